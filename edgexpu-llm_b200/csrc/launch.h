// launch.h -- host-side launchers of the edgexpu CUDA kernels (internal to libedgexpu_cuda.so).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace ex {

// Activation quantizers (device buffers, stream ordered).
//   x: [m][n] fp32 rows; dst: [m][n/32 * 34] (Q8_0) or [m][n/256 * 292] (Q8_K), GGUF layout.
cudaError_t launch_quantize_q8_0(const float* x, int m, int n, uint8_t* dst, cudaStream_t st);
cudaError_t launch_quantize_q8_k(const float* x, int m, int n, uint8_t* dst, cudaStream_t st);

// Element-wise row decoding (dequant.cu) for every GGUF type the path accepts (F32, F16, Q8_0,
// Q4_0, Q5_0, Q4_K, Q5_K, Q6_K), with the reference's float expressions.
//   out[i][e] = row ids[i] of w (row i if ids is null) dequantized; ids outside [0, n_rows) give NaN
//   rows and set ST_BAD_INDEX in *status.
cudaError_t launch_dequant_rows(uint32_t type, const uint8_t* w, size_t row_bytes, long long n_rows,
                                const int32_t* ids, int n_ids, int n, float* out, uint32_t* status, cudaStream_t st);
//   out[t*n_out + o] = bias[o] + dot(dequantized row o, x_t) with fp32 activations x [m][n].
cudaError_t launch_dot_f32(uint32_t type, const uint8_t* w, size_t row_bytes, int n_out, int n, const float* x, int m,
                           const float* bias, float* out, cudaStream_t st);
//   atomicMax of argmax_key(scores[i], row0 + i) over i < n into *key (the caller zeroes *key).
cudaError_t launch_argmax_key(const float* scores, int n, long long row0, unsigned long long* key, cudaStream_t st);

// Temperature sampling over n scores (sample.cu): softmax of io (divided by temperature when
// > 0) in place, then the reference's top_p truncation and pick with the draw u in [0, 1);
// the id into out_dev[0], the softmax denominator and the picked prefix's sum and length into
// stats_dev[0], [2], [3].  scratch: sample_scratch_bytes(n) bytes.
size_t sample_scratch_bytes(int n);
cudaError_t launch_sample(float* io, int n, float temperature, float top_p, double u, void* scratch, size_t scratch_bytes,
                          uint32_t* out_dev, double* stats_dev, cudaStream_t st);

struct ExpTab;  // exptab.cuh

// Llama layer ops on the device (layers.cu).
//   hidden += add (add nullable); out = rmsnorm(hidden) * w.  One CTA; n <= NORM_MAX_N.
constexpr int NORM_MAX_N = 8192;
cudaError_t launch_add_rmsnorm(float* hidden, const float* add, const float* w, float* out, int n, float eps,
                               cudaStream_t st);
//   step[0] = token, step[1] = pos (one thread).
cudaError_t launch_set_step(int* step, int token, int pos, cudaStream_t st);
//   RoPE (adjacent pairs) of q and k at pos = step[1] (device; rope: [window][hd] cos/sin table), k
//   and v into the caches at pos, then out[h][d] = sum_s softmax_s(dot(rot(q_h), K[s][h/rep]) * scale) *
//   V[s][h/rep][d], s = 0..pos.  Cache layout per layer: [n_kv][window][hd]; scores: [n_heads][ld]
//   scratch, ld > pos.  prepare_attention(window, hd) once before the first launch.
cudaError_t launch_attention(const float* q, const float* k, const float* v, const float* rope, float* kc, float* vc,
                             const int* step, int window, int n_heads, int n_kv, int hd, float attn_scale, float* scores,
                             int ld, float* out, const ExpTab& et, cudaStream_t st);
cudaError_t prepare_attention(int window, int hd);
size_t attention_smem_bytes(int window, int hd);
//   g = silu(g) * u.
cudaError_t launch_swiglu(float* g, const float* u, int n, const ExpTab& et, cudaStream_t st);

// Synchronous host-buffer calls through one mapped pinned buffer (zerocopy.cu).
constexpr int ZC_FINISH_THREADS = 128;  // small enough to share an SM with a running GEMV CTA
constexpr int ZC_PULL_MAX_CTAS = 16;
constexpr size_t ZC_MAX_BYTES = 256 * 1024;  // per direction; larger calls use copy-engine transfers
//   dst[0 .. n) = src[0 .. n): src in mapped host memory, both 16-byte aligned.
cudaError_t launch_zc_pull(const float* src, float* dst, int n, cudaStream_t st);
//   After the previous grid completes: dst[0 .. n) = src[0 .. n) (dst in mapped host memory),
//   ctrl[1] = *d_status (and *d_status = 0), then ctrl[0] = *seq_dev (device memory, written by the
//   call's pull).
cudaError_t launch_zc_finish(const float* src, float* dst, int n, uint32_t* d_status, uint32_t* ctrl,
                             const uint32_t* seq_dev, cudaStream_t st);

// What the row-stream kernel does with each finished row.
enum class RowOut : int {
  Store = 0,     // out[t*out_stride + r] = bias[r] + dot
  Argmax = 1,    // atomicMax of argmax_key(bias[r] + dot, row0 + r) into *key (m == 1)
  Partials = 2,  // per-block int32 partials instead of the float dot (test hook)
  StoreTp = 3,   // Store of the sum over the tensor-parallel group (RowStreamArgs::tp), one tensor
};

enum class Fmt : int {
  Q8_0xQ8_0 = 0,  // Q8_0 weight . Q8_0 activation   (gguf_dot_q8.c:436-480)
  Q4_KxQ8_K = 1,  // Q4_K weight . Q8_K activation   (gguf_dot_q8.c:603-762)
  Q4_KxF32 = 2,   // Q4_K weight . fp32 activation   (gguf_quant.c:704-752, logits path)
  Q4_0xQ8_0 = 3,  // Q4_0 weight . Q8_0 activation   (gguf_dot_q8.c:552-601)
  Q5_0xQ8_0 = 4,  // Q5_0 weight . Q8_0 activation   (gguf_dot_q8.c:482-550)
  Q5_KxQ8_K = 5,  // Q5_K weight . Q8_K activation   (gguf_dot_q8.c:764-895)
  Q6_KxQ8_K = 6,  // Q6_K weight . Q8_K activation   (gguf_dot_q8.c:897-1002)
  Q5_KxF32 = 7,   // Q5_K weight . fp32 activation   (gguf_quant.c:837-892, logits path)
  Q6_KxF32 = 8,   // Q6_K weight . fp32 activation   (gguf_quant.c:754-794, logits path)
};

// Activations a format reads: GGUF Q8_0 rows, GGUF Q8_K rows, or fp32 rows.
enum class Act : int { Q8_0 = 0, Q8_K = 1, F32 = 2 };

__host__ __device__ constexpr Act act_of(Fmt f) {
  return (f == Fmt::Q8_0xQ8_0 || f == Fmt::Q4_0xQ8_0 || f == Fmt::Q5_0xQ8_0) ? Act::Q8_0
         : (f == Fmt::Q4_KxF32 || f == Fmt::Q5_KxF32 || f == Fmt::Q6_KxF32) ? Act::F32
                                                                              : Act::Q8_K;
}

// Formats instantiated in rowstream.cu (the original two types); the rest are in rowstream_more.cu.
__host__ __device__ constexpr bool fmt_is_core(Fmt f) {
  return f == Fmt::Q8_0xQ8_0 || f == Fmt::Q4_KxQ8_K || f == Fmt::Q4_KxF32;
}

// One weight tensor of a grouped launch: the segments share K, the weight type and the
// activations, and each writes its own output (row stride = its n_rows).
struct RowSeg {
  const uint8_t* w;
  long long n_rows;
  const float* bias;
  float* out;
  long long tile0;        // first tile of this segment (filled by launch_rowstream)
};
constexpr int MAX_SEGS = 4;

// Tensor-parallel all-reduce over peer memory (tp_p2p.cu).  Every rank holds one region of the
// same layout; peer[r] is rank r's region mapped into this process (peer[rank] = the local one).
constexpr int TP_MAX_WORLD = 8;
constexpr size_t TP_SLOT_BYTES = 512 * 1024;                             // one rank's partials: 65536 u64 entries
constexpr size_t TP_DATA_BYTES = 2 * TP_MAX_WORLD * TP_SLOT_BYTES;       // [parity][rank] (value, tag) words
constexpr size_t TP_CTRL_OFF = TP_DATA_BYTES;                            // u32 CTA counter, u32 epoch
constexpr int TP_DIRECT_WORLD = 4;  // up to this many ranks each output goes to the peers as it is computed
constexpr size_t TP_REGION_BYTES = TP_CTRL_OFF + 256;

struct TpArgs {
  int world;                       // 0 or 1: no all-reduce
  int rank;
  uint8_t* peer[TP_MAX_WORLD];
};

struct RowStreamArgs {
  Fmt fmt;
  RowOut mode;
  const uint8_t* w;       // first weight row (device)
  long long n_rows;
  long long row0;         // global id of the first row (argmax ids)
  int row_bytes;
  int K;
  int m;                  // activation rows (tokens)
  const void* act;        // quantized GGUF activations [m][act_row_bytes], or fp32 [m][K] (act_f32)
  int act_row_bytes;
  bool act_f32;           // Q8 formats: the kernel quantizes fp32 rows itself (m <= 2); Q4_KxF32: always
  const float* bias;      // [n_rows] or nullptr
  float* out;             // Store: [m][out_stride]
  long long out_stride;
  unsigned long long* key;  // Argmax
  int32_t* partials;      // Partials: Q8_0 [m][n_rows][nb]; Q4_K [m][n_rows][nb][2] (sumi, summ)
  uint32_t* status;       // device-visible status word
  int n_seg;              // 0: one tensor (w, n_rows, bias, out, out_stride); 1..MAX_SEGS: seg[] (Store only)
  RowSeg seg[MAX_SEGS];
  TpArgs tp;              // Store, one tensor: sum the outputs of all ranks into out (column-sharded weights)
  bool exact;             // Store / Argmax: reproduce the reference x86 build's float order bit for bit
};

struct DeviceInfo {
  int sm_count;
  int max_smem_optin;
};

// Q8_0 x Q8_0 tensor-core GEMM for prefill batches (gemm_q8_tc.cu).  The weight rows are repacked
// once into q8_weight_pack_bytes(n_rows, K) bytes; the activations into q8_act_pack_bytes(m, K).
size_t q8_weight_pack_bytes(int n_rows, int K);
size_t q8_act_pack_bytes(int m, int K);
cudaError_t launch_q8_repack_weight(const uint8_t* w, int n_rows, int K, uint8_t* pack, cudaStream_t st);
//   From fp32 rows x, or (x == nullptr) from Q8_0 rows xq.
cudaError_t launch_q8_pack_act(const float* x, const uint8_t* xq, int m, int K, uint8_t* pack, cudaStream_t st);
//   out[t*out_stride + r] = bias[r] + sum_b d_w[r][b] d_x[t][b] ip[t][r][b]
cudaError_t launch_q8_gemm(const uint8_t* wpack, int n_rows, const uint8_t* apack, int m, int K, const float* bias,
                           float* out, long long out_stride, uint32_t* status, const DeviceInfo& dev, cudaStream_t st);

// Largest number of activation rows one row-stream launch keeps in shared memory for this K.
int rowstream_max_m(Fmt fmt, int K, const DeviceInfo& dev);

// True when a launch with m activation rows quantizes fp32 activations in its own prologue.
bool rowstream_quantizes_itself(Fmt fmt, int m);

cudaError_t launch_rowstream(const RowStreamArgs& a, const DeviceInfo& dev, cudaStream_t st);

// ---- tensor-core GEMM (gemm_tc.cu): Q4_K weights x Q8_K activations for prefill batches ----

// Smallest batch routed to the tensor-core GEMM instead of the row-stream GEMV.
constexpr int TC_MIN_M = 64;
// Smallest batch routed to the tensor-core GEMM's 16-token tiles (batches below TC_MIN_M; the K
// range of a row tile is split over several CTAs whose partial sums a second kernel adds).
constexpr int TC_SMALL_MIN_M = 9;

// Bytes of the packed activations of m rows of length K (swizzled int8 tiles + per-block d).
size_t tc_act_bytes(int m, int K);

// fp32 rows -> packed activations, quantized exactly as edgexpu_gguf_quantize_q8_k.
cudaError_t launch_tc_pack_f32(const float* x, int m, int K, uint8_t* act, cudaStream_t st);
// Q8_K rows (GGUF blocks) -> packed activations.
cudaError_t launch_tc_pack_q8k(const uint8_t* xq, int m, int K, uint8_t* act, cudaStream_t st);

struct TcGemmArgs {
  const uint8_t* w;      // Q4_K rows, 16-byte aligned, row_bytes = K/256*144
  int n_rows;
  int K;
  const uint8_t* act;    // packed activations of m rows
  int m;
  const float* bias;     // nullable
  float* out;            // out[t*out_stride + row]
  long long out_stride;
  int32_t* partials;     // non-null: (sumi, summ) per [t][row][super-block] instead of out
  uint32_t* status;      // device status word
  float* part;           // tc_split_bytes(m, n_rows, K) bytes of scratch (when nonzero) for K-split sums
};

// Scratch for the partial sums of a K-split launch (0: the launch is not split).
size_t tc_split_bytes(int m, int n_rows, int K, const DeviceInfo& dev);

cudaError_t launch_tc_gemm(const TcGemmArgs& a, const DeviceInfo& dev, cudaStream_t st);

}  // namespace ex
