// session.cu -- a llama decoder that runs whole on the device: the reference's layer loop
// (forward_decode_token, src/native.c:2404-2600, and the per-token arithmetic of
// edgexpu_native_forward_prefill / apply_transformer_layer, :1917-2253) over weights streamed into
// HBM by the GGUF loader.  Per token:
//   embedding row (dequant_rows, gguf_quant.c:428-466)
//   per layer: rmsnorm -> q|k|v GEMV -> RoPE, K/V into the cache -> attention over 0..pos ->
//              o GEMV -> residual add + rmsnorm -> gate|up GEMV -> SwiGLU -> down GEMV
//   residual add + output norm -> the next token: greedy logits (native.c:2355-2397) or the
//   temperature branch's softmax sampling (native.c:2322-2353)
// The GEMVs are the library's (the process's float order: by default the x86 order, bit-identical
// to the reference); the other ops are layers.cu.  A prompt runs token by token at positions
// pos0.. (the prefill's per-token operations are the decode's: every dot, norm and softmax sees the
// same operands in the same order, so the KV cache holds the same values).  The RoPE cos/sin
// table is computed on the host by rope_fill_cache's arithmetic (cpu_kernel.c:659-669) with the
// process's libm, as the reference does, once per position at open.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/edgexpu_cuda.h"
#include "capi_internal.h"
#include "exptab.cuh"
#include "launch.h"

namespace {

struct W {
  const uint8_t* p = nullptr;
  uint32_t type = 0;
  int n_out = 0, n_in = 0;
};

struct Layer {
  W q, k, v, o, gate, up, down;
  const float* attn_norm = nullptr;
  const float* ffn_norm = nullptr;
};

struct Session {
  void* model = nullptr;
  int n_layers = 0, n_embd = 0, n_ff = 0, n_heads = 0, n_kv = 0, hd = 0, vocab = 0, window = 0;
  float eps = 1e-6f, theta = 10000.0f, attn_scale = 1.0f;
  std::vector<Layer> layers;
  W embd, out;
  const float* out_norm = nullptr;
  float* buf = nullptr;  // device: hidden, normed, q, k, v, attn, proj, gate, up, down, last, scores
  float *hidden, *normed, *q, *k, *v, *attn, *proj, *gate, *up, *down, *last, *scores;
  float* kc = nullptr;   // [layers][n_kv][window][hd]
  float* vc = nullptr;
  float* rope = nullptr;  // [window][hd]: cos, sin of each pair
  float* att = nullptr;   // [n_heads][window]: attention scores
  int32_t* step = nullptr;  // device: {token, position} of the step being run
  uint64_t* key_dev = nullptr;
  ex::ExpTab et{};
  bool et_held = false;
  uint64_t* key_host = nullptr;
  int eager_steps = 0;      // single-token steps run without the graph (the first one instantiates every kernel)
  cudaGraphExec_t graph = nullptr;  // the layers of one token, for any position
};

int find(void* model, const std::string& name, W* w, char* error, size_t error_size, bool required = true) {
  const int i = edgexpu_cuda_gguf_find(model, name.c_str());
  if (i < 0) {
    if (!required) return 1;
    return ex::api_fail(error, error_size, "llama_open: tensor %s missing", name.c_str());
  }
  int64_t n_in = 0, n_out = 0;
  uint64_t nbytes = 0;
  if (!edgexpu_cuda_gguf_tensor_at(model, i, nullptr, &w->p, &w->type, &n_in, &n_out, nullptr, &nbytes) || nbytes == 0)
    return ex::api_fail(error, error_size, "llama_open: tensor %s has a type this library does not read", name.c_str());
  w->n_in = static_cast<int>(n_in);
  w->n_out = static_cast<int>(n_out);
  return 1;
}

uint64_t meta_u(void* model, const std::string& key, uint64_t dflt) {
  uint64_t v = 0;
  return edgexpu_cuda_gguf_meta(model, key.c_str(), &v, nullptr, nullptr) ? v : dflt;
}

double meta_f(void* model, const std::string& key, double dflt) {
  double v = 0;
  return edgexpu_cuda_gguf_meta(model, key.c_str(), nullptr, &v, nullptr) ? v : dflt;
}

void release(Session* s) {
  if (s == nullptr) return;
  cudaStreamSynchronize(ex::api_stream());
  cudaFree(s->buf);
  cudaFree(s->kc);
  cudaFree(s->vc);
  cudaFree(s->rope);
  cudaFree(s->att);
  if (s->graph != nullptr) cudaGraphExecDestroy(s->graph);
  cudaFree(s->step);
  cudaFree(s->key_dev);
  cudaFreeHost(s->key_host);
  if (s->model != nullptr) edgexpu_cuda_gguf_free(s->model);
  if (s->et_held) ex::exptab_release();
  delete s;
}

#define SX(call)                                                                                     \
  do {                                                                                               \
    const cudaError_t e_ = (call);                                                                   \
    if (e_ != cudaSuccess) return ex::api_fail(error, error_size, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

// The token and position in s->step through every layer; leaves the output-normed hidden state
// in s->last.  Every launch reads the position from s->step, so one captured graph serves all.
int forward_layers(Session* s, cudaStream_t st, char* error, size_t error_size) {
  SX(ex::launch_dequant_rows(s->embd.type, s->embd.p, ex::api_row_bytes(s->embd.type, s->n_embd), s->embd.n_out, s->step,
                             1, s->n_embd, s->hidden, ex::api_status_word(), st));
  const size_t kv_row = static_cast<size_t>(s->n_kv) * s->hd;
  for (int l = 0; l < s->n_layers; ++l) {
    const Layer& L = s->layers[static_cast<size_t>(l)];
    SX(ex::launch_add_rmsnorm(s->hidden, l == 0 ? nullptr : s->down, L.attn_norm, s->normed, s->n_embd, s->eps, st));
    if (L.q.type == L.k.type && L.k.type == L.v.type) {
      float* outs[3] = {s->q, s->k, s->v};
      const uint8_t* ws[3] = {L.q.p, L.k.p, L.v.p};
      const int nouts[3] = {L.q.n_out, L.k.n_out, L.v.n_out};
      if (!edgexpu_cuda_linear_quant_multi_dev(3, outs, ws, nouts, nullptr, L.q.type, s->normed, 1, s->n_embd, st))
        return ex::api_fail(error, error_size, "layer %d q|k|v: %s", l, edgexpu_cuda_last_error());
    } else {
      const W* w3[3] = {&L.q, &L.k, &L.v};
      float* o3[3] = {s->q, s->k, s->v};
      for (int i = 0; i < 3; ++i)
        if (!edgexpu_cuda_linear_quant_batch_dev(o3[i], s->normed, w3[i]->p, w3[i]->type, nullptr, 1, w3[i]->n_out, s->n_embd, st))
          return ex::api_fail(error, error_size, "layer %d q/k/v: %s", l, edgexpu_cuda_last_error());
    }
    float* kl = s->kc + static_cast<size_t>(l) * s->window * kv_row;  // [n_kv][window][hd]
    float* vl = s->vc + static_cast<size_t>(l) * s->window * kv_row;
    SX(ex::launch_attention(s->q, s->k, s->v, s->rope, kl, vl, s->step, s->window, s->n_heads, s->n_kv, s->hd,
                            s->attn_scale, s->att, s->window, s->attn, s->et, st));
    if (!edgexpu_cuda_linear_quant_batch_dev(s->proj, s->attn, L.o.p, L.o.type, nullptr, 1, L.o.n_out, L.o.n_in, st))
      return ex::api_fail(error, error_size, "layer %d o: %s", l, edgexpu_cuda_last_error());
    SX(ex::launch_add_rmsnorm(s->hidden, s->proj, L.ffn_norm, s->normed, s->n_embd, s->eps, st));
    if (L.gate.type == L.up.type) {
      float* outs[2] = {s->gate, s->up};
      const uint8_t* ws[2] = {L.gate.p, L.up.p};
      const int nouts[2] = {L.gate.n_out, L.up.n_out};
      if (!edgexpu_cuda_linear_quant_multi_dev(2, outs, ws, nouts, nullptr, L.gate.type, s->normed, 1, s->n_embd, st))
        return ex::api_fail(error, error_size, "layer %d gate|up: %s", l, edgexpu_cuda_last_error());
    } else if (!edgexpu_cuda_linear_quant_batch_dev(s->gate, s->normed, L.gate.p, L.gate.type, nullptr, 1, s->n_ff, s->n_embd, st) ||
               !edgexpu_cuda_linear_quant_batch_dev(s->up, s->normed, L.up.p, L.up.type, nullptr, 1, s->n_ff, s->n_embd, st)) {
      return ex::api_fail(error, error_size, "layer %d gate/up: %s", l, edgexpu_cuda_last_error());
    }
    SX(ex::launch_swiglu(s->gate, s->up, s->n_ff, s->et, st));
    if (!edgexpu_cuda_linear_quant_batch_dev(s->down, s->gate, L.down.p, L.down.type, nullptr, 1, s->n_embd, s->n_ff, st))
      return ex::api_fail(error, error_size, "layer %d down: %s", l, edgexpu_cuda_last_error());
  }
  SX(ex::launch_add_rmsnorm(s->hidden, s->down, s->out_norm, s->last, s->n_embd, s->eps, st));
  return 1;
}

// Capture forward_layers into s->graph (after eager steps have instantiated and configured every
// kernel, so the capture makes no other CUDA calls).
int capture(Session* s, cudaStream_t st, char* error, size_t error_size) {
  SX(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  const int ok = forward_layers(s, st, error, error_size);
  cudaGraph_t g = nullptr;
  const cudaError_t e = cudaStreamEndCapture(st, &g);
  if (!ok || e != cudaSuccess) {
    if (g != nullptr) cudaGraphDestroy(g);
    return ok ? ex::api_fail(error, error_size, "capturing the decode step: %s", cudaGetErrorString(e)) : 0;
  }
  const cudaError_t ie = cudaGraphInstantiate(&s->graph, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) {
    s->graph = nullptr;
    return ex::api_fail(error, error_size, "instantiating the decode step: %s", cudaGetErrorString(ie));
  }
  return 1;
}

}  // namespace

extern "C" {

int edgexpu_cuda_llama_open(const char* gguf_path, int window, void** session, char* error, size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(ex::api_mutex());
  if (!ex::api_ready(error, error_size)) return 0;
  if (gguf_path == nullptr || session == nullptr || window < 1) return ex::api_fail(error, error_size, "llama_open: invalid arguments");
  *session = nullptr;
  auto s = std::unique_ptr<Session, void (*)(Session*)>(new Session(), release);
  if (!edgexpu_cuda_gguf_load(gguf_path, window, &s->model, nullptr, error, error_size)) return 0;
  const char* arch = nullptr;
  if (!edgexpu_cuda_gguf_meta(s->model, "general.architecture", nullptr, nullptr, &arch) || arch == nullptr ||
      std::string(arch) != "llama")
    return ex::api_fail(error, error_size, "llama_open: architecture %s is not llama", arch != nullptr ? arch : "?");
  const std::string a = arch;
  s->n_layers = static_cast<int>(meta_u(s->model, a + ".block_count", 0));
  s->n_embd = static_cast<int>(meta_u(s->model, a + ".embedding_length", 0));
  s->n_ff = static_cast<int>(meta_u(s->model, a + ".feed_forward_length", 0));
  s->n_heads = static_cast<int>(meta_u(s->model, a + ".attention.head_count", 0));
  s->n_kv = static_cast<int>(meta_u(s->model, a + ".attention.head_count_kv", static_cast<uint64_t>(s->n_heads)));
  if (s->n_layers <= 0 || s->n_embd <= 0 || s->n_ff <= 0 || s->n_heads <= 0 || s->n_kv <= 0 || s->n_heads % s->n_kv != 0)
    return ex::api_fail(error, error_size, "llama_open: incomplete llama metadata");
  s->hd = static_cast<int>(meta_u(s->model, a + ".attention.key_length", static_cast<uint64_t>(s->n_embd / s->n_heads)));
  // native.c: rms_eps > 0 ? rms_eps : 1e-6f; default_rope_freq (:383-392): freq_base > 0, else 10000 for llama
  const double eps = meta_f(s->model, a + ".attention.layer_norm_rms_epsilon", 0.0);
  s->eps = eps > 0.0 ? static_cast<float>(eps) : 1e-6f;
  const double th = meta_f(s->model, a + ".rope.freq_base", 0.0);
  s->theta = th > 0.0 ? static_cast<float>(th) : 10000.0f;
  s->attn_scale = 1.0f / sqrtf(static_cast<float>(s->hd));
  s->window = window;
  uint64_t n_tok = 0;
  edgexpu_cuda_gguf_meta(s->model, "tokenizer.ggml.tokens", &n_tok, nullptr, nullptr);
  if (s->hd % 4 != 0 || s->hd > 256) return ex::api_fail(error, error_size, "llama_open: head_dim %d unsupported", s->hd);
  if (s->n_embd > ex::NORM_MAX_N)
    return ex::api_fail(error, error_size, "llama_open: n_embd %d unsupported (at most %d)", s->n_embd, ex::NORM_MAX_N);
  if (ex::attention_smem_bytes(window, s->hd) > 200u * 1024)  // the attention kernel's shared memory
    return ex::api_fail(error, error_size, "llama_open: window %d too long for head_dim %d", window, s->hd);
  if (!find(s->model, "token_embd.weight", &s->embd, error, error_size)) return 0;
  if (!find(s->model, "output.weight", &s->out, error, error_size, false)) return 0;
  if (s->out.p == nullptr) s->out = s->embd;  // tied embeddings (native.c:415-426)
  s->vocab = n_tok > 0 ? static_cast<int>(n_tok) : s->out.n_out;
  if (s->vocab > s->out.n_out) return ex::api_fail(error, error_size, "llama_open: vocabulary larger than the logits weight");
  W onorm;
  if (!find(s->model, "output_norm.weight", &onorm, error, error_size)) return 0;
  s->out_norm = reinterpret_cast<const float*>(onorm.p);
  s->layers.resize(static_cast<size_t>(s->n_layers));
  for (int l = 0; l < s->n_layers; ++l) {
    Layer& L = s->layers[static_cast<size_t>(l)];
    const std::string p = "blk." + std::to_string(l) + ".";
    W an, fn;
    if (!find(s->model, p + "attn_norm.weight", &an, error, error_size) || !find(s->model, p + "ffn_norm.weight", &fn, error, error_size) ||
        !find(s->model, p + "attn_q.weight", &L.q, error, error_size) || !find(s->model, p + "attn_k.weight", &L.k, error, error_size) ||
        !find(s->model, p + "attn_v.weight", &L.v, error, error_size) ||
        !find(s->model, p + "attn_output.weight", &L.o, error, error_size) ||
        !find(s->model, p + "ffn_gate.weight", &L.gate, error, error_size) ||
        !find(s->model, p + "ffn_up.weight", &L.up, error, error_size) || !find(s->model, p + "ffn_down.weight", &L.down, error, error_size))
      return 0;
    L.attn_norm = reinterpret_cast<const float*>(an.p);
    L.ffn_norm = reinterpret_cast<const float*>(fn.p);
  }
  // device buffers
  const size_t kv_row = static_cast<size_t>(s->n_kv) * s->hd;
  const size_t nf = static_cast<size_t>(s->n_embd) * 3 + static_cast<size_t>(s->n_heads) * s->hd * 2 + kv_row * 2 +
                    static_cast<size_t>(s->n_ff) * 2 + static_cast<size_t>(s->n_embd) * 2 + static_cast<size_t>(s->out.n_out) + 64;
  SX(cudaMalloc(&s->buf, nf * 4));
  float* b = s->buf;
  s->hidden = b; b += s->n_embd;
  s->normed = b; b += s->n_embd;
  s->proj = b; b += s->n_embd;
  s->q = b; b += static_cast<size_t>(s->n_heads) * s->hd;
  s->attn = b; b += static_cast<size_t>(s->n_heads) * s->hd;
  s->k = b; b += kv_row;
  s->v = b; b += kv_row;
  s->gate = b; b += s->n_ff;
  s->up = b; b += s->n_ff;
  s->down = b; b += s->n_embd;
  s->last = b; b += s->n_embd;
  s->scores = b;
  const size_t cache = static_cast<size_t>(s->n_layers) * window * kv_row * 4;
  SX(cudaMalloc(&s->kc, cache));
  SX(cudaMalloc(&s->vc, cache));
  SX(cudaMemset(s->kc, 0, cache));
  SX(cudaMemset(s->vc, 0, cache));
  // rope_fill_cache (cpu_kernel.c:659-669) for every position of the window
  std::vector<float> rope(static_cast<size_t>(window) * s->hd);
  const float theta_scale = powf(s->theta, -2.0f / static_cast<float>(s->hd));
  for (int pos = 0; pos < window; ++pos) {
    float t = static_cast<float>(pos);
    float* c = rope.data() + static_cast<size_t>(pos) * s->hd;
    for (int i = 0; i < s->hd; i += 2) {
      c[i] = cosf(t);
      c[i + 1] = sinf(t);
      t *= theta_scale;
    }
  }
  SX(cudaMalloc(&s->rope, rope.size() * 4));
  SX(cudaMalloc(&s->att, static_cast<size_t>(s->n_heads) * window * 4));
  SX(cudaMemcpy(s->rope, rope.data(), rope.size() * 4, cudaMemcpyHostToDevice));
  if (!ex::exptab_acquire(&s->et, error, error_size)) return 0;
  s->et_held = true;
  SX(ex::prepare_attention(window, s->hd));
  SX(cudaMalloc(&s->step, 16));
  SX(cudaMalloc(&s->key_dev, 16));
  SX(cudaHostAlloc(reinterpret_cast<void**>(&s->key_host), 16, cudaHostAllocDefault));
  *session = s.release();
  return 1;
}

int edgexpu_cuda_llama_forward(void* session, const uint32_t* tokens, int n_tokens, int pos0, float temperature,
                               float top_p, uint64_t* rng, uint32_t* next_token, float* last_hidden, char* error,
                               size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(ex::api_mutex());
  if (!ex::api_ready(error, error_size)) return 0;
  Session* s = static_cast<Session*>(session);
  if (s == nullptr || tokens == nullptr || n_tokens <= 0 || pos0 < 0 || next_token == nullptr)
    return ex::api_fail(error, error_size, "llama_forward: invalid arguments");
  if (pos0 + n_tokens > s->window)
    return ex::api_fail(error, error_size, "llama_forward: positions %d..%d exceed the window of %d", pos0,
                        pos0 + n_tokens - 1, s->window);
  const bool sample = temperature > 1e-4f;
  if (sample && rng == nullptr) return ex::api_fail(error, error_size, "llama_forward: sampling needs an rng state");
  cudaStream_t st = ex::api_stream();
  for (int t = 0; t < n_tokens; ++t) {
    SX(ex::launch_set_step(s->step, static_cast<int>(tokens[t]), pos0 + t, st));
    if (n_tokens == 1 && s->eager_steps >= 1 && s->graph == nullptr && !capture(s, st, error, error_size)) return 0;
    if (n_tokens == 1 && s->graph != nullptr) {
      SX(cudaGraphLaunch(s->graph, st));
    } else {
      if (!forward_layers(s, st, error, error_size)) return 0;
      if (n_tokens == 1) ++s->eager_steps;
    }
  }
  if (last_hidden != nullptr)
    SX(cudaMemcpyAsync(last_hidden, s->last, static_cast<size_t>(s->n_embd) * 4, cudaMemcpyDeviceToHost, st));
  if (sample) {
    if (!ex::api_logit_scores(s->out.p, s->out.type, s->last, s->n_embd, s->vocab, nullptr, s->scores, st, error, error_size))
      return 0;
    return ex::api_sample(s->scores, s->vocab, temperature, top_p, rng, next_token, st, error, error_size);
  }
  if (!edgexpu_cuda_logits_argmax_dev(s->out.p, s->out.type, s->last, s->n_embd, s->vocab, nullptr, 0, s->key_dev, st))
    return ex::api_fail(error, error_size, "logits: %s", edgexpu_cuda_last_error());
  SX(cudaMemcpyAsync(s->key_host, s->key_dev, 8, cudaMemcpyDeviceToHost, st));
  if (!edgexpu_cuda_stream_sync(st, error, error_size)) return 0;
  *next_token = edgexpu_cuda_argmax_key_id(*s->key_host);
  return 1;
}

int edgexpu_cuda_llama_close(void* session) {
  std::lock_guard<std::recursive_mutex> lk(ex::api_mutex());
  if (session == nullptr) return 0;
  release(static_cast<Session*>(session));
  return 1;
}

}  // extern "C"
