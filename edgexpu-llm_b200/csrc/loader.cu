// loader.cu -- a GGUF model file streamed into HBM in one pass, after an HBM budget check.
//
// The reference maps the file (native.c:115-163), copies every layer of every token into one
// staging buffer (stage_copy_bytes, native.c:350-380) and admits a model when its working set,
// KV cache and scratch fit 85 % of the machine's RAM (fill_native_plan, scheduler.c:320-422).
// On a B200 the whole model stays resident, so:
//   * the budget is the same plan with the weight term = every tensor byte (all resident) and the
//     limit = 85 % of the device's HBM (edgexpu_cuda_hbm_plan_native);
//   * the loader parses the GGUF header (gguf.c:359-610: magic, version, counts, key/values,
//     tensor infos, aligned data section), allocates one arena for the data section, streams the
//     file into it through two pinned buffers (a read of one overlaps the copy of the other), and
//     registers every tensor of a supported type with the weight registry, so any of its rows is
//     a valid `weight` argument of the other entry points.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/edgexpu_cuda.h"
#include "capi_internal.h"

namespace {

constexpr uint32_t GGUF_MAGIC = 0x46554747u;  // "GGUF" little-endian
enum : uint32_t {
  GT_U8 = 0, GT_I8 = 1, GT_U16 = 2, GT_I16 = 3, GT_U32 = 4, GT_I32 = 5, GT_F32 = 6, GT_BOOL = 7,
  GT_STRING = 8, GT_ARRAY = 9, GT_U64 = 10, GT_I64 = 11, GT_F64 = 12
};
constexpr size_t STREAM_CHUNK = 64u << 20;  // bytes per pinned buffer

// Sequential reader over a file descriptor with a 1 MiB window (the header can hold a
// vocabulary of a few hundred thousand strings).
struct Reader {
  int fd = -1;
  uint64_t size = 0, pos = 0;
  std::vector<uint8_t> win;
  uint64_t win_at = 0;
  size_t win_len = 0;
  bool ok = true;

  bool fill(uint64_t at) {
    win.resize(1u << 20);
    const ssize_t n = pread(fd, win.data(), win.size(), static_cast<off_t>(at));
    if (n <= 0) return false;
    win_at = at;
    win_len = static_cast<size_t>(n);
    return true;
  }
  bool bytes(void* dst, size_t n) {
    uint8_t* d = static_cast<uint8_t*>(dst);
    while (n > 0) {
      if (pos >= size) return ok = false;
      if (pos < win_at || pos >= win_at + win_len) {
        if (!fill(pos)) return ok = false;
      }
      const size_t off = static_cast<size_t>(pos - win_at), take = std::min(n, win_len - off);
      if (d != nullptr) {
        std::memcpy(d, win.data() + off, take);
        d += take;
      }
      pos += take;
      n -= take;
    }
    return true;
  }
  bool skip(uint64_t n) {
    if (pos + n > size) return ok = false;
    pos += n;
    return true;
  }
  template <class T>
  T get() {
    T v{};
    bytes(&v, sizeof v);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || n > (1u << 24)) {
      ok = false;
      return {};
    }
    std::string s(static_cast<size_t>(n), '\0');
    bytes(s.data(), s.size());
    return s;
  }
};

size_t scalar_size(uint32_t t) {
  switch (t) {
    case GT_U8: case GT_I8: case GT_BOOL: return 1;
    case GT_U16: case GT_I16: return 2;
    case GT_U32: case GT_I32: case GT_F32: return 4;
    case GT_U64: case GT_I64: case GT_F64: return 8;
    default: return 0;
  }
}

// Read a value of type t: integers into *as_int, f32/f64 into *as_f, strings into *as_str, the
// element count of an array into *as_int; everything else is skipped.
bool read_value(Reader& r, uint32_t t, uint64_t* as_int, std::string* as_str, double* as_f = nullptr, int depth = 0) {
  if (t == GT_STRING) {
    std::string s = r.str();
    if (as_str != nullptr) *as_str = s;
    return r.ok;
  }
  if (t == GT_ARRAY) {
    const uint32_t et = r.get<uint32_t>();
    const uint64_t n = r.get<uint64_t>();
    if (!r.ok || depth > 2) return false;
    if (as_int != nullptr) *as_int = n;
    if (et == GT_STRING || et == GT_ARRAY) {
      for (uint64_t i = 0; i < n && r.ok; ++i) read_value(r, et, nullptr, nullptr, nullptr, depth + 1);
      return r.ok;
    }
    const size_t es = scalar_size(et);
    return es != 0 && r.skip(n * es);
  }
  const size_t sz = scalar_size(t);
  if (sz == 0) return false;
  uint64_t v = 0;
  r.bytes(&v, sz);
  if (t == GT_F32) {
    float f;
    std::memcpy(&f, &v, 4);
    if (as_f != nullptr) *as_f = f;
  } else if (t == GT_F64) {
    double d;
    std::memcpy(&d, &v, 8);
    if (as_f != nullptr) *as_f = d;
  } else if (as_int != nullptr) {
    *as_int = v;
  }
  return r.ok;
}

struct Tensor {
  std::string name;
  uint32_t type;
  int n_dims;
  uint64_t dims[4];
  uint64_t offset;  // inside the data section
  uint64_t nbytes;  // 0 for types this library does not read
  bool registered;
};

struct Meta {
  std::string key;
  uint32_t type;
  uint64_t u;   // integers; element count of arrays
  double f;     // f32 / f64
  std::string s;
};

struct Model {
  uint8_t* arena = nullptr;
  uint64_t data_start = 0, data_bytes = 0;
  std::vector<Tensor> tensors;
  std::vector<Meta> meta;
  edgexpu_cuda_hbm_plan plan{};
};

uint64_t mul_sat(uint64_t a, uint64_t b) { return (a != 0 && b > UINT64_MAX / a) ? UINT64_MAX : a * b; }
uint64_t add_sat(uint64_t a, uint64_t b) { return a > UINT64_MAX - b ? UINT64_MAX : a + b; }

}  // namespace

extern "C" {

int edgexpu_cuda_hbm_plan_native(uint64_t file_bytes, uint64_t weight_bytes, uint32_t n_kv_layers, uint32_t n_kv_heads,
                                 int head_dim, uint32_t n_embd, uint32_t n_ff, uint32_t n_heads, int window,
                                 uint64_t hbm_total_bytes, edgexpu_cuda_hbm_plan* plan) {
  if (plan == nullptr) return 0;
  std::memset(plan, 0, sizeof *plan);
  // The terms of fill_native_plan (scheduler.c:320-422): fp32 K and V per KV layer and position,
  // scratch of min(window, EDGEXPU_BUDGET_SCRATCH_SEQ = 64) positions.
  if (window < 1) window = 1;
  if (head_dim <= 0 && n_embd > 0 && n_heads > 0) head_dim = static_cast<int>(n_embd / n_heads);
  if (n_ff == 0 && n_embd > 0) n_ff = n_embd * 4u;
  plan->window = window;
  plan->file_bytes = file_bytes;
  plan->weight_bytes = weight_bytes;
  plan->kv_bytes = mul_sat(2u, mul_sat(n_kv_layers, mul_sat(n_kv_heads, mul_sat(static_cast<uint64_t>(head_dim),
                                                                                 mul_sat(static_cast<uint64_t>(window), 4u)))));
  const uint64_t seq = window > 64 ? 64u : static_cast<uint64_t>(window);
  const uint64_t per_pos = static_cast<uint64_t>(n_embd) * 6u + static_cast<uint64_t>(n_ff) * 2u +
                           static_cast<uint64_t>(n_heads) * head_dim + 2u * static_cast<uint64_t>(n_kv_heads) * head_dim;
  plan->scratch_bytes = mul_sat(seq, mul_sat(per_pos, 4u));
  plan->total_bytes = add_sat(add_sat(plan->weight_bytes, plan->kv_bytes), plan->scratch_bytes);
  const uint64_t MB = 1024u * 1024u;
  if (std::getenv("EDGEXPU_BUDGET_DISABLE") != nullptr) {
    plan->limit_bytes = UINT64_MAX;
    plan->admitted = 1;
    std::snprintf(plan->reason, sizeof plan->reason, "budget disabled by EDGEXPU_BUDGET_DISABLE");
    return 1;
  }
  const uint64_t total_mb = hbm_total_bytes / MB, usable_mb = total_mb * 85u / 100u;
  if (usable_mb == 0) {  // as the reference does when the device's memory is unknown
    plan->admitted = 1;
    std::snprintf(plan->reason, sizeof plan->reason, "device memory unknown; admit the load");
    return 1;
  }
  plan->limit_bytes = usable_mb * MB;
  plan->admitted = plan->total_bytes <= plan->limit_bytes;
  std::snprintf(plan->reason, sizeof plan->reason,
                "HBM budget %llu MB %s %llu MB (85%% of %llu MB; weights resident %llu KV %llu scratch %llu, window %d)",
                static_cast<unsigned long long>(plan->total_bytes / MB), plan->admitted ? "within" : "exceeds",
                static_cast<unsigned long long>(plan->limit_bytes / MB), static_cast<unsigned long long>(total_mb),
                static_cast<unsigned long long>(plan->weight_bytes / MB), static_cast<unsigned long long>(plan->kv_bytes / MB),
                static_cast<unsigned long long>(plan->scratch_bytes / MB), window);
  return plan->admitted;
}

int edgexpu_cuda_gguf_load(const char* path, int window, void** model, edgexpu_cuda_hbm_plan* plan_out, char* error,
                           size_t error_size) {
  std::lock_guard<std::recursive_mutex> lk(ex::api_mutex());
  if (!ex::api_ready(error, error_size)) return 0;
  if (path == nullptr || model == nullptr) return ex::api_fail(error, error_size, "gguf_load: invalid arguments");
  *model = nullptr;
  Reader r;
  r.fd = open(path, O_RDONLY);
  if (r.fd < 0) return ex::api_fail(error, error_size, "gguf_load: cannot open %s", path);
  struct stat st {};
  if (fstat(r.fd, &st) != 0) {
    close(r.fd);
    return ex::api_fail(error, error_size, "gguf_load: cannot stat %s", path);
  }
  r.size = static_cast<uint64_t>(st.st_size);
  auto bail = [&](const char* what) {
    close(r.fd);
    return ex::api_fail(error, error_size, "gguf_load: %s: %s", path, what);
  };
  // Header (gguf.c:359-610).
  if (r.get<uint32_t>() != GGUF_MAGIC || !r.ok) return bail("not a GGUF file");
  const uint32_t version = r.get<uint32_t>();
  if (version < 2 || version > 3) return bail("unsupported GGUF version");
  const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
  if (!r.ok || n_tensors > (1u << 20) || n_kv > (1u << 20)) return bail("bad header counts");
  std::string arch;
  uint64_t alignment = 32;
  auto m = std::make_unique<Model>();
  for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
    Meta e{};
    e.key = r.str();
    e.type = r.get<uint32_t>();
    if (!read_value(r, e.type, &e.u, e.type == GT_STRING ? &e.s : nullptr, &e.f)) return bail("bad metadata value");
    if (e.key == "general.architecture") arch = e.s;
    else if (e.key == "general.alignment" && e.u != 0) alignment = e.u;
    m->meta.push_back(std::move(e));
  }
  auto dim = [&](const char* suffix) -> uint64_t {
    const std::string k = arch + "." + suffix;
    for (const Meta& e : m->meta)
      if (e.key == k && e.type != GT_STRING && e.type != GT_ARRAY && e.type != GT_F32 && e.type != GT_F64) return e.u;
    return 0;
  };
  m->tensors.reserve(static_cast<size_t>(n_tensors));
  for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
    Tensor t{};
    t.name = r.str();
    t.n_dims = static_cast<int>(r.get<uint32_t>());
    if (!r.ok || t.n_dims < 1 || t.n_dims > 4) return bail("bad tensor info");
    for (int d = 0; d < t.n_dims; ++d) t.dims[d] = r.get<uint64_t>();
    t.type = r.get<uint32_t>();
    t.offset = r.get<uint64_t>();
    uint64_t rows = 1;
    for (int d = 1; d < t.n_dims; ++d) rows = mul_sat(rows, t.dims[d]);
    const size_t rb = t.dims[0] <= (1u << 30) ? ex::api_row_bytes(t.type, static_cast<int>(t.dims[0])) : 0;
    t.nbytes = rb != 0 ? mul_sat(rb, rows) : 0;
    m->tensors.push_back(std::move(t));
  }
  if (!r.ok || alignment == 0 || (alignment & (alignment - 1)) != 0) return bail("bad tensor infos");
  m->data_start = (r.pos + alignment - 1) / alignment * alignment;
  if (m->data_start > r.size) return bail("data section past the end of the file");
  m->data_bytes = r.size - m->data_start;
  for (const Tensor& t : m->tensors)
    if (t.nbytes != 0 && t.offset + t.nbytes > m->data_bytes) return bail("tensor data past the end of the file");

  // Budget: every tensor byte resident, KV and scratch as the reference plans them.
  size_t free_b = 0, total_b = 0;
  if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return bail("cudaMemGetInfo failed");
  const uint64_t n_embd = dim("embedding_length"), n_heads = dim("attention.head_count");
  uint64_t n_kv_heads = dim("attention.head_count_kv");
  if (n_kv_heads == 0) n_kv_heads = n_heads;
  const int head_dim = static_cast<int>(dim("attention.key_length"));
  edgexpu_cuda_hbm_plan_native(r.size, m->data_bytes, static_cast<uint32_t>(dim("block_count")),
                               static_cast<uint32_t>(n_kv_heads), head_dim, static_cast<uint32_t>(n_embd),
                               static_cast<uint32_t>(dim("feed_forward_length")), static_cast<uint32_t>(n_heads), window,
                               total_b, &m->plan);
  if (plan_out != nullptr) *plan_out = m->plan;
  if (!m->plan.admitted) {
    close(r.fd);
    return ex::api_fail(error, error_size, "%s", m->plan.reason);
  }
  if (m->data_bytes + 256 > free_b) return bail("not enough free HBM for the model");

  // One arena for the data section (+256 bytes so a 16-byte-rounded copy of the last rows stays
  // inside it), streamed through two pinned buffers.
  cudaStream_t s = ex::api_stream();
  if (cudaMalloc(reinterpret_cast<void**>(&m->arena), m->data_bytes + 256) != cudaSuccess) return bail("cudaMalloc of the arena failed");
  uint8_t* pin[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  bool ok = true;
  for (int k = 0; k < 2 && ok; ++k)
    ok = cudaHostAlloc(reinterpret_cast<void**>(&pin[k]), STREAM_CHUNK, cudaHostAllocDefault) == cudaSuccess &&
         cudaEventCreateWithFlags(&ev[k], cudaEventDisableTiming) == cudaSuccess;
  uint64_t done = 0;
  for (int k = 0; ok && done < m->data_bytes; k ^= 1) {
    const size_t len = static_cast<size_t>(std::min<uint64_t>(STREAM_CHUNK, m->data_bytes - done));
    ok = cudaEventSynchronize(ev[k]) == cudaSuccess;  // the copy that last used this buffer has finished
    size_t got = 0;
    while (ok && got < len) {
      const ssize_t n = pread(r.fd, pin[k] + got, len - got, static_cast<off_t>(m->data_start + done + got));
      if (n <= 0) ok = false;
      else got += static_cast<size_t>(n);
    }
    ok = ok && cudaMemcpyAsync(m->arena + done, pin[k], len, cudaMemcpyHostToDevice, s) == cudaSuccess &&
         cudaEventRecord(ev[k], s) == cudaSuccess;
    done += len;
  }
  ok = ok && cudaMemsetAsync(m->arena + m->data_bytes, 0, 256, s) == cudaSuccess && cudaStreamSynchronize(s) == cudaSuccess;
  for (int k = 0; k < 2; ++k) {
    if (ev[k] != nullptr) cudaEventDestroy(ev[k]);
    if (pin[k] != nullptr) cudaFreeHost(pin[k]);
  }
  close(r.fd);
  if (!ok) {
    cudaFree(m->arena);
    return ex::api_fail(error, error_size, "gguf_load: %s: reading or copying the data section failed", path);
  }
  for (Tensor& t : m->tensors) {
    if (t.nbytes == 0 || t.offset % 16 != 0) continue;
    uint64_t rows = 1;
    for (int d = 1; d < t.n_dims; ++d) rows *= t.dims[d];
    if (rows > 0x7FFFFFFFu) continue;
    t.registered = edgexpu_cuda_register_weight(m->arena + t.offset, t.nbytes + 16, t.type, static_cast<int>(rows),
                                                static_cast<int>(t.dims[0]), nullptr, 0) == 1;
  }
  *model = m.release();
  return 1;
}

int edgexpu_cuda_gguf_tensor_count(const void* model) {
  return model == nullptr ? 0 : static_cast<int>(static_cast<const Model*>(model)->tensors.size());
}

int edgexpu_cuda_gguf_tensor_at(const void* model, int index, const char** name, const uint8_t** dev, uint32_t* type,
                                int64_t* n_in, int64_t* n_out, uint64_t* file_offset, uint64_t* nbytes) {
  if (model == nullptr) return 0;
  const Model* m = static_cast<const Model*>(model);
  if (index < 0 || index >= static_cast<int>(m->tensors.size())) return 0;
  const Tensor& t = m->tensors[static_cast<size_t>(index)];
  uint64_t rows = 1;
  for (int d = 1; d < t.n_dims; ++d) rows *= t.dims[d];
  if (name != nullptr) *name = t.name.c_str();
  if (dev != nullptr) *dev = m->arena + t.offset;
  if (type != nullptr) *type = t.type;
  if (n_in != nullptr) *n_in = static_cast<int64_t>(t.dims[0]);
  if (n_out != nullptr) *n_out = static_cast<int64_t>(rows);
  if (file_offset != nullptr) *file_offset = m->data_start + t.offset;
  if (nbytes != nullptr) *nbytes = t.registered ? t.nbytes : 0;
  return 1;
}

int edgexpu_cuda_gguf_find(const void* model, const char* name) {
  if (model == nullptr || name == nullptr) return -1;
  const Model* m = static_cast<const Model*>(model);
  for (size_t i = 0; i < m->tensors.size(); ++i)
    if (m->tensors[i].name == name) return static_cast<int>(i);
  return -1;
}

int edgexpu_cuda_gguf_meta(const void* model, const char* key, uint64_t* as_int, double* as_float, const char** as_str) {
  if (model == nullptr || key == nullptr) return 0;
  for (const Meta& e : static_cast<const Model*>(model)->meta) {
    if (e.key != key) continue;
    if (as_int != nullptr) *as_int = e.u;
    if (as_float != nullptr) *as_float = (e.type == GT_F32 || e.type == GT_F64) ? e.f : static_cast<double>(e.u);
    if (as_str != nullptr) *as_str = e.type == GT_STRING ? e.s.c_str() : nullptr;
    return static_cast<int>(e.type) + 1;
  }
  return 0;
}

int edgexpu_cuda_gguf_free(void* model) {
  if (model == nullptr) return 0;
  std::lock_guard<std::recursive_mutex> lk(ex::api_mutex());
  Model* m = static_cast<Model*>(model);
  for (const Tensor& t : m->tensors)
    if (t.registered) edgexpu_cuda_free_weight(m->arena + t.offset);
  cudaStreamSynchronize(ex::api_stream());
  cudaFree(m->arena);
  delete m;
  return 1;
}

}  // extern "C"
