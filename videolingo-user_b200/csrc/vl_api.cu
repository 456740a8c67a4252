// C ABI of libvlasr.so (declared in include/vl_api.h).
//
// Every entry point validates its arguments on the host before touching
// CUDA, maps failures onto the reference CLI's status taxonomy
// (native/asr/src/main_m0.cu:696-703: 2 = invalid input, 1 = execution
// failure) and records a message for vl_last_error().  No exception crosses
// the boundary, nothing is allocated and nothing synchronises.
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <tuple>

#include "vl_common.cuh"
#include "vl_kernels.h"

namespace {

thread_local char g_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_error[0] = '\0';
  return VL_OK;
}

int exec_status(cudaError_t err, const char* op) {
  if (err == cudaSuccess) return ok();
  return fail(VL_ERR_EXEC, "%s: CUDA error %d (%s)", op, static_cast<int>(err),
              cudaGetErrorString(err));
}

bool valid_dtype(int dtype) {
  return dtype == VL_F32 || dtype == VL_F16 || dtype == VL_BF16;
}

int64_t dtype_size(int dtype) { return dtype == VL_F32 ? 4 : 2; }

bool overlaps(const void* a, int64_t a_bytes, const void* b, int64_t b_bytes) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return x < y + static_cast<uintptr_t>(b_bytes) && y < x + static_cast<uintptr_t>(a_bytes);
}

constexpr int64_t kMaxRows = int64_t(1) << 40;
constexpr int64_t kMaxCols = int64_t(1) << 30;
constexpr int64_t kMaxMelChunks = int64_t(1) << 20;

}  // namespace

namespace vl {

int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
    v = 148;
  cache[dev].store(v, std::memory_order_relaxed);
  return v;
}

int resident_blocks(const void* kernel, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, int, size_t>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return sm_count();
  const auto key = std::make_tuple(dev, kernel, threads, smem);
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess ||
      per_sm <= 0) {
    (void)cudaGetLastError();
    per_sm = 1;
  }
  const int blocks = per_sm * sm_count();
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = blocks;
  return blocks;
}

}  // namespace vl

extern "C" {

int vl_version(void) { return 100; }

const char* vl_last_error(void) { return g_error; }

int vl_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  return n;
}

int vl_init(int device) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    (void)cudaGetLastError();
    count = 0;
  }
  if (device < 0 || device >= count)
    return fail(VL_ERR_INVALID, "vl_init: device %d not in [0, %d)", device, count);
  int prev = 0;
  cudaError_t err = cudaGetDevice(&prev);
  if (err == cudaSuccess) err = cudaSetDevice(device);
  if (err != cudaSuccess) return exec_status(err, "vl_init");
  (void)vl::sm_count();
  err = vl::prepare_gelu();
  if (err == cudaErrorStreamCaptureUnsupported) {
    (void)cudaSetDevice(prev);
    return fail(VL_ERR_INVALID, "vl_init: called while the legacy stream is being captured");
  }
  if (err == cudaSuccess) err = vl::prepare_logmel();
  const cudaError_t restore = cudaSetDevice(prev);
  if (err == cudaSuccess) err = restore;
  return exec_status(err, "vl_init");
}

int vl_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return fail(VL_ERR_INVALID, "vl_ipc_export: null pointer");
  return exec_status(vl::ipc_export(ptr, handle_out, offset_out), "vl_ipc_export");
}

int vl_ipc_open(const void* handle, void** base_out) {
  if (handle == nullptr || base_out == nullptr)
    return fail(VL_ERR_INVALID, "vl_ipc_open: null pointer");
  return exec_status(vl::ipc_open(handle, base_out), "vl_ipc_open");
}

int vl_ipc_close(void* base) {
  if (base == nullptr) return fail(VL_ERR_INVALID, "vl_ipc_close: null pointer");
  return exec_status(vl::ipc_close(base), "vl_ipc_close");
}

int vl_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return ok();
  if (dst == nullptr || src == nullptr) return fail(VL_ERR_INVALID, "vl_copy_async: null pointer");
  if (overlaps(dst, static_cast<int64_t>(bytes), src, static_cast<int64_t>(bytes)))
    return fail(VL_ERR_INVALID, "vl_copy_async: source and destination overlap");
  return exec_status(vl::copy_async(dst, src, bytes, static_cast<cudaStream_t>(stream)),
                     "vl_copy_async");
}

size_t vl_logmel_workspace_bytes(int64_t chunks) {
  if (chunks <= 0 || chunks > kMaxMelChunks) return 0;
  return vl::logmel_workspace_bytes(chunks);
}

int vl_logmel(const float* pcm, int64_t chunks, float* out, void* workspace,
              size_t workspace_bytes, void* stream) {
  if (pcm == nullptr || out == nullptr || workspace == nullptr)
    return fail(VL_ERR_INVALID, "vl_logmel: null pointer (pcm=%p out=%p workspace=%p)", pcm, out,
                workspace);
  if (chunks <= 0 || chunks > kMaxMelChunks)
    return fail(VL_ERR_INVALID, "vl_logmel: chunks must be in [1, %lld], got %lld",
                static_cast<long long>(kMaxMelChunks), static_cast<long long>(chunks));
  if (!vl::aligned16(pcm) || !vl::aligned16(out) || !vl::aligned16(workspace))
    return fail(VL_ERR_INVALID, "vl_logmel: pcm, out and workspace must be 16-byte aligned");
  const size_t need = vl::logmel_workspace_bytes(chunks);
  if (workspace_bytes < need)
    return fail(VL_ERR_INVALID, "vl_logmel: workspace holds %zu bytes, %zu needed", workspace_bytes,
                need);
  const int64_t in_bytes = chunks * VL_MEL_CHUNK_SAMPLES * 4;
  const int64_t out_bytes = chunks * VL_MEL_BINS * VL_MEL_FRAMES * 4;
  if (overlaps(pcm, in_bytes, out, out_bytes) || overlaps(workspace, static_cast<int64_t>(need), out, out_bytes) ||
      overlaps(workspace, static_cast<int64_t>(need), pcm, in_bytes))
    return fail(VL_ERR_INVALID, "vl_logmel: pcm, out and workspace must not overlap");
  return exec_status(vl::launch_logmel(pcm, chunks, out, static_cast<float*>(workspace),
                                       static_cast<cudaStream_t>(stream)),
                     "vl_logmel");
}

int vl_logmel_noalloc(const float* pcm, int64_t chunks, float* out, void* stream) {
  if (pcm == nullptr || out == nullptr)
    return fail(VL_ERR_INVALID, "vl_logmel_noalloc: null pointer (pcm=%p out=%p)", pcm, out);
  if (chunks <= 0 || chunks > VL_LOGMEL_NOALLOC_MAX_CHUNKS)
    return fail(VL_ERR_INVALID,
                "vl_logmel_noalloc: chunks must be in [1, %d] (the size of its fixed scratch "
                "array), got %lld; use vl_logmel with a workspace for more",
                VL_LOGMEL_NOALLOC_MAX_CHUNKS, static_cast<long long>(chunks));
  if (!vl::aligned16(pcm) || !vl::aligned16(out))
    return fail(VL_ERR_INVALID, "vl_logmel_noalloc: pcm and out must be 16-byte aligned");
  const int64_t in_bytes = chunks * VL_MEL_CHUNK_SAMPLES * 4;
  const int64_t out_bytes = chunks * VL_MEL_BINS * VL_MEL_FRAMES * 4;
  if (overlaps(pcm, in_bytes, out, out_bytes))
    return fail(VL_ERR_INVALID, "vl_logmel_noalloc: pcm and out must not overlap");
  return exec_status(vl::launch_logmel_noalloc(pcm, chunks, out, static_cast<cudaStream_t>(stream)),
                     "vl_logmel_noalloc");
}

static int check_norm(const char* op, void* residual, const void* delta, const void* weight,
                      void* out, int64_t rows, int64_t cols, float eps, int dtype) {
  if (residual == nullptr || weight == nullptr || out == nullptr)
    return fail(VL_ERR_INVALID, "%s: null pointer (residual=%p weight=%p out=%p)", op, residual,
                weight, out);
  if (!valid_dtype(dtype)) return fail(VL_ERR_INVALID, "%s: unsupported dtype %d", op, dtype);
  if (rows < 0 || rows > kMaxRows || cols <= 0 || cols > kMaxCols)
    return fail(VL_ERR_INVALID, "%s: bad shape rows=%lld cols=%lld", op,
                static_cast<long long>(rows), static_cast<long long>(cols));
  if (!(eps >= 0.f) || !std::isfinite(eps))
    return fail(VL_ERR_INVALID, "%s: eps must be finite and >= 0", op);
  if (delta != nullptr) {
    const int64_t bytes = rows * cols * dtype_size(dtype);
    if (overlaps(out, bytes, residual, bytes))
      return fail(VL_ERR_INVALID, "%s: out must not alias residual when delta is given", op);
    if (delta != out && overlaps(delta, bytes, residual, bytes))
      return fail(VL_ERR_INVALID, "%s: delta must not alias residual", op);
  }
  return VL_OK;
}

int vl_add_layernorm(void* residual, const void* delta, const void* gamma, const void* beta,
                     void* out, int64_t rows, int64_t cols, float eps, int dtype, void* stream) {
  const int st = check_norm("vl_add_layernorm", residual, delta, gamma, out, rows, cols, eps, dtype);
  if (st != VL_OK) return st;
  return exec_status(vl::launch_add_norm(residual, delta, gamma, beta, out, rows, cols, eps, false,
                                         dtype, static_cast<cudaStream_t>(stream)),
                     "vl_add_layernorm");
}

int vl_add_rmsnorm(void* residual, const void* delta, const void* weight, void* out, int64_t rows,
                   int64_t cols, float eps, int dtype, void* stream) {
  const int st = check_norm("vl_add_rmsnorm", residual, delta, weight, out, rows, cols, eps, dtype);
  if (st != VL_OK) return st;
  return exec_status(vl::launch_add_norm(residual, delta, weight, nullptr, out, rows, cols, eps,
                                         true, dtype, static_cast<cudaStream_t>(stream)),
                     "vl_add_rmsnorm");
}

int vl_gelu_erf(const void* in, const void* bias, void* out, int64_t rows, int64_t cols, int dtype,
                void* stream) {
  if (in == nullptr || out == nullptr)
    return fail(VL_ERR_INVALID, "vl_gelu_erf: null pointer (in=%p out=%p)", in, out);
  if (!valid_dtype(dtype)) return fail(VL_ERR_INVALID, "vl_gelu_erf: unsupported dtype %d", dtype);
  if (rows < 0 || rows > kMaxRows || cols < 0 || cols > kMaxCols)
    return fail(VL_ERR_INVALID, "vl_gelu_erf: bad shape rows=%lld cols=%lld",
                static_cast<long long>(rows), static_cast<long long>(cols));
  if (in != out) {
    const int64_t bytes = rows * cols * dtype_size(dtype);
    if (overlaps(in, bytes, out, bytes))
      return fail(VL_ERR_INVALID, "vl_gelu_erf: in and out overlap without being equal");
  }
  return exec_status(vl::launch_gelu(in, bias, out, rows, cols, dtype, static_cast<cudaStream_t>(stream)),
                     "vl_gelu_erf");
}

int vl_swiglu(const void* gate, const void* up, void* out, int64_t rows, int64_t cols,
              int64_t gate_stride, int64_t up_stride, int64_t out_stride, int dtype, void* stream) {
  if (gate == nullptr || up == nullptr || out == nullptr)
    return fail(VL_ERR_INVALID, "vl_swiglu: null pointer (gate=%p up=%p out=%p)", gate, up, out);
  if (!valid_dtype(dtype)) return fail(VL_ERR_INVALID, "vl_swiglu: unsupported dtype %d", dtype);
  if (rows < 0 || rows > kMaxRows || cols < 0 || cols > kMaxCols)
    return fail(VL_ERR_INVALID, "vl_swiglu: bad shape rows=%lld cols=%lld",
                static_cast<long long>(rows), static_cast<long long>(cols));
  if (gate_stride < cols || up_stride < cols || out_stride < cols)
    return fail(VL_ERR_INVALID, "vl_swiglu: row strides must be >= cols");
  if (out != gate && out != up && rows > 0 && cols > 0) {
    const int64_t es = dtype_size(dtype);
    const int64_t ob = ((rows - 1) * out_stride + cols) * es;
    if (overlaps(out, ob, gate, ((rows - 1) * gate_stride + cols) * es) ||
        overlaps(out, ob, up, ((rows - 1) * up_stride + cols) * es))
      return fail(VL_ERR_INVALID, "vl_swiglu: out overlaps an input without being equal to it");
  }
  return exec_status(vl::launch_swiglu(gate, up, out, rows, cols, gate_stride, up_stride, out_stride,
                                       dtype, static_cast<cudaStream_t>(stream)),
                     "vl_swiglu");
}

static int check_rope(const char* op, const void* q, const void* k, int64_t tokens, int n_q_heads,
                      int n_k_heads, int head_dim, int rotary_dim, double base,
                      int64_t q_row_stride, int64_t k_row_stride, int dtype) {
  if (q == nullptr && n_q_heads > 0) return fail(VL_ERR_INVALID, "%s: q is null", op);
  if ((k == nullptr) != (n_k_heads == 0))
    return fail(VL_ERR_INVALID, "%s: k must be null exactly when n_k_heads == 0", op);
  if (!valid_dtype(dtype)) return fail(VL_ERR_INVALID, "%s: unsupported dtype %d", op, dtype);
  if (tokens < 0 || tokens > kMaxRows || n_q_heads < 0 || n_k_heads < 0 ||
      n_q_heads + n_k_heads == 0)
    return fail(VL_ERR_INVALID, "%s: bad shape tokens=%lld heads=%d/%d", op,
                static_cast<long long>(tokens), n_q_heads, n_k_heads);
  if (head_dim <= 0 || rotary_dim <= 0 || rotary_dim % 2 != 0 || rotary_dim > head_dim ||
      rotary_dim > 256)
    return fail(VL_ERR_INVALID,
                "%s: rotary_dim must be even, in (0, min(head_dim, 256)] (head_dim=%d rotary_dim=%d)",
                op, head_dim, rotary_dim);
  if (!(base > 0.0) || !std::isfinite(base))
    return fail(VL_ERR_INVALID, "%s: base must be finite and > 0", op);
  if (q_row_stride < static_cast<int64_t>(n_q_heads) * head_dim ||
      (n_k_heads > 0 && k_row_stride < static_cast<int64_t>(n_k_heads) * head_dim))
    return fail(VL_ERR_INVALID, "%s: row strides must cover heads * head_dim", op);
  return VL_OK;
}

int vl_rope_inplace(void* q, void* k, const int32_t* positions, const int32_t* row_map,
                    int64_t positions_stride, int64_t pos_offset, int64_t tokens, int64_t seq_len,
                    int n_q_heads, int n_k_heads, int head_dim, int rotary_dim, double base,
                    int64_t q_row_stride, int64_t k_row_stride, int dtype, void* stream) {
  const int st = check_rope("vl_rope_inplace", q, k, tokens, n_q_heads, n_k_heads, head_dim,
                            rotary_dim, base, q_row_stride, k_row_stride, dtype);
  if (st != VL_OK) return st;
  if (seq_len < 0 || positions_stride < 0)
    return fail(VL_ERR_INVALID, "vl_rope_inplace: seq_len and positions_stride must be >= 0");
  if (row_map != nullptr && positions == nullptr)
    return fail(VL_ERR_INVALID, "vl_rope_inplace: row_map requires positions");
  if (n_q_heads == 0 && q == nullptr) q = k;  // only K rotates; q is never dereferenced
  vl::RopeArgs a{};
  a.q = q;
  a.k = k;
  a.positions = positions;
  a.row_map = row_map;
  a.positions_stride = positions_stride;
  a.pos_offset = pos_offset;
  a.tokens = tokens;
  a.seq_len = seq_len;
  a.n_q_heads = n_q_heads;
  a.n_k_heads = n_k_heads;
  a.head_dim = head_dim;
  a.rotary_dim = rotary_dim;
  a.base = base;
  a.q_row_stride = q_row_stride;
  a.k_row_stride = k_row_stride;
  return exec_status(vl::launch_rope(a, dtype, static_cast<cudaStream_t>(stream)), "vl_rope_inplace");
}

int vl_embed_gather(const int64_t* ids, int64_t batch, int64_t seq, int64_t ids_batch_stride,
                    const int32_t* row_map, const void* table, int64_t vocab, int64_t dim,
                    const void* audio, int64_t audio_token_id, int64_t audio_rows,
                    int64_t audio_batch_stride, void* out, int dtype, int32_t* status,
                    void* stream) {
  if (ids == nullptr || table == nullptr || out == nullptr)
    return fail(VL_ERR_INVALID, "vl_embed_gather: null pointer (ids=%p table=%p out=%p)", ids,
                table, out);
  if (!valid_dtype(dtype)) return fail(VL_ERR_INVALID, "vl_embed_gather: unsupported dtype %d", dtype);
  if (batch < 0 || seq < 0 || batch * seq > kMaxRows || vocab <= 0 || dim <= 0 || dim > kMaxCols ||
      ids_batch_stride < 0)
    return fail(VL_ERR_INVALID, "vl_embed_gather: bad shape batch=%lld seq=%lld vocab=%lld dim=%lld",
                static_cast<long long>(batch), static_cast<long long>(seq),
                static_cast<long long>(vocab), static_cast<long long>(dim));
  if (audio_token_id >= 0 && (audio == nullptr || audio_rows < 0 || audio_batch_stride < 0))
    return fail(VL_ERR_INVALID,
                "vl_embed_gather: audio substitution needs audio rows (audio=%p rows=%lld)", audio,
                static_cast<long long>(audio_rows));
  const int64_t es = dtype_size(dtype);
  return exec_status(
      vl::launch_embed_gather(ids, batch, seq, ids_batch_stride, row_map, table, vocab, dim * es,
                              audio, audio_token_id, audio_rows, audio_batch_stride * es, out,
                              status, static_cast<cudaStream_t>(stream)),
      "vl_embed_gather");
}

int vl_kv_append(const void* k, const void* v, void* k_cache, void* v_cache,
                 const int64_t* slot_mapping, int64_t tokens, int kv_heads, int head_dim,
                 int64_t k_row_stride, int64_t v_row_stride, int64_t num_slots, int dtype,
                 int32_t* status, void* stream) {
  if (k == nullptr || v == nullptr || k_cache == nullptr || v_cache == nullptr ||
      slot_mapping == nullptr)
    return fail(VL_ERR_INVALID, "vl_kv_append: null pointer");
  if (!valid_dtype(dtype)) return fail(VL_ERR_INVALID, "vl_kv_append: unsupported dtype %d", dtype);
  const int64_t row = static_cast<int64_t>(kv_heads) * head_dim;
  if (tokens < 0 || tokens > kMaxRows || kv_heads <= 0 || head_dim <= 0 || num_slots < 0 ||
      k_row_stride < row || v_row_stride < row)
    return fail(VL_ERR_INVALID, "vl_kv_append: bad shape tokens=%lld kv_heads=%d head_dim=%d",
                static_cast<long long>(tokens), kv_heads, head_dim);
  const int64_t es = dtype_size(dtype);
  return exec_status(vl::launch_kv_append(k, v, k_cache, v_cache, slot_mapping, tokens, row * es,
                                          k_row_stride * es, v_row_stride * es, num_slots, status,
                                          static_cast<cudaStream_t>(stream)),
                     "vl_kv_append");
}

int vl_rope_kv_append(void* q, void* k, const void* v, void* k_cache, void* v_cache,
                      const int32_t* positions, const int64_t* slot_mapping, int64_t tokens,
                      int n_q_heads, int n_k_heads, int head_dim, int rotary_dim, double base,
                      int64_t num_slots, int dtype, int32_t* status, void* stream) {
  const int64_t qs = static_cast<int64_t>(n_q_heads) * head_dim;
  const int64_t ks = static_cast<int64_t>(n_k_heads) * head_dim;
  const int st = check_rope("vl_rope_kv_append", q, k, tokens, n_q_heads, n_k_heads, head_dim,
                            rotary_dim, base, qs, ks, dtype);
  if (st != VL_OK) return st;
  if (k == nullptr || v == nullptr || k_cache == nullptr || v_cache == nullptr ||
      positions == nullptr || slot_mapping == nullptr)
    return fail(VL_ERR_INVALID, "vl_rope_kv_append: null pointer");
  if (num_slots < 0) return fail(VL_ERR_INVALID, "vl_rope_kv_append: num_slots must be >= 0");
  if (n_q_heads == 0 && q == nullptr) q = k;
  vl::RopeArgs a{};
  a.q = q;
  a.k = k;
  a.positions = positions;
  a.positions_stride = 1;
  a.tokens = tokens;
  a.n_q_heads = n_q_heads;
  a.n_k_heads = n_k_heads;
  a.head_dim = head_dim;
  a.rotary_dim = rotary_dim;
  a.base = base;
  a.q_row_stride = qs;
  a.k_row_stride = ks;
  a.v = v;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.slot_mapping = slot_mapping;
  a.num_slots = num_slots;
  a.status = status;
  return exec_status(vl::launch_rope(a, dtype, static_cast<cudaStream_t>(stream)),
                     "vl_rope_kv_append");
}

int vl_decode_rows(void* residual, const void* delta, const void* weight, void* out,
                   int64_t rows, int64_t cols, float eps, void* q, void* k, const void* v,
                   void* k_cache, void* v_cache, const int32_t* positions,
                   const int64_t* slot_mapping, int64_t tokens, int n_q_heads, int n_kv_heads,
                   int head_dim, int rotary_dim, double base, int64_t q_row_stride,
                   int64_t kv_row_stride, int64_t num_slots, int dtype, int32_t* status,
                   void* stream) {
  const char* op = "vl_decode_rows";
  if (!valid_dtype(dtype)) return fail(VL_ERR_INVALID, "%s: unsupported dtype %d", op, dtype);
  const int64_t E = 16 / dtype_size(dtype);
  if (rows < 0 || tokens < 0 || rows > (int64_t(1) << 30) || tokens > (int64_t(1) << 30))
    return fail(VL_ERR_INVALID, "%s: rows and tokens must be in [0, 2^30]", op);
  if (rows > 0) {
    const int st = check_norm(op, residual, delta, weight, out, rows, cols, eps, dtype);
    if (st != VL_OK) return st;
    if (cols % E != 0 || cols / E > 4 * 256)
      return fail(VL_ERR_INVALID, "%s: cols must be a multiple of %lld and at most %lld", op,
                  static_cast<long long>(E), static_cast<long long>(4 * 256 * E));
    if (!vl::aligned16(residual) || !vl::aligned16(weight) || !vl::aligned16(out) ||
        (delta != nullptr && !vl::aligned16(delta)))
      return fail(VL_ERR_INVALID, "%s: residual, delta, weight and out must be 16-byte aligned",
                  op);
  }
  if (tokens > 0) {
    const int st = check_rope(op, q, k, tokens, n_q_heads, n_kv_heads, head_dim, rotary_dim, base,
                              q_row_stride, kv_row_stride, dtype);
    if (st != VL_OK) return st;
    if (n_q_heads <= 0 || n_kv_heads <= 0 || v == nullptr || k_cache == nullptr ||
        v_cache == nullptr || positions == nullptr || slot_mapping == nullptr)
      return fail(VL_ERR_INVALID, "%s: q, k, v, caches, positions and slots are all needed", op);
    if (head_dim % E != 0 || (rotary_dim / 2) % E != 0 || q_row_stride % E != 0 ||
        kv_row_stride % E != 0)
      return fail(VL_ERR_INVALID,
                  "%s: head_dim, rotary_dim / 2 and the row strides must be multiples of %lld",
                  op, static_cast<long long>(E));
    if (!vl::aligned16(q) || !vl::aligned16(k) || !vl::aligned16(v) || !vl::aligned16(k_cache) ||
        !vl::aligned16(v_cache))
      return fail(VL_ERR_INVALID, "%s: q, k, v and the caches must be 16-byte aligned", op);
    if (num_slots < 0) return fail(VL_ERR_INVALID, "%s: num_slots must be >= 0", op);
    if (rows > 0) {
      const int64_t es = dtype_size(dtype);
      const int64_t nb = rows * cols * es;
      const void* norm_bufs[3] = {residual, out, delta};
      const void* tok_bufs[3] = {q, k, v};
      const int64_t tok_bytes[3] = {tokens * q_row_stride * es, tokens * kv_row_stride * es,
                                    tokens * kv_row_stride * es};
      for (const void* a : norm_bufs)
        for (int i = 0; i < 3; ++i)
          if (a != nullptr && overlaps(a, nb, tok_bufs[i], tok_bytes[i]))
            return fail(VL_ERR_INVALID, "%s: the norm rows must not overlap q, k or v", op);
    }
  }
  vl::DecodeRowsArgs a{};
  a.residual = residual;
  a.delta = delta;
  a.weight = weight;
  a.out = out;
  a.rows = rows;
  a.cols = static_cast<int>(cols);
  a.eps = eps;
  a.q = q;
  a.k = k;
  a.v = v;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.positions = positions;
  a.slot_mapping = slot_mapping;
  a.tokens = tokens;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.rotary_dim = rotary_dim;
  a.rope_base = base;
  a.q_row_stride = q_row_stride;
  a.kv_row_stride = kv_row_stride;
  a.num_slots = num_slots;
  a.status = status;
  return exec_status(vl::launch_decode_rows(a, dtype, static_cast<cudaStream_t>(stream)), op);
}

size_t vl_decode_attention_workspace_bytes(int64_t tokens, int n_q_heads, int n_kv_heads,
                                           int head_dim, int64_t max_seq_len) {
  if (tokens <= 0 || n_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % n_kv_heads != 0 ||
      head_dim <= 0 || max_seq_len <= 0 || max_seq_len > VL_DECODE_MAX_SEQ_LEN ||
      tokens > kMaxRows)
    return 0;
  return vl::decode_attention_workspace_bytes(tokens, n_q_heads, n_kv_heads, head_dim,
                                              max_seq_len);
}

int vl_decode_attention(const void* q, const void* k, const void* v, void* k_cache,
                        void* v_cache, const int32_t* positions, const int64_t* seq_start,
                        int64_t tokens, int n_q_heads, int n_kv_heads, int head_dim,
                        int rotary_dim, double rope_base, float scale, int64_t q_row_stride,
                        int64_t kv_row_stride, int64_t cache_row_stride, int64_t max_seq_len,
                        int64_t num_slots, void* out, int64_t out_row_stride, int dtype,
                        void* workspace, size_t workspace_bytes, int32_t* status, int flags,
                        void* stream) {
  const char* op = "vl_decode_attention";
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || positions == nullptr ||
      seq_start == nullptr || out == nullptr)
    return fail(VL_ERR_INVALID, "%s: null pointer", op);
  if ((k == nullptr) != (v == nullptr))
    return fail(VL_ERR_INVALID, "%s: k and v must both be given or both be null", op);
  if (dtype != VL_F16 && dtype != VL_BF16)
    return fail(VL_ERR_INVALID, "%s: unsupported dtype %d (f16 or bf16)", op, dtype);
  if ((flags & ~VL_LAUNCH_PDL) != 0)
    return fail(VL_ERR_INVALID, "%s: unknown flags 0x%x", op, flags);
  if (tokens < 0 || tokens > 0x7fffffff || n_q_heads <= 0 || n_kv_heads <= 0 ||
      n_kv_heads > 65535 || n_q_heads % n_kv_heads != 0)
    return fail(VL_ERR_INVALID, "%s: bad shape tokens=%lld heads=%d/%d", op,
                static_cast<long long>(tokens), n_q_heads, n_kv_heads);
  if (!vl::decode_attention_supported(head_dim, n_q_heads / n_kv_heads))
    return fail(VL_ERR_INVALID,
                "%s: unsupported head_dim %d / group %d (head_dim 64 or 128 with 1, 2, 4 or 8 "
                "query heads per kv head)", op, head_dim,
                n_q_heads / n_kv_heads);
  if (rotary_dim < 0 || rotary_dim % 2 != 0 || rotary_dim > head_dim)
    return fail(VL_ERR_INVALID, "%s: rotary_dim must be even, in [0, head_dim]", op);
  if (rotary_dim > 0 && k == nullptr)
    return fail(VL_ERR_INVALID, "%s: RoPE needs the new k row (k is null)", op);
  if (rotary_dim > 0 && (!(rope_base > 0.0) || !std::isfinite(rope_base)))
    return fail(VL_ERR_INVALID, "%s: rope_base must be finite and > 0", op);
  if (!std::isfinite(scale) || scale < 0.0f)
    return fail(VL_ERR_INVALID, "%s: scale must be finite and >= 0", op);
  if (max_seq_len <= 0 || max_seq_len > VL_DECODE_MAX_SEQ_LEN || num_slots < 0)
    return fail(VL_ERR_INVALID, "%s: max_seq_len must be in [1, %d], num_slots >= 0", op,
                VL_DECODE_MAX_SEQ_LEN);
  const int64_t qw = static_cast<int64_t>(n_q_heads) * head_dim;
  const int64_t kw = static_cast<int64_t>(n_kv_heads) * head_dim;
  if (q_row_stride < qw || out_row_stride < qw || cache_row_stride < kw ||
      (k != nullptr && kv_row_stride < kw))
    return fail(VL_ERR_INVALID, "%s: row strides must cover heads * head_dim", op);
  if (q_row_stride % 8 || out_row_stride % 8 || cache_row_stride % 8 ||
      (k != nullptr && kv_row_stride % 8))
    return fail(VL_ERR_INVALID, "%s: row strides must be multiples of 8 elements", op);
  if (!vl::aligned16(q) || !vl::aligned16(k_cache) || !vl::aligned16(v_cache) ||
      !vl::aligned16(out) || (k != nullptr && (!vl::aligned16(k) || !vl::aligned16(v))))
    return fail(VL_ERR_INVALID, "%s: q, k, v, caches and out must be 16-byte aligned", op);
  if (tokens == 0) return ok();
  const size_t need = vl::decode_attention_workspace_bytes(tokens, n_q_heads, n_kv_heads,
                                                           head_dim, max_seq_len);
  if (workspace == nullptr || workspace_bytes < need || !vl::aligned16(workspace))
    return fail(VL_ERR_INVALID, "%s: workspace of %zu bytes (16-byte aligned) required", op,
                need);
  if (overlaps(out, tokens * out_row_stride * 2, k_cache, num_slots * cache_row_stride * 2) ||
      overlaps(out, tokens * out_row_stride * 2, v_cache, num_slots * cache_row_stride * 2))
    return fail(VL_ERR_INVALID, "%s: out overlaps a cache", op);
  vl::DecodeAttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.positions = positions;
  a.seq_start = seq_start;
  a.out = out;
  a.tokens = tokens;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.rotary_dim = rotary_dim;
  a.rope_base = rope_base;
  a.scale = scale > 0.0f ? scale : 1.0f / std::sqrt(static_cast<float>(head_dim));
  a.q_row_stride = q_row_stride;
  a.kv_row_stride = kv_row_stride;
  a.cache_row_stride = cache_row_stride;
  a.out_row_stride = out_row_stride;
  a.max_seq_len = max_seq_len;
  a.num_slots = num_slots;
  a.status = status;
  return exec_status(
      vl::launch_decode_attention(a, dtype, workspace, (flags & VL_LAUNCH_PDL) != 0,
                                  static_cast<cudaStream_t>(stream)),
      op);
}

int vl_decode_linear_timeouts(uint32_t* count) {
  if (count == nullptr) return fail(VL_ERR_INVALID, "vl_decode_linear_timeouts: null pointer");
  unsigned int v = 0;
  const cudaError_t err = vl::read_linear_timeouts(&v);
  if (err == cudaSuccess) *count = v;
  return exec_status(err, "vl_decode_linear_timeouts");
}

int vl_decode_linear(const void* x, int64_t x_row_stride, const void* norm_weight,
                     const float* ssq_in, int ssq_in_parts, float eps, const void* w, int64_t n,
                     int64_t k, void* y, int64_t y_row_stride, float* ssq_out, int64_t rows,
                     int epilogue, int dtype, int flags, void* stream) {
  const char* op = "vl_decode_linear";
  if (x == nullptr || w == nullptr || y == nullptr)
    return fail(VL_ERR_INVALID, "%s: null pointer", op);
  if (dtype != VL_F16 && dtype != VL_BF16)
    return fail(VL_ERR_INVALID, "%s: unsupported dtype %d (f16 or bf16)", op, dtype);
  if ((flags & ~(VL_LAUNCH_PDL | VL_LINEAR_TCGEN05)) != 0)
    return fail(VL_ERR_INVALID, "%s: unknown flags 0x%x", op, flags);
  if (epilogue != VL_LINEAR_STORE && epilogue != VL_LINEAR_SWIGLU &&
      epilogue != VL_LINEAR_RESIDUAL)
    return fail(VL_ERR_INVALID, "%s: unknown epilogue %d", op, epilogue);
  if (rows < 0 || rows > VL_LINEAR_MAX_ROWS)
    return fail(VL_ERR_INVALID, "%s: rows must be in [0, %d]", op, VL_LINEAR_MAX_ROWS);
  if (k <= 0 || k % 512 != 0 || k > kMaxCols)
    return fail(VL_ERR_INVALID, "%s: k must be a positive multiple of 512", op);
  const int64_t align_n = epilogue == VL_LINEAR_SWIGLU ? 32 : 16;
  if (n <= 0 || n % align_n != 0 || n > (int64_t(1) << 28))
    return fail(VL_ERR_INVALID, "%s: n must be a positive multiple of %lld", op,
                static_cast<long long>(align_n));
  const int64_t out_cols = epilogue == VL_LINEAR_SWIGLU ? n / 2 : n;
  if (x_row_stride < k || x_row_stride % 8 != 0 || y_row_stride < out_cols)
    return fail(VL_ERR_INVALID, "%s: bad row strides", op);
  if (!vl::aligned16(x) || !vl::aligned16(w))
    return fail(VL_ERR_INVALID, "%s: x and w must be 16-byte aligned", op);
  if (norm_weight != nullptr) {
    if (ssq_in == nullptr || ssq_in_parts <= 0)
      return fail(VL_ERR_INVALID, "%s: the RMSNorm prologue needs ssq_in partial sums", op);
    if (!vl::aligned16(norm_weight))
      return fail(VL_ERR_INVALID, "%s: norm_weight must be 16-byte aligned", op);
    if (!(eps >= 0.0f) || !std::isfinite(eps))
      return fail(VL_ERR_INVALID, "%s: eps must be finite and >= 0", op);
  }
  if (ssq_out != nullptr && epilogue != VL_LINEAR_RESIDUAL)
    return fail(VL_ERR_INVALID, "%s: ssq_out is written by the RESIDUAL epilogue only", op);
  if (rows > 0 && overlaps(x, ((rows - 1) * x_row_stride + k) * 2, y,
                           ((rows - 1) * y_row_stride + out_cols) * 2))
    return fail(VL_ERR_INVALID, "%s: x overlaps y", op);
  vl::LinearArgs a{};
  a.x = x;
  a.x_row_stride = x_row_stride;
  a.norm_weight = norm_weight;
  a.ssq_in = ssq_in;
  a.ssq_in_parts = ssq_in_parts;
  a.eps = eps;
  a.w = w;
  a.n = n;
  a.k = k;
  a.y = y;
  a.y_row_stride = y_row_stride;
  a.ssq_out = ssq_out;
  a.rows = rows;
  a.epilogue = epilogue;
  return exec_status(vl::launch_decode_linear(a, dtype, (flags & VL_LAUNCH_PDL) != 0,
                                              (flags & VL_LINEAR_TCGEN05) != 0,
                                              static_cast<cudaStream_t>(stream)),
                     op);
}

int vl_argmax_eos(const void* logits, int64_t rows, int64_t vocab, int64_t row_stride,
                  const int32_t* row_chunk, int64_t chunks, uint8_t* finished,
                  int64_t* current_ids, int64_t* out_ids, int64_t out_rows, int64_t out_stride,
                  const int32_t* positions, const int64_t* prompt_length,
                  const int64_t* eos_ids, int n_eos, int64_t freeze_id, int dtype,
                  int32_t* status, void* stream) {
  const char* op = "vl_argmax_eos";
  if (logits == nullptr || current_ids == nullptr)
    return fail(VL_ERR_INVALID, "%s: null pointer", op);
  if (dtype != VL_F32 && dtype != VL_F16 && dtype != VL_BF16)
    return fail(VL_ERR_INVALID, "%s: unsupported dtype %d", op, dtype);
  if (rows < 0 || rows > 0x7fffffff || chunks < 0 || (row_chunk == nullptr && chunks < rows))
    return fail(VL_ERR_INVALID, "%s: bad rows=%lld chunks=%lld", op,
                static_cast<long long>(rows), static_cast<long long>(chunks));
  if (vocab <= 0 || vocab % 8 != 0 || vocab > (int64_t(1) << 24))
    return fail(VL_ERR_INVALID, "%s: vocab must be a positive multiple of 8, at most 2^24", op);
  if (row_stride < vocab || row_stride % 8 != 0)
    return fail(VL_ERR_INVALID, "%s: bad row stride", op);
  if (!vl::aligned16(logits))
    return fail(VL_ERR_INVALID, "%s: logits must be 16-byte aligned", op);
  if (n_eos < 0 || n_eos > 8 || (n_eos > 0 && eos_ids == nullptr))
    return fail(VL_ERR_INVALID, "%s: n_eos must be in [0, 8] with eos_ids given", op);
  if (out_ids != nullptr) {
    if (finished == nullptr || positions == nullptr || prompt_length == nullptr)
      return fail(VL_ERR_INVALID, "%s: out_ids needs finished, positions and prompt_length", op);
    if (out_rows <= 0 || out_stride < chunks)
      return fail(VL_ERR_INVALID, "%s: bad out_rows / out_stride", op);
  }
  vl::ArgmaxArgs a{};
  a.logits = logits;
  a.rows = rows;
  a.vocab = vocab;
  a.row_stride = row_stride;
  a.row_chunk = row_chunk;
  a.chunks = chunks;
  a.finished = finished;
  a.current_ids = current_ids;
  a.out_ids = out_ids;
  a.out_rows = out_rows;
  a.out_stride = out_stride;
  a.positions = positions;
  a.prompt_length = prompt_length;
  for (int e = 0; e < n_eos; ++e) a.eos[e] = eos_ids[e];
  a.n_eos = n_eos;
  a.freeze_id = freeze_id;
  a.status = status;
  return exec_status(vl::launch_argmax_eos(a, dtype, static_cast<cudaStream_t>(stream)), op);
}

}  // extern "C"
