// Reference-kernel harness, decoder ops.  TEST INFRASTRUCTURE ONLY.
//
// Compiles the reference's own decoder.cu (VideoLingo-user
// native/asr/src/decoder.cu, included from where it lies; nothing is copied)
// and re-exports its anonymous-namespace kernels with the reference's launch
// shapes (decoder.cu:1497,1511,1520,1524,1601,1692,1710,1715).  The kernels
// have the GLM-ASR decoder's compile-time shapes: hidden 2048, 16 query and
// 4 KV heads of 128, full rotary 128, 1024-position tables, audio token
// 59260.  Default stream; the caller synchronises.
#include "decoder.cu"

namespace {

struct RopeTables {
  float* cos = nullptr;
  float* sin = nullptr;
  cudaError_t err = cudaSuccess;
  RopeTables() {
    const std::vector<float> c = build_full_rope_table(true), s = build_full_rope_table(false);
    err = cudaMalloc(&cos, c.size() * sizeof(float));
    if (err == cudaSuccess) err = cudaMalloc(&sin, s.size() * sizeof(float));
    if (err == cudaSuccess)
      err = cudaMemcpy(cos, c.data(), c.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (err == cudaSuccess)
      err = cudaMemcpy(sin, s.data(), s.size() * sizeof(float), cudaMemcpyHostToDevice);
  }
  ~RopeTables() {
    cudaDeviceSynchronize();
    cudaFree(cos);
    cudaFree(sin);
  }
};

}  // namespace

extern "C" {

int vlref_rmsnorm(void* x, const void* w, int rows, int hidden) {
  rmsnorm_kernel<<<rows, 256, 257 * sizeof(float)>>>(static_cast<half*>(x),
                                                     static_cast<const half*>(w), hidden);
  return static_cast<int>(cudaGetLastError());
}

int vlref_residual_add_dec(void* x, const void* delta, unsigned long long count) {
  residual_add_kernel<<<static_cast<unsigned>((count + 255) / 256), 256>>>(
      static_cast<half*>(x), static_cast<const half*>(delta), count);
  return static_cast<int>(cudaGetLastError());
}

int vlref_silu_mul(void* gate, const void* up, unsigned long long count) {
  silu_mul_kernel<<<static_cast<unsigned>((count + 255) / 256), 256>>>(
      static_cast<half*>(gate), static_cast<const half*>(up), count);
  return static_cast<int>(cudaGetLastError());
}

// Prefill RoPE: q [rows, 16*128], k [rows, 4*128], position = row % frames (< 1024).
int vlref_rope_rows(void* q, void* k, int rows, int frames) {
  RopeTables t;
  if (t.err != cudaSuccess) return static_cast<int>(t.err);
  rope_rows_kernel<<<rows, 64>>>(static_cast<half*>(q), static_cast<half*>(k), t.cos, t.sin, rows,
                                 frames);
  cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  return static_cast<int>(err);
}

// Decode RoPE at positions[active[r]] (< 1024).
int vlref_rope_map(void* q, void* k, const int* positions, const int* active, int rows) {
  RopeTables t;
  if (t.err != cudaSuccess) return static_cast<int>(t.err);
  rope_at_position_map_kernel<<<rows, 64>>>(static_cast<half*>(q), static_cast<half*>(k), t.cos,
                                            t.sin, positions, active, rows);
  cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  return static_cast<int>(err);
}

// Prompt gather for `group` chunks sharing ids [L]; audio [group, 375, 2048].
int vlref_gather_batch(const int64_t* ids, int L, const void* embed, const void* audio,
                       int audio_chunk_stride, void* out, int group) {
  gather_batch_kernel<<<dim3(L, group), 128>>>(ids, L, static_cast<const half*>(embed),
                                               static_cast<const half*>(audio), audio_chunk_stride,
                                               static_cast<half*>(out), group);
  return static_cast<int>(cudaGetLastError());
}

int vlref_gather_ids_mapped(const int64_t* ids, const int* active, const void* embed, void* out,
                            int rows) {
  gather_ids_mapped_kernel<<<rows, 128>>>(ids, active, static_cast<const half*>(embed),
                                          static_cast<half*>(out), rows);
  return static_cast<int>(cudaGetLastError());
}

// Decode KV append: row r -> cache + active[r]*chunk_stride + positions[active[r]]*512.
int vlref_append_kv_mapped(const void* k, const void* v, void* k_cache, void* v_cache,
                           const int* positions, const int* active, int rows,
                           unsigned long long chunk_stride) {
  const unsigned long long total = static_cast<unsigned long long>(rows) * 512;
  append_kv_mapped_kernel<<<static_cast<unsigned>((total + 255) / 256), 256>>>(
      static_cast<const half*>(k), static_cast<const half*>(v), static_cast<half*>(k_cache),
      static_cast<half*>(v_cache), positions, active, rows, chunk_stride);
  return static_cast<int>(cudaGetLastError());
}

// Decode attention (decoder.cu:1719-1722 launch shape): cache layout
// [chunk][layer][K|V][1024][512]; row r attends chunk active[r] over positions
// 0..positions[active[r]] (< 1024); q / out [rows][2048].
int vlref_attention_mapped(const void* q, const void* kv_cache, void* out, const int* positions,
                           const int* active, int rows, int layer,
                           unsigned long long layer_stride, unsigned long long chunk_stride) {
  attention_step_mapped_kernel<<<rows * kTextHeads, 128, (kMaxSequence + 128) * sizeof(float)>>>(
      static_cast<const half*>(q), static_cast<const half*>(kv_cache), static_cast<half*>(out),
      positions, active, rows, layer, layer_stride, chunk_stride);
  return static_cast<int>(cudaGetLastError());
}

// Kernel-only RoPE launchers for timing (bench.py --impl reference --ops):
// the reference's tables (kMaxSequence x 64 floats each) are built once into
// caller device buffers, so a timed launch is the kernel alone.
int vlref_fill_rope_tables(float* cos_dev, float* sin_dev) {
  const std::vector<float> c = build_full_rope_table(true), s = build_full_rope_table(false);
  cudaError_t err = cudaMemcpy(cos_dev, c.data(), c.size() * sizeof(float), cudaMemcpyHostToDevice);
  if (err == cudaSuccess)
    err = cudaMemcpy(sin_dev, s.data(), s.size() * sizeof(float), cudaMemcpyHostToDevice);
  return static_cast<int>(err);
}

int vlref_rope_rows_t(void* q, void* k, const float* cos_dev, const float* sin_dev, int rows,
                      int frames) {
  rope_rows_kernel<<<rows, 64>>>(static_cast<half*>(q), static_cast<half*>(k), cos_dev, sin_dev,
                                 rows, frames);
  return static_cast<int>(cudaGetLastError());
}

int vlref_rope_map_t(void* q, void* k, const float* cos_dev, const float* sin_dev,
                     const int* positions, const int* active, int rows) {
  rope_at_position_map_kernel<<<rows, 64>>>(static_cast<half*>(q), static_cast<half*>(k), cos_dev,
                                            sin_dev, positions, active, rows);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
