// Reference-kernel harness, encoder ops.  TEST INFRASTRUCTURE ONLY.
//
// Compiles the reference's own engine.cu (VideoLingo-user
// native/asr/src/engine.cu, included from where it lies via -I; nothing is
// copied) and re-exports its anonymous-namespace kernels through extern "C"
// launchers with the reference's own launch shapes (engine.cu:1013,1103,
// 1116, 881, 1365-1371), so GPU parity tests can run the reference
// implementation on the same inputs as libvlasr.  Default stream; the caller
// synchronises.
#include "engine.cu"

extern "C" {

int vlref_layer_norm(void* x, const void* w, const void* b, int rows, int cols) {
  layer_norm_kernel<<<rows, 256, 2 * 256 * sizeof(float)>>>(
      static_cast<half*>(x), static_cast<const half*>(w), static_cast<const half*>(b), rows, cols);
  return static_cast<int>(cudaGetLastError());
}

int vlref_residual_add_enc(void* x, const void* delta, unsigned long long count) {
  residual_add_kernel<<<static_cast<unsigned>((count + 255) / 256), 256>>>(
      static_cast<half*>(x), static_cast<const half*>(delta), count);
  return static_cast<int>(cudaGetLastError());
}

int vlref_gelu(void* x, unsigned long long count) {
  gelu_kernel<<<static_cast<unsigned>((count + 255) / 256), 256>>>(static_cast<half*>(x), count);
  return static_cast<int>(cudaGetLastError());
}

int vlref_add_bias(void* x, const void* bias, unsigned long long rows, int cols) {
  const unsigned long long count = rows * cols;
  add_bias_kernel<<<static_cast<unsigned>((count + 255) / 256), 256>>>(
      static_cast<half*>(x), static_cast<const half*>(bias), rows, cols);
  return static_cast<int>(cudaGetLastError());
}

// Encoder partial RoPE (20 heads x 64, rotary 32) on rows = chunks*1500,
// position = row % 1500, with the reference's host-built fp32 tables.
int vlref_encoder_rope(void* x, int rows) {
  const std::vector<float> cos_t = build_rope_table(true), sin_t = build_rope_table(false);
  float *d_cos = nullptr, *d_sin = nullptr;
  cudaError_t err = cudaMalloc(&d_cos, cos_t.size() * sizeof(float));
  if (err == cudaSuccess) err = cudaMalloc(&d_sin, sin_t.size() * sizeof(float));
  if (err == cudaSuccess)
    err = cudaMemcpy(d_cos, cos_t.data(), cos_t.size() * sizeof(float), cudaMemcpyHostToDevice);
  if (err == cudaSuccess)
    err = cudaMemcpy(d_sin, sin_t.data(), sin_t.size() * sizeof(float), cudaMemcpyHostToDevice);
  if (err == cudaSuccess) {
    const dim3 blocks((kRotaryDim / 2 + 63) / 64, rows);
    rope_kernel<<<blocks, 64>>>(static_cast<half*>(x), d_cos, d_sin, rows, kFrames);
    err = cudaGetLastError();
  }
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  cudaFree(d_cos);
  cudaFree(d_sin);
  return static_cast<int>(err);
}

}  // extern "C"
