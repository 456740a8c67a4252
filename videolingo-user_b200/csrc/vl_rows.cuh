// Block-per-row device routines for the few-row (decode-step) launches:
// residual add + LayerNorm / RMSNorm of one row by one block, shared by
// vl_norm.cu (its few-row path) and vl_decode_rows.cu (the fused decode-row
// launch).
//
// Reference semantics (VideoLingo-user native/asr/src):
//   residual_add_kernel (engine.cu:207-212, decoder.cu:933-938)
//   layer_norm_kernel (engine.cu:162-192), rmsnorm_kernel (decoder.cu:81-101)
// With one block per row every thread holds at most NV 16-byte vectors, and
// the norm weights are requested together with the row, so the launch
// costs one memory round trip and one block reduction however cold the
// caches are - the regime of a 64-row decode step, where a warp-per-row
// launch would put all rows on 8 SMs and fetch gamma only after the
// reduction.
#pragma once

#include "vl_common.cuh"

namespace vl {

constexpr int kRowBlockThreads = 256;

// Normalises row `row` of residual (+ delta) into out.  Every thread of the
// block must call it (it contains a barrier); `red` is 2 * warps floats of
// shared memory.  The block reduction sums the warps' partials in warp
// order, so a row's result does not depend on which launch computes it.
template <typename T, int NV, bool kDelta, bool kRms>
__device__ __forceinline__ void add_norm_row_block(T* residual, const T* delta,
                                                   const T* __restrict__ gamma,
                                                   const T* __restrict__ beta, T* out,
                                                   int64_t row, int cols, float eps,
                                                   float* red) {
  using S = Storage<T>;
  constexpr int E = S::kVec;
  constexpr int kWarps = kRowBlockThreads / 32;
  const int tid = threadIdx.x;
  const int nvec = cols / E;
  uint4* xrow = reinterpret_cast<uint4*>(residual + row * cols);
  const uint4* drow = reinterpret_cast<const uint4*>(kDelta ? delta + row * cols : nullptr);
  const uint4* gvec = reinterpret_cast<const uint4*>(gamma);
  const uint4* bvec = reinterpret_cast<const uint4*>(beta);

  uint4 h[NV], d[NV], g[NV], b[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = tid + kRowBlockThreads * i;
    if (v < nvec) {
      h[i] = ld_vec(xrow + v);
      if (kDelta) d[i] = ld_vec(drow + v);
      g[i] = __ldg(gvec + v);
      if (!kRms && beta != nullptr) b[i] = __ldg(bvec + v);
    }
  }
  float sum = 0.f, sq = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = tid + kRowBlockThreads * i;
    if (v < nvec) {
      float a[E];
      S::unpack(h[i], a);
      if (kDelta) {
        float c[E];
        S::unpack(d[i], c);
#pragma unroll
        for (int e = 0; e < E; ++e) a[e] = a[e] + c[e];
        h[i] = S::pack(a);  // rounded residual, as the reference stores it
        S::unpack(h[i], a); // statistics use the rounded value
        st_vec(xrow + v, h[i]);
      }
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if (!kRms) sum += a[e];
        sq += a[e] * a[e];
      }
    }
  }
  if (!kRms) sum = warp_sum(sum);
  sq = warp_sum(sq);
  const int warp = tid >> 5, lane = tid & 31;
  if (lane == 0) {
    red[warp] = sum;
    red[kWarps + warp] = sq;
  }
  __syncthreads();
  sum = 0.f;
  sq = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    if (!kRms) sum += red[w];
    sq += red[kWarps + w];
  }
  float mean = 0.f, inv;
  if (kRms) {
    inv = rsqrtf(sq / static_cast<float>(cols) + eps);
  } else {
    mean = sum / static_cast<float>(cols);
    const float var = fmaxf(sq / static_cast<float>(cols) - mean * mean, 0.f);
    inv = rsqrtf(var + eps);
  }
  uint4* orow = reinterpret_cast<uint4*>(out + row * cols);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = tid + kRowBlockThreads * i;
    if (v < nvec) {
      float a[E], gw[E], y[E];
      S::unpack(h[i], a);
      S::unpack(g[i], gw);
      if (kRms) {
#pragma unroll
        for (int e = 0; e < E; ++e) y[e] = a[e] * inv * gw[e];
      } else {
        float bw[E];
        if (beta != nullptr) {
          S::unpack(b[i], bw);
        } else {
#pragma unroll
          for (int e = 0; e < E; ++e) bw[e] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float normalized = (a[e] - mean) * inv;
          y[e] = normalized * gw[e] + bw[e];
        }
      }
      st_vec(orow + v, S::pack(y));
    }
  }
}

}  // namespace vl
