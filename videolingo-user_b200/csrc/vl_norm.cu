// Fused residual-add + LayerNorm / RMSNorm for sm_100a.
//
// Reference semantics (VideoLingo-user native/asr/src):
//   residual_add_kernel   engine.cu:207-212, decoder.cu:933-938
//       x = half(float(x) + float(delta))
//   layer_norm_kernel     engine.cu:162-192
//       mean = sum(x)/n, var = sum(x^2)/n - mean^2, inv = rsqrtf(var + eps)
//       y = half((x - mean) * inv * w + b)
//   rmsnorm_kernel        decoder.cu:81-101
//       inv = rsqrtf(sum(x^2)/n + eps), y = half(x * inv * w)
// The engine runs add -> memcpy -> norm as three passes plus a copy
// (engine.cu:1544-1552, decoder.cu:1591-1597); here it is one pass that
// reads residual and delta once and writes the new residual and the
// normalised row once (4 row transfers instead of 7).
//
// Layout: one warp owns one row (few-row launches: one block per row, see
// vl_rows.cuh).  The row is held in registers as packed
// 16-byte vectors (NV per lane), the moments are reduced with warp shuffles
// (no shared memory, no block barrier), and the output pass re-reads only the
// L1/L2-resident gamma/beta.  Rows that do not fit the register path (length
// not a multiple of the 16-byte vector, unaligned pointers, > 16 vectors per
// lane) take a block-per-row fallback that streams the row twice.
#include "vl_common.cuh"
#include "vl_kernels.h"
#include "vl_rows.cuh"

namespace vl {
namespace {

constexpr int kNormThreads = 256;  // 8 rows per block
// Up to this many rows per SM take the block-per-row path: a launch of that
// size is latency-bound (one memory round trip), and spreading the rows over
// more SMs shortens it; above it the warp-per-row stream is the faster one.
constexpr int kFewRowsPerSm = 2;

template <typename T, int NV, bool kDelta, bool kRms>
__global__ void __launch_bounds__(kNormThreads)
    add_norm_warp_kernel(T* residual, const T* delta, const T* __restrict__ gamma,
                         const T* __restrict__ beta, T* out, int64_t rows, int cols, float eps) {
  using S = Storage<T>;
  constexpr int E = S::kVec;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kNormThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = cols / E;
  const uint4* xrow = reinterpret_cast<const uint4*>(residual + row * cols);
  const uint4* drow = reinterpret_cast<const uint4*>(kDelta ? delta + row * cols : nullptr);

  uint4 h[NV];
  uint4 d[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
      h[i] = ld_vec(xrow + v);
      if (kDelta) d[i] = ld_vec(drow + v);
    }
  }

  float sum = 0.f, sq = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
      float a[E];
      S::unpack(h[i], a);
      if (kDelta) {
        float b[E];
        S::unpack(d[i], b);
#pragma unroll
        for (int e = 0; e < E; ++e) a[e] = a[e] + b[e];
        h[i] = S::pack(a);          // rounded residual, as the reference stores it
        S::unpack(h[i], a);         // statistics use the rounded value
        st_vec(reinterpret_cast<uint4*>(residual + row * cols) + v, h[i]);
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

  float mean = 0.f, inv;
  if (kRms) {
    inv = rsqrtf(sq / static_cast<float>(cols) + eps);
  } else {
    mean = sum / static_cast<float>(cols);
    const float var = fmaxf(sq / static_cast<float>(cols) - mean * mean, 0.f);
    inv = rsqrtf(var + eps);
  }

  uint4* orow = reinterpret_cast<uint4*>(out + row * cols);
  const uint4* gvec = reinterpret_cast<const uint4*>(gamma);
  const uint4* bvec = reinterpret_cast<const uint4*>(beta);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = lane + 32 * i;
    if (v < nvec) {
      float a[E], g[E], y[E];
      S::unpack(h[i], a);
      S::unpack(__ldg(gvec + v), g);
      if (kRms) {
#pragma unroll
        for (int e = 0; e < E; ++e) y[e] = a[e] * inv * g[e];
      } else {
        float b[E];
        if (beta != nullptr) {
          S::unpack(__ldg(bvec + v), b);
        } else {
#pragma unroll
          for (int e = 0; e < E; ++e) b[e] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float normalized = (a[e] - mean) * inv;
          y[e] = normalized * g[e] + b[e];
        }
      }
      st_vec(orow + v, S::pack(y));
    }
  }
}

// Any length / alignment: one block per row, two passes over global memory
// (the second pass hits L1/L2).
template <typename T, bool kRms>
__global__ void __launch_bounds__(kNormThreads)
    add_norm_block_kernel(T* residual, const T* delta, const T* __restrict__ gamma,
                          const T* __restrict__ beta, T* out, int64_t rows, int64_t cols,
                          float eps) {
  using S = Storage<T>;
  __shared__ float red_sum[kNormThreads / 32];
  __shared__ float red_sq[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  if (row >= rows) return;
  T* xrow = residual + row * cols;
  const T* drow = delta ? delta + row * cols : nullptr;
  float sum = 0.f, sq = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    float a = S::to_float(xrow[c]);
    if (drow) {
      const T r = S::from_float(a + S::to_float(drow[c]));
      xrow[c] = r;
      a = S::to_float(r);
    }
    sum += a;
    sq += a * a;
  }
  sum = warp_sum(sum);
  sq = warp_sum(sq);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red_sum[warp] = sum;
    red_sq[warp] = sq;
  }
  __syncthreads();
  sum = 0.f;
  sq = 0.f;
  for (int w = 0; w < kNormThreads / 32; ++w) {
    sum += red_sum[w];
    sq += red_sq[w];
  }
  float mean = 0.f, inv;
  if (kRms) {
    inv = rsqrtf(sq / static_cast<float>(cols) + eps);
  } else {
    mean = sum / static_cast<float>(cols);
    const float var = fmaxf(sq / static_cast<float>(cols) - mean * mean, 0.f);
    inv = rsqrtf(var + eps);
  }
  // Each thread re-reads exactly the elements it wrote in pass 1, so the
  // residual update is visible to it without a barrier.
  T* orow = out + row * cols;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float a = S::to_float(xrow[c]);
    const float g = S::to_float(gamma[c]);
    float y;
    if (kRms) {
      y = a * inv * g;
    } else {
      const float b = beta ? S::to_float(beta[c]) : 0.f;
      const float normalized = (a - mean) * inv;
      y = normalized * g + b;
    }
    orow[c] = S::from_float(y);
  }
}

// Few rows (a decode step): one block per row (vl_rows.cuh), so 64 rows run
// on 64 SMs with the norm weights fetched alongside the row.
template <typename T, int NV, bool kDelta, bool kRms>
__global__ void __launch_bounds__(kRowBlockThreads)
    add_norm_row_kernel(T* residual, const T* delta, const T* __restrict__ gamma,
                        const T* __restrict__ beta, T* out, int cols, float eps) {
  __shared__ float red[2 * kRowBlockThreads / 32];
  add_norm_row_block<T, NV, kDelta, kRms>(residual, delta, gamma, beta, out, blockIdx.x, cols,
                                          eps, red);
}

template <typename T, int NV, bool kRms>
cudaError_t launch_row(void* residual, const void* delta, const void* gamma, const void* beta,
                       void* out, int64_t rows, int64_t cols, float eps, cudaStream_t stream) {
  if (delta)
    add_norm_row_kernel<T, NV, true, kRms><<<static_cast<unsigned>(rows), kRowBlockThreads, 0,
                                             stream>>>(
        static_cast<T*>(residual), static_cast<const T*>(delta), static_cast<const T*>(gamma),
        static_cast<const T*>(beta), static_cast<T*>(out), static_cast<int>(cols), eps);
  else
    add_norm_row_kernel<T, NV, false, kRms><<<static_cast<unsigned>(rows), kRowBlockThreads, 0,
                                              stream>>>(
        static_cast<T*>(residual), nullptr, static_cast<const T*>(gamma),
        static_cast<const T*>(beta), static_cast<T*>(out), static_cast<int>(cols), eps);
  return cudaGetLastError();
}

template <typename T, int NV, bool kRms>
cudaError_t launch_warp(void* residual, const void* delta, const void* gamma, const void* beta,
                        void* out, int64_t rows, int64_t cols, float eps, cudaStream_t stream) {
  const int64_t blocks = (rows + kNormThreads / 32 - 1) / (kNormThreads / 32);
  if (delta) {
    add_norm_warp_kernel<T, NV, true, kRms><<<static_cast<unsigned>(blocks), kNormThreads, 0, stream>>>(
        static_cast<T*>(residual), static_cast<const T*>(delta), static_cast<const T*>(gamma),
        static_cast<const T*>(beta), static_cast<T*>(out), rows, static_cast<int>(cols), eps);
  } else {
    add_norm_warp_kernel<T, NV, false, kRms><<<static_cast<unsigned>(blocks), kNormThreads, 0, stream>>>(
        static_cast<T*>(residual), nullptr, static_cast<const T*>(gamma),
        static_cast<const T*>(beta), static_cast<T*>(out), rows, static_cast<int>(cols), eps);
  }
  return cudaGetLastError();
}

template <typename T, bool kRms>
cudaError_t dispatch(void* residual, const void* delta, const void* gamma, const void* beta,
                     void* out, int64_t rows, int64_t cols, float eps, cudaStream_t stream) {
  constexpr int E = Storage<T>::kVec;
  const bool vec_ok = (cols % E == 0) && aligned16(residual) && aligned16(out) &&
                      aligned16(gamma) && (delta == nullptr || aligned16(delta)) &&
                      (beta == nullptr || aligned16(beta));
  const int64_t per_lane = (cols / E + 31) / 32;
  const int64_t per_thread = (cols / E + kRowBlockThreads - 1) / kRowBlockThreads;
  if (vec_ok && rows <= kFewRowsPerSm * sm_count() && per_thread <= 4) {
    switch (per_thread) {
      case 1: return launch_row<T, 1, kRms>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
      case 2: return launch_row<T, 2, kRms>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
      default: return launch_row<T, 4, kRms>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
    }
  }
  if (vec_ok && per_lane <= 16) {
    switch (per_lane) {
      case 1: return launch_warp<T, 1, kRms>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
      case 2: return launch_warp<T, 2, kRms>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
      case 3:
      case 4: return launch_warp<T, 4, kRms>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
      case 5: return launch_warp<T, 5, kRms>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
      case 6:
      case 7:
      case 8: return launch_warp<T, 8, kRms>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
      case 9:
      case 10: return launch_warp<T, 10, kRms>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
      default: return launch_warp<T, 16, kRms>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
    }
  }
  add_norm_block_kernel<T, kRms><<<static_cast<unsigned>(rows), kNormThreads, 0, stream>>>(
      static_cast<T*>(residual), static_cast<const T*>(delta), static_cast<const T*>(gamma),
      static_cast<const T*>(beta), static_cast<T*>(out), rows, cols, eps);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_add_norm(void* residual, const void* delta, const void* gamma,
                            const void* beta, void* out, int64_t rows, int64_t cols, float eps,
                            bool rms, int dtype, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  switch (dtype) {
    case kDtypeF32:
      return rms ? dispatch<float, true>(residual, delta, gamma, beta, out, rows, cols, eps, stream)
                 : dispatch<float, false>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
    case kDtypeF16:
      return rms ? dispatch<__half, true>(residual, delta, gamma, beta, out, rows, cols, eps, stream)
                 : dispatch<__half, false>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
    default:
      return rms ? dispatch<__nv_bfloat16, true>(residual, delta, gamma, beta, out, rows, cols, eps, stream)
                 : dispatch<__nv_bfloat16, false>(residual, delta, gamma, beta, out, rows, cols, eps, stream);
  }
}

}  // namespace vl
