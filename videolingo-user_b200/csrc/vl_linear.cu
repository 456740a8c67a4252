// Decode-step linear layers for sm_100a: y = x W^T for a few token rows
// (M <= 64) against a large weight matrix, with the neighbouring memory-bound
// steps fused in.
//
// Reference semantics (VideoLingo-user native/asr/src/decoder.cu, the
// per-layer decode sequence at :1692-1760): rmsnorm_kernel (:81-101,
// y = half(x * rsqrtf(sum(x^2)/H + 1e-5) * w)), cuBLAS GEMMs for q/k/v, o,
// gate, up, down and lm_head (`gemm`, :1002-1033: outputs rounded to the
// storage type), residual_add_kernel (:933-938, x = half(x + delta)) and
// silu_mul_kernel (:103-109, g = half(g / (1 + __expf(-g)) * u)).
//
// At decode the token rows are few, so the GEMM is a weight stream: every
// weight is read once and used M times.  One CTA owns 16 output columns (16
// rows of W with 8 warps; 16 gate + 16 up rows with 4 warps for the SwiGLU
// epilogue); each warp takes an equal slice of K and streams its part of
// those W rows, and of the x rows, through a private 3-stage cp.async ring
// of 64-wide k chunks (XOR-swizzled rows, warp-level waits only: no block
// barrier in the loop).  With the RMSNorm prologue the ring also carries the
// chunk's 64 norm weights, so the loop makes no dependent global load.
// The products run on the tensor cores (mma.sync m16n8k16, fp32
// accumulate): A = x rows from ldmatrix, B = W rows from ldmatrix.  The
// warps' partial sums meet in shared memory for the epilogue:
//   STORE     y = round(acc)
//   SWIGLU    y = round(silu(round(acc_gate)) * round(acc_up))
//   RESIDUAL  h = round(h + round(acc)) in place (each CTA owns its columns)
//             and the CTA's sum of squares of its 16 new h values per row
//             goes to ssq_out[cta][row], in a fixed order;
// and the optional RMSNorm prologue normalises x on the fly from those
// partial sums of the producer (summed in a fixed order, so results are
// deterministic): A = round(x * rsqrtf(sum/K + eps) * w[k]).
#include <atomic>

#include "vl_common.cuh"
#include "vl_kernels.h"

namespace vl {
namespace {

// Warps per CTA: 8 for the 16-row weight tiles (more bytes in flight per
// SM), 4 for the 32-row gate|up tiles of the SwiGLU epilogue (whose larger
// ring would otherwise leave one CTA per SM).
template <int EPI>
constexpr int lin_warps() { return EPI == VL_LINEAR_SWIGLU ? 4 : 8; }
#ifndef VL_LINEAR_STAGES
#define VL_LINEAR_STAGES 3
#endif
constexpr int kKc = 64;       // k per ring stage
constexpr int kCols = 16;     // output columns per CTA
constexpr size_t kLinRingBudget = 200 * 1024;

__device__ __forceinline__ unsigned lin_smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void lin_cp16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(lin_smem_u32(smem)),
               "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void lin_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void lin_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void lin_ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(lin_smem_u32(p)));
}
template <typename T>
__device__ __forceinline__ void lin_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                        uint32_t b1);
template <>
__device__ __forceinline__ void lin_mma<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void lin_mma<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2 storage values <-> 2 floats (low half = lower index)
template <typename T>
__device__ __forceinline__ float2 lin_unpack2(uint32_t w);
template <>
__device__ __forceinline__ float2 lin_unpack2<__nv_bfloat16>(uint32_t w) {
  return make_float2(bf16_lo(w), bf16_hi(w));
}
template <>
__device__ __forceinline__ float2 lin_unpack2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <typename T>
__device__ __forceinline__ uint32_t lin_pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t lin_pack2<__nv_bfloat16>(float lo, float hi) {
  return pack_bf16x2(lo, hi);
}
template <>
__device__ __forceinline__ uint32_t lin_pack2<__half>(float lo, float hi) {
  return pack_f16x2(lo, hi);
}

// offset (elements) of 16-byte chunk c of a 64-wide tile row r
__device__ __forceinline__ int lin_swz(int r, int c) { return r * kKc + ((c ^ (r & 7)) << 3); }

// Elements of one ring stage: W rows, x rows (padded to 16 * MT) and, with
// the RMSNorm prologue, the chunk's norm weights.
template <int MT, int EPI, bool NORM>
constexpr int lin_stage_elems() {
  return ((EPI == VL_LINEAR_SWIGLU ? 2 * kCols : kCols) + 16 * MT + (NORM ? 1 : 0)) * kKc;
}

// Ring stages per warp: VL_LINEAR_STAGES, fewer when the ring would not fit.
template <int MT, int EPI, bool NORM>
constexpr int lin_stages() {
  constexpr size_t per_stage = static_cast<size_t>(lin_warps<EPI>()) * lin_stage_elems<MT, EPI, NORM>() * 2;
  constexpr int fit = static_cast<int>(kLinRingBudget / per_stage);
  return fit < VL_LINEAR_STAGES ? (fit < 2 ? 2 : fit) : VL_LINEAR_STAGES;
}

template <int MT, int EPI, bool NORM>
constexpr size_t lin_ring_bytes() {
  return static_cast<size_t>(lin_warps<EPI>()) * lin_stages<MT, EPI, NORM>() *
         lin_stage_elems<MT, EPI, NORM>() * 2;
}

// Shared memory after the ring: 64 inverse RMS values, and for the RESIDUAL
// epilogue the [64][16] new residual values.  Keeping the SwiGLU CTA at
// about 73 KB lets three of them share an SM, so the 384 gate|up tiles of
// the decoder run in one wave.
template <int MT, int EPI, bool NORM>
constexpr size_t lin_smem_bytes() {
  return lin_ring_bytes<MT, EPI, NORM>() +
         (64 + (EPI == VL_LINEAR_RESIDUAL ? 64 * kCols : 0)) * sizeof(float);
}

template <typename T, int MT, int EPI, bool NORM>
__global__ void __launch_bounds__(lin_warps<EPI>() * 32)
    decode_linear_kernel(const __grid_constant__ LinearArgs a) {
  constexpr int kLinWarps = lin_warps<EPI>();
  constexpr int kLinThreads = kLinWarps * 32;
  using S = Storage<T>;
  constexpr int NTW = EPI == VL_LINEAR_SWIGLU ? 2 * kCols : kCols;  // W rows per CTA
  constexpr int MR = 16 * MT;                                          // x rows (padded)
  constexpr int W_EL = NTW * kKc, X_EL = MR * kKc, ST_EL = lin_stage_elems<MT, EPI, NORM>();
  constexpr int kStages = lin_stages<MT, EPI, NORM>();
  extern __shared__ __align__(128) unsigned char smem[];
  T* ring = reinterpret_cast<T*>(smem);
  float* inv_s = reinterpret_cast<float*>(smem + lin_ring_bytes<MT, EPI, NORM>());  // [64]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int cta = blockIdx.x;
  const int64_t col0 = static_cast<int64_t>(cta) * kCols;  // first output column
  const int kw = static_cast<int>(a.k / kLinWarps);
  const int kbase = warp * kw;
  const int nchunks = kw / kKc;
  T* my = ring + warp * kStages * ST_EL;
  const T* x = static_cast<const T*>(a.x);
  const T* w = static_cast<const T*>(a.w);
  const T* gam = static_cast<const T*>(a.norm_weight);

  // chunk c: the W rows and norm weights (inputs of the model), then the x rows
  auto issue_w = [&](int c) {
    T* st = my + (c % kStages) * ST_EL;
    const int64_t kk = kbase + static_cast<int64_t>(c) * kKc;
#pragma unroll
    for (int i = lane; i < NTW * 8; i += 32) {
      const int r = i >> 3, ch = i & 7;
      const int64_t wrow = (EPI == VL_LINEAR_SWIGLU && r >= kCols)
                               ? a.n / 2 + col0 + (r - kCols)
                               : col0 + r;
      lin_cp16(st + lin_swz(r, ch), w + wrow * a.k + kk + ch * 8, 16);
    }
    if (NORM && lane < kKc / 8) lin_cp16(st + W_EL + X_EL + lane * 8, gam + kk + lane * 8, 16);
  };
  auto issue_x = [&](int c) {
    T* st = my + (c % kStages) * ST_EL;
    const int64_t kk = kbase + static_cast<int64_t>(c) * kKc;
#pragma unroll
    for (int i = lane; i < MR * 8; i += 32) {
      const int r = i >> 3, ch = i & 7;
      const bool ok = r < a.rows;
      lin_cp16(st + W_EL + lin_swz(r, ch), x + (ok ? r : 0) * a.x_row_stride + kk + ch * 8,
               ok ? 16 : 0);
    }
  };
  // The first kStages-1 chunks: their weights in one group, issued before
  // the wait for the previous kernel (which may still be producing x and the
  // sums of squares), then their x rows in one group each.  Chunk c's data is
  // complete with commit group c + 1 before the loop and in it alike.
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s)
    if (s < nchunks) issue_w(s);
  lin_commit();
  pdl_wait();
  pdl_release();
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < nchunks) issue_x(s);
    lin_commit();
  }

  if (NORM) {
    // with the first weight tiles in flight: a warp per row, lane l sums the
    // partials l, l+32, ... in order, then a fixed xor tree (deterministic)
    for (int r = warp; r < a.rows; r += kLinWarps) {
      float ssq = 0.0f;
      for (int p = lane; p < a.ssq_in_parts; p += 32)
        ssq += a.ssq_in[static_cast<int64_t>(p) * a.rows + r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
      if (lane == 0) inv_s[r] = rsqrtf(ssq / static_cast<float>(a.k) + a.eps);
    }
    __syncthreads();
  }

  float acc[MT][NTW / 8][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NTW / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[mt][nt][e] = 0.0f;

  for (int c = 0; c < nchunks; ++c) {
    lin_wait<kStages - 2>();
    __syncwarp();  // the chunk is visible to the warp; the stage of chunk c-1 is free
    if (c + kStages - 1 < nchunks) {
      issue_w(c + kStages - 1);
      issue_x(c + kStages - 1);
    }
    lin_commit();
    const T* wt = my + (c % kStages) * ST_EL;
    const T* xt = wt + W_EL;
    const int mi = lane >> 3;
#pragma unroll
    for (int ks = 0; ks < kKc / 16; ++ks) {
      uint32_t bf[NTW / 8][2];
#pragma unroll
      for (int t2 = 0; t2 < NTW / 16; ++t2) {
        // matrices: (n-tile 2*t2, k 0-7), (2*t2, k 8-15), (2*t2+1, k 0-7), (2*t2+1, k 8-15)
        const int r = (2 * t2 + (mi >> 1)) * 8 + (lane & 7);
        uint32_t q[4];
        lin_ldsm_x4(q, wt + lin_swz(r, ks * 2 + (mi & 1)));
        bf[2 * t2][0] = q[0];
        bf[2 * t2][1] = q[1];
        bf[2 * t2 + 1][0] = q[2];
        bf[2 * t2 + 1][1] = q[3];
      }
      uint32_t g01 = 0u, g89 = 0u;
      if (NORM) {
        const T* gt = xt + X_EL + ks * 16 + 2 * tig;
        g01 = *reinterpret_cast<const uint32_t*>(gt);
        g89 = *reinterpret_cast<const uint32_t*>(gt + 8);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        uint32_t af[4];
        // matrices: (rows 0-7, k 0-7), (rows 8-15, k 0-7), (rows 0-7, k 8-15), (rows 8-15, k 8-15)
        const int r = mt * 16 + (mi & 1) * 8 + (lane & 7);
        lin_ldsm_x4(af, xt + lin_swz(r, ks * 2 + (mi >> 1)));
        if (NORM) {
          const int r0 = mt * 16 + gid, r1 = r0 + 8;
          const float i0 = r0 < a.rows ? inv_s[r0] : 0.0f;
          const float i1 = r1 < a.rows ? inv_s[r1] : 0.0f;
          const float2 ga = lin_unpack2<T>(g01), gb = lin_unpack2<T>(g89);
          float2 v;
          v = lin_unpack2<T>(af[0]);
          af[0] = lin_pack2<T>(v.x * i0 * ga.x, v.y * i0 * ga.y);
          v = lin_unpack2<T>(af[1]);
          af[1] = lin_pack2<T>(v.x * i1 * ga.x, v.y * i1 * ga.y);
          v = lin_unpack2<T>(af[2]);
          af[2] = lin_pack2<T>(v.x * i0 * gb.x, v.y * i0 * gb.y);
          v = lin_unpack2<T>(af[3]);
          af[3] = lin_pack2<T>(v.x * i1 * gb.x, v.y * i1 * gb.y);
        }
#pragma unroll
        for (int nt = 0; nt < NTW / 8; ++nt) lin_mma<T>(acc[mt][nt], af, bf[nt][0], bf[nt][1]);
      }
    }
  }
  lin_wait<0>();
  __syncthreads();  // every warp is done with its ring: reuse it for the cross-warp sums

  float* red = reinterpret_cast<float*>(smem);  // [warps][MR][NTW]
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NTW / 8; ++nt) {
      const int r0 = mt * 16 + gid, cc = nt * 8 + 2 * tig;
      red[(warp * MR + r0) * NTW + cc] = acc[mt][nt][0];
      red[(warp * MR + r0) * NTW + cc + 1] = acc[mt][nt][1];
      red[(warp * MR + r0 + 8) * NTW + cc] = acc[mt][nt][2];
      red[(warp * MR + r0 + 8) * NTW + cc + 1] = acc[mt][nt][3];
    }
  __syncthreads();
  auto total = [&](int row, int col) {
    float v = red[row * NTW + col];
#pragma unroll
    for (int wv = 1; wv < kLinWarps; ++wv) v += red[(wv * MR + row) * NTW + col];
    return v;
  };
  T* y = static_cast<T*>(a.y);
  float* hnew = inv_s + 64;  // [rows][16] new residual values (RESIDUAL)
  for (int i = tid; i < a.rows * kCols; i += kLinThreads) {
    const int row = i / kCols, j = i % kCols;
    T* dst = y + row * a.y_row_stride + col0 + j;
    if (EPI == VL_LINEAR_STORE) {
      *dst = S::from_float(total(row, j));
    } else if (EPI == VL_LINEAR_SWIGLU) {
      const float g = S::round_trip(total(row, j));
      const float u = S::round_trip(total(row, kCols + j));
      *dst = S::from_float(__fdividef(g, 1.0f + __expf(-g)) * u);
    } else {
      const float hv = S::round_trip(S::to_float(*dst) + S::round_trip(total(row, j)));
      *dst = S::from_float(hv);
      hnew[row * kCols + j] = hv;
    }
  }
  if (EPI == VL_LINEAR_RESIDUAL && a.ssq_out != nullptr) {
    __syncthreads();
    if (tid < a.rows) {
      float ssq = 0.0f;
#pragma unroll
      for (int j = 0; j < kCols; ++j) ssq = fmaf(hnew[tid * kCols + j], hnew[tid * kCols + j], ssq);
      a.ssq_out[static_cast<int64_t>(cta) * a.rows + tid] = ssq;
    }
  }
}

template <typename T, int MT, int EPI, bool NORM>
cudaError_t linear_launch(const LinearArgs& a, bool pdl, cudaStream_t stream) {
  constexpr size_t smem = lin_smem_bytes<MT, EPI, NORM>();
  static_assert(static_cast<size_t>(lin_warps<EPI>()) * 16 * MT * (EPI == VL_LINEAR_SWIGLU ? 2 * kCols : kCols) * 4 <=
                    lin_ring_bytes<MT, EPI, NORM>(),
                "the cross-warp sums must fit in the ring");
  static_assert(smem <= 227 * 1024, "decode linear shared memory");
  auto kernel = decode_linear_kernel<T, MT, EPI, NORM>;
  if (smem > 48 * 1024) {
    static std::atomic<bool> configured[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || !configured[dev].load(std::memory_order_acquire)) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      if (dev >= 0 && dev < 64) configured[dev].store(true, std::memory_order_release);
    }
  }
  const int64_t cols = a.epilogue == VL_LINEAR_SWIGLU ? a.n / 2 : a.n;
  return launch_kernel(kernel, dim3(static_cast<unsigned>(cols / kCols)),
                       dim3(lin_warps<EPI>() * 32), smem, stream, pdl, a);
}

template <typename T, int MT>
cudaError_t linear_mt(const LinearArgs& a, bool pdl, cudaStream_t stream) {
  const bool norm = a.norm_weight != nullptr;
  switch (a.epilogue) {
    case VL_LINEAR_STORE:
      return norm ? linear_launch<T, MT, VL_LINEAR_STORE, true>(a, pdl, stream)
                  : linear_launch<T, MT, VL_LINEAR_STORE, false>(a, pdl, stream);
    case VL_LINEAR_SWIGLU:
      return norm ? linear_launch<T, MT, VL_LINEAR_SWIGLU, true>(a, pdl, stream)
                  : linear_launch<T, MT, VL_LINEAR_SWIGLU, false>(a, pdl, stream);
    default:
      return norm ? linear_launch<T, MT, VL_LINEAR_RESIDUAL, true>(a, pdl, stream)
                  : linear_launch<T, MT, VL_LINEAR_RESIDUAL, false>(a, pdl, stream);
  }
}

template <typename T>
cudaError_t linear_typed(const LinearArgs& a, bool pdl, cudaStream_t stream) {
  if (a.rows <= 16) return linear_mt<T, 1>(a, pdl, stream);
  if (a.rows <= 32) return linear_mt<T, 2>(a, pdl, stream);
  return linear_mt<T, 4>(a, pdl, stream);
}

}  // namespace

cudaError_t launch_decode_linear(const LinearArgs& a, int dtype, bool pdl, bool tcgen05,
                                 cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  // On request, output columns in tiles of 128: the tcgen05 kernel
  // (vl_linear_tc.cu).  This kernel is the default: it streams a few-row
  // weight matrix over more SMs and measured faster at every row count (the
  // tcgen05 kernel's split-K clusters are limited to 15 of 8 CTAs).
  if (tcgen05 && decode_linear_tc_supported(a, dtype))
    return launch_decode_linear_tc(a, dtype, pdl, stream);
  if (dtype == kDtypeBF16) return linear_typed<__nv_bfloat16>(a, pdl, stream);
  if (dtype == kDtypeF16) return linear_typed<__half>(a, pdl, stream);
  return cudaErrorInvalidValue;
}

}  // namespace vl
