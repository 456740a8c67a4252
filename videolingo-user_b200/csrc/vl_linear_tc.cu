// Decode-step linear layers on the Blackwell tensor cores (tcgen05 + TMA +
// TMEM), for sm_100a: y = x W^T for a few token rows (<= 64) against a large
// weight matrix, with the same fused prologue and epilogues as vl_linear.cu.
//
// Reference semantics (VideoLingo-user native/asr/src/decoder.cu, the
// per-layer decode sequence at :1692-1760): rmsnorm_kernel (:81-101), the
// cuBLAS projections (`gemm`, :1002-1033, outputs rounded to the storage
// type), residual_add_kernel (:933-938) and silu_mul_kernel (:103-109).
//
// Shape of the problem: the weights stream once from HBM and every weight
// is used by only a handful of token rows, so the kernel is a weight stream
// with a tiny matrix product attached.  Design ("swap AB"):
//   * the 128 output columns of a CTA are the MMA's M = 128 (the weight rows,
//     operand A) and the token rows, padded to 16 / 32 / 64, are its N
//     (operand B) - so a 16-row decode step still fills the M=128 tile;
//   * K is split over a thread-block cluster of S CTAs (S <= 8) so that the
//     small weight matrices of a decode step still spread over ~150 SMs; the
//     S partial accumulators are summed through distributed shared memory,
//     each CTA of the cluster finishing NR / S of the token rows, in a fixed
//     order (deterministic);
//   * one thread streams the CTA's weight tiles (128 rows x 64 k, 128-byte
//     swizzle) with TMA into a ring of up to 6 stages guarded by mbarriers -
//     for most decode projections the whole K slice is in flight at once,
//     issued before the programmatic-dependent-launch wait because weights
//     never depend on the previous kernel;
//   * the CTA's slice of x (and, with the RMSNorm prologue, x normalised by
//     the producer's partial sums of squares and the norm weight) is written
//     by all threads into shared memory in the same swizzled K-major layout;
//   * one thread issues tcgen05.mma (kind::f16, fp32 accumulate in TMEM);
//     tcgen05.commit frees ring stages and signals the end;
//   * the four warps read the accumulator back with tcgen05.ld (warp w owns
//     TMEM lanes 32w..32w+31 = output columns) for the cluster reduction and
//     the epilogue: STORE, SWIGLU (gate and up tiles accumulate side by side)
//     or RESIDUAL (h += y in place, plus the per-16-column sums of squares
//     the next RMSNorm prologue consumes, in the same format as vl_linear.cu).
// Every mbarrier wait is bounded: on expiry the CTA stops issuing, waits (also
// bounded) for its own copies, still meets its cluster barriers, frees its
// TMEM, writes NaN for its outputs and counts the event in a device word
// (vl_decode_linear_timeouts()).  No TMA load here uses cluster multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <map>
#include <mutex>
#include <tuple>

#include "vl_common.cuh"
#include "vl_kernels.h"

namespace vl {

// Bounded-wait expiries of the tensor-core decode linear, per device.
__device__ unsigned int g_linear_wait_timeouts;

namespace {

constexpr int kTcThreads = 128;
constexpr int kTileM = 128;                 // output columns per CTA (MMA M)
constexpr int kTileK = 64;                  // k per stage: 64 x 2 B = one 128-byte swizzle row
constexpr int kTileBytes = kTileM * kTileK * 2;  // 16 KB per weight tile
constexpr int kMaxStages = 8;
constexpr size_t kSmemBudget = 220 * 1024;
constexpr uint32_t kWaitLimit = 1u << 22;   // try_wait polls before a wait gives up (~seconds)

__device__ __forceinline__ uint32_t su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity to complete; false if the bound ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle
// layout: 8-row groups 1024 bytes apart (stride byte offset), version 1,
// layout type 2 (SWIZZLE_128B).  The k-th 16-element step inside the
// 128-byte row is the same descriptor with the start address + 32 k bytes.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3fff);          // start address
  d |= static_cast<uint64_t>(1) << 16;                          // leading byte offset (unused)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;                  // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;                          // version (sm100)
  d |= static_cast<uint64_t>(2) << 61;                          // SWIZZLE_128B
  return d;
}

// Instruction descriptor of kind::f16 with fp32 accumulation, both operands
// K-major, M = 128, N = n.
template <typename T>
__host__ __device__ constexpr uint32_t mma_idesc(int n) {
  return (1u << 4)                                            // D format F32
         | ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 7)   // A format
         | ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 10)  // B format
         | (static_cast<uint32_t>(n >> 3) << 17)              // N >> 3
         | (static_cast<uint32_t>(kTileM >> 4) << 24);        // M >> 4
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   su32(bar))
               : "memory");
}

// 16 consecutive fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Store a float to CTA `rank`'s shared memory at the address of `local` in
// this CTA (visible to it after the next cluster barrier).
__device__ __forceinline__ void st_cluster_f32(float* local, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(su32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(su32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}

template <typename T>
__device__ __forceinline__ float2 tc_unpack2(uint32_t w);
template <>
__device__ __forceinline__ float2 tc_unpack2<__nv_bfloat16>(uint32_t w) {
  return make_float2(bf16_lo(w), bf16_hi(w));
}
template <>
__device__ __forceinline__ float2 tc_unpack2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <typename T>
__device__ __forceinline__ uint32_t tc_pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t tc_pack2<__nv_bfloat16>(float lo, float hi) {
  return pack_bf16x2(lo, hi);
}
template <>
__device__ __forceinline__ uint32_t tc_pack2<__half>(float lo, float hi) {
  return pack_f16x2(lo, hi);
}

struct TcLayout {
  int stages;
  int chunks;        // k tiles of this CTA
  size_t ring;       // bytes
  size_t xs;         // bytes of the x slice
  size_t part;       // bytes of the partial accumulators
  size_t norm;       // RMSNorm prologue: the partial sums [k/16][rows] and this CTA's norm weights
  size_t total;      // dynamic shared memory (incl. 1 KB alignment slack)
};

// budget: shared memory one CTA may take (so that the grid's CTAs are
// resident in one wave, see tc_budget).
__host__ __device__ inline TcLayout tc_layout(int nr, int epi, int64_t k, int splits,
                                              int max_stages, size_t budget, bool norm) {
  TcLayout L{};
  L.chunks = static_cast<int>(k / kTileK / splits);
  const int tiles = epi == VL_LINEAR_SWIGLU ? 2 : 1;
  L.xs = static_cast<size_t>(nr) * 128 * L.chunks;
  L.part = static_cast<size_t>(tiles) * nr * kTileM * 4;
  L.norm = norm ? static_cast<size_t>(k / 16) * nr * 4 + static_cast<size_t>(L.chunks) * 128 : 0;
  L.stages = L.chunks < max_stages ? L.chunks : max_stages;
  while (L.stages > 1 && static_cast<size_t>(L.stages) * tiles * kTileBytes + L.xs + L.part +
                                 L.norm + 2048 > budget)
    --L.stages;
  L.ring = static_cast<size_t>(L.stages) * tiles * kTileBytes;
  L.total = L.ring + L.xs + L.part + L.norm + 1024 /*align*/ + 1024 /*barriers, tmem slot, inv*/;
  return L;
}

template <typename T, int NR, int EPI, bool NORM>
__global__ void __launch_bounds__(kTcThreads, 1)
    decode_linear_tc_kernel(const __grid_constant__ LinearArgs a,
                            const __grid_constant__ CUtensorMap wmap, int splits, int max_stages,
                            unsigned int budget) {
  using S = Storage<T>;
  constexpr int kTiles = EPI == VL_LINEAR_SWIGLU ? 2 : 1;
  constexpr int kAccCols = kTiles * NR;
  constexpr uint32_t kTmemCols = kAccCols <= 32 ? 32 : (kAccCols <= 64 ? 64 : 128);
  const TcLayout L = tc_layout(NR, EPI, a.k, splits, max_stages, budget, NORM);

  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* ring = base;
  unsigned char* xs = ring + L.ring;
  float* part = reinterpret_cast<float*>(xs + L.xs);  // [kTiles][NR][128]
  // NORM: the producer's partial sums of squares [k/16][rows], then this
  // CTA's k slice of the norm weight
  float* ssq_s = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(part) + L.part);
  T* gam_s = reinterpret_cast<T*>(ssq_s + (NORM ? (a.k / 16) * NR : 0));
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(part) + L.part +
                                               L.norm);
  uint64_t* full = bars;                    // [stages]
  uint64_t* empty = bars + kMaxStages;      // [stages]
  uint64_t* done = bars + 2 * kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 1);
  int* bad = reinterpret_cast<int*>(tmem_slot + 1);
  int* issued_s = reinterpret_cast<int*>(tmem_slot + 2);
  float* inv_s = reinterpret_cast<float*>(tmem_slot + 3);  // [64]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * kTileM;
  const uint32_t rank = splits > 1 ? cluster_rank() : 0u;
  const int64_t kbase = static_cast<int64_t>(rank) * L.chunks * kTileK;
  const int64_t up_row = EPI == VL_LINEAR_SWIGLU ? a.n / 2 : 0;

  // Weight tile c into ring stage c % stages (thread 0).
  auto issue = [&](int c) {
    const int s = c % L.stages;
    unsigned char* dst = ring + static_cast<size_t>(s) * kTiles * kTileBytes;
    mbar_expect_tx(&full[s], kTiles * kTileBytes);
    const int kx = static_cast<int>(kbase + static_cast<int64_t>(c) * kTileK);
    tma_load_2d(dst, &wmap, kx, static_cast<int>(col0), &full[s]);
    if (EPI == VL_LINEAR_SWIGLU)
      tma_load_2d(dst + kTileBytes, &wmap, kx, static_cast<int>(up_row + col0), &full[s]);
  };
  int issued = 0;  // producer (thread 0): weight tiles requested so far
  if (tid == 0) {
    for (int s = 0; s < L.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *bad = 0;
    *issued_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // the first stages' weight tiles go out at once, before the tensor
    // memory allocation and the dependency wait (weights never depend on the
    // previous kernel)
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
    for (; issued < L.stages; ++issued) issue(issued);
  }
  __syncwarp();
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     su32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (NORM) {  // the norm weight is a model input: fetched before the dependency wait
    const T* gam = static_cast<const T*>(a.norm_weight) + kbase;
    for (int i = tid; i < L.chunks * 8; i += kTcThreads) cp_async16_zfill(gam_s + 8 * i, gam + 8 * i, true);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  pdl_wait();
  pdl_release();

  // This CTA's x slice into shared memory with cp.async (rows past a.rows
  // zero-filled): k tile c, row r, 16-byte vector v at
  // c * NR * 128 + r * 128 + ((v ^ (r & 7)) * 16) - the 128-byte swizzle TMA
  // writes for the weight tiles.  In flight while the RMSNorm sums load.
  const int nvec = NR * L.chunks * 8;
  {
    const T* x = static_cast<const T*>(a.x);
    for (int i = tid; i < nvec; i += kTcThreads) {
      const int v = i & 7, r = (i >> 3) % NR, c = (i >> 3) / NR;
      const int64_t kk = kbase + static_cast<int64_t>(c) * kTileK + v * 8;
      const bool ok = r < a.rows;
      cp_async16_zfill(xs + static_cast<size_t>(c) * NR * 128 + r * 128 + ((v ^ (r & 7)) << 4),
                       x + (ok ? r : 0) * a.x_row_stride + kk, ok);
    }
    if (NORM) {  // the producer's partial sums, [parts][rows] as one contiguous block
      const int nf = a.ssq_in_parts * static_cast<int>(a.rows);
      if ((reinterpret_cast<uintptr_t>(a.ssq_in) & 15) == 0 && nf % 4 == 0) {
        for (int i = tid; i < nf / 4; i += kTcThreads) cp_async16_zfill(ssq_s + 4 * i, a.ssq_in + 4 * i, true);
      } else {
        for (int i = tid; i < nf; i += kTcThreads) ssq_s[i] = a.ssq_in[i];
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // RMSNorm prologue: 1 / rms of every row from the producer's partial sums
  // (a warp per row, lane l sums parts l, l+32, ... in order, then a fixed
  // xor tree), the same order as vl_linear.cu; then x = round(x * inv * w)
  // in place in shared memory.
  if (NORM) {
    for (int r = warp; r < a.rows; r += kTcThreads / 32) {
      float ssq = 0.0f;
      for (int p = lane; p < a.ssq_in_parts; p += 32) ssq += ssq_s[p * a.rows + r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
      if (lane == 0) inv_s[r] = rsqrtf(ssq / static_cast<float>(a.k) + a.eps);
    }
  }
  __syncthreads();
  if (NORM) {
    for (int i = tid; i < nvec; i += kTcThreads) {
      const int v = i & 7, r = (i >> 3) % NR, c = (i >> 3) / NR;
      if (r >= a.rows) continue;
      const int64_t kk = kbase + static_cast<int64_t>(c) * kTileK + v * 8;
      uint4* slot = reinterpret_cast<uint4*>(xs + static_cast<size_t>(c) * NR * 128 + r * 128 +
                                             ((v ^ (r & 7)) << 4));
      const uint4 val = *slot;
      const uint4 g = *reinterpret_cast<const uint4*>(gam_s + (kk - kbase));
      const float iv = inv_s[r];
      uint32_t w[4] = {val.x, val.y, val.z, val.w};
      const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 xv = tc_unpack2<T>(w[j]), gv = tc_unpack2<T>(gw[j]);
        w[j] = tc_pack2<T>(xv.x * iv * gv.x, xv.y * iv * gv.y);
      }
      *slot = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  // the x slice (written by cp.async and, with NORM, by these threads) is
  // read by the tensor cores through the async proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();

  constexpr uint32_t kIdesc = mma_idesc<T>(NR);
  // Roles: lane 0 of warp 1 issues the MMAs, lane 0 of warp 0 refills the
  // ring; the other lanes of those two warps park at __syncwarp (a spinning
  // lane in the same warp would hold the issuing lane back).
  if (tid == 32) {
    // MMA issuer: 4 k-steps of 16 per stage, fp32 accumulation in TMEM.
    for (int c = 0; c < L.chunks; ++c) {
      const int s = c % L.stages;
      if (!mbar_wait(&full[s], static_cast<uint32_t>((c / L.stages) & 1))) {
        atomicExch(bad, 1);
        break;
      }
      tc_fence_after();
      const uint32_t a0 = su32(ring + static_cast<size_t>(s) * kTiles * kTileBytes);
      const uint32_t b0 = su32(xs + static_cast<size_t>(c) * NR * 128);
#pragma unroll
      for (int kk = 0; kk < kTileK / 16; ++kk) {
        const uint64_t bdesc = sw128_desc(b0 + kk * 32);
        const uint32_t acc = (c > 0 || kk > 0) ? 1u : 0u;
        mma_f16(tmem, sw128_desc(a0 + kk * 32), bdesc, kIdesc, acc);
        if (EPI == VL_LINEAR_SWIGLU)
          mma_f16(tmem + NR, sw128_desc(a0 + kTileBytes + kk * 32), bdesc, kIdesc, acc);
      }
      mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
    }
    mma_commit(done);
  } else if (tid == 0) {
    // Producer: refill each stage once the MMAs of its previous tile are done.
    for (int c = L.stages; c < L.chunks; ++c) {
      const int s = c % L.stages;
      if (*reinterpret_cast<volatile int*>(bad) ||
          !mbar_wait(&empty[s], static_cast<uint32_t>(((c / L.stages) - 1) & 1))) {
        atomicExch(bad, 1);
        break;
      }
      issue(c);
      issued = c + 1;
    }
    *issued_s = issued;
  }
  if (warp < 2) __syncwarp();

  // Accumulators: warp w holds TMEM lanes (= output columns) 32w..32w+31.
  const bool finished = mbar_wait(done, 0);
  __syncwarp();
  tc_fence_after();
  float acc[kTiles][NR];
#pragma unroll
  for (int t = 0; t < kTiles; ++t)
#pragma unroll
    for (int j0 = 0; j0 < NR; j0 += 16) {
      float v[16];
      tmem_ld16(tmem + (static_cast<uint32_t>(warp * 32) << 16) + t * NR + j0, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[t][j0 + i] = v[i];
    }
  tmem_ld_wait();
  if (!finished) atomicExch(bad, 1);
  // Split-K reduction, push form: token row j belongs to cluster rank
  // j / rp, which receives every rank's partial of it at
  // part[((t * rp + j % rp) * splits + rank) * 128 + column]; after one
  // cluster barrier each CTA sums what it received in rank order, so no CTA
  // reads another's shared memory and none has to wait for the others to
  // finish.
  const int rp = NR / splits;
  const int lrp = __ffs(rp) - 1;
#pragma unroll
  for (int t = 0; t < kTiles; ++t)
#pragma unroll
    for (int j = 0; j < NR; ++j) {
      const int owner = j >> lrp, jj = j & (rp - 1);
      float* dst = part + ((t * rp + jj) * splits + static_cast<int>(rank)) * kTileM + tid;
      if (splits == 1)
        *dst = acc[t][j];
      else
        st_cluster_f32(dst, static_cast<uint32_t>(owner), acc[t][j]);
    }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  if (*reinterpret_cast<volatile int*>(bad) && tid == 0) {
    // Error path: let this CTA's copies still in flight land before its
    // shared memory goes away (bounded): the last tile issued into each
    // stage, whose phase is the latest one; then count the event.
    const int n = *issued_s;
    for (int c = n - L.stages < 0 ? 0 : n - L.stages; c < n; ++c)
      (void)mbar_wait(&full[c % L.stages], static_cast<uint32_t>((c / L.stages) & 1));
    atomicAdd(&g_linear_wait_timeouts, 1u);
  }

  // Sum the partials of this CTA's NR / splits token rows in rank order and
  // finish them.
  if (splits > 1) cluster_sync();
  const int r_begin = static_cast<int>(rank) * rp;
  T* y = static_cast<T*>(a.y);
  const bool ok = !*reinterpret_cast<volatile int*>(bad);  // read once, before any store
  float* hbuf = part;  // RESIDUAL: this CTA's new h values, [rp][128], after a barrier
  float hv_keep[NR];
  // RESIDUAL: every old h value of this thread is requested before any new
  // one is stored (a store could alias the next row's load otherwise, which
  // would serialise the rows)
  float h_old[EPI == VL_LINEAR_RESIDUAL ? NR : 1];
  if (EPI == VL_LINEAR_RESIDUAL) {
#pragma unroll
    for (int jj = 0; jj < NR; ++jj) {
      const int j = r_begin + jj;
      h_old[jj] = (jj < rp && j < a.rows) ? S::to_float(y[j * a.y_row_stride + col0 + tid]) : 0.0f;
    }
  }
  // All of this thread's rows are summed and finished first, then stored:
  // a partial-sum load issued after a global store waits for it, which cost
  // about a microsecond per row when the two alternated.
  float outv[NR];
#pragma unroll
  for (int jj = 0; jj < NR; ++jj) {
    outv[jj] = 0.0f;
    hv_keep[jj] = 0.0f;
    if (jj >= rp) continue;
    float v[kTiles];
#pragma unroll
    for (int t = 0; t < kTiles; ++t) {
      const float* src = part + (t * rp + jj) * splits * kTileM + tid;
      float sum = 0.0f;
      for (int q = 0; q < splits; ++q) {  // explicit shared-memory loads (measured faster)
        float pv;
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(pv) : "r"(su32(src + q * kTileM)));
        sum += pv;
      }
      v[t] = sum;
    }
    if (EPI == VL_LINEAR_STORE) {
      outv[jj] = v[0];
    } else if (EPI == VL_LINEAR_SWIGLU) {
      const float g = S::round_trip(v[0]);
      const float u = S::round_trip(v[kTiles - 1]);
      outv[jj] = __fdividef(g, 1.0f + __expf(-g)) * u;
    } else {
      const float hv = S::round_trip(h_old[EPI == VL_LINEAR_RESIDUAL ? jj : 0] + S::round_trip(v[0]));
      outv[jj] = hv;
      hv_keep[jj] = hv;
    }
  }
#pragma unroll
  for (int jj = 0; jj < NR; ++jj) {
    const int j = r_begin + jj;
    if (jj < rp && j < a.rows)
      y[j * a.y_row_stride + col0 + tid] = S::from_float(ok ? outv[jj] : __int_as_float(0x7fc00000));
  }
  if (EPI == VL_LINEAR_RESIDUAL && a.ssq_out != nullptr) {
    __syncthreads();
#pragma unroll
    for (int jj = 0; jj < NR; ++jj)
      if (jj < rp) hbuf[jj * kTileM + tid] = hv_keep[jj];
    __syncthreads();
    // per row and 16-column group, sum of squares in column order (fmaf),
    // as vl_linear.cu writes it: ssq_out[col / 16][row]
    for (int i = tid; i < rp * (kTileM / 16); i += kTcThreads) {
      const int jj = i / (kTileM / 16), g = i % (kTileM / 16);
      const int j = r_begin + jj;
      if (j >= a.rows) continue;
      float ssq = 0.0f;
#pragma unroll
      for (int c = 0; c < 16; ++c) ssq = fmaf(hbuf[jj * kTileM + g * 16 + c],
                                              hbuf[jj * kTileM + g * 16 + c], ssq);
      a.ssq_out[(col0 / 16 + g) * a.rows + j] = ssq;
    }
  }
}

using EncodeTiled = PFN_cuTensorMapEncodeTiled_v12000;

EncodeTiled encode_fn() {
  static std::atomic<EncodeTiled> fn{nullptr};
  EncodeTiled f = fn.load(std::memory_order_acquire);
  if (f != nullptr) return f;
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
          cudaSuccess ||
      q != cudaDriverEntryPointSuccess || p == nullptr) {
    (void)cudaGetLastError();
    return nullptr;
  }
  f = reinterpret_cast<EncodeTiled>(p);
  fn.store(f, std::memory_order_release);
  return f;
}

// K splits: the fewest (a power of two, at most 8, dividing the k tiles) that
// give at least one CTA per SM, keeping at least 2 k tiles per CTA.
int tc_splits(int64_t tiles, int64_t ktiles, int nr) {
  const int64_t want = sm_count();
  int s = 1;
  while (s < 8 && tiles * s < want && ktiles % (2 * s) == 0 && ktiles / (2 * s) >= 2 &&
         nr / (2 * s) >= 1)
    s *= 2;
  return s;
}

// Split count and ring depth of a launch, chosen together: clusters of 8
// CTAs are scarce on this part (cudaOccupancyMaxActiveClusters reports 15 on
// a B200 whatever a CTA's shared memory), so a grid of more clusters than
// can be resident runs in two waves.  Search the split counts from the one
// that gives every SM a CTA (tc_splits) down to 1 and take the first whose
// clusters are all resident, with the deepest ring that keeps them so; if
// none is, the largest split with its deepest ring.  Cached per (device,
// kernel, shape).
struct TcPlan {
  int splits;
  int stages;
};

TcPlan tc_plan(const void* kernel, int nr, int epi, bool norm, int64_t k, int64_t tiles) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, int64_t, int64_t>, TcPlan> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TcPlan{1, 1};
  const auto key = std::make_tuple(dev, kernel, k, tiles);
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const int64_t ktiles = k / kTileK;
  TcPlan best{0, 0}, fallback{0, 0};
  for (int sp = tc_splits(tiles, ktiles, nr); sp >= 1 && best.splits == 0; sp /= 2) {
    if (ktiles % sp != 0 || nr / sp < 1) continue;
    for (int st = kMaxStages; st >= 1; --st) {
      const TcLayout L = tc_layout(nr, epi, k, sp, st, kSmemBudget, norm);
      if (L.total > kSmemBudget + 2048) continue;       // does not fit at all
      if (L.stages < st && st > 1) continue;            // this depth does not fit
      if (fallback.splits == 0) fallback = TcPlan{sp, L.stages};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1;
      attr[0].val.clusterDim.y = static_cast<unsigned>(sp);
      attr[0].val.clusterDim.z = 1;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(tiles), static_cast<unsigned>(sp), 1);
      cfg.blockDim = dim3(kTcThreads, 1, 1);
      cfg.dynamicSmemBytes = L.total;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        continue;
      }
      if (n >= tiles) {
        best = TcPlan{sp, L.stages};
        break;
      }
    }
  }
  if (best.splits == 0) best = fallback.splits != 0 ? fallback : TcPlan{1, 1};
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = best;
  return best;
}

template <typename T, int NR, int EPI, bool NORM>
cudaError_t tc_launch(const LinearArgs& a, const CUtensorMap& map, bool pdl, cudaStream_t stream) {
  const int64_t cols = EPI == VL_LINEAR_SWIGLU ? a.n / 2 : a.n;
  const int64_t tiles = cols / kTileM;
  auto kernel = decode_linear_tc_kernel<T, NR, EPI, NORM>;
  static std::atomic<bool> configured[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBudget + 2048));
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev].store(true, std::memory_order_release);
  }
  const TcPlan plan = tc_plan(reinterpret_cast<const void*>(kernel), NR, EPI, NORM, a.k, tiles);
  const int splits = plan.splits, stages = plan.stages;
  const TcLayout L = tc_layout(NR, EPI, a.k, splits, stages, kSmemBudget, NORM);
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = 1;
  attr[na].val.clusterDim.y = static_cast<unsigned>(splits);
  attr[na].val.clusterDim.z = 1;
  ++na;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(tiles), static_cast<unsigned>(splits), 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kernel, a, map, splits, stages,
                            static_cast<unsigned int>(kSmemBudget));
}

template <typename T, int NR>
cudaError_t tc_epi(const LinearArgs& a, const CUtensorMap& map, bool pdl, cudaStream_t stream) {
  const bool norm = a.norm_weight != nullptr;
  switch (a.epilogue) {
    case VL_LINEAR_STORE:
      return norm ? tc_launch<T, NR, VL_LINEAR_STORE, true>(a, map, pdl, stream)
                  : tc_launch<T, NR, VL_LINEAR_STORE, false>(a, map, pdl, stream);
    case VL_LINEAR_SWIGLU:
      return norm ? tc_launch<T, NR, VL_LINEAR_SWIGLU, true>(a, map, pdl, stream)
                  : tc_launch<T, NR, VL_LINEAR_SWIGLU, false>(a, map, pdl, stream);
    default:
      return norm ? tc_launch<T, NR, VL_LINEAR_RESIDUAL, true>(a, map, pdl, stream)
                  : tc_launch<T, NR, VL_LINEAR_RESIDUAL, false>(a, map, pdl, stream);
  }
}

template <typename T>
cudaError_t tc_typed(const LinearArgs& a, const CUtensorMap& map, bool pdl, cudaStream_t stream) {
  if (a.rows <= 16) return tc_epi<T, 16>(a, map, pdl, stream);
  if (a.rows <= 32) return tc_epi<T, 32>(a, map, pdl, stream);
  return tc_epi<T, 64>(a, map, pdl, stream);
}

}  // namespace

cudaError_t read_linear_timeouts(unsigned int* count) {
  return cudaMemcpyFromSymbol(count, g_linear_wait_timeouts, sizeof(unsigned int));
}

bool decode_linear_tc_supported(const LinearArgs& a, int dtype) {
  if (dtype != kDtypeBF16 && dtype != kDtypeF16) return false;
  const int64_t cols = a.epilogue == VL_LINEAR_SWIGLU ? a.n / 2 : a.n;
  if (a.rows < 1 || a.rows > 64 || cols % kTileM != 0 || a.k % (2 * kTileK) != 0) return false;
  if (a.n > (int64_t(1) << 31) - 1 || a.k > (int64_t(1) << 31) - 1) return false;
  if (!aligned16(a.w) || !aligned16(a.x) || a.x_row_stride % 8 != 0) return false;
  if (a.norm_weight != nullptr && !aligned16(a.norm_weight)) return false;
  // the RMSNorm prologue stages the partial sums in a [k/16][rows] buffer
  if (a.norm_weight != nullptr && (a.ssq_in_parts < 1 || a.ssq_in_parts > a.k / 16)) return false;
  const int nr = a.rows <= 16 ? 16 : (a.rows <= 32 ? 32 : 64);
  // some split count must fit one k tile per stage
  bool fits = false;
  for (int sp = tc_splits(cols / kTileM, a.k / kTileK, nr); sp >= 1 && !fits; sp /= 2)
    fits = (a.k / kTileK) % sp == 0 &&
           tc_layout(nr, a.epilogue, a.k, sp, 1, kSmemBudget, a.norm_weight != nullptr).total <=
               kSmemBudget + 2048;
  if (!fits) return false;
  return encode_fn() != nullptr;
}

cudaError_t launch_decode_linear_tc(const LinearArgs& a, int dtype, bool pdl,
                                    cudaStream_t stream) {
  EncodeTiled encode = encode_fn();
  if (encode == nullptr) return cudaErrorNotSupported;
  CUtensorMap map;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.k), static_cast<cuuint64_t>(a.n)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.k) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileK), static_cast<cuuint32_t>(kTileM)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(&map,
                            dtype == kDtypeBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                            2, const_cast<void*>(a.w), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (dtype == kDtypeBF16) return tc_typed<__nv_bfloat16>(a, map, pdl, stream);
  return tc_typed<__half>(a, map, pdl, stream);
}

}  // namespace vl
