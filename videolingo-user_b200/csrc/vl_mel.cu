// Whisper log-mel frontend for sm_100a.
//
// Reference: compute_mel_batched (VideoLingo-user
// native/asr/src/mel_frontend.cu:209-291) runs five kernels per call:
// a 400-tap direct DFT per (bin, frame) (stft_power_kernel :164-184), a dense
// 201-term filterbank product (mel_matmul_kernel :187-201), log10 + per-bin
// max, per-chunk max and the normalise pass (:108-153), with the power and
// mel spectra making full HBM round trips in between.
//
// Here the whole per-frame pipeline is one kernel over tiles of 32 frames:
//   samples (reflect-padded) -> shared memory, one copy per frame pair
//   two real frames packed as one complex 400-point FFT (x_a + i*x_b),
//     400 = 20 x 20: stage 1 = 20 DFT-20s over stride-20 samples + W400
//     twiddles, stage 2 = 20 DFT-20s (each DFT-20 a prime-factor 4 x 5 in
//     registers, in packed fp32x2 arithmetic: one instruction per complex
//     add/fma)
//   |X_a|^2, |X_b|^2 from the packed spectrum's conjugate symmetry, in
//     registers: the stage-2 lanes of k1 and 20 - k1 are neighbours and swap
//     the mirror half of their outputs with one shuffle per bin
//   sparse Slaney projection (394 nonzeros instead of 201 x 128 dense),
//     one task per (frame, run of mel bins) with runs of equal cost
//   log10(max(., 1e-10)) -> out, tile max -> workspace
// The stage-1 transpose and the power spectra share one 53 KB region; with the per-pair samples (prefetched for the next tile) and
// the tables a tile takes ~93 KB, two tiles per SM.  A second, light
// kernel folds the tile maxima of each chunk and applies max(x, max-8) then
// (x+4)/4 in place.  Chunks are processed in equal batches of at most 64
// whose log-mel (1.5 MB per chunk, <= 98 MB) stays resident in the 126 MB L2
// between the two kernels, so HBM sees the PCM once and the features once.
#include <atomic>
#include <mutex>

#include "vl_common.cuh"
#include "vl_kernels.h"
#include "mel_tables.inc"

namespace vl {
namespace mel {
// log10(max(x, 1e-10)) through the hardware log2 (|error| < 1e-6 here).
__device__ __forceinline__ float log10_floor(float x) {
  return __log2f(fmaxf(x, 1e-10f)) * 0.30102999566398119521f;
}
}  // namespace mel
}  // namespace vl

#include "mel_runs.inc"

namespace vl {
namespace {

constexpr int kChunkSamples = 480000;
constexpr int kHop = 160;
constexpr int kPad = 200;
constexpr int kFrames = 3000;              // frames kept (the 3001st is dropped)
constexpr int kTileFrames = 32;            // frames per tile: one per lane in the mel stage
constexpr int kPairs = kTileFrames / 2;    // complex FFTs per tile
constexpr int kTilesPerChunk = (kFrames + kTileFrames - 1) / kTileFrames;  // 94 (last: 24 frames)
constexpr int kTileSamples = kHop * (kTileFrames - 1) + 400;  // 5360
constexpr int kPairSamples = kHop + 400;   // 560: the samples of one frame pair
// Each pair's samples are kept as their own copy, 564 floats apart: 564 = 20
// (mod 32), so in stage 1 lane t of a warp reads bank t mod 32 whichever
// pairs the warp spans (pair offsets 320 p would all start at one bank).
constexpr int kPairStride = 564;
constexpr int kBins = 201;
constexpr int kMel = 128;
constexpr int kThreads = kPairs * 20;      // 320: one FFT task per thread, 10 warps
constexpr int kTRow = 21;                  // padded row (complex) of the stage-1 transpose
constexpr int kNormSlices = 16;            // normalise blocks per chunk
constexpr int kBatchChunks = 64;           // chunks per L2-resident batch, at most (98 MB of log-mel)
constexpr int kMaxTilesPerChunk = 125;     // capacity per chunk of the no-alloc scratch
static_assert(kTilesPerChunk <= kMaxTilesPerChunk, "no-alloc scratch too small");
static_assert(VL_MEL_GROUPS == kThreads / 32, "one mel-bin run per warp");

struct MelSmem {
  float samples[kPairs * kPairStride];     // next tile's samples per pair, filled by cp.async
  // stage-1 output t[p][slot][n2] -> power spectra p[frame][bin]; stage 2
  // reads the first into registers and passes a barrier before writing the
  // second.
  union {
    float2 t[kPairs][20][kTRow];
    float p[kTileFrames][kBins];
  } u;
  float window[400];
  float2 tw[20][20];                       // W400^(k1 n2) at [k1][n2]: lanes n2 read consecutive entries
  float red[kThreads / 32];
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Complex value (re, im) in one 64-bit register pair, operated on with the
// sm_100 packed fp32x2 instructions: a complex add, subtract or
// multiply-add by a real pair is a single instruction.
struct c2 {
  unsigned long long v;
};
__device__ __forceinline__ c2 mk(float re, float im) {
  c2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(re), "f"(im));
  return r;
}
__device__ __forceinline__ float2 split(c2 a) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(a.v));
  return r;
}
__device__ __forceinline__ c2 add(c2 a, c2 b) {
  c2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ c2 sub(c2 a, c2 b) {
  c2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ c2 mul(c2 a, c2 b) {
  c2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
  return r;
}
__device__ __forceinline__ c2 fma2(c2 a, c2 b, c2 c) {  // a * b + c, per lane of the pair
  c2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
  return r;
}
__device__ __forceinline__ c2 swap(c2 a) {
  const float2 f = split(a);
  return mk(f.y, f.x);
}
// a - i*b and a + i*b
__device__ __forceinline__ c2 sub_i(c2 a, c2 b) { return fma2(swap(b), mk(1.f, -1.f), a); }
__device__ __forceinline__ c2 add_i(c2 a, c2 b) { return fma2(swap(b), mk(-1.f, 1.f), a); }
// a * conj(w) with w = (cos, sin): multiplies by exp(-i*theta).
__device__ __forceinline__ c2 cmul_conj(c2 a, float c, float s) {
  return fma2(swap(a), mk(s, -s), mul(a, mk(c, c)));
}

// In-place forward DFT of 20 complex points: X[k] = sum_n x[n] exp(-2 pi i k n / 20),
// by the prime-factor (Good-Thomas) split 20 = 4 x 5: with gcd(4, 5) = 1,
// n = (5 n1 + 4 n2) mod 20 and k = (5 k1 + 16 k2) mod 20 turn the DFT-20
// into DFT-4s over n1 followed by DFT-5s over n2 with no twiddle factors in
// between (W20^(nk) = W4^(n1 k1) W5^(n2 k2)).  The index maps are fixed,
// so they cost nothing in unrolled register code.
__device__ __forceinline__ void dft20(c2 (&x)[20]) {
  c2 u[5][4];  // u[n2][k1]
#pragma unroll
  for (int n2 = 0; n2 < 5; ++n2) {
    const c2 a0 = x[(4 * n2) % 20], a1 = x[(5 + 4 * n2) % 20];
    const c2 a2 = x[(10 + 4 * n2) % 20], a3 = x[(15 + 4 * n2) % 20];
    const c2 t0 = add(a0, a2), t1 = sub(a0, a2);
    const c2 t2 = add(a1, a3), t3 = sub(a1, a3);
    u[n2][0] = add(t0, t2);
    u[n2][2] = sub(t0, t2);
    u[n2][1] = sub_i(t1, t3);
    u[n2][3] = add_i(t1, t3);
  }
  const c2 C1 = mk(mel::kC1, mel::kC1), C2 = mk(mel::kC2, mel::kC2);
  const c2 S1 = mk(mel::kS1, mel::kS1), S2 = mk(mel::kS2, mel::kS2);
  const c2 NS1 = mk(-mel::kS1, -mel::kS1);
#pragma unroll
  for (int k1 = 0; k1 < 4; ++k1) {
    const c2 x0 = u[0][k1];
    const c2 a1 = add(u[1][k1], u[4][k1]), a2 = add(u[2][k1], u[3][k1]);
    const c2 b1 = sub(u[1][k1], u[4][k1]), b2 = sub(u[2][k1], u[3][k1]);
    const c2 m1 = fma2(a2, C2, fma2(a1, C1, x0));
    const c2 m2 = fma2(a2, C1, fma2(a1, C2, x0));
    const c2 n1 = fma2(b2, S2, mul(b1, S1));
    const c2 n2 = fma2(b2, NS1, mul(b1, S2));
    x[(5 * k1) % 20] = add(x0, add(a1, a2));        // k2 = 0
    x[(5 * k1 + 16) % 20] = sub_i(m1, n1);          // k2 = 1
    x[(5 * k1 + 4) % 20] = add_i(m1, n1);           // k2 = 4
    x[(5 * k1 + 12) % 20] = sub_i(m2, n2);          // k2 = 2
    x[(5 * k1 + 8) % 20] = add_i(m2, n2);           // k2 = 3
  }
}

// Stage-1 rows in mirror-pair order: slot 2m holds k1 = m and slot 2m + 1
// holds k1 = 20 - m (m = 1..9); slots 0 and 1 hold k1 = 0 and 10, each its
// own mirror.
__device__ __forceinline__ constexpr int mirror_slot(int k1) {
  return k1 == 0 ? 0 : (k1 == 10 ? 1 : (k1 < 10 ? 2 * k1 : 2 * (20 - k1) + 1));
}
__device__ __forceinline__ int slot_k1(int slot) {
  const int m = slot >> 1;
  if (slot == 1) return 10;
  return (slot & 1) ? 20 - m : m;
}

__device__ __forceinline__ int reflect(int j) {
  if (j < 0) return -j;
  if (j >= kChunkSamples) return 2 * kChunkSamples - 2 - j;
  return j;
}

// Asynchronous copy of one tile's samples (reflect-padded at the chunk edges)
// into shared memory; the copy overlaps the previous tile's compute.
__device__ __forceinline__ void prefetch_samples(float* dst, const float* __restrict__ pcm,
                                                 int64_t chunk, int tile, int tid) {
  const float* src = pcm + chunk * kChunkSamples;
  const int j0 = tile * kTileFrames * kHop - kPad;
  if (j0 >= 0 && j0 + kTileSamples <= kChunkSamples) {
    // pair q: samples j0 + 320 q .. + 560, as 140 16-byte pieces
    for (int i = tid; i < kPairs * (kPairSamples / 4); i += kThreads) {
      const int q = i / (kPairSamples / 4), c = i - q * (kPairSamples / 4);
      cp_async16(dst + q * kPairStride + 4 * c, src + j0 + 2 * kHop * q + 4 * c);
    }
  } else {
    for (int i = tid; i < kPairs * kPairSamples; i += kThreads) {
      const int q = i / kPairSamples, c = i - q * kPairSamples;
      cp_async4(dst + q * kPairStride + c, src + reflect(j0 + 2 * kHop * q + c));
    }
  }
  cp_async_commit();
}

// Persistent: each block walks tiles blockIdx.x, +gridDim.x, ... of the batch
// (chunk-major), prefetching the next tile's samples while it computes.
__global__ void __launch_bounds__(kThreads, 2)
    mel_tile_kernel(const float* __restrict__ pcm, float* __restrict__ out,
                    float* __restrict__ tile_max, int chunk0, int n_chunks) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  MelSmem& sm = *reinterpret_cast<MelSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int total = n_chunks * kTilesPerChunk;
  int w = blockIdx.x;
  if (w < total) prefetch_samples(sm.samples, pcm, chunk0 + w / kTilesPerChunk, w % kTilesPerChunk, tid);
  for (int i = tid; i < 400; i += kThreads) sm.window[i] = mel::kWindow[i];
  for (int i = tid; i < 400; i += kThreads) sm.tw[i / 20][i % 20] = mel::kTwiddle400[(i / 20) * (i % 20)];
  const int p = tid / 20, lane20 = tid - 20 * (tid / 20);
  const int warp = tid >> 5, lane = tid & 31;

  for (; w < total; w += gridDim.x) {
    const int64_t chunk = chunk0 + w / kTilesPerChunk;
    const int tile = w % kTilesPerChunk;
    const int f0 = tile * kTileFrames;
    cp_async_wait_all();
    __syncthreads();  // this tile's samples (and, first time, the tables) are in smem

    // ---- stage 1: per (pair, n2) DFT-20 over n1 of z[20 n1 + n2], twiddle W400^(k1 n2)
    c2 x[20];
    {
      const float* sa = sm.samples + p * kPairStride;
      const float* sb = sa + kHop;
#pragma unroll
      for (int n1 = 0; n1 < 20; ++n1) {
        const int n = 20 * n1 + lane20;
        const float wv = sm.window[n];
        x[n1] = mul(mk(sa[n], sb[n]), mk(wv, wv));
      }
    }
    __syncthreads();  // samples consumed: start fetching the next tile's
    if (w + static_cast<int>(gridDim.x) < total) {
      const int nw = w + gridDim.x;
      prefetch_samples(sm.samples, pcm, chunk0 + nw / kTilesPerChunk, nw % kTilesPerChunk, tid);
    }
    dft20(x);
#pragma unroll
    for (int k1 = 0; k1 < 20; ++k1) {
      const float2 tw = sm.tw[k1][lane20];
      *reinterpret_cast<unsigned long long*>(&sm.u.t[p][mirror_slot(k1)][lane20]) =
          cmul_conj(x[k1], tw.x, tw.y).v;
    }
    __syncthreads();

    // ---- stage 2: per (pair, k1) DFT-20 over n2 -> Z[k1 + 20 k2].  Slot
    // lane20 of the pair holds row k1 = slot_k1(lane20), so the lanes of a
    // mirror pair (k1, 20 - k1) are neighbours (lane ^ 1, same warp).
#pragma unroll
    for (int n2 = 0; n2 < 20; ++n2)
      x[n2].v = *reinterpret_cast<const unsigned long long*>(&sm.u.t[p][lane20][n2]);
    __syncthreads();  // stage-1 output consumed: the region now takes the power spectra
    dft20(x);

    // ---- power: X_a = (Z[k] + conj Z[400-k]) / 2, X_b = (Z[k] - conj Z[400-k]) / 2i.
    // This lane holds Z[k1 + 20 k2]; the mirror Z[400 - k1 - 20 k2] is
    // Z[k1' + 20 (19 - k2)] of the neighbour lane (k1' = 20 - k1), or of
    // this lane itself when k1 is 0 (Z[20 ((20 - k2) mod 20)]) or 10
    // (Z[10 + 20 (19 - k2)]).  Bins k1 + 20 k2 <= 200: k2 = 0..9, and for
    // k1 = 0 also k2 = 10 (bin 200, its own mirror).
    {
      const int k1 = slot_k1(lane20);
      const bool self = k1 == 0 || k1 == 10;
      float* pa_row = sm.u.p[2 * p];
      float* pb_row = sm.u.p[2 * p + 1];
#pragma unroll
      for (int k2 = 0; k2 < 10; ++k2) {
        c2 m;
        m.v = __shfl_xor_sync(0xffffffffu, x[19 - k2].v, 1);
        if (self) m = k1 == 0 ? x[(20 - k2) % 20] : x[19 - k2];
        const float2 a = split(x[k2]), b = split(m);
        const float ar = a.x + b.x, ai = a.y - b.y;
        const float br = a.x - b.x, bi = a.y + b.y;
        pa_row[k1 + 20 * k2] = (ar * ar + ai * ai) * 0.25f;
        pb_row[k1 + 20 * k2] = (br * br + bi * bi) * 0.25f;
      }
      if (k1 == 0) {  // bin 200: Z[200] is its own mirror
        const float2 a = split(x[10]), b = a;
        const float ar = a.x + b.x, ai = a.y - b.y;
        const float br = a.x - b.x, bi = a.y + b.y;
        pa_row[200] = (ar * ar + ai * ai) * 0.25f;
        pb_row[200] = (br * br + bi * bi) * 0.25f;
      }
    }
    __syncthreads();

    // ---- mel projection + log10: warp w = run of bins w, lane = frame
    float local_max = -INFINITY;
    if (f0 + lane < kFrames) {
      const float* pw = sm.u.p[lane];
      float* dst = out + chunk * (static_cast<int64_t>(kMel) * kFrames) + f0 + lane;
      switch (warp) {
        case 0: local_max = mel::mel_run<0>(pw, dst); break;
        case 1: local_max = mel::mel_run<1>(pw, dst); break;
        case 2: local_max = mel::mel_run<2>(pw, dst); break;
        case 3: local_max = mel::mel_run<3>(pw, dst); break;
        case 4: local_max = mel::mel_run<4>(pw, dst); break;
        case 5: local_max = mel::mel_run<5>(pw, dst); break;
        case 6: local_max = mel::mel_run<6>(pw, dst); break;
        case 7: local_max = mel::mel_run<7>(pw, dst); break;
        case 8: local_max = mel::mel_run<8>(pw, dst); break;
        default: local_max = mel::mel_run<9>(pw, dst); break;
      }
    }
    local_max = warp_max(local_max);
    if (lane == 0) sm.red[warp] = local_max;
    __syncthreads();
    if (tid == 0) {
      float mx = sm.red[0];
#pragma unroll
      for (int v = 1; v < kThreads / 32; ++v) mx = fmaxf(mx, sm.red[v]);
      tile_max[chunk * kTilesPerChunk + tile] = mx;
    }
  }
  cp_async_wait_all();
}

// Fold the chunk's tile maxima, then out = (max(x, max - 8) + 4) / 4 over a
// slice of the chunk.  The slice was written by mel_tile_kernel moments
// before and is read from L2.
__global__ void __launch_bounds__(kThreads)
    mel_normalize_kernel(float* __restrict__ out, const float* __restrict__ tile_max,
                         int chunk0) {
  __shared__ float red[kThreads / 32];
  const int tid = threadIdx.x;
  const int64_t chunk = chunk0 + blockIdx.y;
  float mx = -INFINITY;
  for (int i = tid; i < kTilesPerChunk; i += kThreads)
    mx = fmaxf(mx, __ldcg(tile_max + chunk * kTilesPerChunk + i));
  mx = warp_max(mx);
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < kThreads / 32; ++w) mx = fmaxf(mx, red[w]);
  const float floor_log = mx - 8.0f;

  constexpr int kVec4PerChunk = kMel * kFrames / 4;  // 96000
  constexpr int kPerSlice = kVec4PerChunk / kNormSlices;  // 6000
  float4* base = reinterpret_cast<float4*>(out + chunk * (static_cast<int64_t>(kMel) * kFrames)) +
                 blockIdx.x * kPerSlice;
  for (int i = tid; i < kPerSlice; i += kThreads) {
    float4 v = __ldcg(base + i);
    v.x = (fmaxf(v.x, floor_log) + 4.0f) / 4.0f;
    v.y = (fmaxf(v.y, floor_log) + 4.0f) / 4.0f;
    v.z = (fmaxf(v.z, floor_log) + 4.0f) / 4.0f;
    v.w = (fmaxf(v.w, floor_log) + 4.0f) / 4.0f;
    __stcs(base + i, v);
  }
}

// Opt the tile kernel into > 48 KB of dynamic shared memory, once per device.
cudaError_t enable_large_smem(size_t smem) {
  static std::atomic<int> done[64];
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev >= 0 && dev < 64 && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
  err = cudaFuncSetAttribute(mel_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
  if (err == cudaSuccess && dev >= 0 && dev < 64) done[dev].store(1, std::memory_order_release);
  return err;
}

// Scratch of vl_logmel_noalloc: the per-tile maxima of up to
// VL_LOGMEL_NOALLOC_MAX_CHUNKS chunks (512,000 bytes), a fixed array inside
// the library so that entry point allocates nothing.  Host code must not
// use the symbol itself as a pointer (it names a host-side shadow); it
// fetches the device address once per device with cudaGetSymbolAddress.
static __device__ __align__(256) float g_noalloc_tile_max[VL_LOGMEL_NOALLOC_MAX_CHUNKS * kMaxTilesPerChunk];

}  // namespace

// Device address of g_noalloc_tile_max on the current device, looked up on
// the first call per device (that device current) and cached.  Later calls
// read the cached address with one acquire load; only the first lookup on a
// device takes the lock.
cudaError_t noalloc_tile_max(float** ptr) {
  static std::mutex mu;
  static std::atomic<float*> addr[64];
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  float* cached = addr[dev].load(std::memory_order_acquire);
  if (cached == nullptr) {
    std::lock_guard<std::mutex> lock(mu);
    cached = addr[dev].load(std::memory_order_relaxed);
    if (cached == nullptr) {
      void* p = nullptr;
      err = cudaGetSymbolAddress(&p, g_noalloc_tile_max);
      if (err != cudaSuccess) return err;
      cached = static_cast<float*>(p);
      addr[dev].store(cached, std::memory_order_release);
    }
  }
  *ptr = cached;
  return cudaSuccess;
}

size_t logmel_workspace_bytes(int64_t chunks) {
  const size_t raw = static_cast<size_t>(chunks) * kTilesPerChunk * sizeof(float);
  return (raw + 255) & ~static_cast<size_t>(255);
}

cudaError_t launch_logmel(const float* pcm, int64_t chunks, float* out, float* tile_max,
                          cudaStream_t stream) {
  static_assert(sizeof(MelSmem) <= 113 * 1024, "two tiles must fit one SM");
  const size_t smem = sizeof(MelSmem);
  cudaError_t err = enable_large_smem(smem);
  if (err != cudaSuccess) return err;
  // equal batches of at most kBatchChunks (a short last batch would run a
  // mostly idle final round of tiles); measured on 256 chunks: 32-chunk
  // batches 628 us, 43-48 602 us, 64 577-582 us, 86-128 595 us (their
  // log-mel no longer stays in L2 for the normalise pass), 256 583 us
  const int64_t nb = (chunks + kBatchChunks - 1) / kBatchChunks;
  for (int64_t b = 0; b < nb; ++b) {
    const int64_t c0 = (chunks * b) / nb;
    const int64_t n = (chunks * (b + 1)) / nb - c0;
    int blocks = resident_blocks(reinterpret_cast<const void*>(mel_tile_kernel), kThreads, smem);
    if (blocks > n * kTilesPerChunk) blocks = static_cast<int>(n * kTilesPerChunk);
    mel_tile_kernel<<<static_cast<unsigned>(blocks), kThreads, smem, stream>>>(
        pcm, out, tile_max, static_cast<int>(c0), static_cast<int>(n));
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    mel_normalize_kernel<<<dim3(kNormSlices, static_cast<unsigned>(n)), kThreads, 0, stream>>>(
        out, tile_max, static_cast<int>(c0));
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
  }
  return cudaSuccess;
}

}  // namespace vl

namespace vl {

cudaError_t prepare_logmel() {
  float* tile_max = nullptr;
  const cudaError_t err = enable_large_smem(sizeof(MelSmem));
  if (err != cudaSuccess) return err;
  return noalloc_tile_max(&tile_max);
}

cudaError_t launch_logmel_noalloc(const float* pcm, int64_t chunks, float* out,
                                  cudaStream_t stream) {
  float* tile_max = nullptr;
  const cudaError_t err = noalloc_tile_max(&tile_max);
  if (err != cudaSuccess) return err;
  return launch_logmel(pcm, chunks, out, tile_max, stream);
}

}  // namespace vl
