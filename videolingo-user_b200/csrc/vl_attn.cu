// Decode-step attention for sm_100a: one query token per sequence against
// its KV cache, with grouped-query heads, optionally fused with the RoPE of
// q / k at the token's position and the append of the new k / v rows.
//
// Reference semantics (VideoLingo-user native/asr/src/decoder.cu):
//   rope_at_position_map_kernel (:471-498)  q, k rotated at positions[chunk]
//   append_kv_mapped_kernel     (:500-514)  k, v -> cache row `position`
//   attention_step_mapped_kernel (:516-572) per (row, q head): scores
//       q.k_t / sqrt(128) over t in [0, position], fp32 softmax (max, exp,
//       sum, normalise), out = sum_t p_t v_t rounded to the storage type;
//       kv head = q head / (16 / 4)
// launched back to back per layer (:1710-1722).  The reference keeps all
// scores of a sequence in shared memory (at most 1024 positions) and runs
// one 128-thread block per (row, q head), so every K/V row is read once per
// q head, with one thread per position for q.k (a 256-byte row per thread).
//
// Here one CTA of 4 warps owns (token, kv head, split of the positions):
// * the G = n_q_heads / n_kv_heads query heads that share the kv head are
//   computed together, so each K and V row is read from HBM once;
// * the split's K and V rows stream through a shared-memory ring of
//   64-position tiles (32 KB each) filled with cp.async (16 bytes per thread,
//   L1 bypassed, rows past the end zero-filled): 2 stages and three CTAs per
//   SM when the grid fills the GPU, 3 or 4 stages when it does not; 16-byte
//   chunks are XOR-swizzled by row so ldmatrix reads are free of bank
//   conflicts;
// * with programmatic dependent launch, the position, the first tiles and
//   the rotation angles are fetched before waiting for the kernel that
//   produces q and the new k / v rows;
// * the products run on the tensor cores (mma.sync m16n8k16, fp32
//   accumulate) with the positions as M and the query heads as N (GQA decode
//   has too few queries for an M dimension): each warp takes 16 positions of
//   a tile, S^T = K q^T (K from ldmatrix, q^T held in registers), then
//   O^T += V^T P^T with V^T from ldmatrix.trans and P^T obtained from the S^T
//   accumulators by movmatrix.trans (no shared-memory round trip);
// * softmax is online per warp and head (log2 domain, exp2); warps and then
//   splits are merged with their maxima;
// * splits are combined by the CTA that finishes last (an atomic counter per
//   (token, kv head) that this CTA resets): no CTA ever waits for another.
// With fused RoPE the new k row is rotated once, written to the cache by
// split 0 and used from shared memory by the split owning the position, so
// no CTA reads a cache row that another CTA of the same launch writes.
//
// q and the probabilities enter the tensor cores in the storage type (the
// reference also rounds the rotated q to it); scores, softmax and the
// output accumulate in fp32.
#include <atomic>
#include <cmath>

#include "vl_common.cuh"
#include "vl_kernels.h"
#include "vl_rope_math.cuh"

namespace vl {
namespace {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
#ifndef VL_ATTN_STAGES
#define VL_ATTN_STAGES 2
#endif
#ifndef VL_ATTN_MIN_SPLIT
#define VL_ATTN_MIN_SPLIT 256
#endif
#ifndef VL_ATTN_TARGET_CTAS
#define VL_ATTN_TARGET_CTAS 2048
#endif
constexpr int kTile = 64;                 // positions per pipeline tile (16 per warp)
#ifndef VL_ATTN_DEEP_RING
#define VL_ATTN_DEEP_RING 1
#endif
// Tiles in the ring: VL_ATTN_STAGES (three CTAs per SM) for grids that fill
// the GPU; with VL_ATTN_DEEP_RING, 3 (two per SM) for grids of at most two
// CTAs per SM and 4 (one per SM) for at most one, so that more of a split's
// tiles are in flight at once.
constexpr int kStagesLarge = VL_ATTN_STAGES;
constexpr int kMaxSplits = 64;
constexpr float kLog2e = 1.4426950408889634f;

template <int HD, int G>
struct AttnSmem {
  float q[G][HD];           // rotated q (fp32 holding storage values)
  float kn[HD];             // fresh k (rotated, rounded to storage) and v
  float vn[HD];
  float2 cs[HD / 2];
  float wm[kAttnWarps][8];  // per-warp running maximum and sum per head column
  float wl[kAttnWarps][8];
  float wscale[kAttnWarps][G];  // warp merge weights exp2(m_w - M)
  float msplit[G];              // this split's maximum and sum
  float l[G];
  float w[kMaxSplits][G];       // split combine weights
  int last;
};

template <int HD, int G>
constexpr size_t attn_fixed_bytes() {
  return (sizeof(AttnSmem<HD, G>) + 127) & ~size_t(127);
}

// ---- PTX wrappers ----------------------------------------------------------
__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
// 16-byte async copy; src_bytes 0 zero-fills the destination
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4],
                                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  return pack_bf16x2(lo, hi);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  return pack_f16x2(lo, hi);
}

template <typename T>
__device__ __forceinline__ void load_row_f32(float* dst, const T* src, int n, int tid) {
  using S = Storage<T>;
  for (int c = tid; c < n / 8; c += kAttnThreads) {
    float f[8];
    S::unpack(ld_vec(src + c * 8), f);
#pragma unroll
    for (int e = 0; e < 8; ++e) dst[c * 8 + e] = f[e];
  }
}

// Shared-memory offset (elements) of 16-byte chunk `c` of tile row `r`.
template <int HD>
__device__ __forceinline__ int swz(int r, int c) {
  return r * HD + ((c ^ (r & 7)) << 3);
}

template <typename T, int HD, int G, int kStages>
__global__ void __launch_bounds__(kAttnThreads, kStages <= 2 ? 3 : (kStages == 3 ? 2 : 1))
    decode_attention_kernel(const __grid_constant__ DecodeAttnArgs a,
                            const __grid_constant__ InvFreq freq) {
  using S = Storage<T>;
  constexpr int KS = HD / 16;              // k-steps of q.k, m-tiles of p.v
  constexpr int CPR = HD / 8;              // 16-byte chunks per row
  constexpr int RPP = kAttnThreads / CPR;  // rows per cp.async pass
  extern __shared__ __align__(128) unsigned char smem_raw[];
  AttnSmem<HD, G>& sm = *reinterpret_cast<AttnSmem<HD, G>*>(smem_raw);
  // tile ring [kStages][K|V][kTile][HD], reused at the end for the per-warp
  // partial outputs [kAttnWarps][G][HD] (fp32)
  T* ring = reinterpret_cast<T*>(smem_raw + attn_fixed_bytes<HD, G>());

  const int64_t t = blockIdx.x;
  const int h = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int64_t pos = a.positions[t];
  const int64_t start = a.seq_start[t];
  T* out = static_cast<T*>(a.out) + t * a.out_row_stride + static_cast<int64_t>(h) * G * HD;

  if (pos < 0 || pos >= a.max_seq_len || start < 0 || start > a.num_slots - 1 - pos) {
    pdl_wait();
    if (s == 0) {
      for (int i = tid; i < G * HD; i += kAttnThreads) out[i] = S::from_float(0.0f);
      if (tid == 0 && a.status) atomicOr(a.status, VL_STATUS_BAD_SLOT);
    }
    return;
  }
  const int len = static_cast<int>(pos) + 1;
  const int nsplit = (len + a.split - 1) / a.split;
  if (s >= nsplit) return;
  const int p0 = s * a.split;
  const int p1 = min(len, p0 + a.split);
  const bool fresh = a.k != nullptr;
  const bool owns_last = p1 == len;
  const bool need_k = fresh && (owns_last || s == 0);
  const int rot = a.rotary_dim, half = rot / 2;
  // positions read from the cache (the owner of the last position takes it
  // from shared memory when the row is fresh)
  const int ncache = (fresh && owns_last) ? len - 1 - p0 : p1 - p0;
  const int ntiles = (ncache + kTile - 1) / kTile;

  // ---- start streaming the first tiles, then q (and the fresh k / v) -------
  const T* kg = static_cast<const T*>(a.k_cache) + (start + p0) * a.cache_row_stride +
                static_cast<int64_t>(h) * HD;
  const T* vg = static_cast<const T*>(a.v_cache) + (start + p0) * a.cache_row_stride +
                static_cast<int64_t>(h) * HD;
  const int my_row = tid / CPR, my_chunk = tid % CPR;
  auto issue = [&](int tile) {
    T* kd = ring + (tile % kStages) * (2 * kTile * HD);
    T* vd = kd + kTile * HD;
#pragma unroll
    for (int pass = 0; pass < kTile / RPP; ++pass) {
      const int r = pass * RPP + my_row;
      const int pr = tile * kTile + r;
      const bool ok = pr < ncache;
      const int64_t off = static_cast<int64_t>(ok ? pr : 0) * a.cache_row_stride + my_chunk * 8;
      cp_async16(kd + swz<HD>(r, my_chunk), kg + off, ok ? 16 : 0);
      cp_async16(vd + swz<HD>(r, my_chunk), vg + off, ok ? 16 : 0);
    }
  };
  // With the fused append the cached rows are those before the position,
  // written by earlier steps: they stream in while the kernel before this
  // one (which may be producing q and the new k / v rows) finishes.  Without
  // it the row at the position may have just been appended: wait first.
  if (!fresh) pdl_wait();
#pragma unroll
  for (int st = 0; st < kStages - 1; ++st) {
    if (st < ntiles) issue(st);
    cp_async_commit();
  }
  // the rotation angles depend on the position only
  for (int d = tid; d < half; d += kAttnThreads)
    sm.cs[d] = rope_cos_sin(static_cast<double>(pos) * freq.v[d]);
  if (fresh) pdl_wait();
  pdl_release();

  const T* qrow = static_cast<const T*>(a.q) + t * a.q_row_stride + static_cast<int64_t>(h) * G * HD;
  load_row_f32<T>(&sm.q[0][0], qrow, G * HD, tid);
  if (need_k) {
    load_row_f32<T>(sm.kn, static_cast<const T*>(a.k) + t * a.kv_row_stride +
                               static_cast<int64_t>(h) * HD, HD, tid);
    load_row_f32<T>(sm.vn, static_cast<const T*>(a.v) + t * a.kv_row_stride +
                               static_cast<int64_t>(h) * HD, HD, tid);
  }
  __syncthreads();
  if (rot > 0) {
    // RoPE on q and the fresh k, rounded to the storage type: the values the
    // tensor cores and the cache see (the reference stores them rounded too)
    const int rows = G + (need_k ? 1 : 0);
    for (int i = tid; i < rows * half; i += kAttnThreads) {
      const int r = i / half, d = i - r * half;
      float* x = r < G ? sm.q[r] : sm.kn;
      const float2 c = sm.cs[d];
      const float x1 = x[d], x2 = x[d + half];
      x[d] = S::round_trip(x1 * c.x - x2 * c.y);
      x[d + half] = S::round_trip(x2 * c.x + x1 * c.y);
    }
    __syncthreads();
  }
  if (fresh && s == 0) {
    const int64_t slot = start + pos;
    T* kc = static_cast<T*>(a.k_cache) + slot * a.cache_row_stride + static_cast<int64_t>(h) * HD;
    T* vc = static_cast<T*>(a.v_cache) + slot * a.cache_row_stride + static_cast<int64_t>(h) * HD;
    for (int c = tid; c < 2 * (HD / 8); c += kAttnThreads) {
      const bool isv = c >= HD / 8;
      const int cc = isv ? c - HD / 8 : c;
      const float* src = isv ? sm.vn : sm.kn;
      float f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = src[cc * 8 + e];
      st_vec((isv ? vc : kc) + cc * 8, S::pack(f));
    }
  }

  // ---- q^T as the B operand: column n = query head gid (zero past G) -------
  uint32_t qb[KS][2];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    const float* qh = sm.q[gid < G ? gid : 0] + ks * 16 + tig * 2;
    qb[ks][0] = gid < G ? pack2<T>(qh[0], qh[1]) : 0u;
    qb[ks][1] = gid < G ? pack2<T>(qh[8], qh[9]) : 0u;
  }
  const float qscale = a.scale * kLog2e;
  const bool h0_ok = 2 * tig < G, h1_ok = 2 * tig + 1 < G;

  // running state for this thread's two head columns 2*tig, 2*tig+1
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
  float o[KS][4];  // O^T: dims ks*16 + gid (+8), heads 2*tig (+1)
#pragma unroll
  for (int ks = 0; ks < KS; ++ks)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[ks][e] = 0.0f;

  for (int tile = 0; tile < ntiles; ++tile) {
    cp_async_wait<kStages - 2>();
    __syncthreads();  // tile visible to all; the buffer of tile-1 is free
    if (tile + kStages - 1 < ntiles) issue(tile + kStages - 1);
    cp_async_commit();
    const T* kt = ring + (tile % kStages) * (2 * kTile * HD);
    const T* vt = kt + kTile * HD;
    const int cnt = min(kTile, ncache - tile * kTile);
    const int wrow = warp * 16;
    if (wrow >= cnt) continue;  // warp-uniform: no positions of this tile for this warp
    const int mi = lane >> 3;   // the 8x8 matrix this lane addresses for ldmatrix

    // S^T (16 positions x 8 head columns) = K q^T
    float sacc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    {
      const int r = wrow + (mi & 1) * 8 + (lane & 7);
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t af[4];
        ldsm_x4(af, kt + swz<HD>(r, ks * 2 + (mi >> 1)));
        mma16816<T>(sacc, af, qb[ks][0], qb[ks][1]);
      }
    }
    // scale, mask, online softmax per head column
    const bool r0_ok = wrow + gid < cnt, r1_ok = wrow + gid + 8 < cnt;
    float sv[4];
    sv[0] = (r0_ok && h0_ok) ? sacc[0] * qscale : -INFINITY;
    sv[1] = (r0_ok && h1_ok) ? sacc[1] * qscale : -INFINITY;
    sv[2] = (r1_ok && h0_ok) ? sacc[2] * qscale : -INFINITY;
    sv[3] = (r1_ok && h1_ok) ? sacc[3] * qscale : -INFINITY;
    float alpha[2];
    bool rescale = false;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float mt = fmaxf(sv[c], sv[c + 2]);
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
      const float m_new = fmaxf(m_run[c], mt);
      alpha[c] = m_new == -INFINITY ? 1.0f : exp2f(m_run[c] - m_new);
      rescale |= alpha[c] != 1.0f;
      m_run[c] = m_new;
      sv[c] = sv[c] == -INFINITY ? 0.0f : exp2f(sv[c] - m_new);
      sv[c + 2] = sv[c + 2] == -INFINITY ? 0.0f : exp2f(sv[c + 2] - m_new);
      l_run[c] = fmaf(l_run[c], alpha[c], sv[c] + sv[c + 2]);
    }
    if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        o[ks][0] *= alpha[0];
        o[ks][1] *= alpha[1];
        o[ks][2] *= alpha[0];
        o[ks][3] *= alpha[1];
      }
    }
    // P^T (16 positions x 8 heads) as the B operand of O^T += V^T P^T
    const uint32_t pb0 = movmatrix_t(pack2<T>(sv[0], sv[1]));
    const uint32_t pb1 = movmatrix_t(pack2<T>(sv[2], sv[3]));
    {
      const int r = wrow + (mi >> 1) * 8 + (lane & 7);
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t af[4];
        ldsm_x4_t(af, vt + swz<HD>(r, ks * 2 + (mi & 1)));
        mma16816<T>(o[ks], af, pb0, pb1);
      }
    }
  }
  cp_async_wait<0>();

  if (fresh && owns_last && warp == 0) {
    // the token's own position, from the fresh (rotated, rounded) k and v:
    // lane holds dims [lane*HD/32, (lane+1)*HD/32) of each head's dot product
    constexpr int DPL = HD / 32;
    float dot[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float acc = 0.0f;
#pragma unroll
      for (int e = 0; e < DPL; ++e) acc = fmaf(sm.q[g][lane * DPL + e], sm.kn[lane * DPL + e], acc);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      dot[g] = acc * qscale;
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int hc = 2 * tig + c;
      float sf = -INFINITY;
#pragma unroll
      for (int g = 0; g < G; ++g)
        if (g == hc) sf = dot[g];
      if (hc < G) {
        const float m_new = fmaxf(m_run[c], sf);
        const float al = exp2f(m_run[c] - m_new);  // 0 when nothing was seen yet
        const float pf = exp2f(sf - m_new);
        m_run[c] = m_new;
        l_run[c] = l_run[c] * al + (gid == 0 ? pf : 0.0f);
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          o[ks][c] = fmaf(pf, sm.vn[ks * 16 + gid], o[ks][c] * al);
          o[ks][c + 2] = fmaf(pf, sm.vn[ks * 16 + gid + 8], o[ks][c + 2] * al);
        }
      }
    }
  }

  // per-warp sums over the 8 position rows held by the lanes of one column
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    l_run[c] += __shfl_xor_sync(0xffffffffu, l_run[c], 4);
    l_run[c] += __shfl_xor_sync(0xffffffffu, l_run[c], 8);
    l_run[c] += __shfl_xor_sync(0xffffffffu, l_run[c], 16);
  }
  __syncthreads();  // every warp is done with the ring: reuse it for the partials
  float* part = reinterpret_cast<float*>(ring);  // [warps][G][HD]
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int hc = 2 * tig + c;
    if (hc < G) {
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        part[(warp * G + hc) * HD + ks * 16 + gid] = o[ks][c];
        part[(warp * G + hc) * HD + ks * 16 + gid + 8] = o[ks][c + 2];
      }
    }
    if (gid == 0) {
      sm.wm[warp][hc] = m_run[c];
      sm.wl[warp][hc] = l_run[c];
    }
  }
  __syncthreads();
  // merge the warps: M = max_w m_w, weights exp2(m_w - M) (0 for empty warps)
  if (tid < G) {
    float M = sm.wm[0][tid];
#pragma unroll
    for (int w = 1; w < kAttnWarps; ++w) M = fmaxf(M, sm.wm[w][tid]);
    float L = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float sw = sm.wm[w][tid] == -INFINITY ? 0.0f : exp2f(sm.wm[w][tid] - M);
      sm.wscale[w][tid] = sw;
      L = fmaf(sm.wl[w][tid], sw, L);
    }
    sm.msplit[tid] = M;
    sm.l[tid] = L;
  }
  __syncthreads();
  auto merged = [&](int idx) {
    const int g = idx / HD;
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) v = fmaf(part[w * G * HD + idx], sm.wscale[w][g], v);
    return v;
  };

  // ---- output, or this split's partial + the last CTA's combine ---------------
  const int64_t pair = t * a.n_kv_heads + h;
  if (nsplit == 1) {
    for (int c = tid; c < G * HD / 8; c += kAttnThreads) {
      const int g = (c * 8) / HD;
      const float inv = 1.0f / sm.l[g];
      float f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = merged(c * 8 + e) * inv;
      st_vec(out + c * 8, S::pack(f));
    }
    return;
  }
  float* o_part = a.o_part + (pair * a.max_splits + s) * (G * HD);
  float2* ml_part = a.ml_part + (pair * a.max_splits + s) * G;
  for (int idx = tid; idx < G * HD; idx += kAttnThreads) o_part[idx] = merged(idx);
  if (tid < G) ml_part[tid] = make_float2(sm.msplit[tid], sm.l[tid]);
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int done = atomicAdd(a.counters + pair, 1);
    sm.last = done == nsplit - 1;
  }
  __syncthreads();
  if (!sm.last) return;
  __threadfence();
  // combine: weights w_s = exp2(m_s - M), L = sum_s l_s w_s
  const float2* ml_all = a.ml_part + pair * a.max_splits * G;
  if (tid < G) {
    float M = -INFINITY;
    for (int q = 0; q < nsplit; ++q) M = fmaxf(M, __ldcg(&ml_all[q * G + tid]).x);
    float L = 0.0f;
    for (int q = 0; q < nsplit; ++q) {
      const float2 ml = __ldcg(&ml_all[q * G + tid]);
      const float w = exp2f(ml.x - M);
      sm.w[q][tid] = w;
      L = fmaf(ml.y, w, L);
    }
    sm.l[tid] = L;
  }
  __syncthreads();
  // every thread owns 4 outputs; 8 splits are loaded before they are summed
  const float4* o_all = reinterpret_cast<const float4*>(a.o_part + pair * a.max_splits * (G * HD));
  for (int c = tid; c < G * HD / 4; c += kAttnThreads) {
    const int g = (c * 4) / HD;
    float4 f = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int q0 = 0; q0 < nsplit; q0 += 8) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        v[u] = q0 + u < nsplit ? __ldcg(o_all + (q0 + u) * (G * HD / 4) + c)
                               : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float w = q0 + u < nsplit ? sm.w[q0 + u][g] : 0.0f;
        f.x = fmaf(v[u].x, w, f.x);
        f.y = fmaf(v[u].y, w, f.y);
        f.z = fmaf(v[u].z, w, f.z);
        f.w = fmaf(v[u].w, w, f.w);
      }
    }
    const float inv = 1.0f / sm.l[g];
    const uint2 packed = make_uint2(pack2<T>(f.x * inv, f.y * inv), pack2<T>(f.z * inv, f.w * inv));
    *reinterpret_cast<uint2*>(out + c * 4) = packed;
  }
  if (tid == 0) a.counters[pair] = 0;  // ready for the next call
}

template <typename T, int HD, int G, int kStages>
cudaError_t launch_staged(const DecodeAttnArgs& a, bool pdl, cudaStream_t stream) {
  const InvFreq freq = make_inv_freq(a.rope_base, a.rotary_dim);
  constexpr size_t ring = static_cast<size_t>(kStages) * 2 * kTile * HD * sizeof(T);
  constexpr size_t partials = static_cast<size_t>(kAttnWarps) * G * HD * sizeof(float);
  constexpr size_t smem = attn_fixed_bytes<HD, G>() + (ring > partials ? ring : partials);
  static_assert(smem <= 227 * 1024, "decode attention shared memory");
  auto kernel = decode_attention_kernel<T, HD, G, kStages>;
  if (smem > 48 * 1024) {
    // once per device and instantiation, so that later launches (and CUDA
    // graph captures) make no further runtime calls
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
  // tokens on x (up to 2^31 - 1), kv heads on y, splits (<= 64) on z
  const dim3 grid(static_cast<unsigned>(a.tokens), static_cast<unsigned>(a.n_kv_heads),
                  static_cast<unsigned>(a.max_splits));
  return launch_kernel(kernel, grid, dim3(kAttnThreads), smem, stream, pdl, a, freq);
}

template <typename T, int HD, int G>
cudaError_t launch_typed(const DecodeAttnArgs& a, bool pdl, cudaStream_t stream) {
  const int64_t ctas = a.tokens * a.n_kv_heads * a.max_splits;
  const int64_t sms = sm_count();
  if (VL_ATTN_DEEP_RING && ctas <= sms) return launch_staged<T, HD, G, 4>(a, pdl, stream);
  if (VL_ATTN_DEEP_RING && ctas <= 2 * sms) return launch_staged<T, HD, G, 3>(a, pdl, stream);
  return launch_staged<T, HD, G, kStagesLarge>(a, pdl, stream);
}

template <typename T>
cudaError_t launch_dtype(const DecodeAttnArgs& a, bool pdl, cudaStream_t stream) {
  const int G = a.n_q_heads / a.n_kv_heads;
  if (a.head_dim == 128) {
    if (G == 1) return launch_typed<T, 128, 1>(a, pdl, stream);
    if (G == 2) return launch_typed<T, 128, 2>(a, pdl, stream);
    if (G == 4) return launch_typed<T, 128, 4>(a, pdl, stream);
    if (G == 8) return launch_typed<T, 128, 8>(a, pdl, stream);
  } else if (a.head_dim == 64) {
    if (G == 1) return launch_typed<T, 64, 1>(a, pdl, stream);
    if (G == 2) return launch_typed<T, 64, 2>(a, pdl, stream);
    if (G == 4) return launch_typed<T, 64, 4>(a, pdl, stream);
    if (G == 8) return launch_typed<T, 64, 8>(a, pdl, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

bool decode_attention_supported(int head_dim, int group) {
  return (head_dim == 128 || head_dim == 64) &&
         (group == 1 || group == 2 || group == 4 || group == 8);
}

// Positions per split: enough CTAs (about VL_ATTN_TARGET_CTAS when every
// sequence is at max_seq_len) to fill the GPU several times over, at most kMaxSplits
// splits, a power of two between 64 (one tile) and 4096.
int64_t decode_attention_split(int64_t tokens, int n_kv_heads, int64_t max_seq_len) {
  const int64_t pairs = tokens * n_kv_heads;
  int64_t want = (pairs * max_seq_len + VL_ATTN_TARGET_CTAS - 1) / VL_ATTN_TARGET_CTAS;
  const int64_t floor_splits = (max_seq_len + kMaxSplits - 1) / kMaxSplits;
  if (want < floor_splits) want = floor_splits;
  int64_t split = VL_ATTN_MIN_SPLIT;
  while (split < want && split < 4096) split <<= 1;
  return split;
}

size_t decode_attention_workspace_bytes(int64_t tokens, int n_q_heads, int n_kv_heads,
                                        int head_dim, int64_t max_seq_len) {
  const int64_t pairs = tokens * n_kv_heads;
  const int64_t split = decode_attention_split(tokens, n_kv_heads, max_seq_len);
  const int64_t splits = (max_seq_len + split - 1) / split;
  const int G = n_q_heads / n_kv_heads;
  const size_t counters = (static_cast<size_t>(pairs) * 4 + 255) & ~size_t(255);
  const size_t o = static_cast<size_t>(pairs) * splits * G * head_dim * 4;
  const size_t ml = static_cast<size_t>(pairs) * splits * G * 8;
  return counters + ((o + 255) & ~size_t(255)) + ml;
}

cudaError_t launch_decode_attention(DecodeAttnArgs a, int dtype, void* workspace, bool pdl,
                                    cudaStream_t stream) {
  if (a.tokens == 0) return cudaSuccess;
  a.split = static_cast<int>(decode_attention_split(a.tokens, a.n_kv_heads, a.max_seq_len));
  a.max_splits = static_cast<int>((a.max_seq_len + a.split - 1) / a.split);
  const int64_t pairs = a.tokens * a.n_kv_heads;
  const int G = a.n_q_heads / a.n_kv_heads;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  const size_t counters = (static_cast<size_t>(pairs) * 4 + 255) & ~size_t(255);
  const size_t o = static_cast<size_t>(pairs) * a.max_splits * G * a.head_dim * 4;
  a.counters = reinterpret_cast<int*>(ws);
  a.o_part = reinterpret_cast<float*>(ws + counters);
  a.ml_part = reinterpret_cast<float2*>(ws + counters + ((o + 255) & ~size_t(255)));
  if (dtype == kDtypeBF16) return launch_dtype<__nv_bfloat16>(a, pdl, stream);
  if (dtype == kDtypeF16) return launch_dtype<__half>(a, pdl, stream);
  return cudaErrorInvalidValue;
}

}  // namespace vl
