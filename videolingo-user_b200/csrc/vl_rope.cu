// Rotate-half rotary embedding applied in place to Q/K, and its decode-step
// fusion with the KV-cache append, for sm_100a.
//
// Reference semantics (VideoLingo-user native/asr/src):
//   rope_kernel (engine.cu:214-233) + build_rope_table (engine.cu:892-905)
//   rope_full / rope_rows / rope_at_position(_dev/_map) kernels
//   (decoder.cu:113-134, 307-333, 471-498, 670-695, 789-814)
//   + build_full_rope_table (decoder.cu:950-961)
//       inv_freq(d) = 1/pow(base, 2d/rot) (fp64), angle = inv_freq * pos (fp64),
//       cos/sin rounded to fp32;  x1' = x1*c - x2*s, x2' = x2*c + x1*s
//       over the pairs (d, d + rot/2), d < rot/2, of every head.
// The reference reads cos/sin from host-built tables of 1024 or 1500 rows;
// here they are evaluated per (token, pair) on the device (no table, no
// position limit): the angle in fp64, reduced modulo 2*pi in fp64, then an
// fp32 sincosf.  One warp owns one token: lane l rotates the 16-byte
// vector l % per_head of the x1 half together with its x2 partner for head
// l / per_head (+ multiples of 32 / per_head), so indexing is shifts only,
// the first vectors are requested before the cos/sin evaluation, and
// the untouched half of each head is never read.  Shapes whose rotated half
// is not a power-of-two number of 16-byte vectors use a scalar block kernel.
#include <cmath>

#include "vl_common.cuh"
#include "vl_kernels.h"
#include "vl_rope_math.cuh"

namespace vl {
namespace {

constexpr int kRopeThreads = 128;
constexpr int kMaxTokensPerBlock = 8;

__device__ __forceinline__ int64_t token_position(const RopeArgs& a, int64_t r) {
  if (a.positions == nullptr) return a.pos_offset + (a.seq_len > 0 ? r % a.seq_len : r);
  const int64_t src = a.row_map ? static_cast<int64_t>(a.row_map[r]) : r;
  return a.pos_offset + static_cast<int64_t>(a.positions[src * a.positions_stride]);
}

// Head row of task i of this block: task = (token t, head h, vector/pair j).
template <typename T>
__device__ __forceinline__ T* task_head(const RopeArgs& a, int64_t t0, int i, int tasks,
                                        int per_head, int* t_out, int* j_out) {
  const int t = i / tasks;
  const int rem = i - t * tasks;
  const int h = rem / per_head;
  *t_out = t;
  *j_out = rem - h * per_head;
  const int64_t r = t0 + t;
  return h < a.n_q_heads
             ? static_cast<T*>(a.q) + r * a.q_row_stride + static_cast<int64_t>(h) * a.head_dim
             : static_cast<T*>(a.k) + r * a.k_row_stride +
                   static_cast<int64_t>(h - a.n_q_heads) * a.head_dim;
}

template <typename T, bool kVec>
__global__ void __launch_bounds__(kRopeThreads)
    rope_kernel(const __grid_constant__ RopeArgs a, const __grid_constant__ InvFreq freq,
                int tokens_per_block) {
  using S = Storage<T>;
  constexpr int E = S::kVec;
  constexpr int G = 4;  // tasks whose vectors are in flight per thread
  extern __shared__ float2 cs[];  // [tokens_per_block][half_rot] (cos, sin)
  const int half_rot = a.rotary_dim / 2;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * tokens_per_block;
  int nt = tokens_per_block;
  if (t0 + nt > a.tokens) nt = static_cast<int>(a.tokens - t0);
  const int heads = a.n_q_heads + a.n_k_heads;
  const int per_head = kVec ? half_rot / E : half_rot;
  const int tasks = heads * per_head;
  const int ntask = nt * tasks;

  // Vector path: the first group of x1/x2 vectors is requested before the
  // cos/sin evaluation, so the HBM latency overlaps it.
  uint4 x1v[G], x2v[G];
  if (kVec) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int i = threadIdx.x + g * kRopeThreads;
      if (i < ntask) {
        int t, j;
        T* head = task_head<T>(a, t0, i, tasks, per_head, &t, &j);
        x1v[g] = ld_vec(head + j * E);
        x2v[g] = ld_vec(head + half_rot + j * E);
      }
    }
  }

  for (int i = threadIdx.x; i < nt * half_rot; i += kRopeThreads) {
    const int t = i / half_rot, d = i % half_rot;
    cs[i] = rope_cos_sin(static_cast<double>(token_position(a, t0 + t)) * freq.v[d]);
  }
  __syncthreads();

  if (kVec) {
    for (int base = threadIdx.x; base < ntask; base += kRopeThreads * G) {
      if (base != static_cast<int>(threadIdx.x)) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const int i = base + g * kRopeThreads;
          if (i < ntask) {
            int t, j;
            T* head = task_head<T>(a, t0, i, tasks, per_head, &t, &j);
            x1v[g] = ld_vec(head + j * E);
            x2v[g] = ld_vec(head + half_rot + j * E);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int i = base + g * kRopeThreads;
        if (i < ntask) {
          int t, j;
          T* head = task_head<T>(a, t0, i, tasks, per_head, &t, &j);
          const float2* cst = cs + t * half_rot + j * E;
          float x1[E], x2[E], y1[E], y2[E];
          S::unpack(x1v[g], x1);
          S::unpack(x2v[g], x2);
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const float c = cst[e].x, s = cst[e].y;
            y1[e] = x1[e] * c - x2[e] * s;
            y2[e] = x2[e] * c + x1[e] * s;
          }
          st_vec(head + j * E, S::pack(y1));
          st_vec(head + half_rot + j * E, S::pack(y2));
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < ntask; i += kRopeThreads) {
      int t, j;
      T* head = task_head<T>(a, t0, i, tasks, per_head, &t, &j);
      const float c = cs[t * half_rot + j].x, s = cs[t * half_rot + j].y;
      const float x1 = S::to_float(head[j]);
      const float x2 = S::to_float(head[j + half_rot]);
      head[j] = S::from_float(x1 * c - x2 * s);
      head[j + half_rot] = S::from_float(x2 * c + x1 * s);
    }
  }

  if (a.v == nullptr) return;
  // Fused KV append: the rotated K rows written above are visible to the
  // whole block after the barrier; copy them and the V rows to their slots.
  __syncthreads();
  const int64_t row_elems = static_cast<int64_t>(a.n_k_heads) * a.head_dim;
  const int64_t vec_per_row = kVec ? row_elems / E : row_elems;
  for (int64_t i = threadIdx.x; i < nt * vec_per_row; i += kRopeThreads) {
    const int t = static_cast<int>(i / vec_per_row);
    const int64_t c = i % vec_per_row;
    const int64_t r = t0 + t;
    const int64_t slot = a.slot_mapping[r];
    if (slot < 0) continue;
    if (slot >= a.num_slots) {
      if (c == 0 && a.status) atomicOr(a.status, VL_STATUS_BAD_SLOT);
      continue;
    }
    const T* krow = static_cast<const T*>(a.k) + r * a.k_row_stride;
    const T* vrow = static_cast<const T*>(a.v) + r * row_elems;
    T* kc = static_cast<T*>(a.k_cache) + slot * row_elems;
    T* vc = static_cast<T*>(a.v_cache) + slot * row_elems;
    if (kVec) {
      st_vec(reinterpret_cast<uint4*>(kc) + c, ld_vec(reinterpret_cast<const uint4*>(krow) + c));
      st_vec(reinterpret_cast<uint4*>(vc) + c, ld_vec(reinterpret_cast<const uint4*>(vrow) + c));
    } else {
      kc[c] = krow[c];
      vc[c] = vrow[c];
    }
  }
}

constexpr int kWarpRopeWarps = 4;         // tokens per block
constexpr int kWarpRopePrefetch = 3;      // head iterations of a token requested ahead

template <typename T>
__device__ __forceinline__ T* head_row(const RopeArgs& a, int64_t r, int h) {
  return h < a.n_q_heads
             ? static_cast<T*>(a.q) + r * a.q_row_stride + static_cast<int64_t>(h) * a.head_dim
             : static_cast<T*>(a.k) + r * a.k_row_stride +
                   static_cast<int64_t>(h - a.n_q_heads) * a.head_dim;
}

// PH = 16-byte vectors per rotated half (a power of two <= 32).
// PH = 16-byte vectors per rotated half (a power of two <= 32).  Persistent:
// warp w handles tokens w, w + total warps, ...; the next token's vectors are
// requested before the current token is rotated, so HBM latency overlaps
// the cos/sin evaluation and the rotation of the previous token.
template <typename T, int PH>
__global__ void __launch_bounds__(kWarpRopeWarps * 32)
    rope_warp_kernel(const __grid_constant__ RopeArgs a, const __grid_constant__ InvFreq freq) {
  using S = Storage<T>;
  constexpr int E = S::kVec;
  constexpr int kHalf = PH * E;            // rotary_dim / 2
  constexpr int kHeadsPerIter = 32 / PH;
  constexpr int P = kWarpRopePrefetch;
  __shared__ float2 cs_all[kWarpRopeWarps][kHalf];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t r = static_cast<int64_t>(blockIdx.x) * kWarpRopeWarps + warp;
  if (r >= a.tokens) return;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarpRopeWarps;
  const int heads = a.n_q_heads + a.n_k_heads;
  const int iters = (heads + kHeadsPerIter - 1) / kHeadsPerIter;
  const int j = lane & (PH - 1);
  const int hl = lane / PH;
  float2* cs = cs_all[warp];

  uint4 x1v[P], x2v[P], n1v[P], n2v[P];
  auto load = [&](int64_t tok, uint4 (&d1)[P], uint4 (&d2)[P]) {
#pragma unroll
    for (int it = 0; it < P; ++it) {
      const int h = it * kHeadsPerIter + hl;
      if (it < iters && h < heads) {
        T* row = head_row<T>(a, tok, h);
        d1[it] = ld_vec(row + j * E);
        d2[it] = ld_vec(row + kHalf + j * E);
      }
    }
  };
  load(r, x1v, x2v);

  for (;;) {
    const int64_t rn = r + stride;
    const double pos = static_cast<double>(token_position(a, r));
    for (int d = lane; d < kHalf; d += 32) cs[d] = rope_cos_sin(pos * freq.v[d]);
    __syncwarp();
    float c[E], sn[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float2 v = cs[j * E + e];
      c[e] = v.x;
      sn[e] = v.y;
    }
    if (rn < a.tokens) load(rn, n1v, n2v);

    auto rotate = [&](int h, const uint4& v1, const uint4& v2) {
      float x1[E], x2[E], y1[E], y2[E];
      S::unpack(v1, x1);
      S::unpack(v2, x2);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        y1[e] = x1[e] * c[e] - x2[e] * sn[e];
        y2[e] = x2[e] * c[e] + x1[e] * sn[e];
      }
      T* row = head_row<T>(a, r, h);
      st_vec(row + j * E, S::pack(y1));
      st_vec(row + kHalf + j * E, S::pack(y2));
    };
#pragma unroll
    for (int it = 0; it < P; ++it) {
      const int h = it * kHeadsPerIter + hl;
      if (it < iters && h < heads) rotate(h, x1v[it], x2v[it]);
    }
    for (int it = P; it < iters; ++it) {  // heads beyond the prefetch depth
      const int h = it * kHeadsPerIter + hl;
      if (h < heads) {
        T* row = head_row<T>(a, r, h);
        rotate(h, ld_vec(row + j * E), ld_vec(row + kHalf + j * E));
      }
    }

    if (a.v != nullptr) {
      // Fused KV append: copy this token's (now rotated) K row and its V row
      // to the slot; the warp's own stores above are visible after the sync.
      __syncwarp();
      const int64_t slot = a.slot_mapping[r];
      if (slot >= a.num_slots) {
        if (lane == 0 && a.status) atomicOr(a.status, VL_STATUS_BAD_SLOT);
      } else if (slot >= 0) {
        const int64_t row_elems = static_cast<int64_t>(a.n_k_heads) * a.head_dim;
        const uint4* krow =
            reinterpret_cast<const uint4*>(static_cast<const T*>(a.k) + r * a.k_row_stride);
        const uint4* vrow =
            reinterpret_cast<const uint4*>(static_cast<const T*>(a.v) + r * row_elems);
        uint4* kc = reinterpret_cast<uint4*>(static_cast<T*>(a.k_cache) + slot * row_elems);
        uint4* vc = reinterpret_cast<uint4*>(static_cast<T*>(a.v_cache) + slot * row_elems);
        for (int64_t i = lane; i < row_elems / E; i += 32) {
          st_vec(kc + i, ld_vec(krow + i));
          st_vec(vc + i, ld_vec(vrow + i));
        }
      }
    }
    if (rn >= a.tokens) break;
#pragma unroll
    for (int it = 0; it < P; ++it) {
      x1v[it] = n1v[it];
      x2v[it] = n2v[it];
    }
    r = rn;
    __syncwarp();  // every lane has read cs before the next token overwrites it
  }
}

template <typename T, int PH>
void launch_warp_rope(const RopeArgs& a, const InvFreq& freq, cudaStream_t stream) {
  const int64_t need = (a.tokens + kWarpRopeWarps - 1) / kWarpRopeWarps;
  const int64_t cap = resident_blocks(reinterpret_cast<const void*>(rope_warp_kernel<T, PH>),
                                      kWarpRopeWarps * 32, 0);
  const int64_t blocks = need < cap ? need : cap;
  rope_warp_kernel<T, PH><<<static_cast<unsigned>(blocks), kWarpRopeWarps * 32, 0, stream>>>(a, freq);
}

template <typename T>
cudaError_t rope_typed(const RopeArgs& a, cudaStream_t stream) {
  constexpr int E = Storage<T>::kVec;
  const int half_rot = a.rotary_dim / 2;
  const InvFreq freq = make_inv_freq(a.base, a.rotary_dim);
  const int64_t row_elems = static_cast<int64_t>(a.n_k_heads) * a.head_dim;
  bool vec = half_rot % E == 0 && a.head_dim % E == 0 && aligned16(a.q) &&
             a.q_row_stride % E == 0 &&
             (a.n_k_heads == 0 || (aligned16(a.k) && a.k_row_stride % E == 0));
  if (a.v != nullptr)
    vec = vec && aligned16(a.v) && aligned16(a.k_cache) && aligned16(a.v_cache) &&
          row_elems % E == 0;
  // Enough blocks to fill every SM's 16 resident blocks, up to 8 tokens each.
  const int64_t want_blocks = static_cast<int64_t>(sm_count()) * 16;
  int64_t tpb = (a.tokens + want_blocks - 1) / want_blocks;
  if (tpb < 1) tpb = 1;
  if (tpb > kMaxTokensPerBlock) tpb = kMaxTokensPerBlock;
  const int64_t blocks = (a.tokens + tpb - 1) / tpb;
  const size_t smem = static_cast<size_t>(tpb) * half_rot * sizeof(float2);
  const int per_head = half_rot / E;
  if (vec && per_head <= 32 && (per_head & (per_head - 1)) == 0) {
    switch (per_head) {
      case 1: launch_warp_rope<T, 1>(a, freq, stream); break;
      case 2: launch_warp_rope<T, 2>(a, freq, stream); break;
      case 4: launch_warp_rope<T, 4>(a, freq, stream); break;
      case 8: launch_warp_rope<T, 8>(a, freq, stream); break;
      case 16: launch_warp_rope<T, 16>(a, freq, stream); break;
      default: launch_warp_rope<T, 32>(a, freq, stream); break;
    }
  } else if (vec)
    rope_kernel<T, true><<<static_cast<unsigned>(blocks), kRopeThreads, smem, stream>>>(
        a, freq, static_cast<int>(tpb));
  else
    rope_kernel<T, false><<<static_cast<unsigned>(blocks), kRopeThreads, smem, stream>>>(
        a, freq, static_cast<int>(tpb));
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_rope(const RopeArgs& args, int dtype, cudaStream_t stream) {
  if (args.tokens == 0) return cudaSuccess;
  switch (dtype) {
    case kDtypeF32: return rope_typed<float>(args, stream);
    case kDtypeF16: return rope_typed<__half>(args, stream);
    default: return rope_typed<__nv_bfloat16>(args, stream);
  }
}

}  // namespace vl
