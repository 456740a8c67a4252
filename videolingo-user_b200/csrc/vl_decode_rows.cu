// The row ops of a decode step in one launch, for sm_100a: residual add +
// RMSNorm of the hidden rows, rotary embedding of the new q/k rows at each
// sequence's position, and the append of the rotated k and of v to the KV
// cache.
//
// Reference semantics (VideoLingo-user native/asr/src/decoder.cu): the step
// at :1702-1733 launches rope_at_position_map_kernel (:471-498),
// append_kv_mapped_kernel (:500-514), and residual_add_kernel (:933-938) +
// cudaMemcpyAsync + rmsnorm_kernel (:81-101) - five launches of a few
// microseconds each, every one a single dependent chain of memory accesses.
// Here one grid runs them side by side: blocks [0, rows) normalise one row
// each (vl_rows.cuh), blocks [rows, rows + tokens) rotate and append one
// token each.  A token block requests all of its q/k/v vectors and its slot
// before it evaluates the cos/sin of the token's position, so the whole
// launch costs about one memory round trip.
//
// The two halves read and write disjoint buffers (the caller guarantees it:
// the norm's rows are not the q/k/v rows), which is what lets them share a
// launch; within a token block the rotated k vector goes to the cache from
// the register that holds it, so no block reads what another writes.
#include "vl_common.cuh"
#include "vl_kernels.h"
#include "vl_rope_math.cuh"
#include "vl_rows.cuh"

namespace vl {
namespace {

constexpr int kPrefetch = 2;  // tasks per thread whose vectors are requested up front

template <typename T>
__device__ __forceinline__ void token_task(const DecodeRowsArgs& a, int64_t t, int task,
                                           int64_t slot, bool load_only, uint4& x1, uint4& x2,
                                           const float2* cs) {
  using S = Storage<T>;
  constexpr int E = S::kVec;
  const int half_rot = a.rotary_dim / 2;
  const int ph = half_rot / E;                  // rotated pair vectors per head
  const int vh = a.head_dim / E;                // vectors per head
  const int heads = a.n_q_heads + a.n_kv_heads;
  const int n_pair = heads * ph;
  const int n_pass = a.n_kv_heads * (vh - 2 * ph);
  const int64_t cache_row = static_cast<int64_t>(a.n_kv_heads) * a.head_dim;
  const bool slot_ok = slot >= 0 && slot < a.num_slots;
  if (task < n_pair) {
    const int h = task / ph, j = task - (task / ph) * ph;
    T* row = h < a.n_q_heads
                 ? static_cast<T*>(a.q) + t * a.q_row_stride + static_cast<int64_t>(h) * a.head_dim
                 : static_cast<T*>(a.k) + t * a.kv_row_stride +
                       static_cast<int64_t>(h - a.n_q_heads) * a.head_dim;
    if (load_only) {
      x1 = ld_vec(row + j * E);
      x2 = ld_vec(row + half_rot + j * E);
      return;
    }
    float v1[E], v2[E], y1[E], y2[E];
    S::unpack(x1, v1);
    S::unpack(x2, v2);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float2 c = cs[j * E + e];
      y1[e] = v1[e] * c.x - v2[e] * c.y;
      y2[e] = v2[e] * c.x + v1[e] * c.y;
    }
    const uint4 o1 = S::pack(y1), o2 = S::pack(y2);
    st_vec(row + j * E, o1);
    st_vec(row + half_rot + j * E, o2);
    if (h >= a.n_q_heads && slot_ok) {
      T* dst = static_cast<T*>(a.k_cache) + slot * cache_row +
               static_cast<int64_t>(h - a.n_q_heads) * a.head_dim;
      st_vec(dst + j * E, o1);
      st_vec(dst + half_rot + j * E, o2);
    }
    return;
  }
  task -= n_pair;
  if (task < n_pass) {  // k vectors past the rotated dims: copied as they are
    const int per = vh - 2 * ph;
    const int kh = task / per, c = 2 * ph + (task - (task / per) * per);
    const int64_t off = static_cast<int64_t>(kh) * a.head_dim + static_cast<int64_t>(c) * E;
    if (load_only) {
      x1 = ld_vec(static_cast<const T*>(a.k) + t * a.kv_row_stride + off);
      return;
    }
    if (slot_ok) st_vec(static_cast<T*>(a.k_cache) + slot * cache_row + off, x1);
    return;
  }
  task -= n_pass;  // v vectors
  const int64_t off = static_cast<int64_t>(task) * E;
  if (load_only) {
    x1 = ld_vec(static_cast<const T*>(a.v) + t * a.kv_row_stride + off);
    return;
  }
  if (slot_ok) st_vec(static_cast<T*>(a.v_cache) + slot * cache_row + off, x1);
}

template <typename T, int NV>
__global__ void __launch_bounds__(kRowBlockThreads)
    decode_rows_kernel(const __grid_constant__ DecodeRowsArgs a,
                       const __grid_constant__ InvFreq freq) {
  using S = Storage<T>;
  constexpr int E = S::kVec;
  __shared__ float red[2 * kRowBlockThreads / 32];
  __shared__ float2 cs[kMaxHalfRot];
  if (static_cast<int64_t>(blockIdx.x) < a.rows) {
    if (a.delta != nullptr)
      add_norm_row_block<T, NV, true, true>(static_cast<T*>(a.residual),
                                            static_cast<const T*>(a.delta),
                                            static_cast<const T*>(a.weight), nullptr,
                                            static_cast<T*>(a.out), blockIdx.x, a.cols, a.eps, red);
    else
      add_norm_row_block<T, NV, false, true>(static_cast<T*>(a.residual), nullptr,
                                             static_cast<const T*>(a.weight), nullptr,
                                             static_cast<T*>(a.out), blockIdx.x, a.cols, a.eps,
                                             red);
    return;
  }
  const int64_t t = static_cast<int64_t>(blockIdx.x) - a.rows;
  const int half_rot = a.rotary_dim / 2;
  const int ph = half_rot / E, vh = a.head_dim / E;
  const int total = (a.n_q_heads + a.n_kv_heads) * ph + a.n_kv_heads * (vh - 2 * ph) +
                    a.n_kv_heads * vh;
  const int64_t slot = __ldg(a.slot_mapping + t);
  uint4 x1[kPrefetch], x2[kPrefetch];
#pragma unroll
  for (int p = 0; p < kPrefetch; ++p) {
    const int task = threadIdx.x + p * kRowBlockThreads;
    if (task < total) token_task<T>(a, t, task, slot, true, x1[p], x2[p], cs);
  }
  if (threadIdx.x < half_rot) {
    const double pos = static_cast<double>(__ldg(a.positions + t));
    cs[threadIdx.x] = rope_cos_sin(pos * freq.v[threadIdx.x]);
  }
  if (threadIdx.x == 0 && slot >= a.num_slots && a.status != nullptr)
    atomicOr(a.status, VL_STATUS_BAD_SLOT);
  __syncthreads();
#pragma unroll
  for (int p = 0; p < kPrefetch; ++p) {
    const int task = threadIdx.x + p * kRowBlockThreads;
    if (task < total) token_task<T>(a, t, task, slot, false, x1[p], x2[p], cs);
  }
  for (int task = threadIdx.x + kPrefetch * kRowBlockThreads; task < total;
       task += kRowBlockThreads) {
    uint4 y1, y2;
    token_task<T>(a, t, task, slot, true, y1, y2, cs);
    token_task<T>(a, t, task, slot, false, y1, y2, cs);
  }
}

template <typename T>
cudaError_t decode_rows_typed(const DecodeRowsArgs& a, cudaStream_t stream) {
  constexpr int E = Storage<T>::kVec;
  const InvFreq freq = make_inv_freq(a.rope_base, a.rotary_dim);
  const int64_t blocks = a.rows + a.tokens;
  const int per_thread = (a.cols / E + kRowBlockThreads - 1) / kRowBlockThreads;
  const dim3 grid(static_cast<unsigned>(blocks));
  if (per_thread <= 1)
    decode_rows_kernel<T, 1><<<grid, kRowBlockThreads, 0, stream>>>(a, freq);
  else if (per_thread == 2)
    decode_rows_kernel<T, 2><<<grid, kRowBlockThreads, 0, stream>>>(a, freq);
  else
    decode_rows_kernel<T, 4><<<grid, kRowBlockThreads, 0, stream>>>(a, freq);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_decode_rows(const DecodeRowsArgs& args, int dtype, cudaStream_t stream) {
  if (args.rows + args.tokens == 0) return cudaSuccess;
  switch (dtype) {
    case kDtypeF32: return decode_rows_typed<float>(args, stream);
    case kDtypeF16: return decode_rows_typed<__half>(args, stream);
    default: return decode_rows_typed<__nv_bfloat16>(args, stream);
  }
}

}  // namespace vl
