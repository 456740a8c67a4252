// Decode-step tail for sm_100a: greedy next token per row with the EOS
// freeze and the per-chunk bookkeeping, in one launch.
//
// Reference semantics (VideoLingo-user native/asr/src/decoder.cu):
// argmax_mapped_kernel (:573-621) and, without the bookkeeping,
// argmax_rows_kernel (:755-782).  Both run 256 threads per row: thread t
// keeps the first strictly greater value over j = t, t+256, ... (from
// -1e30), then thread 0 keeps the first strictly greater thread in thread
// order.  The winner is therefore the largest value above -1e30 (NaN never
// wins), ties going to the smallest j mod 256 and then the smallest j - an
// order this kernel reproduces with any block shape by reducing (value,
// key) pairs, key = (j mod 256) << 24 | j.  A finished chunk skips the scan
// and yields the freeze id; otherwise the id is stored at output row
// positions[c] - prompt_length + 1 and an EOS id finishes the chunk.
//
// One CTA of 512 threads per row streams the row with 16-byte loads; the
// whole step's bookkeeping (freeze, id store, finished flag, current id)
// is done by thread 0, replacing the float conversion, argmax and six
// small bookkeeping kernels of a torch tail.
#include "vl_common.cuh"
#include "vl_kernels.h"

namespace vl {
namespace {

constexpr int kArgmaxThreads = 512;
constexpr uint32_t kNoKey = 0xffffffffu;

__device__ __forceinline__ bool argmax_better(float v, uint32_t key, float bv, uint32_t bkey) {
  return v > bv || (v == bv && key < bkey);
}

template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads) argmax_eos_kernel(const __grid_constant__ ArgmaxArgs a) {
  using S = Storage<T>;
  constexpr int kVec = S::kVec;
  const int64_t r = blockIdx.x;
  const int tid = threadIdx.x;
  const int64_t c = a.row_chunk ? static_cast<int64_t>(a.row_chunk[r]) : r;
  if (c < 0 || c >= a.chunks) {
    if (tid == 0 && a.status) atomicOr(a.status, VL_STATUS_BAD_SLOT);
    return;
  }
  const bool tracked = a.finished != nullptr;
  if (tracked && a.finished[c]) {  // the reference skips the scan of a finished chunk
    if (tid == 0) a.current_ids[c] = a.freeze_id;
    return;
  }

  float best = -1e30f;
  uint32_t key = kNoKey;
  const T* row = static_cast<const T*>(a.logits) + r * a.row_stride;
  const int64_t nvec = a.vocab / kVec;
  for (int64_t i = tid; i < nvec; i += kArgmaxThreads) {
    float f[kVec];
    S::unpack(ld_stream(row + i * kVec), f);
#pragma unroll
    for (int e = 0; e < kVec; ++e) {
      const uint32_t j = static_cast<uint32_t>(i * kVec + e);
      const uint32_t kj = ((j & 255u) << 24) | j;
      if (f[e] > -1e30f && argmax_better(f[e], kj, best, key)) {
        best = f[e];
        key = kj;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const uint32_t ok = __shfl_xor_sync(0xffffffffu, key, o);
    if (argmax_better(ov, ok, best, key)) {
      best = ov;
      key = ok;
    }
  }
  __shared__ float warp_best[kArgmaxThreads / 32];
  __shared__ uint32_t warp_key[kArgmaxThreads / 32];
  const int lane = tid & 31, warp = tid >> 5;
  if (lane == 0) {
    warp_best[warp] = best;
    warp_key[warp] = key;
  }
  __syncthreads();
  if (tid != 0) return;
  for (int w = 1; w < kArgmaxThreads / 32; ++w)
    if (argmax_better(warp_best[w], warp_key[w], best, key)) {
      best = warp_best[w];
      key = warp_key[w];
    }
  const int64_t id = key != kNoKey ? static_cast<int64_t>(key & 0xffffffu)
                                   : (tracked ? a.freeze_id : 0);
  if (tracked) {
    if (a.out_ids) {
      const int64_t orow = static_cast<int64_t>(a.positions[c]) - *a.prompt_length + 1;
      if (orow >= 0 && orow < a.out_rows)
        a.out_ids[orow * a.out_stride + c] = id;
      else if (a.status)
        atomicOr(a.status, VL_STATUS_BAD_SLOT);
    }
    for (int e = 0; e < a.n_eos; ++e)
      if (id == a.eos[e]) a.finished[c] = 1;
  }
  a.current_ids[c] = id;
}

}  // namespace

cudaError_t launch_argmax_eos(const ArgmaxArgs& a, int dtype, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(a.rows));
  if (dtype == kDtypeBF16)
    argmax_eos_kernel<__nv_bfloat16><<<grid, kArgmaxThreads, 0, stream>>>(a);
  else if (dtype == kDtypeF16)
    argmax_eos_kernel<__half><<<grid, kArgmaxThreads, 0, stream>>>(a);
  else if (dtype == kDtypeF32)
    argmax_eos_kernel<float><<<grid, kArgmaxThreads, 0, stream>>>(a);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace vl
