// Bit-exact row movers for sm_100a: token-embedding gather (with audio
// placeholder substitution) and slot-mapped KV-cache append.
//
// Reference semantics (VideoLingo-user native/asr/src/decoder.cu):
//   gather_inputs_kernel :60-78, gather_batch_kernel :636-654,
//   gather_ids_batched_kernel :659-667, gather_ids_mapped_kernel :460-469
//       out[pos] = id == audio_token ? audio[#placeholders before pos] : embed[id]
//   append_kv_kernel :940-948, append_kv_rows_kernel :873-882,
//   append_kv_batched(_dev)_kernel :857-870/:335-351, append_kv_mapped_kernel :500-514
//       cache[chunk][pos] = k/v row
// One warp moves one row with the widest access its alignment allows
// (16-byte vectors for 2048-wide bf16 rows: 8 per lane); a KV append of
// few tokens takes one block per token instead.  The reference
// counts placeholders with a serial O(pos) loop for every position; here
// only placeholder rows count, 32 ids per step with a warp ballot.
#include "vl_common.cuh"
#include "vl_kernels.h"

namespace vl {
namespace {

constexpr int kRowThreads = 256;  // 8 rows per block

// Copy `bytes` from src to dst with one warp.  `width` is the access size
// the caller proved legal for both pointers and the byte count.
__device__ __forceinline__ void warp_copy(void* dst, const void* src, int64_t bytes, int width,
                                          int lane) {
  if (width == 16) {
    const uint4* s = static_cast<const uint4*>(src);
    uint4* d = static_cast<uint4*>(dst);
    const int n = static_cast<int>(bytes >> 4);
#pragma unroll 4
    for (int i = lane; i < n; i += 32) st_vec(d + i, ld_vec(s + i));
  } else if (width == 4) {
    const uint32_t* s = static_cast<const uint32_t*>(src);
    uint32_t* d = static_cast<uint32_t*>(dst);
    for (int64_t i = lane; i < (bytes >> 2); i += 32) d[i] = s[i];
  } else {
    const uint16_t* s = static_cast<const uint16_t*>(src);
    uint16_t* d = static_cast<uint16_t*>(dst);
    for (int64_t i = lane; i < (bytes >> 1); i += 32) d[i] = s[i];
  }
}

__device__ __forceinline__ void warp_zero(void* dst, int64_t bytes, int width, int lane) {
  if (width == 16) {
    uint4* d = static_cast<uint4*>(dst);
    for (int64_t i = lane; i < (bytes >> 4); i += 32) st_vec(d + i, make_uint4(0, 0, 0, 0));
  } else if (width == 4) {
    uint32_t* d = static_cast<uint32_t*>(dst);
    for (int64_t i = lane; i < (bytes >> 2); i += 32) d[i] = 0u;
  } else {
    uint16_t* d = static_cast<uint16_t*>(dst);
    for (int64_t i = lane; i < (bytes >> 1); i += 32) d[i] = 0u;
  }
}

__global__ void __launch_bounds__(kRowThreads)
    embed_gather_kernel(const int64_t* __restrict__ ids, int64_t batch, int64_t seq,
                        int64_t ids_batch_stride, const int32_t* __restrict__ row_map,
                        const char* __restrict__ table, int64_t vocab, int64_t row_bytes,
                        const char* __restrict__ audio, int64_t audio_token_id,
                        int64_t audio_rows, int64_t audio_batch_stride_bytes, char* out,
                        int32_t* status, int width) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kRowThreads / 32) + (threadIdx.x >> 5);
  if (row >= batch * seq) return;
  const int64_t b = row / seq, s = row % seq;
  const int64_t src = row_map ? static_cast<int64_t>(row_map[b]) : b;
  const int64_t* id_row = ids + src * ids_batch_stride;
  const int64_t id = id_row[s];
  char* dst = out + row * row_bytes;
  const char* from = nullptr;
  int bad = 0;
  if (audio_token_id >= 0 && id == audio_token_id) {
    // j = number of placeholders strictly before s in this sequence.
    int64_t j = 0;
    for (int64_t base = 0; base < s; base += 32) {
      const int64_t p = base + lane;
      const bool hit = p < s && id_row[p] == audio_token_id;
      j += __popc(__ballot_sync(0xffffffffu, hit));
    }
    if (j < audio_rows) {
      from = audio + src * audio_batch_stride_bytes + j * row_bytes;
    } else {
      bad = VL_STATUS_BAD_AUDIO;
    }
  } else if (id >= 0 && id < vocab) {
    from = table + id * row_bytes;
  } else {
    bad = VL_STATUS_BAD_ID;
  }
  if (from) {
    warp_copy(dst, from, row_bytes, width, lane);
  } else {
    warp_zero(dst, row_bytes, width, lane);
    if (lane == 0 && status) atomicOr(status, bad);
  }
}

__global__ void __launch_bounds__(kRowThreads)
    kv_append_kernel(const char* __restrict__ k, const char* __restrict__ v, char* k_cache,
                     char* v_cache, const int64_t* __restrict__ slot_mapping, int64_t tokens,
                     int64_t row_bytes, int64_t ks, int64_t vs, int64_t num_slots,
                     int32_t* status, int width) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * (kRowThreads / 32) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const int64_t slot = slot_mapping[t];
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (lane == 0 && status) atomicOr(status, VL_STATUS_BAD_SLOT);
    return;
  }
  warp_copy(k_cache + slot * row_bytes, k + t * ks, row_bytes, width, lane);
  warp_copy(v_cache + slot * row_bytes, v + t * vs, row_bytes, width, lane);
}

// Few tokens (a decode step): one block per token, one 16-byte vector of K
// or V per thread.  The row vectors and the slot are requested together -
// only the stores depend on the slot - so a launch costs one memory round
// trip instead of two, and 64 tokens occupy 64 SMs instead of 8.
__global__ void __launch_bounds__(kRowThreads)
    kv_append_token_kernel(const char* __restrict__ k, const char* __restrict__ v,
                           char* k_cache, char* v_cache, const int64_t* __restrict__ slot_mapping,
                           int vec_per_row, int64_t ks, int64_t vs, int64_t num_slots,
                           int32_t* status) {
  const int64_t t = blockIdx.x;
  const int64_t row_bytes = static_cast<int64_t>(vec_per_row) * 16;
  for (int i = threadIdx.x; i < 2 * vec_per_row; i += blockDim.x) {
    const bool is_v = i >= vec_per_row;
    const int c = is_v ? i - vec_per_row : i;
    const uint4 val =
        ld_vec((is_v ? v + t * vs : k + t * ks) + static_cast<int64_t>(c) * 16);
    const int64_t slot = __ldg(slot_mapping + t);
    if (slot < 0) continue;
    if (slot >= num_slots) {
      if (i == 0 && status) atomicOr(status, VL_STATUS_BAD_SLOT);
      continue;
    }
    st_vec((is_v ? v_cache : k_cache) + slot * row_bytes + static_cast<int64_t>(c) * 16, val);
  }
}

int access_width(int64_t a, int64_t b, int64_t c, int64_t d) {
  const int64_t m = a | b | c | d;
  if ((m & 15) == 0) return 16;
  if ((m & 3) == 0) return 4;
  return 2;
}

}  // namespace

cudaError_t launch_embed_gather(const int64_t* ids, int64_t batch, int64_t seq,
                                int64_t ids_batch_stride, const int32_t* row_map,
                                const void* table, int64_t vocab, int64_t row_bytes,
                                const void* audio, int64_t audio_token_id, int64_t audio_rows,
                                int64_t audio_batch_stride_bytes, void* out, int32_t* status,
                                cudaStream_t stream) {
  const int64_t rows = batch * seq;
  if (rows == 0) return cudaSuccess;
  const int width = access_width(reinterpret_cast<intptr_t>(table), reinterpret_cast<intptr_t>(out),
                                 row_bytes,
                                 audio ? (reinterpret_cast<intptr_t>(audio) | audio_batch_stride_bytes) : 0);
  const int64_t blocks = (rows + kRowThreads / 32 - 1) / (kRowThreads / 32);
  embed_gather_kernel<<<static_cast<unsigned>(blocks), kRowThreads, 0, stream>>>(
      ids, batch, seq, ids_batch_stride, row_map, static_cast<const char*>(table), vocab,
      row_bytes, static_cast<const char*>(audio), audio_token_id, audio_rows,
      audio_batch_stride_bytes, static_cast<char*>(out), status, width);
  return cudaGetLastError();
}

cudaError_t launch_kv_append(const void* k, const void* v, void* k_cache, void* v_cache,
                             const int64_t* slot_mapping, int64_t tokens, int64_t row_bytes,
                             int64_t k_row_stride_bytes, int64_t v_row_stride_bytes,
                             int64_t num_slots, int32_t* status, cudaStream_t stream) {
  if (tokens == 0) return cudaSuccess;
  const int width = access_width(
      reinterpret_cast<intptr_t>(k) | reinterpret_cast<intptr_t>(v),
      reinterpret_cast<intptr_t>(k_cache) | reinterpret_cast<intptr_t>(v_cache), row_bytes,
      k_row_stride_bytes | v_row_stride_bytes);
  if (width == 16 && tokens <= 2 * static_cast<int64_t>(sm_count()) &&
      row_bytes / 16 <= (int64_t(1) << 20)) {
    const int vpr = static_cast<int>(row_bytes / 16);
    int threads = ((2 * vpr + 31) / 32) * 32;
    if (threads > kRowThreads) threads = kRowThreads;
    kv_append_token_kernel<<<static_cast<unsigned>(tokens), threads, 0, stream>>>(
        static_cast<const char*>(k), static_cast<const char*>(v), static_cast<char*>(k_cache),
        static_cast<char*>(v_cache), slot_mapping, vpr, k_row_stride_bytes, v_row_stride_bytes,
        num_slots, status);
    return cudaGetLastError();
  }
  const int64_t blocks = (tokens + kRowThreads / 32 - 1) / (kRowThreads / 32);
  kv_append_kernel<<<static_cast<unsigned>(blocks), kRowThreads, 0, stream>>>(
      static_cast<const char*>(k), static_cast<const char*>(v), static_cast<char*>(k_cache),
      static_cast<char*>(v_cache), slot_mapping, tokens, row_bytes, k_row_stride_bytes,
      v_row_stride_bytes, num_slots, status, width);
  return cudaGetLastError();
}

}  // namespace vl
