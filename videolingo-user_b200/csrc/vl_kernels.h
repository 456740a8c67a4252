// Internal launcher interface between the C ABI (vl_api.cu) and the kernel
// translation units.  Arguments arrive already validated; every launcher only
// enqueues work on `stream` and returns the launch status.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace vl {

cudaError_t launch_add_norm(void* residual, const void* delta, const void* gamma,
                            const void* beta, void* out, int64_t rows, int64_t cols, float eps,
                            bool rms, int dtype, cudaStream_t stream);

cudaError_t launch_gelu(const void* in, const void* bias, void* out, int64_t rows, int64_t cols,
                        int dtype, cudaStream_t stream);

cudaError_t launch_swiglu(const void* gate, const void* up, void* out, int64_t rows, int64_t cols,
                          int64_t gate_stride, int64_t up_stride, int64_t out_stride, int dtype,
                          cudaStream_t stream);

struct RopeArgs {
  void* q;
  void* k;
  const int32_t* positions;
  const int32_t* row_map;
  int64_t positions_stride;
  int64_t pos_offset;
  int64_t tokens;
  int64_t seq_len;
  int n_q_heads;
  int n_k_heads;
  int head_dim;
  int rotary_dim;
  double base;
  int64_t q_row_stride;
  int64_t k_row_stride;
  // Fused KV append (vl_rope_kv_append); v == nullptr disables it.
  const void* v;
  void* k_cache;
  void* v_cache;
  const int64_t* slot_mapping;
  int64_t num_slots;
  int32_t* status;
};
cudaError_t launch_rope(const RopeArgs& args, int dtype, cudaStream_t stream);

cudaError_t launch_embed_gather(const int64_t* ids, int64_t batch, int64_t seq,
                                int64_t ids_batch_stride, const int32_t* row_map,
                                const void* table, int64_t vocab, int64_t row_bytes,
                                const void* audio, int64_t audio_token_id, int64_t audio_rows,
                                int64_t audio_batch_stride_bytes, void* out, int32_t* status,
                                cudaStream_t stream);

cudaError_t launch_kv_append(const void* k, const void* v, void* k_cache, void* v_cache,
                             const int64_t* slot_mapping, int64_t tokens, int64_t row_bytes,
                             int64_t k_row_stride_bytes, int64_t v_row_stride_bytes,
                             int64_t num_slots, int32_t* status, cudaStream_t stream);

// Decode-step attention (vl_attn.cu).
struct DecodeAttnArgs {
  const void* q;            // [tokens][n_q_heads * head_dim], row stride q_row_stride
  const void* k;            // new rows [tokens][n_kv_heads * head_dim] or nullptr
  const void* v;
  void* k_cache;            // [num_slots][cache_row_stride]
  void* v_cache;
  const int32_t* positions; // [tokens]
  const int64_t* seq_start; // [tokens] slot of position 0
  void* out;                // [tokens][n_q_heads * head_dim], row stride out_row_stride
  int64_t tokens;
  int n_q_heads;
  int n_kv_heads;
  int head_dim;
  int rotary_dim;           // 0: no RoPE
  double rope_base;
  float scale;
  int64_t q_row_stride;
  int64_t kv_row_stride;
  int64_t cache_row_stride;
  int64_t out_row_stride;
  int64_t max_seq_len;
  int64_t num_slots;
  int32_t* status;
  // filled by launch_decode_attention
  int split;
  int max_splits;
  int* counters;
  float* o_part;
  float2* ml_part;
};
bool decode_attention_supported(int head_dim, int group);
int64_t decode_attention_split(int64_t tokens, int n_kv_heads, int64_t max_seq_len);
size_t decode_attention_workspace_bytes(int64_t tokens, int n_q_heads, int n_kv_heads,
                                        int head_dim, int64_t max_seq_len);
// pdl: launch as a programmatic dependent of the stream's previous kernel
// (VL_LAUNCH_PDL of the C ABI).
cudaError_t launch_decode_attention(DecodeAttnArgs args, int dtype, void* workspace, bool pdl,
                                    cudaStream_t stream);

// Decode-step linear layers (vl_linear.cu).
struct LinearArgs {
  const void* x;             // [rows][x_row_stride], k used
  int64_t x_row_stride;
  const void* norm_weight;   // [k] RMSNorm weight, or nullptr
  const float* ssq_in;       // [ssq_in_parts][rows] partial sums of squares of x's rows
  int ssq_in_parts;
  float eps;
  const void* w;             // [n][k]
  int64_t n;
  int64_t k;
  void* y;                   // [rows][y_row_stride]
  int64_t y_row_stride;
  float* ssq_out;            // RESIDUAL: [n / 16][rows], or nullptr
  int64_t rows;
  int epilogue;              // VL_LINEAR_STORE / _SWIGLU / _RESIDUAL
};
cudaError_t launch_decode_linear(const LinearArgs& args, int dtype, bool pdl, bool tcgen05,
                                 cudaStream_t stream);
// The tensor-core (tcgen05 / TMA / TMEM) form of the same op (vl_linear_tc.cu),
// used by launch_decode_linear on request for the shapes it supports.
bool decode_linear_tc_supported(const LinearArgs& args, int dtype);
cudaError_t launch_decode_linear_tc(const LinearArgs& args, int dtype, bool pdl,
                                    cudaStream_t stream);
// Bounded-wait expiries of the tensor-core kernel on the current device.
cudaError_t read_linear_timeouts(unsigned int* count);

// Decode-step tail: argmax with the EOS freeze (vl_argmax.cu).
struct ArgmaxArgs {
  const void* logits;            // [rows][row_stride], vocab used
  int64_t rows;
  int64_t vocab;
  int64_t row_stride;
  const int32_t* row_chunk;      // [rows] chunk of each row, or nullptr (row = chunk)
  int64_t chunks;
  uint8_t* finished;             // [chunks] or nullptr (plain argmax)
  int64_t* current_ids;          // [chunks]
  int64_t* out_ids;              // [out_rows][out_stride] or nullptr
  int64_t out_rows;
  int64_t out_stride;
  const int32_t* positions;      // [chunks]
  const int64_t* prompt_length;  // device scalar
  int64_t eos[8];
  int n_eos;
  int64_t freeze_id;
  int32_t* status;
};
cudaError_t launch_argmax_eos(const ArgmaxArgs& args, int dtype, cudaStream_t stream);

// The row ops of a decode step in one launch (vl_decode_rows.cu): residual
// add + RMSNorm of `rows` hidden rows, and RoPE of q/k at each token's
// position with the append of the rotated k and of v to the KV cache.
struct DecodeRowsArgs {
  void* residual;            // [rows][cols]
  const void* delta;         // [rows][cols] or nullptr
  const void* weight;        // [cols]
  void* out;                 // [rows][cols]
  int64_t rows;
  int cols;
  float eps;
  void* q;                   // [tokens][q_row_stride], n_q_heads * head_dim used
  void* k;                   // [tokens][kv_row_stride], n_kv_heads * head_dim used
  const void* v;             // [tokens][kv_row_stride]
  void* k_cache;             // [num_slots][n_kv_heads * head_dim]
  void* v_cache;
  const int32_t* positions;  // [tokens]
  const int64_t* slot_mapping;  // [tokens]
  int64_t tokens;
  int n_q_heads;
  int n_kv_heads;
  int head_dim;
  int rotary_dim;
  double rope_base;
  int64_t q_row_stride;
  int64_t kv_row_stride;
  int64_t num_slots;
  int32_t* status;
};
cudaError_t launch_decode_rows(const DecodeRowsArgs& args, int dtype, cudaStream_t stream);

// Peer-memory plumbing of the sharded pipeline (vl_peer.cu).
cudaError_t ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out);
cudaError_t ipc_open(const void* handle, void** base_out);
cudaError_t ipc_close(void* base);
cudaError_t copy_async(void* dst, const void* src, size_t bytes, cudaStream_t stream);

// Once-per-device set-up done ahead of the first op call (vl_init): the
// GELU tables (a private stream, one kernel, one stream synchronise) and the
// log-mel kernel's shared-memory limit and scratch address.
cudaError_t prepare_gelu();
cudaError_t prepare_logmel();

size_t logmel_workspace_bytes(int64_t chunks);
cudaError_t launch_logmel(const float* pcm, int64_t chunks, float* out, float* tile_max,
                          cudaStream_t stream);
// Same, with the library's fixed scratch array instead of a caller workspace.
cudaError_t launch_logmel_noalloc(const float* pcm, int64_t chunks, float* out,
                                  cudaStream_t stream);

}  // namespace vl
