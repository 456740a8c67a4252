/*
 * vl_api.h - C ABI of libvlasr.so, the sm_100a (B200) implementation of the
 * memory-bound layer ops of the GLM-ASR native engine:
 *
 *   log-mel frontend, residual-add + LayerNorm, residual-add + RMSNorm,
 *   exact-erf GELU (optionally with a fused bias add), SwiGLU, rotary
 *   embedding on Q/K in place, token-embedding gather and KV-cache append.
 *
 * Reference interfaces replaced (paths inside the VideoLingo-user project):
 *   native/asr/src/mel_frontend.h:26-32   compute_mel / compute_mel_batched
 *   native/asr/src/engine.cu:162-233      layer_norm / gelu / add_bias /
 *                                         residual_add / rope kernels
 *   native/asr/src/decoder.cu:60-134,307-351,460-514,636-695,789-814,
 *                            857-882,933-948
 *                                         embedding gathers, rmsnorm,
 *                                         silu_mul, RoPE and KV-append kernels
 * In the reference those ops are anonymous-namespace __global__ functions
 * launched by the engine's host code with compile-time shapes; this header is
 * the stable, shape-parameterised boundary a host (Python via ctypes, C, C++)
 * binds instead.
 *
 * Conventions shared by every entry point
 *   - Return value: VL_OK (0) on success, VL_ERR_EXEC (1) when a CUDA launch
 *     fails, VL_ERR_INVALID (2) for an invalid argument.  These mirror the
 *     reference CLI's exit codes (native/asr/src/main_m0.cu:6-7,696-703:
 *     0 ok, 1 ModelExecutionError, 2 ModelInputError).  vl_last_error()
 *     returns the message of the last failure on the calling thread.
 *   - Invalid arguments are detected on the host before any CUDA call, so a
 *     rejected call has no side effects and needs no GPU.
 *   - Buffers are caller-owned DEVICE pointers; ops never allocate device
 *     memory and run on the caller's stream (`stream` is a cudaStream_t
 *     passed as void*; NULL = the legacy default stream).  After an op's
 *     first call on a device they never synchronise either.  The first call
 *     does per-device set-up, cached for the life of the process: kernel
 *     attributes and occupancy queries for every op, and for vl_gelu_erf
 *     (f16/bf16) a one-time table build that launches one kernel on a
 *     private stream and waits for it.  vl_init() does all of it up front.
 *   - Apart from that per-device set-up (built once, read-only afterwards),
 *     ops keep no state between calls and are thread-safe; launches on one
 *     stream are ordered.  The exceptions that keep device state across
 *     calls (vl_decode_attention's split counters in the caller's
 *     workspace, vl_logmel_noalloc's fixed scratch array) say so below.
 *   - Float ops compute in fp32 and round once to the storage type (RNE);
 *     the rounding points are those of the reference kernels (documented per
 *     op below).  Index ops (gather, KV append) are bit-exact copies.
 *   - Index values that live in device memory (token ids, slots, audio
 *     placeholder counts) cannot be checked on the host.  The kernels never
 *     access memory out of bounds: an offending row is zero-filled (gather)
 *     or skipped (KV append) and, when `status` is non-NULL, a bit is OR-ed
 *     into *status (a device int32 the caller zeroes and later reads).
 */
#ifndef VL_API_H_
#define VL_API_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VL_EXPORT __attribute__((visibility("default")))
#else
#define VL_EXPORT
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define VL_OK 0
#define VL_ERR_EXEC 1
#define VL_ERR_INVALID 2

/* Element types of activation tensors. */
#define VL_F32 0
#define VL_F16 1
#define VL_BF16 2

/* Bits OR-ed into a device-side *status word by the index ops. */
#define VL_STATUS_BAD_ID 1      /* token id outside [0, vocab)              */
#define VL_STATUS_BAD_AUDIO 2   /* more audio placeholders than audio rows  */
#define VL_STATUS_BAD_SLOT 4    /* KV slot >= num_slots                      */

/* Whisper/GLM-ASR log-mel geometry (native/asr/src/mel_frontend.h:34-42). */
#define VL_MEL_BINS 128
#define VL_MEL_FFT 400
#define VL_MEL_HOP 160
#define VL_MEL_CHUNK_SAMPLES 480000
#define VL_MEL_FRAMES 3000

/* Library version (major*10000 + minor*100 + patch). */
VL_EXPORT int vl_version(void);

/* Message of the last failed call on this thread ("" when none). */
VL_EXPORT const char* vl_last_error(void);

/* Number of CUDA devices visible to the library (0 on a host without GPU). */
VL_EXPORT int vl_device_count(void);

/*
 * Once-per-device set-up, ahead of the first op call on `device` (the
 * caller's current device is restored on return).  Optional: each op does
 * its own part of it on its first call on a device, which is what this call
 * moves out of the hot path and out of any stream capture.  What it does:
 *   - builds the GELU lookup tables that vl_gelu_erf uses for f16/bf16
 *     inputs of 1M elements or more: creates a private stream, launches one
 *     kernel on it, synchronises that stream and destroys it (the only op
 *     set-up that launches work or waits); the tables live in a fixed
 *     256 KB array inside the library, so nothing is allocated;
 *   - raises the shared-memory limit of the log-mel kernel
 *     (cudaFuncSetAttribute) and looks up the address of
 *     vl_logmel_noalloc's fixed scratch array (cudaGetSymbolAddress).
 * The other ops' first-call set-up only sets kernel attributes and queries
 * occupancy (host calls that neither launch, allocate nor wait).
 * Without vl_init, the first vl_gelu_erf call on a device made while its
 * stream is being captured cannot build the tables; that call and the graph
 * captured with it evaluate erff directly, with bit-identical results but
 * at lower speed, and the tables are built by the first later call that is
 * not captured.  Returns VL_ERR_INVALID for a bad device index or when
 * called during a capture of the legacy stream.
 */
VL_EXPORT int vl_init(int device);

/* ------------------------------------------------------------------------ */
/* Peer memory for the chunk-sharded pipeline                                */
/* ------------------------------------------------------------------------ */
/*
 * The multi-GPU run of the layer chain shards chunks over one process per
 * GPU and then gives every rank all ranks' encoder-norm outputs.  These four
 * calls let a host do that exchange with the GPUs' copy engines over
 * NVLink - no kernel, so the shard transfers take no SM time from the layer
 * kernels that run beside them.  They have no counterpart in the reference,
 * whose engine runs on one GPU (native/asr/src/engine.cu:1166-1616).
 *
 * vl_ipc_export: CUDA IPC handle (VL_IPC_HANDLE_BYTES opaque bytes) of the
 *   device allocation that contains `ptr`, and ptr's byte offset in it.
 * vl_ipc_open: maps another process's exported allocation into this one
 *   (on the current device; peer access is enabled on first use) and
 *   returns its base address; add the exported offset.
 * vl_ipc_close: unmaps an address vl_ipc_open returned.
 * vl_copy_async: cudaMemcpyAsync device-to-device of `bytes` on `stream`;
 *   src or dst may be a mapped peer address.  They must not overlap.
 * The host orders the copies against the producer's kernels (e.g. a
 * collective barrier on the copying stream); these calls do no ordering of
 * their own.
 */
#define VL_IPC_HANDLE_BYTES 64
VL_EXPORT int vl_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out);
VL_EXPORT int vl_ipc_open(const void* handle, void** base_out);
VL_EXPORT int vl_ipc_close(void* base);
VL_EXPORT int vl_copy_async(void* dst, const void* src, size_t bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Log-mel frontend                                                          */
/* ------------------------------------------------------------------------ */

/* Workspace bytes vl_logmel needs for `chunks` chunks (per-tile maxima). */
VL_EXPORT size_t vl_logmel_workspace_bytes(int64_t chunks);

/*
 * Whisper log-mel features of `chunks` independent 30 s chunks.
 * Replaces compute_mel_batched (native/asr/src/mel_frontend.cu:209-291;
 * declared native/asr/src/mel_frontend.h:30-32).
 *
 *   pcm  [chunks][480000] f32, 16 kHz mono, already zero-padded per chunk
 *        (the reference throws unless size == chunks*480000).
 *   out  [chunks][128][3000] f32.
 *
 * Per chunk: reflect pad 200, periodic Hann, |rfft_400|^2 on hop-160 frames,
 * 128-bin Slaney mel filterbank (0-8000 Hz), log10(max(x,1e-10)) over
 * frames 0..2999 (the 3001st frame is dropped), clamp to (chunk max - 8),
 * then (x+4)/4.  pcm and out must be 16-byte aligned; workspace must hold
 * vl_logmel_workspace_bytes(chunks) bytes (16-byte aligned) and needs no
 * initialisation.  `out` must not overlap `pcm`.
 */
VL_EXPORT int vl_logmel(const float* pcm, int64_t chunks, float* out, void* workspace,
              size_t workspace_bytes, void* stream);

/* Largest chunk count vl_logmel_noalloc accepts in one call. */
#define VL_LOGMEL_NOALLOC_MAX_CHUNKS 1024

/*
 * vl_logmel for callers that cannot allocate device memory.  This entry
 * point has no counterpart in the reference.
 *
 * Some hosts cannot call cudaMalloc or hand this library a scratch buffer:
 * a process whose GPU memory is all reserved up front by a fixed budget or
 * arena (a serving process, or an engine sharing the GPU under a VRAM cap as
 * the reference's native engine does), a plugin running inside another
 * framework's callback where allocating is not allowed, or a latency-
 * critical path that must never wait on the allocator.  Such callers pass
 * only pcm and out (the same layouts as vl_logmel); the per-tile maxima the
 * kernel needs live in one fixed array inside the library, sized for
 * VL_LOGMEL_NOALLOC_MAX_CHUNKS chunks (512,000 bytes, held on every GPU that
 * loads the library until the process exits).  chunks above that limit
 * return VL_ERR_INVALID.  Nothing is allocated, freed or synchronised.
 *
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and raises the kernel's shared-memory limit; make
 * that first call before any stream capture.  Every call shares the one
 * array and it keeps whatever the previous call left there; nothing in it
 * has to start at zero because each call writes every slot before reading
 * it.  Calls that can overlap on the GPU (several streams, or several host
 * threads on one device) race on the array: serialise them.
 */
VL_EXPORT int vl_logmel_noalloc(const float* pcm, int64_t chunks, float* out, void* stream);

/* ------------------------------------------------------------------------ */
/* Norms                                                                     */
/* ------------------------------------------------------------------------ */

/*
 * Residual add + LayerNorm over the last dimension (rows x cols, row-major,
 * contiguous).  Replaces residual_add_kernel -> cudaMemcpy -> layer_norm_kernel
 * (native/asr/src/engine.cu:207-212, :162-192, sequence :1544-1552).
 *
 *   delta != NULL:  h = round(residual + delta); residual := h;
 *                   out = round((h - mean) * rsqrt(var + eps) * gamma + beta)
 *   delta == NULL:  out = LayerNorm(residual); residual is only read
 *                   (out == residual gives the reference's in-place LN).
 * mean = sum(h)/cols and var = sum(h^2)/cols - mean^2 in fp32, computed from
 * the ROUNDED h exactly as the reference normalises the stored half value;
 * var is clamped at 0 (the reference would produce NaN on a degenerate row).
 * `out` may alias `delta`; with delta != NULL it must not alias `residual`.
 * gamma/beta are [cols] of the same dtype; beta may be NULL (no bias).
 */
VL_EXPORT int vl_add_layernorm(void* residual, const void* delta, const void* gamma,
                     const void* beta, void* out, int64_t rows, int64_t cols,
                     float eps, int dtype, void* stream);

/*
 * Residual add + RMSNorm.  Replaces residual_add_kernel -> cudaMemcpy ->
 * rmsnorm_kernel (native/asr/src/decoder.cu:933-938, :81-101, sequence
 * :1591-1597 and :1727-1733).
 *   h as above; out = round((h * rsqrt(sum(h^2)/cols + eps)) * weight).
 * Same aliasing rules as vl_add_layernorm.
 */
VL_EXPORT int vl_add_rmsnorm(void* residual, const void* delta, const void* weight,
                   void* out, int64_t rows, int64_t cols, float eps, int dtype,
                   void* stream);

/* ------------------------------------------------------------------------ */
/* Activations                                                               */
/* ------------------------------------------------------------------------ */

/*
 * Exact-erf GELU, optionally after a bias add.  Replaces add_bias_kernel +
 * gelu_kernel (native/asr/src/engine.cu:200-205, :194-198, gelu :110-112).
 *   bias == NULL:  out = round(0.5*x*(1+erf(x/sqrt(2))))
 *   bias != NULL:  t = round(x + bias[col]); out = round(gelu(t))
 *                  (the reference stores the biased value before GELU).
 * in/out are rows x cols contiguous; out may equal in (in place).
 */
VL_EXPORT int vl_gelu_erf(const void* in, const void* bias, void* out, int64_t rows,
                int64_t cols, int dtype, void* stream);

/*
 * SwiGLU: out = round(g / (1 + exp(-g)) * u) with g = gate, u = up (the
 * division by a fast reciprocal, within 2 ulp of IEEE division in fp32).
 * Replaces silu_mul_kernel (native/asr/src/decoder.cu:103-109), which writes
 * into the gate buffer (out == gate is allowed).  Row strides are in
 * elements, so a packed [rows, 2*cols] gate|up buffer is expressed as
 * gate = buf, up = buf + cols, gate_stride = up_stride = 2*cols.
 */
VL_EXPORT int vl_swiglu(const void* gate, const void* up, void* out, int64_t rows,
              int64_t cols, int64_t gate_stride, int64_t up_stride,
              int64_t out_stride, int dtype, void* stream);

/* ------------------------------------------------------------------------ */
/* Rotary embedding                                                          */
/* ------------------------------------------------------------------------ */

/*
 * Rotate-half RoPE applied in place to q [tokens][n_q_heads][head_dim] and
 * k [tokens][n_k_heads][head_dim] (row strides in elements; k may be NULL
 * with n_k_heads == 0).  For every head the first `rotary_dim` dims rotate
 * in pairs (d, d + rotary_dim/2):
 *   x1' = x1*cos - x2*sin,  x2' = x2*cos + x1*sin   (fp32, one rounding)
 * with angle = pos * base^(-2d/rotary_dim) formed in fp64 as the reference's
 * host tables are (native/asr/src/engine.cu:892-905,
 * native/asr/src/decoder.cu:950-961), reduced modulo 2*pi in fp64 and
 * evaluated with fp32 sincosf (within 3e-7 of the tables' fp32 values).
 * Dims >= rotary_dim are untouched.
 *
 * Position of row r:
 *   positions == NULL:  pos_offset + (seq_len > 0 ? r % seq_len : r)
 *   positions != NULL:  pos_offset + positions[(row_map ? row_map[r] : r) * positions_stride]
 * This covers every reference variant: rope_kernel (row % 1500, rotary 32 of
 * 64), rope_rows_kernel (row % L), rope_full_kernel / rope_at_position_kernel
 * (seq_len = 1, pos_offset = position), rope_at_position_dev_kernel
 * (positions_stride = 0), rope_at_position_map_kernel (row_map = active ids)
 * (engine.cu:217-233; decoder.cu:113-134,307-333,471-498,670-695,789-814).
 */
VL_EXPORT int vl_rope_inplace(void* q, void* k, const int32_t* positions,
                    const int32_t* row_map, int64_t positions_stride,
                    int64_t pos_offset, int64_t tokens, int64_t seq_len,
                    int n_q_heads, int n_k_heads, int head_dim, int rotary_dim,
                    double base, int64_t q_row_stride, int64_t k_row_stride,
                    int dtype, void* stream);

/* ------------------------------------------------------------------------ */
/* Index ops (bit-exact)                                                     */
/* ------------------------------------------------------------------------ */

/*
 * Token-embedding gather with audio-placeholder substitution.
 * Output row (b, s), b < batch, s < seq, is out[(b*seq + s)*dim ..]:
 *   src = row_map ? row_map[b] : b
 *   id  = ids[src*ids_batch_stride + s]
 *   id == audio_token_id (>= 0):  audio[src*audio_batch_stride + j*dim ..]
 *        with j = number of placeholders in ids[src][0..s)
 *   otherwise:                    table[id*dim ..]
 * Replaces gather_inputs_kernel, gather_batch_kernel (ids shared by every
 * chunk: ids_batch_stride = 0), gather_ids_batched_kernel (seq = 1) and
 * gather_ids_mapped_kernel (row_map = active ids)
 * (native/asr/src/decoder.cu:60-78, :636-654, :659-667, :460-469).
 * audio_token_id < 0 disables substitution (audio may then be NULL).
 * Bad ids (outside [0,vocab)) and placeholders beyond audio_rows give a
 * zero row and set VL_STATUS_BAD_ID / VL_STATUS_BAD_AUDIO in *status.
 * dtype only fixes the element size; rows are copied bit for bit.
 */
VL_EXPORT int vl_embed_gather(const int64_t* ids, int64_t batch, int64_t seq,
                    int64_t ids_batch_stride, const int32_t* row_map,
                    const void* table, int64_t vocab, int64_t dim,
                    const void* audio, int64_t audio_token_id,
                    int64_t audio_rows, int64_t audio_batch_stride, void* out,
                    int dtype, int32_t* status, void* stream);

/*
 * KV-cache append through a slot mapping.  Caches are
 * [num_slots][kv_heads*head_dim]; token t's K row (k + t*k_row_stride) and
 * V row go to slot slot_mapping[t].  slot < 0 skips the token (padding);
 * slot >= num_slots skips it and sets VL_STATUS_BAD_SLOT.
 * Replaces append_kv_kernel, append_kv_rows_kernel, append_kv_batched_kernel,
 * append_kv_batched_dev_kernel and append_kv_mapped_kernel
 * (native/asr/src/decoder.cu:940-948, :873-882, :857-870, :335-351,
 * :500-514): their position/chunk-stride addressing is the slot
 * chunk*(chunk_stride/row) + position.
 */
VL_EXPORT int vl_kv_append(const void* k, const void* v, void* k_cache, void* v_cache,
                 const int64_t* slot_mapping, int64_t tokens, int kv_heads,
                 int head_dim, int64_t k_row_stride, int64_t v_row_stride,
                 int64_t num_slots, int dtype, int32_t* status, void* stream);

/*
 * Decode-step fusion of RoPE and KV append (one launch instead of
 * rope_at_position_map_kernel + append_kv_mapped_kernel,
 * native/asr/src/decoder.cu:1710-1718): q is rotated in place; k is rotated,
 * written back in place AND stored to k_cache[slot]; v is copied to
 * v_cache[slot].  Row r uses position positions[r] and slot
 * slot_mapping[r] (slot < 0: q/k still rotate, nothing is cached).
 */
VL_EXPORT int vl_rope_kv_append(void* q, void* k, const void* v, void* k_cache,
                      void* v_cache, const int32_t* positions,
                      const int64_t* slot_mapping, int64_t tokens,
                      int n_q_heads, int n_k_heads, int head_dim,
                      int rotary_dim, double base, int64_t num_slots,
                      int dtype, int32_t* status, void* stream);

/*
 * The row ops of a decode step in ONE launch: residual add + RMSNorm of the
 * hidden rows (as vl_add_rmsnorm), and RoPE of q/k at each token's position
 * with the KV append (as vl_rope_kv_append).  Replaces the five launches the
 * reference's decode step spends on them (native/asr/src/decoder.cu:1702-1733:
 * rope_at_position_map_kernel :471-498, append_kv_mapped_kernel :500-514,
 * residual_add_kernel :933-938 + cudaMemcpyAsync + rmsnorm_kernel :81-101).
 *
 * Norm part (rows may be 0): residual/delta/out [rows][cols], weight [cols];
 *   h = round(residual + delta) (delta NULL: h = residual); residual := h;
 *   out = round((h * rsqrt(sum(h^2)/cols + eps)) * weight).
 * Token part (tokens may be 0): q [tokens][q_row_stride] (n_q_heads *
 *   head_dim used), k and v [tokens][kv_row_stride] (n_kv_heads * head_dim
 *   used), caches [num_slots][n_kv_heads * head_dim]; q and k are rotated in
 *   place at positions[t] (rotate-half on the first rotary_dim dims of every
 *   head, base `base`), the rotated k row and the v row are stored to slot
 *   slot_mapping[t] (slot < 0: not cached; slot >= num_slots: not cached and
 *   VL_STATUS_BAD_SLOT set in *status).
 * The two parts run side by side, so the norm rows must not overlap q, k or
 * v (checked).  Each part computes exactly what its own entry point
 * computes: the same rounding points, the same cos/sin.  Requirements:
 * 16-byte aligned pointers; cols, head_dim, rotary_dim / 2 and the row
 * strides multiples of the 16-byte vector (8 for f16/bf16, 4 for f32);
 * cols at most 1024 vectors.  No allocation, no synchronisation.
 */
VL_EXPORT int vl_decode_rows(void* residual, const void* delta, const void* weight, void* out,
                             int64_t rows, int64_t cols, float eps, void* q, void* k,
                             const void* v, void* k_cache, void* v_cache,
                             const int32_t* positions, const int64_t* slot_mapping,
                             int64_t tokens, int n_q_heads, int n_kv_heads, int head_dim,
                             int rotary_dim, double base, int64_t q_row_stride,
                             int64_t kv_row_stride, int64_t num_slots, int dtype,
                             int32_t* status, void* stream);

/*
 * Launch flags of the decode-step entry points (vl_decode_attention,
 * vl_decode_linear).
 *
 * VL_LAUNCH_PDL  launch as a programmatic dependent of the kernel before it
 *                in the stream: the new kernel's blocks may start while that
 *                kernel finishes and prefetch inputs it cannot be writing,
 *                and they wait for its completion (and its writes) before
 *                reading anything else.  The caller guarantees that the
 *                kernel before it in the stream writes none of:
 *                  vl_decode_linear     w, norm_weight;
 *                  vl_decode_attention  positions, seq_start and, with k / v
 *                                       given, the cache rows before each
 *                                       token's position.
 *                Results are identical with and without the flag.  In a
 *                chain of such launches (a decode step captured in a CUDA
 *                graph) each kernel's weight or cache stream overlaps the
 *                tail of the kernel before it.
 */
#define VL_LAUNCH_PDL 1

/*
 * Decode-step attention: one query token per sequence against its KV cache,
 * grouped-query heads (n_q_heads / n_kv_heads query heads share a kv head),
 * optionally fused with the RoPE of q and k at the token's position and the
 * append of the new k / v rows.  One launch replaces the reference's
 * rope_at_position_map_kernel + append_kv_mapped_kernel +
 * attention_step_mapped_kernel (native/asr/src/decoder.cu:471-572, launched
 * at :1710-1722), without its 1024-position limit.
 *
 * Token t (query row q + t*q_row_stride, [n_q_heads][head_dim]) sits at
 * position p = positions[t] of a sequence whose cache rows are the slots
 * seq_start[t] + 0 .. seq_start[t] + p of k_cache / v_cache
 * ([num_slots][cache_row_stride] elements, kv head h at h*head_dim).
 * out row t = softmax(scale * q . K^T) V over positions 0..p (scale 0 means
 * 1/sqrt(head_dim)), per query head, fp32 arithmetic, rounded once.
 *
 * With k and v given (rows k/v + t*kv_row_stride, [n_kv_heads][head_dim]),
 * q and k are first rotated at p (rotate-half over the first rotary_dim
 * dims, base rope_base; rotary_dim 0 = no RoPE), and the rotated k and the v
 * row are stored to slot seq_start[t] + p; the inputs are not modified.
 * With k = v = NULL the cache must already hold position p.
 *
 * A token with p outside [0, max_seq_len) or a slot outside [0, num_slots)
 * gets zero output and sets VL_STATUS_BAD_SLOT in *status (if given).
 * Supported: f16 / bf16; head_dim 64 or 128 with 1, 2, 4 or 8 query heads
 * per kv head; max_seq_len <= VL_DECODE_MAX_SEQ_LEN.  One call must not
 * read a slot that another token of the same call appends (one token per
 * sequence per call, as in a decode step).
 * workspace: vl_decode_attention_workspace_bytes(...) bytes, zero-filled
 * before its first use; every call leaves it zero-filled again (the split
 * counters reset themselves), so one workspace serves calls in stream order.
 * flags: 0 or VL_LAUNCH_PDL.
 */
#define VL_DECODE_MAX_SEQ_LEN 262144

VL_EXPORT size_t vl_decode_attention_workspace_bytes(int64_t tokens, int n_q_heads,
                                                     int n_kv_heads, int head_dim,
                                                     int64_t max_seq_len);

VL_EXPORT int vl_decode_attention(const void* q, const void* k, const void* v,
                                  void* k_cache, void* v_cache, const int32_t* positions,
                                  const int64_t* seq_start, int64_t tokens, int n_q_heads,
                                  int n_kv_heads, int head_dim, int rotary_dim,
                                  double rope_base, float scale, int64_t q_row_stride,
                                  int64_t kv_row_stride, int64_t cache_row_stride,
                                  int64_t max_seq_len, int64_t num_slots, void* out,
                                  int64_t out_row_stride, int dtype, void* workspace,
                                  size_t workspace_bytes, int32_t* status, int flags,
                                  void* stream);

/*
 * Decode-step linear layer: y = x W^T for rows <= 64 token rows (W [n][k]
 * row-major, as nn.Linear and the checkpoint store it), fp32 accumulation,
 * one rounding to the storage type, with the neighbouring memory-bound steps
 * of the reference's decode layer fused in (native/asr/src/decoder.cu:
 * rmsnorm_kernel :81-101, the `gemm` projections :1002-1033,
 * residual_add_kernel :933-938, silu_mul_kernel :103-109):
 *
 * prologue  norm_weight NULL: A = x.
 *           norm_weight given: A = round(x * rsqrtf(S/k + eps) * w_norm[k])
 *           with S = sum over p < ssq_in_parts of ssq_in[p*rows + row] (the
 *           partial sums written by a RESIDUAL call, summed in order).
 * epilogue  VL_LINEAR_STORE    y[row][j] = round(acc), j < n
 *           VL_LINEAR_SWIGLU   W = [gate rows n/2; up rows n/2];
 *                              y[row][j] = round(silu(round(acc_gate)) *
 *                              round(acc_up)), j < n/2
 *           VL_LINEAR_RESIDUAL y is the residual stream, updated in place:
 *                              y[row][j] = round(y + round(acc)); if
 *                              ssq_out, ssq_out[(j/16)*rows + row] = sum of
 *                              the squares of the 16 new values j..j+15.
 * Requires k % 512 == 0, n % 16 == 0 (n % 32 for SWIGLU), x / w / y and
 * norm_weight 16-byte aligned with row strides that are multiples of 8 elements, x not
 * overlapping y.  f16 / bf16.  No allocation, no synchronisation.
 * flags: VL_LAUNCH_PDL and / or VL_LINEAR_TCGEN05.
 * Kernels: by default a tensor-core kernel of the previous generation
 * (mma.sync), which spreads a few-row weight stream over many SMs.  With
 * VL_LINEAR_TCGEN05, when the output columns (n, or n/2 for SWIGLU) are a
 * multiple of 128, the 5th-generation tensor cores compute it instead
 * (tcgen05.mma with the accumulator in tensor memory, weights streamed by
 * TMA, K split over a thread-block cluster whose partial sums meet in
 * distributed shared memory); other shapes ignore the flag.  On a B200 the
 * tcgen05 kernel measured slower per launch than the default at every row
 * count (its split-K clusters reach at most 15 x 8 CTAs, and each CTA's
 * prologue, reduction and epilogue are serial latencies), so it is opt-in.
 * Both keep the rounding points above; their fp32 summation orders differ,
 * each is deterministic.
 */
#define VL_LINEAR_TCGEN05 2
#define VL_LINEAR_STORE 0
#define VL_LINEAR_SWIGLU 1
#define VL_LINEAR_RESIDUAL 2
#define VL_LINEAR_MAX_ROWS 64

VL_EXPORT int vl_decode_linear(const void* x, int64_t x_row_stride, const void* norm_weight,
                               const float* ssq_in, int ssq_in_parts, float eps,
                               const void* w, int64_t n, int64_t k, void* y,
                               int64_t y_row_stride, float* ssq_out, int64_t rows,
                               int epilogue, int dtype, int flags, void* stream);

/*
 * Number of waits of the tensor-core vl_decode_linear kernel on the current
 * device that gave up (each is bounded to a few seconds; on expiry the kernel
 * writes NaN for the outputs of the tile it could not finish, releases its
 * resources and returns instead of hanging).  0 in normal operation.  Reads
 * a device counter with a synchronous copy.
 */
VL_EXPORT int vl_decode_linear_timeouts(uint32_t* count);

/*
 * Decode-step tail: the greedy next token of each row with the EOS freeze,
 * replacing the reference's argmax_mapped_kernel (native/asr/src/
 * decoder.cu:573-621, launched at :1749) and, with finished = NULL, its
 * argmax_rows_kernel (:755-782).
 *
 * Row r of logits ([rows][row_stride], vocab used; f32 / f16 / bf16) belongs
 * to chunk c = row_chunk[r] (row_chunk NULL: c = r; c must be in
 * [0, chunks)).  The id is the largest logit above -1e30 (NaN never wins);
 * ties go to the smallest j mod 256, then the smallest j - the order of the
 * reference's 256-thread reduction.  A row with no logit above -1e30 gives
 * freeze_id (finished given) or 0.
 * finished given ([chunks] bytes, 0/1): a finished chunk gives freeze_id
 * without a scan and changes nothing else; otherwise, with out_ids, the id
 * is stored at out_ids[(positions[c] - *prompt_length + 1) * out_stride + c]
 * (an output row outside [0, out_rows) sets VL_STATUS_BAD_SLOT in *status
 * instead), and an id in eos_ids[0..n_eos) marks the chunk finished.
 * current_ids[c] = the id in every case.
 * eos_ids is a HOST array (n_eos <= 8); prompt_length is a device scalar so
 * a captured CUDA graph serves every prompt length.  With finished given,
 * row_chunk entries must be distinct: two rows of one chunk would both write
 * finished[c], current_ids[c] and the chunk's out_ids slot with no order
 * between them, and which id lands there is unspecified (row_chunk lives in
 * device memory, so this is not checked).  Requires vocab % 8 == 0,
 * vocab <= 2^24, row_stride % 8 == 0, 16-byte aligned logits.  No
 * allocation, no synchronisation.
 */
VL_EXPORT int vl_argmax_eos(const void* logits, int64_t rows, int64_t vocab, int64_t row_stride,
                            const int32_t* row_chunk, int64_t chunks, uint8_t* finished,
                            int64_t* current_ids, int64_t* out_ids, int64_t out_rows,
                            int64_t out_stride, const int32_t* positions,
                            const int64_t* prompt_length, const int64_t* eos_ids, int n_eos,
                            int64_t freeze_id, int dtype, int32_t* status, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* VL_API_H_ */
