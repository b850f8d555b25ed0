/*
 * vtx_fa.h — C ABI of the B200 (sm_100a) attention node for voxtral.cpp.
 *
 * This library replaces exactly one ggml graph node: GGML_OP_FLASH_ATTN_EXT,
 * created by
 *     ggml_flash_attn_ext(ctx, q, k, v, mask, scale, max_bias, logit_softcap)
 * at the two call sites of voxtral.cpp:
 *     src/voxtral.cpp:1611  encoder self-attention (offline: mask = NULL;
 *                           realtime: F16 sliding-causal mask, window 750)
 *     src/voxtral.cpp:1802  decoder GQA attention over the KV cache
 *                           (prefill: F16 causal mask; decode step: NULL)
 * The arithmetic it replaces lives in ggml (fetched by CMake FetchContent at
 * ggml-org/ggml@5cecdad, reference CMakeLists.txt:33-41): the CPU kernel
 * ggml_compute_forward_flash_attn_ext_f16 and the ggml-cuda fattn-* kernels.
 *
 * Tensor descriptors mirror ggml_tensor's geometry: ne[0] is the fastest
 * dimension, nb[i] are byte strides, any permuted view is accepted as is
 * (the call sites pass ggml_permute views, src/voxtral.cpp:1601-1605 and
 * :1783-1794).  Type ids are ggml's (GGML_TYPE_F32 = 0, F16 = 1, Q8_0 = 8).
 *
 * Operator contract (ggml semantics):
 *   q    [Dk, n_q,  Hq,  B]   F32 or F16
 *   k    [Dk, n_kv, Hkv, B]   F32, F16 or Q8_0 (Hq % Hkv == 0 -> GQA broadcast)
 *   v    [Dv, n_kv, Hkv, B]   same type as k, rows are tokens (not transposed)
 *   mask [n_kv, >= n_q, 1|Hq, 1|B]  F16, additive, -inf = skip; may be NULL
 *   dst  [Dv, Hq, n_q, B]     F32, written by the call (ggml permutes the
 *                             result so one token's heads are contiguous);
 *                             F16 is accepted where the tcgen05 kernel runs
 *                             (n_q * Hq/Hkv >= 64, no mask tensor, no softcap):
 *                             the F32 result rounded to nearest even, as ggml
 *                             rounds the activations of the F16 projection
 *                             weight that consumes it (VTX_ERR_TYPE elsewhere)
 *   O[b,i,h,:] = sum_j softmax_j(scale*q.k_j [softcap] + slope_h*mask[i,j]) v_j
 *
 * All device pointers belong to the caller.  No entry point allocates device
 * memory, synchronises the host or aborts: errors are returned as negative
 * codes (vtx_strerror).  Scratch memory for split-KV partials and dtype
 * conversion is passed in as `workspace`; its size comes from the matching
 * *_workspace() query.  `stream` is a cudaStream_t (NULL = legacy stream).
 */
#ifndef VTX_FA_H
#define VTX_FA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define VTX_API __attribute__((visibility("default")))
#else
#define VTX_API
#endif

#define VTX_FA_ABI_VERSION 2

/* ggml type ids (ggml/include/ggml.h enum ggml_type) */
enum vtx_type {
    VTX_TYPE_F32  = 0,
    VTX_TYPE_F16  = 1,
    VTX_TYPE_Q8_0 = 8
};

/* Q8_0 block, identical to ggml's block_q8_0: 32 values = d * qs[i]. */
#define VTX_QK8_0 32
typedef struct {
    uint16_t d;              /* IEEE half scale */
    int8_t   qs[VTX_QK8_0];
} vtx_block_q8_0;            /* 34 bytes, 2-byte aligned */

/* Status codes. */
enum vtx_status {
    VTX_OK                  =  0,
    VTX_ERR_NULL            = -1,  /* a required pointer is NULL            */
    VTX_ERR_TYPE            = -2,  /* unsupported or mismatched dtype       */
    VTX_ERR_SHAPE           = -3,  /* inconsistent shapes                   */
    VTX_ERR_STRIDE          = -4,  /* stride/alignment not supported        */
    VTX_ERR_UNSUPPORTED     = -5,  /* head_dim / parameter not supported    */
    VTX_ERR_WORKSPACE       = -6,  /* workspace too small or misaligned     */
    VTX_ERR_CUDA            = -7,  /* a CUDA launch/runtime call failed     */
    VTX_ERR_NO_DEVICE       = -8,  /* no sm_100 device is current           */
    VTX_ERR_SCRATCH_LIMIT   = -9   /* problem needs more than the built-in
                                      no-alloc scratch buffer holds         */
};

/* Mirrors the geometry of a ggml_tensor (ggml.h struct ggml_tensor:
 * type, ne[GGML_MAX_DIMS], nb[GGML_MAX_DIMS], data). */
typedef struct vtx_tensor {
    int32_t type;            /* enum vtx_type */
    int32_t reserved;
    int64_t ne[4];           /* elements per dim, ne[0] fastest */
    size_t  nb[4];           /* byte strides; nb[0] = type size (34 for a Q8_0 block) */
    void   *data;            /* device pointer */
} vtx_tensor;

/* Operator parameters.  scale/max_bias/logit_softcap are ggml_flash_attn_ext's
 * op_params (ggml.h).  causal/window are an exact, tensor-free encoding of the
 * masks voxtral.cpp builds on the host:
 *   causal = 1 : query i may see key j iff j <= i + (n_kv - n_q)
 *                (src/voxtral.cpp:2103-2111 fill_causal_mask, n_kv == n_q)
 *   window = W : additionally j >= i + (n_kv - n_q) - (W - 1)
 *                (src/voxtral.cpp:2181-2188, VOXTRAL_ENC_WINDOW = 750)
 * An explicit mask tensor, if given, is applied on top. */
typedef struct vtx_fa_params {
    float   scale;
    float   max_bias;        /* ALiBi; 0 = off (both voxtral call sites) */
    float   logit_softcap;   /* 0 = off (both voxtral call sites) */
    int32_t causal;          /* 0 / 1 */
    int32_t window;          /* 0 = no window, else W > 0 (requires causal) */
    int32_t reserved[3];
} vtx_fa_params;

/* ggml_flash_attn_ext replacement (reference: ggml.h ggml_flash_attn_ext,
 * called at src/voxtral.cpp:1611 and src/voxtral.cpp:1802).
 * Returns VTX_OK or a negative vtx_status.  Asynchronous on `stream`. */
VTX_API int vtx_flash_attn_ext(const vtx_tensor *q, const vtx_tensor *k, const vtx_tensor *v,
                       const vtx_tensor *mask, const vtx_fa_params *params,
                       vtx_tensor *dst, void *workspace, size_t workspace_bytes,
                       void *stream);

/* Bytes of workspace vtx_flash_attn_ext needs for these operands (0 is a valid
 * answer).  Pure host computation; never touches the device.  Returns
 * (size_t)-1 if the operands are rejected. */
VTX_API size_t vtx_flash_attn_ext_workspace(const vtx_tensor *q, const vtx_tensor *k,
                                    const vtx_tensor *v, const vtx_fa_params *params);

/* Batched ragged decode: one new token per stream, each stream with its own
 * KV cache and length.  This is the decode node of src/voxtral.cpp:1802
 * (n_tokens = 1, mask = NULL, reached from run_decoder_step :2438 and
 * run_offline_step :2506) executed for many independent streams in one call.
 *   q        : device F32 [n_seq][n_head_q][head_dim], contiguous
 *   k_ptrs   : device array of n_seq device pointers, one per stream; the
 *              stream's keys are rows at k_ptrs[s] + t*kv_nb1 + g*kv_nb2
 *   v_ptrs   : same for values
 *   kv_len   : device int32 [n_seq], keys 0..kv_len[s]-1 are attended
 *   dst      : device F32 [n_seq][n_head_q][head_dim]
 *   fresh_row: optional device int32 [n_seq]: the one key row of each stream
 *              (index t, or -1 for none) that the kernel launched just before
 *              this call on the stream writes, together with q -- the KV
 *              append of the same decode step.  When given, the streaming
 *              decode kernels start copying the other rows while that kernel
 *              still runs (programmatic dependent launch) and wait for it only
 *              before reading q and the fresh row; kv_len, the pointer arrays
 *              and every other row must then be complete before that kernel.
 *              NULL: nothing is read before the preceding kernel completes.
 * max_kv_len bounds every kv_len[s] (host-known upper bound used for sizing). */
typedef struct vtx_decode_batch {
    int32_t n_seq;
    int32_t n_head_q;
    int32_t n_head_kv;
    int32_t head_dim;
    int32_t kv_type;         /* VTX_TYPE_F16, VTX_TYPE_Q8_0 or VTX_TYPE_F32 */
    int32_t max_kv_len;
    size_t  kv_nb1;          /* byte stride between tokens */
    size_t  kv_nb2;          /* byte stride between kv heads */
    const float        *q;
    const void * const *k_ptrs;
    const void * const *v_ptrs;
    const int32_t      *kv_len;
    float              *dst;
    float   scale;
    int32_t reserved;
    const int32_t      *fresh_row;   /* optional, see above (added in ABI version 2) */
} vtx_decode_batch;

VTX_API int vtx_flash_attn_decode_batched(const vtx_decode_batch *batch, void *workspace,
                                  size_t workspace_bytes, void *stream);

VTX_API size_t vtx_flash_attn_decode_batched_workspace(const vtx_decode_batch *batch);

/* Batched ragged decode for callers that cannot allocate device memory.
 *
 * No counterpart in the reference (ggml takes scratch from its backend pool).
 * Some callers have no way to obtain scratch: a plugin running inside a host
 * application that owns all device memory, code running under a strict
 * memory budget or a custom allocator that forbids extra cudaMalloc calls,
 * or a real-time decode loop where an allocation could block.  This entry
 * point computes exactly what vtx_flash_attn_decode_batched computes but
 * keeps its split-KV partials in a buffer compiled into the library
 * (VTX_NOALLOC_SCRATCH_BYTES per GPU, held by every GPU that loads the
 * library until the process exits).  The caller still passes inputs and
 * outputs; nothing is allocated.
 *
 * - Problems whose partials exceed VTX_NOALLOC_SCRATCH_BYTES are rejected
 *   with VTX_ERR_SCRATCH_LIMIT (vtx_flash_attn_decode_batched_workspace tells
 *   how many bytes a batch needs).
 * - The first call on a device looks up the buffer's device address once
 *   (cudaGetSymbolAddress); make that first call before any stream capture.
 * - Every call on a device shares the one buffer: calls that overlap on the
 *   GPU (different streams, or concurrent host threads) race on it.  Order
 *   them on one stream or synchronise between them. */
#define VTX_NOALLOC_SCRATCH_BYTES (32u << 20)
VTX_API int vtx_flash_attn_decode_batched_noalloc(const vtx_decode_batch *batch, void *stream);

/* Decoder KV-cache update: RoPE of Q and K, then the K/V cache write, in one
 * pass.  Replaces per decoder layer the ggml_rope_ext of Q and K (mode 0,
 * freq_base = dec_rope_theta, freq_scale 1, no YaRN) and the ggml_cpy of K
 * and V into the cache rows at kv_offset (src/voxtral.cpp:1744-1770), and the
 * shift-left memmove of the full cache window (src/voxtral.cpp:1237-1266).
 * - Token t of q / k / v is a row of heads x head_dim F32 values (heads
 *   contiguous, token stride *_nb1 bytes).  It is rotated with positions[t].
 * - K and V go to cache row slots[t] (a ring slot).  With
 *   slots[t] = (tokens so far + t) % window the cache holds the same rows as
 *   the reference after its shift-left, and decode attention does not depend
 *   on their order.  Prefill writes rows 0..n-1 in order.
 * - A cache row is ggml's [kv_dim] row: n_head_kv heads of head_dim values in
 *   the cache type (F32, F16, or Q8_0 blocks of 34 bytes).  Row r is at
 *   k_cache + r * cache_nb1, or at k_cache_ptrs[t] + r * cache_nb1 when the
 *   per-token base array is given (one cache per stream in batched decode).
 * - q_out receives the rotated Q (it may equal q); with q_out NULL only K
 *   and V are processed.
 * - Tokens of one call are written concurrently: two tokens of a call must
 *   not target the same cache row (a prefill longer than the window writes
 *   only its last `window` tokens).
 * positions, slots and the pointer arrays are device memory.  Asynchronous
 * on `stream`; no allocation. */
typedef struct {
    int32_t n_tokens, n_head_q, n_head_kv, head_dim;
    int32_t kv_type;                    /* VTX_TYPE_F32 / VTX_TYPE_F16 / VTX_TYPE_Q8_0 */
    float freq_base;                    /* RoPE base (voxtral.cpp: 1e6) */
    const float *q; size_t q_nb1;
    float *q_out; size_t q_out_nb1;
    const float *k; size_t k_nb1;
    const float *v; size_t v_nb1;
    const int32_t *positions;
    const int32_t *slots;
    void *k_cache, *v_cache;
    const void *const *k_cache_ptrs;    /* optional, [n_tokens] */
    const void *const *v_cache_ptrs;
    size_t cache_nb1;
    int32_t reserved[4];
} vtx_kv_append_args;
VTX_API int vtx_kv_append(const vtx_kv_append_args *args, void *stream);

/* Advances the device-side decode counters of n streams by one token, so a
 * captured decode step (vtx_kv_append + vtx_flash_attn_decode_batched per
 * layer, then this) can be replayed token after token with no host work:
 *   positions[i] += 1;  slots[i] = (slots[i] + 1) % window;
 *   kv_len[i] = min(kv_len[i] + 1, window).
 * Any of the three pointers may be NULL.  Replaces the host-side bookkeeping
 * of run_decoder_step (kv_used += 1 and the shift-left when full,
 * src/voxtral.cpp:2444-2471). */
VTX_API int vtx_decode_advance(int32_t *positions, int32_t *slots, int32_t *kv_len, int32_t n, int32_t window,
                               void *stream);

/* One decoder layer's attention for one new token per stream, in one launch:
 * what vtx_kv_append (RoPE of Q and K, K/V into ring row slots[s]) followed by
 * vtx_flash_attn_decode_batched computes, without the two dependent launches
 * and the split-merge launch between them.  Replaces per layer and decoded
 * token the ggml_rope_ext of Q and K and the ggml_cpy of K and V into the
 * cache at kv_offset (src/voxtral.cpp:1744-1770) and the decode
 * ggml_flash_attn_ext node (src/voxtral.cpp:1783-1805, n_tokens = 1,
 * mask = NULL), inside run_decoder_step (:2438-2473).
 * - q: [n_seq] rows of n_head_q * head_dim F32 (un-rotated; heads contiguous,
 *   token stride q_nb1 bytes); k, v: [n_seq] rows of n_head_kv * head_dim.
 * - The new K (rotated) and V are written to row slots[s] of the stream's
 *   caches k_cache_ptrs[s] / v_cache_ptrs[s] (rows cache_nb1 bytes apart,
 *   heads contiguous, F16 or Q8_0), then attention runs over rows
 *   [0, kv_len[s]) with kv_len[s] counting the new row (slots[s] < kv_len[s]).
 * - dst: [n_seq] rows of n_head_q * head_dim F32 (ggml's result for n_q = 1).
 * - head_dim 128, n_head_q / n_head_kv <= 8; Q8_0 needs an even n_head_kv.
 *   q, k, v, dst, the cache bases and every stride 16-byte aligned.
 * - early = 1: the cache rows other than slots[s], positions, kv_len, slots
 *   and the pointer arrays may be read while the kernel launched just before
 *   still runs (they must be complete before it); only q, k and v are waited
 *   for.  early = 0 reads nothing before that kernel completes.
 * - max_kv_len: a bound on every kv_len[s] for the calls made with these
 *   arguments.  It sizes the workspace and picks the key splits: when few are
 *   needed (short bounds) the splits of a (stream, KV head) run as one
 *   thread-block cluster and merge through distributed shared memory, else
 *   they merge through the workspace.  A longer kv_len[s] still gives the
 *   exact result, over the bound's splits.  The first call on a device
 *   queries the device's cluster capacity once (make it before a capture).
 * - workspace: vtx_decode_layer_workspace(args) bytes, 256-byte aligned:
 *   split partials and one arrival counter per stream and KV head.  Zero it
 *   once before the first call (cudaMemset); every completed call leaves it
 *   zeroed again.  After a call that reported a device error
 *   (vtx_read_device_error), zero it again.  Calls sharing a workspace must
 *   not overlap on the GPU.
 * Asynchronous on `stream`; no allocation, no host synchronisation. */
typedef struct {
    int32_t n_seq, n_head_q, n_head_kv, head_dim;
    int32_t kv_type;                    /* VTX_TYPE_F16 or VTX_TYPE_Q8_0 */
    int32_t max_kv_len;                 /* bound on every kv_len[s] (picks the key splits) */
    float freq_base;                    /* RoPE base (voxtral.cpp: 1e6) */
    float scale;                        /* softmax scale, 1/sqrt(head_dim) */
    const float *q; size_t q_nb1;
    const float *k; size_t k_nb1;
    const float *v; size_t v_nb1;
    const int32_t *positions;           /* RoPE position of each stream's new token */
    const int32_t *slots;               /* cache row the new token goes to */
    const int32_t *kv_len;              /* rows attended, the new one included */
    const void *const *k_cache_ptrs;    /* [n_seq] */
    const void *const *v_cache_ptrs;
    size_t cache_nb1;
    float *dst; size_t dst_nb1;
    int32_t early;
    int32_t reserved[3];
} vtx_decode_layer_args;
VTX_API size_t vtx_decode_layer_workspace(const vtx_decode_layer_args *args);
VTX_API int vtx_decode_layer(const vtx_decode_layer_args *args, void *workspace, size_t workspace_bytes,
                             void *stream);

/* ---- realtime encoder: chunk plan and device-side stitch ------------------ */

/* One chunk of the realtime model's chunked encoder run (run_encoder_chunked,
 * src/voxtral.cpp:2234-2335): chunks of 3000 mel frames every 1500 frames;
 * every chunk but the first skips the 750 encoder tokens that overlap the
 * previous one (:26-27).  Token counts follow mel_frames_to_enc_tokens
 * (:1300-1305: two causal convolutions, then a multiple of 4). */
typedef struct vtx_enc_chunk {
    int32_t mel_offset;       /* first mel frame of the chunk */
    int32_t mel_frames;       /* mel frames in the chunk, <= 3000 */
    int32_t n_tokens;         /* encoder tokens of the chunk (its attention length) */
    int32_t skip;             /* leading tokens already produced by the previous chunk */
    int32_t stride;           /* tokens the chunk adds to the stitched output */
    int32_t rope_offset;      /* absolute position of the chunk's token 0 */
    int32_t write_offset;     /* stitched-output row of the chunk's token `skip` */
    int32_t reserved;
} vtx_enc_chunk;

/* Plans the chunks of an utterance of total_mel_frames mel frames, exactly as
 * run_encoder_chunked walks them (including its early stop and its clamp to
 * compute_total_enc_tokens, :1308-1325).  Writes min(n, max_chunks) entries
 * (chunks may be NULL to query n) and returns n >= 0, or a negative
 * vtx_status.  *n_tokens_total (optional) gets the stitched token count (the
 * reference's output allocation); *n_tokens_used (optional) that count
 * trimmed to a multiple of the downsample factor (enc_seq_used, :2331-2332).
 * Host only: no CUDA call, no allocation. */
VTX_API int vtx_encoder_chunk_plan(int32_t total_mel_frames, vtx_enc_chunk *chunks, int32_t max_chunks,
                                   int32_t *n_tokens_total, int32_t *n_tokens_used);

/* Stitches per-chunk encoder rows into the long-form output on the device,
 * replacing the device -> host -> device copy of :2318-2328: for each chunk c,
 * rows [skip, skip + stride) of chunk c (src + c * src_chunk_bytes
 * + row * src_row_bytes) are copied to rows [write_offset, write_offset +
 * stride) of dst (row pitch dst_row_bytes), row_bytes bytes per row.  chunks
 * is the host array from vtx_encoder_chunk_plan.  One kernel launch per 64
 * chunks on `stream`; no allocation, no host sync, graph-capturable. */
VTX_API int vtx_encoder_stitch(const void *src, size_t src_chunk_bytes, size_t src_row_bytes, void *dst,
                               size_t dst_row_bytes, size_t row_bytes, const vtx_enc_chunk *chunks,
                               int32_t n_chunks, void *stream);

/* ---- attention output projection ------------------------------------------ */

/* The output projection that consumes each attention node's result:
 *     attn_out  = ggml_cont(attn_out); reshape to [Dv*Hq, n]
 *     attn_proj = ggml_mul_mat(attn_o_weight, attn_out)     // [dim, n]
 *     attn_proj = ggml_add(attn_proj, attn_o_bias)          // encoder only
 *     x         = ggml_add(residual, attn_proj)
 * (src/voxtral.cpp:1612-1617 encoder, src/voxtral.cpp:1804-1809 decoder) as
 * one tcgen05 GEMM: dst[t][n] = residual[t][n] + bias[n]
 *                              + sum_k f16(attn[t][k]) * w[n][k]
 * with f32 accumulation (ggml rounds the activations to f16 for an F16
 * weight).  The attention output is read in place -- no contiguous copy --
 * from the layout vtx_flash_attn_ext writes (heads at attn->nb[1], tokens
 * at attn->nb[2]), or, with head_block = h > 0, from heads stored in blocks
 * of h at a stride of block_nb bytes (head i = block i / h, head i % h in
 * it): the rank-major result of a KV-head-split prefill after its
 * all-gather.
 *   attn     F32 [Dv, Hq, n, 1], Dv a multiple of 64; or F16 (vtx_flash_attn_ext
 *            with an F16 dst: the same rounding done once, in the attention
 *            epilogue; the projection reads it by TMA with no conversion)
 *   w        F16 [K = Dv * Hq, N] (ggml's weight: row r = output feature r)
 *   bias     optional F32 [N]
 *   residual optional F32 [N, n]; may be dst itself
 *   dst      F32 [N, n]
 * Asynchronous on `stream`; no allocation, no workspace. */
typedef struct vtx_out_proj_args {
    const vtx_tensor *attn;
    int32_t head_block;          /* 0: one head stride; h > 0: blocks of h heads */
    int32_t reserved;
    size_t block_nb;             /* byte stride between head blocks (head_block > 0) */
    const vtx_tensor *w;
    const vtx_tensor *bias;
    const vtx_tensor *residual;
    vtx_tensor *dst;
} vtx_out_proj_args;
VTX_API int vtx_attn_out_proj(const vtx_out_proj_args *args, void *stream);

/* Diagnostic: synchronises `stream`, returns and clears the device-side error
 * word of the current device (0 = none).  Kernels set it instead of hanging
 * when a bounded pipeline wait runs out, or when a batched-decode stream base
 * is not aligned to the copy width.  No counterpart in ggml (ggml aborts). */
VTX_API int vtx_read_device_error(void *stream);

/* Human-readable text for a vtx_status. */
VTX_API const char *vtx_strerror(int status);

/* VTX_FA_ABI_VERSION of the loaded library. */
VTX_API int vtx_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* VTX_FA_H */
