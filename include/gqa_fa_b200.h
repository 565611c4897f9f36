/*
 * gqa_fa_b200.h - C ABI of the B200 (sm_100a) GQA flash-attention library.
 *
 * The library replaces the three Triton launches of the reference's training
 * path and the one launch of its inference path (zzhhjjj/gemma-triton-flash-attn):
 *
 *   gqafa_fwd  <- FlashAttnGQAFunction.forward launch of _flash_attn_gqa_kernel
 *                 with STORE_LSE=True          (flash_attn/attention.py:1454-1468)
 *              <- attention_flash_gqa launch with STORE_LSE=False, lse == NULL
 *                                              (flash_attn/attention.py:583-603)
 *   gqafa_bwd  <- FlashAttnGQAFunction.backward: the dQ launch with the delta
 *                 prologue (flash_attn/attention.py:1506-1523) followed by the
 *                 packed dK/dV launch (flash_attn/attention.py:1602-1620)
 *
 * Conventions (all taken from the reference):
 *   - q is [B, H_Q, N, D]; k, v are [B, H_KV, N, D]; H_Q % H_KV == 0 and query
 *     head h reads KV head h / (H_Q / H_KV)   (attention.py:272).
 *   - Tensors are fp16 or bf16 (dtype code below) with arbitrary strides in
 *     elements, given as {stride_b, stride_h, stride_n, stride_d}; stride_d must
 *     be 1, the others multiples of 8 elements (16 bytes), pointers 16-byte
 *     aligned. Transposed views such as HF's [B, N, H, D] storage are accepted
 *     without a copy.
 *   - head_dim is 64, 128, 256 or 512 (the reference accepts powers of two up to
 *     512, docs/api.md:63); other values return GQAFA_ERR_UNSUPPORTED.
 *   - causal != 0 applies k <= q. window > 0 additionally applies q - k < window,
 *     and only when causal != 0 (attention.py:289-293, 347-356). window >= N is
 *     treated as full causal (attention.py:1442-1443).
 *   - softmax_scale multiplies Q K^T. The reference fixes it at 1/sqrt(D)
 *     (attention.py:1461); passing another value is how the HF adapter avoids
 *     pre-multiplying q (hf_integration.py:55-58).
 *   - lse is fp32 [B, H_Q, N] contiguous, natural log, including the scale
 *     (attention.py:384-388). delta is fp32 [B, H_Q, N] contiguous scratch that
 *     gqafa_bwd fills with rowsum(dO * O) (attention.py:738-742).
 *   - Outputs have the dtype of q. dq/dk/dv have the shapes of q/k/v.
 *   - Work is launched on `stream` (a cudaStream_t, NULL = legacy default) of
 *     the current CUDA device; nothing is allocated and nothing synchronises.
 *
 * Return value: GQAFA_OK, or an error code; gqafa_last_error() then returns a
 * message (thread-local).
 */
#ifndef GQA_FA_B200_H
#define GQA_FA_B200_H

#if defined(__GNUC__)
#define GQAFA_API __attribute__((visibility("default")))
#else
#define GQAFA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define GQAFA_DTYPE_FP16 0
#define GQAFA_DTYPE_BF16 1

#define GQAFA_OK 0
#define GQAFA_ERR_INVALID 1     /* bad shape, stride, pointer or flag   */
#define GQAFA_ERR_UNSUPPORTED 2 /* valid but not implemented (head_dim) */
#define GQAFA_ERR_CUDA 3        /* a CUDA runtime / driver call failed   */

/* Forward. lse may be NULL (inference path, no LSE written). */
GQAFA_API int gqafa_fwd(const void* q, const long long* q_strides, const void* k, const long long* k_strides,
              const void* v, const long long* v_strides, void* o, const long long* o_strides, float* lse,
              int batch, int heads_q, int heads_kv, int seqlen, int head_dim, float softmax_scale,
              int causal, int window, int dtype, void* stream);

/* Forward with a key length different from the query length (a KV cache:
 * decode or chunked prefill). q and o are [B, H_Q, seqlen_q, D], k and v
 * [B, H_KV, seqlen_k, D], lse (may be NULL) [B, H_Q, seqlen_q]. With causal
 * != 0 the queries are the last seqlen_q of the seqlen_k positions (query row
 * r sits at key position r + seqlen_k - seqlen_q, so seqlen_k >= seqlen_q is
 * required) and a window counts back from that position; without causal every
 * query sees all seqlen_k keys. Replaces the same forward launch as gqafa_fwd
 * (flash_attn/attention.py:583-603): the reference takes the key length from q
 * (attention.py:552-553) and so reads the wrong range of a longer cache; this
 * entry takes both lengths. There is no backward for seqlen_k != seqlen_q. */
GQAFA_API int gqafa_fwd_kv(const void* q, const long long* q_strides, const void* k, const long long* k_strides,
              const void* v, const long long* v_strides, void* o, const long long* o_strides, float* lse,
              int batch, int heads_q, int heads_kv, int seqlen_q, int seqlen_k, int head_dim,
              float softmax_scale, int causal, int window, int dtype, void* stream);

/* Backward. Reads q, k, v, o, dout and lse; writes dq, dk, dv and delta. */
GQAFA_API int gqafa_bwd(const void* q, const long long* q_strides, const void* k, const long long* k_strides,
              const void* v, const long long* v_strides, const void* o, const long long* o_strides,
              const void* dout, const long long* dout_strides, const float* lse, void* dq,
              const long long* dq_strides, void* dk, const long long* dk_strides, void* dv,
              const long long* dv_strides, float* delta, int batch, int heads_q, int heads_kv,
              int seqlen, int head_dim, float softmax_scale, int causal, int window, int dtype,
              void* stream);

/* One stage of gqafa_bwd, same arguments: stage 0 = dQ with the delta
 * prologue (replaces the dQ launch, flash_attn/attention.py:1506-1523),
 * 1 = dK and 2 = dV (together they replace the packed dK/dV launch,
 * flash_attn/attention.py:1602-1620). Stage 0 must run before 1 (dK reads
 * delta). For per-kernel timing and profiling; gqafa_bwd runs all three. */
GQAFA_API int gqafa_bwd_stage(int stage, const void* q, const long long* q_strides, const void* k,
                              const long long* k_strides, const void* v, const long long* v_strides,
                              const void* o, const long long* o_strides, const void* dout,
                              const long long* dout_strides, const float* lse, void* dq,
                              const long long* dq_strides, void* dk, const long long* dk_strides, void* dv,
                              const long long* dv_strides, float* delta, int batch, int heads_q,
                              int heads_kv, int seqlen, int head_dim, float softmax_scale, int causal,
                              int window, int dtype, void* stream);

/* gqafa_bwd without the delta argument, for callers that cannot allocate
 * device memory (an FFI binding that only holds its input and output tensors,
 * or a process whose device memory is planned up front and may not call
 * cudaMalloc). No counterpart in the reference. The delta workspace lives in
 * a fixed 4 MiB device array inside the library, which limits B * H_Q * N to
 * 1,048,576 (larger sizes return GQAFA_ERR_INVALID). The first call on a
 * device looks up the array's address, so make it before any CUDA stream
 * capture. All calls share the array: calls whose kernels overlap on the GPU
 * race on it. Allocates nothing. */
GQAFA_API int gqafa_bwd_noalloc(const void* q, const long long* q_strides, const void* k,
                                const long long* k_strides, const void* v, const long long* v_strides,
                                const void* o, const long long* o_strides, const void* dout,
                                const long long* dout_strides, const float* lse, void* dq,
                                const long long* dq_strides, void* dk, const long long* dk_strides, void* dv,
                                const long long* dv_strides, int batch, int heads_q, int heads_kv, int seqlen,
                                int head_dim, float softmax_scale, int causal, int window, int dtype,
                                void* stream);

/* Materialised backward. The reference's dK/dV launch recomputes
 * S = Q K^T and dP = dO V^T for every (key tile, query block)
 * (flash_attn/attention.py:1602-1620) after its dQ launch already computed
 * them (flash_attn/attention.py:1506-1523). gqafa_bwd_ws instead has the dQ
 * kernel also write P and dS (16-bit, the attended 128 x 256 blocks only) to a
 * caller-provided workspace and computes dK and dV from them in one kernel:
 * 10 instead of 16 head_dim-sized MACs per attended (query, key) pair, and
 * the softmax elementwise work done once. Same arguments and results as
 * gqafa_bwd, plus the workspace (256-byte aligned device memory, any
 * contents). gqafa_bwd_workspace_size returns the bytes it needs
 * (2 * B * H_Q * blocks * 64 KiB, independent of head_dim), 0 where the
 * materialised path does not apply (gqafa_bwd_ws then runs gqafa_bwd and
 * ignores the workspace), or -1 for invalid or unsupported sizes. */
GQAFA_API long long gqafa_bwd_workspace_size(int batch, int heads_q, int heads_kv, int seqlen, int head_dim,
                                             int causal, int window);
GQAFA_API int gqafa_bwd_ws(const void* q, const long long* q_strides, const void* k, const long long* k_strides,
                           const void* v, const long long* v_strides, const void* o, const long long* o_strides,
                           const void* dout, const long long* dout_strides, const float* lse, void* dq,
                           const long long* dq_strides, void* dk, const long long* dk_strides, void* dv,
                           const long long* dv_strides, float* delta, int batch, int heads_q, int heads_kv,
                           int seqlen, int head_dim, float softmax_scale, int causal, int window, int dtype,
                           void* stream, void* workspace, long long workspace_bytes);
/* gqafa_bwd_ws (workspace non-NULL) or gqafa_bwd (workspace NULL) with dk and
 * dv written as fp32 (float, element strides as for the 16-bit tensors; dq
 * stays in the input dtype). No counterpart in the reference: for callers
 * that split the query heads of one KV group over several devices and add the
 * partial dK / dV up (the multi-GPU head split), so that the partials are not
 * rounded to 16 bits before the sum. */
GQAFA_API int gqafa_bwd_partial(const void* q, const long long* q_strides, const void* k,
                                const long long* k_strides, const void* v, const long long* v_strides,
                                const void* o, const long long* o_strides, const void* dout,
                                const long long* dout_strides, const float* lse, void* dq,
                                const long long* dq_strides, void* dk, const long long* dk_strides, void* dv,
                                const long long* dv_strides, float* delta, int batch, int heads_q, int heads_kv,
                                int seqlen, int head_dim, float softmax_scale, int causal, int window, int dtype,
                                void* stream, void* workspace, long long workspace_bytes);
/* One kernel of gqafa_bwd_ws: stage 0 = dQ + delta + P/dS, 1 = dK + dV
 * (needs stage 0's workspace contents). For per-kernel timing. */
GQAFA_API int gqafa_bwd_ws_stage(int stage, const void* q, const long long* q_strides, const void* k,
                                 const long long* k_strides, const void* v, const long long* v_strides,
                                 const void* o, const long long* o_strides, const void* dout,
                                 const long long* dout_strides, const float* lse, void* dq,
                                 const long long* dq_strides, void* dk, const long long* dk_strides, void* dv,
                                 const long long* dv_strides, float* delta, int batch, int heads_q, int heads_kv,
                                 int seqlen, int head_dim, float softmax_scale, int causal, int window, int dtype,
                                 void* stream, void* workspace, long long workspace_bytes);

/* Row-range variants for splitting one (batch, KV-group) unit across GPUs
 * by sequence blocks (no counterpart in the reference, whose launches always
 * cover every row). Same arguments as gqafa_fwd / gqafa_bwd_stage plus
 * [row_begin, row_end): row_begin a multiple of 128, row_end a multiple of 128
 * or N. gqafa_fwd_rows writes the O and LSE rows of that query range (keys:
 * all). gqafa_bwd_stage_rows stage 0 writes the dQ and delta rows of that
 * query range; stages 1 and 2 write the dK / dV rows of that key range and
 * read lse and delta of every query row, so those must be complete. */
GQAFA_API int gqafa_fwd_rows(const void* q, const long long* q_strides, const void* k, const long long* k_strides,
                             const void* v, const long long* v_strides, void* o, const long long* o_strides,
                             float* lse, int batch, int heads_q, int heads_kv, int seqlen, int head_dim,
                             float softmax_scale, int causal, int window, int dtype, void* stream, int row_begin,
                             int row_end);
GQAFA_API int gqafa_bwd_stage_rows(int stage, const void* q, const long long* q_strides, const void* k,
                                   const long long* k_strides, const void* v, const long long* v_strides,
                                   const void* o, const long long* o_strides, const void* dout,
                                   const long long* dout_strides, const float* lse, void* dq,
                                   const long long* dq_strides, void* dk, const long long* dk_strides, void* dv,
                                   const long long* dv_strides, float* delta, int batch, int heads_q,
                                   int heads_kv, int seqlen, int head_dim, float softmax_scale, int causal,
                                   int window, int dtype, void* stream, int row_begin, int row_end);

/* 1 if (head_dim, dtype) has a compiled kernel set, else 0. */
GQAFA_API int gqafa_supported(int head_dim, int dtype);

/* Message of the last failed call on this thread ("" if none). */
GQAFA_API const char* gqafa_last_error(void);

/* Synchronises `device` and returns its kernel status word (0 = every kernel
 * finished its pipeline; otherwise the code of the first bounded wait that
 * timed out). reset != 0 clears the word afterwards. Returns -1 on a CUDA
 * error. Not for the hot path. */
GQAFA_API int gqafa_device_status(int device, int reset);

/* Diagnostics, not for the hot path: point the kernels at a device buffer of
 * 9 zeroed unsigned 64-bit counters (NULL turns it off). Kernels that support
 * it (the head_dim-512 backward) then add the cycles each role spends waiting:
 * [0] producer on free ring stages, [1] MMA issuer on score operands, [2] on
 * accumulate operands, [3] on the row warps, [4] row warps on scores, [5] row
 * warps' elementwise work, [6] epilogue, [7] CTA lifetime, [8] CTA count. */
GQAFA_API int gqafa_set_wait_counters(void* device_counters);

/* Test knob (no counterpart in the reference, whose Triton kernels have no
 * bounded waits): every mbarrier wait of later launches gives up after
 * `wait_limit_cycles` clock cycles (<= 0 restores the default of 2e9, about
 * one second), and with `skip_loads` != 0 the kernels' TMA producers issue
 * nothing, so every wait runs into that bound. A timed-out launch records a
 * non-zero code in the status word (gqafa_device_status), frees its tensor
 * memory and returns; its outputs are undefined. Used by the tests of the
 * timeout path; process-wide, not for production use. */
GQAFA_API int gqafa_set_test_waits(long long wait_limit_cycles, int skip_loads);

/* Library version string. */
GQAFA_API const char* gqafa_version(void);

#ifdef __cplusplus
}
#endif
#endif /* GQA_FA_B200_H */
