/*
 * ee_b200.h - C ABI of the B200 (sm_100a) entropy-gated mixed-precision engine.
 *
 * Library: libee_b200.so (built in-tree by triton-kernels-optimization_b200/build.py).
 *
 * Conventions
 *  - Every compute entry point takes a CUDA stream as `void* stream` (a cudaStream_t;
 *    NULL = the legacy default stream) and only enqueues work on it: the call returns
 *    before the GPU is done.  Nothing here synchronises the device.
 *  - All buffers are device pointers owned by the caller; nothing allocates device
 *    memory.  Matrices are row-major with an explicit leading dimension in ELEMENTS.
 *  - Returns EE_OK (0) or a negative EE_ERR_* status; ee_last_error() gives the text
 *    of the last failure on the calling thread.  Nothing is enqueued when a call
 *    returns an error.
 *  - fp16 buffers are passed as `void*` (IEEE binary16), e4m3 buffers as uint8_t
 *    (OCP FP8 E4M3FN bytes).
 *  - Entry points are thread-safe; calls on different streams may run concurrently
 *    when they use different output and workspace buffers.
 *
 * Reference surface each entry point replaces ("EE/" = the reference's
 * entropy-engine/ directory):
 *   EE/python/kernels.py:264-312  fused_softmax_entropy_kernel -> ee_softmax_entropy
 *   EE/python/kernels.py:416-453  fused_softmax_entropy        -> ee_fused_softmax_entropy_4d
 *   EE/python/dispatch.py:243-245 Llama-path attention entropy -> ee_attention_entropy
 *   EE/python/dispatch.py:55-82   PipelinedEntropyDispatcher   -> ee_route_batch_max, ee_route
 *   EE/python/dispatch.py:43-48   quantize_weights_int8        -> ee_quantize_weights_int8
 *   EE/python/kernels.py:330-351  triton_int8_gemm             -> ee_linear_int8
 *   EE/python/kernels.py:354-373  triton_fp8_gemm              -> ee_linear_fp8
 *   EE/python/kernels.py:380-409  triton_fp16_gemm             -> ee_gemm_fp16
 *   EE/csrc/engine.cpp:106-166    CubinEngine::forward         -> ee_gemm_int8
 *   EE/python/dispatch.py:126-140 EntropyDispatchedLinear      -> ee_gated_linear
 */
#ifndef EE_B200_H_
#define EE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define EE_API __attribute__((visibility("default")))
#else
#define EE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define EE_ABI_VERSION 1

#define EE_OK 0
#define EE_ERR_INVALID (-1)     /* bad argument (null pointer, negative or zero size, bad flag) */
#define EE_ERR_MISALIGNED (-2)  /* pointer / leading dimension misses the required alignment */
#define EE_ERR_UNSUPPORTED (-3) /* shape outside what the kernels support (see each entry) */
#define EE_ERR_CUDA (-4)        /* a CUDA runtime / driver call failed (text in ee_last_error) */
#define EE_ERR_DEVICE (-5)      /* a kernel reported an error word (see ee_device_check) */

/* Precision buckets = route ids = the reference's PrecisionTier values. */
#define EE_INT8 0
#define EE_FP8 1
#define EE_FP16 2

/* element types of ee_attention_entropy's probabilities */
#define EE_DTYPE_F16 0
#define EE_DTYPE_F32 1

EE_API int ee_abi_version(void);
EE_API const char* ee_last_error(void);

/* GEMM tiling policy for every later call in the process (no counterpart in the
 * reference): 0 = automatic (CTA-pair 256 x 256 tiles above 128 rows; 65 .. 128 rows
 * single-CTA 128 x 256 tiles, or 128 x 64 tiles when the wide ones would leave SMs idle;
 * at most 64 rows -- the call streams its weights -- the weight-streaming kernel:
 * 128-channel tiles against all of a bucket's rows, K split over a thread-block
 * cluster), 1 = always
 * single-CTA 128 x 256, 2 = always CTA pairs, 3 = always single-CTA 128 x 64, 4 = the
 * weight-streaming kernel where the call has at most 128 rows (else automatic).  INT8
 * results are identical under every policy; FP8 / FP16 results of the weight-streaming
 * kernel with K split differ from the others in the last bits (fp32 partial sums added
 * in rank order: deterministic, not the single-pass accumulation order). */
EE_API int ee_set_gemm_policy(int policy);

/* K splits per 128-channel tile of the weight-streaming kernel for every later call:
 * 0 = chosen per call (about one CTA per resident slot), 1 .. 8 = forced. */
EE_API int ee_set_gemm_splits(int splits);

/* Reads and clears the current device's error word (set by a kernel whose bounded
 * wait gave up).  Synchronous.  EE_OK if clear, EE_ERR_DEVICE otherwise; *value
 * (nullable) receives the word. */
EE_API int ee_device_check(int* value);

/* Failure-detection test hook (no counterpart in the reference, whose kernels have no
 * bounded waits).  Arms a one-shot fault for the next launch of the single-CTA gated
 * GEMM kernel (ee_set_gemm_policy(1) forces that kernel): its CTA `cta` issues neither
 * the TMA copies nor the barrier arrival of its first K stage, so the MMA warp's bounded
 * wait on that stage gives up after 2 s, the CTA unwinds (drains its MMAs and copies,
 * frees its tensor memory) and sets the error word ee_device_check reports.  Nothing
 * faults or hangs; that call's output is incomplete, every later call runs normally.
 * After the error, re-zero each gated workspace's header (ee_gate_rows does) before
 * routing with it again. */
EE_API int ee_debug_drop_next_gemm_load(int cta);

/* ---------------------------------------------------------------- softmax + entropy
 * Per row r of the fp16 matrix x [rows, n] (row stride ld):
 *   p = softmax(x[r]), H[r] = -sum p log p   (fp32 math)
 * causal != 0 masks column j of row r when j > r % S (the reference's query_pos).
 * probs (fp16 [rows, n], stride ldp) is written when non-NULL (masked entries = 0).
 * route (int8 [rows]) is written when non-NULL: H < tau_low -> EE_INT8,
 * H < tau_high -> EE_FP8, else EE_FP16 (strict comparisons).
 * Any n >= 1; the fast path wants n % 8 == 0, ld % 8 == 0 and 16-byte aligned rows.
 * Replaces EE/python/kernels.py:264-312. */
EE_API int ee_softmax_entropy(const void* x, int64_t rows, int64_t n, int64_t ld, int causal, int64_t S, void* probs,
                       int64_t ldp, float* H, int8_t* route, double tau_low, double tau_high, void* stream);

/* The reference's 4-D surface: logits [B, Hh, S, S] contiguous fp16 ->
 * probs [B, Hh, S, S] fp16 (nullable), row_entropy [B*Hh*S] fp32 (caller scratch,
 * required), batch_entropy [B] = mean of row_entropy over (Hh, S).
 * Replaces EE/python/kernels.py:416-453. */
EE_API int ee_fused_softmax_entropy_4d(const void* logits, int64_t B, int64_t Hh, int64_t S, int causal, void* probs,
                                float* row_entropy, float* batch_entropy, void* stream);

/* Entropy of given attention probabilities, the Llama block's router input:
 *   row_entropy[r] = -sum_j p[r, j] * ln(p[r, j] + 1e-10)   (fp32 arithmetic)
 * for `rows` rows of n probabilities (row stride ld elements, dtype EE_DTYPE_F16 or
 * EE_DTYPE_F32), then batch_entropy[b] = mean of row_entropy over the rows / batches
 * consecutive rows of batch b (nullable; rows % batches == 0).  row_entropy is
 * required.  For [B, Hh, S, S] probabilities: rows = B*Hh*S, n = ld = S, batches = B.
 * Replaces EE/python/dispatch.py:243-245. */
EE_API int ee_attention_entropy(const void* probs, int dtype, int64_t rows, int64_t n, int64_t ld, float* row_entropy,
                                int64_t batches, float* batch_entropy, void* stream);

/* Causal (or full) attention with the entropy of every query row, in one pass over K
 * and V (flash attention on tcgen05): the Llama block's attention output and router
 * input without the [B, Hq, S, S] probabilities the reference materialises
 * (EE/python/dispatch.py:236-245).  Q fp16 [B, Hq, S, head_dim], K and V fp16
 * [B, Hkv, S, head_dim] (contiguous; Hq % Hkv == 0: grouped-query heads), head_dim 64 or
 * 128.  Scores follow the reference's eager path -- fp16(Q K^T), times `scale`, rounded
 * to fp16, causal mask, softmax in fp32 -- and O = softmax . V is written fp16
 * [B, S, Hq, head_dim] (the layout o_proj reads); H fp32 [B, Hq, S] receives
 * -sum_k p_k ln p_k of each row.  Workspace: ee_attention_workspace_bytes (V transposed),
 * 256-byte aligned.  No counterpart in the reference's kernels (its entropy needs the
 * probabilities in HBM). */
EE_API size_t ee_attention_workspace_bytes(int64_t B, int64_t Hkv, int64_t S, int64_t head_dim);
EE_API int ee_flash_attention_entropy(const void* Q, const void* K, const void* V, int64_t B, int64_t Hq, int64_t Hkv,
                                      int64_t S, int64_t head_dim, int causal, float scale, void* O, float* H,
                                      void* workspace, size_t workspace_bytes, void* stream);
/* ee_flash_attention_entropy on the projections' outputs as they come: q rows
 * [B*S, Hq*head_dim] (row stride ldq), k and v rows [B*S, Hkv*head_dim] (ldk, ldv), and
 * the rotary tables cos / sin [B*S, head_dim] (row stride ld_cs, fp16: what transformers'
 * LlamaRotaryEmbedding returns).  One pass applies the rotary embedding to q and k with
 * the roundings of transformers' apply_rotary_pos_emb on fp16 tensors --
 * fp16(fp16(x * cos) + fp16(rotate_half(x) * sin)) -- and writes them in the [B, H, S,
 * head_dim] layouts, V is transposed from its rows, then the attention runs as above.
 * Replaces the block's reshape / transpose / rotate_half / cat / multiply / add chain
 * (EE/python/dispatch.py:237 through transformers' attention).  Workspace:
 * ee_attention_rope_workspace_bytes, 256-byte aligned; all rows 16-byte aligned with
 * strides that are multiples of 8 elements. */
EE_API size_t ee_attention_rope_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t head_dim);
EE_API int ee_flash_attention_rope_entropy(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                                           int64_t ldv, const void* cos, const void* sin, int64_t ld_cs, int64_t B,
                                           int64_t Hq, int64_t Hkv, int64_t S, int64_t head_dim, int causal,
                                           float scale, void* O, float* H, void* workspace, size_t workspace_bytes,
                                           void* stream);

/* The block's router inputs from the attention's row entropies H fp32 [B, Hq, S]:
 * token_entropy[b * S + s] = (sum over heads of H[b, h, s]) / Hq, heads added in
 * ascending order (per-token routing), and batch_entropy[b] (nullable) = the mean of
 * H[b] over heads and positions -- the reference's entropy_batch
 * (EE/python/dispatch.py:244-245), the input of its batch-max dispatcher. */
EE_API int ee_head_mean_entropy(const float* H, int64_t B, int64_t Hq, int64_t S, float* token_entropy,
                                float* batch_entropy, void* stream);

/* ee_flash_attention_rope_entropy with the reference's entropy exactly: H receives
 * -sum_j p_j ln(p_j + 1e-10) (fp32) of the fp16-ROUNDED probabilities
 * p_j = fp16(softmax_fp32(scores)_j) that transformers' eager attention returns and the
 * reference's block reduces (EE/python/dispatch.py:236-245), instead of the entropy of
 * the unrounded softmax.  Rounding a probability needs its row's normaliser, known only
 * after the last key, so a second tcgen05 pass over the keys recomputes the scores and
 * reduces the rounded probabilities (about half the first pass's tensor work plus an
 * exponential and a logarithm per score).  O is the same as without it.  Workspace:
 * ee_attention_exact_workspace_bytes (each row's exponent reference and sum after the
 * rotary / attention workspace).  No counterpart in the reference's kernels. */
EE_API size_t ee_attention_exact_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t head_dim);
EE_API int ee_flash_attention_rope_entropy_exact(const void* q, int64_t ldq, const void* k, int64_t ldk,
                                                 const void* v, int64_t ldv, const void* cos, const void* sin,
                                                 int64_t ld_cs, int64_t B, int64_t Hq, int64_t Hkv, int64_t S,
                                                 int64_t head_dim, int causal, float scale, void* O, float* H,
                                                 void* workspace, size_t workspace_bytes, void* stream);

/* The Llama block's RMSNorm with the residual add before it folded in (transformers'
 * LlamaRMSNorm.forward and the block's `residual + x`, EE/python/dispatch.py:166-210):
 * with residual: s = fp16(residual + x), stored to sum_out when given; without: s = x;
 * y = fp16(weight * fp16(fp32(s) * rsqrt(mean(fp32(s)^2) + eps))).  x, residual,
 * sum_out, y: fp16 rows of d (8 .. 8192, a multiple of 8) with the given strides; weight
 * fp16 [d].  The sum of squares is taken in a different order than torch's reduction,
 * so an output may differ from transformers' by up to two fp16 ulps (one in the
 * normalised value, carried through the weight product); over 99 % are equal. */
EE_API int ee_add_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ldr, void* sum_out, int64_t lds,
                          const void* weight, float eps, void* y, int64_t ldy, int64_t M, int64_t d, void* stream);

/* ---------------------------------------------------------------- routing
 * route[i] = dual-threshold tier of H[i]                (per-row granularity) */
EE_API int ee_route(const float* H, int64_t rows, double tau_low, double tau_high, int8_t* route, void* stream);
/* The reference dispatcher's granularity: tier of max(H[0..n)).  max_out (fp32[1])
 * and tier_out (int8[1]) are device pointers (either may be NULL; both may point to
 * mapped pinned host memory).  Replaces EE/python/dispatch.py:63-82. */
EE_API int ee_route_batch_max(const float* H, int64_t n, double tau_low, double tau_high, float* max_out, int8_t* tier_out,
                       void* stream);

/* ---------------------------------------------------------------- weights (offline)
 * Per-output-channel INT8 quantisation of W fp16 [N, K] (nn.Linear layout, row
 * stride ldw):  s[n] = max(amax_k |W[n,k]| / 127, 1e-8),
 * q = clamp(round_half_even(W / s), -127, 127).
 * div_mode 0 evaluates amax/127 as amax * fp32(1/127) (what torch does on CUDA),
 * 1 as an IEEE division (what torch does on CPU).
 * w_kn: int8 [K, N] (the reference's returned layout), w_nk: int8 [N, K]; either may
 * be NULL.  Replaces EE/python/dispatch.py:43-48. */
EE_API int ee_quantize_weights_int8(const void* W, int64_t N, int64_t K, int64_t ldw, int8_t* w_kn, int8_t* w_nk,
                             float* scale, int div_mode, void* stream);

/* From the reference's weight format (int8 [K, N] + fp32 scale [N]) build the
 * K-major [N, K] operand packs of the three buckets (each nullable):
 *   w_i8_nk   = q,   w_e4m3_nk = e4m3(fp16(q)),   w_f16_nk = fp16(fp16(q) * fp16(s)).
 * These equal, bit for bit, the operands the reference's Triton kernels build per
 * tile (EE/python/kernels.py:166, :233). */
EE_API int ee_pack_weights(const int8_t* w_kn, const float* scale, int64_t K, int64_t N, int8_t* w_i8_nk,
                    uint8_t* w_e4m3_nk, void* w_f16_nk, void* stream);

/* ---------------------------------------------------------------- activations
 * Per-row symmetric quantisation of A fp16 [M, K] (row stride lda, K % 8 == 0):
 *   INT8: s = fp16(amax/127), q = trunc(A / s)               (EE/python/kernels.py:336-338)
 *   e4m3: s = fp16(amax/448), q = e4m3(fp16(A * fp16(1/s)))  (EE/python/kernels.py:361, :144-160)
 * q: [M, K] contiguous, scale: fp32 [M]. */
EE_API int ee_quant_rows_int8(const void* A, int64_t M, int64_t K, int64_t lda, int8_t* q, float* scale, void* stream);
EE_API int ee_quant_rows_e4m3(const void* A, int64_t M, int64_t K, int64_t lda, uint8_t* q, float* scale, void* stream);

/* ---------------------------------------------------------------- tcgen05 GEMMs
 * Y fp16 [M, N] (row stride ldy) = A [M, K] . W_nk [N, K]^T with the bucket's
 * epilogue.  Requirements: K % 16 == 0, N % 8 == 0, ldy % 8 == 0, every matrix and
 * scale pointer 16-byte aligned; M, N, K < 2^31.  M == 0 is a no-op.
 *   ee_gemm_int8 : y = fp16((fp32(acc_i32) * a_scale[m]) * w_scale[n])
 *                  (EE/python/kernels.py:52-110, EE/csrc/engine.cpp:106-166)
 *   ee_gemm_fp8  : y = fp16((acc_f32 * a_scale[m]) * w_scale[n])  (EE/python/kernels.py:120-180)
 *   ee_gemm_fp16 : y = fp16(acc_f32)                              (EE/python/kernels.py:194-246)
 * The *_acc variants store the raw accumulators (int32 / fp32 [M, N], ldy = N) for
 * verification. */
EE_API int ee_gemm_int8(const int8_t* A, const float* a_scale, const int8_t* W_nk, const float* w_scale, void* Y,
                 int64_t M, int64_t N, int64_t K, int64_t ldy, void* stream);
EE_API int ee_gemm_fp8(const uint8_t* A, const float* a_scale, const uint8_t* W_nk, const float* w_scale, void* Y,
                int64_t M, int64_t N, int64_t K, int64_t ldy, void* stream);
EE_API int ee_gemm_fp16(const void* A, const void* W_nk, void* Y, int64_t M, int64_t N, int64_t K, int64_t ldy,
                 void* stream);
EE_API int ee_gemm_int8_acc(const int8_t* A, const int8_t* W_nk, int32_t* acc, int64_t M, int64_t N, int64_t K,
                     void* stream);
EE_API int ee_gemm_fp8_acc(const uint8_t* A, const uint8_t* W_nk, float* acc, int64_t M, int64_t N, int64_t K,
                    void* stream);
EE_API int ee_gemm_fp16_acc(const void* A, const void* W_nk, float* acc, int64_t M, int64_t N, int64_t K, void* stream);

/* fp16 activations in, quantisation fused in front of the GEMM (the reference's
 * launchers).  Workspace: ee_linear_workspace_bytes(M, K) bytes, 256-byte aligned.
 * Replace EE/python/kernels.py:330-351 (INT8) and :354-373 (FP8). */
EE_API size_t ee_linear_workspace_bytes(int64_t M, int64_t K);
EE_API int ee_linear_int8(const void* A, int64_t lda, const int8_t* W_nk, const float* w_scale, void* Y, int64_t M,
                   int64_t N, int64_t K, int64_t ldy, void* workspace, size_t workspace_bytes, void* stream);
EE_API int ee_linear_fp8(const void* A, int64_t lda, const uint8_t* W_e4m3_nk, const float* w_scale, void* Y, int64_t M,
                  int64_t N, int64_t K, int64_t ldy, void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free variant of ee_linear_int8 (this entry point has no counterpart in
 * the reference).  Same inputs, output and result; instead of a caller-provided
 * workspace it keeps the quantised activations and their scales in a fixed block of
 * device memory compiled into this library (16 MiB + 64 KiB per device, held until
 * the process exits).  It is for callers that cannot hand out device memory: e.g. a
 * serving process that reserves all of the GPU's memory for its own pool at start-up
 * and forbids any further allocation, or a plug-in hosted by another runtime that owns
 * the allocator and gives the plug-in no way to borrow from it.
 * Limits: M <= 16384 rows and M * K <= 2^24; larger calls return EE_ERR_UNSUPPORTED
 * (use ee_linear_int8 then).  The first call on a device looks up the block's device
 * address (cudaGetSymbolAddress, once per device context: again after a
 * cudaDeviceReset, which unloads the block); make that first call before any stream
 * capture begins.  All calls share the one block and each call overwrites what
 * the previous left there (nothing in it needs to start at zero): calls that can
 * overlap on the GPU -- on different streams, or from different threads -- race on it
 * and must be serialised by the caller. */
EE_API int ee_linear_int8_noalloc(const void* A, int64_t lda, const int8_t* W_nk, const float* w_scale, void* Y,
                                  int64_t M, int64_t N, int64_t K, int64_t ldy, void* stream);

/* ---------------------------------------------------------------- entropy-gated linear
 * The on-device dispatcher: per-row routing of A's rows by the entropy of the
 * matching logits rows, per-row quantisation into three compacted buckets, one
 * persistent tcgen05 GEMM over all buckets, results scattered back in row order:
 *   Y[i] = gemm_{route[i]}(A, W)[i].
 * Workspace: ee_gated_workspace_bytes(M, K) bytes, 256-byte aligned, one per
 * concurrently running call.  After ee_gate_rows the workspace holds the routing of
 * M rows; any number of ee_gated_gemm calls (one per projection that shares the
 * routing, with its own A of M rows and width K) may follow on the same stream.
 * ee_gated_linear = ee_gate_rows + ee_gated_gemm.
 * H (fp32 [M]) and route (int8 [M]) are outputs; NULL keeps them in the workspace.
 * bucket_counts (int32 [3], device, nullable) receives the rows per bucket.
 * K split: a workspace larger than ee_gated_workspace_bytes(M, K) of the call lends
 * the rest to its GEMM for K-split partial sums.  When a call has few tiles for the SMs
 * (mid-size M: e.g. 128 or 1024 rows at Llama-3-8B widths) the GEMM then cuts each
 * tile's K loop into ranges run by different CTAs and adds the ranges' int32 / fp32
 * partials in range order in a second kernel: INT8 results bit-identical to the unsplit
 * run, FP8 / FP16 within the last bits (deterministic).  ee_gated_workspace_split_bytes
 * (M, K) is the recommended size (the base plus four 128 KiB partial blocks per SM;
 * just the base for M <= 64, where the weight-streaming kernel splits K itself, and for
 * M > 4096, where the tiles already fill the SMs). */
EE_API size_t ee_gated_workspace_bytes(int64_t M, int64_t K);
EE_API size_t ee_gated_workspace_split_bytes(int64_t M, int64_t K);
EE_API int ee_gate_rows(const void* logits, int64_t M, int64_t n, int64_t ld, double tau_low, double tau_high, float* H,
                 int8_t* route, int32_t* bucket_counts, void* workspace, size_t workspace_bytes, void* stream);
/* ee_gate_rows without zeroing the workspace head (its first
 * ee_gated_workspace_head_bytes() bytes: bucket counters, tile counters and the router's
 * single-pass scan state), for callers that zeroed it once -- every kernel of the path
 * leaves it consistent after a clean run -- and saw no device error since (after one,
 * zero it again or call ee_gate_rows).  Saves the memset, and lets the router launch
 * start while the previous kernel of the stream drains. */
EE_API int ee_gate_rows_keep(const void* logits, int64_t M, int64_t n, int64_t ld, double tau_low, double tau_high,
                             float* H, int8_t* route, int32_t* bucket_counts, void* workspace,
                             size_t workspace_bytes, void* stream);
EE_API size_t ee_gated_workspace_head_bytes(void);
/* ee_gate_rows for callers that already hold one entropy per row (the Llama block's
 * per-token router: the mean over heads of the attention entropy of each query
 * position): routes the M rows of H (fp32, device) into the workspace, ready for
 * ee_gated_gemm / ee_gated_pack.  No counterpart in the reference, which gates whole
 * batches (EE/python/dispatch.py:64). */
EE_API int ee_gate_entropies(const float* H, int64_t M, double tau_low, double tau_high, int8_t* route,
                             int32_t* bucket_counts, void* workspace, size_t workspace_bytes, void* stream);
EE_API int ee_gated_gemm(const void* A, int64_t lda, int64_t M, int64_t K, const int8_t* W_i8_nk,
                  const uint8_t* W_e4m3_nk, const void* W_f16_nk, const float* w_scale, int64_t N, void* Y,
                  int64_t ldy, void* workspace, size_t workspace_bytes, void* stream);
/* The two halves of ee_gated_gemm, for callers that time or schedule them apart:
 * ee_gated_pack quantises / copies A's rows into the workspace's bucket buffers
 * (per the routing left there by ee_gate_rows); ee_gated_gemm_packed runs the
 * persistent tcgen05 GEMM over the packed buckets and scatters Y. */
EE_API int ee_gated_pack(const void* A, int64_t lda, int64_t M, int64_t K, void* workspace, size_t workspace_bytes,
                         void* stream);
EE_API int ee_gated_gemm_packed(int64_t M, int64_t K, const int8_t* W_i8_nk, const uint8_t* W_e4m3_nk,
                                const void* W_f16_nk, const float* w_scale, int64_t N, void* Y, int64_t ldy,
                                void* workspace, size_t workspace_bytes, void* stream);
/* The gated SwiGLU MLP's first half in one GEMM over the rows packed by
 * ee_gated_pack: Y[i, c] = fp16(silu(gate[i, c]) * up[i, c]) for c < I, where gate / up
 * are what ee_gated_gemm_packed would write for the gate and up weights (each row in
 * its bucket's precision) and silu(g) = fp16(g / (1 + exp(-g))) -- the roundings of
 * torch.nn.functional.silu(gate) * up on those fp16 outputs (EE/python/dispatch.py:
 * 201-203).  The weight packs and scales hold 2I rows: gate and up interleaved in
 * groups of 128 (rows 256t .. 256t+127 = gate channels 128t .., the next 128 = the same
 * up channels); I % 128 == 0.  Y: fp16 [M, I], row stride ldy. */
EE_API int ee_gated_swiglu_packed(int64_t M, int64_t K, const int8_t* Wgu_i8_nk, const uint8_t* Wgu_e4m3_nk,
                                  const void* Wgu_f16_nk, const float* wgu_scale, int64_t I, void* Y, int64_t ldy,
                                  void* workspace, size_t workspace_bytes, void* stream);
/* Byte offsets, inside a gated workspace for (M, K), of: [0] bucket counts int32[3],
 * [1] perm int32[M] (position -> row), [2] slot int32[M] (row -> position),
 * [3] route int8[M], [4] H fp32[M], [5] activation scales fp32[M], [6] 8-bit rows
 * [M, K], [7] fp16 rows [M, K].  Lets a caller read the routing in place. */
EE_API int ee_gated_workspace_layout(int64_t M, int64_t K, int64_t* offsets);
EE_API int ee_gated_linear(const void* logits, int64_t n, int64_t ld_logits, const void* A, int64_t lda, int64_t M,
                    int64_t K, const int8_t* W_i8_nk, const uint8_t* W_e4m3_nk, const void* W_f16_nk,
                    const float* w_scale, int64_t N, double tau_low, double tau_high, float* H, int8_t* route,
                    int32_t* bucket_counts, void* Y, int64_t ldy, void* workspace, size_t workspace_bytes,
                    void* stream);

/* ---------------------------------------------------------------- gated layer loop (engine)
 * The reference runs its layer loop in Python with a host synchronisation per layer
 * (EE/python/dispatch.py:192-203, EE/python/quality_eval.py:133-141) and launches
 * one cubin at a time from C++ (EE/csrc/engine.cpp:64-200).  The engine takes a fixed
 * description of L gated layers -- per layer the routing logits and P projections,
 * every buffer at a fixed device address owned by the caller -- and enqueues the
 * whole loop with no host round trip: eagerly (ee_engine_run) or as a CUDA graph
 * recorded once and replayed (ee_engine_capture / ee_engine_launch).  Layers run in
 * order on one stream and share one workspace (ee_engine_workspace_bytes). */
typedef struct ee_engine ee_engine;

typedef struct ee_projection {
  int64_t K, N;
  const void* A;           /* fp16 [rows, K] input, row stride lda */
  int64_t lda;
  const int8_t* w_i8_nk;   /* the three packs of ee_pack_weights and the weight scale */
  const uint8_t* w_e4m3_nk;
  const void* w_f16_nk;
  const float* w_scale;
  void* Y;                 /* fp16 [rows, N] output, row stride ldy */
  int64_t ldy;
} ee_projection;

typedef struct ee_gated_layer {
  const void* logits;      /* fp16 [rows, n_logits], row stride ld_logits: routes this layer's rows */
  int64_t n_logits, ld_logits;
  int32_t n_proj;
  const ee_projection* proj;
} ee_gated_layer;

EE_API size_t ee_engine_workspace_bytes(int64_t rows, int32_t n_layers, const ee_gated_layer* layers);
/* Copies the descriptions; the buffers they point to must outlive the engine. */
EE_API int ee_engine_create(int64_t rows, double tau_low, double tau_high, int32_t n_layers,
                            const ee_gated_layer* layers, void* workspace, size_t workspace_bytes, ee_engine** out);
EE_API int ee_engine_run(ee_engine* engine, void* stream);
/* Records the loop into a CUDA graph; stream must be a created (non-default) stream. */
EE_API int ee_engine_capture(ee_engine* engine, void* stream);
/* Replays the recorded graph (records it first if needed). */
EE_API int ee_engine_launch(ee_engine* engine, void* stream);
EE_API int ee_engine_destroy(ee_engine* engine);

/* ---------------------------------------------------------------- entropy-tied KV cache
 * The reference lists "dynamic KV-cache compression tied to the entropy metric" as its
 * next step (README, Work In Progress) and has no code for it.  Here every cached token
 * keeps its keys and values at the precision of its entropy tier -- the same dual-
 * threshold route ids as the linears (0 INT8, 1 FP8-e4m3, 2 FP16): INT8 codes
 * q = rn(x / s), s = amax / 127, or e4m3 codes of x / s, s = amax / 448, with one fp32
 * scale per (token, KV head), or the fp16 values -- in two slot pools (8-bit: slots8
 * token slots, fp16: slots16) shared by the batch's sequences and addressed through a
 * per-sequence slot table, so the cache holds about 1 byte per value for 8-bit tokens
 * and the decode attention reads that much less.  One device allocation of
 * ee_kv_cache_bytes, carved by ee_kv_cache_init; the caller keeps the struct. */
typedef struct ee_kv_cache {
  int64_t batch, kv_heads, head_dim, max_tokens, slots8, slots16;
  uint8_t* k8;         /* [slots8, kv_heads, head_dim] INT8 / e4m3 codes */
  uint8_t* v8;
  void* k16;           /* [slots16, kv_heads, head_dim] fp16 */
  void* v16;
  float* k_scale;      /* [slots8, kv_heads] */
  float* v_scale;
  int32_t* slot;       /* [batch, max_tokens]: (tier << 28) | slot in its pool */
  int32_t* length;     /* [batch] tokens stored */
  uint32_t* pool_used; /* [2] slots taken in the 8-bit and fp16 pools */
} ee_kv_cache;

EE_API size_t ee_kv_cache_bytes(int64_t batch, int64_t kv_heads, int64_t head_dim, int64_t max_tokens,
                                int64_t slots8, int64_t slots16);
/* Lays the cache out in `memory` (256-byte aligned, ee_kv_cache_bytes) and empties it
 * (every length and pool counter zero) on `stream`.  head_dim 64 or 128. */
EE_API int ee_kv_cache_init(ee_kv_cache* cache, void* memory, size_t bytes, int64_t batch, int64_t kv_heads,
                            int64_t head_dim, int64_t max_tokens, int64_t slots8, int64_t slots16, void* stream);
/* Appends t_new tokens to every sequence: row b * t_new + t of k_rows / v_rows (fp16
 * [batch * t_new, kv_heads * head_dim], row strides ldk / ldv; K after the rotary
 * embedding) at tier[b * t_new + t].  A token that finds its pool or its sequence full
 * is not stored and sets the device error word (ee_device_check, bit 8). */
EE_API int ee_kv_append(const ee_kv_cache* cache, const void* k_rows, int64_t ldk, const void* v_rows, int64_t ldv,
                        const int8_t* tier, int64_t t_new, void* stream);
/* One decode step's attention: query row b (fp16 q [batch, heads * head_dim], row stride
 * ldq; heads a multiple of kv_heads: 1, 2, 4 or 8 query heads per KV head) against the
 * sequence's cached tokens and its own new K / V rows (k_new / v_new fp16 [batch,
 * kv_heads * head_dim], row stride ld_new, not yet appended), softmax(scale q k) v ->
 * out fp16 [batch, heads * head_dim] (row stride ldo), and H (nullable, fp32 [batch,
 * heads]) the entropy of each softmax row: the router input of the new token.  The
 * tokens are split over CTAs (flash-decoding) whose partials merge in a second launch;
 * workspace: ee_kv_decode_workspace_bytes.  The cache's K / V pools must be 16-byte
 * aligned (the layout of ee_kv_cache_init is); EE_ERR_MISALIGNED otherwise. */
EE_API size_t ee_kv_decode_workspace_bytes(const ee_kv_cache* cache, int64_t heads);
EE_API int ee_kv_decode_attention(const ee_kv_cache* cache, const void* q, int64_t ldq, int64_t heads,
                                  const void* k_new, const void* v_new, int64_t ld_new, float scale, void* out,
                                  int64_t ldo, float* H, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- decoder-stack engine
 * The whole decoder stack of a Llama-architecture model for one fixed batch shape
 * [batch, seq] as one native object: the reference's Python layer loop
 * (EE/python/quality_eval.py:133-141 over EntropyDispatchedLlamaBlock.forward,
 * EE/python/dispatch.py:166-210; the C++ port its README lists as the next step) with
 * every step on the device and no host round trip, eagerly (ee_decoder_run) or as one
 * CUDA graph recorded once and replayed (ee_decoder_capture / ee_decoder_launch).
 * Per layer, on M = batch * seq rows of width hidden:
 *   x  = RMSNorm(h) (h = s_prev + mlp_prev folded into the norm pass, ee_add_rmsnorm)
 *   qkv = x W_qkv^T                  fp16 GEMM of the fp16 weights (route_all = 0) or
 *                                    gated GEMM routed by the previous layer's entropies
 *                                    (route_all = 1; the first layer's rows take FP16)
 *   o, H = flash attention with rotary embedding and row entropies
 *                                    (ee_flash_attention_rope_entropy, causal)
 *   Ht = mean over heads of H (per token), Hb = mean over heads and positions (per batch)
 *   a  = o W_o^T                     as qkv, routed by this layer's entropies
 *   s  = h + a, x2 = RMSNorm(s)      (one pass)
 *   routes: per token by Ht (routing 0), or every row in the tier of max_b Hb
 *           (routing 1, the reference dispatcher's batch-max rule, decided on the device)
 *   m  = gated SwiGLU GEMM (gate / up interleaved) of x2, then gated GEMM down
 *   h' = s + m                       (folded into the next layer's norm pass)
 * then hidden_out = RMSNorm_final(h_last) and residual_out (nullable) = h_last.  The
 * result equals running EntropyDispatchedLlamaBlock(attention="flash", routing=...,
 * route_all=...) layer by layer through the same kernels, bit for bit. */
typedef struct ee_decoder ee_decoder;

typedef struct ee_weight_pack {
  const int8_t* w_i8;      /* int8 [N, K] */
  const uint8_t* w_e4m3;   /* e4m3 codes [N, K] */
  const void* w_f16;       /* fp16 [N, K] */
  const float* scale;      /* fp32 [N] */
} ee_weight_pack;

typedef struct ee_decoder_layer {
  const void* input_norm;  /* fp16 [hidden] */
  const void* post_norm;   /* fp16 [hidden] */
  const void* qkv_f16;     /* route_all = 0: fp16 [(heads + 2 kv_heads) head_dim, hidden] (q, k, v rows) */
  const void* o_f16;       /* route_all = 0: fp16 [hidden, heads head_dim] */
  ee_weight_pack qkv;      /* route_all = 1: packs of the concatenated q / k / v weight */
  ee_weight_pack o;        /* route_all = 1 */
  ee_weight_pack gate_up;  /* gate and up interleaved in 128-row groups: N = 2 intermediate, K = hidden */
  ee_weight_pack down;     /* N = hidden, K = intermediate */
} ee_decoder_layer;

#define EE_ROUTE_TOKEN 0
#define EE_ROUTE_BATCH 1

typedef struct ee_decoder_config {
  int64_t batch, seq, hidden, heads, kv_heads, head_dim, intermediate;
  float rms_eps;           /* every RMSNorm of the stack */
  float attn_scale;        /* softmax scale (head_dim^-0.5 for Llama) */
  double tau_low, tau_high;
  int32_t routing;         /* EE_ROUTE_TOKEN or EE_ROUTE_BATCH */
  int32_t route_all;       /* 0: MLP only (the reference's mode), 1: q / k / v and o too */
  int32_t exact_entropy;   /* 1: route by the reference's entropy of fp16-rounded probabilities
                              (ee_flash_attention_rope_entropy_exact), 0: by the online entropy */
} ee_decoder_config;

EE_API size_t ee_decoder_workspace_bytes(const ee_decoder_config* cfg);
/* Copies the descriptions; the weights, final_norm (fp16 [hidden]), the rotary tables
 * cos / sin (fp16 [batch * seq, head_dim]) and layer_counts (nullable: device int32
 * [n_layers, 3], the MLP's INT8 / FP8 / FP16 row counts of every layer, written by each
 * forward) must outlive the engine.  workspace: 256-byte aligned, ee_decoder_workspace_bytes. */
EE_API int ee_decoder_create(const ee_decoder_config* cfg, int32_t n_layers, const ee_decoder_layer* layers,
                             const void* final_norm, const void* cos, const void* sin, int32_t* layer_counts,
                             void* workspace, size_t workspace_bytes, ee_decoder** out);
/* One forward: hidden_in fp16 [batch * seq, hidden] (read only) -> hidden_out fp16
 * [batch * seq, hidden] and residual_out (nullable, fp16, same shape), on `stream`. */
EE_API int ee_decoder_run(ee_decoder* dec, const void* hidden_in, void* hidden_out, void* residual_out, void* stream);
/* Records one forward over these buffers into a CUDA graph (stream: a created stream). */
EE_API int ee_decoder_capture(ee_decoder* dec, const void* hidden_in, void* hidden_out, void* residual_out,
                              void* stream);
/* Replays the recorded forward. */
EE_API int ee_decoder_launch(ee_decoder* dec, void* stream);
EE_API int ee_decoder_destroy(ee_decoder* dec);

#ifdef __cplusplus
}
#endif

#endif /* EE_B200_H_ */
