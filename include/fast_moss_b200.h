/*
 * fast_moss_b200.h -- C ABI of the B200 (sm_100a) kernels for the MOSS Audio
 * Tokenizer v2 data-parallel hot path.
 *
 * Conventions shared by every entry point:
 *   - All tensor pointers are DEVICE pointers owned by the caller; nothing is
 *     allocated inside a call and nothing is freed.
 *   - Sizes are int64_t element counts; strides are int64_t element strides.
 *   - `stream` is a cudaStream_t passed as void*; NULL means the legacy default
 *     stream.  Unless its declaration says otherwise, every call is
 *     stream-ordered, never synchronises the host and is therefore legal
 *     inside CUDA-graph capture.
 *   - Return value: MOSS_OK (0) on success, otherwise a status code below; a
 *     human-readable message for the calling thread is in moss_last_error().
 *     The Python host layer maps MOSS_ERR_VALUE -> ValueError and the others
 *     -> RuntimeError, the same exception classes the reference raises.
 *   - Calls on distinct streams are independent.  The only state shared
 *     between calls is read-only after its first use on a device: the SM
 *     count and the bf16 activation tables of moss_gated_act (also read by
 *     moss_linear's activation epilogue).  The tables
 *     are built by one kernel at the first moss_gated_act call on a device
 *     that is large enough to use them (2^22 outputs) and is not inside a
 *     stream capture; that call waits for the caller's stream once.  Calls
 *     captured before then use a kernel without the tables (same results).
 *
 * Dtype codes: MOSS_F32 = float32, MOSS_BF16 = bfloat16 (stored as uint16).
 *
 * Each declaration names the reference function (path within the reference
 * project, file:line) whose behaviour it reproduces.
 */
#ifndef FAST_MOSS_B200_H
#define FAST_MOSS_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define MOSS_API __attribute__((visibility("default")))
#else
#define MOSS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MOSS_OK 0
#define MOSS_ERR_VALUE 1       /* bad shape / dtype / stride / alignment  */
#define MOSS_ERR_UNSUPPORTED 2 /* valid input this kernel does not cover  */
#define MOSS_ERR_CUDA 3        /* kernel launch or device error           */
#define MOSS_ERR_TIMEOUT 4     /* a bounded device-side wait ran out      */

#define MOSS_F32 0
#define MOSS_BF16 1

#define MOSS_ACT_SILU 0
#define MOSS_ACT_GELU_ERF 1
#define MOSS_ACT_GELU_TANH 2

#define MOSS_LINEAR_BIAS 0      /* y = x w^T + bias                       */
#define MOSS_LINEAR_BIAS_ACT 1  /* y = act(bf16(x w^T) + bias), ungated   */

#define MOSS_RVQ_AUTO 0    /* tensor-core quantizer: the faster kernel (SINGLE)         */
#define MOSS_RVQ_SINGLE 1  /* one CTA per row block, the whole codebook each         */
#define MOSS_RVQ_PAIR 2    /* a CTA pair per row block, each half of the codebook     */

/* Library ABI version (major*100 + minor). */
MOSS_API int moss_version(void);

/* Message describing the last non-OK status returned on this host thread. */
MOSS_API const char* moss_last_error(void);

/* Reads and clears the device-side error word that bounded waits set when
 * they give up (MOSS_ERR_TIMEOUT).  Synchronises `stream`; not for use inside
 * graph capture. */
MOSS_API int moss_check_device_error(void* stream);

/* Self-test of the failure path -- no counterpart in the reference (its
 * kernels never wait on the device).  Runs one warp that waits on an
 * mbarrier through the same bounded wait every kernel here uses, with a
 * limit of limit_ns (1 us to 100 ms) instead of the kernels' ~2 s.  With
 * arrive != 0 the phase is completed first and nothing is recorded; with
 * arrive == 0 nothing completes it, the wait gives up after limit_ns,
 * records MOSS_ERR_TIMEOUT in the device error word (read and cleared by
 * moss_check_device_error) and the kernel returns: the context stays
 * usable.  Stream-ordered; for tests. */
MOSS_API int moss_test_bounded_wait(int64_t limit_ns, int arrive, void* stream);

/* ---------------------------------------------------------------------------
 * Residual update with per-channel layer scale.
 * Replaces fast_moss/v2_pointwise.py:92-122 (`_scale_add` / `scale_add`):
 *   y[i] = float(x[i]) + float(u[i]) * scale[i % c]
 * with the product and the sum rounded separately (no FMA), y float32.
 * x, u contiguous with n elements, scale contiguous [c], n % c == 0.
 * ------------------------------------------------------------------------- */
MOSS_API int moss_scale_add(const void* x, int x_dtype, const void* u, int u_dtype,
                   const float* scale, float* y, int64_t n, int64_t c,
                   void* stream);

/* ---------------------------------------------------------------------------
 * LayerNorm over the last dimension, float32, identical to the arithmetic of
 * PyTorch's CUDA vectorised layer-norm forward that the reference calls
 * through nn.LayerNorm (fast_moss/v2_runtime.py:259, type-checked at :330).
 * x [rows, n] contiguous, n % 4 == 0, gamma/beta [n] 16-byte aligned (NULL
 * gamma => 1, NULL beta => 0).  mean/rstd [rows] are optional (NULL = skip).
 * ------------------------------------------------------------------------- */
MOSS_API int moss_layer_norm(const float* x, const float* gamma, const float* beta,
                    float eps, int64_t rows, int64_t n, float* y, float* mean,
                    float* rstd, void* stream);

/* ---------------------------------------------------------------------------
 * Fused residual + layer scale + LayerNorm: one pass computes
 *   residual = x + u * scale          (as moss_scale_add)
 *   normed   = LayerNorm(residual)    (as moss_layer_norm)
 * Replaces the pair `scale_add(residual, update, scale)` followed by the next
 * `norm(x)` in the patched transformer layer (fast_moss/v2_runtime.py:254-276).
 * residual_out may be NULL when only the normalised output is needed.
 * ------------------------------------------------------------------------- */
MOSS_API int moss_residual_layer_norm(const void* x, int x_dtype, const void* u,
                             int u_dtype, const float* scale,
                             const float* gamma, const float* beta, float eps,
                             int64_t rows, int64_t n, float* residual_out,
                             float* normed_out, float* mean, float* rstd,
                             void* stream);

/* ---------------------------------------------------------------------------
 * moss_residual_layer_norm (u != NULL) or moss_layer_norm (u == NULL, x
 * float32) with the normalised output stored in normed_dtype: MOSS_F32, or
 * MOSS_BF16 rounded to nearest even -- the bits of the bf16 cast that the
 * patched layer's next Linear applies to norm(x) under autocast
 * (fast_moss/v2_runtime.py:104, :259), so the cast needs no kernel of its
 * own.  A bf16 normed_out must be 8-byte aligned.
 * ------------------------------------------------------------------------- */
MOSS_API int moss_residual_layer_norm_out(const void* x, int x_dtype, const void* u,
                             int u_dtype, const float* scale,
                             const float* gamma, const float* beta, float eps,
                             int64_t rows, int64_t n, float* residual_out,
                             void* normed_out, int normed_dtype, float* mean,
                             float* rstd, void* stream);

/* ---------------------------------------------------------------------------
 * Rotary embedding on q and k with caller-supplied tables.
 * Replaces fast_moss/v2_pointwise.py:50-89 (`_rotate` / `rotate`):
 *   o[2p]   = q[2p]*cos - q[2p+1]*sin
 *   o[2p+1] = q[2p]*sin + q[2p+1]*cos     (float32, no FMA)
 * q, k: [b,h,t,d] with arbitrary element strides (q_strides/k_strides: 4
 * int64 each, host memory); cos/sin: contiguous float32 [b,t,d/2];
 * oq/ok: contiguous [b,h,t,d] of the input dtype (MOSS_F32 or MOSS_BF16).
 * ------------------------------------------------------------------------- */
MOSS_API int moss_rotate(const void* q, const void* k, int dtype, const float* cos_t,
                const float* sin_t, void* oq, void* ok, int64_t b, int64_t h,
                int64_t t, int64_t d, const int64_t* q_strides,
                const int64_t* k_strides, void* stream);

/* ---------------------------------------------------------------------------
 * Rotary embedding with the phase tables computed inside the kernel.
 * Replaces the patched rotary forward fast_moss/v2_runtime.py:186-224:
 *   freq[j]  = expf(j * freq_coef)                 (freq_coef = float32 of
 *                                                   -ln(max_period)*2/d)
 *   ts       = float(offset[b]) + t
 *   phase    = freq[j] * ts ; cos = cosf(phase) ; sin = sinf(phase)
 * followed by the rotation of moss_rotate.  offset: device pointer to b
 * values of dtype offset_dtype (0 = int64, 1 = int32, 2 = float32).
 * ------------------------------------------------------------------------- */
MOSS_API int moss_rope(const void* q, const void* k, int dtype, const void* offset,
              int offset_dtype, float freq_coef, void* oq, void* ok, int64_t b,
              int64_t h, int64_t t, int64_t d, const int64_t* q_strides,
              const int64_t* k_strides, void* stream);

/* ---------------------------------------------------------------------------
 * moss_rope whose rotated keys, and the values, go straight into the
 * attention history instead of new tensors.  Replaces the patched rotary
 * forward (fast_moss/v2_runtime.py:186-224) followed by the streaming
 * attention's key/value cache update (the upstream state that
 * fast_moss/streaming.py:14-26 keeps at stable addresses): oq contiguous
 * [b,h,t,d]; k rotated into k_cache and v copied into v_cache at
 * [b, h, slots[b*t + t_i], :], both caches contiguous [b, h, cache_slots, d]
 * of the input dtype.  slots: device int64 [b, t]; a slot outside
 * [0, cache_slots) is skipped and reported through moss_check_device_error.
 * q, k, v: [b,h,t,d] with arbitrary element strides (4 int64 each, host).
 * ------------------------------------------------------------------------- */
MOSS_API int moss_rope_kv(const void* q, const void* k, const void* v, int dtype,
              const void* offset, int offset_dtype, float freq_coef,
              const int64_t* slots, void* oq, void* k_cache, void* v_cache,
              int64_t b, int64_t h, int64_t t, int64_t d, int64_t cache_slots,
              const int64_t* q_strides, const int64_t* k_strides,
              const int64_t* v_strides, void* stream);

/* ---------------------------------------------------------------------------
 * Fused qkv projection with the rotary embedding in its epilogue (bf16).
 * Replaces the cached bf16 Linear of the attention input
 * (fast_moss/v2_runtime.py:77-106, F.linear at :104) followed by the
 * patched rotary forward (fast_moss/v2_runtime.py:186-224) and the
 * streaming attention's key/value cache update, i.e. the Linear followed by
 * moss_rope_kv:
 *   y = bf16(x W^T + bias)   x [b*t, k] bf16 rows (row = b_i*t + t_i),
 *                            W [3*h*64, k] bf16, FP32 accumulation on the
 *                            tensor cores (tcgen05), one bf16 rounding
 *   q = y[:, :64h], k = y[:, 64h:128h], v = y[:, 128h:], heads of 64
 *   q, k rotated with the in-kernel phase of moss_rope (offset[b_i] + t_i)
 *   oq [b, h, t, 64]; k_cache / v_cache [b, h, cache_slots, 64] at slot
 *   slots[b_i*t + t_i] (a slot out of range is skipped and reported).
 * w_image: W pre-packed by the host into blocks of 32 rows x 64 columns in
 * the MMA's no-swizzle K-major core-matrix order ([3h*2][k/64][4][8][8][8]
 * bf16: row group, k core, row, element).  bias: [3*h*64] bf16 or NULL.
 * k must be a multiple of 64 and at most 1536; buffers 16-byte aligned.
 * The dot products are summed in this kernel's order, not cuBLAS's, so a
 * projection output can differ from F.linear's by the rounding of a
 * different sum.  Built for skinny inputs (one 32-row tile of tokens per
 * CTA, all operands resident): on B200 at 4 rows it takes about as long
 * as the cuBLAS GEMM + moss_rope_kv, and well above 32 rows it loses.
 * ------------------------------------------------------------------------- */
MOSS_API int moss_qkv_rope(const void* x, const void* w_image, const void* bias, int64_t b,
              int64_t t, int64_t h, int64_t k, const void* offset, int offset_dtype,
              float freq_coef, const int64_t* slots, void* oq, void* k_cache,
              void* v_cache, int64_t cache_slots, void* stream);

/* ---------------------------------------------------------------------------
 * Attention of a chunk's queries over a streaming history ring.
 * Replaces the SDPA call of the streaming layer's attention over its
 * bounded history (fast_moss/v2_runtime.py:40-41 validates SDPA,
 * :254-262 calls the attention block; fast_moss/streaming.py:68-79 keeps
 * the history bounded and at stable addresses).
 *   query t of stream s sits at position pos[s] + t; it attends to ring slot
 *   j iff 0 <= slot_pos[s, j] <= pos[s] + t and slot_pos[s, j] > pos[s] + t
 *   - context (slot_pos = -1 marks an empty slot);
 *   out[s, t, h] = sum_j softmax_j(scale * q[s, h, t] . k[s, h, j]) v[s, h, j]
 * q [s, h, t, 64] bf16 contiguous; k_cache, v_cache [s, h, n, 64] bf16
 * contiguous and 16-byte aligned; slot_pos int64 [s, n]; pos int64 [s];
 * out [s, t, h, 64] bf16 (the layout the output projection reads).
 * d must be 64, 1 <= t <= 8, 1 <= n <= 512.  FP32 arithmetic throughout,
 * one bf16 rounding, so results can differ from SDPA's (which rounds the
 * weights to bf16 before P.V) by a bf16 unit.  A query with no attended
 * slot gets NaN.
 * ------------------------------------------------------------------------- */
MOSS_API int moss_history_attention(const void* q, const void* k_cache, const void* v_cache,
              const int64_t* slot_pos, const int64_t* pos, int64_t s, int64_t h,
              int64_t t, int64_t n, int64_t d, int64_t context, float scale, void* out,
              void* stream);

/* ---------------------------------------------------------------------------
 * moss_rope_kv followed by moss_history_attention in one kernel: the
 * streaming layer's rotary forward (fast_moss/v2_runtime.py:186-224), the
 * history's key/value update (fast_moss/streaming.py:68-79) and the
 * attention over the history (fast_moss/v2_runtime.py:40-41, :254-262).
 *   qkv [s * t, 3 * h * 64] bf16, 16-byte aligned: the qkv projection's
 *     output (row s_i * t + t_i; q, k, v of every head of 64)
 *   slots int64 [s, t]: each token's ring slot; freq_coef: as moss_rope_kv
 *   pos int64 [s]: the chunk's first position, both the rotary offset and
 *     the queries' position
 * q and k are rotated exactly as moss_rope_kv does; the rotated keys and
 * the values are written into k_cache / v_cache at their slots (a slot out
 * of range is skipped and reported in the device error word) and the
 * attention is that of moss_history_attention on the rotated q: the same
 * bits as the two calls.  Covers the persistent kernel's range only (at
 * most 8 queries, rings of at most 256 slots, at least two (stream, head)
 * items per resident CTA: 2 x the SM count); MOSS_ERR_UNSUPPORTED otherwise.
 * ------------------------------------------------------------------------- */
MOSS_API int moss_history_attention_qkv(const void* qkv, const int64_t* slots, float freq_coef,
              void* k_cache, void* v_cache, const int64_t* slot_pos,
              const int64_t* pos, int64_t s, int64_t h, int64_t t, int64_t n,
              int64_t d, int64_t context, float scale, void* out, void* stream);

/* ---------------------------------------------------------------------------
 * Linear layer on cached bf16 weights, tcgen05 tensor cores, bias or bias +
 * activation in the epilogue.
 * Replaces the cached bf16 Linear of the patched model
 * (fast_moss/v2_runtime.py:77-106, F.linear at :104) and, with
 * MOSS_LINEAR_BIAS_ACT, the Linear followed by the feed-forward's
 * bias + activation (moss_gated_act, ungated):
 *   MOSS_LINEAR_BIAS      y = bf16(x w^T + bias)          (bias may be NULL)
 *   MOSS_LINEAR_BIAS_ACT  y = bf16(act(bf16(bf16(x w^T) + bias)))
 * x [m, k], bias [n], y [m, n]: bf16, row-major, 16-byte aligned; w_image:
 * the weight w [n, k] packed once by moss_linear_pack_weight (n * k bf16:
 * per 128-row tile and 64-column chunk a 16 KB block in the tensor cores'
 * 128-byte-swizzled K-major layout, a tile's chunks back to back); k a
 * multiple of 64, n of 128 (MOSS_ERR_UNSUPPORTED otherwise).  FP32
 * accumulation; K is split across the CTAs of a thread-block cluster
 * (moss_linear_cluster(m, n, k) CTAs) whose partial sums are added in a
 * fixed order, so results are deterministic but summed in another order
 * than cuBLAS's: an output can differ from F.linear's by the rounding of a
 * different FP32 sum.  The activation epilogue looks act(h) up in the
 * activation tables of moss_gated_act when they are built (same bits); like
 * there, the first such call on a device outside a stream capture builds
 * them and waits for the caller's stream once.
 * ------------------------------------------------------------------------- */
MOSS_API int moss_linear_pack_weight(const void* w, int64_t n, int64_t k, void* w_image,
                            void* stream);
MOSS_API int moss_linear(const void* x, int64_t m, int64_t k, const void* w_image, int64_t n,
                const void* bias, int epilogue, int act, void* y, void* stream);
MOSS_API int moss_linear_cluster(int64_t m, int64_t n, int64_t k);

/* ---------------------------------------------------------------------------
 * Bias + gated activation, bf16 or float32 in and out.
 * No kernel in the reference (its FFN activation is upstream model code);
 * this is the eager-PyTorch chain it replaces, one rounding per torch op:
 *   h = x + bias                      (rounded to dtype)
 *   gated:   y = act(h[:, :w]) * h[:, w:]   (each op rounded to dtype)
 *   ungated: y = act(h)
 * x [rows, width], bias [width] (or NULL), y [rows, width/2] if gated.
 * act: MOSS_ACT_SILU, MOSS_ACT_GELU_ERF, MOSS_ACT_GELU_TANH.
 * ------------------------------------------------------------------------- */
MOSS_API int moss_gated_act(const void* x, const void* bias, void* y, int dtype,
                   int64_t rows, int64_t width, int act, int gated,
                   void* stream);

/* ---------------------------------------------------------------------------
 * LFQ latent preparation for eight-channel latents x [b,8,t] (contiguous).
 * Replaces fast_moss/quantizer_prepare.py:111-157 (`prepare`, kernel source
 * :16-58): denom = max(sqrt(sum x^2), 1e-12) (NaN-propagating), e = x/denom,
 * twice = 2e, norm = sum e^2, with the reference's summation orders.
 * Layout of e/twice: [8,t] transposed (column j = row j) when b == 1 and
 * t > 1, else [b*t, 8].  norm, denom: [b*t].
 * ------------------------------------------------------------------------- */
MOSS_API int moss_lfq_prepare(const float* x, int64_t b, int64_t t, float* e,
                     float* norm, float* twice, float* denom, void* stream);

/* ---------------------------------------------------------------------------
 * Nearest-codeword selection from precomputed dot products.
 * Replaces fast_moss/quantizer.py:52-108 (`_select` / `select`):
 *   distance = (row_norm - dots) + code_norm ; the first NaN wins, otherwise
 *   the first minimum ; indices int64 ; out = codebook[index].
 * dots [b*t, k], row_norm [b*t], code_norm [k], codebook [k, d] contiguous;
 * latents [b,d,t] with strides latent_strides (3 int64, host) used only when
 * straight_through != 0, in which case out is [b,d,t] contiguous holding
 * latents + (codebook[index] - latents); otherwise out is [b*t, d].
 * ------------------------------------------------------------------------- */
MOSS_API int moss_lfq_select(const float* dots, const float* row_norm,
                    const float* code_norm, const float* codebook,
                    const float* latents, const int64_t* latent_strides,
                    int64_t b, int64_t d, int64_t t, int64_t k,
                    int straight_through, float* out, int64_t* indices,
                    void* stream);

/* ---------------------------------------------------------------------------
 * Fused LFQ decode: preparation + dot products + selection in one kernel,
 * no [b*t, k] dot-product matrix in HBM.
 * Replaces fast_moss/v2_runtime.py:143-181 (patched `decode_latents`).
 * x [b,8,t] contiguous float32; book_normed [k,8] (F.normalize of the
 * weight), code_norm [k] (sum of squares of book_normed rows), weight [k,8]
 * (raw codebook, gathered into the output).  Dots use a sequential FMA over
 * the 8 channels.  out [b*t, 8] (the reference returns its B,8,T transpose
 * view), indices int64 [b*t].
 * ------------------------------------------------------------------------- */
MOSS_API int moss_lfq_decode(const float* x, const float* book_normed,
                    const float* code_norm, const float* weight, int64_t b,
                    int64_t t, int64_t k, float* out, int64_t* indices,
                    void* stream);

/* ---------------------------------------------------------------------------
 * Multi-stage LFQ quantizer of the real codec, every stage in one kernel.
 * Replaces, per stage, the upstream quantizer's input projection, the
 * patched LFQ decode (fast_moss/v2_runtime.py:143-181: prepare,
 * fast_moss/quantizer_prepare.py:111-157; the FP32 dot-product GEMM; select,
 * fast_moss/quantizer.py:52-108), the output projection and the residual
 * update -- the stage loop the reference leaves to the upstream quantizer
 * (fast_moss/v2_codec.py:45).  Per frame (b, t), r = x[b, :, t], and for
 * every stage s:
 *   z_j = dot(w_in[s, j, :], r) + b_in[s, j]  (32 lane partial sums over
 *         d = l, l + 32, ..., sequential FMA from +0, then added pairwise
 *         across lanes 16, 8, 4, 2, 1 apart)
 *   index = the LFQ decode of z viewed as a [b, 8, t] latent (the
 *         reference's prepare orders, transposed when b == 1 and t > 1;
 *         dots = product + 7 FMAs; first NaN, else first minimum)
 *   o_d = (FMA chain over j of w_out[s, d, j] * weight[s, index, j] from
 *         +0) + b_out[s, d] ;  r_d -= o_d ;  codes[s, b * t + t_i] = index
 * x, residual_out [b, d, t] FP32 (residual_out may be NULL); w_in [s, 8, d],
 * b_in [s, 8], book_normed [s, k, 8] (F.normalize of the codebook weight),
 * code_norm [s, k] (sum of squares of book_normed rows), weight [s, k, 8]
 * (raw codebooks), w_out [s, d, 8], b_out [s, d]; book_normed and w_out
 * 16-byte aligned; codes int64 [s, b * t].  d <= 2048, k <= 65536.
 * ------------------------------------------------------------------------- */
MOSS_API int moss_lfq_rvq_encode(const float* x, int64_t b, int64_t d, int64_t t, int64_t stages,
                        int64_t k, const float* w_in, const float* b_in,
                        const float* book_normed, const float* code_norm,
                        const float* weight, const float* w_out, const float* b_out,
                        int64_t* codes, float* residual_out, void* stream);

/* ---------------------------------------------------------------------------
 * Codebook preparation for the multi-stage residual vector quantizer,
 * the analogue of the one-off codebook normalisation the reference performs
 * when its optimisation context is entered (fast_moss/v2_runtime.py:401-403).
 * books [stages, k, d] float32 contiguous.  Writes
 *   code_norm [stages, kpad]  sum_d c[d]^2 (sequential FMA; +inf for padding)
 *   packed    moss_rvq_packed_floats() floats: the k-major copy
 *             [stages, kpad/256, d, 256] read by moss_rvq_encode_ffma, then
 *             the 128-byte-swizzled 256-code tile images read by the
 *             tensor cores in moss_rvq_encode
 *   stats     [stages, 4]     {max code norm, non-finite flag, 0, 0}
 * with kpad = k rounded up to a multiple of 256.  Only d == 64 is supported.
 * ------------------------------------------------------------------------- */
MOSS_API int64_t moss_rvq_packed_floats(int64_t stages, int64_t k, int64_t d);
MOSS_API int moss_rvq_prepare_codebooks(const float* books, int64_t stages, int64_t k,
                               int64_t d, float* code_norm, float* packed,
                               float* stats, void* stream);

/* ---------------------------------------------------------------------------
 * Multi-stage residual vector quantizer, encode + decode in one kernel.
 * The stage loop the reference delegates to the upstream quantizer
 * (fast_moss/v2_codec.py:45), each stage with the selection rule of
 * fast_moss/quantizer.py:33-39: for every row r (residual kept on chip):
 *   norm = sum_d r[d]^2, dot_j = sum_d (2 r[d]) c_j[d]  (sequential FMA, d
 *   ascending), dist_j = (norm - dot_j) + code_norm_j, index = first NaN,
 *   else first minimum; r -= c_index; recon += c_index.
 * x [rows, d]; codes int32 [stages, rows]; recon [rows, d];
 * residual_out [rows, d] optional (NULL = skip); all 16-byte aligned.
 *
 * moss_rvq_encode screens the codes with TF32 tensor-core dot products
 * (tcgen05, accumulators in tensor memory) under a proven error margin and
 * resolves the surviving candidates with the exact arithmetic above, so its
 * codes equal those of moss_rvq_encode_ffma, which evaluates every distance
 * with FP32 FMAs.  k <= 4096 for the tensor-core path.
 * ------------------------------------------------------------------------- */
MOSS_API int moss_rvq_encode(const float* x, int64_t rows, int64_t d,
                    const float* books, const float* packed,
                    const float* code_norm, const float* stats,
                    int64_t stages, int64_t k, int32_t* codes, float* recon,
                    float* residual_out, void* stream);
/* moss_rvq_encode with the tensor-core kernel chosen (same results): MOSS_RVQ_AUTO
 * (what moss_rvq_encode does: the single-CTA kernel, measured faster at
 * 8192 rows x 32 stages x 1024 codes), MOSS_RVQ_SINGLE (one CTA holds its rows for the
 * whole codebook), MOSS_RVQ_PAIR (two CTAs of a cluster hold the same <= 128
 * rows and each screens half of every codebook; needs k > 256 and rows within
 * one wave of pairs, else MOSS_ERR_UNSUPPORTED).  Same reference row as
 * moss_rvq_encode (fast_moss/v2_codec.py:45 with fast_moss/quantizer.py:33-39). */
MOSS_API int moss_rvq_encode_kernel(const float* x, int64_t rows, int64_t d,
                    const float* books, const float* packed,
                    const float* code_norm, const float* stats,
                    int64_t stages, int64_t k, int32_t* codes, float* recon,
                    float* residual_out, int kernel, void* stream);
MOSS_API int moss_rvq_encode_ffma(const float* x, int64_t rows, int64_t d,
                    const float* books, const float* packed,
                    const float* code_norm, const float* stats,
                    int64_t stages, int64_t k, int32_t* codes, float* recon,
                    float* residual_out, void* stream);

/* ---------------------------------------------------------------------------
 * moss_rvq_encode_static -- no reference counterpart.  The quantizer of
 * moss_rvq_encode for callers that cannot allocate device memory (a host
 * binding that owns only its input and output buffers, or a process held to
 * a fixed device-memory budget): the prepared codebooks live in a static
 * device array of this library instead of caller buffers, and each call runs
 * moss_rvq_prepare_codebooks into it and then moss_rvq_encode, both on
 * `stream`.  Same arguments and results as moss_rvq_encode minus the
 * prepared buffers.
 *   - Capacity: at most 32 stages x 1024 codes, d == 64; other sizes return
 *     MOSS_ERR_UNSUPPORTED (bad shapes and null pointers MOSS_ERR_VALUE).
 *     The array takes 17,957,376 bytes of device memory on every device the
 *     library is used on.
 *   - Cost: every call prepares the codebooks again (two small kernels,
 *     one CTA per 256-code chunk and stage, then one per stage) before the
 *     encode; callers that quantize many batches against one codebook set
 *     and can allocate should prepare once and call moss_rvq_encode.
 *   - Nothing in the array has to start at zero: every call rewrites all of
 *     it that the encode reads.
 *   - The first call on each device looks up the array's address
 *     (cudaGetSymbolAddress) and keeps it for the life of the process (calls
 *     after cudaDeviceReset are not supported); make that first call before
 *     any stream capture on the device.
 *   - Calls that overlap in time on one device (other streams or host
 *     threads) race on the shared array; serialise them.
 * ------------------------------------------------------------------------- */
MOSS_API int moss_rvq_encode_static(const float* x, int64_t rows, int64_t d,
                    const float* books, int64_t stages, int64_t k,
                    int32_t* codes, float* recon, float* residual_out,
                    void* stream);

/* ---------------------------------------------------------------------------
 * Residual-VQ dequantisation: recon[r] = sum_s books[s][codes[s][r]] in
 * stage order (float32 adds starting from zero).  Codes outside [0, k) are
 * reported through the device error word and contribute nothing.
 * ------------------------------------------------------------------------- */
MOSS_API int moss_rvq_decode(const int32_t* codes, int64_t rows, const float* books,
                    int64_t stages, int64_t k, int64_t d, float* recon,
                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FAST_MOSS_B200_H */
