/*
 * b200moe — C ABI of the B200 (sm_100a) Qwen3-MoE expert layer.
 *
 * Drop-in kernels for the MoE path of spark-gpt's train.py.  Every entry
 * point takes raw device pointers, plain sizes and a CUDA stream
 * (cudaStream_t passed as void*), enqueues its kernels on that stream and
 * returns 0 on success or a positive error code; b200moe_last_error() gives
 * the message of the calling thread's last failure.  No entry point allocates
 * device memory: outputs and the scratch areas sized by the *_scratch_bytes
 * helpers belong to the caller.
 *
 * Tensors are row-major and contiguous unless a leading dimension is given.
 * "bf16" buffers hold IEEE bfloat16 values.  Shapes: T tokens, H hidden, E
 * experts, k top-k, I moe_intermediate, R = T*k routed slots, Rcap =
 * b200moe_padded_rows(R, E) padded routed rows (each expert's block of rows is
 * padded with zero rows to a multiple of 128).
 *
 * Shape limits of the GPU path: H % 128 == 0, I % 64 == 0, E <= 256,
 * k <= 16, 1 <= k <= E.
 */
#ifndef B200MOE_H_
#define B200MOE_H_

#ifdef __cplusplus
extern "C" {
#endif

#define B200MOE_OK 0
#define B200MOE_ERR_INVALID_ARG 1
#define B200MOE_ERR_CUDA 2
#define B200MOE_ERR_UNSUPPORTED 3

/* Library version (major*10000 + minor*100 + patch). */
int b200moe_version(void);

/* Expert GEMMs run as two-CTA (cta_group::2) 256-row pair tiles when the
 * shape allows (default 1); 0 selects the single-CTA 128-row kernel.  Both
 * give identical results.  Returns the previous setting; process-wide. */
int b200moe_set_pair_gemm(int enable);

/* Grids of the persistent kernels (expert and router GEMMs, the row
 * reductions of combine / gather backward) span at most `sms` SMs (0 = all,
 * the default), leaving the rest to kernels that run beside them on other
 * streams, such as the NCCL all-to-all of the expert-parallel layer: every
 * CTA of a persistent grid is then resident at once and no statically
 * scheduled tile waits for the collective to finish.  Results do not depend
 * on it.  Returns the previous setting; process-wide. */
int b200moe_set_persistent_sm_limit(int sms);

/* The peer-memory transfer kernels (b200moe_ep_p2p_send / _send_part,
 * b200moe_ep_p2p_reduce_return / _src) launch at most 8 blocks per SM of
 * `sms` SMs (0 = a grid over every SM, the default): for a transfer on a copy
 * stream beside the compute stream, whose kernels then keep the other SMs
 * instead of waiting for the transfer's blocks.  Results do not depend on
 * it.  Returns the previous setting; process-wide. */
int b200moe_set_transfer_sm_limit(int sms);

/* Message of this thread's last failed call ("" if none). */
const char* b200moe_last_error(void);

/* Reads and clears the device fault word of the current device (synchronous).
 * Bits: 1 = a bounded wait gave up, 2 = an expert id outside [0, E),
 * 4 = inconsistent sizes.  Kernels never trap; they record and return. */
int b200moe_fault_read_and_clear(unsigned int* fault);

/* Enqueues on `stream` an asynchronous copy of the device fault word into
 * *dst (pinned host memory, or device memory); nothing is cleared and the
 * host is not synchronised.  The layer ends every call with one, and checks
 * the copy at its next call.  Replaces the reference's only failure signal on
 * this path, a collective that times out (train.py:3561-3562, :3655). */
int b200moe_fault_snapshot(unsigned int* dst, void* stream);

/* Rows of the padded routed-row buffers: R + E*127 rounded up to 128. */
long long b200moe_padded_rows(long long routed_rows, int num_experts);

/* Router logits width used on the device: E rounded up to 64, 128 or 256. */
int b200moe_router_width(int num_experts);

/* fp32 master -> bf16 compute copy (the `.to(bfloat16)` of the expert and
 * router weights, train.py:2306, :2309 and autocast's F.linear at :2145).
 * dst has rows_out >= rows_in rows of `cols`; rows >= rows_in are zeroed.
 * rows_out*cols must be a multiple of 4. */
int b200moe_cast_f32_to_bf16(const float* src, long long rows_in, long long cols,
                             long long rows_out, void* dst_bf16, void* stream);

/* ---- router: TopKRouter.forward / backward (train.py:2134-2158) ---------- */

/* logits (T, W) bf16 = x (T,H) bf16 . w_router (W,H) bf16 ^T, W = router width
 * (rows >= E of w_router are zero).  Replaces F.linear at train.py:2145. */
int b200moe_router_logits(const void* x, const void* w_router, long long T, int H, int W,
                          void* logits, void* stream);

/* fp32 softmax over the first E of `ld` logit columns, top-k (probability
 * desc, lower index first on ties), optional renormalisation.  logits are
 * bf16 (logits_f32 = 0) or fp32 (1).  selected (T,k) int64, weights (T,k)
 * bf16.  Replaces train.py:2146-2157. */
int b200moe_router_topk_fwd(const void* logits, int logits_f32, long long ld, long long T,
                            int E, int k, int norm_topk_prob, long long* selected,
                            void* weights, void* stream);

/* d logits (T, ld) bf16 from d(routing weights) (T,k) fp32, plus an optional
 * extra bf16 logit gradient d_extra (T, ld) (the load-balancing loss); columns
 * >= E are written as zero.  Backward of train.py:2146-2157. */
int b200moe_router_topk_bwd(const void* logits, long long ld, const long long* selected,
                            const float* d_weights, const void* d_extra, long long T, int E,
                            int k, int norm_topk_prob, void* d_logits, void* stream);

/* dx (T,H) bf16 = d_logits (T,W) bf16 . w_router (W,H) bf16.  Backward of
 * F.linear at train.py:2145 w.r.t. its input. */
int b200moe_router_dgrad(const void* d_logits, const void* w_router, long long T, int H, int W,
                         void* dx, void* stream);

/* Bytes of scratch b200moe_router_wgrad needs (per-split fp32 partials). */
long long b200moe_router_wgrad_scratch_bytes(long long T, int H, int E);

/* dw_router (E,H) fp32 (+)= d_logits[:, :E]^T . x, split over the T rows into
 * per-split partials in `scratch` and summed in a fixed order (deterministic).
 * Backward of F.linear at train.py:2145 w.r.t. the router weight. */
int b200moe_router_wgrad(const void* x, const void* d_logits, long long T, int H, int E, int W,
                         float* dw_router, int accumulate, void* scratch,
                         long long scratch_bytes, void* stream);

/* ---- dispatch: Experts.forward sort / histc / cumsum (train.py:2271-2290) - */

long long b200moe_dispatch_scratch_bytes(long long T, int k, int E);

/* Stable counting sort of the flat expert ids selected (T,k) int64.
 *   counts (E) int32         rows per expert (histc, train.py:2283)
 *   offsets (E) int32        inclusive cumulative counts (train.py:2289)
 *   pad_offsets (E+1) int32  first padded row of each expert; [E] = total
 *   row_flat (Rcap) int32    padded row -> flat slot t*k+s, -1 for padding
 *   inv_pad (R) int32        flat slot -> padded row
 *   tile_expert (Rcap/128)   expert of each 128-row tile
 * Inside an expert, rows keep flat-slot order (= torch.sort(stable=True)).
 * A negative id marks a slot that goes to no expert: it gets no row and
 * inv_pad = -1; the gather, combine and gather-backward entry points skip such
 * slots (the combine backward gives them d_weights = 0).  Ids >= E set fault
 * bit 2. */
int b200moe_dispatch(const long long* selected, long long T, int k, int E, int* counts,
                     int* offsets, int* pad_offsets, int* row_flat, int* inv_pad,
                     int* tile_expert, void* scratch, long long scratch_bytes, void* stream);

/* b200moe_dispatch without caller scratch; it has no counterpart in the reference.
 * For callers that hold only the input and output buffers and cannot allocate device
 * memory: a host runtime bound through FFI that owns a fixed device arena and has no
 * caching allocator, or code that must not call cudaMalloc/cudaFree because those can
 * synchronize the device or fail under memory pressure in the middle of a step.  Outputs
 * are identical to b200moe_dispatch's.  The per-chunk counts go to a 1 MiB array built into
 * the library (held on every GPU that loads it until exit), so ceil(T*k/4096) * E must be
 * <= 262144 (e.g. T*k <= 16.7M slots at E = 64, <= 4.19M at E = 256); larger sizes are
 * rejected with B200MOE_ERR_INVALID_ARG.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress); make that first call before any stream capture.
 * The address is kept per device ordinal until the process exits, so resetting a device
 * (cudaDeviceReset, or releasing and re-creating its primary context) after that first
 * call is not supported: the next call would write through the old context's address.
 * All calls share the array: calls that overlap on the GPU (different streams, or different
 * host threads, without ordering between them) race and give wrong results.  No call
 * allocates or frees device memory. */
int b200moe_dispatch_noalloc(const long long* selected, long long T, int k, int E, int* counts,
                             int* offsets, int* pad_offsets, int* row_flat, int* inv_pad,
                             int* tile_expert, void* stream);

/* ---- gather: _GatherTopK (train.py:2195-2217) ---------------------------- */

/* xs (Rcap,H) bf16: xs[p] = x[row_flat[p]/k], zero rows for padding.  With
 * inv_pad (T*k, from dispatch) the copy runs in token order (each of the T x
 * rows read once, written to its k rows; k <= 32); with inv_pad == NULL, in
 * padded-row order (T unused). */
int b200moe_gather_rows(const void* x, const int* row_flat, const int* inv_pad,
                        const int* pad_offsets, long long T, int E, int k, int H,
                        long long rows_cap, void* xs, void* stream);

/* dx (T,H) bf16 = sum_s dxs[inv_pad[t*k+s]] (+ addend (T,H) bf16 if given).
 * With inv_pad == NULL, dxs is token-major: slot t*k+s in row t*k+s.
 * partial = 1 when some slots have no row (inv_pad -1, skipped); with
 * partial = 0 every inv_pad entry must be a row. */
int b200moe_gather_rows_bwd(const void* dxs, const int* inv_pad, const void* addend, long long T,
                            int k, int H, int partial, void* dx, void* stream);

/* ---- post-attention RMSNorm folded into the layer ------------------------ */
/* Replaces the block's RMSNorm (train.py:162-170) applied to the layer's input
 * (Block.forward, train.py:2370).
 *
 * x_n (T,H) bf16 = bf16(bf16(x * r) * bf16(w)), r = rsqrt(sum(x^2) * (1/H) + eps)
 * per token, written to rstd (T) fp32; x bf16, w (H) fp32.  H % 8 == 0. */
int b200moe_rmsnorm_fwd(const void* x, const float* w, long long T, int H, float eps, void* x_n,
                        float* rstd, void* stream);

/* Scratch of b200moe_gather_rows_bwd_rmsnorm: per-block partial rows of the
 * norm weight's gradient. */
long long b200moe_gather_rows_bwd_rmsnorm_scratch_bytes(long long T, int H);

/* b200moe_gather_rows_bwd with the RMSNorm backward folded in: with
 * g = bf16(sum_s dxs[inv_pad[t*k+s]] + addend[t]) (the norm output's gradient,
 * not written), dx (T,H) bf16 = the norm input's gradient
 * bf16(r * dy - (r^3/H) * x * <dy, x>), dy = bf16(g * bf16(w)), and dw (H) fp32
 * = sum_t g * bf16(x * r) (deterministic order).  x, w, rstd as given to and
 * returned by b200moe_rmsnorm_fwd.  Needs H % 32 == 0, H <= 4096 and
 * H * k <= 18432 (the shared-memory row ring); other shapes return
 * B200MOE_ERR_UNSUPPORTED. */
int b200moe_gather_rows_bwd_rmsnorm(const void* dxs, const int* inv_pad, const void* addend,
                                    const void* x, const float* w, const float* rstd, long long T,
                                    int k, int H, int partial, void* dx, float* dw, void* scratch,
                                    long long scratch_bytes, void* stream);

/* ---- combine: _CombineTopK (train.py:2220-2241) -------------------------- */

/* out (T,H) bf16 = sum_s bf16(y[inv_pad[t*k+s]] * weights[t,s]).  With
 * inv_pad == NULL, y is token-major: slot t*k+s in row t*k+s.  partial as in
 * b200moe_gather_rows_bwd. */
int b200moe_combine_fwd(const void* y, const int* inv_pad, const void* weights, long long T,
                        int k, int H, int partial, void* out, void* stream);

/* dy (Rcap,H) bf16 = bf16(d_out[t] * w), zero for padding rows;
 * d_weights (T*k) fp32 = <d_out[t], y[row of slot]> in flat-slot order.
 * y is in padded-row order (y_token_major = 0: row p holds slot row_flat[p])
 * or token-major (1: row t*k+s holds slot t*k+s; inv_pad required). */
int b200moe_combine_bwd(const void* d_out, const void* y, const int* row_flat,
                        const int* inv_pad, const int* pad_offsets, const void* weights, int E,
                        long long T, int k, int H, long long rows_cap, int y_token_major,
                        void* dy, float* d_weights, void* stream);

/* ---- expert products: _FusedSwiGLU / _GroupedLinear (train.py:1625-2090) - */

/* gu (Rcap,2I) bf16 = xs . W_gu[e]^T per expert; h (Rcap,I) bf16 =
 * silu(g)*u from the bf16-rounded g,u.  w_gate_up (E,2I,H) bf16.
 * Replaces _swiglu_gemm (train.py:1719). */
int b200moe_expert_gate_up_fwd(const void* xs, const void* w_gate_up, const int* tile_expert,
                               const int* pad_offsets, long long rows_cap, int E, int H, int I,
                               void* gu, void* h, void* stream);

/* y = h . W_d[e]^T per expert; w_down (E,H,I) bf16.  row_flat_out NULL: y is
 * (Rcap,H) in padded-row order; else padded row p is written to row
 * row_flat_out[p] of a token-major (T*k,H) y and padding rows are skipped.
 * Replaces _grouped_gemm (train.py:1803) in _GroupedLinear.forward. */
int b200moe_expert_down_fwd(const void* h, const void* w_down, const int* tile_expert,
                            const int* pad_offsets, const int* row_flat_out, long long rows_cap,
                            int E, int H, int I, void* y, void* stream);

/* dh = dy . W_d[e] (rounded to bf16), then the SwiGLU backward in the
 * epilogue: d_gu (Rcap,2I) bf16 = [dh*u*s*(1+g*(1-s)), dh*g*s], s = sigmoid(g).
 * Replaces _grouped_gemm(transpose_w) (train.py:1894) + _swiglu_tiles (:1899). */
int b200moe_expert_down_dgrad_swiglu(const void* dy, const void* w_down, const void* gu,
                                     const int* tile_expert, const int* pad_offsets,
                                     long long rows_cap, int E, int H, int I, void* d_gu,
                                     void* stream);

/* dxs = d_gu . W_gu[e] per expert, (Rcap,H) padded order, or token-major
 * (T*k,H) when row_flat_out is given (as b200moe_expert_down_fwd).  Replaces
 * _swiglu_dgrad (train.py:2029). */
int b200moe_expert_gate_up_dgrad(const void* d_gu, const void* w_gate_up, const int* tile_expert,
                                 const int* pad_offsets, const int* row_flat_out,
                                 long long rows_cap, int E, int H, int I, void* dxs,
                                 void* stream);

/* dw (E,M,N) fp32 (+)= a_e^T . b_e over the padded rows of expert e;
 * a (Rcap,M) bf16, b (Rcap,N) bf16, M % 128 == 0, N % 64 == 0.  Replaces
 * _grouped_wgrad (train.py:1863) and _swiglu_wgrad (:2047). */
int b200moe_expert_wgrad(const void* a, int M, const void* b, int N, const int* pad_offsets,
                         int E, long long rows_cap, float* dw, int accumulate, void* stream);

/* The same weight gradient when each expert's rows lie in several row
 * segments of one (rows_total, M) / (rows_total, N) allocation: seg_offsets
 * is (segments, E+1) int32 of absolute row offsets, and expert e's K rows are
 * the union over s of [seg_offsets[s][e], seg_offsets[s][e+1]) (each a
 * multiple of 128 rows long), in segment order.  The expert-parallel layer's
 * per-source chunks use it for one weight gradient over all of them (no
 * accumulation pass per chunk); the reference computes the same product per
 * expert over one contiguous block (_grouped_wgrad, train.py:1863).
 * M % 128 == 0, N % 64 == 0, 1 <= segments <= 64.  Shapes the two-CTA tiles
 * do not take (N < 128, an odd number of 128-row M tiles, E > 256) run one
 * b200moe_expert_wgrad per segment, adding into dw after the first. */
int b200moe_expert_wgrad_segments(const void* a, int M, const void* b, int N,
                                  const int* seg_offsets, int segments, int E,
                                  long long rows_total, float* dw, int accumulate, void* stream);

/* ---- the fp8 expert path: _FP8Experts (train.py:1543-1604) --------------
 * spark-gpt's --fp8-mlp on MoE layers.  x, gu, h and the expert weights are
 * e4m3, d_gu and the rows' gradient dy e5m2.  `scale` points at the layer's
 * five delayed per-site scales (x, gu, h, d_gu, dy: the Experts module's
 * fp8_scale buffer) and `amax` at its five amax slots (fp8_amax), which the
 * kernels raise with the absolute maxima of the unquantized values
 * (train.py:914-946).  Quantization is clamp(v * scale) with a round to
 * nearest even; every dequantization divides by powers of two.  Shapes:
 * H % 256 == 0, I % 128 == 0, E <= 256; fp8 buffers are one byte per element
 * in the padded expert-order row layout of b200moe_dispatch. */

long long b200moe_fp8_quantize_experts_scratch_bytes(int E);

/* Per-expert e4m3 copies of fp32 master weights w (E, per_expert):
 * q[e] = 2^floor(log2(448 / max|w_e|)), w8 = e4m3(w * q[e]).  Replaces
 * _fp8_quantize_experts (train.py:1536-1540). */
int b200moe_fp8_quantize_experts(const float* w, int E, long long per_expert, void* w8, float* q,
                                 void* scratch, long long scratch_bytes, void* stream);

/* x8 (Rcap,H) e4m3 = e4m3(x[token] * scale[0]) in padded expert order,
 * padding rows zero; amax[0] raised.  Replaces _fp8_moe_gather_quant_kernel
 * (train.py:1301-1313). */
int b200moe_fp8_gather_quant(const void* x, const int* row_flat, const int* inv_pad,
                             const int* pad_offsets, long long T, int E, int k, int H,
                             long long rows_cap, const float* scale, float* amax, void* x8,
                             void* stream);

/* dst (rows,cols) fp8 = fp8(src * scale[0]) for a bf16 src, amax[0] raised;
 * fmt 0 = e4m3, 1 = e5m2.  total_rows (device int, or NULL for all rows)
 * limits the rows read and written: the padded total pad_offsets[E] of a
 * padded-row buffer, whose spare rows hold no data.  The e5m2 copy of the
 * rows' gradient that the down weight gradient reads (the in-register
 * quantization of _fp8_moe_wgrad_rows_kernel, train.py:1504-1530). */
int b200moe_fp8_quantize_rows(const void* src, long long rows, int cols, const int* total_rows,
                              const float* scale, float* amax, int fmt, void* dst, void* stream);

/* b200moe_combine_bwd (padded-row y) that also writes dy8 (Rcap,H) e5m2 =
 * e5m2(dy * scale_dy[0]), padding rows zero, and raises amax_dy[0] with
 * max|dy|: the combine backward of _CombineTopK (train.py:2235-2241) fused
 * with the e5m2 quantization of its rows that _fp8_moe_wgrad_rows_kernel does
 * in registers (train.py:1504-1530), so dy is not read a second time.  Pass
 * scale + 4 and amax + 4 of the layer's five slots. */
int b200moe_fp8_combine_bwd(const void* d_out, const void* y, const int* row_flat,
                            const int* inv_pad, const int* pad_offsets, const void* weights,
                            int E, long long T, int k, int H, long long rows_cap,
                            const float* scale_dy, float* amax_dy, void* dy, float* d_weights,
                            void* dy8, void* stream);

/* gu = x8 . W8_gu[e]^T / (scale[0] q_gu[e]) rounded to bf16, h = silu(g) u;
 * gu8 (Rcap,2I), h8 (Rcap,I) e4m3 with scale[1], scale[2]; amax[1], amax[2]
 * raised.  Replaces _fp8_moe_swiglu_fwd_kernel (train.py:1317-1354). */
int b200moe_fp8_expert_gate_up_fwd(const void* x8, const void* w8_gate_up, const float* q_gu,
                                   const int* tile_expert, const int* pad_offsets,
                                   long long rows_cap, int E, int H, int I, const float* scale,
                                   float* amax, void* gu8, void* h8, void* stream);

/* y (Rcap,H) bf16 = h8 . W8_d[e]^T / (scale[2] q_d[e]).  Replaces
 * _fp8_moe_down_fwd_kernel (train.py:1357-1379). */
int b200moe_fp8_expert_down_fwd(const void* h8, const void* w8_down, const float* q_d,
                                const int* tile_expert, const int* pad_offsets, long long rows_cap,
                                int E, int H, int I, const float* scale, void* y, void* stream);

/* dh = bf16(dy . W_d[e]) (bf16 operands); g, u = gu8 / scale[1]; the SwiGLU
 * backward; d_gu8 (Rcap,2I) e5m2 with scale[3]; amax[3] raised.  Replaces
 * _fp8_moe_down_dgrad_swiglu_kernel (train.py:1382-1423); the dy amax it
 * records comes from b200moe_fp8_quantize_rows. */
int b200moe_fp8_expert_down_dgrad_swiglu(const void* dy, const void* w_down, const void* gu8,
                                         const int* tile_expert, const int* pad_offsets,
                                         long long rows_cap, int E, int H, int I,
                                         const float* scale, float* amax, void* d_gu8,
                                         void* stream);

/* dxs (Rcap,H) bf16 = d_gu8 . W8_gu[e] / (scale[3] q_gu[e]).  Replaces
 * _fp8_moe_dgrad_kernel (train.py:1426-1448). */
int b200moe_fp8_expert_gate_up_dgrad(const void* d_gu8, const void* w8_gate_up, const float* q_gu,
                                     const int* tile_expert, const int* pad_offsets,
                                     long long rows_cap, int E, int H, int I, const float* scale,
                                     void* dxs, void* stream);

/* dw (E,M,N) fp32 (+)= a8_e^T . b8_e / (scale_a[0] scale_b[0]) over the padded
 * rows of expert e; a8 (Rcap,M) e4m3 (a_fmt 0) or e5m2 (1), b8 (Rcap,N) e4m3;
 * M % 256 == 0, N % 128 == 0.  Replaces _fp8_moe_wgrad_kernel (train.py:1451-1478)
 * and _fp8_moe_wgrad_rows_kernel (:1504-1530). */
int b200moe_fp8_expert_wgrad(const void* a8, int a_fmt, int M, const void* b8, int N,
                             const int* pad_offsets, int E, long long rows_cap,
                             const float* scale_a, const float* scale_b, float* dw, int accumulate,
                             void* stream);

/* ---- expert products with the row gather / combine backward fused in ----
 * These read token-major tensors (x, d_out) row by row with TMA tile::gather4
 * in the GEMM's load stage, so the gathered (Rcap,H) copies of the reference's
 * _GatherTopK forward and _CombineTopK backward (train.py:2206, :2237-2239) are
 * never written.  Padding rows read as zero. */

/* gate_up fwd with xs[p] = x[row_flat[p]/k] gathered on the fly (x (T,H) bf16).
 * Replaces _GatherTopK.forward + _swiglu_gemm (train.py:2301-2306). */
int b200moe_expert_gate_up_fwd_gather(const void* x, const int* row_flat, long long T, int k,
                                      const void* w_gate_up, const int* tile_expert,
                                      const int* pad_offsets, long long rows_cap, int E, int H,
                                      int I, void* gu, void* h, void* stream);

long long b200moe_down_dgrad_combine_scratch_bytes(long long rows_cap, int I);

/* Combine backward + down dgrad + SwiGLU backward.  With d_out (T,H) gathered per
 * row and w = weights[row_flat[p]] (bf16, flat slot order): acc = d_out[t] . W_d[e];
 * dh = bf16(w*acc); d_gu (Rcap,2I) as in b200moe_expert_down_dgrad_swiglu;
 * hw (Rcap,I) = bf16(w*h) (the down weight-gradient operand);
 * d_weights (T*k) fp32 = <acc, h[p]> = <d_out[t], y[p]> (the routing-weight
 * gradient).  Replaces _CombineTopK.backward (train.py:2235-2241) +
 * _grouped_gemm(transpose_w) (:1894) + _swiglu_tiles (:1899). */
int b200moe_expert_down_dgrad_combine(const void* d_out, const int* row_flat, const void* weights,
                                      long long T, int k, const void* w_down, const void* gu,
                                      const void* h, const int* tile_expert,
                                      const int* pad_offsets, long long rows_cap, int E, int H,
                                      int I, void* d_gu, void* hw, float* d_weights,
                                      void* scratch, long long scratch_bytes, void* stream);

/* dw (E,M,N) fp32 (+)= a_e^T . x[tokens of expert e]: a (Rcap,M) bf16, x (T,N)
 * bf16 gathered per row.  Replaces _swiglu_wgrad (train.py:2047) on xs. */
int b200moe_expert_wgrad_gather_b(const void* a, int M, const void* x, int N, const int* row_flat,
                                  long long T, int k, const int* pad_offsets, int E,
                                  long long rows_cap, float* dw, int accumulate, void* stream);

/* dw (E,M,N) fp32 (+)= src[tokens of expert e]^T . b_e: src (T,M) bf16 gathered
 * per row, b (Rcap,N) bf16.  With src = d_out and b = hw this is the down
 * weight gradient dy^T h of _grouped_wgrad (train.py:1863). */
int b200moe_expert_wgrad_gather_a(const void* src, int M, const int* row_flat, long long T, int k,
                                  const void* b, int N, const int* pad_offsets, int E,
                                  long long rows_cap, float* dw, int accumulate, void* stream);

/* ---- expert parallel: experts sharded over P ranks -----------------------
 * The reference trains data-parallel only (experts replicated; Experts.forward,
 * train.py:2262-2322, runs every expert on every rank).  These entry points
 * serve the expert-parallel layout of the same layer: rank r owns experts
 * [r*Er, (r+1)*Er), Er = experts_per_rank; each token travels once to every
 * rank that owns one of its k experts, as one row with k packed slot words
 * (uint32: bf16 routing-weight bits << 16 | local expert id, or 0xFFFF in the
 * low half when the slot's expert lives elsewhere).  The rows cross the fabric
 * with NCCL all-to-all; the owner runs its experts on the received rows as a
 * k-slot layer whose foreign slots are skipped. */

/* dest (T,P) int64: dest[t*P+r] = r if token t selected an expert of rank r,
 * else -1; b200moe_dispatch(dest, T, P, P, ...) then gives the send layout
 * (rank-major, token order within a rank, 128-row padded blocks).
 * slot_counts (P) int32 = routed slots per destination rank (set here). */
int b200moe_ep_route(const long long* selected, long long T, int k, int experts_per_rank,
                     int ranks, long long* dest, int* slot_counts, void* stream);

/* meta (rows_cap, k) uint32 slot words of the send rows p < pad_offsets[P]
 * (row_flat/pad_offsets from the dispatch of dest); padding rows get 0xFFFF
 * words.  weights (T,k) bf16 routing weights. */
int b200moe_ep_pack(const long long* selected, const void* weights, const int* row_flat,
                    const int* pad_offsets, long long rows_cap, int k, int experts_per_rank,
                    int ranks, unsigned int* meta, void* stream);

/* Owner side: meta (rows, k) -> selected_local (rows, k) int64 local expert ids
 * (-1 for foreign slots) and weights_local (rows, k) bf16 (0 for foreign slots). */
int b200moe_ep_unpack(const unsigned int* meta, long long rows, int k, long long* selected_local,
                      void* weights_local, void* stream);

/* Source side: d_weights (T,k) fp32 of the routing weights from the owners'
 * per-row slot gradients dw_rows (send rows, k) fp32 (returned in the send
 * layout): d_weights[t*k+s] = dw_rows[inv_send[t*P + sel[t,s]/Er]*k + s];
 * inv_send (T*P) is the inv_pad of the dispatch of dest. */
int b200moe_ep_weight_grad(const float* dw_rows, const int* inv_send, const long long* selected,
                           long long T, int k, int experts_per_rank, int ranks, float* d_weights,
                           void* stream);

/* ---- expert parallel over peer memory (NVLink / NVSwitch) ---------------
 * The exchange of the expert-parallel layer without a collective library:
 * rows are stored by these kernels straight into buffers of the other ranks
 * that every rank has mapped (symmetric memory), and a bounded barrier over
 * flag words in that memory orders the phases.  Per rank the mapped buffers are
 * recv rows (P*T_cap, H) bf16 + recv meta (P*T_cap, k) uint32 (rows sent to
 * this rank's experts) and back rows (P*T_cap, H) bf16 + back dw (P*T_cap, k)
 * fp32 (results returned to this rank).  counts (P, ld) int32: row s = the
 * unpadded rows rank s sends to each rank (gathered on every rank).  No
 * counterpart in the reference, which is data-parallel only. */

/* plan (2 + 4P ints) of this rank from the gathered counts: [0] rows received,
 * [1, 1+P) where this rank's rows start at each owner, [1+P, 2+2P) where each
 * source's rows start here (P+1 entries), [2+2P, 2+3P) where this rank's
 * results for each source start in that source's back rows, [2+3P, 2+4P) where
 * each owner's results start in this rank's back rows. */
int b200moe_ep_p2p_plan(const int* counts, int ld, int me, int ranks, int* plan, void* stream);

/* Source side: each token's row src[t] (T,H) bf16 is stored into the recv rows
 * of every rank it selected (peer_rows[r] = rank r's recv rows, mapped here),
 * at the row given by the send layout (inv_send (T*P), send_pad_offsets (P+1)
 * from the dispatch of b200moe_ep_route's dest) and the plan; with selected
 * (T,k) and weights (T,k) bf16, its k slot words go to peer_meta[r] likewise
 * (selected == NULL: rows only).  ranks <= 32. */
int b200moe_ep_p2p_send(const void* src, const int* inv_send, const int* send_pad_offsets,
                        const int* plan, void* const* peer_rows, long long T, int H, int ranks,
                        const long long* selected, const void* weights, int k,
                        int experts_per_rank, unsigned int* const* peer_meta, void* stream);

/* Owner side: the first plan[0] rows of rows (rows_cap, H) bf16 (and of dw_rows
 * (rows_cap, k) fp32 if given) are stored into the back rows (back dw) of the
 * ranks they came from, at the rows the plan gives. */
int b200moe_ep_p2p_return(const void* rows, const float* dw_rows, const int* plan,
                          void* const* peer_rows, float* const* peer_dw, long long rows_cap,
                          int H, int k, int ranks, void* stream);

/* Owner side, reduction fused with the return: for received row i < plan[0],
 * sum_s bf16(rows[inv_pad[i*k+s]] * weights[i,s]) (the combine; weights (n,k)
 * bf16) or sum_s rows[inv_pad[i*k+s]] (weights NULL: the gather backward),
 * over the slots with inv_pad >= 0, fp32 in slot order, rounded once, is
 * stored into the back rows of the rank row i came from; dw_rows (n,k) fp32,
 * if given, into its back dw.  H in {256, 512, 1024, 2048}. */
int b200moe_ep_p2p_reduce_return(const void* rows, const int* inv_pad, const void* weights, int k,
                                 const float* dw_rows, const int* plan, void* const* peer_rows,
                                 float* const* peer_dw, long long rows_cap, int H, int ranks,
                                 void* stream);

/* Pipelined exchange (no counterpart in the reference, which is data-parallel
 * only).  b200moe_ep_p2p_send with a destination filter: dest_mode 0 stores
 * every row, 1 only the rows of this rank (`me`) itself, 2 only the other
 * ranks' rows -- so a rank's own share is copied at once and the rest crosses
 * NVLink beside the experts' compute. */
int b200moe_ep_p2p_send_part(const void* src, const int* inv_send, const int* send_pad_offsets,
                             const int* plan, void* const* peer_rows, long long T, int H,
                             int ranks, const long long* selected, const void* weights, int k,
                             int experts_per_rank, unsigned int* const* peer_meta, int me,
                             int dest_mode, void* stream);

/* b200moe_ep_p2p_reduce_return for one source's rows only: rows [0, n_rows)
 * (inv_pad and weights indexed by that chunk) all came from rank `src`; row i
 * goes to row back_base[src] + i of src's back rows (and back dw). */
int b200moe_ep_p2p_reduce_return_src(const void* rows, const int* inv_pad, const void* weights,
                                     int k, const float* dw_rows, const int* plan,
                                     void* const* peer_rows, float* const* peer_dw,
                                     long long n_rows, int src, int H, int ranks, void* stream);

/* Point-to-point completion flags: each rank's flag area holds one u64 per
 * (phase 1..4, source rank) at flags[phase * 64 + source].  ep_signal writes
 * epoch into word (phase, me) of peer `dest` (every peer when dest < 0),
 * system-scope release after this stream's earlier stores into that peer.
 * ep_wait waits until word (phase, src) of my_flags -- every source's word
 * when src < 0 -- reaches epoch (acquire); at most 4 s, then fault bit 1 and
 * return.  ranks <= 32. */
int b200moe_ep_signal(unsigned long long* const* peer_flags, int phase, int me, int ranks,
                      int dest, unsigned long long epoch, void* stream);
int b200moe_ep_wait(const unsigned long long* my_flags, int phase, int src, int ranks,
                    unsigned long long epoch, void* stream);

/* inv_back (T*P) int32: the row of this rank's back rows that holds owner r's
 * result for token t, or -1 (for b200moe_gather_rows_bwd with k = P). */
int b200moe_ep_p2p_back_inv(const int* inv_send, const int* send_pad_offsets, const int* plan,
                            long long T, int ranks, int* inv_back, void* stream);

/* Group barrier over peer memory: writes epoch (> every earlier epoch) into
 * every peer's flag word for this rank (system-scope release, after this
 * stream's earlier stores into peers) and waits until every peer has written
 * epoch into my_flags (ranks words).  Waits at most 4 s, then sets fault bit 1
 * and returns.  ranks <= 32. */
int b200moe_ep_barrier(unsigned long long* const* peer_flags, unsigned long long* my_flags, int me,
                       int ranks, unsigned long long epoch, void* stream);

/* ---- Muon on the packed expert weights (train.py:2877-3024) --------------
 * The optimizer step of the 3-D expert tensors (Muon groups, train.py:3066-3070):
 * momentum, then the batched Newton-Schulz orthogonalisation of each matrix,
 * then p -= lr * result. */

/* momentum_buf (n) fp32 <- lerp(momentum_buf, grad, 1 - momentum); staged (n)
 * bf16 <- lerp(grad, momentum_buf, momentum) (nesterov) or momentum_buf, with
 * fp32 math and one rounding.  n % 4 == 0.  Replaces _momentum_stage
 * (train.py:2806-2839) / the lerp pair of MuonAdamWHybrid._muon_group (:3001-3005). */
int b200moe_muon_momentum(const float* grad, float* momentum_buf, void* staged, long long n,
                          double momentum, int nesterov, void* stream);

long long b200moe_newton_schulz_scratch_bytes(int batch, int rows, int cols);

/* Newton-Schulz orthogonalisation of a stack x (batch, rows, cols) bf16 of
 * same-shape matrices (_newtonschulz5_batched, train.py:2877-2927): x is
 * normalised in place by its Frobenius norm (bf16, + 1e-7) and then used as a
 * work buffer; `steps` iterations of A = X X^T, P = c*A.A + b*A, X = P.X + a*X
 * (for rows > cols the same on X^T, computed without transposing: A = X^T X,
 * X = X.P^T + a*X), each product in fp32 with one bf16 rounding.  The result
 * goes to out (batch, rows, cols) bf16, or, when update (batch, rows, cols)
 * fp32 is given, is applied as update += neg_lr * bf16(result) instead.
 * rows and cols are multiples of 128. */
int b200moe_newton_schulz(void* x, int batch, int rows, int cols, int steps, float a, float b,
                          float c, void* out, float* update, float neg_lr, void* scratch,
                          long long scratch_bytes, void* stream);

/* ---- load-balancing loss: global_load_balancing_loss (train.py:3098-3197) */

long long b200moe_lb_scratch_bytes(long long T, int E);

/* packed (2E+2) fp32 += [hard counts (E), soft sums (E), entropy, valid rows]
 * of one layer; valid (T) uint8 or NULL (all tokens valid). */
int b200moe_lb_stats(const void* logits, long long ld, const long long* selected,
                     const unsigned char* valid, long long T, int E, int k, float* packed,
                     void* scratch, long long scratch_bytes, void* stream);

/* From the (all-reduced) packed sums: aux (1), stats (5: min_frac, max_frac,
 * cv, entropy, unused) and coef (E): d(local proxy)/d(soft sums). */
int b200moe_lb_finalize(const float* packed, int E, int k, int world_size, float* aux,
                        float* stats, float* coef, void* stream);

/* d_logits (T, ld) bf16 = grad * mask * p * (coef - <p, coef>); grad is a
 * device fp32 scalar. */
int b200moe_lb_grad(const void* logits, long long ld, const unsigned char* valid, long long T,
                    int E, const float* coef, const float* grad, void* d_logits, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200MOE_H_ */
