/*
 * tpp_b200.h — C-ABI of the B200 (sm_100a) kernels behind torchpp's
 * transformer-inference hot path.
 *
 * Every entry point takes plain device pointers, 64-bit sizes and strides
 * (in ELEMENTS, not bytes), a dtype code and a cudaStream_t passed as void*.
 * Nothing here allocates or frees device memory: outputs and workspaces are
 * caller-allocated.  All launches go to the given stream (NULL = legacy
 * default stream) and are asynchronous.  The return value is a tpp_status;
 * on failure tpp_last_error() gives a human-readable message (thread-local).
 *
 * Reference interfaces replaced (paths relative to the torchpp project root):
 *   rmsnormFused.rmsnormFused        csrc/dlops/rmsnorm/rmsnorm_binding.cu:20-73
 *   layernormFused.applyLayernorm    csrc/dlops/layernorm/layernorm_binding.cu:8-47
 *   ropeApplyFunction.rope_apply_cuda   csrc/dlops/rope/rope_binding.cu:10-72
 *   qkropeApplyFunction.qkrope_apply_cuda csrc/dlops/qkrope/qkrope_binding.cu:14-101
 *   linearActvationFp16.LinearGelu/LinearSilu/LinearRelu
 *                                    csrc/activation/binding.cu:11-166
 *   launchHgemv / launchHgemvCute    csrc/blas/hgemv/hgemv_kernels.cuh:69-85,240-262
 *   flash_attn_func (third-party flash-attn 2.x, called at
 *     torchpp/attention/gqa.py:128, swa.py:85-89, mha.py:84, mqa.py:87, ca.py:83)
 *   KVCache.update                   torchpp/llmops/kvcache.py:50-108
 */
#ifndef TPP_B200_H
#define TPP_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  TPP_OK = 0,
  TPP_ERR_SHAPE = 1,        /* bad/mismatched sizes                          */
  TPP_ERR_DTYPE = 2,        /* unsupported dtype code                        */
  TPP_ERR_ALIGN = 3,        /* pointer or stride not suitably aligned        */
  TPP_ERR_LAUNCH = 4,       /* CUDA launch/runtime error                     */
  TPP_ERR_TIMEOUT = 5,      /* a bounded device-side wait gave up            */
  TPP_ERR_UNSUPPORTED = 6,  /* valid request the library does not implement  */
  TPP_ERR_WORKSPACE = 7     /* caller workspace too small / missing          */
} tpp_status;

typedef enum { TPP_F16 = 0, TPP_BF16 = 1, TPP_F32 = 2 } tpp_dtype;

typedef enum {
  TPP_ACT_NONE = 0,
  TPP_ACT_SILU = 1,     /* x / (1 + exp(-x))            csrc/activation/activation.cuh:45-56 */
  TPP_ACT_GELU = 2,     /* tanh GeLU                    csrc/activation/activation.cuh:26-43 */
  TPP_ACT_RELU = 3,     /* max(x, 0)                    csrc/activation/activation.cuh:59-67 */
  TPP_ACT_SWIGLU = 4    /* W holds [gate; up] (2N rows): y = silu(x.Wg^T) * (x.Wu^T)       */
} tpp_act;

/* ---- library info --------------------------------------------------------- */
const char* tpp_last_error(void);
const char* tpp_version(void);
/* Number of kernel launches this library has issued in the calling process. */
uint64_t tpp_launch_count(void);
/* SM budget for the launches the calling host thread makes next (0 = the
 * whole device, the default): decode linears and decode attention size
 * their grids for `sms` SMs.  Lets independent sub-batches recorded as
 * parallel CUDA-graph branches each plan for their share of the GPU.  No
 * reference counterpart. */
int tpp_set_sm_budget(int sms);
/* Reads and clears (synchronising `stream`) the current device's error flag,
 * which a kernel sets when one of its bounded device-side waits runs out
 * instead of spinning forever.  Returns 0 if no wait expired, the nonzero
 * site code of the last expiry otherwise, or TPP_ERR_LAUNCH (negated: -4) if
 * the flag could not be read.  No reference counterpart (the reference has
 * no device-side waits). */
int tpp_device_error(void* stream);
/* Test hook for the path above: launches one CTA whose mbarrier wait can
 * never complete (nothing arrives, no copy is in flight) with a limit of
 * `polls` (1..65536) try_wait polls; the wait gives up, sets the flag to
 * `code` (nonzero) and the kernel returns.  No reference counterpart. */
int tpp_debug_expire_wait(uint32_t polls, int code, void* stream);

/* ---- normalisation -------------------------------------------------------- */
/* y[r,:] = x[r,:] * rsqrt(mean(x[r,:]^2) + eps) * w     (fp32 statistics)
 * Replaces rmsnormFused.rmsnormFused (rmsnorm_binding.cu:20-68; kernel
 * rmsnorm_fp16.cuh:43-115).  x,y: [rows, cols] with row strides; w: [cols]. */
int tpp_rmsnorm(const void* x, int64_t x_row_stride, const void* w, void* y,
                int64_t y_row_stride, int64_t rows, int64_t cols, float eps,
                int dtype, void* stream);

/* Fused residual add + RMSNorm (decode-step fusion):
 *   res[r,:] += x[r,:];  y[r,:] = rmsnorm(res[r,:]) * w
 * res is read and written in place (the residual stream).  When x is NULL the
 * add is skipped.  No reference counterpart as one kernel: it fuses the
 * "x = x + x_res; x = self.rms_norm2(x)" pair of examples/LLM/fastqwen3.py:111-114. */
int tpp_add_rmsnorm(const void* x, void* res, const void* w, void* y,
                    int64_t rows, int64_t cols, float eps, int dtype, void* stream);

/* y = (x - mean) * rsqrt(var + eps) * w (+ b)    (two-pass fp32 statistics)
 * Replaces layernormFused.applyLayernorm (layernorm_binding.cu:8-43; kernel
 * layernorm_fp16.cuh:46-176, which has no bias; b may be NULL). */
int tpp_layernorm(const void* x, const void* w, const void* b, void* y,
                  int64_t rows, int64_t cols, float eps, int dtype, void* stream);

/* ---- rotary position embedding -------------------------------------------- */
/* NeoX rotate-half RoPE:  out = x*cos + rotate_half(x)*sin, rotate_half(x) =
 * cat(-x[D/2:], x[:D/2]).  x is [B,H,S,D] addressed by strides (sb, sh, ss; D
 * contiguous); out is contiguous [B,H,S,D].  cos/sin are [*, D] tables (row
 * stride cs_stride) read at row (s + pos_offset).  Math in fp32.
 * Replaces ropeApplyFunction.rope_apply_cuda (rope_binding.cu:10-67; kernel
 * apply_rope.cuh:4-63). */
int tpp_rope(const void* x, int64_t sb, int64_t sh, int64_t ss,
             const void* cos, const void* sin, int64_t cs_stride, int cs_dtype,
             void* out, int64_t B, int64_t H, int64_t S, int64_t D,
             int64_t pos_offset, int dtype, void* stream);

/* RoPE on Q [B,Hq,S,D] and K [B,Hk,S,D] (contiguous) in one launch; Hq may
 * differ from Hk (GQA).  Replaces qkropeApplyFunction.qkrope_apply_cuda
 * (qkrope_binding.cu:14-92, kernel qkrope.cuh:8-67, which required Hq == Hk). */
int tpp_qkrope(const void* q, const void* k, const void* cos, const void* sin,
               int64_t cs_stride, int cs_dtype, void* q_out, void* k_out,
               int64_t B, int64_t Hq, int64_t Hk, int64_t S, int64_t D,
               int64_t pos_offset, int dtype, void* stream);

/* ---- linear layers --------------------------------------------------------- */
/* y[M,N] = act(x[M,K] . w[N,K]^T + bias) + residual
 * x row-major with row stride ldx (>= K); w row-major [N,K] (or [2N,K] for
 * TPP_ACT_SWIGLU, gate rows first); bias [N] or NULL (for SWIGLU: [2N]);
 * residual [M,N] (row stride ldy) or NULL and may alias y; y row stride ldy.
 * fp32 accumulation.  Replaces linearActvationFp16.LinearGelu/LinearSilu/
 * LinearRelu (activation/binding.cu:11-166, CUTLASS Sm80 GEMM of
 * fused_gemm.cuh:143-170) and the nn.Linear projections of
 * torchpp/attention/gqa.py:41-60.  M <= 64 runs the streaming decode kernel,
 * larger M the tcgen05/TMEM GEMM. */
int tpp_linear(const void* x, int64_t ldx, const void* w, const void* bias,
               const void* residual, void* y, int64_t ldy, int64_t M, int64_t N,
               int64_t K, int act, int dtype, void* stream);

/* Decode-step fusion of RMSNorm into the following linear (M <= 64 rows):
 *   y = act( rsqrt(mean(x[m,:]^2) + eps) * (x[m,:] . w_folded^T) + bias ) + residual
 * where the caller has folded the norm weight into the matrix once,
 * w_folded[n,k] = w[n,k] * gamma[k]; activations/bias/residual/SwiGLU as in
 * tpp_linear.  The statistics come from the x tiles the GEMM already stages,
 * so the separate norm kernel (and its round trip through HBM) disappears.
 * Replaces the rms_norm1/rms_norm2 -> projection pairs of
 * examples/LLM/fastqwen3.py:108-115 (RmsNormFused, torchpp/dlops/
 * normalization.py:30-50, followed by nn.Linear / LinearSILU). */
int tpp_rmsnorm_linear(const void* x, int64_t ldx, const void* w_folded, const void* bias,
                       const void* residual, void* y, int64_t ldy, int64_t M, int64_t N,
                       int64_t K, float eps, int act, int dtype, void* stream);

/* ---- packed decode linears ---------------------------------------------------
 * A decode step (M <= 64 tokens) is bound by how fast each SM can pull its
 * operands, and on B200 a CTA's TMA loads of strided 128-byte rows run at
 * ~25 GB/s while contiguous bulk copies run at >150 GB/s.  The packed forms
 * below lay the operands out in HBM exactly as the tensor-core kernel stages
 * them (128-byte-swizzled K-major tiles), so every load is one contiguous copy:
 *   weights:     per-CTA images, packed once (static);
 *   activations: [K/64][T][64] with T = 16 or 32 (M <= 32 rounded up),
 *                written by the previous decode linear as a second output.
 * Every CTA computes whole outputs (no split-K).  K must be a multiple of 64;
 * tpp_packed_weight_bytes returns 0 when a layer is too wide for this form
 * (then use tpp_linear / tpp_rmsnorm_linear).  No reference counterpart: the
 * reference decodes with nn.Linear / LinearSILU on row-major weights
 * (examples/LLM/fastqwen3.py:108-115). */
int64_t tpp_packed_weight_bytes(int64_t N, int64_t K, int act);
int64_t tpp_packed_activation_bytes(int64_t M, int64_t K);
/* w [N,K] (or [2N,K] gate rows then up rows for SwiGLU) -> packed image. */
int tpp_pack_weight(const void* w, int64_t N, int64_t K, int act, int dtype, void* w_packed,
                    void* stream);
/* x [M,K] (row stride ldx) -> packed activation. */
int tpp_pack_activation(const void* x, int64_t ldx, int64_t M, int64_t K, int dtype,
                        void* x_packed, void* stream);
/* y = act(scale * (x . W^T) + bias) + residual, x and W packed; scale =
 * rsqrt(mean(x^2) + eps) when eps >= 0 (fused RMSNorm, norm weight folded
 * into W as for tpp_rmsnorm_linear), else 1.  y_packed (optional) receives y
 * in packed form for the next decode linear (needs N % 64 == 0). */
int tpp_linear_packed(const void* x_packed, const void* w_packed, const void* bias,
                      const void* residual, void* y, int64_t ldy, void* y_packed, int64_t M,
                      int64_t N, int64_t K, float eps, int act, int dtype, void* stream);

/* ---- fp8 (e4m3) decode weights -------------------------------------------
 * Weight-only fp8 for the decode linears (the reference lists quantized
 * GEMMs as future work, todo.md:24-29).  Format: per-row fp32 scale =
 * amax(|w[n,:]|) / 448 (1 for a zero row); q[n,:] = e4m3(w / scale) with
 * round-to-nearest-even and saturation.  Storage (tpp_fp8_weight_bytes):
 * 32-row groups, [ceil(rows/32)][K/64][32 rows][64 B] (rows past `rows`
 * zero), so a group is one contiguous block; inside each 64-wide k-block
 * byte 16c + 4s + j of a row holds k = 16s + {2c, 2c+1, 2c+8, 2c+9}[j] (the
 * MMA fragment order).  K must be a multiple of 64. */
int64_t tpp_fp8_weight_bytes(int64_t rows, int64_t K);
int tpp_quantize_weight_fp8(const void* w, int64_t rows, int64_t K, int dtype, void* q,
                            float* scale, void* stream);
/* w[n, k] = dtype(e4m3(q) * scale[n]) in natural k order. */
int tpp_dequantize_weight_fp8(const void* q, const float* scale, int64_t rows, int64_t K,
                              int dtype, void* w, void* stream);
/* y = act(r * scale[n] * (x . q[n]) + bias) + residual for 1..32 tokens, as
 * tpp_linear / tpp_rmsnorm_linear with the weight in the fp8 format above:
 * r = rsqrt(mean(x^2) + eps) when eps >= 0 (norm weight folded into w
 * before quantizing), else 1; SwiGLU: q and scale hold 2N rows, gate first
 * (N a multiple of 8).  Larger M: tpp_dequantize_weight_fp8 + tpp_linear. */
int tpp_linear_fp8(const void* x, int64_t ldx, const void* q, const float* scale,
                   const void* bias, const void* residual, void* y, int64_t ldy, int64_t M,
                   int64_t N, int64_t K, float eps, int act, int dtype, void* stream);

/* One sampled token per row of logits [B, V] (row stride ld; V, ld multiples
 * of 8): softmax(logits / temperature) restricted to the top_k largest
 * logits (0 = no limit) and to the smallest descending prefix whose
 * cumulative probability exceeds top_p (1 = no limit), the crossing token
 * included -- LLMInference.sample_top_k / sample_top_p
 * (torchpp/llmops/llm.py:114-203).  Tokens tied with a threshold are all
 * kept.  The uniform draw is SplitMix64(seed, row, counters[row]) (counters
 * may be NULL), so a CUDA graph replays with fresh randomness when the
 * counters (e.g. positions) advance.  Greedy decoding: tpp_argmax. */
int tpp_sample(const void* logits, int64_t ld, int64_t B, int64_t V, float temperature,
               int64_t top_k, float top_p, uint64_t seed, const int32_t* counters, int64_t* out,
               int dtype, void* stream);

/* Bulk-prefetch [ptr, ptr + bytes) into L2 (16-byte aligned, bytes % 16 ==
 * 0); no data reaches the SMs.  Meant for a parallel branch of a decode
 * graph that warms the next layers' weights.  No reference counterpart. */
int tpp_l2_prefetch(const void* ptr, int64_t bytes, void* stream);

/* y[N] = W[N,K] . x[K]   (fp32 accumulation; y in dtype)
 * Replaces launchHgemv / launchHgemvCute (hgemv_kernels.cuh:69-85, 240-262),
 * which accumulated in fp16. */
int tpp_hgemv(const void* W, const void* x, void* y, int64_t N, int64_t K,
              int dtype, void* stream);

/* ---- attention ----------------------------------------------------------- */
/* Prefill / general flash attention (q_len >= 1), GQA by head mapping
 * kv = h / (Hq/Hkv) (what repeat_interleave does at gqa.py:120-121).
 *   q [B,Sq,Hq,D], k/v [B,Sk,Hkv,D], o [B,Sq,Hq,D], each addressed by
 *   (batch, seq, head) element strides with D contiguous.
 * causal: bottom-right aligned (query i sits at key position i + Sk - Sq);
 * window_left >= 0 limits keys to [p - window_left, p] (flash-attn
 * window_size=(w-1,0) at swa.py:88 ⇒ window_left = w-1); -1 = unlimited.
 * Replaces flash_attn_func(q,k,v,causal,window_size). D must be 64 or 128. */
int tpp_attention_prefill(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh,
                          const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh,
                          const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
                          void* o, int64_t o_sb, int64_t o_ss, int64_t o_sh,
                          int64_t B, int64_t Sq, int64_t Sk, int64_t Hq, int64_t Hkv,
                          int64_t D, int causal, int64_t window_left, float scale,
                          int dtype, void* stream);

/* Bytes of workspace tpp_attention_decode needs for the given shape. */
int64_t tpp_attention_decode_workspace(int64_t B, int64_t Hq, int64_t max_seqlen,
                                       int64_t D);

/* Exact workspace bytes for one decode-attention shape (this Hkv and window);
 * 0 when the key range is merged without a workspace.  Never more than
 * tpp_attention_decode_workspace(B, Hq, max_seqlen, D). */
int64_t tpp_attention_decode_workspace_exact(int64_t B, int64_t Hq, int64_t Hkv,
                                             int64_t max_seqlen, int64_t D,
                                             int64_t window_left);

/* Decode attention: one query token per sequence against the KV cache.
 *   q [B,Hq,D] (strides q_sb, q_sh); caches [B,Hkv,Smax,D] (strides c_sb,
 *   c_sh, c_ss); seqlens: device int32[B] (number of valid cache rows per
 *   sequence, the query sits at position seqlens[b]-1) or NULL to use
 *   max_seqlen for every sequence; o [B,Hq,D] (strides o_sb, o_sh).
 *   window_left as in tpp_attention_prefill.  The key range is split across
 *   CTAs (split-KV); partial results go to the caller's workspace
 *   (tpp_attention_decode_workspace bytes) and a second kernel merges them.
 * Replaces flash_attn_func at q_len = 1 (gqa.py:128 in the decode loop of
 * torchpp/llmops/llm.py:263-282; sliding window swa.py:85-89). */
int tpp_attention_decode(const void* q, int64_t q_sb, int64_t q_sh,
                         const void* k_cache, const void* v_cache, int64_t c_sb,
                         int64_t c_sh, int64_t c_ss, const int32_t* seqlens,
                         int64_t max_seqlen, void* o, int64_t o_sb, int64_t o_sh,
                         int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                         int64_t window_left, float scale, void* workspace,
                         int64_t workspace_bytes, int dtype, void* stream);

/* Decode attention with the step's q/k RMSNorm + RoPE + KV append fused in:
 * one launch replaces tpp_qk_norm_rope_cache (S = 1) + tpp_attention_decode.
 * qkv[b] is the raw QKV projection row [q (Hq*D) | k (Hkv*D) | v (Hkv*D)]
 * (row stride ld_qkv); q/k are normalised with qn_w / kn_w (either may be
 * NULL = no norm) and rotated at positions[b] (fp16 tables [ctx, D], row
 * stride cs_stride, NeoX rotate-half), the new k/v are written to the cache
 * row positions[b], and attention covers keys [.., positions[b]].  Requires
 * positions[b] == seqlens[b] - 1 and D = 64 or 128.  Other arguments as
 * tpp_attention_decode.  Replaces the q_norm/k_norm + qkrope + KVCache.update
 * + flash_attn_func sequence of torchpp/attention/gqa.py:96-128. */
int tpp_attention_decode_qkv(const void* qkv, int64_t ld_qkv, const void* qn_w,
                             const void* kn_w, float eps, const void* cos, const void* sin,
                             int64_t cs_stride, int cs_dtype, const int32_t* positions,
                             void* k_cache, void* v_cache, int64_t c_sb, int64_t c_sh,
                             int64_t c_ss, const int32_t* seqlens, int64_t max_seqlen, void* o,
                             int64_t o_sb, int64_t o_sh, int64_t B, int64_t Hq, int64_t Hkv,
                             int64_t D, int64_t window_left, float scale, void* workspace,
                             int64_t workspace_bytes, int dtype, void* stream);

/* ---- paged KV cache --------------------------------------------------------
 * K and V live in block pools [num_blocks][Hkv][64][D] (64 keys a block);
 * sequence b's key k sits in block block_table[b * table_stride + k / 64],
 * row k % 64.  The decode kernels read one 64-key tile per block with one
 * TMA request.  Blocks must exist for every position < seqlens[b].  No
 * reference counterpart (the reference lists a paged cache as a TODO,
 * todo.md:8); semantics as the contiguous entry points. */
int tpp_attention_decode_paged(const void* q, int64_t q_sb, int64_t q_sh, const void* k_pool,
                               const void* v_pool, int64_t num_blocks,
                               const int32_t* block_table, int64_t table_stride,
                               const int32_t* seqlens, int64_t max_seqlen, void* o,
                               int64_t o_sb, int64_t o_sh, int64_t B, int64_t Hq, int64_t Hkv,
                               int64_t D, int64_t window_left, float scale, void* workspace,
                               int64_t workspace_bytes, int dtype, void* stream);
int tpp_attention_decode_qkv_paged(const void* qkv, int64_t ld_qkv, const void* qn_w,
                                   const void* kn_w, float eps, const void* cos, const void* sin,
                                   int64_t cs_stride, int cs_dtype, const int32_t* positions,
                                   void* k_pool, void* v_pool, int64_t num_blocks,
                                   const int32_t* block_table, int64_t table_stride,
                                   const int32_t* seqlens, int64_t max_seqlen, void* o,
                                   int64_t o_sb, int64_t o_sh, int64_t B, int64_t Hq,
                                   int64_t Hkv, int64_t D, int64_t window_left, float scale,
                                   void* workspace, int64_t workspace_bytes, int dtype,
                                   void* stream);
/* Prompt K/V [B, Hkv, S, D] (element strides) into the pools at positions
 * (positions[b] if given, else start_pos) + s. */
int tpp_kv_append_paged(const void* k, int64_t k_sb, int64_t k_sh, int64_t k_ss, const void* v,
                        int64_t v_sb, int64_t v_sh, int64_t v_ss, void* k_pool, void* v_pool,
                        int64_t num_blocks, const int32_t* block_table, int64_t table_stride,
                        const int32_t* positions, int64_t start_pos, int64_t B, int64_t Hkv,
                        int64_t S, int64_t D, int dtype, void* stream);

/* Allocation-free decode attention: the same computation and arguments as
 * tpp_attention_decode, minus the workspace.  For callers that cannot
 * allocate device memory when they decode (allocator / memory-pool
 * callbacks, runtimes with a fixed memory budget that forbid cudaMalloc after
 * start-up, plain-C hosts without an allocator to carve a workspace from).
 * The split-KV partials go to a fixed 8 MiB scratch array inside the
 * library's device image, held by every GPU that loads the library until
 * exit; shapes needing more (see tpp_attention_decode_workspace) are rejected
 * with TPP_ERR_WORKSPACE.  All calls on a device share that array, so calls
 * that overlap on the GPU race -- serialise them.  The first call on each
 * device looks the array's address up; make it before any stream capture.
 * Allocates nothing.  No counterpart in the reference. */
int tpp_attention_decode_noalloc(const void* q, int64_t q_sb, int64_t q_sh,
                                 const void* k_cache, const void* v_cache, int64_t c_sb,
                                 int64_t c_sh, int64_t c_ss, const int32_t* seqlens,
                                 int64_t max_seqlen, void* o, int64_t o_sb, int64_t o_sh,
                                 int64_t B, int64_t Hq, int64_t Hkv, int64_t D,
                                 int64_t window_left, float scale, int dtype, void* stream);
/* Size in bytes of that fixed scratch array.  No counterpart in the reference. */
int64_t tpp_attention_decode_noalloc_max_bytes(void);

/* ---- KV cache / decode-step helpers --------------------------------------- */
/* Fused per-head q/k RMSNorm + RoPE + KV-cache append for S new tokens.
 *   qkv [B,S,(Hq+2*Hkv)*D] rows (row stride ld_qkv): q heads, then k, then v.
 *   qn_w/kn_w: [D] RMSNorm weights or NULL (no q/k norm).
 *   positions: device int32[B], the cache row of token 0 of each sequence
 *   (token s goes to row positions[b]+s and uses cos/sin row positions[b]+s).
 *   q_out [B,S,Hq,D] contiguous.  Caches [B,Hkv,Smax,D] (strides c_sb,c_sh,c_ss).
 * Replaces the q_norm/k_norm (gqa.py:90-94), rope_apply (gqa.py:108-115) and
 * KVCache.update (kvcache.py:83-108) sequence of GroupedQueryAttention.forward. */
int tpp_qk_norm_rope_cache(const void* qkv, int64_t ld_qkv, const void* qn_w,
                           const void* kn_w, float eps, const void* cos,
                           const void* sin, int64_t cs_stride, int cs_dtype,
                           const int32_t* positions, void* q_out, void* k_cache,
                           void* v_cache, int64_t c_sb, int64_t c_sh, int64_t c_ss,
                           int64_t B, int64_t S, int64_t Hq, int64_t Hkv, int64_t D,
                           int dtype, void* stream);

/* Copy new K/V rows [B,Hkv,S,D] (strided) into the caches at row start_pos
 * (host scalar) or at positions[b] when positions != NULL.
 * Replaces the slice assignment of KVCache.update (kvcache.py:73-74, 101-102). */
int tpp_kv_append(const void* k, int64_t k_sb, int64_t k_sh, int64_t k_ss,
                  const void* v, int64_t v_sb, int64_t v_sh, int64_t v_ss,
                  void* k_cache, void* v_cache, int64_t c_sb, int64_t c_sh, int64_t c_ss,
                  int64_t B, int64_t Hkv, int64_t S, int64_t D, int64_t start_pos,
                  const int32_t* positions, int dtype, void* stream);

/* Greedy sampling: out[b] = argmax_v logits[b, v] (first index on ties), as
 * torch.argmax in LLMInference.sample_greedy (torchpp/llmops/llm.py:181-186).
 * logits row stride ld; out int64[B]. */
int tpp_argmax(const void* logits, int64_t ld, int64_t B, int64_t V, int64_t* out,
               int dtype, void* stream);

/* Token embedding gather: out[t,:] = table[ids[t],:]  (nn.Embedding at
 * examples/LLM/fastqwen3.py:128,178).  ids int64[T] on the device.  The ids
 * are only visible on the device, so an id outside [0,V) cannot be reported
 * synchronously: it produces a zero row instead of reading out of bounds. */
int tpp_embedding(const int64_t* ids, int64_t T, const void* table, int64_t V,
                  int64_t D, void* out, int dtype, void* stream);

/* End-of-step bookkeeping for a device-resident (CUDA-graph) decode loop:
 *   p = positions[b] + 1;  out_ids[b*ld_out + p] = next_tokens[b] (if p < out_cap);
 *   positions[b] = p;  seqlens[b] = p + 1 (if seqlens != NULL).
 * positions[b] is the cache row of the token being decoded, so after the step
 * it points at the row of the token just produced.  Replaces the host-side
 * torch.cat bookkeeping and per-token .item() of torchpp/llmops/llm.py:263-285. */
int tpp_decode_advance(const int64_t* next_tokens, int64_t* out_ids, int64_t ld_out,
                       int64_t out_cap, int32_t* positions, int32_t* seqlens, int64_t B,
                       void* stream);

/* ---- persistent single-sequence decode step ------------------------------- */
/* Row pitch of the persistent step's weights: `in` + TPP_PERSISTENT_ROW_PAD
 * elements.  The padding (never read) shifts consecutive rows by 16
 * shared-memory banks, so the kernel's tensor-core operand loads from a
 * bulk-copied weight slice are conflict-free. */
#define TPP_PERSISTENT_ROW_PAD 32

/* One decoder layer's operands for tpp_decode_step_persistent (device
 * pointers; the array of these lives in device memory).  Weights are
 * [out, in] row-major in the step's dtype with a row pitch of
 * in + TPP_PERSISTENT_ROW_PAD elements, with the RMSNorm weight in front
 * of a projection folded into it (w[r, k] * gamma[k]): wqkv [(Hq+2Hkv)*D, E]
 * (q rows, k rows, v rows), wo [E, Hq*D], wgu [2F, E] (gate rows, then up
 * rows), wdown [E, F]; qn / kn the per-head q / k RMSNorm weights [D] (may
 * be NULL); kc / vc the layer's cache [Hkv, Smax, D] (one sequence).  Every
 * pointer 16-byte aligned: the kernel bulk-copies weight slices, cached K/V
 * rows and the norm weights into shared memory. */
typedef struct {
  const void* wqkv;
  const void* qn;
  const void* kn;
  const void* wo;
  const void* wgu;
  const void* wdown;
  void* kc;
  void* vc;
} tpp_decode_layer;

/* Bytes of device workspace tpp_decode_step_persistent needs (zero it once
 * before the first step), or 0 when the model shape is outside its plan. */
int64_t tpp_decode_step_persistent_workspace(int64_t E, int64_t Hq, int64_t Hkv, int64_t D,
                                             int64_t F, int64_t Smax);

/* The whole greedy decode step of one sequence in ONE cooperative launch of
 * one CTA per SM: embedding of tokens[0] -> per layer [RMSNorm + QKV ->
 * q/k RMSNorm + RoPE at positions[0] + K/V append + attention over keys
 * 0..positions[0] (split over CTAs, merged by every CTA that needs it) ->
 * o-proj + residual -> RMSNorm + gate/up + SwiGLU -> down + residual] ->
 * final RMSNorm + LM head (lm_head = W_head * final-norm weight, logits
 * written, [V] in dtype; pitch E + TPP_PERSISTENT_ROW_PAD) -> argmax -> tokens[0] = next, out_ids[p+1] = next
 * (if p+1 < out_cap), positions[0] = p+1, seqlens[0] = p+2.  The phases
 * exchange their outputs as epoch-tagged words in the workspace, so a phase
 * starts once the words it reads carry its producer phase's epoch, and CTA
 * 0 picks the token once every CTA's tagged best logit has arrived (bounded
 * waits; an expiry raises the device error flag and the kernel returns)
 * instead of kernel boundaries,
 * and each CTA's producer warp streams the weight slices of the coming
 * phases (paced: TPP_DP_PACE="<KiB>,<in flight>", default "16,8") and its
 * attention unit's cached K/V rows into shared memory across the barriers.  cos/sin: fp16 RoPE tables
 * [ctx, D] (row stride cs_stride); dtype bf16 or fp16.  Replaces the
 * reference's per-token loop of torchpp/llmops/llm.py:263-282 over
 * examples/LLM/fastqwen3.py:99-118 at batch 1.  Returns TPP_ERR_UNSUPPORTED
 * for shapes outside its plan (a phase's weight slice must fit 96 KB). */
int tpp_decode_step_persistent(const tpp_decode_layer* layers, int64_t n_layers,
                               const void* emb, const void* lm_head, const void* cos,
                               const void* sin, int64_t cs_stride, int64_t* tokens,
                               int32_t* positions, int32_t* seqlens, int64_t* out_ids,
                               int64_t out_cap, void* logits, void* workspace,
                               int64_t workspace_bytes, int64_t E, int64_t Hq, int64_t Hkv,
                               int64_t D, int64_t F, int64_t V, int64_t Smax, float eps,
                               int dtype, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TPP_B200_H */
