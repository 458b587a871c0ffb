/*
 * libd3b200 — C ABI of the B200 (sm_100a) kernels for d3's prefill hot path.
 *
 * Every entry point takes raw device pointers, element strides and sizes, and
 * a CUDA stream (passed as an opaque pointer; 0 = legacy default stream). All
 * work is enqueued on that stream; nothing synchronises the device. The caller
 * owns every buffer. Each function returns D3B_OK (0) or a negative status;
 * d3b_error_string() turns a status into text. Argument problems (shape,
 * stride, alignment, unsupported dtype) are reported before any launch and
 * never reach the GPU. A device-side wait that runs past its wall-clock limit
 * records a site code that d3b_device_error() returns after the stream is
 * synchronised. The word is sticky: while it is set, every later launch's
 * waits stop early and that launch's outputs are undefined (entry points
 * still return D3B_OK, since the launch itself was valid). Callers check
 * d3b_device_error() after a pass (or a batch of passes) and discard the
 * results it covers when it is non-zero; reading it with reset != 0 clears it.
 *
 * Dtype codes (x_dtype, dtype, h_dtype, out_kind):
 *   D3B_F32 = 0, D3B_F16 = 1, D3B_BF16 = 2, D3B_I32 = 3
 * Quantisation modes (mode):
 *   D3B_MODE_FP8 = 0  (e4m3fn, max 448)
 *   D3B_MODE_INT8 = 1 (symmetric int8, max 127)
 */
#ifndef D3B200_H_
#define D3B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define D3B_API __attribute__((visibility("default")))
#else
#define D3B_API
#endif

typedef void* d3b_stream_t;

enum {
  D3B_OK = 0,
  D3B_EINVAL = -1,       /* bad shape, size or argument */
  D3B_EALIGN = -2,       /* pointer or stride not aligned as the kernel needs */
  D3B_EUNSUPPORTED = -3, /* dtype / head_dim / group size the kernels do not cover */
  D3B_ECUDA = -4,        /* a CUDA runtime or driver call failed */
  D3B_ETIMEOUT = -5,     /* a device-side wait ran past its limit */
  D3B_ENOSPACE = -6      /* workspace or fixed scratch too small for the request */
};

enum { D3B_F32 = 0, D3B_F16 = 1, D3B_BF16 = 2, D3B_I32 = 3 };
enum { D3B_MODE_FP8 = 0, D3B_MODE_INT8 = 1, D3B_MODE_NONE = 2 /* fused producers: bf16 rows only */ };

/* Library version (major*10000 + minor*100 + patch). */
D3B_API int d3b_version(void);

/* Static text for a status code. */
D3B_API const char* d3b_error_string(int status);

/* Returns the device error word of the current device (0 = none) after
 * synchronising `stream`; clears it when `reset` is non-zero. A non-zero
 * value is the site code of the wait that gave up. */
D3B_API int d3b_device_error(d3b_stream_t stream, int reset);

/*
 * Per-token (per-row) dynamic activation quantisation.
 * Replaces d3trt/model/quant.py:92-100 (quantize_rows) and, applied to a
 * weight matrix, quant.py:77-89 (quantize_weight).
 *   x     [M, K] rows of `ldx` elements, dtype x_dtype (f32, f16 or bf16)
 *   q     [M, K] contiguous, e4m3fn bytes (mode FP8) or int8 (mode INT8)
 *   scale [M] float32: max(max|x_row|, 1e-12) / 448 (or / 127)
 * q = e4m3_rn_satfinite(clamp(x / scale, ±448)) or int8(clamp(rint(x / scale), ±127)),
 * IEEE division, bit-identical to the reference on the same input.
 */
D3B_API int d3b_act_quant(const void* x, int x_dtype, int64_t ldx, void* q, float* scale, int64_t M, int64_t K,
                  int mode, d3b_stream_t stream);

/*
 * Residual add + zero-centred RMSNorm fused with the per-row activation quant
 * of the linear that consumes the normed rows (q/k/v_proj, gate/up_proj).
 * Replaces reference/d3_kernels.py:97-170 (add_rmsnorm, the bf16-exact
 * restatement of Qwen3_5RMSNorm with a preceding bf16 residual add) followed
 * by d3trt/model/quant.py:92-100 (quantize_rows) on its output.
 *   residual, delta [M, K] bf16 rows of ld_res / ld_delta elements (delta may
 *     be NULL: hidden = residual, no hidden_out)
 *   hidden_out [M, K] bf16 = bf16(residual + delta) (required with delta)
 *   normed = bf16((hidden * rsqrt(mean(hidden^2) + eps)) * weight_plus_one),
 *     fp32 math, mean over an fp64 sum of squares, rsqrt correctly rounded;
 *     rows whose rowmask entry is 0 are zero (rowmask may be NULL)
 *   normed_out [M, K] bf16, optional (required with mode D3B_MODE_NONE)
 *   q [M, K] contiguous codes + scale [M] of normed, as d3b_act_quant
 *     (not written with mode D3B_MODE_NONE)
 * bf16 only, K % 8 == 0, K <= 6144, 16-byte aligned rows (else
 * D3B_EUNSUPPORTED / D3B_EALIGN).
 */
D3B_API int d3b_add_rmsnorm_quant(const void* residual, int64_t ld_res, const void* delta, int64_t ld_delta,
                                  const float* weight_plus_one, float eps, const int32_t* rowmask, void* hidden_out,
                                  int64_t ld_hidden, void* normed_out, int64_t ld_normed, void* q, float* scale,
                                  int64_t M, int64_t K, int mode, d3b_stream_t stream);

/*
 * Attention output gate fused with the per-row activation quant of o_proj.
 * Replaces reference/d3_kernels.py:467-525 (sigmoid_gate; d3trt/model/core.py:297)
 * followed by d3trt/model/quant.py:92-100 on its output.
 *   attn, gate: [B, T, H, D] bf16 views with unit last stride and element
 *     strides attn_strides / gate_strides = {b, t, h} (multiples of 8)
 *   gated = bf16(attn * bf16(1 / (1 + exp(-gate)))) as rows [B*T, H*D]
 *   gated_out [B*T, H*D] bf16 contiguous, optional (required with D3B_MODE_NONE)
 *   q [B*T, H*D] contiguous codes + scale [B*T] of gated, as d3b_act_quant
 * D % 8 == 0, H*D <= 6144.
 */
D3B_API int d3b_sigmoid_gate_quant(const void* attn, const int64_t* attn_strides, const void* gate,
                                   const int64_t* gate_strides, void* gated_out, void* q, float* scale, int B, int T,
                                   int H, int D, int mode, d3b_stream_t stream);

/*
 * W8A8 scaled GEMM: y[m, n] = (sum_k qa[m,k] * qw[n,k]) * sa[m] * sw[n].
 * Replaces the torch._scaled_mm rowwise call in quant.py:164-179 (mode FP8)
 * and torch._int_mm plus its dequant chain in quant.py:190-197 (mode INT8).
 *   qa [M, K] row-major 8-bit, qw [N, K] row-major 8-bit (K-major both)
 *   sa [M] f32, sw [N] f32
 *   y  [M, N] with row stride ldy elements; out_kind D3B_BF16 / D3B_F16 /
 *      D3B_F32 (dequantised) or D3B_I32 (raw int32 accumulator, INT8 only,
 *      scales ignored and may be NULL)
 * Requires K % 16 == 0, N % 16 == 0, 16-byte aligned qa/qw/y.
 */
D3B_API int d3b_w8a8_gemm(const void* qa, const void* qw, const float* sa, const float* sw, void* y, int64_t ldy,
                  int64_t M, int64_t N, int64_t K, int mode, int out_kind, d3b_stream_t stream);

/*
 * Prefix-bidirectional GQA attention (question pass), one launch.
 * Replaces d3trt/kernels/prefix_bidir.py:187-260 (prefix_bidir_attention and
 * the Triton _prefix_bidir_fwd kernel at :47-131, without the pack/unpack
 * gathers). For block b, head h, token i < lengths[b]:
 *   out[b,h,i] = softmax_j(scale * q[b,h,i] . key_j) . value_j over
 *   j in {state keys 0..S-1 of kv head h/(H/Hkv)} U {own keys 0..lengths[b]-1}
 * Tokens i >= lengths[b] get zero rows. S == 0 gives plain bidirectional
 * attention within each block (the state pass, ops.py:107-124 / :174-193).
 *   q        [B, H, L, D]   strides q_strides   = {b, h, l} in elements, d contiguous
 *   k_state  [Hkv, S, D]    strides kv_strides  = {h, s}
 *   v_state  [Hkv, S, D]    same strides as k_state
 *   k_q, v_q [B, Hkv, L, D] strides kq_strides  = {b, h, l}
 *   lengths  [B] int32 on the device (the block-offset table)
 *   out      [B, H, L, D]   strides out_strides = {b, h, l}
 * dtype: D3B_F16 or D3B_BF16 for all of q/k/v/out. D in {32, 64, 128, 256};
 * H % Hkv == 0 and H/Hkv <= 128. Strides must be multiples of 8 elements.
 * The kernel reads `lengths` itself: an entry outside [0, L] is clamped and
 * sets the device error word (site 2010, see d3b_device_error).
 * Work unit: one (block, head group, 128-row Q tile), one CTA per SM at a
 * time. A head group is the kv head's whole GQA group, or, when the group does
 * not divide 128 rows and fewer tiles result, a divisor of it (G = 6 at 64
 * tokens: 3 groups of 2 heads x 64 tokens).
 */
D3B_API int d3b_prefix_bidir(const void* q, const int64_t* q_strides, const void* k_state, const void* v_state,
                     const int64_t* kv_strides, const void* k_q, const void* v_q, const int64_t* kq_strides,
                     const int32_t* lengths, int B, int H, int Hkv, int S, int L, int D, int dtype, float scale,
                     void* out, const int64_t* out_strides, d3b_stream_t stream);

/*
 * Bytes of workspace d3b_prefix_bidir_ws uses for this shape on the current
 * device; 0 when the shape gains nothing from one (units fill whole waves of
 * the SMs, or are too short to cut).
 */
D3B_API size_t d3b_prefix_bidir_workspace_size(int B, int H, int Hkv, int S, int L, int D);

/*
 * d3b_prefix_bidir with a workspace: same arguments, results within rounding
 * of it, same reference function (d3trt/kernels/prefix_bidir.py:187-260).
 * One CTA runs per SM. When the units do not fill whole waves of the SMs, the
 * units of the last partial wave are cut into pieces along their key tiles
 * (sized by a host-side model of the dispatch), so that wave keeps every SM
 * busy; the piece that finishes a unit last merges the pieces' partial
 * results (O, row max, row sum) through the workspace.
 *   workspace  256-byte aligned, >= d3b_prefix_bidir_workspace_size(...)
 *              bytes, ZERO-FILLED before its first use; every launch leaves
 *              it zeroed again. After a device-side error (d3b_device_error
 *              non-zero) zero it again before reuse. Launches that share a
 *              workspace must be ordered (one stream, or events).
 *              NULL: runs as d3b_prefix_bidir.
 * Returns D3B_ENOSPACE if workspace_bytes is too small.
 */
D3B_API int d3b_prefix_bidir_ws(const void* q, const int64_t* q_strides, const void* k_state, const void* v_state,
                        const int64_t* kv_strides, const void* k_q, const void* v_q, const int64_t* kq_strides,
                        const int32_t* lengths, int B, int H, int Hkv, int S, int L, int D, int dtype, float scale,
                        void* out, const int64_t* out_strides, void* workspace, size_t workspace_bytes,
                        d3b_stream_t stream);

/*
 * Causal depthwise convolution + SiLU of the GDN layers over token-major rows.
 * Replaces d3trt/model/ops.py:266-285 (causal_conv1d: F.conv1d with groups=C
 * and padding W-1, cut to L, then SiLU) as called at d3trt/model/core.py:311-330,
 * including the question pass's torch.cat of the snapshot tail.
 *   x      [rows, T, C] bf16, channels contiguous, strides {row, token} in
 *          elements (multiples of 8, token stride >= C)
 *   tail   NULL (state pass: zeros before the first token) or the last W-1
 *          inputs [rows or 1, C, W-1] bf16 with strides {row (0 = shared), c, k}
 *   weight [C, W] bf16 contiguous (conv1d.weight squeezed)
 *   out    [rows, T, C] bf16 contiguous
 *   out[r,t,c] = bf16(silu(bf16(sum_j weight[c,j] * in(r, t-(W-1)+j, c))))
 * C % 8 == 0, 2 <= W <= 8, 16-byte aligned x and out.
 */
D3B_API int d3b_causal_conv1d_silu(const void* x, const int64_t* x_strides, const void* tail,
                                   const int64_t* tail_strides, const void* weight, void* out, int rows, int T,
                                   int C, int W, d3b_stream_t stream);

/*
 * SiLU(gate) * up fused with the per-row quantisation of down_proj's input.
 * Replaces the MLP's act_fn(gate_proj(x)) * up_proj(x) (transformers Qwen3_5MLP,
 * d3trt/model/trtllm_stack.py:118-120) followed by d3trt/model/quant.py:92-100.
 *   gate_up [M, 2I] bf16 rows of ld elements: gate in [0, I), up in [I, 2I)
 *   act = bf16(bf16(silu(gate)) * up); act_out [M, I] bf16 contiguous, optional
 *   (required with D3B_MODE_NONE); q [M, I] codes + scale [M] of act
 * I % 8 == 0, I <= 24576.
 */
D3B_API int d3b_silu_mul_quant(const void* gate_up, int64_t ld, void* act_out, void* q, float* scale, int64_t M,
                               int64_t I, int mode, d3b_stream_t stream);

/*
 * Gated RMSNorm of the GDN output fused with out_proj's per-row quantisation.
 * Replaces Qwen3_5RMSNormGated (called at d3trt/model/core.py:400-401) followed
 * by d3trt/model/quant.py:92-100 on the token rows it produces.
 *   x, z [M, K] bf16 token rows (K = heads * head_dim) of ldx / ldz elements
 *   per head: out = bf16(bf16(weight * bf16(x * rsqrt(mean(x^2) + eps))) * silu(z))
 *   weight [head_dim] bf16; out [M, K] bf16 contiguous, optional (required with
 *   D3B_MODE_NONE); q [M, K] codes + scale [M] of out
 * head_dim in {64, 128, 256}, K % head_dim == 0, K <= 6144.
 */
D3B_API int d3b_gated_rmsnorm_quant(const void* x, int64_t ldx, const void* z, int64_t ldz, const void* weight,
                                    float eps, int head_dim, void* out, void* q, float* scale, int64_t M, int64_t K,
                                    int mode, d3b_stream_t stream);

/*
 * Gated DeltaNet gates of every (token row, value head). Replaces the module's
 * beta = b.sigmoid() and g = -A_log.float().exp() * softplus(a.float() + dt_bias)
 * (d3trt/model/core.py:341-342).
 *   a, b [M, HV] bf16 rows of lda / ldb elements (slices of the input projection)
 *   neg_exp_a [HV] f32 = -exp(float(A_log)); dt_bias [HV] f32
 *   g [M, HV] f32 = neg_exp_a * softplus(float(a) + dt_bias) (softplus: x > 20 ? x : log1p(exp(x)))
 *   beta [M, HV] bf16 = bf16(1 / (1 + exp(-b)))
 */
D3B_API int d3b_gdn_gates(const void* a, int64_t lda, const void* b, int64_t ldb, const float* neg_exp_a,
                          const float* dt_bias, float* g, void* beta, int64_t M, int HV, d3b_stream_t stream);

/*
 * Per-head RMSNorm of queries or keys followed by the partial rotary embedding,
 * one pass. Replaces q_norm / k_norm (transformers Qwen3_5RMSNorm) and
 * apply_rotary_pos_emb in D3Core._attention (d3trt/model/core.py:233-237).
 *   x [rows, T, heads, head_dim] bf16, element strides x_strides = {row, token,
 *     head}, head_dim contiguous (the query half of q_proj's output is a slice)
 *   y = bf16(float(x * rsqrt(mean(x^2) + eps)) * (1 + weight))   weight [head_dim] bf16
 *   for i < rotary_dim: out_i = bf16(bf16(y_i * cos_i) + bf16(rot(y)_i * sin_i)),
 *     rot(y) = (-y[rd/2 .. rd), y[0 .. rd/2)); out_i = y_i beyond rotary_dim
 *   cos, sin [rows, T, rotary_dim] bf16, element strides cs_strides = {row, token}
 *   out [rows, T, heads, head_dim] bf16 contiguous (token-major)
 * head_dim == 128, rotary_dim in {16, 32, 64, 128}.
 */
D3B_API int d3b_qk_norm_rope(const void* x, const int64_t* x_strides, const void* weight, const void* cos,
                             const void* sin, const int64_t* cs_strides, void* out, int rows, int T, int heads,
                             int head_dim, int rotary_dim, float eps, d3b_stream_t stream);

/*
 * 255-way (any n_opt <= 1024) fp32 readout softmax at the selected positions.
 * Replaces the probabilities body of d3trt/model/trtllm_stack.py:451-468
 * (= hf_stack.py:67-84): logits = f32(hidden) @ readout^T; logits[b, j] = -inf
 * for j >= counts[b]; probs = softmax(logits / temperature).
 *   hidden  [B, K] contiguous, dtype h_dtype (f32, f16, bf16)
 *   readout [n_opt, K] f32 contiguous
 *   counts  [B] int32 device
 *   probs   [B, n_opt] f32 contiguous
 *   workspace: device scratch of d3b_readout_workspace_size(B, n_opt) bytes,
 *   zero-filled before its first use; the kernel leaves it ready for the next
 *   call. Calls that share a workspace must not overlap on the GPU.
 */
D3B_API size_t d3b_readout_workspace_size(int B, int n_opt);
D3B_API int d3b_readout(const void* hidden, int h_dtype, const float* readout, const int32_t* counts, float temperature,
                float* probs, int B, int K, int n_opt, void* workspace, size_t workspace_bytes,
                d3b_stream_t stream);

/*
 * The same readout on the tensor cores for bf16 hidden rows (the model's
 * final-norm output; trtllm_stack.py:451-468 as above). The fp32 readout matrix
 * is first split, once, into three bf16 planes r0 + r1 + r2 = readout (all 24
 * bits): d3b_readout_split writes them as [3][o_pad][K] bf16 (o_pad = n_opt
 * rounded up to 256, padding rows zero) into a buffer of
 * d3b_readout_planes_size(n_opt, K) bytes. d3b_readout_planes then computes
 * every logit as sum_p hidden . r_p with exact bf16 x bf16 products and fp32
 * accumulation (an fp32 dot product in another summation order), split over K
 * across the SMs, and applies the mask, temperature and softmax like d3b_readout.
 *   hidden [B, K] bf16 contiguous, 16-byte aligned; K % 8 == 0
 *   workspace: d3b_readout_planes_workspace_size(B, K, n_opt) bytes (the K
 *   splits' partial logits; no zero-filling needed), 16-byte aligned
 */
D3B_API size_t d3b_readout_planes_size(int n_opt, int K);
D3B_API int d3b_readout_split(const float* readout, int n_opt, int K, void* planes, d3b_stream_t stream);
D3B_API size_t d3b_readout_planes_workspace_size(int B, int K, int n_opt);
D3B_API int d3b_readout_planes(const void* hidden, const void* planes, const int32_t* counts, float temperature,
                               float* probs, int B, int K, int n_opt, void* workspace, size_t workspace_bytes,
                               d3b_stream_t stream);

/*
 * The readout above for callers that cannot allocate device memory when they
 * call (for example code that runs during CUDA graph capture, or a host
 * runtime that only hands over its input and output buffers). It has no
 * counterpart in the reference. Same arguments and results as d3b_readout,
 * without the workspace: the scratch is one fixed 1 MiB array inside the
 * library, held by every GPU that loads it until the process exits.
 *   Limit: 16 KiB of counters plus B * n_opt * 4 bytes of logits must fit in
 *   1 MiB (B * n_opt up to 258048 logits), otherwise D3B_ENOSPACE and nothing
 *   is enqueued.
 *   Calls on one device share the array: calls whose work overlaps on the
 *   GPU (unordered streams) race and give wrong results.
 *   The first call on a device looks up the array's device address; make it
 *   before any stream capture begins. The address is kept per device ordinal
 *   for the life of the process and is not looked up again after a
 *   cudaDeviceReset; do not call this entry point on a device after resetting it.
 * Calls no allocating routine (no cudaMalloc / cudaFree).
 */
D3B_API int d3b_readout_noalloc(const void* hidden, int h_dtype, const float* readout, const int32_t* counts,
                                float temperature, float* probs, int B, int K, int n_opt, d3b_stream_t stream);

/*
 * Self-test of the device wait limit: launches one CTA that waits on an
 * mbarrier nothing arrives on, with a limit of `limit_ms` milliseconds; the
 * kernel gives up, records its site code and returns. After synchronising,
 * d3b_device_error() returns that code. Used by the failure-detection test.
 */
D3B_API int d3b_selftest_wait_timeout(int limit_ms, d3b_stream_t stream);

/*
 * Gated delta rule: the GDN layers' scan, token-recurrent, fp32 state. Replaces
 * FLA's fused_recurrent_gated_delta_rule as the reference calls it
 * (d3trt/model/ops.py:327-360, d3trt/model/core.py:360-372) and, for the same
 * math, chunk_gated_delta_rule (ops.py:287-324). Per (row, value head), over t:
 *   S <- exp(g_t) S;  v' = beta_t (v_t - S^T k_t);  S <- S + k_t v'^T;  o_t = S^T q_t
 *   q, k [B, T, H, K]; v, o [B, T, HV, V]: `dtype` (D3B_BF16 / D3B_F16), innermost
 *     dim contiguous, *_strides = element strides of (b, t, head); the q/k head
 *     of value head hv is hv / (HV / H) (no repeated q/k needed)
 *   g [B, T, HV] f32 (log decay); beta [B, T, HV] in beta_dtype (F32/BF16/F16)
 *   h0 [B, HV, K, V] f32 or NULL (zeros); h0_strides = (b, hv, k-row), V
 *     contiguous; a b stride of 0 shares one state across rows
 *   ht [B, HV, K, V] f32 contiguous or NULL: the final state
 *   K in {64, 128}, V % 32 == 0, HV % H == 0. l2norm != 0 divides q and k by
 *   sqrt(sum x^2 + 1e-6); q is then multiplied by scale.
 *   algo: 1 = token recurrence (fp32 throughout, FLA's fused recurrent numerics);
 *   2 = chunked form on the tensor cores (bf16 products, fp32 accumulate and
 *   solve; T <= 64, K = V = 128, h0 NULL or shared by all rows, ht NULL, 16-byte
 *   rows, a workspace of d3b_gated_delta_workspace_size() bytes when h0 is given,
 *   else D3B_EUNSUPPORTED); 3 = chunked form with the inter-chunk state
 *   recurrence (FLA's chunk_gated_delta_rule numerics: 64-token chunks, bf16
 *   products, fp32 accumulation and state; any T, K = V = 128, per-row or shared
 *   h0, ht allowed, 16-byte rows, a 256-byte aligned workspace of
 *   d3b_gated_delta_state_workspace_size() bytes, else D3B_EUNSUPPORTED);
 *   0 = form 2 where it applies, else form 3 where it applies, else 1.
 */
D3B_API int d3b_gated_delta_rule(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                 const void* v, const int64_t* v_strides, const float* g, const int64_t* g_strides,
                                 const void* beta, int beta_dtype, const int64_t* beta_strides, const float* h0,
                                 const int64_t* h0_strides, void* o, const int64_t* o_strides, float* ht, int B,
                                 int T, int H, int HV, int K, int V, int dtype, float scale, int l2norm, int algo,
                                 void* workspace, size_t workspace_bytes, d3b_stream_t stream);

/* Device workspace the chunked form needs with an initial state: HV bf16 copies of
 * the state, 32 KiB each (0 where the chunked form does not apply). */
D3B_API size_t d3b_gated_delta_workspace_size(int HV, int K, int V);

/* Device workspace of the chunked form with the inter-chunk recurrence (algo 3;
 * the state pass, ops.py:287-324 with output_final_state): 74752 bytes per
 * (row, value head, 64-token chunk), the chunk's operand tiles (0 where the form
 * does not apply). */
D3B_API size_t d3b_gated_delta_state_workspace_size(int B, int T, int HV, int K, int V);

/*
 * State snapshots (the per-layer K/V and GDN states one state pass leaves
 * behind; replaces the tensor lists that d3trt/model/core.py:28-40 defines and
 * d3trt/model/cache.py:50-184 caches).
 *
 * d3b_copy_segments: one launch copies `n` strided byte segments. Segment i
 * moves outer x rows rows of row_bytes contiguous bytes; the row (o, r) starts
 * at src + o*src_outer_stride + r*src_row_stride and lands at
 * dst + o*dst_outer_stride + r*dst_row_stride (byte strides, any sign). Source
 * and destination ranges must not overlap. The widest access (16, 8, 4, 2 or 1
 * bytes) that divides every address, row size and used stride of a segment is
 * chosen per segment. Empty segments are skipped. Up to 128 segments go into
 * one launch (the table travels as the kernel's parameter, so the call
 * allocates and copies nothing else and can be captured in a CUDA graph).
 */
typedef struct d3b_copy_segment {
  const void* src;
  void* dst;
  int64_t outer, rows, row_bytes;
  int64_t src_outer_stride, src_row_stride;
  int64_t dst_outer_stride, dst_row_stride;
} d3b_copy_segment;

D3B_API int d3b_copy_segments(const d3b_copy_segment* segments, int n, d3b_stream_t stream);

/*
 * Snapshot arena: host-side bookkeeping of one caller-owned device buffer of
 * `capacity` bytes. Blocks are `alignment`-aligned (a power of two >= 16),
 * placed best-fit and coalesced on free. The arena touches no device memory;
 * it only hands out offsets. Thread-safe.
 *   d3b_arena_alloc  -> D3B_ENOSPACE when no free range holds `bytes`
 *   d3b_arena_free   -> D3B_EINVAL when `offset` is not a live block
 *   d3b_arena_stats  -> stats[0] bytes in live blocks, [1] free bytes,
 *                       [2] largest free range, [3] live blocks
 */
D3B_API int d3b_arena_create(uint64_t capacity, uint64_t alignment, void** arena);
D3B_API int d3b_arena_alloc(void* arena, uint64_t bytes, uint64_t* offset);
D3B_API int d3b_arena_free(void* arena, uint64_t offset);
D3B_API int d3b_arena_stats(void* arena, uint64_t* stats);
D3B_API void d3b_arena_destroy(void* arena);

#ifdef __cplusplus
}
#endif

#endif /* D3B200_H_ */
