/*
 * qf2b200.h -- C ABI of libqf2b200.so, the B200 (sm_100a) kernels behind the
 * DiT inference hot path of quantfun2 (Flux / Lumina-Image-2.0).
 *
 * Conventions (all entry points):
 *   - Plain device pointers, element strides (not bytes), int64 sizes.
 *   - Every call is asynchronous and ordered on `stream` (a cudaStream_t;
 *     NULL = legacy default stream).  Nothing is allocated: outputs and any
 *     workspace are owned by the caller.
 *   - Return 0 on success or a negative qf2_status.  Shape/dtype/alignment
 *     problems are reported before anything is launched.
 *   - Kernels that wait on mbarriers bound every wait (~2 s); a timed-out
 *     kernel writes a nonzero code into the status word at the start of the
 *     caller's workspace and returns.  qf2_workspace_status() reads it back.
 *
 * Each entry point names the reference interface it replaces
 * (paths are relative to the gabe56f/quantfun2 source tree).
 */
#ifndef QF2B200_H
#define QF2B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* qf2_stream_t; /* == cudaStream_t */

enum qf2_status {
  QF2_OK = 0,
  QF2_ERR_SHAPE = -1,       /* unsupported or inconsistent sizes           */
  QF2_ERR_DTYPE = -2,       /* unsupported dtype code                      */
  QF2_ERR_LAUNCH = -3,      /* CUDA launch / runtime error                 */
  QF2_ERR_TIMEOUT = -4,     /* a bounded device-side wait gave up          */
  QF2_ERR_ALIGN = -5,       /* pointer or stride alignment not met         */
  QF2_ERR_WORKSPACE = -6,   /* workspace missing or too small              */
  QF2_ERR_DEVICE = -7,      /* current device is not an sm_100 part        */
  QF2_ERR_ARG = -8          /* NULL or otherwise invalid argument          */
};

enum qf2_dtype {
  QF2_F32 = 0,
  QF2_F16 = 1,
  QF2_BF16 = 2,
  QF2_I8 = 3,
  QF2_E4M3 = 4,
  QF2_I32 = 5
};

/* ---------------------------------------------------------------- misc -- */
const char* qf2_version(void);
const char* qf2_status_string(int status);
/* Text of the CUDA error behind the last QF2_ERR_LAUNCH returned on this host thread
 * (empty if none). */
const char* qf2_last_error(void);
/* 0 when the current CUDA device is compute capability 10.0, else QF2_ERR_DEVICE. */
int qf2_device_check(void);
/* Synchronizes `stream`, then reads (and clears) the status word at the start of
 * `workspace`: QF2_ERR_TIMEOUT if a bounded wait gave up, QF2_ERR_ARG if a kernel met an
 * index outside its range (and skipped it), else QF2_OK. */
int qf2_workspace_status(void* workspace, qf2_stream_t stream);

/* ---------------------------------------------------------------- RoPE --
 * Replaces rope_apply (src/kernels/__init__.py:126-142, eager) and its Triton
 * body rope_triton (src/kernels/triton/rope.py:83-134).
 * Rotates interleaved pairs (x[2p], x[2p+1]) of the last dim by the complex
 * freqs_cis[b, s, p] (complex64, interleaved re/im floats), fp32 math, result
 * rounded to `dtype`.  x*_strides = {batch, seq, head} in elements; the last
 * dim is contiguous.  freqs_strides = {batch, seq} in complex elements (batch
 * stride 0 broadcasts).  xk may be NULL.  Out may alias in (in-place, as the
 * Triton path does).  flags & QF2_ROPE_FP16_TRIG rounds cos/sin to fp16 first,
 * which is what the reference's Triton path computes with (rope.py:91-92).
 */
#define QF2_ROPE_FP16_TRIG 1
int qf2_rope_apply(const void* xq, void* xq_out, int64_t Hq, const int64_t* xq_strides,
                   const int64_t* xq_out_strides, const void* xk, void* xk_out, int64_t Hk,
                   const int64_t* xk_strides, const int64_t* xk_out_strides, const void* freqs_cis,
                   const int64_t* freqs_strides, int64_t B, int64_t S, int64_t D, int dtype, int flags,
                   qf2_stream_t stream);

/* Fused per-head q/k RMSNorm + RoPE on a fused QKV projection output, replacing the
 * q_norm / k_norm + rope_apply sequence of the attention blocks (src/models/flux/mmdit.py
 * :133-149, src/models/common/attn.py:209-212): qkv [B*L, (Hq + 2*Hkv)*D] bf16 (q heads,
 * k heads, v heads; row stride qkv_row_stride); q and k rows -> x * rsqrt(mean(x^2) +
 * eps) * w, rotated by freqs_cis[b, s] (complex64, strides {batch, seq} in complex
 * elements), rounded once; v copied.  Outputs through {batch, seq, head} element
 * strides with head dim Dout >= D (extra columns written as zero, e.g. head_dim 96
 * padded to the attention kernel's 128).  D, Dout multiples of 8, <= 128; bf16. */
int qf2_qkv_norm_rope(const void* qkv, int64_t qkv_row_stride, int64_t B, int64_t L, int64_t Hq, int64_t Hkv,
                      int64_t D, int64_t Dout, void* q_out, const int64_t* q_strides, void* k_out,
                      const int64_t* k_strides, void* v_out, const int64_t* v_strides, const void* q_weight,
                      const void* k_weight, float eps, const void* freqs_cis, const int64_t* freqs_strides,
                      qf2_stream_t stream);

/* RoPE with row scatter, the RoPE of the reference's RAS partial ops (PYCUDA_ROPE_KERNEL,
 * src/kernels/cuda/ras.cu:12-52): y[b, idx[n], h, :] = rotate(x[b, n, h, :], f[n]) for the
 * N rows of x [B, N, H, D] into y [B, M, H, D]; f holds D/2 complex factors per row as
 * interleaved (cos, sin) floats, row stride f_stride floats; idx int64 [N] on the device.
 * bf16 only (as the reference); strides {batch, row, head} in elements, D % 8 == 0, 16-byte
 * aligned rows.  Rows of y not named by idx are left untouched.  workspace (optional, a
 * 256-byte status word area): an index outside [0, M) skips its row and makes
 * qf2_workspace_status return QF2_ERR_ARG. */
int qf2_rope_scatter(const void* x, const int64_t* x_strides, const float* f, int64_t f_stride, const int64_t* idx,
                     void* y, const int64_t* y_strides, int64_t B, int64_t N, int64_t M, int64_t H, int64_t D,
                     int dtype, void* workspace, qf2_stream_t stream);

/* ------------------------------------------------------------- RMSNorm --
 * Replaces rmsnorm_apply (src/kernels/__init__.py:73-80) and the Triton
 * apply_rmsnorm (src/kernels/triton/rmsnorm.py:72-95).
 * out[m, :] = x[m, :] * rsqrt(mean(x[m, :]^2) + eps) * w, with fp32 sum of squares.
 *   mode QF2_RMS_EAGER : normalized row rounded to x's dtype, then multiplied
 *                        by w and rounded to out_dtype (the eager body).
 *   mode QF2_RMS_FUSED : product formed in fp32, rounded once (the Triton body).
 * Rows are N contiguous elements; row strides in elements.
 */
#define QF2_RMS_EAGER 0
#define QF2_RMS_FUSED 1
int qf2_rmsnorm(const void* x, int64_t x_row_stride, int x_dtype, const void* weight, int w_dtype, void* out,
                int64_t out_row_stride, int out_dtype, int64_t M, int64_t N, float eps, int mode,
                qf2_stream_t stream);

/* Gated residual + RMSNorm-modulate of the Lumina joint block (src/models/lumina/image_two/
 * model.py:82-101), one pass over rows of `dim` bf16 (dim a multiple of 256, <= 8192;
 * contiguous rows; batch b = row / rows_per_batch):
 *   if y:  x = bf16(x + g * RMSNorm(y; w_post, eps_post))   g = tanh(gate[b]) when
 *          gate_tanh, gate[b] otherwise, 1 without gate; w_post NULL = no norm on y
 *   if h:  h = bf16(RMSNorm(x; w_pre, eps_pre) * (1 + scale[b]))   (scale NULL = 0)
 * gate / scale rows are gate_stride / scale_stride elements apart. */
int qf2_rms_gate_residual(const void* y, void* x, void* h, int64_t rows, int64_t dim, int64_t rows_per_batch,
                          const void* w_post, float eps_post, const void* gate, int64_t gate_stride, int gate_tanh,
                          const void* w_pre, float eps_pre, const void* scale, int64_t scale_stride,
                          qf2_stream_t stream);

/* ------------------------------------------------------------- softmax --
 * Replaces inplace_softmax (src/kernels/__init__.py:83-87) and
 * inplace_tiled_softmax (src/kernels/triton/softmax.py:82-91): in-place
 * softmax over each of `rows` rows of `n` elements (row stride in elements).
 */
int qf2_softmax_inplace(void* x, int64_t rows, int64_t n, int64_t row_stride, int dtype, qf2_stream_t stream);

/* ------------------------------------------------ Sage-style attention --
 * Replaces sageattention.sageattn (called at src/models/flux/attn.py:39-41)
 * and sageattn_varlen (src/models/common/attn.py:109-120).
 * Algorithm: K smoothed by its per-(sequence, head, channel) token mean; Q
 * (pre-multiplied by sm_scale*log2(e)) and smoothed K quantized to INT8 per
 * 64-token block by the published SageAttention rule (scale = amax/127,
 * t = x / scale, code = trunc(t + 0.5 * sign(t)), each step rounded in fp32); V quantized
 * to FP8 e4m3 per channel (code = e4m3(v * (448/amax)), scale = amax/448);
 * S = Qi8.Ki8^T on tcgen05 kind::i8 into
 * TMEM; online softmax in base 2; P quantized to e4m3 (x448) and P.V on
 * tcgen05 kind::f8f6f4 with fp32 accumulation in TMEM.  D = 64, 96 or 128 (the
 * Flux blocks' 128, Lumina's 96): channels past D are zero in the code tiles, QK^T
 * runs D/32 MMA K-steps, the output has D columns.
 *
 * Dense: q/k/v/out strides = {batch, head, seq} in elements (HND and NHD both
 * expressible); dtype QF2_BF16 or QF2_F16; Hq % Hkv == 0 (GQA).
 * Varlen: q [total_q, Hq, D], k/v [total_k, Hkv, D], strides = {token, head};
 * cu_seqlens_* are int32 device arrays of batch+1 offsets.
 * Workspace: caller-owned device memory of qf2_sage_workspace_bytes(); it
 * holds the quantized codes, scales and the status word.
 */
int64_t qf2_sage_workspace_bytes(int64_t batch, int64_t Hq, int64_t Hkv, int64_t total_q, int64_t total_k,
                                 int64_t max_seqlen_q, int64_t max_seqlen_k, int64_t D);
int qf2_sageattn(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides, const void* v,
                 const int64_t* v_strides, void* out, const int64_t* out_strides, int64_t B, int64_t Hq,
                 int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D, float sm_scale, int dtype, void* workspace,
                 int64_t workspace_bytes, qf2_stream_t stream);
int qf2_sageattn_varlen(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                        const void* v, const int64_t* v_strides, void* out, const int64_t* out_strides,
                        const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int64_t batch,
                        int64_t total_q, int64_t total_k, int64_t max_seqlen_q, int64_t max_seqlen_k, int64_t Hq,
                        int64_t Hkv, int64_t D, float sm_scale, int dtype, void* workspace,
                        int64_t workspace_bytes, qf2_stream_t stream);

/* Byte offsets inside the Sage workspace (for inspecting the quantized codes):
 * offsets[0..10] = status, q codes, q scales, k codes, k scales, v codes,
 * v scales, k mean, v inverse scales, split-KV partial rows, split-KV row max/sum;
 * offsets[11] = total. */
int qf2_sage_workspace_layout(int64_t batch, int64_t Hq, int64_t Hkv, int64_t total_q, int64_t total_k,
                              int64_t max_seqlen_q, int64_t max_seqlen_k, int64_t D, int64_t* offsets);

/* Failure injection for tests of the bounded waits (no counterpart in the reference; the
 * reference has no failure detection).  Process-wide, read by every later Sage attention
 * launch: wait_limit_us > 0 bounds each of the attention kernel's mbarrier waits to about
 * that many microseconds (<= 0: the default, about 2 s); skip_kv_tile >= 0 makes the
 * producer never issue the load of that K/V tile of each CTA, so the waits on it run out,
 * the kernel records a timeout in the workspace status word (qf2_workspace_status then
 * returns QF2_ERR_TIMEOUT), lets its issued copies land, drains its MMAs, frees its TMEM
 * and returns; the output of that call is undefined.  Nothing faults: the context stays
 * usable.  qf2_sage_fault_injection(0, -1) restores normal operation. */
int qf2_sage_fault_injection(int64_t wait_limit_us, int skip_kv_tile);

/* Quantization stage alone (same arguments as qf2_sageattn / _varlen; pass
 * cu_seqlens NULL for the dense form).  Leaves codes and scales in the
 * workspace, laid out as qf2_sage_workspace_layout() describes. */
int qf2_sage_quantize(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                      const void* v, const int64_t* v_strides, const int32_t* cu_seqlens_q,
                      const int32_t* cu_seqlens_k, int64_t batch, int64_t Sq, int64_t Skv, int64_t total_q,
                      int64_t total_k, int64_t max_seqlen_q, int64_t max_seqlen_k, int64_t Hq, int64_t Hkv,
                      int64_t D, float sm_scale, int dtype, void* workspace, int64_t workspace_bytes,
                      qf2_stream_t stream);

/* Attention stage alone, reading the codes qf2_sage_quantize() left in `workspace`
 * (the second half of qf2_sageattn / qf2_sageattn_varlen; same layout rules). */
int qf2_sage_attn_quantized(void* out, const int64_t* out_strides, const int32_t* cu_seqlens_q,
                            const int32_t* cu_seqlens_k, int64_t batch, int64_t Sq, int64_t Skv, int64_t total_q,
                            int64_t total_k, int64_t max_seqlen_q, int64_t max_seqlen_k, int64_t Hq, int64_t Hkv,
                            int64_t D, int dtype, void* workspace, int64_t workspace_bytes, qf2_stream_t stream);

/* ------------------------------------------ top-k block-sparse attention --
 * Replaces topk_attn (src/kernels/__init__.py:146-195) and its mask cache POS_DICT
 * (src/models/common/attn.py:20, :24-56), in block form with 128-token blocks:
 *   qf2_blocktopk_select: mean-pool Q and K per block (fp64 sums, fp32 means), block
 *     scores pooled_q . pooled_k^T (fp64, d ascending, rounded to fp32), keep the top
 *     `keep` key blocks per query block (lower index wins ties) and write them in
 *     ascending order to idx_out [B, Hq, ceil(S/128), keep] (int32).  The caller may
 *     cache idx across layers as the reference caches POS_DICT.
 *   qf2_blocksparse_attn: exact softmax attention of every query block over its kept
 *     key blocks (keys beyond S masked); bf16/fp16, D = 128, tcgen05 kind::f16.
 * q/k/v/out strides = {batch, head, seq} in elements, multiples of 8.  The select
 * workspace holds the pooled blocks (qf2_blocktopk_workspace_bytes); the attention
 * workspace holds only the status word (256 bytes). */
int64_t qf2_blocktopk_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t D);
int qf2_blocktopk_select(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides, int64_t B,
                         int64_t Hq, int64_t Hkv, int64_t S, int64_t D, int64_t keep, int dtype, int32_t* idx_out,
                         void* workspace, int64_t workspace_bytes, qf2_stream_t stream);
int qf2_blocksparse_attn(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                         const void* v, const int64_t* v_strides, void* out, const int64_t* out_strides, int64_t B,
                         int64_t Hq, int64_t Hkv, int64_t S, int64_t D, const int32_t* idx, int64_t keep,
                         float sm_scale, int dtype, void* workspace, int64_t workspace_bytes, qf2_stream_t stream);

/* ------------------------------------------------------ quantized linears --
 * Replace the torchao weight subclasses the reference swaps into nn.Linear.weight
 * (src/quant.py:131-148; int8 weight-only :209-224, float8 weight-only :227-241).
 *
 * qf2_quantize_rows: per-row symmetric quantization of x [M, K] (row stride ldx):
 *   QF2_I8:   scale = max(amax / 127.5, FLT_EPSILON), code = rint(x / scale) in [-128, 127]
 *   QF2_E4M3: scale = amax / 448 (1 for a zero row), code = e4m3(x * (448 / amax))
 * One fp32 scale per row in `scales` (weights: per output channel; activations: per token).
 *
 * qf2_codes_to_bf16: int8 / e4m3 codes -> bf16 (exact).
 *
 * qf2_gemm: D[M, N] = (A . B^T) * row_scale[m] * col_scale[n] + bias[n] on tcgen05 tensor
 * cores, A [M, K] and B [N, K] both QF2_BF16, both QF2_F16 or both QF2_E4M3 with K
 * contiguous (row strides lda/ldb in elements), fp32 accumulation, D QF2_BF16, QF2_F16
 * or QF2_F32 (row stride ldd; the residual and SwiGLU epilogues need QF2_BF16).  row_scale, col_scale and bias may be NULL; bias is QF2_BF16 or QF2_F32.
 * N % 8 == 0.  Workspace: >= 256 bytes (status word).
 * Weight-only INT8/FP8 linear: D = qf2_gemm_codes(x, codes, col_scale = w_scale) for M <= 128,
 * else D = qf2_gemm_ex(x, qf2_codes_convert(codes), col_scale = w_scale).
 * W8A8 FP8 linear: D = qf2_gemm(e4m3(x), e4m3 codes, row_scale = x_scale, col_scale = w_scale). */
int qf2_quantize_rows(const void* x, int64_t ldx, int x_dtype, int64_t M, int64_t K, void* q, int64_t ldq,
                      int q_dtype, float* scales, qf2_stream_t stream);
int qf2_codes_to_bf16(const void* q, int64_t ldq, int q_dtype, int64_t M, int64_t K, void* out, int64_t ldo,
                      qf2_stream_t stream);
/* Weight quantizer of the reference's quantize-on-load (src/quant.py:209-241 through
 * torchao 0.7.0 choose_qparams_affine / quantize_affine, with the model already cast to
 * the qdtype's activation dtype at src/quant.py:383).  w [M, K] in w_dtype T (QF2_F16,
 * QF2_BF16 or QF2_F32), every step rounded in T as the library's tensor ops do:
 *   scale = max(T(amax / D), FLT_EPSILON)   D = 127.5 (QF2_I8) or 448 (QF2_E4M3)
 *   y = T(w * T(1 / scale));  QF2_I8: code = clamp(round_half_even(y), -128, 127)
 *                             QF2_E4M3: code = e4m3(clamp(y, -448, 448))
 * scales[m] = float(scale). */
int qf2_quantize_weight_rows(const void* w, int64_t ldw, int w_dtype, int64_t M, int64_t K, void* q, int64_t ldq,
                             int q_dtype, float* scales, qf2_stream_t stream);
/* Codes -> QF2_BF16 or QF2_F16 values (exact for int8 and e4m3 codes); the fp16 form
 * needs K % 16 == 0 and 16-byte aligned rows. */
int qf2_codes_convert(const void* q, int64_t ldq, int q_dtype, int64_t M, int64_t K, void* out, int64_t ldo,
                      int out_dtype, qf2_stream_t stream);
int qf2_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, void* d, int64_t ldd, int64_t M, int64_t N,
             int64_t K, int ab_dtype, int d_dtype, const float* row_scale, const float* col_scale, const void* bias,
             int bias_dtype, void* workspace, int64_t workspace_bytes, qf2_stream_t stream);
/* qf2_gemm with the DiT block epilogues fused (src/models/flux/mmdit.py:152-160, :226-231):
 * y = (A . B^T) * row_scale * col_scale + bias;  y = gelu_tanh(y) on columns >= gelu_col0
 * (gelu_col0 < 0: none);  D = residual + gate[m / rows_per_gate][n] * y when residual is
 * non-NULL (bf16, row stride ldr; gate bf16 with row stride gate_stride, NULL = 1).
 * D may alias residual.  glu != 0 fuses the SwiGLU of src/models/common/nextdit.py:124-125:
 * B's rows come in groups of 256 = [128 rows of w1 | the matching 128 rows of w3], and
 * D[m, 128 j + i] = silu(y[m, 256 j + i]) * y[m, 256 j + 128 + i] (N % 256 == 0, D has
 * N / 2 bf16 columns, no residual, no GELU). */
int qf2_gemm_ex(const void* a, int64_t lda, const void* b, int64_t ldb, void* d, int64_t ldd, int64_t M, int64_t N,
                int64_t K, int ab_dtype, int d_dtype, const float* row_scale, const float* col_scale,
                const void* bias, int bias_dtype, int64_t gelu_col0, int glu, const void* residual, int64_t ldr,
                const void* gate, int64_t gate_stride, int64_t rows_per_gate, void* workspace,
                int64_t workspace_bytes, qf2_stream_t stream);
/* Weight-only linear on 8-bit weight codes, the compute of the reference's torchao
 * int8 / float8 weight-only linears (src/quant.py:209-241: y = F.linear(x, T(codes)) *
 * scale, T the activation dtype).  A [M, K] is a_dtype (QF2_BF16 or QF2_F16); B [N, K]
 * holds codes of b_dtype (QF2_I8, or QF2_E4M3 as bytes), row stride ldb bytes (a multiple
 * of 16); the kernel converts them in shared memory to exact a_dtype values (every int8
 * and e4m3 code is one), so D equals qf2_gemm_ex(A, a_dtype(codes), ...) bit for bit
 * while reading 1 byte per weight.  Epilogue arguments as qf2_gemm_ex.  The conversion is
 * repeated for every 128-row tile of A: it is the faster route up to M = 128 (the
 * adaLN / embedding linears); for M of thousands qf2_codes_convert once and qf2_gemm_ex
 * take about half the time. */
int qf2_gemm_codes(const void* a, int64_t lda, const void* b_codes, int64_t ldb, int b_dtype, void* d, int64_t ldd,
                   int64_t M, int64_t N, int64_t K, int a_dtype, int d_dtype, const float* row_scale,
                   const float* col_scale, const void* bias, int bias_dtype, int64_t gelu_col0, int glu,
                   const void* residual, int64_t ldr, const void* gate, int64_t gate_stride, int64_t rows_per_gate,
                   void* workspace, int64_t workspace_bytes, qf2_stream_t stream);
/* Row-indexed product of the reference's RAS partial ops (_partially_linear,
 * src/kernels/triton/ras.py:28-128): for each of `batch` blocks of M rows of A (row stride
 * lda; A [batch*M, K]), D[b * out_rows + row_idx[m], :] = A[b*M + m, :] . B^T * col_scale + bias,
 * written to the row-strided D (ldd); rows of D not named by row_idx are left untouched.
 * row_idx: int64 device array of M entries; an entry outside [0, out_rows) is skipped and
 * reported through qf2_workspace_status (QF2_ERR_ARG).  Operands and output dtypes as
 * qf2_gemm (the reference: bf16 x bf16 -> bf16, no scale, no bias). */
int qf2_gemm_rows_indexed(const void* a, int64_t lda, const void* b, int64_t ldb, void* d, int64_t ldd, int64_t batch,
                          int64_t M, int64_t N, int64_t K, int ab_dtype, int d_dtype, const int64_t* row_idx,
                          int64_t out_rows, const float* col_scale, const void* bias, int bias_dtype, void* workspace,
                          int64_t workspace_bytes, qf2_stream_t stream);
/* Fused adaLN input (src/models/flux/mmdit.py:127-128, src/models/common/utilities.py:4-5):
 * y = LayerNorm(x) * (1 + scale[b]) + shift[b] over rows of N (no affine, eps), b = row /
 * rows_per_batch, shift/scale bf16 with row stride mod_stride; out QF2_BF16, or QF2_E4M3
 * with a per-row scale in `scales` (ready for the FP8 GEMM).  N % 8 == 0, N <= 16384. */
int qf2_ln_modulate(const void* x, int64_t ldx, int x_dtype, const void* shift, const void* scale, int64_t mod_stride,
                    int64_t rows_per_batch, int64_t M, int64_t N, float eps, void* out, int64_t ldo, int out_dtype,
                    float* scales, qf2_stream_t stream);

/* Chunk permutation copy: dims[0..3] (dims[3] fastest) index n = d0*d1*d2*d3 chunks
 * of chunk_bytes bytes; chunk (i0, i1, i2, i3) is copied from
 * src + sum_k i_k * src_strides[k] to dst + sum_k i_k * dst_strides[k] (strides in bytes).
 * chunk_bytes, the strides and both pointers must be multiples of 16 (QF2_ERR_ALIGN);
 * source and destination must not overlap.  Used for the layout changes around the
 * head-parallel all-to-all of the multi-GPU DiT step; the reference runs on one GPU and
 * has no counterpart. */
int qf2_copy_chunks(void* dst, const void* src, int64_t chunk_bytes, const int64_t* dims, const int64_t* src_strides,
                    const int64_t* dst_strides, qf2_stream_t stream);

/* No counterpart in the reference.  qf2_sageattn without a caller workspace, for
 * callers that cannot allocate device memory: programs that reserve all device memory
 * in their own pool, code that must avoid the device synchronization an allocation
 * can cause, and bindings that only hold the tensors they pass.  The quantized codes
 * and scales live in one static device array of QF2_SAGE_NOALLOC_SCRATCH_BYTES that
 * every GPU loading the library keeps until the process exits.  Dense form only,
 * same arguments and results as qf2_sageattn; a problem whose workspace
 * (qf2_sage_workspace_bytes) exceeds the array less 1 KiB is rejected with
 * QF2_ERR_WORKSPACE before anything runs (48 MiB holds one 4608-token, 24-head,
 * head_dim 128 sequence).  The first call on a device looks the array's address up
 * for that device (it must be the current device); make that first call before any
 * stream capture.  All calls share the array and leave their contents in it; the
 * status word is cleared at the start of each call.  Calls that overlap on the GPU
 * (different streams, or host threads) race on the array: serialize them.  The array's
 * device address is looked up on every call with the calling thread's current device
 * (after a cudaDeviceReset the next call finds the new address by itself; like the
 * first call on a device, make it outside stream capture). */
#define QF2_SAGE_NOALLOC_SCRATCH_BYTES (48ll << 20)
int qf2_sageattn_noalloc(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                         const void* v, const int64_t* v_strides, void* out, const int64_t* out_strides, int64_t B,
                         int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D, float sm_scale, int dtype,
                         qf2_stream_t stream);
/* Error report of qf2_sageattn_noalloc on the current device: synchronizes `stream`,
 * then returns QF2_ERR_TIMEOUT (and clears the word) if a kernel of the last call gave
 * up a bounded wait, else QF2_OK -- qf2_workspace_status() for the static array, whose
 * address callers do not see.  Call it before the next qf2_sageattn_noalloc call, which
 * clears the word. */
int qf2_sageattn_noalloc_status(qf2_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QF2B200_H */
