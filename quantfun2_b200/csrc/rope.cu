// Rotary position embedding over interleaved pairs (sm_100a).
//
// Replaces rope_apply (src/kernels/__init__.py:126-142) and the Triton body
// rope_kernel_inplace / rope_triton (src/kernels/triton/rope.py:20-134).
// One launch rotates both q and k: the flat index runs over
// (batch, seq, head in [0, Hq + Hk), 16-byte chunk of the head row); each thread
// moves one 16-byte vector (8 bf16/f16 or 4 fp32 elements) with the matching
// complex factors read once per (batch, seq) from freqs_cis.  HBM-bound: every
// element is read once and written once.
#include "qf2_common.cuh"

namespace qf2 {
namespace rope {

struct Side {
  const void* x;
  void* y;
  int64_t sb, ss, sh;     // input strides (elements)
  int64_t ob, os, oh;     // output strides
  int64_t H;
};

template <typename T, int VEC, bool FP16_TRIG>
__global__ void __launch_bounds__(256) rope_kernel(Side q, Side k, const float2* __restrict__ freqs, int64_t fsb,
                                                   int64_t fss, int64_t B, int64_t S, int64_t D) {
  const int64_t chunks = D / VEC;
  const int64_t H = q.H + k.H;
  const int64_t total = B * S * H * chunks;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = idx;
    const int64_t c = t % chunks; t /= chunks;
    const int64_t h = t % H; t /= H;
    const int64_t s = t % S;
    const int64_t b = t / S;
    const bool is_q = h < q.H;
    const Side& sd = is_q ? q : k;
    const int64_t hh = is_q ? h : h - q.H;
    const T* src = reinterpret_cast<const T*>(sd.x) + b * sd.sb + s * sd.ss + hh * sd.sh + c * VEC;
    T* dst = reinterpret_cast<T*>(sd.y) + b * sd.ob + s * sd.os + hh * sd.oh + c * VEC;
    const float2* f = freqs + b * fsb + s * fss + c * (VEC / 2);

    T in[VEC];
    if constexpr (VEC * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(in) = *reinterpret_cast<const uint4*>(src);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) in[i] = src[i];
    }
    T out[VEC];
#pragma unroll
    for (int p = 0; p < VEC / 2; ++p) {
      float2 cs = __ldg(f + p);
      if (FP16_TRIG) {
        cs.x = __half2float(__float2half_rn(cs.x));
        cs.y = __half2float(__float2half_rn(cs.y));
      }
      const float x0 = to_f32(in[2 * p]), x1 = to_f32(in[2 * p + 1]);
      // (x0 + i x1) * (c + i s), each product rounded separately
      const float re = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
      const float im = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
      out[2 * p] = from_f32<T>(re);
      out[2 * p + 1] = from_f32<T>(im);
    }
    if constexpr (VEC * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(out);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) dst[i] = out[i];
    }
  }
}

template <typename T, int VEC>
static void launch(const Side& q, const Side& k, const float2* f, int64_t fsb, int64_t fss, int64_t B, int64_t S,
                   int64_t D, bool fp16_trig, cudaStream_t st) {
  const int64_t total = B * S * (q.H + k.H) * (D / VEC);
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 64) blocks = 148 * 64;  // grid-stride beyond 64 CTAs per SM
  if (blocks < 1) blocks = 1;
  if (fp16_trig)
    rope_kernel<T, VEC, true><<<(unsigned)blocks, threads, 0, st>>>(q, k, f, fsb, fss, B, S, D);
  else
    rope_kernel<T, VEC, false><<<(unsigned)blocks, threads, 0, st>>>(q, k, f, fsb, fss, B, S, D);
}

static bool al(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace rope
}  // namespace qf2

extern "C" int qf2_rope_apply(const void* xq, void* xq_out, int64_t Hq, const int64_t* xq_strides,
                              const int64_t* xq_out_strides, const void* xk, void* xk_out, int64_t Hk,
                              const int64_t* xk_strides, const int64_t* xk_out_strides, const void* freqs_cis,
                              const int64_t* freqs_strides, int64_t B, int64_t S, int64_t D, int dtype, int flags,
                              qf2_stream_t stream) {
  using namespace qf2::rope;
  if (!xq || !xq_out || !xq_strides || !xq_out_strides || !freqs_cis || !freqs_strides) return QF2_ERR_ARG;
  if (B < 0 || S < 0 || Hq < 0 || D <= 0 || (D & 1)) return QF2_ERR_SHAPE;
  const bool has_k = xk != nullptr && Hk > 0;
  if (has_k && (!xk_out || !xk_strides || !xk_out_strides)) return QF2_ERR_ARG;
  if (B == 0 || S == 0) return QF2_OK;
  Side q{xq, xq_out, xq_strides[0], xq_strides[1], xq_strides[2],
         xq_out_strides[0], xq_out_strides[1], xq_out_strides[2], Hq};
  Side k{nullptr, nullptr, 0, 0, 0, 0, 0, 0, 0};
  if (has_k)
    k = Side{xk, xk_out, xk_strides[0], xk_strides[1], xk_strides[2],
             xk_out_strides[0], xk_out_strides[1], xk_out_strides[2], Hk};
  const float2* f = reinterpret_cast<const float2*>(freqs_cis);
  if (!al(f, 8)) return QF2_ERR_ALIGN;
  const bool fp16 = (flags & QF2_ROPE_FP16_TRIG) != 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int esz;
  switch (dtype) {
    case QF2_F32: esz = 4; break;
    case QF2_F16: case QF2_BF16: esz = 2; break;
    default: return QF2_ERR_DTYPE;
  }
  // 16-byte vector path when every row start is 16-byte aligned
  const int vec16 = 16 / esz;
  bool vec_ok = (D % vec16) == 0 && al(xq, 16) && al(xq_out, 16);
  const int64_t* all_strides[4] = {xq_strides, xq_out_strides, xk_strides, xk_out_strides};
  for (int i = 0; i < (has_k ? 4 : 2); ++i)
    for (int j = 0; j < 3; ++j) vec_ok = vec_ok && ((all_strides[i][j] * esz) % 16 == 0);
  if (has_k) vec_ok = vec_ok && al(xk, 16) && al(xk_out, 16);
  if (dtype == QF2_F32) {
    if (vec_ok) launch<float, 4>(q, k, f, freqs_strides[0], freqs_strides[1], B, S, D, fp16, st);
    else launch<float, 2>(q, k, f, freqs_strides[0], freqs_strides[1], B, S, D, fp16, st);
  } else if (dtype == QF2_BF16) {
    if (vec_ok) launch<__nv_bfloat16, 8>(q, k, f, freqs_strides[0], freqs_strides[1], B, S, D, fp16, st);
    else launch<__nv_bfloat16, 2>(q, k, f, freqs_strides[0], freqs_strides[1], B, S, D, fp16, st);
  } else {
    if (vec_ok) launch<__half, 8>(q, k, f, freqs_strides[0], freqs_strides[1], B, S, D, fp16, st);
    else launch<__half, 2>(q, k, f, freqs_strides[0], freqs_strides[1], B, S, D, fp16, st);
  }
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}

// ------------------------------------------------ fused QK RMSNorm + RoPE --
// Replaces the per-head q_norm / k_norm (src/models/flux/mmdit.py:133-134,
// src/models/common/attn.py:209-210) followed by rope_apply (:149 / :212): one pass over
// the fused QKV projection output [rows, (Hq + 2*Hkv)*D] (row = b * L + s; q heads, then
// k heads, then v heads).  q and k rows get y = x * rsqrt(mean(x^2) + eps) * w (fp32)
// rotated by freqs[b, s, :], then rounded once; v rows are copied.  Outputs are written
// through {batch, seq, head} strides with head dim Dout >= D (columns D..Dout-1 zero),
// so they can land inside a larger joint-sequence buffer and be padded to the
// attention kernel's head dim.
namespace qf2 {
namespace rope {

struct QkvDst {
  __nv_bfloat16* p[3];
  int64_t sb[3], ss[3], sh[3];
};

// One CTA per token row: 16 groups of 16 lanes; group g handles head rows g, g + 16, ...
// (up to 8 passes, Hq + 2 Hkv <= 128), lane `sub` holds 8 elements of its head row.  The
// token's RoPE factors and the q / k norm weights are per-lane constants loaded once; all
// of the row's loads are issued before any arithmetic.
constexpr int kQkvPasses = 8;

QF2_DEV void unpack_bf16x8(const uint4& v, float* f) {
  const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = __bfloat162float(e[j]);
}

template <int NP>
__global__ void __launch_bounds__(256, 4) qkv_norm_rope_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld,
                                                            int64_t rows, int64_t L, int Hq, int Hkv, int D, int Dout,
                                                            QkvDst dst, const __nv_bfloat16* __restrict__ qw,
                                                            const __nv_bfloat16* __restrict__ kw, float eps,
                                                            const float2* __restrict__ freqs, int64_t fb, int64_t fs) {
  const int sub = threadIdx.x & 15, grp = threadIdx.x >> 4;
  const int Ht = Hq + 2 * Hkv;
  const int npass = (Ht + 15) >> 4;
  const int64_t row = blockIdx.x;
  const uint32_t b32 = (uint32_t)row / (uint32_t)L;
  const int64_t b = b32, s = (int64_t)((uint32_t)row - b32 * (uint32_t)L);
  const int nin = D / 8, nout = Dout / 8;
  const bool lane_in = sub < nin;
  uint4 raw[NP];
#pragma unroll
  for (int u = 0; u < NP; ++u) {
    const int hr = grp + 16 * u;
    raw[u] = (u < npass && hr < Ht && lane_in)
                 ? *reinterpret_cast<const uint4*>(qkv + row * ld + (int64_t)hr * D + sub * 8)
                 : make_uint4(0, 0, 0, 0);
  }
  float2 cs[4];
  uint4 wq = make_uint4(0, 0, 0, 0), wk = make_uint4(0, 0, 0, 0);
  if (lane_in) {
    const float2* f = freqs + b * fb + s * fs + sub * 4;
#pragma unroll
    for (int p = 0; p < 4; ++p) cs[p] = __ldg(f + p);
    wq = __ldg(reinterpret_cast<const uint4*>(qw + sub * 8));
    wk = __ldg(reinterpret_cast<const uint4*>(kw + sub * 8));
  } else {
#pragma unroll
    for (int p = 0; p < 4; ++p) cs[p] = make_float2(0.f, 0.f);
  }
#pragma unroll
  for (int u = 0; u < NP; ++u) {
    if (u >= npass) break;  // CTA-uniform: every lane reaches the shuffles below
    const int hr = grp + 16 * u;
    float x[8];
    unpack_bf16x8(raw[u], x);
    float ss_ = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss_ = fmaf(x[j], x[j], ss_);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss_ += __shfl_xor_sync(0xffffffffu, ss_, o, 16);
    if (hr >= Ht || sub >= nout) continue;
    const int kind = hr < Hq ? 0 : (hr < Hq + Hkv ? 1 : 2);
    const int head = kind == 0 ? hr : (kind == 1 ? hr - Hq : hr - Hq - Hkv);
    uint4 outv = raw[u];  // zeros on the padding lanes
    if (kind != 2 && lane_in) {
      const float r = __frsqrt_rn(ss_ / (float)D + eps);
      float w[8];
      unpack_bf16x8(kind == 0 ? wq : wk, w);
      uint32_t* op = reinterpret_cast<uint32_t*>(&outv);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float x0 = x[2 * p] * r * w[2 * p];
        const float x1 = x[2 * p + 1] * r * w[2 * p + 1];
        const float re = __fsub_rn(__fmul_rn(x0, cs[p].x), __fmul_rn(x1, cs[p].y));
        const float im = __fadd_rn(__fmul_rn(x0, cs[p].y), __fmul_rn(x1, cs[p].x));
        __nv_bfloat162 t = __floats2bfloat162_rn(re, im);
        op[p] = *reinterpret_cast<uint32_t*>(&t);
      }
    }
    // select by kind without indexing the parameter arrays (keeps them out of local memory)
    __nv_bfloat16* d = kind == 0 ? dst.p[0] + b * dst.sb[0] + s * dst.ss[0] + (int64_t)head * dst.sh[0]
                     : kind == 1 ? dst.p[1] + b * dst.sb[1] + s * dst.ss[1] + (int64_t)head * dst.sh[1]
                                 : dst.p[2] + b * dst.sb[2] + s * dst.ss[2] + (int64_t)head * dst.sh[2];
    *reinterpret_cast<uint4*>(d + sub * 8) = outv;
  }
}

}  // namespace rope
}  // namespace qf2

extern "C" int qf2_qkv_norm_rope(const void* qkv, int64_t qkv_row_stride, int64_t B, int64_t L, int64_t Hq,
                                 int64_t Hkv, int64_t D, int64_t Dout, void* q_out, const int64_t* q_strides,
                                 void* k_out, const int64_t* k_strides, void* v_out, const int64_t* v_strides,
                                 const void* q_weight, const void* k_weight, float eps, const void* freqs_cis,
                                 const int64_t* freqs_strides, qf2_stream_t stream) {
  using namespace qf2::rope;
  if (!qkv || !q_out || !k_out || !v_out || !q_strides || !k_strides || !v_strides || !q_weight || !k_weight ||
      !freqs_cis || !freqs_strides)
    return QF2_ERR_ARG;
  if (D % 8 || D <= 0 || D > 128 || Dout < D || Dout % 8 || Dout > 128 || B <= 0 || L <= 0 || Hq <= 0 || Hkv <= 0)
    return QF2_ERR_SHAPE;
  if (qkv_row_stride < (Hq + 2 * Hkv) * D || qkv_row_stride % 8) return QF2_ERR_ALIGN;
  const void* ps[4] = {qkv, q_out, k_out, v_out};
  for (const void* p : ps)
    if (!al(p, 16)) return QF2_ERR_ALIGN;
  if (!al(q_weight, 16) || !al(k_weight, 16) || !al(freqs_cis, 16)) return QF2_ERR_ALIGN;
  QkvDst dst;
  const int64_t* st[3] = {q_strides, k_strides, v_strides};
  void* outs[3] = {q_out, k_out, v_out};
  for (int i = 0; i < 3; ++i) {
    dst.p[i] = reinterpret_cast<__nv_bfloat16*>(outs[i]);
    dst.sb[i] = st[i][0]; dst.ss[i] = st[i][1]; dst.sh[i] = st[i][2];
    if ((dst.sb[i] % 8) || (dst.ss[i] % 8) || (dst.sh[i] % 8)) return QF2_ERR_ALIGN;
  }
  if (freqs_strides[0] % 2 || freqs_strides[1] % 2) return QF2_ERR_ALIGN;
  const int64_t rows = B * L;
  const int64_t units = rows * (Hq + 2 * Hkv);
  if (units >= (int64_t)1 << 31 || L >= (int64_t)1 << 31) return QF2_ERR_SHAPE;
  if (Hq + 2 * Hkv > 16 * kQkvPasses) return QF2_ERR_SHAPE;
  const int npass = (int)((Hq + 2 * Hkv + 15) / 16);
  auto kern = npass <= 3 ? qkv_norm_rope_kernel<3> : npass <= 5 ? qkv_norm_rope_kernel<5> : qkv_norm_rope_kernel<8>;
  kern<<<(unsigned)rows, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv), qkv_row_stride, rows, L, (int)Hq, (int)Hkv, (int)D, (int)Dout, dst,
      reinterpret_cast<const __nv_bfloat16*>(q_weight), reinterpret_cast<const __nv_bfloat16*>(k_weight), eps,
      reinterpret_cast<const float2*>(freqs_cis), freqs_strides[0], freqs_strides[1]);
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}

// ------------------------------------------------------- RoPE with row scatter --
// The RoPE of the reference's RAS partial ops (PYCUDA_ROPE_KERNEL, src/kernels/cuda/ras.cu:
// 12-52): y[b, idx[n], h, :] = x[b, n, h, :] rotated by f[n] (interleaved pairs times the
// complex f[n, p], fp32 products, each pair rounded to bf16).  One warp per (b, n) row of
// H * D elements, 8 elements (4 pairs) per 16-byte vector; rows of y not named by idx are
// left untouched; an index outside [0, M) skips its row and sets the status word.
// The complex product is rounded step by step (no fused multiply-add): re = x0 f0 - x1 f1,
// im = x0 f1 + x1 f0, each product and the sum rounded to fp32.
namespace qf2 {
namespace rope {

struct ScatterArgs {
  const __nv_bfloat16* x;
  const float* f;
  const int64_t* idx;
  __nv_bfloat16* y;
  int64_t xb, xn, xh;   // x strides (elements)
  int64_t yb, ym, yh;   // y strides (elements)
  int64_t fn;           // f stride per n (floats)
  int64_t B, N, M;
  int H, D;
  int* status;
};

__global__ void __launch_bounds__(256) rope_scatter_kernel(ScatterArgs A) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= A.B * A.N) return;
  const int lane = threadIdx.x & 31;
  const int64_t b = row / A.N, n = row - b * A.N;
  const int64_t m = A.idx[n];
  if (m < 0 || m >= A.M) {
    if (lane == 0 && A.status) atomicExch(A.status, kDevBadIndex);
    return;
  }
  const int vpr = A.D / 8;               // vectors per head row
  const int nvec = A.H * vpr;
  for (int v = lane; v < nvec; v += 32) {
    const int h = v / vpr, d = (v - h * vpr) * 8;
    const uint4 raw = *reinterpret_cast<const uint4*>(A.x + b * A.xb + n * A.xn + h * A.xh + d);
    const float4 f01 = *reinterpret_cast<const float4*>(A.f + n * A.fn + d);
    const float4 f23 = *reinterpret_cast<const float4*>(A.f + n * A.fn + d + 4);
    const float fr[8] = {f01.x, f01.y, f01.z, f01.w, f23.x, f23.y, f23.z, f23.w};
    const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&raw);
    uint4 out;
    __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float2 a = __bfloat1622float2(xp[p]);
      const float c = fr[2 * p], sn = fr[2 * p + 1];
      const float re = __fsub_rn(__fmul_rn(a.x, c), __fmul_rn(a.y, sn));
      const float im = __fadd_rn(__fmul_rn(a.x, sn), __fmul_rn(a.y, c));
      op[p] = __floats2bfloat162_rn(re, im);
    }
    *reinterpret_cast<uint4*>(A.y + b * A.yb + m * A.ym + h * A.yh + d) = out;
  }
}

}  // namespace rope
}  // namespace qf2

extern "C" int qf2_rope_scatter(const void* x, const int64_t* x_strides, const float* f, int64_t f_stride,
                                const int64_t* idx, void* y, const int64_t* y_strides, int64_t B, int64_t N,
                                int64_t M, int64_t H, int64_t D, int dtype, void* workspace, qf2_stream_t stream) {
  using namespace qf2::rope;
  if (!x || !x_strides || !f || !idx || !y || !y_strides) return QF2_ERR_ARG;
  if (dtype != QF2_BF16) return QF2_ERR_DTYPE;
  if (B < 0 || N < 0 || M < 0 || H <= 0 || D <= 0 || D % 8 || H * D > (1 << 24)) return QF2_ERR_SHAPE;
  if (B == 0 || N == 0) return QF2_OK;
  const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                       reinterpret_cast<uintptr_t>(f);
  if ((al & 15) || (f_stride % 4)) return QF2_ERR_ALIGN;
  for (int i = 0; i < 3; ++i)
    if ((x_strides[i] % 8) || (y_strides[i] % 8)) return QF2_ERR_ALIGN;
  ScatterArgs A;
  A.x = reinterpret_cast<const __nv_bfloat16*>(x);
  A.f = f;
  A.idx = idx;
  A.y = reinterpret_cast<__nv_bfloat16*>(y);
  A.xb = x_strides[0]; A.xn = x_strides[1]; A.xh = x_strides[2];
  A.yb = y_strides[0]; A.ym = y_strides[1]; A.yh = y_strides[2];
  A.fn = f_stride;
  A.B = B; A.N = N; A.M = M;
  A.H = (int)H; A.D = (int)D;
  A.status = reinterpret_cast<int*>(workspace);
  const int64_t blocks = (B * N + 7) / 8;
  if (blocks > 2147483647ll) return QF2_ERR_SHAPE;
  rope_scatter_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(A);
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}
