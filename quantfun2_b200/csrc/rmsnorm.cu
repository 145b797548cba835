// Row RMSNorm (sm_100a).
//
// Replaces rmsnorm_apply (src/kernels/__init__.py:73-80) and the Triton
// rms_norm_kernel / apply_rmsnorm (src/kernels/triton/rmsnorm.py:22-95).
// A group of LPR lanes owns one row; each lane keeps its slice of the row in
// registers (16-byte vectors), so x is read from HBM exactly once.  Sum of
// squares in fp32, warp-shuffle reduction, rsqrt correctly rounded.
// Rows too long for registers take a two-pass path (second read hits L2).
#include "qf2_common.cuh"

namespace qf2 {
namespace rms {

template <typename T>
QF2_DEV void load_vec(const T* p, float* f, int n) {
  // n elements (16 bytes) -> fp32
  if constexpr (sizeof(T) == 4) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
  } else {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = to_f32(e[i]);
  }
}

template <typename T>
QF2_DEV void store_vec(T* p, const float* f) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  } else {
    uint4 v;
    T* e = reinterpret_cast<T*>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(f[i]);
    *reinterpret_cast<uint4*>(p) = v;
  }
}

template <typename T>
QF2_DEV float round_to(float v) { return to_f32(from_f32<T>(v)); }

// V weights starting at element i as fp32: 16-byte vector loads when the weight is aligned
template <typename TW, int V>
QF2_DEV void load_w(const TW* w, int64_t i, bool vec, float* f) {
  if (vec && sizeof(TW) * V % 16 == 0) {
#pragma unroll
    for (int b = 0; b < (int)(sizeof(TW) * V / 16); ++b) {
      const uint4 r = __ldg(reinterpret_cast<const uint4*>(w + i) + b);
      const TW* e = reinterpret_cast<const TW*>(&r);
#pragma unroll
      for (int j = 0; j < (int)(16 / sizeof(TW)); ++j) f[b * (16 / sizeof(TW)) + j] = to_f32(e[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < V; ++j) f[j] = to_f32(w[i + j]);
  }
}

// EAGER: y = round_O( float(round_X(x * r)) * w );  FUSED: y = round_O((x * r) * w)
template <typename TX, typename TW, typename TO, int LPR, int MAXC, bool EAGER>
__global__ void __launch_bounds__(256) rmsnorm_reg_kernel(const TX* __restrict__ x, int64_t xs, const TW* __restrict__ w,
                                                          TO* __restrict__ y, int64_t ys, int64_t M, int64_t N, float eps,
                                                          int w_vec) {
  constexpr int V = 16 / sizeof(TX);
  const int64_t nvec = N / V;
  const int rows_per_block = blockDim.x / LPR;
  const int sub = threadIdx.x % LPR;
  for (int64_t row = (int64_t)blockIdx.x * rows_per_block + threadIdx.x / LPR; row < M;
       row += (int64_t)gridDim.x * rows_per_block) {
    const TX* xr = x + row * xs;
    float v[MAXC][V];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      const int64_t vi = sub + (int64_t)c * LPR;
      if (vi < nvec) {
        load_vec(xr + vi * V, v[c], V);
#pragma unroll
        for (int i = 0; i < V; ++i) ss = fmaf(v[c][i], v[c][i], ss);
      }
    }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o, LPR);
    const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)N), eps));
    TO* yr = y + row * ys;
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      const int64_t vi = sub + (int64_t)c * LPR;
      if (vi < nvec) {
        float o[V], wv[V];
        load_w<TW, V>(w, vi * V, w_vec != 0, wv);
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const float n = __fmul_rn(v[c][i], r);
          o[i] = EAGER ? __fmul_rn(round_to<TX>(n), wv[i]) : __fmul_rn(n, wv[i]);
        }
        if constexpr (sizeof(TO) == sizeof(TX)) {
          store_vec(yr + vi * V, o);
        } else {
#pragma unroll
          for (int i = 0; i < V; ++i) yr[vi * V + i] = from_f32<TO>(o[i]);
        }
      }
    }
  }
}

// Scalar two-pass fallback: any N, any alignment.  One warp per row.
template <typename TX, typename TW, typename TO, bool EAGER>
__global__ void __launch_bounds__(256) rmsnorm_generic_kernel(const TX* __restrict__ x, int64_t xs,
                                                              const TW* __restrict__ w, TO* __restrict__ y, int64_t ys,
                                                              int64_t M, int64_t N, float eps) {
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x / 32;
  for (int64_t row = (int64_t)blockIdx.x * wpb + threadIdx.x / 32; row < M; row += (int64_t)gridDim.x * wpb) {
    const TX* xr = x + row * xs;
    float ss = 0.f;
    for (int64_t i = lane; i < N; i += 32) {
      const float v = to_f32(xr[i]);
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)N), eps));
    TO* yr = y + row * ys;
    for (int64_t i = lane; i < N; i += 32) {
      const float n = __fmul_rn(to_f32(xr[i]), r);
      const float wv = to_f32(w[i]);
      yr[i] = from_f32<TO>(EAGER ? __fmul_rn(round_to<TX>(n), wv) : __fmul_rn(n, wv));
    }
  }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename TX, typename TW, typename TO, bool EAGER>
static void dispatch(const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t M, int64_t N, float eps,
                     cudaStream_t st) {
  constexpr int V = 16 / sizeof(TX);
  const TX* X = reinterpret_cast<const TX*>(x);
  const TW* W = reinterpret_cast<const TW*>(w);
  TO* Y = reinterpret_cast<TO*>(y);
  const bool vec_ok = (N % V) == 0 && al16(x) && al16(y) && ((xs * (int64_t)sizeof(TX)) % 16) == 0 &&
                      ((ys * (int64_t)sizeof(TO)) % 16) == 0 && (sizeof(TO) == sizeof(TX) || true);
  const int64_t nvec = N / V;
  auto grid_for = [&](int rows_per_block) {
    int64_t g = (M + rows_per_block - 1) / rows_per_block;
    if (g > 148 * 16) g = 148 * 16;
    return (unsigned)(g < 1 ? 1 : g);
  };
  const int wv = al16(w) ? 1 : 0;
  // a warp per row for wide rows, the per-lane register tile sized to the row (one HBM read)
  if (vec_ok && nvec <= 8) {
    rmsnorm_reg_kernel<TX, TW, TO, 8, 1, EAGER><<<grid_for(32), 256, 0, st>>>(X, xs, W, Y, ys, M, N, eps, wv);
  } else if (vec_ok && nvec <= 16) {
    rmsnorm_reg_kernel<TX, TW, TO, 16, 1, EAGER><<<grid_for(16), 256, 0, st>>>(X, xs, W, Y, ys, M, N, eps, wv);
  } else if (vec_ok && nvec <= 32 * 4) {
    rmsnorm_reg_kernel<TX, TW, TO, 32, 4, EAGER><<<grid_for(8), 256, 0, st>>>(X, xs, W, Y, ys, M, N, eps, wv);
  } else if (vec_ok && nvec <= 32 * 9) {
    rmsnorm_reg_kernel<TX, TW, TO, 32, 9, EAGER><<<grid_for(8), 256, 0, st>>>(X, xs, W, Y, ys, M, N, eps, wv);
  } else if (vec_ok && nvec <= 32 * 16) {
    rmsnorm_reg_kernel<TX, TW, TO, 32, 16, EAGER><<<grid_for(8), 256, 0, st>>>(X, xs, W, Y, ys, M, N, eps, wv);
  } else {
    rmsnorm_generic_kernel<TX, TW, TO, EAGER><<<grid_for(8), 256, 0, st>>>(X, xs, W, Y, ys, M, N, eps);
  }
}

template <typename TX, typename TW, bool EAGER>
static int by_out(int od, const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t M, int64_t N,
                  float eps, cudaStream_t st) {
  switch (od) {
    case QF2_F32: dispatch<TX, TW, float, EAGER>(x, xs, w, y, ys, M, N, eps, st); return QF2_OK;
    case QF2_F16: dispatch<TX, TW, __half, EAGER>(x, xs, w, y, ys, M, N, eps, st); return QF2_OK;
    case QF2_BF16: dispatch<TX, TW, __nv_bfloat16, EAGER>(x, xs, w, y, ys, M, N, eps, st); return QF2_OK;
  }
  return QF2_ERR_DTYPE;
}

template <typename TX, bool EAGER>
static int by_w(int wd, int od, const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t M, int64_t N,
                float eps, cudaStream_t st) {
  switch (wd) {
    case QF2_F32: return by_out<TX, float, EAGER>(od, x, xs, w, y, ys, M, N, eps, st);
    case QF2_F16: return by_out<TX, __half, EAGER>(od, x, xs, w, y, ys, M, N, eps, st);
    case QF2_BF16: return by_out<TX, __nv_bfloat16, EAGER>(od, x, xs, w, y, ys, M, N, eps, st);
  }
  return QF2_ERR_DTYPE;
}

template <bool EAGER>
static int by_x(int xd, int wd, int od, const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t M,
                int64_t N, float eps, cudaStream_t st) {
  switch (xd) {
    case QF2_F32: return by_w<float, EAGER>(wd, od, x, xs, w, y, ys, M, N, eps, st);
    case QF2_F16: return by_w<__half, EAGER>(wd, od, x, xs, w, y, ys, M, N, eps, st);
    case QF2_BF16: return by_w<__nv_bfloat16, EAGER>(wd, od, x, xs, w, y, ys, M, N, eps, st);
  }
  return QF2_ERR_DTYPE;
}

}  // namespace rms
}  // namespace qf2

extern "C" int qf2_rmsnorm(const void* x, int64_t x_row_stride, int x_dtype, const void* weight, int w_dtype, void* out,
                           int64_t out_row_stride, int out_dtype, int64_t M, int64_t N, float eps, int mode,
                           qf2_stream_t stream) {
  if (!x || !weight || !out) return QF2_ERR_ARG;
  if (M < 0 || N <= 0) return QF2_ERR_SHAPE;
  if (mode != QF2_RMS_EAGER && mode != QF2_RMS_FUSED) return QF2_ERR_ARG;
  if (M == 0) return QF2_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int r = mode == QF2_RMS_EAGER
                    ? qf2::rms::by_x<true>(x_dtype, w_dtype, out_dtype, x, x_row_stride, weight, out, out_row_stride, M,
                                           N, eps, st)
                    : qf2::rms::by_x<false>(x_dtype, w_dtype, out_dtype, x, x_row_stride, weight, out, out_row_stride,
                                            M, N, eps, st);
  if (r != QF2_OK) return r;
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}

// ------------------------------------------- gated residual + RMSNorm modulate --
// The glue of the Lumina joint block (src/models/lumina/image_two/model.py:82-101):
//   x = x + g * RMSNorm_post(y)          g = tanh(gate[b]) (or gate, or 1)
//   h = RMSNorm_pre(x) * (1 + scale[b])  (the next linear's input)
// in one pass: one CTA per row, one 8-element (16-byte) vector of y and x per thread
// (dim / 8 threads), sums of squares reduced through shared memory; x is rounded to bf16
// once and stored, h is computed from that rounded x (as the reference's next norm sees
// it) and stored.  Math in fp32.
namespace qf2 {
namespace rms {

struct GateResArgs {
  const __nv_bfloat16* y;
  __nv_bfloat16* x;
  __nv_bfloat16* h;
  int64_t rows, rows_per_batch;
  int dim;
  const __nv_bfloat16* w_post;
  float eps_post;
  const __nv_bfloat16* gate;
  int64_t gate_stride;
  int gate_tanh;
  const __nv_bfloat16* w_pre;
  float eps_pre;
  const __nv_bfloat16* scale;
  int64_t scale_stride;
};

QF2_DEV void ld8(const __nv_bfloat16* p, float* f) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = __bfloat162float(e[i]);
}

QF2_DEV void st8(__nv_bfloat16* p, const float* f) {
  uint4 v;
  uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 t = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&t);
  }
  *reinterpret_cast<uint4*>(p) = v;
}

// sum over the CTA (blockDim.x a multiple of 32, <= 1024); `red` holds 32 floats
QF2_DEV float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

__global__ void __launch_bounds__(1024) gate_residual_kernel(GateResArgs a) {
  __shared__ float red[2][32];
  const int64_t row = blockIdx.x;
  const int64_t b = row / a.rows_per_batch;
  const int c = threadIdx.x * 8;
  float xv[8];
  ld8(a.x + row * a.dim + c, xv);
  if (a.y != nullptr) {
    float yv[8], w[8], g[8];
    ld8(a.y + row * a.dim + c, yv);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(yv[j], yv[j], ss);
    if (a.w_post != nullptr) {
      ld8(a.w_post + c, w);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = 1.0f;
    }
    if (a.gate != nullptr) {
      ld8(a.gate + b * a.gate_stride + c, g);
      if (a.gate_tanh) {
#pragma unroll
        for (int j = 0; j < 8; ++j) asm("tanh.approx.f32 %0, %1;" : "=f"(g[j]) : "f"(g[j]));  // ~2^-11 rel.
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) g[j] = 1.0f;
    }
    const float tot = block_sum(ss, red[0]);
    const float r = a.w_post != nullptr ? __frsqrt_rn(tot / (float)a.dim + a.eps_post) : 1.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) xv[j] = __bfloat162float(__float2bfloat16_rn(fmaf(g[j], yv[j] * r * w[j], xv[j])));
    st8(a.x + row * a.dim + c, xv);
  }
  if (a.h != nullptr) {
    float w[8], sc[8], o[8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(xv[j], xv[j], ss);
    if (a.w_pre != nullptr) {
      ld8(a.w_pre + c, w);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = 1.0f;
    }
    if (a.scale != nullptr) {
      ld8(a.scale + b * a.scale_stride + c, sc);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) sc[j] = 0.0f;
    }
    const float tot = block_sum(ss, red[1]);
    const float r = __frsqrt_rn(tot / (float)a.dim + a.eps_pre);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = xv[j] * r * w[j] * (1.0f + sc[j]);
    st8(a.h + row * a.dim + c, o);
  }
}

// One warp per row (dim = NV * 256): y is read once into registers for its sum of squares,
// the updated x is kept packed (bf16) for the second norm, and the per-channel vectors
// (weights, gate, scale) come from L1.  No CTA-wide barrier.
QF2_DEV float warp_sum32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int NV>
__global__ void __launch_bounds__(256, 2) gate_residual_warp_kernel(GateResArgs a) {
  constexpr int D = NV * 256;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const int64_t b = row / a.rows_per_batch;
  uint4 xn[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) xn[i] = *reinterpret_cast<const uint4*>(a.x + row * D + (i * 32 + lane) * 8);
  if (a.y != nullptr) {
    uint4 yr[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) yr[i] = *reinterpret_cast<const uint4*>(a.y + row * D + (i * 32 + lane) * 8);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&yr[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(__bfloat162float(e[j]), __bfloat162float(e[j]), ss);
    }
    const float r = a.w_post != nullptr ? __frsqrt_rn(warp_sum32(ss) / (float)D + a.eps_post) : 1.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      float xv[8], yv[8], w[8], g[8];
      const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&xn[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) xv[j] = __bfloat162float(xe[j]);
      const __nv_bfloat16* ye = reinterpret_cast<const __nv_bfloat16*>(&yr[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) yv[j] = __bfloat162float(ye[j]);
      if (a.w_post != nullptr) {
        ld8(a.w_post + c, w);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j] = 1.0f;
      }
      if (a.gate != nullptr) {
        ld8(a.gate + b * a.gate_stride + c, g);
        if (a.gate_tanh) {
#pragma unroll
          for (int j = 0; j < 8; ++j) asm("tanh.approx.f32 %0, %1;" : "=f"(g[j]) : "f"(g[j]));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = 1.0f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) xv[j] = fmaf(g[j], yv[j] * r * w[j], xv[j]);
      uint32_t* wp = reinterpret_cast<uint32_t*>(&xn[i]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __nv_bfloat162 t = __floats2bfloat162_rn(xv[2 * q], xv[2 * q + 1]);
        wp[q] = *reinterpret_cast<uint32_t*>(&t);
      }
      *reinterpret_cast<uint4*>(a.x + row * D + c) = xn[i];
    }
  }
  if (a.h != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&xn[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(__bfloat162float(e[j]), __bfloat162float(e[j]), ss);
    }
    const float r = __frsqrt_rn(warp_sum32(ss) / (float)D + a.eps_pre);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = (i * 32 + lane) * 8;
      float xv[8], w[8], sc[8], o[8];
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&xn[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) xv[j] = __bfloat162float(e[j]);
      if (a.w_pre != nullptr) {
        ld8(a.w_pre + c, w);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j] = 1.0f;
      }
      if (a.scale != nullptr) {
        ld8(a.scale + b * a.scale_stride + c, sc);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) sc[j] = 0.0f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = xv[j] * r * w[j] * (1.0f + sc[j]);
      st8(a.h + row * D + c, o);
    }
  }
}

}  // namespace rms
}  // namespace qf2

extern "C" int qf2_rms_gate_residual(const void* y, void* x, void* h, int64_t rows, int64_t dim,
                                     int64_t rows_per_batch, const void* w_post, float eps_post, const void* gate,
                                     int64_t gate_stride, int gate_tanh, const void* w_pre, float eps_pre,
                                     const void* scale, int64_t scale_stride, qf2_stream_t stream) {
  using namespace qf2::rms;
  if (!x || (!y && !h)) return QF2_ERR_ARG;
  if (rows < 0 || dim <= 0 || dim % 256 || dim > 8192 || rows_per_batch <= 0) return QF2_ERR_SHAPE;
  if (rows == 0) return QF2_OK;
  const void* ps[] = {y, x, h, w_post, gate, w_pre, scale};
  for (const void* p : ps)
    if (p && (reinterpret_cast<uintptr_t>(p) & 15)) return QF2_ERR_ALIGN;
  if ((gate && gate_stride % 8) || (scale && scale_stride % 8)) return QF2_ERR_ALIGN;
  GateResArgs a;
  a.y = reinterpret_cast<const __nv_bfloat16*>(y);
  a.x = reinterpret_cast<__nv_bfloat16*>(x);
  a.h = reinterpret_cast<__nv_bfloat16*>(h);
  a.rows = rows;
  a.rows_per_batch = rows_per_batch;
  a.w_post = reinterpret_cast<const __nv_bfloat16*>(w_post);
  a.eps_post = eps_post;
  a.gate = reinterpret_cast<const __nv_bfloat16*>(gate);
  a.gate_stride = gate_stride;
  a.gate_tanh = gate_tanh;
  a.w_pre = reinterpret_cast<const __nv_bfloat16*>(w_pre);
  a.eps_pre = eps_pre;
  a.scale = reinterpret_cast<const __nv_bfloat16*>(scale);
  a.scale_stride = scale_stride;
  a.dim = (int)dim;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (rows > 0x7fffffff) return QF2_ERR_SHAPE;
  switch (dim / 256) {
    case 8: gate_residual_warp_kernel<8><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(a); break;
    case 9: gate_residual_warp_kernel<9><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(a); break;
    case 12: gate_residual_warp_kernel<12><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(a); break;
    default: gate_residual_kernel<<<(unsigned)rows, (unsigned)(dim / 8), 0, st>>>(a); break;
  }
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}
