// Per-row symmetric quantization and code conversion for the quantized linears.
//
// Replaces the quantize-on-load transforms of the reference (src/quant.py):
//   _int8_weight_only_transform   :209-224  (torchao symmetric int8, one scale per output row)
//   _float8_weight_only_transform :227-241  (e4m3, one scale per output row)
// with quantize_weight_rows_kernel (torchao's steps in the weight's dtype, below), and
// provides the per-token e4m3 activation quantizer of the W8A8 FP8 path (fp32 rule):
//   int8:  scale = max(amax / 127.5, FLT_EPSILON)   code = rint(x / scale) clamped to [-128, 127]
//   e4m3:  scale = amax / 448 (1 for an all-zero row)   code = e4m3(x * (448 / amax)), RNE, saturating
// amax is the row's max |x| in fp32; one CTA per row, the row is read twice (the
// second read hits L2).
#include "qf2_common.cuh"

#include <cfloat>

namespace qf2 {
namespace quant {

template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const T* __restrict__ x, int64_t ldx, int64_t K, void* q,
                                                            int64_t ldq, int fp8, float* __restrict__ scales) {
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ldx;
  __shared__ float red[8];
  float am = 0.f;
  for (int64_t i = threadIdx.x; i < K; i += blockDim.x) am = fmaxf(am, fabsf(to_f32(xr[i])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = am;
  __syncthreads();
  am = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) am = fmaxf(am, red[w]);
  if (fp8) {
    const float inv = am > 0.f ? __fdiv_rn(448.0f, am) : 1.0f;
    if (threadIdx.x == 0) scales[row] = am > 0.f ? __fdiv_rn(am, 448.0f) : 1.0f;
    uint8_t* qr = reinterpret_cast<uint8_t*>(q) + row * ldq;
    for (int64_t i = threadIdx.x; i < K; i += blockDim.x)
      qr[i] = (uint8_t)(f32x2_to_e4m3x2(__fmul_rn(to_f32(xr[i]), inv), 0.f) & 0xff);
  } else {
    const float sc = fmaxf(__fdiv_rn(am, 127.5f), FLT_EPSILON);
    if (threadIdx.x == 0) scales[row] = sc;
    int8_t* qr = reinterpret_cast<int8_t*>(q) + row * ldq;
    for (int64_t i = threadIdx.x; i < K; i += blockDim.x) {
      const int c = __float2int_rn(__fdiv_rn(to_f32(xr[i]), sc));
      qr[i] = (int8_t)max(-128, min(127, c));
    }
  }
}

// Fast path: 16-bit rows with K % 8 == 0 and K <= 256 * 8 * kRowVecs, 16-byte aligned.
// The row stays in registers (one HBM read), 16-byte loads, 8-byte e4m3 stores.
constexpr int kRowVecs = 8;

template <typename T>
QF2_DEV float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  v = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) v = fmaxf(v, red[w]);
  return v;
}

QF2_DEV float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  v = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += red[w];
  return v;
}

// store 8 values of a row either as bf16 (16 bytes) or e4m3 (8 bytes, * inv)
QF2_DEV void store8(void* out, int64_t off, const float* y, bool fp8, float inv) {
  if (fp8) {
    uint2 w;
    w.x = (uint32_t)f32x2_to_e4m3x2(__fmul_rn(y[0], inv), __fmul_rn(y[1], inv)) |
          ((uint32_t)f32x2_to_e4m3x2(__fmul_rn(y[2], inv), __fmul_rn(y[3], inv)) << 16);
    w.y = (uint32_t)f32x2_to_e4m3x2(__fmul_rn(y[4], inv), __fmul_rn(y[5], inv)) |
          ((uint32_t)f32x2_to_e4m3x2(__fmul_rn(y[6], inv), __fmul_rn(y[7], inv)) << 16);
    *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(out) + off) = w;
  } else {
    uint4 w;
    uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 t = __floats2bfloat162_rn(y[2 * j], y[2 * j + 1]);
      wp[j] = *reinterpret_cast<uint32_t*>(&t);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out) + off) = w;
  }
}

template <typename T, int NV>
__global__ void __launch_bounds__(256) quantize_rows_vec_kernel(const T* __restrict__ x, int64_t ldx, int K, void* q,
                                                                int64_t ldq, int fp8, float* __restrict__ scales) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ldx;
  const int nv = K / 8;
  uint4 raw[NV];
  float am = 0.f;
#pragma unroll
  for (int c = 0; c < NV; ++c) {
    const int vi = threadIdx.x + c * 256;
    raw[c] = vi < nv ? *reinterpret_cast<const uint4*>(xr + vi * 8) : make_uint4(0, 0, 0, 0);
    const T* e = reinterpret_cast<const T*>(&raw[c]);
#pragma unroll
    for (int j = 0; j < 8; ++j) am = fmaxf(am, fabsf(to_f32(e[j])));
  }
  am = block_max<T>(am, red);
  const float inv = fp8 ? (am > 0.f ? __fdiv_rn(448.0f, am) : 1.0f) : 0.f;
  const float sc = fp8 ? (am > 0.f ? __fdiv_rn(am, 448.0f) : 1.0f) : fmaxf(__fdiv_rn(am, 127.5f), FLT_EPSILON);
  if (threadIdx.x == 0) scales[row] = sc;
#pragma unroll
  for (int c = 0; c < NV; ++c) {
    const int vi = threadIdx.x + c * 256;
    if (vi >= nv) continue;
    const T* e = reinterpret_cast<const T*>(&raw[c]);
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = to_f32(e[j]);
    if (fp8) {
      store8(q, row * ldq + vi * 8, y, true, inv);
    } else {
      uint2 w = make_uint2(0u, 0u);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int cc = max(-128, min(127, __float2int_rn(__fdiv_rn(y[j], sc))));
        (j < 4 ? w.x : w.y) |= (uint32_t)(cc & 0xff) << ((j & 3) * 8);
      }
      *reinterpret_cast<uint2*>(reinterpret_cast<int8_t*>(q) + row * ldq + vi * 8) = w;
    }
  }
}

// adaLN: y = LayerNorm(x) * (1 + scale[b]) + shift[b] (LayerNorm without affine, fp32
// statistics), written as bf16 or as e4m3 with a per-row scale for the next GEMM.
// Same row constraints as the fast quantizer.
template <typename T, int NV>
__global__ void __launch_bounds__(256) ln_modulate_kernel(const T* __restrict__ x, int64_t ldx, int N,
                                                          const __nv_bfloat16* __restrict__ shift,
                                                          const __nv_bfloat16* __restrict__ scale, int64_t mod_stride,
                                                          int64_t rows_per_batch, float eps, void* out, int64_t ldo,
                                                          int fp8, float* __restrict__ scales) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ldx;
  const int64_t bi = row / rows_per_batch;
  const __nv_bfloat16* sh = shift + bi * mod_stride;
  const __nv_bfloat16* scl = scale + bi * mod_stride;
  const int nv = N / 8;
  float v[NV][8];
  float sum = 0.f;
#pragma unroll
  for (int c = 0; c < NV; ++c) {
    const int vi = threadIdx.x + c * 256;
    uint4 raw = vi < nv ? *reinterpret_cast<const uint4*>(xr + vi * 8) : make_uint4(0, 0, 0, 0);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[c][j] = to_f32(e[j]);
      sum += v[c][j];
    }
  }
  const float mean = block_sum(sum, red) / (float)N;
  float sq = 0.f;
#pragma unroll
  for (int c = 0; c < NV; ++c) {
    const int vi = threadIdx.x + c * 256;
    if (vi < nv) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[c][j] - mean;
        sq = fmaf(d, d, sq);
      }
    }
  }
  const float rstd = rsqrtf(block_sum(sq, red) / (float)N + eps);
  float am = 0.f;
#pragma unroll
  for (int c = 0; c < NV; ++c) {
    const int vi = threadIdx.x + c * 256;
    if (vi < nv) {
      const uint4 a = *reinterpret_cast<const uint4*>(sh + vi * 8);
      const uint4 b = *reinterpret_cast<const uint4*>(scl + vi * 8);
      const __nv_bfloat16* ae = reinterpret_cast<const __nv_bfloat16*>(&a);
      const __nv_bfloat16* be = reinterpret_cast<const __nv_bfloat16*>(&b);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[c][j] = fmaf((v[c][j] - mean) * rstd, 1.0f + __bfloat162float(be[j]), __bfloat162float(ae[j]));
        am = fmaxf(am, fabsf(v[c][j]));
      }
    }
  }
  float inv = 1.f;
  if (fp8) {
    am = block_max<T>(am, red);
    inv = am > 0.f ? __fdiv_rn(448.0f, am) : 1.0f;
    if (threadIdx.x == 0) scales[row] = am > 0.f ? __fdiv_rn(am, 448.0f) : 1.0f;
  }
#pragma unroll
  for (int c = 0; c < NV; ++c) {
    const int vi = threadIdx.x + c * 256;
    if (vi < nv) store8(out, row * ldo + vi * 8, v[c], fp8 != 0, inv);
  }
}

// Same operation, one warp per row for N % 256 == 0 (NV = N / 256 vectors per lane): the
// statistics are warp shuffles (no CTA-wide barrier between the load and the store) and
// the row is re-read from L1 in the later passes instead of being held in registers, so
// many rows stay resident per SM.  Mean and variance come from sums shifted by the row's
// first element (stable when the mean is large against the spread).
QF2_DEV float warp_allsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
QF2_DEV float warp_allmax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <typename T, int NV>
__global__ void __launch_bounds__(256, 2) ln_modulate_warp_kernel(const T* __restrict__ x, int64_t ldx, int64_t M,
                                                                  const __nv_bfloat16* __restrict__ shift,
                                                                  const __nv_bfloat16* __restrict__ scale,
                                                                  int64_t mod_stride, int64_t rows_per_batch,
                                                                  float eps, void* out, int64_t ldo, int fp8,
                                                                  float* __restrict__ scales) {
  constexpr int N = NV * 256;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= M) return;
  const T* xr = x + row * ldx;
  const int64_t bi = row / rows_per_batch;
  const __nv_bfloat16* sh = shift + bi * mod_stride;
  const __nv_bfloat16* scl = scale + bi * mod_stride;
  const float x0 = to_f32(xr[0]);
  float s1 = 0.f, s2 = 0.f;
  {
    uint4 raw[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) raw[i] = *reinterpret_cast<const uint4*>(xr + (i * 32 + lane) * 8);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const T* e = reinterpret_cast<const T*>(&raw[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = to_f32(e[j]) - x0;
        s1 += d;
        s2 = fmaf(d, d, s2);
      }
    }
  }
  const float m1 = warp_allsum(s1) / (float)N;
  const float var = fmaxf(warp_allsum(s2) / (float)N - m1 * m1, 0.f);
  const float mean = x0 + m1;
  const float rstd = rsqrtf(var + eps);
  auto modulated = [&](int i, float* y) {
    const int c = (i * 32 + lane) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(sh + c));
    const uint4 bsc = __ldg(reinterpret_cast<const uint4*>(scl + c));
    const __nv_bfloat16* ae = reinterpret_cast<const __nv_bfloat16*>(&a);
    const __nv_bfloat16* be = reinterpret_cast<const __nv_bfloat16*>(&bsc);
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      y[j] = fmaf((to_f32(e[j]) - mean) * rstd, 1.0f + __bfloat162float(be[j]), __bfloat162float(ae[j]));
  };
  float inv = 1.f;
  if (fp8) {
    float am = 0.f;
#pragma unroll 4
    for (int i = 0; i < NV; ++i) {
      float y[8];
      modulated(i, y);
#pragma unroll
      for (int j = 0; j < 8; ++j) am = fmaxf(am, fabsf(y[j]));
    }
    am = warp_allmax(am);
    inv = am > 0.f ? __fdiv_rn(448.0f, am) : 1.0f;
    if (lane == 0) scales[row] = am > 0.f ? __fdiv_rn(am, 448.0f) : 1.0f;
  }
#pragma unroll 4
  for (int i = 0; i < NV; ++i) {
    float y[8];
    modulated(i, y);
    store8(out, row * ldo + (i * 32 + lane) * 8, y, fp8 != 0, inv);
  }
}

// code -> bf16 (exact for int8 and e4m3 codes)
__global__ void __launch_bounds__(256) codes_to_bf16_kernel(const void* q, int64_t ldq, int fp8, int64_t M, int64_t K,
                                                            __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int64_t total = M * K;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / K, c = idx % K;
    float v;
    if (fp8) {
      const __nv_fp8_e4m3 e = *reinterpret_cast<const __nv_fp8_e4m3*>(reinterpret_cast<const uint8_t*>(q) + r * ldq + c);
      v = (float)e;
    } else {
      v = (float)reinterpret_cast<const int8_t*>(q)[r * ldq + c];
    }
    out[r * ldo + c] = __float2bfloat16_rn(v);
  }
}

// 16 codes per thread: one 16-byte load, two 16-byte stores (K % 16 == 0, aligned rows)
__global__ void __launch_bounds__(256) codes_to_bf16_vec_kernel(const uint8_t* __restrict__ q, int64_t ldq, int fp8,
                                                                int64_t M, int64_t kv, __nv_bfloat16* __restrict__ out,
                                                                int64_t ldo) {
  const int64_t total = M * kv;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / kv, c = (idx - r * kv) * 16;
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(q + r * ldq + c));
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&raw);
    uint4 o[2];
    uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float lo, hi;
      if (fp8) {
        lo = (float)*reinterpret_cast<const __nv_fp8_e4m3*>(b + 2 * i);
        hi = (float)*reinterpret_cast<const __nv_fp8_e4m3*>(b + 2 * i + 1);
      } else {
        lo = (float)(int8_t)b[2 * i];
        hi = (float)(int8_t)b[2 * i + 1];
      }
      __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
      ow[i] = *reinterpret_cast<uint32_t*>(&t);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + r * ldo + c);
    dst[0] = o[0];
    dst[1] = o[1];
  }
}

// ------------------------------------------------ weight quantizer (torchao) --
// Per-output-row symmetric quantization of a weight [M, K] by the steps of torchao 0.7.0
// (quant_primitives.py: choose_qparams_affine, then quantize_affine), which the reference
// runs on weights it has already cast to the activation dtype T (fp16 for qint8 and
// qfloat8: supported_dtypes at src/quant.py:326,331, applied by model.to(dtype) at :383),
// with every tensor op in T and its fp32 opmath:
//   amax   = max(-min(min_row, 0), max(max_row, 0))                         (exact in T)
//   scale  = T(amax / D) (fp32 division, rounded to T), then max(scale, FLT_EPSILON)
//            D = (qmax - qmin) / 2: 127.5 for int8 [-128, 127], 448 for e4m3 [-448, 448]
//   recip  = T(1 / scale)                     (`1.0 / scale`, `scale.reciprocal()`)
//   y      = T(w * recip)                     (the product of two T values, rounded to T)
//   int8:  code = clamp(round_half_even(y), -128, 127);  NaN (0 * inf) -> 0
//   e4m3:  code = e4m3_rne(clamp(y, -448, 448))
// The fp32 scale written per row is float(scale).  An overflowing reciprocal (fp16 scale
// below 1/65504) gives inf there too, and the same saturated codes.
template <typename T>
__global__ void __launch_bounds__(256) quantize_weight_rows_kernel(const T* __restrict__ w, int64_t ldw, int64_t K,
                                                                   void* q, int64_t ldq, int fp8,
                                                                   float* __restrict__ scales) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const T* wr = w + row * ldw;
  float am = 0.f;
  for (int64_t i = threadIdx.x; i < K; i += blockDim.x) am = fmaxf(am, fabsf(to_f32(wr[i])));
  am = block_max<T>(am, red);
  const float scale_t = fmaxf(to_f32(from_f32<T>(__fdiv_rn(am, fp8 ? 448.0f : 127.5f))), FLT_EPSILON);
  const float recip_t = to_f32(from_f32<T>(__fdiv_rn(1.0f, scale_t)));
  if (threadIdx.x == 0) scales[row] = scale_t;
  for (int64_t i = threadIdx.x; i < K; i += blockDim.x) {
    const float y = to_f32(from_f32<T>(__fmul_rn(to_f32(wr[i]), recip_t)));
    if (fp8) {
      const float c = fminf(fmaxf(y, -448.0f), 448.0f);  // fminf/fmaxf would drop a NaN: keep it
      reinterpret_cast<uint8_t*>(q)[row * ldq + i] = (uint8_t)(f32x2_to_e4m3x2(y != y ? y : c, 0.f) & 0xff);
    } else {
      const float r = fminf(fmaxf(rintf(y), -128.0f), 127.0f);
      reinterpret_cast<int8_t*>(q)[row * ldq + i] = y != y ? (int8_t)0 : (int8_t)(int)r;
    }
  }
}

// code -> fp16 (exact for int8 and e4m3 codes), 16 codes per thread as in the bf16 form
__global__ void __launch_bounds__(256) codes_to_f16_vec_kernel(const uint8_t* __restrict__ q, int64_t ldq, int fp8,
                                                               int64_t M, int64_t kv, __half* __restrict__ out,
                                                               int64_t ldo) {
  const int64_t total = M * kv;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / kv, c = (idx - r * kv) * 16;
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(q + r * ldq + c));
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&raw);
    uint4 o[2];
    uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float lo, hi;
      if (fp8) {
        lo = (float)*reinterpret_cast<const __nv_fp8_e4m3*>(b + 2 * i);
        hi = (float)*reinterpret_cast<const __nv_fp8_e4m3*>(b + 2 * i + 1);
      } else {
        lo = (float)(int8_t)b[2 * i];
        hi = (float)(int8_t)b[2 * i + 1];
      }
      __half2 t = __floats2half2_rn(lo, hi);
      ow[i] = *reinterpret_cast<uint32_t*>(&t);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + r * ldo + c);
    dst[0] = o[0];
    dst[1] = o[1];
  }
}

// Rows are held in registers, NV 16-byte vectors per thread of 256: the smallest NV that
// covers the row keeps the register count (and so the number of resident rows per SM) up.
static int vecs_per_thread(int64_t n) {
  const int64_t v = (n / 8 + 255) / 256;
  return v <= 1 ? 1 : v <= 2 ? 2 : v <= 4 ? 4 : 8;
}

template <typename T>
static void launch_rows(int nv, const T* x, int64_t ldx, int K, void* q, int64_t ldq, int fp8, float* scales,
                        int64_t M, cudaStream_t s) {
  switch (nv) {
    case 1: quantize_rows_vec_kernel<T, 1><<<(unsigned)M, 256, 0, s>>>(x, ldx, K, q, ldq, fp8, scales); break;
    case 2: quantize_rows_vec_kernel<T, 2><<<(unsigned)M, 256, 0, s>>>(x, ldx, K, q, ldq, fp8, scales); break;
    case 4: quantize_rows_vec_kernel<T, 4><<<(unsigned)M, 256, 0, s>>>(x, ldx, K, q, ldq, fp8, scales); break;
    default: quantize_rows_vec_kernel<T, 8><<<(unsigned)M, 256, 0, s>>>(x, ldx, K, q, ldq, fp8, scales); break;
  }
}

template <typename T>
static void launch_ln(int nv, const T* x, int64_t ldx, int N, const __nv_bfloat16* sh, const __nv_bfloat16* sc,
                      int64_t mod_stride, int64_t rpb, float eps, void* out, int64_t ldo, int fp8, float* scales,
                      int64_t M, cudaStream_t s) {
  if (N % 256 == 0 && N / 256 <= 16) {
    const unsigned grid = (unsigned)((M + 7) / 8);
#define QF2_LNW(V) ln_modulate_warp_kernel<T, V><<<grid, 256, 0, s>>>(x, ldx, M, sh, sc, mod_stride, rpb, eps, out, \
                                                                     ldo, fp8, scales)
    switch (N / 256) {
      case 1: QF2_LNW(1); return;
      case 2: QF2_LNW(2); return;
      case 3: QF2_LNW(3); return;
      case 4: QF2_LNW(4); return;
      case 6: QF2_LNW(6); return;
      case 8: QF2_LNW(8); return;
      case 9: QF2_LNW(9); return;
      case 12: QF2_LNW(12); return;
      case 16: QF2_LNW(16); return;
      default: break;
    }
#undef QF2_LNW
  }
#define QF2_LN(V) ln_modulate_kernel<T, V><<<(unsigned)M, 256, 0, s>>>(x, ldx, N, sh, sc, mod_stride, rpb, eps, out, \
                                                                     ldo, fp8, scales)
  switch (nv) {
    case 1: QF2_LN(1); break;
    case 2: QF2_LN(2); break;
    case 4: QF2_LN(4); break;
    default: QF2_LN(8); break;
  }
#undef QF2_LN
}

}  // namespace quant
}  // namespace qf2

extern "C" int qf2_quantize_rows(const void* x, int64_t ldx, int x_dtype, int64_t M, int64_t K, void* q, int64_t ldq,
                                 int q_dtype, float* scales, qf2_stream_t stream) {
  using namespace qf2::quant;
  if (!x || !q || !scales) return QF2_ERR_ARG;
  if (q_dtype != QF2_I8 && q_dtype != QF2_E4M3) return QF2_ERR_DTYPE;
  if (M < 0 || K <= 0 || ldx < K || ldq < K) return QF2_ERR_SHAPE;
  if (M == 0) return QF2_OK;
  if (M > 0x7fffffff) return QF2_ERR_SHAPE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int fp8 = q_dtype == QF2_E4M3;
  const bool vec = (x_dtype == QF2_BF16 || x_dtype == QF2_F16) && K % 8 == 0 && K <= 256 * 8 * kRowVecs &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (ldx % 8) == 0 &&
                   (reinterpret_cast<uintptr_t>(q) & 7) == 0 && (ldq % 8) == 0;
  if (vec) {
    if (x_dtype == QF2_BF16)
      launch_rows<__nv_bfloat16>(vecs_per_thread(K), (const __nv_bfloat16*)x, ldx, (int)K, q, ldq, fp8, scales, M, s);
    else
      launch_rows<__half>(vecs_per_thread(K), (const __half*)x, ldx, (int)K, q, ldq, fp8, scales, M, s);
    QF2_LAUNCH_CHECK();
    return QF2_OK;
  }
  switch (x_dtype) {
    case QF2_F32: quantize_rows_kernel<float><<<(unsigned)M, 256, 0, s>>>((const float*)x, ldx, K, q, ldq, fp8, scales); break;
    case QF2_F16: quantize_rows_kernel<__half><<<(unsigned)M, 256, 0, s>>>((const __half*)x, ldx, K, q, ldq, fp8, scales); break;
    case QF2_BF16:
      quantize_rows_kernel<__nv_bfloat16><<<(unsigned)M, 256, 0, s>>>((const __nv_bfloat16*)x, ldx, K, q, ldq, fp8, scales);
      break;
    default: return QF2_ERR_DTYPE;
  }
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}

extern "C" int qf2_quantize_weight_rows(const void* w, int64_t ldw, int w_dtype, int64_t M, int64_t K, void* q,
                                        int64_t ldq, int q_dtype, float* scales, qf2_stream_t stream) {
  using namespace qf2::quant;
  if (!w || !q || !scales) return QF2_ERR_ARG;
  if (q_dtype != QF2_I8 && q_dtype != QF2_E4M3) return QF2_ERR_DTYPE;
  if (M < 0 || K <= 0 || ldw < K || ldq < K || M > 0x7fffffff) return QF2_ERR_SHAPE;
  if (M == 0) return QF2_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int fp8 = q_dtype == QF2_E4M3;
  switch (w_dtype) {
    case QF2_F16:
      quantize_weight_rows_kernel<__half><<<(unsigned)M, 256, 0, s>>>((const __half*)w, ldw, K, q, ldq, fp8, scales);
      break;
    case QF2_BF16:
      quantize_weight_rows_kernel<__nv_bfloat16><<<(unsigned)M, 256, 0, s>>>((const __nv_bfloat16*)w, ldw, K, q, ldq,
                                                                            fp8, scales);
      break;
    case QF2_F32:
      quantize_weight_rows_kernel<float><<<(unsigned)M, 256, 0, s>>>((const float*)w, ldw, K, q, ldq, fp8, scales);
      break;
    default: return QF2_ERR_DTYPE;
  }
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}

extern "C" int qf2_codes_convert(const void* q, int64_t ldq, int q_dtype, int64_t M, int64_t K, void* out,
                                 int64_t ldo, int out_dtype, qf2_stream_t stream) {
  using namespace qf2::quant;
  if (out_dtype == QF2_BF16) return qf2_codes_to_bf16(q, ldq, q_dtype, M, K, out, ldo, stream);
  if (out_dtype != QF2_F16) return QF2_ERR_DTYPE;
  if (!q || !out) return QF2_ERR_ARG;
  if (q_dtype != QF2_I8 && q_dtype != QF2_E4M3) return QF2_ERR_DTYPE;
  if (M < 0 || K <= 0 || ldq < K || ldo < K) return QF2_ERR_SHAPE;
  if (M == 0) return QF2_OK;
  if (K % 16 || ldq % 16 || ldo % 8 || (reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return QF2_ERR_ALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t total = M * (K / 16);
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  codes_to_f16_vec_kernel<<<(unsigned)blocks, 256, 0, s>>>(reinterpret_cast<const uint8_t*>(q), ldq,
                                                           q_dtype == QF2_E4M3, M, K / 16,
                                                           reinterpret_cast<__half*>(out), ldo);
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}

extern "C" int qf2_codes_to_bf16(const void* q, int64_t ldq, int q_dtype, int64_t M, int64_t K, void* out, int64_t ldo,
                                 qf2_stream_t stream) {
  using namespace qf2::quant;
  if (!q || !out) return QF2_ERR_ARG;
  if (q_dtype != QF2_I8 && q_dtype != QF2_E4M3) return QF2_ERR_DTYPE;
  if (M < 0 || K <= 0 || ldq < K || ldo < K) return QF2_ERR_SHAPE;
  if (M == 0) return QF2_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = K % 16 == 0 && ldq % 16 == 0 && ldo % 8 == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  if (vec) {
    const int64_t total = M * (K / 16);
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    codes_to_bf16_vec_kernel<<<(unsigned)blocks, 256, 0, s>>>(reinterpret_cast<const uint8_t*>(q), ldq,
                                                              q_dtype == QF2_E4M3, M, K / 16,
                                                              reinterpret_cast<__nv_bfloat16*>(out), ldo);
  } else {
    const int64_t total = M * K;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    codes_to_bf16_kernel<<<(unsigned)blocks, 256, 0, s>>>(q, ldq, q_dtype == QF2_E4M3, M, K,
                                                           reinterpret_cast<__nv_bfloat16*>(out), ldo);
  }
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}

extern "C" int qf2_ln_modulate(const void* x, int64_t ldx, int x_dtype, const void* shift, const void* scale,
                               int64_t mod_stride, int64_t rows_per_batch, int64_t M, int64_t N, float eps, void* out,
                               int64_t ldo, int out_dtype, float* scales, qf2_stream_t stream) {
  using namespace qf2::quant;
  if (!x || !shift || !scale || !out) return QF2_ERR_ARG;
  if (x_dtype != QF2_BF16 && x_dtype != QF2_F16) return QF2_ERR_DTYPE;
  if (out_dtype != QF2_BF16 && out_dtype != QF2_E4M3) return QF2_ERR_DTYPE;
  if (out_dtype == QF2_E4M3 && !scales) return QF2_ERR_ARG;
  if (M < 0 || N <= 0 || N % 8 || N > 256 * 8 * kRowVecs || rows_per_batch <= 0 || M > 0x7fffffff)
    return QF2_ERR_SHAPE;
  const int osz = out_dtype == QF2_E4M3 ? 1 : 2;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(shift) & 15) ||
      (reinterpret_cast<uintptr_t>(scale) & 15) || (reinterpret_cast<uintptr_t>(out) & (osz == 1 ? 7 : 15)) ||
      (ldx % 8) || (mod_stride % 8) || (ldo % 8))
    return QF2_ERR_ALIGN;
  if (M == 0) return QF2_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __nv_bfloat16* sh = reinterpret_cast<const __nv_bfloat16*>(shift);
  const __nv_bfloat16* sc = reinterpret_cast<const __nv_bfloat16*>(scale);
  const int fp8 = out_dtype == QF2_E4M3;
  if (x_dtype == QF2_BF16)
    launch_ln<__nv_bfloat16>(vecs_per_thread(N), (const __nv_bfloat16*)x, ldx, (int)N, sh, sc, mod_stride,
                             rows_per_batch, eps, out, ldo, fp8, scales, M, s);
  else
    launch_ln<__half>(vecs_per_thread(N), (const __half*)x, ldx, (int)N, sh, sc, mod_stride, rows_per_batch, eps, out,
                      ldo, fp8, scales, M, s);
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}
