// In-place row softmax over the last dim (sm_100a).
//
// Replaces inplace_softmax (src/kernels/__init__.py:83-87) and the Triton
// softmax_kernel / inplace_tiled_softmax (src/kernels/triton/softmax.py:22-91).
// The reference Triton kernel makes three passes over each row (max, sum,
// normalize).  Rows that fit in the registers of one CTA (softmax_reg_kernel, up to
// 16384 16-bit or 8192 fp32 elements) are read once and written once; longer or
// unaligned rows (softmax_rows_kernel) keep a running (max, sum) pair per thread and
// merge them with shuffles, reading the row twice.  fp32 math; result rounded to the
// row dtype.
#include "qf2_common.cuh"

namespace qf2 {
namespace smax {

QF2_DEV void merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) { m = mn; s = 0.f; return; }
  s = s * expf(m - mn) + s2 * expf(m2 - mn);
  m = mn;
}

// one CTA (256 threads) per row, grid-stride over rows
template <typename T>
__global__ void __launch_bounds__(256) softmax_rows_kernel(T* __restrict__ x, int64_t rows, int64_t n, int64_t rs) {
  __shared__ float s_m[8], s_s[8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    T* xr = x + row * rs;
    float m = -INFINITY, s = 0.f;
    for (int64_t i = tid; i < n; i += blockDim.x) {
      const float v = to_f32(xr[i]);
      if (v > m) {
        s = (m == -INFINITY ? 0.f : s * expf(m - v)) + 1.f;
        m = v;
      } else if (v != -INFINITY) {
        s += expf(v - m);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      merge(m, s, m2, s2);
    }
    if (lane == 0) { s_m[warp] = m; s_s[warp] = s; }
    __syncthreads();
    m = s_m[0]; s = s_s[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) merge(m, s, s_m[w], s_s[w]);
    __syncthreads();
    for (int64_t i = tid; i < n; i += blockDim.x) {
      const float v = to_f32(xr[i]);
      xr[i] = from_f32<T>(__fdiv_rn(expf(v - m), s));
    }
  }
}

// Register-resident rows: 256 threads, each holding NV 16-byte vectors of the row, so the
// row is read once and written once.  Rows of n <= 256 * NV * (16 / sizeof(T)) elements,
// n a multiple of the vector width, 16-byte aligned rows.  exp through __expf (the SFU
// exponential intrinsic), one IEEE reciprocal of the row sum per row.
template <typename T>
QF2_DEV void unpack_vec(const uint4& r, float* f);
template <>
QF2_DEV void unpack_vec<float>(const uint4& r, float* f) {
  f[0] = __uint_as_float(r.x); f[1] = __uint_as_float(r.y); f[2] = __uint_as_float(r.z); f[3] = __uint_as_float(r.w);
}
template <>
QF2_DEV void unpack_vec<__nv_bfloat16>(const uint4& r, float* f) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) { f[2 * j] = __uint_as_float(w[j] << 16); f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u); }
}
template <>
QF2_DEV void unpack_vec<__half>(const uint4& r, float* f) {
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) { const float2 t = __half22float2(h[j]); f[2 * j] = t.x; f[2 * j + 1] = t.y; }
}
template <typename T>
QF2_DEV uint4 pack_vec(const float* f);
template <>
QF2_DEV uint4 pack_vec<float>(const float* f) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
}
template <>
QF2_DEV uint4 pack_vec<__nv_bfloat16>(const float* f) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 t = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
    w[j] = *reinterpret_cast<uint32_t*>(&t);
  }
  return r;
}
template <>
QF2_DEV uint4 pack_vec<__half>(const float* f) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __half2 t = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
    w[j] = *reinterpret_cast<uint32_t*>(&t);
  }
  return r;
}

template <typename T, int NV>
__global__ void __launch_bounds__(256) softmax_reg_kernel(T* __restrict__ x, int64_t rows, int n, int64_t rs) {
  constexpr int VE = 16 / sizeof(T);
  __shared__ float red[2][8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nvec = n / VE;
  int par = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x, par ^= 1) {
    uint4* xr = reinterpret_cast<uint4*>(x + row * rs);
    float f[NV][VE];
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < NV; ++c) {
      const int vi = tid + c * 256;
      if (vi < nvec) {
        unpack_vec<T>(xr[vi], f[c]);
      } else {
#pragma unroll
        for (int j = 0; j < VE; ++j) f[c][j] = -INFINITY;
      }
#pragma unroll
      for (int j = 0; j < VE; ++j) m = fmaxf(m, f[c][j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[par][warp] = m;
    __syncthreads();
    m = red[par][0];
#pragma unroll
    for (int w = 1; w < 8; ++w) m = fmaxf(m, red[par][w]);
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NV; ++c)
#pragma unroll
      for (int j = 0; j < VE; ++j) {
        f[c][j] = __expf(f[c][j] - m);
        s += f[c][j];
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __syncthreads();  // every warp has read red[par] (max) before it holds sums
    if (lane == 0) red[par][warp] = s;
    __syncthreads();
    s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[par][w];
    const float inv = __fdiv_rn(1.0f, s);
#pragma unroll
    for (int c = 0; c < NV; ++c) {
      const int vi = tid + c * 256;
      if (vi < nvec) {
#pragma unroll
        for (int j = 0; j < VE; ++j) f[c][j] *= inv;
        xr[vi] = pack_vec<T>(f[c]);
      }
    }
  }
}

template <typename T>
static void launch_reg(T* x, int64_t rows, int64_t n, int64_t rs, unsigned grid, cudaStream_t st) {
  constexpr int VE = 16 / sizeof(T);
  const int64_t per = (n / VE + 255) / 256;
  if (per <= 1) softmax_reg_kernel<T, 1><<<grid, 256, 0, st>>>(x, rows, (int)n, rs);
  else if (per <= 2) softmax_reg_kernel<T, 2><<<grid, 256, 0, st>>>(x, rows, (int)n, rs);
  else if (per <= 4) softmax_reg_kernel<T, 4><<<grid, 256, 0, st>>>(x, rows, (int)n, rs);
  else softmax_reg_kernel<T, 8><<<grid, 256, 0, st>>>(x, rows, (int)n, rs);
}

}  // namespace smax
}  // namespace qf2

extern "C" int qf2_softmax_inplace(void* x, int64_t rows, int64_t n, int64_t row_stride, int dtype,
                                   qf2_stream_t stream) {
  using namespace qf2::smax;
  if (!x) return QF2_ERR_ARG;
  if (rows < 0 || n < 0) return QF2_ERR_SHAPE;
  if (rows == 0 || n == 0) return QF2_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)(rows < 148 * 8 ? rows : 148 * 8);
  const int64_t esz = dtype == QF2_F32 ? 4 : 2, ve = 16 / esz;
  if ((dtype == QF2_F32 || dtype == QF2_F16 || dtype == QF2_BF16) && n % ve == 0 && row_stride % ve == 0 &&
      n <= 256 * 8 * ve && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    if (dtype == QF2_F32) launch_reg<float>((float*)x, rows, n, row_stride, grid, st);
    else if (dtype == QF2_F16) launch_reg<__half>((__half*)x, rows, n, row_stride, grid, st);
    else launch_reg<__nv_bfloat16>((__nv_bfloat16*)x, rows, n, row_stride, grid, st);
    QF2_LAUNCH_CHECK();
    return QF2_OK;
  }
  switch (dtype) {
    case QF2_F32: softmax_rows_kernel<float><<<grid, 256, 0, st>>>((float*)x, rows, n, row_stride); break;
    case QF2_F16: softmax_rows_kernel<__half><<<grid, 256, 0, st>>>((__half*)x, rows, n, row_stride); break;
    case QF2_BF16:
      softmax_rows_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((__nv_bfloat16*)x, rows, n, row_stride);
      break;
    default: return QF2_ERR_DTYPE;
  }
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}
