// In-place row softmax over the last dim (sm_100a).
//
// Replaces inplace_softmax (src/kernels/__init__.py:83-87) and the Triton
// softmax_kernel / inplace_tiled_softmax (src/kernels/triton/softmax.py:22-91).
// The reference Triton kernel makes three passes over each row (max, sum,
// normalize).  Here pass 1 keeps a running (max, sum) pair per thread and
// merges them with shuffles, so each row is read twice and written once.
// fp32 math, expf (library), IEEE division; result rounded to the row dtype.
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
