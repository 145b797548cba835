// Per-row symmetric quantization and code conversion for the quantized linears.
//
// Replaces the quantize-on-load transforms of the reference (src/quant.py):
//   _int8_weight_only_transform   :209-224  (torchao symmetric int8, one scale per output row)
//   _float8_weight_only_transform :227-241  (e4m3, one scale per output row)
// and provides the per-token e4m3 activation quantizer of the W8A8 FP8 path.
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

extern "C" int qf2_codes_to_bf16(const void* q, int64_t ldq, int q_dtype, int64_t M, int64_t K, void* out, int64_t ldo,
                                 qf2_stream_t stream) {
  using namespace qf2::quant;
  if (!q || !out) return QF2_ERR_ARG;
  if (q_dtype != QF2_I8 && q_dtype != QF2_E4M3) return QF2_ERR_DTYPE;
  if (M < 0 || K <= 0 || ldq < K || ldo < K) return QF2_ERR_SHAPE;
  if (M == 0) return QF2_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t total = M * K;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  codes_to_bf16_kernel<<<(unsigned)blocks, 256, 0, s>>>(q, ldq, q_dtype == QF2_E4M3, M, K,
                                                         reinterpret_cast<__nv_bfloat16*>(out), ldo);
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}
