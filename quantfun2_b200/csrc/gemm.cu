// Scaled GEMM for the quantized linears (sm_100a).
//
// D[M, N] = (A[M, K] . B[N, K]^T) * row_scale[m] * col_scale[n] + bias[n]
// with A, B both bf16 (tcgen05.mma kind::f16) or both e4m3 (kind::f8f6f4), fp32
// accumulation in TMEM, bf16 or fp32 output.  It is the compute core behind the
// reference's torchao linears (src/quant.py:209-241 int8 / float8 weight-only, bound
// into nn.Linear at :131-148): weight-only INT8/FP8 runs it on bf16 activations and
// bf16 copies of the weight codes with the per-channel scale in the epilogue; the
// W8A8 FP8 path runs it on e4m3 activations (per-token scale) and e4m3 weights.
//
// Persistent kernel, one CTA per SM, 128x256 output tiles:
//   warp 0     TMA producer: A box [128 B of K, 128 rows], B box [128 B of K, 256 rows],
//              128-byte swizzle, 4-stage ring
//   warp 1     MMA issuer: 4 x (M128 N256) per stage into one of two TMEM accumulators
//   warps 2-9  epilogue: TMEM -> registers -> scales/bias/GELU/gated residual -> global,
//              overlapped with the next tile's main loop through the second accumulator
#include "qf2_common.cuh"

#include <algorithm>
#include <climits>

namespace qf2 {
namespace gemm {

constexpr int BM = 128, BN = 256;
constexpr int kStages = 4;
constexpr int kABytes = BM * 128;   // 128 rows x 128 bytes of K
constexpr int kBBytes = BN * 128;   // 256 rows x 128 bytes of K
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 320;           // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kEpilogueWarps = 8;
constexpr uint32_t kTmemCols = 512;  // two 256-column fp32 accumulators

struct Smem {
  static constexpr int stages = 0;
  static constexpr int bars = kStages * kStageBytes;
  static constexpr int nbars = 2 * kStages + 4 + 1;
  static constexpr int misc = bars + nbars * 8;
  static constexpr int total = misc + 64;
  static constexpr int alloc = total + 1024;
};

struct Args {
  void* d;
  int64_t ldd;
  int64_t M, N, K;
  const float* row_scale;
  const float* col_scale;
  const void* bias;
  int bias_f32;   // 1: fp32 bias, 0: bf16 bias
  int d_f32;      // 1: fp32 output, 0: bf16 output
  int fp8;        // operand type: 1 e4m3, 0 bf16
  int64_t gelu_col0;                 // GELU (tanh form) on columns >= gelu_col0
  const __nv_bfloat16* residual;     // D = residual + gate * y when non-null
  int64_t ldr;
  const __nv_bfloat16* gate;         // per (row / rows_per_gate, column); null = 1
  int64_t gate_stride, rows_per_gate;
  int glu;        // SwiGLU: per 256-column tile, [128 gate | 128 up] -> 128 output columns
  int vec_ok;     // scale / bias / residual / gate rows 16-byte aligned: vector loads
  int* status;
};

QF2_DEV void load_f32x32(const float* p, float* o) {
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p + i));
    o[i] = v.x; o[i + 1] = v.y; o[i + 2] = v.z; o[i + 3] = v.w;
  }
}

QF2_DEV void load_bf16x32(const __nv_bfloat16* p, float* o) {
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(p + i);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[i + j] = __bfloat162float(e[j]);
  }
}

// GELU, tanh form, with the SFU tanh (tanh.approx.f32: ~2^-11 relative error, below
// the bf16 rounding of the output)
QF2_DEV float gelu_tanh_fast(float x) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * x * (1.0f + t);
}

// SiLU through the SFU tanh: x * sigmoid(x) = 0.5 x (1 + tanh(x / 2))
QF2_DEV float silu_fast(float x) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * x));
  return 0.5f * x * (1.0f + t);
}

// scale + bias of 32 accumulator columns starting at source column n (vector loads)
QF2_DEV void scale_bias32(const Args& A, int64_t n, float* o) {
  if (A.col_scale != nullptr) {
    float cs[32];
    load_f32x32(A.col_scale + n, cs);
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] *= cs[i];
  }
  if (A.bias != nullptr) {
    float bb[32];
    if (A.bias_f32)
      load_f32x32(reinterpret_cast<const float*>(A.bias) + n, bb);
    else
      load_bf16x32(reinterpret_cast<const __nv_bfloat16*>(A.bias) + n, bb);
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] += bb[i];
  }
}


__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb, Args A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + Smem::bars);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* acc_full = bars + 2 * kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + Smem::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + Smem::misc + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int64_t mt = (A.M + BM - 1) / BM, nt = (A.N + BN - 1) / BN;
  const int64_t ntiles = mt * nt;
  const int bk = A.fp8 ? 128 : 64;  // K elements per stage (128 bytes)
  const int64_t nk = (A.K + bk - 1) / bk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(acc_full + b, 1); mbar_init(acc_empty + b, kEpilogueWarps); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&](int code) {
    atomicExch(A.status, code);
    *abort_flag = 1;
  };
  auto wwait = [&](uint64_t* bar, uint32_t parity) -> bool {
    const bool w = mbar_wait(bar, parity) && (*abort_flag == 0);
    return __all_sync(0xffffffffu, w);
  };

  if (warp == 0) {
    // ------------------------------------------------------- producer --
    if (lane == 0) {
      prefetch_tmap(&tma);
      prefetch_tmap(&tmb);
    }
    int64_t g = 0;
    bool ok = true;
    for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      const int m0 = (int)((tile % mt) * BM), n0 = (int)((tile / mt) * BN);
      for (int64_t kb = 0; kb < nk; ++kb, ++g) {
        const int s = (int)(g % kStages);
        if (!wwait(empty + s, (uint32_t)(((g / kStages) & 1) ^ 1))) { ok = false; break; }
        if (lane == 0) {
          uint8_t* st = base + s * kStageBytes;
          mbar_arrive_expect_tx(full + s, kStageBytes);
          tma_load_2d(st, &tma, (int)(kb * bk), m0, full + s);
          tma_load_2d(st + kABytes, &tmb, (int)(kb * bk), n0, full + s);
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      fail(kDevTimeoutProducer);
      // let issued copies land before the CTA's shared memory goes away
      for (int64_t j = g > kStages ? g - kStages : 0; j < g; ++j) mbar_wait(full + (j % kStages), (j / kStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA --
    const uint32_t idesc = A.fp8 ? make_idesc(1, 0, 0, 0, 0, BM, BN)   // e4m3 x e4m3 -> f32
                                 : make_idesc(1, 1, 1, 0, 0, BM, BN);  // bf16 x bf16 -> f32
    const uint64_t d0 = sdesc_sw128_kmajor(smem_u32(base));
    constexpr uint64_t kStageStep = kStageBytes >> 4, kBOff = kABytes >> 4;
    int64_t g = 0;
    int it = 0;
    bool ok = true;
    for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      if (!wwait(acc_empty + buf, (uint32_t)(((it >> 1) & 1) ^ 1))) { ok = false; break; }
      tc_fence_after();
      const uint32_t dt = tmem + buf * BN;
      for (int64_t kb = 0; kb < nk; ++kb, ++g) {
        const int s = (int)(g % kStages);
        if (!wwait(full + s, (uint32_t)((g / kStages) & 1))) { ok = false; break; }
        tc_fence_after();
        const uint64_t da = d0 + (uint64_t)s * kStageStep, db = da + kBOff;
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            if (A.fp8)
              mma_f8f6f4(dt, da + 2 * kk, db + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            else
              mma_f16(dt, da + 2 * kk, db + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(empty + s);
        }
        __syncwarp();
      }
      if (ok && lane == 0) tc_commit(acc_full + buf);
      __syncwarp();
    }
    if (lane == 0) {
      if (!ok) fail(kDevTimeoutMma);
      tc_commit(drain);
      mbar_wait(drain, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------- epilogue --
    // 8 warps: lane quarter = warp & 3 (TMEM lanes / tile rows), column half = (warp - 2) / 4
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    int it = 0;
    bool ok = true;
    for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      const int64_t m = (tile % mt) * BM + r;
      const int64_t n0 = (tile / mt) * BN + half * (BN / 2);
      if (!wwait(acc_full + buf, (uint32_t)((it >> 1) & 1))) { ok = false; break; }
      tc_fence_after();
      const float rs = (A.row_scale != nullptr && m < A.M) ? A.row_scale[m] : 1.0f;
      if (A.glu) {
        // output columns (tile_n * 128 + half * 64 + c * 32 ...): gate at accumulator
        // column half * 64 + c * 32, up 128 columns further (N % 256 == 0, vec_ok)
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t vg[32], vu[32];
          const int col = half * 64 + c * 32;
          tmem_ld32(tmem + lane_off + buf * BN + col, vg);
          tmem_ld32(tmem + lane_off + buf * BN + 128 + col, vu);
          tmem_wait_ld();
          if (m >= A.M) continue;
          const int64_t ns = (tile / mt) * BN + col;
          float g[32], u[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            g[i] = __uint_as_float(vg[i]) * rs;
            u[i] = __uint_as_float(vu[i]) * rs;
          }
          scale_bias32(A, ns, g);
          scale_bias32(A, ns + 128, u);
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(A.d) + m * A.ldd + (tile / mt) * (BN / 2) + col;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              __nv_bfloat162 t = __floats2bfloat162_rn(silu_fast(g[i + 2 * j]) * u[i + 2 * j],
                                                       silu_fast(g[i + 2 * j + 1]) * u[i + 2 * j + 1]);
              wp[j] = *reinterpret_cast<uint32_t*>(&t);
            }
            *reinterpret_cast<uint4*>(dst + i) = w;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + buf);
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < BN / 64; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + buf * BN + half * (BN / 2) + c * 32, v);
        tmem_wait_ld();
        const int64_t nc = n0 + c * 32;
        if (m >= A.M || nc >= A.N) continue;
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(v[i]) * rs;
        const int ncols = (int)min((int64_t)32, A.N - nc);
        if (ncols == 32 && A.vec_ok) {
          scale_bias32(A, nc, o);
          if (nc + 32 > A.gelu_col0) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (nc + i >= A.gelu_col0) o[i] = gelu_tanh_fast(o[i]);
          }
          if (A.residual != nullptr) {
            float rr[32], gg[32];
            load_bf16x32(A.residual + m * A.ldr + nc, rr);
            if (A.gate != nullptr) {
              load_bf16x32(A.gate + (m / A.rows_per_gate) * A.gate_stride + nc, gg);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) gg[i] = 1.0f;
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = fmaf(gg[i], o[i], rr[i]);
          }
        } else {
          // ragged or unaligned columns: element-wise with bounds
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (i >= ncols) continue;
            if (A.col_scale != nullptr) o[i] *= A.col_scale[nc + i];
            if (A.bias != nullptr)
              o[i] += A.bias_f32 ? reinterpret_cast<const float*>(A.bias)[nc + i]
                                 : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(A.bias)[nc + i]);
            if (nc + i >= A.gelu_col0) o[i] = gelu_tanh_fast(o[i]);
            if (A.residual != nullptr) {
              const float g = A.gate != nullptr
                                  ? __bfloat162float(A.gate[(m / A.rows_per_gate) * A.gate_stride + nc + i])
                                  : 1.0f;
              o[i] = fmaf(g, o[i], __bfloat162float(A.residual[m * A.ldr + nc + i]));
            }
          }
        }
        if (A.d_f32) {
          float* dst = reinterpret_cast<float*>(A.d) + m * A.ldd + nc;
          if (ncols == 32) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < ncols) dst[i] = o[i];
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(A.d) + m * A.ldd + nc;
          if (ncols == 32) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 w;
              uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                __nv_bfloat162 t = __floats2bfloat162_rn(o[i + 2 * j], o[i + 2 * j + 1]);
                wp[j] = *reinterpret_cast<uint32_t*>(&t);
              }
              *reinterpret_cast<uint4*>(dst + i) = w;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < ncols) dst[i] = __float2bfloat16_rn(o[i]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty + buf);
    }
    if (!ok && lane == 0) fail(kDevTimeoutEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace gemm
}  // namespace qf2

using namespace qf2::gemm;

extern "C" int qf2_gemm_ex(const void* a, int64_t lda, const void* b, int64_t ldb, void* d, int64_t ldd, int64_t M,
                           int64_t N, int64_t K, int ab_dtype, int d_dtype, const float* row_scale,
                           const float* col_scale, const void* bias, int bias_dtype, int64_t gelu_col0, int glu,
                           const void* residual, int64_t ldr, const void* gate, int64_t gate_stride,
                           int64_t rows_per_gate, void* workspace, int64_t workspace_bytes, qf2_stream_t stream) {
  if (!a || !b || !d) return QF2_ERR_ARG;
  if (ab_dtype != QF2_BF16 && ab_dtype != QF2_E4M3) return QF2_ERR_DTYPE;
  if (d_dtype != QF2_BF16 && d_dtype != QF2_F32) return QF2_ERR_DTYPE;
  if (bias && bias_dtype != QF2_BF16 && bias_dtype != QF2_F32) return QF2_ERR_DTYPE;
  if (M <= 0 || N <= 0 || K <= 0 || (N % 8)) return QF2_ERR_SHAPE;
  if (residual && (ldr < N || (gate && rows_per_gate <= 0))) return QF2_ERR_SHAPE;
  if (glu && (N % BN || residual || gelu_col0 >= 0 || d_dtype != QF2_BF16)) return QF2_ERR_SHAPE;
  const int esz = ab_dtype == QF2_E4M3 ? 1 : 2;
  if (!al16(a) || !al16(b) || !al16(d) || (lda * esz) % 16 || (ldb * esz) % 16 || (ldd % 8) || lda < K || ldb < K ||
      ldd < (glu ? N / 2 : N))
    return QF2_ERR_ALIGN;
  if (!workspace || workspace_bytes < 256 || !al16(workspace)) return QF2_ERR_WORKSPACE;
  const CUtensorMapDataType tdt =
      ab_dtype == QF2_E4M3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t bk = ab_dtype == QF2_E4M3 ? 128 : 64;
  CUtensorMap ma, mb;
  const uint64_t da[2] = {(uint64_t)K, (uint64_t)M}, db[2] = {(uint64_t)K, (uint64_t)N};
  const uint32_t ba[2] = {bk, (uint32_t)BM}, bb[2] = {bk, (uint32_t)BN};
  if (!qf2_make_tmap_2d(&ma, tdt, a, da, (uint64_t)lda * esz, ba) ||
      !qf2_make_tmap_2d(&mb, tdt, b, db, (uint64_t)ldb * esz, bb))
    return QF2_ERR_ALIGN;
  Args args;
  args.d = d;
  args.ldd = ldd;
  args.M = M; args.N = N; args.K = K;
  args.row_scale = row_scale;
  args.col_scale = col_scale;
  args.bias = bias;
  args.bias_f32 = bias_dtype == QF2_F32;
  args.d_f32 = d_dtype == QF2_F32;
  args.fp8 = ab_dtype == QF2_E4M3;
  args.gelu_col0 = gelu_col0 < 0 ? INT64_MAX : gelu_col0;
  args.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  args.ldr = ldr;
  args.gate = reinterpret_cast<const __nv_bfloat16*>(gate);
  args.gate_stride = gate_stride;
  args.rows_per_gate = rows_per_gate > 0 ? rows_per_gate : 1;
  args.glu = glu != 0;
  args.vec_ok = al16(col_scale) && al16(bias) && al16(residual) && al16(gate) && (ldr % 8) == 0 &&
                (gate_stride % 8) == 0;
  if (glu && !args.vec_ok) return QF2_ERR_ALIGN;
  args.status = reinterpret_cast<int*>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  QF2_CUDA_CHECK(cudaMemsetAsync(workspace, 0, sizeof(int), s));
  static std::atomic<uint64_t> attr_done{0};
  QF2_CUDA_CHECK(qf2_set_smem_once(gemm_kernel, Smem::alloc, &attr_done));
  int sms = 148;
  QF2_CUDA_CHECK(qf2_sm_count(&sms));
  const int64_t ntiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const unsigned grid = (unsigned)std::min<int64_t>(ntiles, sms);
  gemm_kernel<<<grid, kThreads, Smem::alloc, s>>>(ma, mb, args);
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}

extern "C" int qf2_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, void* d, int64_t ldd, int64_t M,
                        int64_t N, int64_t K, int ab_dtype, int d_dtype, const float* row_scale,
                        const float* col_scale, const void* bias, int bias_dtype, void* workspace,
                        int64_t workspace_bytes, qf2_stream_t stream) {
  return qf2_gemm_ex(a, lda, b, ldb, d, ldd, M, N, K, ab_dtype, d_dtype, row_scale, col_scale, bias, bias_dtype, -1, 0,
                     nullptr, 0, nullptr, 0, 1, workspace, workspace_bytes, stream);
}
