// Scaled GEMM for the quantized linears (sm_100a).
//
// D[M, N] = (A[M, K] . B[N, K]^T) * row_scale[m] * col_scale[n] + bias[n]
// with A, B both bf16 or both fp16 (tcgen05.mma kind::f16) or both e4m3 (kind::f8f6f4),
// fp32 accumulation in TMEM, bf16, fp16 or fp32 output.  It is the compute core behind the
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

// per epilogue warp: two 32 x 32 bf16 output staging tiles (64-byte swizzle) for TMA stores
constexpr int kStagingBytes = kEpilogueWarps * 2 * 2048;

struct Smem {
  static constexpr int stages = 0;
  static constexpr int staging = kStages * kStageBytes;
  static constexpr int bars = staging + kStagingBytes;
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
  int d_f32;      // 1: fp32 output, 0: 16-bit output
  int d_f16;      // 16-bit output: 1 fp16, 0 bf16
  int fp8;        // operand type: 1 e4m3, 0 16-bit
  int f16;        // 16-bit operands: 1 fp16, 0 bf16
  int64_t gelu_col0;                 // GELU (tanh form) on columns >= gelu_col0
  const __nv_bfloat16* residual;     // D = residual + gate * y when non-null
  int64_t ldr;
  const __nv_bfloat16* gate;         // per (row / rows_per_gate, column); null = 1
  int64_t gate_stride, rows_per_gate;
  int glu;        // SwiGLU: per 256-column tile, [128 gate | 128 up] -> 128 output columns
  int bn;         // tile width: 256, or 192 / 128 for CTA-pair tiles (fewer idle SMs in the last wave)
  int vec_ok;     // scale / bias / residual / gate rows 16-byte aligned: vector loads
  int* status;
  // row scatter (the row-indexed product of the reference's RAS ops): row m of the product
  // goes to output row (m / idx_rows) * out_rows + row_idx[m % idx_rows]; null = none
  const int64_t* row_idx;
  int64_t idx_rows, out_rows;
};

// 32 output values of one row to a scattered row: 16-bit (bf16 / fp16) or fp32, vector
// stores when the whole chunk is in range and aligned
QF2_DEV void store_row32(const Args& A, int64_t row, int64_t nc, int ncols, const float* o) {
  if (A.d_f32) {
    float* dst = reinterpret_cast<float*>(A.d) + row * A.ldd + nc;
    for (int i = 0; i < 32; ++i)
      if (i < ncols) dst[i] = o[i];
    return;
  }
  uint16_t h[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if (A.d_f16) {
      __half t = __float2half_rn(o[i]);
      h[i] = *reinterpret_cast<uint16_t*>(&t);
    } else {
      __nv_bfloat16 t = __float2bfloat16_rn(o[i]);
      h[i] = *reinterpret_cast<uint16_t*>(&t);
    }
  }
  uint16_t* dst = reinterpret_cast<uint16_t*>(A.d) + row * A.ldd + nc;
  if (ncols == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
    for (int v = 0; v < 4; ++v) *reinterpret_cast<uint4*>(dst + 8 * v) = *reinterpret_cast<const uint4*>(h + 8 * v);
  } else {
    for (int i = 0; i < 32; ++i)
      if (i < ncols) dst[i] = h[i];
  }
}

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


// Output staging for one 32-row x 32-column bf16 / fp16 chunk of a warp: each lane writes its
// row (64 bytes) into a 64-byte-swizzled tile, then lane 0 stores the tile with TMA.
// Row-per-thread stores straight to global memory issue 32 scattered 16-byte writes per
// warp instruction and stall the tensor pipe; one bulk store per chunk does not.
struct Stager {
  uint8_t* buf;            // this warp's two 2 KB tiles
  const CUtensorMap* map;  // D, box {32 columns, 32 rows}, 64-byte swizzle
  uint32_t ctr;
  int64_t rows;            // M: boxes starting at or below it are not issued
  int f16;                 // 1: fp16 output, 0: bf16
};

QF2_DEV void stage_store(Stager& st, const float* o, int lane, int64_t col, int64_t row0) {
  uint8_t* b = st.buf + (st.ctr & 1) * 2048;
  if (lane == 0) bulk_wait_read<1>();  // the store issued from this tile two chunks ago has read it
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 w;
    uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
    if (st.f16) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __half2 t = __floats2half2_rn(o[8 * j + 2 * q], o[8 * j + 2 * q + 1]);
        wp[q] = *reinterpret_cast<uint32_t*>(&t);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __nv_bfloat162 t = __floats2bfloat162_rn(o[8 * j + 2 * q], o[8 * j + 2 * q + 1]);
        wp[q] = *reinterpret_cast<uint32_t*>(&t);
      }
    }
    *reinterpret_cast<uint4*>(b + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = w;
  }
  fence_async_smem();
  __syncwarp();
  if (lane == 0 && row0 < st.rows) {
    tma_store_2d(st.map, b, (int32_t)col, (int32_t)row0);
    bulk_commit();
  }
  ++st.ctr;
}

// One accumulator tile's epilogue for the calling thread: TMEM lane = tile row (row m of
// D, m0w = row of lane 0 of the warp), column half `half` of the 256 accumulator columns
// starting at tile column n_tile.  tacc = TMEM address of (lane quarter, accumulator
// buffer).  Scales, bias, GELU / SwiGLU, gated residual; bf16 output through the stager,
// fp32 output with direct stores.
QF2_DEV void epilogue_tile(const Args& A, Stager& st, uint32_t tacc, int64_t m0w, int64_t n_tile, int half) {
  const int lane = threadIdx.x & 31;
  const int64_t m = m0w + lane;
  const bool row_ok = m < A.M;
  const float rs = (A.row_scale != nullptr && row_ok) ? A.row_scale[m] : 1.0f;
  if (A.glu) {
    // output columns n_tile / 2 + half * 64 + c * 32 ...: gate at accumulator column
    // half * 64 + c * 32, up 128 columns further (N % 256 == 0, vec_ok)
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t vg[32], vu[32];
      const int col = half * 64 + c * 32;
      tmem_ld32(tacc + col, vg);
      tmem_ld32(tacc + 128 + col, vu);
      tmem_wait_ld();
      const int64_t ns = n_tile + col;
      float g[32], u[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        g[i] = __uint_as_float(vg[i]) * rs;
        u[i] = __uint_as_float(vu[i]) * rs;
      }
      scale_bias32(A, ns, g);
      scale_bias32(A, ns + 128, u);
#pragma unroll
      for (int i = 0; i < 32; ++i) g[i] = silu_fast(g[i]) * u[i];
      stage_store(st, g, lane, n_tile / 2 + col, m0w);
    }
    return;
  }
  const int hw = A.bn / 2;  // columns per half
  const int64_t n0 = n_tile + half * hw;
#pragma unroll 1
  for (int c = 0; c < hw / 32; ++c) {
    uint32_t v[32];
    tmem_ld32(tacc + half * hw + c * 32, v);
    tmem_wait_ld();
    const int64_t nc = n0 + c * 32;
    if (nc >= A.N) continue;  // warp-uniform
    float o[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(v[i]) * rs;
    const int ncols = (int)min((int64_t)32, A.N - nc);
    if (!row_ok) {
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = 0.f;
    } else if (ncols == 32 && A.vec_ok) {
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
    if (A.row_idx != nullptr) {  // warp-uniform: scattered rows, direct stores
      if (row_ok) {
        const int64_t ri = A.row_idx[m % A.idx_rows];
        if (ri >= 0 && ri < A.out_rows)
          store_row32(A, (m / A.idx_rows) * A.out_rows + ri, nc, ncols, o);
        else
          atomicExch(A.status, kDevBadIndex);  // skipped; the status word reports it
      }
      continue;
    }
    if (!A.d_f32) {
      stage_store(st, o, lane, nc, m0w);  // TMA clips rows >= M and columns >= N
      continue;
    }
    if (!row_ok) continue;
    float* dst = reinterpret_cast<float*>(A.d) + m * A.ldd + nc;
    if (ncols == 32) {
#pragma unroll
      for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < ncols) dst[i] = o[i];
    }
  }
}

// ------------------------------------------------------- single-CTA tiles --
// 128 x 256 tiles, one CTA per SM (small M: the adaLN / embedding linears).
template <bool FP8>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                const __grid_constant__ CUtensorMap tmd, Args A) {
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
  constexpr int bk = FP8 ? 128 : 64;  // K elements per stage (128 bytes)
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
    // e4m3 x e4m3, bf16 x bf16 or fp16 x fp16 -> f32 (the 16-bit format is a descriptor
    // field, not a branch between the MMAs)
    const uint32_t fmt16 = A.f16 ? 0u : 1u;
    const uint32_t idesc = FP8 ? make_idesc(1, 0, 0, 0, 0, BM, BN) : make_idesc(1, fmt16, fmt16, 0, 0, BM, BN);
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
            if constexpr (FP8)
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
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    Stager stg{base + Smem::staging + (warp - 2) * 4096, &tmd, 0, A.M, A.d_f16};
    int it = 0;
    bool ok = true;
    for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      if (!wwait(acc_full + buf, (uint32_t)((it >> 1) & 1))) { ok = false; break; }
      tc_fence_after();
      epilogue_tile(A, stg, tmem + lane_off + buf * BN, (tile % mt) * BM + quarter * 32, (tile / mt) * BN, half);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty + buf);
    }
    if (!ok && lane == 0) fail(kDevTimeoutEpilogue);
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------- CTA-pair tiles --
// 256 x 256 tiles on a cluster of two CTAs (one per SM).  CTA r of the pair loads A rows
// [m0 + 128 r, +128) and B rows [n0 + 128 r, +128) into its own shared memory; the even
// CTA issues M256 x N256 tcgen05.mma.cta_group::2, which reads both CTAs' tiles and
// leaves rows 128 r .. 128 r + 127 of the accumulator in CTA r's TMEM.  Each SM thus reads
// half of the B tile instead of all of it, and a stage is 32 KB per CTA (6 stages).
//   full[s]      on the even CTA: its producer's expect_tx(64 KB) + both CTAs' TMA bytes
//   empty[s]     on each CTA: arrived by the even CTA's MMA commit
//   acc_full[b]  on each CTA: arrived by the even CTA's MMA commit
//   acc_empty[b] on the even CTA: 8 epilogue warps of each CTA (16 arrivals)
namespace pair {
constexpr int kStages = 6;
constexpr int kABytes = 128 * 128;   // this CTA's 128 rows x 128 bytes of K
constexpr int kBBytes = 128 * 128;   // this CTA's half of the 256 B rows
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int staging = kStages * kStageBytes;
constexpr int bars = staging + kStagingBytes;
constexpr int nbars = 2 * kStages + 4 + 1;
constexpr int misc = bars + nbars * 8;
constexpr int alloc = misc + 64 + 1024;
}  // namespace pair

template <bool FP8>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                     const __grid_constant__ CUtensorMap tmd, Args A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars_p = reinterpret_cast<uint64_t*>(base + pair::bars);
  uint64_t* full = bars_p;
  uint64_t* empty = bars_p + pair::kStages;
  uint64_t* acc_full = bars_p + 2 * pair::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + pair::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + pair::misc + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const uint32_t peer = rank ^ 1;

  const int bn = A.bn;
  const int64_t mt = (A.M + 2 * BM - 1) / (2 * BM), nt = (A.N + bn - 1) / bn;
  const int64_t ntiles = mt * nt;
  const int64_t cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  constexpr int bk = FP8 ? 128 : 64;
  const int64_t nk = (A.K + bk - 1) / bk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < pair::kStages; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(acc_full + b, 1); mbar_init(acc_empty + b, 2 * kEpilogueWarps); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
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
    // --------------------------------------------- producer (both CTAs) --
    if (lane == 0) {
      prefetch_tmap(&tma);
      prefetch_tmap(&tmb);
    }
    const uint32_t full0 = mapa_shared(smem_u32(full), 0);  // the even CTA's full[0]
    int64_t g = 0;
    bool ok = true;
    for (int64_t tile = cid; ok && tile < ntiles; tile += ncl) {
      const int m0 = (int)((tile % mt) * (2 * BM) + rank * BM), n0 = (int)((tile / mt) * bn + rank * (bn / 2));
      for (int64_t kb = 0; kb < nk; ++kb, ++g) {
        const int s = (int)(g % pair::kStages);
        if (!wwait(empty + s, (uint32_t)(((g / pair::kStages) & 1) ^ 1))) { ok = false; break; }
        if (lane == 0) {
          uint8_t* st = base + s * pair::kStageBytes;
          if (leader) mbar_arrive_expect_tx(full + s, 2 * (pair::kABytes + (bn / 2) * 128));
          tma_load_2d_pair(st, &tma, (int)(kb * bk), m0, full0 + s * 8);
          tma_load_2d_pair(st + pair::kABytes, &tmb, (int)(kb * bk), n0, full0 + s * 8);
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      fail(kDevTimeoutProducer);
      if (leader)
        for (int64_t j = g > pair::kStages ? g - pair::kStages : 0; j < g; ++j) mbar_wait(full + (j % pair::kStages), (j / pair::kStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA (even CTA) --
    if (leader) {
      const uint32_t fmt16 = A.f16 ? 0u : 1u;
      const uint32_t idesc = FP8 ? make_idesc(1, 0, 0, 0, 0, 2 * BM, bn)
                                 : make_idesc(1, fmt16, fmt16, 0, 0, 2 * BM, bn);
      const uint64_t d0 = sdesc_sw128_kmajor(smem_u32(base));
      constexpr uint64_t kStageStep = pair::kStageBytes >> 4, kBOff = pair::kABytes >> 4;
      const uint32_t empty_own = smem_u32(empty), empty_peer = mapa_shared(smem_u32(empty), peer);
      const uint32_t accf_own = smem_u32(acc_full), accf_peer = mapa_shared(smem_u32(acc_full), peer);
      int64_t g = 0;
      int it = 0;
      bool ok = true;
      for (int64_t tile = cid; ok && tile < ntiles; tile += ncl, ++it) {
        const int buf = it & 1;
        if (!wwait(acc_empty + buf, (uint32_t)(((it >> 1) & 1) ^ 1))) { ok = false; break; }
        tc_fence_after();
        const uint32_t dt = tmem + buf * BN;
        for (int64_t kb = 0; kb < nk; ++kb, ++g) {
          const int s = (int)(g % pair::kStages);
          if (!wwait(full + s, (uint32_t)((g / pair::kStages) & 1))) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = d0 + (uint64_t)s * kStageStep, db = da + kBOff;
          if (lane == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              if constexpr (FP8)
                mma_f8f6f4_pair(dt, da + 2 * kk, db + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
              else
                mma_f16_pair(dt, da + 2 * kk, db + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            }
            tc_commit_pair(empty_own + s * 8);
            tc_commit_pair(empty_peer + s * 8);
          }
          __syncwarp();
        }
        if (ok && lane == 0) {
          tc_commit_pair(accf_own + buf * 8);
          tc_commit_pair(accf_peer + buf * 8);
        }
        __syncwarp();
      }
      if (lane == 0) {
        if (!ok) fail(kDevTimeoutMma);
        tc_commit_pair(smem_u32(drain));
        mbar_wait(drain, 0);
      }
      __syncwarp();
    }
  } else {
    // --------------------------------------------- epilogue (both CTAs) --
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t acce0 = mapa_shared(smem_u32(acc_empty), 0);
    Stager stg{base + pair::staging + (warp - 2) * 4096, &tmd, 0, A.M, A.d_f16};
    int it = 0;
    bool ok = true;
    for (int64_t tile = cid; ok && tile < ntiles; tile += ncl, ++it) {
      const int buf = it & 1;
      if (!wwait(acc_full + buf, (uint32_t)((it >> 1) & 1))) { ok = false; break; }
      tc_fence_after();
      const int64_t m0w = (tile % mt) * (2 * BM) + rank * BM + quarter * 32;
      epilogue_tile(A, stg, tmem + lane_off + buf * BN, m0w, (tile / mt) * bn, half);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce0 + buf * 8);
    }
    if (!ok && lane == 0) fail(kDevTimeoutEpilogue);
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the pair's MMAs and both epilogues are done with TMEM
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
template <typename K>
static cudaError_t pair_clusters(K* kern, int* out);

// Shared-memory attribute of the pair kernel (per device) and the resident pair count.
static cudaError_t pair_setup(bool fp8, int* clusters) {
  static std::atomic<uint64_t> attr{0}, attr8{0};
  auto kern = fp8 ? gemm_pair_kernel<true> : gemm_pair_kernel<false>;
  cudaError_t e = qf2_set_smem_once(kern, pair::alloc, fp8 ? &attr8 : &attr);
  if (e != cudaSuccess) return e;
  return pair_clusters(kern, clusters);
}

// Tile width of the CTA-pair kernel: among 256 / 192 / 128 the one with the least
// estimated time, rounds of the persistent grid x per-tile cost.  Narrower tiles keep
// fewer MMA cycles in flight per stage against the same TMA latency; measured per-column
// costs on bf16 and e4m3 problems of 2304-15360 columns are about 1.0 / 1.25 / 1.8.
static int pick_bn(int64_t M, int64_t N, int clusters) {
  const int cand[3] = {256, 192, 128};
  const double cost[3] = {1.0, 1.25, 1.8};
  const int64_t mt = (M + 2 * BM - 1) / (2 * BM);
  int best = 256;
  double best_t = 1e300;
  for (int i = 0; i < 3; ++i) {
    const int64_t tiles = mt * ((N + cand[i] - 1) / cand[i]);
    const int64_t rounds = (tiles + clusters - 1) / clusters;
    const double t = (double)rounds * cand[i] * cost[i];
    if (t < best_t - 1e-9) { best_t = t; best = cand[i]; }
  }
  return best;
}

// How many CTA pairs of gemm_pair_kernel are resident at once on the current device
// (the persistent grid's size), cached per device.  Needs the smem attribute set.
template <typename K>
static cudaError_t pair_clusters(K* kern, int* out) {
  static std::atomic<int> cache[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int v = cache[dev & 63].load(std::memory_order_relaxed);
  if (v == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = pair::alloc;
    e = cudaOccupancyMaxActiveClusters(&v, kern, &cfg);
    if (e != cudaSuccess) return e;
    if (v <= 0) return cudaErrorInvalidConfiguration;
    cache[dev & 63].store(v, std::memory_order_relaxed);
  }
  *out = v;
  return cudaSuccess;
}

}  // namespace gemm
}  // namespace qf2

using namespace qf2::gemm;

static int gemm_run(const void* a, int64_t lda, const void* b, int64_t ldb, void* d, int64_t ldd, int64_t M, int64_t N,
                    int64_t K, int ab_dtype, int d_dtype, const float* row_scale, const float* col_scale,
                    const void* bias, int bias_dtype, int64_t gelu_col0, int glu, const void* residual, int64_t ldr,
                    const void* gate, int64_t gate_stride, int64_t rows_per_gate, const int64_t* row_idx,
                    int64_t idx_rows, int64_t out_rows, void* workspace, int64_t workspace_bytes,
                    qf2_stream_t stream) {
  if (!a || !b || !d) return QF2_ERR_ARG;
  if (ab_dtype != QF2_BF16 && ab_dtype != QF2_F16 && ab_dtype != QF2_E4M3) return QF2_ERR_DTYPE;
  if (d_dtype != QF2_BF16 && d_dtype != QF2_F16 && d_dtype != QF2_F32) return QF2_ERR_DTYPE;
  // the fused residual / SwiGLU epilogues read and write bf16 only
  if (d_dtype == QF2_F16 && (residual || glu)) return QF2_ERR_DTYPE;
  if (bias && bias_dtype != QF2_BF16 && bias_dtype != QF2_F32) return QF2_ERR_DTYPE;
  if (M <= 0 || N <= 0 || K <= 0 || (N % 8)) return QF2_ERR_SHAPE;
  if (residual && (ldr < N || (gate && rows_per_gate <= 0))) return QF2_ERR_SHAPE;
  if (glu && (N % BN || residual || gelu_col0 >= 0 || d_dtype != QF2_BF16)) return QF2_ERR_SHAPE;
  const int esz = ab_dtype == QF2_E4M3 ? 1 : 2;
  if (!al16(a) || !al16(b) || !al16(d) || (lda * esz) % 16 || (ldb * esz) % 16 || (ldd % 8) || lda < K || ldb < K ||
      ldd < (glu ? N / 2 : N))
    return QF2_ERR_ALIGN;
  if (!workspace || workspace_bytes < 256 || !al16(workspace)) return QF2_ERR_WORKSPACE;
  const CUtensorMapDataType tdt = ab_dtype == QF2_E4M3  ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                  : ab_dtype == QF2_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t bk = ab_dtype == QF2_E4M3 ? 128 : 64;
  // CTA pairs (256-row tiles) once there are two 128-row tiles of A; single CTAs for the
  // thin products (adaLN / embedding linears on a few rows)
  const bool use_pair = M > BM;
  CUtensorMap ma, mb;
  const uint64_t da[2] = {(uint64_t)K, (uint64_t)M}, db[2] = {(uint64_t)K, (uint64_t)N};
  int clusters = 0, bn = BN;
  if (use_pair) {
    QF2_CUDA_CHECK(pair_setup(ab_dtype == QF2_E4M3, &clusters));
    if (!glu) bn = pick_bn(M, N, clusters);
  }
  const uint32_t ba[2] = {bk, (uint32_t)BM}, bb[2] = {bk, (uint32_t)(use_pair ? bn / 2 : BN)};
  if (!qf2_make_tmap_2d(&ma, tdt, a, da, (uint64_t)lda * esz, ba) ||
      !qf2_make_tmap_2d(&mb, tdt, b, db, (uint64_t)ldb * esz, bb))
    return QF2_ERR_ALIGN;
  // 16-bit output goes out through 32 x 32 TMA stores; the fp32 output map is never used
  CUtensorMap md;
  const uint64_t dd[2] = {(uint64_t)(glu ? N / 2 : N), (uint64_t)M};
  const uint32_t bd[2] = {32, 32};
  if (d_dtype != QF2_F32 && !row_idx &&
      !qf2_make_tmap_2d_sw64(&md, d_dtype == QF2_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                             d, dd, (uint64_t)ldd * 2, bd))
    return QF2_ERR_ALIGN;
  if (d_dtype == QF2_F32 || row_idx) md = ma;
  Args args;
  args.d = d;
  args.ldd = ldd;
  args.M = M; args.N = N; args.K = K;
  args.row_scale = row_scale;
  args.col_scale = col_scale;
  args.bias = bias;
  args.bias_f32 = bias_dtype == QF2_F32;
  args.d_f32 = d_dtype == QF2_F32;
  args.d_f16 = d_dtype == QF2_F16;
  args.fp8 = ab_dtype == QF2_E4M3;
  args.f16 = ab_dtype == QF2_F16;
  args.gelu_col0 = gelu_col0 < 0 ? INT64_MAX : gelu_col0;
  args.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  args.ldr = ldr;
  args.gate = reinterpret_cast<const __nv_bfloat16*>(gate);
  args.gate_stride = gate_stride;
  args.rows_per_gate = rows_per_gate > 0 ? rows_per_gate : 1;
  args.glu = glu != 0;
  args.bn = bn;
  args.vec_ok = al16(col_scale) && al16(bias) && al16(residual) && al16(gate) && (ldr % 8) == 0 &&
                (gate_stride % 8) == 0;
  if (glu && !args.vec_ok) return QF2_ERR_ALIGN;
  args.status = reinterpret_cast<int*>(workspace);
  args.row_idx = row_idx;
  args.idx_rows = idx_rows > 0 ? idx_rows : 1;
  args.out_rows = out_rows;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  QF2_CUDA_CHECK(cudaMemsetAsync(workspace, 0, sizeof(int), s));
  if (use_pair) {
    auto kern = args.fp8 ? gemm_pair_kernel<true> : gemm_pair_kernel<false>;
    const int64_t ntiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + bn - 1) / bn);
    const unsigned grid = 2 * (unsigned)std::min<int64_t>(ntiles, clusters);
    kern<<<grid, kThreads, pair::alloc, s>>>(ma, mb, md, args);
  } else {
    static std::atomic<uint64_t> attr_done{0}, attr_done8{0};
    auto kern = args.fp8 ? gemm_kernel<true> : gemm_kernel<false>;
    QF2_CUDA_CHECK(qf2_set_smem_once(kern, Smem::alloc, args.fp8 ? &attr_done8 : &attr_done));
    int sms = 148;
    QF2_CUDA_CHECK(qf2_sm_count(&sms));
    const int64_t ntiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const unsigned grid = (unsigned)std::min<int64_t>(ntiles, sms);
    kern<<<grid, kThreads, Smem::alloc, s>>>(ma, mb, md, args);
  }
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}

extern "C" int qf2_gemm_ex(const void* a, int64_t lda, const void* b, int64_t ldb, void* d, int64_t ldd, int64_t M,
                           int64_t N, int64_t K, int ab_dtype, int d_dtype, const float* row_scale,
                           const float* col_scale, const void* bias, int bias_dtype, int64_t gelu_col0, int glu,
                           const void* residual, int64_t ldr, const void* gate, int64_t gate_stride,
                           int64_t rows_per_gate, void* workspace, int64_t workspace_bytes, qf2_stream_t stream) {
  return gemm_run(a, lda, b, ldb, d, ldd, M, N, K, ab_dtype, d_dtype, row_scale, col_scale, bias, bias_dtype, gelu_col0,
                  glu, residual, ldr, gate, gate_stride, rows_per_gate, nullptr, 0, 0, workspace, workspace_bytes,
                  stream);
}

extern "C" int qf2_gemm_rows_indexed(const void* a, int64_t lda, const void* b, int64_t ldb, void* d, int64_t ldd,
                                     int64_t batch, int64_t M, int64_t N, int64_t K, int ab_dtype, int d_dtype,
                                     const int64_t* row_idx, int64_t out_rows, const float* col_scale,
                                     const void* bias, int bias_dtype, void* workspace, int64_t workspace_bytes,
                                     qf2_stream_t stream) {
  if (!row_idx) return QF2_ERR_ARG;
  if (batch <= 0 || M <= 0 || out_rows < 1) return QF2_ERR_SHAPE;
  // a's rows are the batch's M rows one after another (row stride lda); a row whose index
  // is outside [0, out_rows) is not written and sets the workspace status word
  return gemm_run(a, lda, b, ldb, d, ldd, batch * M, N, K, ab_dtype, d_dtype, nullptr, col_scale, bias, bias_dtype, -1,
                  0, nullptr, 0, nullptr, 0, 1, row_idx, M, out_rows, workspace, workspace_bytes, stream);
}

extern "C" int qf2_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, void* d, int64_t ldd, int64_t M,
                        int64_t N, int64_t K, int ab_dtype, int d_dtype, const float* row_scale,
                        const float* col_scale, const void* bias, int bias_dtype, void* workspace,
                        int64_t workspace_bytes, qf2_stream_t stream) {
  return qf2_gemm_ex(a, lda, b, ldb, d, ldd, M, N, K, ab_dtype, d_dtype, row_scale, col_scale, bias, bias_dtype, -1, 0,
                     nullptr, 0, nullptr, 0, 1, workspace, workspace_bytes, stream);
}
