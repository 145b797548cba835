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
//   warps 10-13 (weight-code kernels only) converters: B arrives as 8-bit weight codes
//              (int8 or e4m3, half the bytes of a 16-bit copy) and is rewritten in shared
//              memory as the exact 16-bit values of the activations' type before the MMA
#include "qf2_common.cuh"

#include <algorithm>
#include <climits>
#include <type_traits>

namespace qf2 {
namespace gemm {

constexpr int BM = 128, BN = 256;
constexpr int kThreads = 320;           // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kEpilogueWarps = 8;
constexpr uint32_t kTmemCols = 512;  // two 256-column fp32 accumulators

// per epilogue warp: two 32 x 32 bf16 output staging tiles (64-byte swizzle) for TMA stores
constexpr int kStagingBytes = kEpilogueWarps * 2 * 2048;

// Operand kinds of the kernels: 16-bit A and B (kind::f16), e4m3 A and B (kind::f8f6f4),
// or 16-bit A with 8-bit weight codes for B, converted in shared memory (kind::f16).
enum Kind { kK16 = 0, kKE4M3 = 1, kKCodes = 2 };
constexpr int kConvWarps = 4;
constexpr int kConvThreads = 32 * kConvWarps;

// Shared-memory layout per kernel kind and tile form.  A stage holds the A tile (128 rows
// x 128 bytes of K) and the B tile this CTA feeds the MMA (256 rows, or 128 in a CTA pair);
// the single-CTA weight-code kernel adds a staging slot per stage for the codes as they
// arrive (256 rows x 64 bytes), and has one stage fewer to make room.
template <int KIND, bool PAIR>
struct Lay {
  static_assert(!(PAIR && KIND == kKCodes), "weight codes run on the single-CTA gemm_kernel");
  static constexpr bool codes = KIND == kKCodes;
  static constexpr int stages = PAIR ? 6 : (codes ? 3 : 4);
  // the single-CTA kernel also runs 128- and 64-column tiles (thin products), whose
  // smaller stages (and code slots) fit more times into the same region
  static constexpr int max_stages = PAIR ? stages : 8;
  static constexpr int a_bytes = BM * 128;
  static constexpr int b_rows = PAIR ? 128 : BN;
  static constexpr int b_bytes = b_rows * 128;
  static constexpr int stage_bytes = a_bytes + b_bytes;
  static constexpr int raw_bytes = codes ? b_rows * 64 : 0;
  static constexpr int raw = stages * stage_bytes;
  static constexpr int staging = raw + stages * raw_bytes;
  static constexpr int bars = staging + kStagingBytes;
  // full, empty, raw_full per stage; acc_full, acc_empty per accumulator; drain
  static constexpr int nbars = 3 * max_stages + 4 + 1;
  static constexpr int misc = bars + nbars * 8;
  static constexpr int alloc = misc + 64 + 1024;
  static constexpr int threads = codes ? kThreads + kConvThreads : kThreads;
  static_assert(alloc <= 227 * 1024, "shared memory");
};

// Two 8-bit codes (bytes 0 and 2 of r; bytes 1 and 3 zero) -> their exact 16-bit values.
//   int8 -> bf16: bf16(128 + (c & 127)) - bf16(c < 0 ? 256 : 128); operands and result are
//                 integers of at most 8 significant bits, so the subtraction is exact
//   int8 -> fp16: fp16(1024 + (c + 128)) - 1152, exact (integers below 2048)
QF2_DEV uint32_t i8x2_to_bf16x2(uint32_t r) {
  const uint32_t hi = (r & 0x007F007Fu) | 0x43004300u;
  const uint32_t lo = (r & 0x00800080u) | 0x43004300u;
  uint32_t o;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(o) : "r"(hi), "r"(lo));
  return o;
}
QF2_DEV uint32_t i8x2_to_f16x2(uint32_t r) {
  const uint32_t v = (r ^ 0x00800080u) | 0x64006400u;
  uint32_t o;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(o) : "r"(v), "r"(0x64806480u));
  return o;
}
// Two e4m3 codes (bytes 0 and 1 of b) -> fp16x2 (exact: every e4m3 value is an fp16 normal)
// or bf16x2 (through fp32, exact likewise).
QF2_DEV uint32_t e4m3x2_to_16(uint32_t b, bool f16) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(b & 0xffffu), __NV_E4M3);
  if (f16) return (uint32_t)h.x | ((uint32_t)h.y << 16);
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
  __nv_bfloat162 t = __floats2bfloat162_rn(f.x, f.y);
  return *reinterpret_cast<uint32_t*>(&t);
}

// Converter side of the weight-code kernels: the codes of a B tile (row-major, 64 bytes of
// K per row, as TMA wrote them without swizzle) -> the K-major 128-byte-swizzled 16-bit
// tile the MMA reads (16-byte chunk j of row r at r * 128 + ((j ^ (r % 8)) * 16)).  Thread
// ct converts 16-byte code chunks ct, ct + kConvThreads, ... (chunk k = row k / 4, codes
// 16 (k % 4) .. + 15 -> output chunks 2 (k % 4) and 2 (k % 4) + 1; the second sits at the
// first's offset ^ 16).  The offsets are fixed for the kernel's life and computed once.
template <int CHUNKS>
struct ConvPlan {
  uint32_t src[CHUNKS];  // byte offset of the code chunk in its staging slot
  uint32_t dst[CHUNKS];  // byte offset of its first output chunk in the 16-bit tile
  int n;                 // chunks this thread converts (the tile may have fewer rows)
  QF2_DEV ConvPlan(int ct, int nchunks) : n(0) {
#pragma unroll
    for (int i = 0; i < CHUNKS; ++i) {
      const uint32_t k = (uint32_t)(ct + i * kConvThreads), r = k >> 2, c = k & 3;
      src[i] = k * 16;
      dst[i] = r * 128 + (((2 * c) ^ (r & 7)) << 4);
      if ((int)k < nchunks) n = i + 1;
    }
  }
};

// One staging slot -> one 16-bit tile.  FMT QF2_I8 / QF2_E4M3, F16: fp16 (else bf16)
// output.  All loads first: the stores cannot alias them, but the compiler cannot tell.
template <int CHUNKS, int FMT, bool F16>
QF2_DEV void convert_codes_tile(const uint8_t* raw, uint8_t* dst, const ConvPlan<CHUNKS>& p) {
  uint4 v[CHUNKS];
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i)
    if (i < p.n) v[i] = *reinterpret_cast<const uint4*>(raw + p.src[i]);
#pragma unroll
  for (int i = 0; i < CHUNKS; ++i) {
    if (i >= p.n) break;
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    uint32_t o[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if constexpr (FMT == QF2_E4M3) {
        o[2 * q] = e4m3x2_to_16(w[q], F16);
        o[2 * q + 1] = e4m3x2_to_16(w[q] >> 16, F16);
      } else {
        const uint32_t r01 = __byte_perm(w[q], 0u, 0x4140), r23 = __byte_perm(w[q], 0u, 0x4342);
        o[2 * q] = F16 ? i8x2_to_f16x2(r01) : i8x2_to_bf16x2(r01);
        o[2 * q + 1] = F16 ? i8x2_to_f16x2(r23) : i8x2_to_bf16x2(r23);
      }
    }
    *reinterpret_cast<uint4*>(dst + p.dst[i]) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(dst + (p.dst[i] ^ 16u)) = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// Calls body(std::integral_constant<int, FMT>, std::integral_constant<bool, F16>) for the
// run-time code format and activation type: the converter loop is compiled once per pair.
template <typename F>
QF2_DEV void with_code_format(int fmt, bool f16, F&& body) {
  if (fmt == QF2_E4M3) {
    if (f16) body(std::integral_constant<int, QF2_E4M3>{}, std::true_type{});
    else body(std::integral_constant<int, QF2_E4M3>{}, std::false_type{});
  } else {
    if (f16) body(std::integral_constant<int, QF2_I8>{}, std::true_type{});
    else body(std::integral_constant<int, QF2_I8>{}, std::false_type{});
  }
}

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
  int b_fmt;      // weight-code kernels: B codes QF2_I8 or QF2_E4M3
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
    // B's rows come in groups of 256: [128 gate rows | their 128 up rows].  A tile of
    // width bn holds bn / 2 gate columns then their bn / 2 up columns (bn = 256: one whole
    // group; bn = 128: the gate and up quarters of one, rows 64 (n_tile % 256) / 128 on):
    // gate at accumulator column col, up at gh + col, weight row src0 + col (+ 128 for
    // up), output column n_tile / 2 + col.  This half takes gh / 2 columns (N % 256 == 0,
    // vec_ok).
    const int gh = A.bn / 2;
    const int64_t src0 = (n_tile / 256) * 256 + (n_tile % 256) / 2;
#pragma unroll 1
    for (int c = 0; c < gh / 64; ++c) {
      uint32_t vg[32], vu[32];
      const int col = half * (gh / 2) + c * 32;
      tmem_ld32(tacc + col, vg);
      tmem_ld32(tacc + gh + col, vu);
      tmem_wait_ld();
      const int64_t ns = src0 + col;
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
// 128 x 256 tiles, one CTA per SM (small M: the adaLN / embedding linears).  Also the
// weight-code kernel (KIND kKCodes), for every M: B arrives as 8-bit codes and warps 10-13
// rewrite each stage's bn x 64 codes as 16-bit values in shared memory.  That conversion
// is repeated for every 128-row tile of A and its shared-memory traffic (1 byte read and 2
// written per code) comes on top of the operand traffic of the tile, so it pays where one
// tile of A covers M (the weight is read at 1 byte instead of 2 and no expansion kernel
// runs); for M of a few thousand rows one expansion per call followed by the 16-bit
// product is faster (measured: 4352 x 12288 x 2304 in 0.44 ms here against 0.21 ms), and
// neither 256 x 128 single-CTA tiles (two M = 128 accumulators sharing the converted B)
// nor CTA pairs (each CTA converting its half of B, handed to the even CTA's MMA issuer
// through a cluster barrier) came near it: 0.31-0.51 ms.
template <int KIND>
__global__ void __launch_bounds__(Lay<KIND, false>::threads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                const __grid_constant__ CUtensorMap tmd, Args A) {
  using L = Lay<KIND, false>;
  constexpr bool FP8 = KIND == kKE4M3, CODES = KIND == kKCodes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + L::bars);
  uint64_t* full = bars;
  uint64_t* empty = bars + L::max_stages;
  uint64_t* acc_full = bars + 2 * L::max_stages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* raw_full = drain + 1;  // weight-code kernels: A tile + B codes landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + L::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + L::misc + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // tile width (256, or 128 / 64 for thin products) and the stages (A + B tiles, and for
  // weight codes a code slot each) that fit into the region at that width
  const int bn = A.bn;
  const int sbytes = L::a_bytes + bn * 128;
  const int rbytes = CODES ? bn * 64 : 0;
  const int ns = min(L::max_stages, L::staging / (sbytes + rbytes));
  uint8_t* const raw_base = base + ns * sbytes;  // code slots after the stages
  const int64_t mt = (A.M + BM - 1) / BM, nt = (A.N + bn - 1) / bn;
  const int64_t ntiles = mt * nt;
  constexpr int bk = FP8 ? 128 : 64;  // K elements per stage (128 bytes)
  const int64_t nk = (A.K + bk - 1) / bk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(full + s, CODES ? kConvWarps : 1);
      mbar_init(empty + s, 1);
      mbar_init(raw_full + s, 1);
    }
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
    // the barrier each stage's copies complete on: full, or raw_full when converters
    // stand between the copies and the MMA
    uint64_t* landed = CODES ? raw_full : full;
    int64_t g = 0;
    bool ok = true;
    for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      const int m0 = (int)((tile % mt) * BM), n0 = (int)((tile / mt) * bn);
      for (int64_t kb = 0; kb < nk; ++kb, ++g) {
        const int s = (int)(g % ns);
        if (!wwait(empty + s, (uint32_t)(((g / ns) & 1) ^ 1))) { ok = false; break; }
        if (lane == 0) {
          uint8_t* st = base + s * sbytes;
          mbar_arrive_expect_tx(landed + s, CODES ? L::a_bytes + rbytes : sbytes);
          tma_load_2d(st, &tma, (int)(kb * bk), m0, landed + s);
          tma_load_2d(CODES ? raw_base + s * rbytes : st + L::a_bytes, &tmb, (int)(kb * bk), n0,
                      landed + s);
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      fail(kDevTimeoutProducer);
      // let issued copies land before the CTA's shared memory goes away
      for (int64_t j = g > ns ? g - ns : 0; j < g; ++j) mbar_wait(landed + (j % ns), (j / ns) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA --
    // e4m3 x e4m3, bf16 x bf16 or fp16 x fp16 -> f32 (the 16-bit format is a descriptor
    // field, not a branch between the MMAs)
    const uint32_t fmt16 = A.f16 ? 0u : 1u;
    const uint32_t idesc = FP8 ? make_idesc(1, 0, 0, 0, 0, BM, bn) : make_idesc(1, fmt16, fmt16, 0, 0, BM, bn);
    const uint64_t d0 = sdesc_sw128_kmajor(smem_u32(base));
    const uint64_t kStageStep = (uint64_t)(sbytes >> 4);
    constexpr uint64_t kBOff = L::a_bytes >> 4;
    int64_t g = 0;
    int it = 0;
    bool ok = true;
    for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      if (!wwait(acc_empty + buf, (uint32_t)(((it >> 1) & 1) ^ 1))) { ok = false; break; }
      tc_fence_after();
      const uint32_t dt = tmem + buf * BN;
      for (int64_t kb = 0; kb < nk; ++kb, ++g) {
        const int s = (int)(g % ns);
        if (!wwait(full + s, (uint32_t)((g / ns) & 1))) { ok = false; break; }
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
  } else if (warp < 2 + kEpilogueWarps) {
    // ------------------------------------------------------- epilogue --
    // 8 warps: lane quarter = warp & 3 (TMEM lanes / tile rows), column half = (warp - 2) / 4
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    Stager stg{base + L::staging + (warp - 2) * 4096, &tmd, 0, A.M, A.d_f16};
    int it = 0;
    bool ok = true;
    for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++it) {
      const int buf = it & 1;
      if (!wwait(acc_full + buf, (uint32_t)((it >> 1) & 1))) { ok = false; break; }
      tc_fence_after();
      epilogue_tile(A, stg, tmem + lane_off + buf * BN, (tile % mt) * BM + quarter * 32, (tile / mt) * bn, half);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty + buf);
    }
    if (!ok && lane == 0) fail(kDevTimeoutEpilogue);
    if (lane == 0) bulk_wait_all();
  } else if constexpr (CODES) {
    // ----------------------------------------------------- converters --
    constexpr int kChunks = L::raw_bytes / 16 / kConvThreads;
    const ConvPlan<kChunks> plan(threadIdx.x - 32 * (2 + kEpilogueWarps), bn * 4);
    bool ok = true;
    with_code_format(A.b_fmt, A.f16 != 0, [&](auto fmt_c, auto f16_c) {
      int64_t g = 0;
      for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
        for (int64_t kb = 0; kb < nk; ++kb, ++g) {
          const int s = (int)(g % ns);
          if (!wwait(raw_full + s, (uint32_t)((g / ns) & 1))) { ok = false; break; }
          convert_codes_tile<kChunks, decltype(fmt_c)::value, decltype(f16_c)::value>(
              raw_base + s * rbytes, base + s * sbytes + L::a_bytes, plan);
          fence_async_smem();  // the generic-proxy writes, before the MMA reads them
          __syncwarp();
          if (lane == 0) mbar_arrive(full + s);
        }
      }
    });
    if (!ok && lane == 0) fail(kDevTimeoutConvert);
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
template <int KIND>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Lay<KIND, true>::threads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                     const __grid_constant__ CUtensorMap tmd, Args A) {
  static_assert(KIND != kKCodes, "weight codes run on the single-CTA gemm_kernel");
  using L = Lay<KIND, true>;
  constexpr bool FP8 = KIND == kKE4M3;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars_p = reinterpret_cast<uint64_t*>(base + L::bars);
  uint64_t* full = bars_p;
  uint64_t* empty = bars_p + L::stages;
  uint64_t* acc_full = bars_p + 2 * L::stages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + L::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + L::misc + 8);
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
    // full[s] of the even CTA completes on its expect_tx and the TMA bytes of both CTAs
    for (int s = 0; s < L::stages; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
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
    const uint32_t full0 = mapa_shared(smem_u32(full), 0);  // the even CTA's full[0]
    if (lane == 0) {
      prefetch_tmap(&tma);
      prefetch_tmap(&tmb);
    }
    int64_t g = 0;
    bool ok = true;
    for (int64_t tile = cid; ok && tile < ntiles; tile += ncl) {
      const int m0 = (int)((tile % mt) * (2 * BM) + rank * BM), n0 = (int)((tile / mt) * bn + rank * (bn / 2));
      for (int64_t kb = 0; kb < nk; ++kb, ++g) {
        const int s = (int)(g % L::stages);
        if (!wwait(empty + s, (uint32_t)(((g / L::stages) & 1) ^ 1))) { ok = false; break; }
        if (lane == 0) {
          uint8_t* st = base + s * L::stage_bytes;
          if (leader) mbar_arrive_expect_tx(full + s, 2 * (L::a_bytes + (bn / 2) * 128));
          tma_load_2d_pair(st, &tma, (int)(kb * bk), m0, full0 + s * 8);
          tma_load_2d_pair(st + L::a_bytes, &tmb, (int)(kb * bk), n0, full0 + s * 8);
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      fail(kDevTimeoutProducer);
      if (leader)
        for (int64_t j = g > L::stages ? g - L::stages : 0; j < g; ++j)
          mbar_wait(full + (j % L::stages), (j / L::stages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA (even CTA) --
    if (leader) {
      const uint32_t fmt16 = A.f16 ? 0u : 1u;
      const uint32_t idesc = FP8 ? make_idesc(1, 0, 0, 0, 0, 2 * BM, bn)
                                 : make_idesc(1, fmt16, fmt16, 0, 0, 2 * BM, bn);
      const uint64_t d0 = sdesc_sw128_kmajor(smem_u32(base));
      constexpr uint64_t kStageStep = L::stage_bytes >> 4, kBOff = L::a_bytes >> 4;
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
          const int s = (int)(g % L::stages);
          if (!wwait(full + s, (uint32_t)((g / L::stages) & 1))) { ok = false; break; }
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
    Stager stg{base + L::staging + (warp - 2) * 4096, &tmd, 0, A.M, A.d_f16};
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
template <typename Kern>
static cudaError_t pair_clusters(Kern* kern, int threads, int smem, std::atomic<int>* cache, int* out);

template <int KIND>
static cudaError_t pair_setup_kind(int* clusters) {
  static std::atomic<uint64_t> attr{0};
  static std::atomic<int> cache[64];
  cudaError_t e = qf2_set_smem_once(gemm_pair_kernel<KIND>, Lay<KIND, true>::alloc, &attr);
  if (e != cudaSuccess) return e;
  return pair_clusters(gemm_pair_kernel<KIND>, Lay<KIND, true>::threads, Lay<KIND, true>::alloc, cache, clusters);
}

// Shared-memory attribute of a CTA-pair kernel (per device) and its resident pair count.
static cudaError_t pair_setup(int kind, int* clusters) {
  return kind == kKE4M3 ? pair_setup_kind<kKE4M3>(clusters) : pair_setup_kind<kK16>(clusters);
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

// Tile width of the single-CTA kernel for products of at most 128 rows: 256, 128 or 64
// columns, the one with the least estimated time = rounds of the one-CTA-per-SM grid x
// the bytes a stage moves (A's 16 KB + B's width x 128 bytes, relative to a 256 tile):
// a thin product's tiles are few and each walks all of K, so narrower tiles (with deeper
// rings: 6 or 8 stages) put more SMs on it.
static int pick_bn_thin(int64_t M, int64_t N, int sms) {
  const int cand[3] = {256, 128, 64};
  const int64_t mt = (M + BM - 1) / BM;
  int best = 256;
  double best_t = 1e300;
  for (int i = 0; i < 3; ++i) {
    const int64_t tiles = mt * ((N + cand[i] - 1) / cand[i]);
    const int64_t rounds = (tiles + sms - 1) / sms;
    const double t = (double)rounds * (128.0 + cand[i]) / 384.0;
    if (t < best_t - 1e-9) { best_t = t; best = cand[i]; }
  }
  return best;
}

// How many CTA pairs of gemm_pair_kernel are resident at once on the current device
// (the persistent grid's size), cached per device.  Needs the smem attribute set.
template <typename Kern>
static cudaError_t pair_clusters(Kern* kern, int threads, int smem, std::atomic<int>* cache, int* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int v = cache[dev & 63].load(std::memory_order_relaxed);
  if (v == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
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

// ab_dtype: the operands' type (A's, and B's unless b_codes); b_codes: 0, or QF2_I8 /
// QF2_E4M3 when B holds 8-bit weight codes that the kernel converts to ab_dtype (16-bit).
static int gemm_run(const void* a, int64_t lda, const void* b, int64_t ldb, void* d, int64_t ldd, int64_t M, int64_t N,
                    int64_t K, int ab_dtype, int d_dtype, const float* row_scale, const float* col_scale,
                    const void* bias, int bias_dtype, int64_t gelu_col0, int glu, const void* residual, int64_t ldr,
                    const void* gate, int64_t gate_stride, int64_t rows_per_gate, const int64_t* row_idx,
                    int64_t idx_rows, int64_t out_rows, void* workspace, int64_t workspace_bytes,
                    qf2_stream_t stream, int b_codes = 0) {
  if (!a || !b || !d) return QF2_ERR_ARG;
  if (ab_dtype != QF2_BF16 && ab_dtype != QF2_F16 && ab_dtype != QF2_E4M3) return QF2_ERR_DTYPE;
  if (b_codes && ((b_codes != QF2_I8 && b_codes != QF2_E4M3) || ab_dtype == QF2_E4M3)) return QF2_ERR_DTYPE;
  if (d_dtype != QF2_BF16 && d_dtype != QF2_F16 && d_dtype != QF2_F32) return QF2_ERR_DTYPE;
  // the fused residual / SwiGLU epilogues read and write bf16 only
  if (d_dtype == QF2_F16 && (residual || glu)) return QF2_ERR_DTYPE;
  if (bias && bias_dtype != QF2_BF16 && bias_dtype != QF2_F32) return QF2_ERR_DTYPE;
  if (M <= 0 || N <= 0 || K <= 0 || (N % 8)) return QF2_ERR_SHAPE;
  if (residual && (ldr < N || (gate && rows_per_gate <= 0))) return QF2_ERR_SHAPE;
  if (glu && (N % BN || residual || gelu_col0 >= 0 || d_dtype != QF2_BF16)) return QF2_ERR_SHAPE;
  const int esz = ab_dtype == QF2_E4M3 ? 1 : 2, bsz = b_codes ? 1 : esz;
  if (!al16(a) || !al16(b) || !al16(d) || (lda * esz) % 16 || (ldb * bsz) % 16 || (ldd % 8) || lda < K || ldb < K ||
      ldd < (glu ? N / 2 : N))
    return QF2_ERR_ALIGN;
  const int kind = ab_dtype == QF2_E4M3 ? kKE4M3 : b_codes ? kKCodes : kK16;
  if (!workspace || workspace_bytes < 256 || !al16(workspace)) return QF2_ERR_WORKSPACE;
  const CUtensorMapDataType tdt = ab_dtype == QF2_E4M3  ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                  : ab_dtype == QF2_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t bk = ab_dtype == QF2_E4M3 ? 128 : 64;
  // CTA pairs (256-row tiles) once there are two 128-row tiles of A; single CTAs for the
  // thin products (adaLN / embedding linears on a few rows)
  // weight codes always run on single-CTA tiles (see gemm_kernel)
  const bool use_pair = M > BM && kind != kKCodes;
  CUtensorMap ma, mb;
  const uint64_t da[2] = {(uint64_t)K, (uint64_t)M}, db[2] = {(uint64_t)K, (uint64_t)N};
  int clusters = 0, bn = BN, sms = 148;
  QF2_CUDA_CHECK(qf2_sm_count(&sms));
  if (use_pair) {
    QF2_CUDA_CHECK(pair_setup(kind, &clusters));
    if (!glu) bn = pick_bn(M, N, clusters);
  } else if (!glu) {
    bn = pick_bn_thin(M, N, sms);
  }
  const uint32_t ba[2] = {bk, (uint32_t)BM},
                 bb[2] = {bk, (uint32_t)(use_pair ? bn / 2 : bn)};
  // weight codes: bk bytes of K per row, unswizzled (the converters rewrite them)
  const bool bmap_ok = b_codes ? qf2_make_tmap_2d_noswizzle(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, db, (uint64_t)ldb, bb)
                               : qf2_make_tmap_2d(&mb, tdt, b, db, (uint64_t)ldb * esz, bb);
  if (!qf2_make_tmap_2d(&ma, tdt, a, da, (uint64_t)lda * esz, ba) || !bmap_ok) return QF2_ERR_ALIGN;
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
  args.b_fmt = b_codes;
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
    const int64_t ntiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + bn - 1) / bn);
    const unsigned grid = 2 * (unsigned)std::min<int64_t>(ntiles, clusters);
    if (kind == kKE4M3)
      gemm_pair_kernel<kKE4M3><<<grid, Lay<kKE4M3, true>::threads, Lay<kKE4M3, true>::alloc, s>>>(ma, mb, md, args);
    else
      gemm_pair_kernel<kK16><<<grid, Lay<kK16, true>::threads, Lay<kK16, true>::alloc, s>>>(ma, mb, md, args);
  } else {
    static std::atomic<uint64_t> attr_done[3];
    const int64_t ntiles = ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
    const unsigned grid = (unsigned)std::min<int64_t>(ntiles, sms);
    if (kind == kKE4M3) {
      QF2_CUDA_CHECK(qf2_set_smem_once(gemm_kernel<kKE4M3>, Lay<kKE4M3, false>::alloc, &attr_done[kind]));
      gemm_kernel<kKE4M3><<<grid, Lay<kKE4M3, false>::threads, Lay<kKE4M3, false>::alloc, s>>>(ma, mb, md, args);
    } else if (kind == kKCodes) {
      QF2_CUDA_CHECK(qf2_set_smem_once(gemm_kernel<kKCodes>, Lay<kKCodes, false>::alloc, &attr_done[kind]));
      gemm_kernel<kKCodes><<<grid, Lay<kKCodes, false>::threads, Lay<kKCodes, false>::alloc, s>>>(ma, mb, md, args);
    } else {
      QF2_CUDA_CHECK(qf2_set_smem_once(gemm_kernel<kK16>, Lay<kK16, false>::alloc, &attr_done[kind]));
      gemm_kernel<kK16><<<grid, Lay<kK16, false>::threads, Lay<kK16, false>::alloc, s>>>(ma, mb, md, args);
    }
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

extern "C" int qf2_gemm_codes(const void* a, int64_t lda, const void* b_codes, int64_t ldb, int b_dtype, void* d,
                              int64_t ldd, int64_t M, int64_t N, int64_t K, int a_dtype, int d_dtype,
                              const float* row_scale, const float* col_scale, const void* bias, int bias_dtype,
                              int64_t gelu_col0, int glu, const void* residual, int64_t ldr, const void* gate,
                              int64_t gate_stride, int64_t rows_per_gate, void* workspace, int64_t workspace_bytes,
                              qf2_stream_t stream) {
  if (a_dtype != QF2_BF16 && a_dtype != QF2_F16) return QF2_ERR_DTYPE;
  if (b_dtype != QF2_I8 && b_dtype != QF2_E4M3) return QF2_ERR_DTYPE;
  return gemm_run(a, lda, b_codes, ldb, d, ldd, M, N, K, a_dtype, d_dtype, row_scale, col_scale, bias, bias_dtype,
                  gelu_col0, glu, residual, ldr, gate, gate_stride, rows_per_gate, nullptr, 0, 0, workspace,
                  workspace_bytes, stream, b_dtype);
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
