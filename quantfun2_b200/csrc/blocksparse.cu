// Top-k block-sparse attention for B200 (sm_100a).
//
// Replaces the reference's sparse attention path, topk_attn
// (src/kernels/__init__.py:146-195) with its mask cache POS_DICT
// (src/models/common/attn.py:20, :24-56), in block form:
//   1. blocktopk_pool_kernel    mean of Q and K over 128-token blocks (fp64 sums, fp32 means)
//   2. blocktopk_select_kernel  block scores pooled_q . pooled_k^T (fp64, fixed order,
//                               rounded to fp32) and the top `keep` key blocks per query
//                               block (lower index wins ties), written ascending (int32)
//   3. blocksparse_attn_kernel  exact softmax attention of each 128-row query block over
//                               its kept key blocks: TMA tiles (bf16/fp16, 128-byte
//                               swizzle) fetched by block index, tcgen05.mma kind::f16
//                               QK^T into TMEM (double-buffered S), P written to TMEM
//                               (two buffers) as PV's A operand, V read as an MN-major
//                               operand, fp32 O in TMEM; 8 softmax warps, lazy rescale.
#include "qf2_common.cuh"

#include <algorithm>
#include <cmath>

namespace qf2 {
namespace bsa {

constexpr int kBlk = 128;       // tokens per block (MMA M and N)
constexpr int kD = 128;         // head dim
constexpr int kMaxBlocks = 1024;

struct S3 { int64_t b, h, s; };

// ------------------------------------------------------------------ pool --
// grid (nb, Hq + Hkv, B), 256 threads: thread = (row slot 0..15, 8-channel chunk 0..15);
// each thread sums 8 rows x 8 channels from 16-byte loads issued together, the 16 row
// slots are combined through shared memory.
template <typename T>
__global__ void __launch_bounds__(256) blocktopk_pool_kernel(const T* __restrict__ q, S3 qs, const T* __restrict__ k,
                                                             S3 ks, int64_t S, int Hq, int Hkv, float* __restrict__ pq,
                                                             float* __restrict__ pk) {
  const int blk = blockIdx.x, job = blockIdx.y, b = blockIdx.z;
  const int slot = threadIdx.x >> 4, c8 = threadIdx.x & 15;
  const bool is_q = job < Hq;
  const int h = is_q ? job : job - Hq;
  const T* src = (is_q ? q : k) + (int64_t)b * (is_q ? qs.b : ks.b) + (int64_t)h * (is_q ? qs.h : ks.h) + c8 * 8;
  const int64_t ss = is_q ? qs.s : ks.s;
  const int64_t r0 = (int64_t)blk * kBlk;
  const int n = (int)min((int64_t)kBlk, S - r0);
  uint4 raw[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int r = slot + 16 * u;
    raw[u] = r < n ? *reinterpret_cast<const uint4*>(src + (r0 + r) * ss) : make_uint4(0, 0, 0, 0);
  }
  double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const T* e = reinterpret_cast<const T*>(&raw[u]);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] += (double)to_f32(e[j]);
  }
  __shared__ double red[16][kD];
#pragma unroll
  for (int j = 0; j < 8; ++j) red[slot][c8 * 8 + j] = acc[j];
  __syncthreads();
  if (threadIdx.x < kD) {
    // every partial sum is exact for 16-bit inputs, so the combination order is immaterial
    double sum = 0.0;
#pragma unroll
    for (int r = 0; r < 16; ++r) sum += red[r][threadIdx.x];
    const int nb = (int)((S + kBlk - 1) / kBlk);
    float* dst = is_q ? pq + (((int64_t)b * Hq + h) * nb + blk) * kD : pk + (((int64_t)b * Hkv + h) * nb + blk) * kD;
    dst[threadIdx.x] = (float)(sum / (double)n);
  }
}

// ---------------------------------------------------------------- select --
// grid (ceil(nb / kSelQ), Hq, B), 256 threads.  A CTA scores kSelQ query blocks against
// every key block: the pooled queries (as fp64) stay in shared memory, the pooled keys go
// through shared memory 64 blocks at a time (rows padded to 129 floats so the lanes of a
// warp, one key block each, hit distinct banks); each thread runs 4 independent dot
// products, each in the fixed order d = 0..127 with separately rounded fp64 products and
// sums, rounded once to fp32.  Ranks and ascending positions follow per query block.
constexpr int kSelQ = 16, kSelK = 64, kSelPad = kD + 1;

struct SelSmem {
  static constexpr int sq = 0;                                         // [kSelQ][kD] double
  static constexpr int skc = sq + kSelQ * kD * 8;                       // [kSelK][kSelPad] float
  static constexpr int sc = skc + kSelK * kSelPad * 4;                  // [kSelQ][nb] float
  static int bytes(int nb) { return sc + kSelQ * nb * 4 + kSelQ * nb; }  // + sel [kSelQ][nb]
};

__global__ void __launch_bounds__(256) blocktopk_select_kernel(const float* __restrict__ pq, const float* __restrict__ pk,
                                                               int nb, int Hq, int Hkv, int keep, int32_t* __restrict__ idx) {
  extern __shared__ __align__(16) uint8_t sm[];
  double* sq = reinterpret_cast<double*>(sm + SelSmem::sq);
  float* skc = reinterpret_cast<float*>(sm + SelSmem::skc);
  float* sc = reinterpret_cast<float*>(sm + SelSmem::sc);
  unsigned char* sel = sm + SelSmem::sc + kSelQ * nb * 4;
  const int q0 = blockIdx.x * kSelQ, h = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  const int hk = h / (Hq / Hkv);
  const int nq = min(kSelQ, nb - q0);
  const float* qsrc = pq + (((int64_t)b * Hq + h) * nb + q0) * kD;
  for (int i = tid; i < kSelQ * kD; i += 256) sq[i] = i < nq * kD ? (double)qsrc[i] : 0.0;
  const float* ksrc = pk + ((int64_t)b * Hkv + hk) * nb * kD;
  const int warp = tid >> 5, lane = tid & 31;
  for (int k0 = 0; k0 < nb; k0 += kSelK) {
    __syncthreads();  // sq written / the previous chunk's reads done
    const int nk = min(kSelK, nb - k0);
    for (int i = tid; i < kSelK * kD; i += 256) {
      const int r = i / kD, d = i % kD;
      skc[r * kSelPad + d] = r < nk ? ksrc[(int64_t)(k0 + r) * kD + d] : 0.f;
    }
    __syncthreads();
    // warp w: query blocks w, w + 8; lane: key blocks lane, lane + 32 of the chunk
    double acc[2][2] = {{0.0, 0.0}, {0.0, 0.0}};
    const double* qa = sq + warp * kD;
    const double* qb2 = sq + (warp + 8) * kD;
    const float* ka = skc + lane * kSelPad;
    const float* kb2 = skc + (lane + 32) * kSelPad;
#pragma unroll 4
    for (int d = 0; d < kD; ++d) {
      const double x0 = qa[d], x1 = qb2[d];
      const double y0 = (double)ka[d], y1 = (double)kb2[d];
      acc[0][0] = __dadd_rn(acc[0][0], __dmul_rn(x0, y0));
      acc[0][1] = __dadd_rn(acc[0][1], __dmul_rn(x0, y1));
      acc[1][0] = __dadd_rn(acc[1][0], __dmul_rn(x1, y0));
      acc[1][1] = __dadd_rn(acc[1][1], __dmul_rn(x1, y1));
    }
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int ql = warp + 8 * a, kl = lane + 32 * c;
        if (kl < nk) sc[ql * nb + k0 + kl] = (float)acc[a][c];
      }
  }
  __syncthreads();
  // rank of every (query block, key block): the lower index wins ties
  for (int i = tid; i < nq * nb; i += 256) {
    const int ql = i / nb, j = i % nb;
    const float* row = sc + ql * nb;
    const float v = row[j];
    int rank = 0;
    for (int t = 0; t < nb; ++t) {
      const float u = row[t];
      rank += (u > v) || (u == v && t < j);
    }
    sel[ql * nb + j] = rank < keep;
  }
  __syncthreads();
  for (int i = tid; i < nq * nb; i += 256) {
    const int ql = i / nb, j = i % nb;
    if (sel[ql * nb + j]) {
      int pos = 0;
      for (int t = 0; t < j; ++t) pos += sel[ql * nb + t];
      idx[(((int64_t)b * Hq + h) * nb + q0 + ql) * keep + pos] = j;
    }
  }
}

// ------------------------------------------------------------- attention --
// One CTA per 128-row query block: warp 0 TMA producer (Q once, K/V of each kept block
// into a 3-stage ring), warp 1 MMA issuer (QK^T into a double-buffered S in TMEM, PV into
// O in TMEM), warps 2-9 softmax.  A row's 128 scores are split over two softmax threads
// of the same TMEM lane quarter (warps w and w + 4), 64 columns each, so two warps per
// SM sub-partition feed the SFU; the halves exchange row maxima through shared memory.
// Lazy rescale: the running max moves (and O is rescaled) only when a block's max
// exceeds it by more than kTau (log2 units); P (bf16/fp16, at most 2^kTau) goes through
// two TMEM buffers so the next block's exps do not wait for the last PV.
constexpr int kThreads = 320;   // warp 0 producer, warp 1 MMA, warps 2-9 softmax
constexpr int kTile = 16384;    // 128 rows x 128 bytes (one 128-byte swizzle atom column)
constexpr int kOpBytes = 2 * kTile;  // 128 x 128 16-bit elements
// P lives in tensor memory as the PV product's A operand, which leaves shared memory for a
// 3-stage K/V ring (measured against P in two shared-memory buffers and 2 K/V stages:
// 0.774 -> 0.729 ms, S=16384, keep 16/128)
constexpr int kKvStages = 3;
// TMEM: S0 [0,128) S1 [128,256) O [256,384) P0 [384,448) P1 [448,512) (a 128 x 128 16-bit
// tile is 64 columns: two elements per column)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemP = 384;
constexpr float kTau = 8.0f;

struct Smem {
  static constexpr int q = 0;
  static constexpr int kv = q + kOpBytes;                   // kKvStages x (K, V)
  static constexpr int xch = kv + kKvStages * 2 * kOpBytes;  // row-max [j & 1][half][row] (row sums reuse it)
  static constexpr int bars = xch + 2 * 2 * 128 * 4;
  static constexpr int nbars = 1 + 2 * kKvStages + 2 + 2 + 2 + 2 + 4 + 4 + 1;
  static constexpr int misc = bars + nbars * 8;
  static constexpr int total = misc + 64;
  static constexpr int alloc = total;  // no alignment slack: the base is declared 1024-aligned
};
static_assert(Smem::alloc <= 227 * 1024, "shared memory");

struct AttnArgs {
  const int32_t* idx;
  void* out;
  S3 os;
  int64_t S;
  int Hq, Hkv, keep, nb;
  float scale_log2;  // sm_scale * log2(e)
  int f16;           // 1: fp16 operands, 0: bf16
  int* status;
};

QF2_DEV uint32_t pack2(float a, float b, bool f16) {
  if (f16) {
    __half2 t = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&t);
  }
  __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&t);
}

// F16: fp16 operands and output (else bf16), a compile-time choice so the P packing of
// the exponent loop carries no per-element select
template <bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    blocksparse_attn_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv, AttnArgs A) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  if (smem_u32(smem_raw) & 1023) {  // the 128-byte swizzle needs 1024-byte aligned tiles
    if (threadIdx.x == 0) atomicExch(A.status, kDevTimeoutProducer);
    return;
  }
  const int hk = h / (A.Hq / A.Hkv);
  const int keep = A.keep;
  const int32_t* idx = A.idx + (((int64_t)b * A.Hq + h) * A.nb + qb) * keep;

  uint8_t* base = smem_raw;
  uint8_t* sQ = base + Smem::q;
  uint8_t* sKV = base + Smem::kv;
  float* xmax = reinterpret_cast<float*>(base + Smem::xch);  // [j & 1][half][row]
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + Smem::bars);
  uint64_t* bar_q = bars;
  uint64_t* bar_kv_full = bars + 1;                   // [kKvStages]
  uint64_t* bar_kv_empty = bar_kv_full + kKvStages;   // [kKvStages]
  uint64_t* bar_s_full = bar_kv_empty + kKvStages;    // [2]
  uint64_t* bar_s_empty = bar_s_full + 2;             // [2]
  uint64_t* bar_p_full = bar_s_empty + 2;             // [P buffer]: P(i) written, i & 1 = buffer
  uint64_t* bar_o_done = bar_p_full + 2;              // [P buffer]: PV(i) completed
  // row-max / row-sum exchange between the two warps of a lane quarter (w and w + 4):
  // one barrier per quarter, so the quarters do not wait on one another
  uint64_t* bar_xm = bar_o_done + 2;  // [4]
  uint64_t* bar_xl = bar_xm + 4;      // [4]
  uint64_t* bar_drain = bar_xl + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + Smem::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + Smem::misc + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < kKvStages; ++s) {
      mbar_init(bar_kv_full + s, 1);
      mbar_init(bar_kv_empty + s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_s_full + s, 1);
      mbar_init(bar_s_empty + s, 8);
      mbar_init(bar_o_done + s, 1);
      mbar_init(bar_p_full + s, 8);
    }
    for (int q = 0; q < 4; ++q) {
      mbar_init(bar_xm + q, 2);
      mbar_init(bar_xl + q, 2);
    }
    mbar_init(bar_drain, 1);
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
  // o_done[i & 1] completes once per PV(i) of that P buffer: phase i >> 1
  auto o_wait = [&](int i) -> bool { return wwait(bar_o_done + (i & 1), (uint32_t)((i >> 1) & 1)); };

  if (warp == 0) {
    // ------------------------------------------------------- producer --
    if (keep > 0) {
      if (lane == 0) {
        prefetch_tmap(&tmq);
        prefetch_tmap(&tmk);
        prefetch_tmap(&tmv);
        mbar_arrive_expect_tx(bar_q, kOpBytes);
        tma_load_4d(sQ, &tmq, 0, qb * kBlk, h, b, bar_q);
        tma_load_4d(sQ + kTile, &tmq, 64, qb * kBlk, h, b, bar_q);
      }
      int issued = 0;
      for (int j = 0; j < keep; ++j) {
        const int s = j % kKvStages;
        if (!wwait(bar_kv_empty + s, ((j / kKvStages) & 1) ^ 1)) { if (lane == 0) fail(kDevTimeoutProducer); break; }
        if (lane == 0) {
          const int kb = idx[j];
          uint8_t* dK = sKV + s * 2 * kOpBytes;
          uint8_t* dV = dK + kOpBytes;
          mbar_arrive_expect_tx(bar_kv_full + s, 2 * kOpBytes);
          tma_load_4d(dK, &tmk, 0, kb * kBlk, hk, b, bar_kv_full + s);
          tma_load_4d(dK + kTile, &tmk, 64, kb * kBlk, hk, b, bar_kv_full + s);
          tma_load_4d(dV, &tmv, 0, kb * kBlk, hk, b, bar_kv_full + s);
          tma_load_4d(dV + kTile, &tmv, 64, kb * kBlk, hk, b, bar_kv_full + s);
        }
        __syncwarp();
        issued = j + 1;
      }
      if (*abort_flag && lane == 0) {
        mbar_wait(bar_q, 0);
        for (int j = issued > kKvStages ? issued - kKvStages : 0; j < issued; ++j)
          mbar_wait(bar_kv_full + (j % kKvStages), (j / kKvStages) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA --
    if (keep > 0) {
      const uint32_t ab = F16 ? 0u : 1u;
      const uint32_t idesc_qk = make_idesc(1, ab, ab, 0, 0, kBlk, kBlk);   // K-major x K-major -> f32
      const uint32_t idesc_pv = make_idesc(1, ab, ab, 0, 1, kBlk, kD);     // P K-major x V MN-major -> f32
      const uint32_t aQ = smem_u32(sQ);
      bool ok = wwait(bar_q, 0);
      auto issue_pv = [&](int i) -> bool {
        if (!wwait(bar_p_full + (i & 1), (uint32_t)((i >> 1) & 1))) return false;
        tc_fence_after();
        const uint32_t aV = smem_u32(sKV + (i % kKvStages) * 2 * kOpBytes + kOpBytes);
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            // A: P rows, 16 keys per step = 8 TMEM columns; B: V rows kk*16.. as MN-major
            // (head-dim halves 16 KB apart, 8-row groups 1 KB apart)
            const uint64_t db = sdesc_sw128_mnmajor(aV + kk * 16 * 128, kTile, 1024);
            mma_f16_tmem_a(tmem + 256, tmem + kTmemP + (i & 1) * 64 + kk * 8, db, idesc_pv,
                           (i > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(bar_o_done + (i & 1));
          tc_commit(bar_kv_empty + (i % kKvStages));
        }
        __syncwarp();
        return true;
      };
      for (int j = 0; ok && j < keep; ++j) {
        const int s = j & 1, ks = j % kKvStages;
        if (!wwait(bar_kv_full + ks, (j / kKvStages) & 1)) { ok = false; break; }
        if (!wwait(bar_s_empty + s, ((j >> 1) & 1) ^ 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t aK = smem_u32(sKV + ks * 2 * kOpBytes);
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * kTile + (kk & 3) * 32;
            mma_f16(tmem + s * kBlk, sdesc_sw128_kmajor(aQ + off), sdesc_sw128_kmajor(aK + off), idesc_qk,
                    kk > 0 ? 1u : 0u);
          }
          tc_commit(bar_s_full + s);
        }
        __syncwarp();
        if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_pv(keep - 1);
      if (lane == 0) {
        if (!ok) fail(kDevTimeoutMma);
        tc_commit(bar_drain);
        mbar_wait(bar_drain, 0);
      }
      __syncwarp();
    }
  } else {
    // -------------------------------------------------------- softmax --
    const int sw = warp - 2;
    const int half = sw >> 2;  // 64-column half of the row (warps 2-5: 0, 6-9: 1)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tO = tmem + lane_off + 256 + half * 64;
    constexpr bool f16 = F16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = keep > 0;
    for (int j = 0; ok && j < keep; ++j) {
      const int s = j & 1;
      if (!wwait(bar_s_full + s, (j >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[64];
      tmem_ld32(tmem + lane_off + s * kBlk + half * 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
      tmem_ld32(tmem + lane_off + s * kBlk + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_s_empty + s);

      const int64_t valid = A.S - (int64_t)idx[j] * kBlk - half * 64;  // keys of this half inside the sequence
      // raw scores; the scale (> 0) is applied to the max and folded into the exponent's fma
      float x[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) x[i] = __uint_as_float(sr[i]);
      if (valid < 64) {  // warp-uniform: the block runs past the sequence end
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i >= valid) x[i] = -INFINITY;
      }
      float mq[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float m = fmax3(x[c * 16], x[c * 16 + 1], x[c * 16 + 2]);
#pragma unroll
        for (int i = 3; i < 15; i += 2) m = fmax3(m, x[c * 16 + i], x[c * 16 + i + 1]);
        mq[c] = fmaxf(m, x[c * 16 + 15]);
      }
      const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * A.scale_log2;
      float* xm = xmax + (j & 1) * 256;
      xm[half * 128 + row] = mx;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_xm + quarter);
      if (!wwait(bar_xm + quarter, j & 1)) { ok = false; break; }
      const float m_tile = fmaxf(mx, xm[(half ^ 1) * 128 + row]);
      const float m_new = fmaxf(m_run, m_tile);
      // both warps of a row pair see the same 32 rows, so they agree on the decision
      const bool rescale = __any_sync(0xffffffffu, m_new > m_run + kTau);
      float alpha = 1.0f;
      if (rescale) {
        alpha = m_run == -INFINITY ? 0.f : fast_exp2(m_run - m_new);
        m_run = m_new;
        l_run *= alpha;
      }
      const float m_use = m_run == -INFINITY ? 0.f : m_run;  // a fully masked row contributes nothing
      // P(j) goes to buffer j & 1, last read by PV(j - 2)
      if (j >= 2 && !o_wait(j - 2)) { ok = false; break; }
      // this half's 64 keys of the row: 32 TMEM columns of packed pairs in P buffer j & 1
      // P = 2^(s * scale - m) as one fma per pair of keys (f32x2)
      const float2 scv = make_float2(A.scale_log2, A.scale_log2), nm = make_float2(-m_use, -m_use);
      float2 rs = make_float2(0.f, 0.f);
      uint32_t w[32];
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const float2 e = ffma2(make_float2(x[2 * q], x[2 * q + 1]), scv, nm);
        const float2 pp = make_float2(fast_exp2(e.x), fast_exp2(e.y));
        rs = fadd2(rs, pp);
        w[q] = pack2(pp.x, pp.y, f16);
      }
      tmem_st32(tmem + lane_off + kTmemP + (j & 1) * 64 + half * 32, w);
      l_run += rs.x + rs.y;
      if (rescale && j > 0) {
        // O holds sum_{i<j} P_i V_i against the old max; PV(j) is issued after p_full(j)
        if (!o_wait(j - 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
        tmem_wait_st();
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p_full + (j & 1));
    }
    if (keep > 0 && !ok) fail(kDevTimeoutSoftmax);
    // ------------------------------------------------------- epilogue --
    float l_tot = l_run;
    if (ok && keep > 0) {
      // row sums of the two halves through the row-max buffer that the last iteration did
      // not use (both halves are past its last read)
      float* xs = xmax + (keep & 1) * 256;
      xs[half * 128 + row] = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_xl + quarter);
      if (!wwait(bar_xl + quarter, 0) || !o_wait(keep - 1)) {
        fail(kDevTimeoutEpilogue);
        ok = false;
      } else {
        l_tot = l_run + xs[(half ^ 1) * 128 + row];
      }
      tc_fence_after();
    }
    const int64_t tok = (int64_t)qb * kBlk + row;
    const float inv_l = (ok && l_tot > 0.f) ? 1.0f / l_tot : 0.f;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t o[32];
      if (ok && keep > 0) {
        tmem_ld32(tO + c * 32, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (tok < A.S) {
        uint8_t* dst = reinterpret_cast<uint8_t*>(A.out) +
                       2 * ((int64_t)b * A.os.b + (int64_t)h * A.os.h + tok * A.os.s + half * 64 + c * 32);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = pack2(__uint_as_float(o[8 * v + 0]) * inv_l, __uint_as_float(o[8 * v + 1]) * inv_l, f16);
          w.y = pack2(__uint_as_float(o[8 * v + 2]) * inv_l, __uint_as_float(o[8 * v + 3]) * inv_l, f16);
          w.z = pack2(__uint_as_float(o[8 * v + 4]) * inv_l, __uint_as_float(o[8 * v + 5]) * inv_l, f16);
          w.w = pack2(__uint_as_float(o[8 * v + 6]) * inv_l, __uint_as_float(o[8 * v + 7]) * inv_l, f16);
          *reinterpret_cast<uint4*>(dst + v * 16) = w;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ host --
static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static int check_common(const void* q, const int64_t* qs, const void* k, const int64_t* ks, int64_t B, int64_t Hq,
                        int64_t Hkv, int64_t S, int64_t D, int dtype) {
  if (!q || !k || !qs || !ks) return QF2_ERR_ARG;
  if (dtype != QF2_BF16 && dtype != QF2_F16) return QF2_ERR_DTYPE;
  if (D != kD || B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || S <= 0) return QF2_ERR_SHAPE;
  if ((S + kBlk - 1) / kBlk > kMaxBlocks || B > 65535 || Hq + Hkv > 65535) return QF2_ERR_SHAPE;
  if (!al16(q) || !al16(k)) return QF2_ERR_ALIGN;
  for (int i = 0; i < 3; ++i)
    if ((qs[i] % 8) || (ks[i] % 8)) return QF2_ERR_ALIGN;
  return QF2_OK;
}

static bool make_map(CUtensorMap* m, const void* base, const int64_t* st, int64_t B, int64_t H, int64_t S, int dtype) {
  const uint64_t dims[4] = {(uint64_t)kD, (uint64_t)S, (uint64_t)H, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)st[2] * 2, (uint64_t)st[1] * 2, (uint64_t)st[0] * 2};
  const uint32_t box[4] = {64, (uint32_t)kBlk, 1, 1};
  return qf2_make_tmap_4d(m, dtype == QF2_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                          base, dims, strides, box);
}

}  // namespace bsa
}  // namespace qf2

using namespace qf2::bsa;

extern "C" int64_t qf2_blocktopk_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t D) {
  if (D != kD || B <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0) return (int64_t)QF2_ERR_SHAPE;
  const int64_t nb = (S + kBlk - 1) / kBlk;
  return 256 + (B * Hq + B * Hkv) * nb * kD * 4;
}

extern "C" int qf2_blocktopk_select(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                    int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t D, int64_t keep, int dtype,
                                    int32_t* idx_out, void* workspace, int64_t workspace_bytes, qf2_stream_t stream) {
  int st = check_common(q, q_strides, k, k_strides, B, Hq, Hkv, S, D, dtype);
  if (st != QF2_OK) return st;
  const int64_t nb = (S + kBlk - 1) / kBlk;
  if (!idx_out || keep <= 0 || keep > nb) return keep <= 0 || keep > nb ? QF2_ERR_SHAPE : QF2_ERR_ARG;
  if (!workspace || workspace_bytes < qf2_blocktopk_workspace_bytes(B, Hq, Hkv, S, D) || !al16(workspace))
    return QF2_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float* pq = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + 256);
  float* pk = pq + B * Hq * nb * kD;
  const S3 qs{q_strides[0], q_strides[1], q_strides[2]}, ks{k_strides[0], k_strides[1], k_strides[2]};
  const dim3 gp((unsigned)nb, (unsigned)(Hq + Hkv), (unsigned)B);
  if (dtype == QF2_BF16)
    blocktopk_pool_kernel<__nv_bfloat16><<<gp, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(q), qs,
                                                             reinterpret_cast<const __nv_bfloat16*>(k), ks, S,
                                                             (int)Hq, (int)Hkv, pq, pk);
  else
    blocktopk_pool_kernel<__half><<<gp, 256, 0, s>>>(reinterpret_cast<const __half*>(q), qs,
                                                      reinterpret_cast<const __half*>(k), ks, S, (int)Hq, (int)Hkv,
                                                      pq, pk);
  QF2_LAUNCH_CHECK();
  const int sel_bytes = SelSmem::bytes((int)nb);
  static std::atomic<uint64_t> sel_attr{0};
  QF2_CUDA_CHECK(qf2_set_smem_once(blocktopk_select_kernel, SelSmem::bytes(kMaxBlocks), &sel_attr));
  blocktopk_select_kernel<<<dim3((unsigned)((nb + kSelQ - 1) / kSelQ), (unsigned)Hq, (unsigned)B), 256, sel_bytes, s>>>(
      pq, pk, (int)nb, (int)Hq, (int)Hkv, (int)keep, idx_out);
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}

extern "C" int qf2_blocksparse_attn(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                    const void* v, const int64_t* v_strides, void* out, const int64_t* out_strides,
                                    int64_t B, int64_t Hq, int64_t Hkv, int64_t S, int64_t D, const int32_t* idx,
                                    int64_t keep, float sm_scale, int dtype, void* workspace,
                                    int64_t workspace_bytes, qf2_stream_t stream) {
  int st = check_common(q, q_strides, k, k_strides, B, Hq, Hkv, S, D, dtype);
  if (st != QF2_OK) return st;
  if (!v || !v_strides || !out || !out_strides || !idx) return QF2_ERR_ARG;
  if (!al16(v) || !al16(out)) return QF2_ERR_ALIGN;
  for (int i = 0; i < 3; ++i)
    if ((v_strides[i] % 8) || (out_strides[i] % 8)) return QF2_ERR_ALIGN;
  const int64_t nb = (S + kBlk - 1) / kBlk;
  if (keep <= 0 || keep > nb) return QF2_ERR_SHAPE;
  if (!workspace || workspace_bytes < 256 || !al16(workspace)) return QF2_ERR_WORKSPACE;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, q, q_strides, B, Hq, S, dtype) || !make_map(&mk, k, k_strides, B, Hkv, S, dtype) ||
      !make_map(&mv, v, v_strides, B, Hkv, S, dtype))
    return QF2_ERR_ALIGN;
  AttnArgs a;
  a.idx = idx;
  a.out = out;
  a.os = S3{out_strides[0], out_strides[1], out_strides[2]};
  a.S = S;
  a.Hq = (int)Hq; a.Hkv = (int)Hkv; a.keep = (int)keep; a.nb = (int)nb;
  a.scale_log2 = (float)((double)sm_scale * 1.4426950408889634);
  a.f16 = dtype == QF2_F16;
  a.status = reinterpret_cast<int*>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  QF2_CUDA_CHECK(cudaMemsetAsync(workspace, 0, sizeof(int), s));
  static std::atomic<uint64_t> attr_done[2];
  auto kern = a.f16 ? blocksparse_attn_kernel<true> : blocksparse_attn_kernel<false>;
  QF2_CUDA_CHECK(qf2_set_smem_once(kern, Smem::alloc, &attr_done[a.f16 ? 1 : 0]));
  kern<<<dim3((unsigned)nb, (unsigned)Hq, (unsigned)B), kThreads, Smem::alloc, s>>>(mq, mk, mv, a);
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}
