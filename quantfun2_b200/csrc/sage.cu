// Sage-style quantized attention for B200 (sm_100a).
//
// Replaces the third-party sageattention calls of the reference:
//   sageattn(q, k, v)                      src/models/flux/attn.py:39-41   (HND)
//   sageattn_varlen(q, k, v, cu_seqlens..) src/models/common/attn.py:109-120
//
// Pipeline (2 launches and a 4-byte memset, all on the caller's stream):
//   1. sage_prep_kernel       persistent, TMA-fed, in thread-block clusters: one cluster
//                             per (seq, kv head) computes the K token mean and the V
//                             per-channel scale (partials exchanged through distributed
//                             shared memory) and then writes smoothed-K INT8 and V e4m3
//                             codes from a second, L2-resident pass over its tiles;
//                             the remaining CTAs write Q INT8 codes.  Codes land in the
//                             128-byte-swizzled tile layout tcgen05 reads directly from
//                             shared memory (one 16 KB bulk copy per tile; Q/K K-major,
//                             V token-major)
//   2. sage_attn_kernel       warp-specialised tcgen05 attention: 1 producer warp
//                             (bulk copies), 1 MMA warp (kind::i8 QK^T and kind::f8f6f4
//                             PV into TMEM), 8 softmax warps (TMEM -> registers, online
//                             base-2 softmax, P -> e4m3 into swizzled smem, O rescale,
//                             epilogue).
#include "qf2_common.cuh"

#include <algorithm>
#include <cmath>

namespace qf2 {
namespace sage {

constexpr int kTile = 128;          // tokens per tile (MMA M and N)
constexpr int kHeadDim = 128;       // channels of a code tile row (D <= 128 is zero-padded there)
// head dims the entry points take: D = 64, 96 or 128 channels are read from the inputs,
// codes of the missing channels are 0 (the TMA box is 128 channels wide over a D-wide
// tensor, so the loads fill them with zeros), QK^T runs D / 32 MMA K-steps and the
// epilogue stores D columns
QF2_DEV_HOST_INLINE bool head_dim_ok(int64_t D) { return D == 64 || D == 96 || D == 128; }
constexpr int kTileBytes = 16384;   // 128 rows x 128 bytes of 8-bit codes
constexpr int kQuantBlock = 64;     // tokens per INT8 scale block
static_assert(kTile == 2 * kQuantBlock, "a Q/K tile holds two INT8 scale blocks");
// P tiles per Q tile in shared memory: 2 lets the softmax write P(j) while PV(j-1) still
// reads P(j-1) (the K/V ring then has 3 stages to stay within shared memory; measured
// 0.4370 -> 0.4332 ms at B=2, H=24, S=4608)
#ifndef QF2_SAGE_PBUF
#define QF2_SAGE_PBUF 2
#endif
constexpr int kPBuf = QF2_SAGE_PBUF;
static_assert(kPBuf == 1 || kPBuf == 2, "one or two P tiles per Q tile");
constexpr int kStages = kPBuf == 2 ? 3 : 4;  // K/V smem ring depth
constexpr int kMaxKvTiles = 512;    // k-scale smem capacity (65536 tokens)
constexpr int kMaxSplits = 8;       // KV splits of the attention
constexpr float kLog2_448 = 8.807354922057604f;

struct SeqGeom {
  const int32_t* cu_q;  // nullptr for dense
  const int32_t* cu_k;
  int64_t Sq, Skv;      // dense lengths
  int64_t tiles_q_dense, tiles_k_dense;
};

struct SeqInfo {
  int64_t tok0;   // first token (varlen) or 0 (dense)
  int64_t len;
  int64_t tile0;  // first tile slot of this sequence in the per-head tile arrays
};

QF2_DEV SeqInfo seq_q(const SeqGeom& g, int b) {
  SeqInfo s;
  if (g.cu_q) {
    const int64_t a = g.cu_q[b], e = g.cu_q[b + 1];
    s.tok0 = a; s.len = e - a; s.tile0 = a / kTile + b;
  } else {
    s.tok0 = 0; s.len = g.Sq; s.tile0 = (int64_t)b * g.tiles_q_dense;
  }
  return s;
}

QF2_DEV SeqInfo seq_k(const SeqGeom& g, int b) {
  SeqInfo s;
  if (g.cu_k) {
    const int64_t a = g.cu_k[b], e = g.cu_k[b + 1];
    s.tok0 = a; s.len = e - a; s.tile0 = a / kTile + b;
  } else {
    s.tok0 = 0; s.len = g.Skv; s.tile0 = (int64_t)b * g.tiles_k_dense;
  }
  return s;
}

struct Strides3 { int64_t b, h, s; };

struct Workspace {
  int* status;
  int8_t* qc; float* qs;
  int8_t* kc; float* ks;
  uint8_t* vc; float* vs;
  float* kmean; float* vinv;
  __nv_bfloat16* part_o; float2* part_ml;  // split-KV partials (see sage_attn_kernel)
  int64_t prows;                           // rows of one split's partials: Hq * tq * 128
  int nsplit;                              // KV splits of the attention (1: none)
  int64_t tq, tk;   // tile slots per head
  int64_t nch;      // stats chunks per sequence
};

// --------------------------------------------------------- packed fp32 math --
// Two-lane fp32 arithmetic (sm_100 f32x2 instructions); each lane rounds like the
// scalar .rn instruction.
QF2_DEV float2 fmul2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}



// The two 16-bit floats of a 32-bit word as fp32 (exact).
template <typename T>
QF2_DEV float2 unpack2(uint32_t w);
template <>
QF2_DEV float2 unpack2<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
QF2_DEV float2 unpack2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// max(|a|, |b|) of the four 16-bit floats of two words, as fp32 (NaN lanes ignored like fmaxf)
template <typename T>
QF2_DEV uint32_t absmax2(uint32_t acc, uint32_t w);
template <>
QF2_DEV uint32_t absmax2<__nv_bfloat16>(uint32_t acc, uint32_t w) {
  __nv_bfloat162 r = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&acc),
                             __habs2(*reinterpret_cast<const __nv_bfloat162*>(&w)));
  return *reinterpret_cast<uint32_t*>(&r);
}
template <>
QF2_DEV uint32_t absmax2<__half>(uint32_t acc, uint32_t w) {
  __half2 r = __hmax2(*reinterpret_cast<const __half2*>(&acc), __habs2(*reinterpret_cast<const __half2*>(&w)));
  return *reinterpret_cast<uint32_t*>(&r);
}

// INT8 code of x in a block with dequant scale s = RN(amax / 127) and r = RN(1 / s), by the
// published SageAttention Triton rule (quant_per_block_int8_kernel: x / scale, += 0.5 *
// sign, truncate): t = RN(x / s); code = trunc(RN(t + 0.5 sign(t))), +0.5 for t >= 0.
// The quotient is RN(x r) corrected once (Markstein 1990: with r the correctly rounded
// reciprocal and q0 = RN(x r) within an ulp of x / s, the fma remainder x - s q0 is exact
// and RN(q0 + rem r) is the correctly rounded quotient).  RN(t + 0.5 sign t) = sign(t)
// RN(|t| + 0.5), and its truncation is sign(t) floor(RN(|t| + 0.5)); the floor of a value
// below 2^22 is the low bits of its round-toward-zero sum with 2^23.  Returns the code as
// a two's-complement int32 (low byte = int8 code); |code| <= 127 since |t| <= 127 (1 + 2^-23).
// The intrinsics are never contracted with one another.
QF2_DEV uint32_t sage_code(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  const float rem = __fmaf_rn(-q0, s, x);
  const float t = __fmaf_rn(rem, r, q0);
  const float v = __fadd_rn(fabsf(t), 0.5f);
  const uint32_t n = __float_as_uint(__fadd_rz(v, 8388608.0f)) - 0x4B000000u;
  const uint32_t neg = (uint32_t)((int32_t)__float_as_uint(t) >> 31);
  return (n ^ neg) - neg;
}

// sage_code on two lanes with the sm_100 f32x2 instructions (each lane rounds like the
// scalar .rn / .rz instruction; the mul feeds only fma multiplicands, so nothing contracts).
// ns = -s.  Returns the two codes in the low bytes of c.x / c.y.
QF2_DEV uint2 sage_code2(float2 x, float2 ns, float2 r) {
  float2 f;
  uint32_t tx, ty;
  asm("{\n\t.reg .b64 rx, rr, rs, rq, rm, rt, rv, rh, rz;\n\t"
      ".reg .b32 ax, ay;\n\t"
      "mov.b64 rx, {%4, %5};\n\tmov.b64 rr, {%6, %7};\n\tmov.b64 rs, {%8, %9};\n\t"
      "mul.rn.f32x2 rq, rx, rr;\n\t"          // q0 = x r
      "fma.rn.f32x2 rm, rq, rs, rx;\n\t"      // rem = x - s q0 (exact)
      "fma.rn.f32x2 rt, rm, rr, rq;\n\t"      // t = RN(x / s)
      "mov.b64 {%2, %3}, rt;\n\t"
      "and.b32 ax, %2, 0x7fffffff;\n\tand.b32 ay, %3, 0x7fffffff;\n\t"
      "mov.b64 rv, {ax, ay};\n\t"
      "mov.b64 rh, {0f3F000000, 0f3F000000};\n\t"
      "add.rn.f32x2 rv, rv, rh;\n\t"         // |t| + 0.5
      "mov.b64 rz, {0f4B000000, 0f4B000000};\n\t"
      "add.rz.f32x2 rv, rv, rz;\n\t"         // 2^23 + floor(|t| + 0.5)
      "mov.b64 {%0, %1}, rv;\n\t}"
      : "=f"(f.x), "=f"(f.y), "=r"(tx), "=r"(ty)
      : "f"(x.x), "f"(x.y), "f"(r.x), "f"(r.y), "f"(ns.x), "f"(ns.y));
  const uint32_t nx = __float_as_uint(f.x) & 0xffu, ny = __float_as_uint(f.y) & 0xffu;
  const uint32_t sx = (uint32_t)((int32_t)tx >> 31), sy = (uint32_t)((int32_t)ty >> 31);
  return make_uint2((nx ^ sx) - sx, (ny ^ sy) - sy);
}

// ------------------------------------------------------------ preparation --
// One persistent, TMA-fed, warp-specialised kernel launched in clusters of C CTAs
// (C <= 8).  Warp 8 produces: it picks the tiles, writes each tile's descriptor next to
// its 32 KB ring slot (128 tokens x 128 channels of 16-bit values, 3-stage ring) and
// starts the TMA load; warps 0-7 consume the slots in order.  thread = (row slot rg
// 0..15, 8-channel chunk c8 0..15); it reads rows rg + 16 i (i < 4: first 64-token block).
//   K/V role (the first clusters): a cluster walks (seq, kv head) pairs one after the
//     other; CTA r owns a contiguous range of the sequence's tiles.  Phase 1 streams its
//     K and V tiles: fp64 channel sums of K and channel amax of V.  An exchange marker in
//     the ring then makes the CTAs swap these partials through distributed shared memory
//     (cluster barrier); each derives the K token mean and the V channel scale (fp64 sums
//     of 16-bit floats are exact, so the order of the partials does not matter), and
//     phase 2 streams the same tiles again -- from L2, where phase 1 left them with
//     evict-last priority and where only a few heads are in flight -- to write the codes:
//     smoothed K -> INT8 per 64-token block, V -> e4m3 per channel.
//   Q tiles -> INT8 per 64-token block (x = q * sm_scale * log2 e): every CTA takes them
//     from a global counter once it has no K/V work left, so the grid finishes together.
// Codes go straight into the 128-byte-swizzled tile layout tcgen05 reads from shared
// memory (Q and K K-major, V token-major = MN-major B operand of the PV product).
constexpr int kPrepThreads = 288;      // warps 0-7 consumers, warp 8 TMA producer
constexpr int kPrepStages = 3;
constexpr int kPrepTile = 32768;       // 128 tokens x 128 channels x 16 bit
constexpr int kPrepCtasPerSm = 2;
constexpr int kMaxCluster = 8;

struct PrepSmem {
  static constexpr int ring = 0;
  static constexpr int red = ring + kPrepStages * kPrepTile;  // 8 warps x 128 doubles
  static constexpr int part_sum = red + 8 * kHeadDim * 8;      // [2 heads] this CTA's K channel sums
  static constexpr int part_amax = part_sum + 2 * kHeadDim * 8;  // [2 heads] this CTA's V channel amax
  static constexpr int stats = part_amax + 2 * kHeadDim * 4;   // K mean, V 448 / amax
  static constexpr int blk = stats + 2 * kHeadDim * 4;         // per-tile block amax [2][16]
  static constexpr int items = blk + 2 * 16 * 4;               // slot descriptors (int4)
  static constexpr int bars = items + kPrepStages * 16;
  static constexpr int nbars = 2 * kPrepStages + 2;            // full, empty, block-amax [2]
  static constexpr int total = bars + nbars * 8;
};
static_assert(kPrepCtasPerSm * (PrepSmem::total + 1024) <= 228 * 1024, "two CTAs per SM");

// Byte offset of (row, 16-byte chunk) in a 128x128-byte tile stored in the
// 128B-swizzle layout: row r at r*128, chunk c at slot c ^ (r & 7).
QF2_DEV int swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

struct PrepArgs {
  SeqGeom g;
  Workspace ws;
  int batch, Hq, Hkv;
  int64_t mtq;           // tiles of the longest q sequence
  float qmul;            // sm_scale * log2(e)
  int varlen;
  int csize;             // CTAs per cluster
  uint32_t n_kv_ctas;    // CTAs with the K/V role (whole clusters)
  uint32_t* q_next;      // Q tile counter (zeroed with the status word)
};

// Slot descriptor: x = kind (0 Q, 1 K, 2 V, 3 statistics exchange; -1 end of work) |
// phase << 4, y = b, z = h, w = tile.  Kinds -1 and 3 carry no tile.
QF2_DEV int4 make_desc(int tensor, int phase, int b, int h, int64_t tile) {
  return make_int4(tensor < 0 ? -1 : (tensor | (phase << 4)), b, h, (int)tile);
}

QF2_DEV float2 ffma2_rn(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}

QF2_DEV void bar_consumers() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// K/V range of CTA `rank` for kv head `hd` (= b * Hkv + h): tiles [t0, t0 + nt)
struct KvRange {
  int b, h;
  int64_t t0, nt;
};

QF2_DEV KvRange kv_range(const PrepArgs& A, uint32_t hd, uint32_t rank) {
  KvRange r;
  r.b = (int)(hd / (uint32_t)A.Hkv);
  r.h = (int)(hd - (uint32_t)r.b * (uint32_t)A.Hkv);
  const int64_t ntiles = (seq_k(A.g, r.b).len + kTile - 1) / kTile;
  const int64_t per = (ntiles + A.csize - 1) / A.csize;
  r.t0 = min(ntiles, (int64_t)rank * per);
  r.nt = min(ntiles, r.t0 + per) - r.t0;
  return r;
}

template <typename T>
__global__ void __launch_bounds__(kPrepThreads, kPrepCtasPerSm)
    sage_prep_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, PrepArgs A) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem + PrepSmem::ring;
  double* red = reinterpret_cast<double*>(smem + PrepSmem::red);
  double* part_sum = reinterpret_cast<double*>(smem + PrepSmem::part_sum);
  float* part_amax = reinterpret_cast<float*>(smem + PrepSmem::part_amax);
  float* s_kmean = reinterpret_cast<float*>(smem + PrepSmem::stats);
  float* s_vinv = s_kmean + kHeadDim;
  float* s_blk = reinterpret_cast<float*>(smem + PrepSmem::blk);
  int4* s_item = reinterpret_cast<int4*>(smem + PrepSmem::items);  // ordered by the full/empty mbarriers
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + PrepSmem::bars);
  uint64_t* empty = full + kPrepStages;
  uint64_t* bar_blk = empty + kPrepStages;  // [2]: the 8 warps' block amax of a Q/K tile
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const Workspace& ws = A.ws;
  if (tid == 0) {
    for (int s = 0; s < kPrepStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 8);
    }
    mbar_init(bar_blk, 8);
    mbar_init(bar_blk + 1, 8);
    fence_mbar_init();
  }
  __syncthreads();

  // K/V role: this cluster walks kv heads cl, cl + ncl, ... (b * Hkv + h order)
  const bool kv = blockIdx.x < A.n_kv_ctas;
  const uint32_t heads = (uint32_t)A.batch * (uint32_t)A.Hkv;
  const uint32_t ncl = A.n_kv_ctas / (uint32_t)A.csize;
  const uint32_t cl = kv ? blockIdx.x / (uint32_t)A.csize : 0u;
  const uint32_t rank = kv ? blockIdx.x - cl * (uint32_t)A.csize : 0u;
  const uint32_t my_heads = kv && cl < heads ? (heads - cl + ncl - 1) / ncl : 0u;

  if (warp == 8) {
    // ------------------------------------------------------------ producer --
    uint32_t n = 0;  // slots filled
    bool dead = false;
    const uint64_t keep = l2_policy_evict_last(), drop = l2_policy_evict_first();
    // lane 0: wait for a free slot, publish the descriptor, start the load (none for the
    // markers; their slot completes on the arrive alone)
    auto push = [&](int kind, int phase, int b, int h, int64_t tile) {
      if (dead) return;
      const int s = (int)(n % kPrepStages);
      if (!mbar_wait(empty + s, ((n / kPrepStages) & 1u) ^ 1u)) {
        atomicExch(ws.status, kDevTimeoutProducer);
        dead = true;
        return;
      }
      s_item[s] = make_desc(kind, phase, b, h, tile);
      ++n;
      if (kind < 0 || kind == 3) {
        mbar_arrive(full + s);
        return;
      }
      mbar_arrive_expect_tx(full + s, kPrepTile);
      const SeqInfo si = kind == 0 ? seq_q(A.g, b) : seq_k(A.g, b);
      const CUtensorMap* tm = kind == 0 ? &tm_q : kind == 1 ? &tm_k : &tm_v;
      // K/V tiles stay in L2 between their two reads; Q tiles and second reads go first
      tma_load_4d_hint(ring + s * kPrepTile, tm, 0, (int32_t)(si.tok0 + tile * kTile), h, A.varlen ? 0 : b, full + s,
                       phase == 1 ? keep : drop);
    };
    if (lane == 0) {
      if (my_heads > 0) {
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
      }
      if (A.mtq > 0) prefetch_tmap(&tm_q);
    }
    for (uint32_t i = 0; i < my_heads; ++i) {
      const KvRange r = kv_range(A, cl + i * ncl, rank);
      if (lane == 0) {
        for (int64_t t = r.t0; t < r.t0 + r.nt; ++t) {
          push(1, 1, r.b, r.h, t);
          push(2, 1, r.b, r.h, t);
        }
        push(3, 1, r.b, r.h, 0);
      }
      __syncwarp();
      cluster_arrive();  // this head's partials exchange (this warp publishes nothing)
      if (lane == 0) {
        for (int64_t t = r.t0; t < r.t0 + r.nt; ++t) {
          push(1, 2, r.b, r.h, t);
          push(2, 2, r.b, r.h, t);
        }
      }
      __syncwarp();
      cluster_wait();
    }
    if (lane == 0) {
      const uint32_t mtq = (uint32_t)A.mtq;
      const uint32_t nq = (uint32_t)A.batch * (uint32_t)A.Hq * mtq;
      while (!dead) {
        const uint32_t gq = atomicAdd(A.q_next, 1u);
        if (gq >= nq) break;
        const uint32_t bh = gq / mtq;
        const int64_t tile = (int64_t)(gq - bh * mtq);
        const int b = (int)(bh / (uint32_t)A.Hq);
        const int h = (int)(bh - (uint32_t)b * (uint32_t)A.Hq);
        if (tile * kTile < seq_q(A.g, b).len) push(0, 2, b, h, tile);
      }
      push(-1, 0, 0, 0, 0);
      // the last loads have landed before this CTA's shared memory goes away (their
      // phases completed already when the consumers took them; bounded if they gave up)
      for (uint32_t i = n > kPrepStages ? n - kPrepStages : 0; i < n; ++i)
        mbar_wait(full + (int)(i % kPrepStages), (i / kPrepStages) & 1u);
    }
    __syncwarp();
    if (kv) {
      cluster_arrive();  // no CTA leaves while another may still read its partials
      cluster_wait();
    }
    return;
  }

  // -------------------------------------------------------------- consumers --
  // Bounded waits only inside the tile loop: a warp that gives up records the error and
  // leaves the loop; the others then give up at their next wait.  Every warp takes each
  // head's exchange exactly once (after the loop for the heads it did not reach).
  const int rg = tid >> 4, c8 = tid & 15;
  bool dead = false;
  uint32_t n = 0;          // slots consumed
  uint32_t nbar = 0;       // Q/K tiles (block-amax exchanges)
  uint32_t heads_done = 0;
  int slot = 0;
  auto next = [&](int4& d) -> bool {
    if (dead) return false;
    slot = (int)(n % kPrepStages);
    const bool ok = mbar_wait(full + slot, (n / kPrepStages) & 1u);
    ++n;
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) atomicExch(ws.status, kDevTimeoutSoftmax);
      dead = true;
      return false;
    }
    d = s_item[slot];
    return true;
  };
  auto release = [&]() {
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + slot);
  };
  // the tile of the current slot into registers, then the slot back to the producer
  auto read_tile = [&](uint4 (&raw)[8]) {
    const uint8_t* src = ring + slot * kPrepTile + rg * 256 + c8 * 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) raw[i] = *reinterpret_cast<const uint4*>(src + i * 16 * 256);
    release();
  };
  // CTA partials of head i of this cluster -> cluster exchange -> its K mean and V scale
  // in shared memory (rank 0 also writes them to the workspace)
  auto exchange = [&](const double (&ksum_in)[8], const uint32_t (&vmax_in)[4]) {
    double ksum[8];
    uint32_t vmax[4];
#pragma unroll
    for (int j = 0; j < 8; ++j) ksum[j] = ksum_in[j] + __shfl_xor_sync(0xffffffffu, ksum_in[j], 16);
#pragma unroll
    for (int j = 0; j < 4; ++j) vmax[j] = absmax2<T>(vmax_in[j], __shfl_xor_sync(0xffffffffu, vmax_in[j], 16));
    const uint32_t par = heads_done & 1u;
    double* psum = part_sum + par * kHeadDim;
    float* pamax = part_amax + par * kHeadDim;
    if (lane < 16) {
#pragma unroll
      for (int j = 0; j < 8; ++j) red[warp * kHeadDim + c8 * 8 + j] = ksum[j];
    }
    bar_consumers();
    if (tid < kHeadDim) {
      double acc = 0.0;
#pragma unroll
      for (int q = 0; q < 8; ++q) acc += red[q * kHeadDim + tid];
      psum[tid] = acc;
    }
    bar_consumers();
    float* redf = reinterpret_cast<float*>(red);
    if (lane < 16) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack2<T>(vmax[j]);
        redf[warp * kHeadDim + c8 * 8 + 2 * j] = f.x;
        redf[warp * kHeadDim + c8 * 8 + 2 * j + 1] = f.y;
      }
    }
    bar_consumers();
    if (tid < kHeadDim) {
      float am = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) am = fmaxf(am, redf[q * kHeadDim + tid]);
      pamax[tid] = am;
    }
    // partials of head i live in buffer i & 1: a CTA rewrites it for head i + 2 only
    // after the exchange of head i + 1, which every CTA joins after reading head i's
    cluster_arrive();
    cluster_wait();
    if (tid < kHeadDim) {
      double acc = 0.0;
      float am = 0.f;
      const uint32_t a_sum = smem_u32(psum + tid), a_amax = smem_u32(pamax + tid);
      for (int r = 0; r < A.csize; ++r) {
        acc += ld_dsmem_f64(mapa_shared(a_sum, (uint32_t)r));
        am = fmaxf(am, ld_dsmem_f32(mapa_shared(a_amax, (uint32_t)r)));
      }
      const uint32_t hd = cl + heads_done * ncl;
      const int b = (int)(hd / (uint32_t)A.Hkv);
      const int h = (int)(hd - (uint32_t)b * (uint32_t)A.Hkv);
      const int64_t len = seq_k(A.g, b).len;
      const float km = len > 0 ? (float)(acc / (double)len) : 0.f;
      const float vinv = am > 0.f ? __fdiv_rn(448.0f, am) : 1.0f;
      s_kmean[tid] = km;
      s_vinv[tid] = vinv;
      if (rank == 0) {
        const int64_t o = ((int64_t)b * A.Hkv + h) * kHeadDim + tid;
        ws.kmean[o] = km;
        ws.vs[o] = am > 0.f ? __fdiv_rn(am, 448.0f) : 1.0f;
        ws.vinv[o] = vinv;
      }
    }
    bar_consumers();  // K mean and V scale in shared memory from here on (read per tile)
    ++heads_done;
  };
  // this thread's 8 channels of the K mean (negated) / V 448 / amax
  auto load_pairs = [&](const float* src, float sign, float2 (&out)[4]) {
    const float4 a = *reinterpret_cast<const float4*>(src + c8 * 8);
    const float4 c = *reinterpret_cast<const float4*>(src + c8 * 8 + 4);
    out[0] = make_float2(sign * a.x, sign * a.y); out[1] = make_float2(sign * a.z, sign * a.w);
    out[2] = make_float2(sign * c.x, sign * c.y); out[3] = make_float2(sign * c.z, sign * c.w);
  };

  const float2 mul = make_float2(A.qmul, A.qmul);
  int4 d = make_int4(-1, 0, 0, 0);
  bool have = next(d);
  while (have && d.x >= 0) {
    if ((d.x >> 4) == 1) {
      // ---- phase 1 of a head: channel statistics of this CTA's K and V tiles ----
      double ksum[8];
      uint32_t vmax[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int j = 0; j < 8; ++j) ksum[j] = 0.0;
      while ((d.x & 15) != 3) {
        const int kind = d.x & 15;
        const int64_t tile = d.w;
        uint4 raw[8];
        read_tile(raw);
        const int valid = (int)min((int64_t)kTile, seq_k(A.g, d.y).len - tile * kTile);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          if (rg + 16 * r < valid) {
            const uint32_t* wd = reinterpret_cast<const uint32_t*>(&raw[r]);
            if (kind == 1) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 f = unpack2<T>(wd[j]);
                ksum[2 * j] += (double)f.x;
                ksum[2 * j + 1] += (double)f.y;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 4; ++j) vmax[j] = absmax2<T>(vmax[j], wd[j]);
            }
          }
        }
        if (!next(d)) break;
      }
      if (dead) break;
      release();  // the exchange marker's slot
      exchange(ksum, vmax);
      have = next(d);
      continue;
    }
    // ---- phase 2: codes ----
    const int kind = d.x & 15, b = d.y, h = d.z;
    const int64_t tile = d.w;
    uint4 raw[8];
    read_tile(raw);
    const SeqInfo si = kind == 0 ? seq_q(A.g, b) : seq_k(A.g, b);
    const int valid = (int)min((int64_t)kTile, si.len - tile * kTile);
    if (kind == 2) {
      // V: e4m3(v * (448 / amax_channel)), token-major
      float2 vinv2[4];
      load_pairs(s_vinv, 1.0f, vinv2);
      uint8_t* dst = ws.vc + ((int64_t)h * ws.tk + si.tile0 + tile) * kTileBytes;
#pragma unroll
      for (int r8 = 0; r8 < 8; ++r8) {
        const int r = rg + 16 * r8;
        const uint32_t* wd = reinterpret_cast<const uint32_t*>(&raw[r8]);
        uint32_t e[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 x = fmul2(unpack2<T>(wd[j]), vinv2[j]);
          e[j] = f32x2_to_e4m3x2(x.x, x.y);
        }
        const bool in = r < valid;  // rows past the sequence end get code 0
        *reinterpret_cast<uint2*>(dst + swz(r, c8 >> 1) + (c8 & 1) * 8) =
            make_uint2(in ? (e[0] | (e[1] << 16)) : 0u, in ? (e[2] | (e[3] << 16)) : 0u);
      }
      have = next(d);
      continue;
    }
    // Q / K: x = q * qmul or k - mean; INT8 per 64-token block
    const bool is_q = kind == 0;
    float2 neg[4];
    if (!is_q) load_pairs(s_kmean, -1.0f, neg);
    float am[2] = {0.f, 0.f};
    if (is_q) {
      // |round(q * qmul)| = round(|q| * |qmul|) and rounding is monotone: the block amax
      // of x is the rounded product of the 16-bit amax.  Rows past the sequence end (the
      // next sequence's tokens in a varlen batch) are left out.
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        uint32_t m[4] = {0u, 0u, 0u, 0u};  // four independent chains
#pragma unroll
        for (int r8 = 4 * hb; r8 < 4 * hb + 4; ++r8) {
          if (rg + 16 * r8 < valid) {
            const uint32_t* wd = reinterpret_cast<const uint32_t*>(&raw[r8]);
#pragma unroll
            for (int j = 0; j < 4; ++j) m[j] = absmax2<T>(m[j], wd[j]);
          }
        }
        const float2 f = unpack2<T>(absmax2<T>(absmax2<T>(m[0], m[1]), absmax2<T>(m[2], m[3])));
        am[hb] = __fmul_rn(fmaxf(f.x, f.y), fabsf(A.qmul));
      }
    } else {
      float a4[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};  // four chains per block
#pragma unroll
      for (int r8 = 0; r8 < 8; ++r8) {
        if (rg + 16 * r8 < valid) {
          const uint32_t* wd = reinterpret_cast<const uint32_t*>(&raw[r8]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 x = fadd2(unpack2<T>(wd[j]), neg[j]);
            a4[r8 >> 2][j] = fmax3(a4[r8 >> 2][j], fabsf(x.x), fabsf(x.y));
          }
        }
      }
      am[0] = fmaxf(fmaxf(a4[0][0], a4[0][1]), fmaxf(a4[0][2], a4[0][3]));
      am[1] = fmaxf(fmaxf(a4[1][0], a4[1][1]), fmaxf(a4[1][2], a4[1][3]));
    }
    // warp max of non-negative floats: their bit patterns order like unsigned integers
    am[0] = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(am[0])));
    am[1] = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(am[1])));
    // block amax across the 8 warps: double-buffered, exchange k completes phase k >> 1
    // of bar_blk[k & 1]; buffer k & 1 is rewritten only after every warp passed exchange
    // k + 1, i.e. after it read buffer k
    const uint32_t kb2 = nbar & 1u;
    float* r2 = s_blk + kb2 * 16;
    if (lane == 0) {
      r2[warp] = am[0];
      r2[8 + warp] = am[1];
      mbar_arrive(bar_blk + kb2);
    }
    const bool got = mbar_wait(bar_blk + kb2, (nbar >> 1) & 1u);
    ++nbar;
    if (!__all_sync(0xffffffffu, got)) {
      if (lane == 0) atomicExch(ws.status, kDevTimeoutSoftmax);
      dead = true;
      break;
    }
    float bm[2] = {0.f, 0.f};
#pragma unroll
    for (int q = 0; q < 8; ++q) { bm[0] = fmaxf(bm[0], r2[q]); bm[1] = fmaxf(bm[1], r2[8 + q]); }
    // dequant scales of the two 64-token blocks and their correctly rounded reciprocals
    const float bs[2] = {bm[0] > 0.f ? __fdiv_rn(bm[0], 127.0f) : 1.0f, bm[1] > 0.f ? __fdiv_rn(bm[1], 127.0f) : 1.0f};
    const float br[2] = {__frcp_rn(bs[0]), __frcp_rn(bs[1])};
    const float2 nbs2[2] = {make_float2(-bs[0], -bs[0]), make_float2(-bs[1], -bs[1])};
    const float2 br2[2] = {make_float2(br[0], br[0]), make_float2(br[1], br[1])};
    const int64_t tslot = (int64_t)h * (is_q ? ws.tq : ws.tk) + si.tile0 + tile;
    int8_t* dst = (is_q ? ws.qc : ws.kc) + tslot * kTileBytes;
#pragma unroll
    for (int r8 = 0; r8 < 8; ++r8) {
      const int r = rg + 16 * r8;
      const float2 nsb = nbs2[r8 >> 2], rb = br2[r8 >> 2];
      const uint32_t* wd = reinterpret_cast<const uint32_t*>(&raw[r8]);
      uint32_t y[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack2<T>(wd[j]);
        const float2 x = is_q ? fmul2(f, mul) : fadd2(f, neg[j]);
        const uint2 c = sage_code2(x, nsb, rb);
        y[2 * j] = c.x;
        y[2 * j + 1] = c.y;
      }
      const uint32_t lo = __byte_perm(__byte_perm(y[0], y[1], 0x0040), __byte_perm(y[2], y[3], 0x0040), 0x5410);
      const uint32_t hi = __byte_perm(__byte_perm(y[4], y[5], 0x0040), __byte_perm(y[6], y[7], 0x0040), 0x5410);
      const bool in = r < valid;  // rows past the sequence end get code 0
      *reinterpret_cast<uint2*>(dst + swz(r, c8 >> 1) + (c8 & 1) * 8) = make_uint2(in ? lo : 0u, in ? hi : 0u);
    }
    if (tid == 0) {
      float* sc = (is_q ? ws.qs : ws.ks) + tslot * 4;
      *reinterpret_cast<float4*>(sc) = make_float4(bs[0], bs[1], 0.f, 0.f);
    }
    have = next(d);
  }
  {
    const double kz[8] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0};
    const uint32_t vz[4] = {0u, 0u, 0u, 0u};
    while (heads_done < my_heads) exchange(kz, vz);  // only after a wait gave up
  }
  if (kv) {
    cluster_arrive();  // no CTA leaves while another may still read its partials
    cluster_wait();
  }
}

// ------------------------------------------------------------- attention --
// One CTA = two 128-row Q tiles of one (sequence, head) sharing every K/V tile.
//   warp 0      producer: bulk copies of Q tiles, K scales, K/V tiles (3-stage ring)
//   warp 1      MMA issuer: per KV tile QK0, QK1 (kind::i8 -> S_t in TMEM), then
//               PV0, PV1 of the previous tile (kind::f8f6f4 -> O_t in TMEM)
//   warps 4-7   softmax for Q tile 0, warps 8-11 softmax for Q tile 1: one row per
//               thread, TMEM -> registers, base-2 online softmax with lazy rescaling
//               (the running max only moves when a row's max grows by more than
//               kTau), P -> e4m3 into a double-buffered swizzled smem tile, epilogue
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
// Registers: 384 threads x 168; a softmax thread holds its full 128-column S row.
constexpr int kAttnThreads = 384;
constexpr uint32_t kTmemCols = 512;
constexpr float kTau = 4.0f;                    // lazy-rescale threshold (log2 units)
constexpr float kPScaleLog2 = kLog2_448 - kTau;  // P_fp8 = 2^(x - m_run + kPScaleLog2) <= 448
constexpr float kMagic = 12582912.0f;           // 1.5 * 2^23
constexpr int kMagicBits = 0x4B400000;

struct AttnSmem {
  static constexpr int q = 0;                                   // 2 Q tiles
  static constexpr int kv = q + 2 * kTileBytes;                 // stages x (K, V)
  static constexpr int p = kv + kStages * 2 * kTileBytes;       // kPBuf P tiles per Q tile ([t][buf])
  static constexpr int kscale = p + 2 * kPBuf * kTileBytes;     // up to kMaxKvTiles x 16 B
  static constexpr int bars = kscale + kMaxKvTiles * 16;
  static constexpr int nbars = 1 + 2 * kStages + 2 * 4 + 2 * kPBuf + 1;
  static constexpr int misc = bars + nbars * 8;
  static constexpr int total = misc + 64;
  static constexpr int alloc = total + 1024;  // slack for manual 1024-B alignment
};
static_assert(AttnSmem::alloc <= 227 * 1024, "attention shared memory exceeds the per-CTA limit");

struct AttnParams {
  Workspace ws;
  SeqGeom g;
  void* out;
  Strides3 os;
  int Hq, Hkv;
  int out_bf16;
  int D;          // head dim of the inputs and output (64, 96 or 128)
  long long wait_clocks;  // bound of every mbarrier wait (SM clocks)
  int skip_kv;    // failure-injection tests only: K/V tile index whose load is never issued (-1: none)
};

QF2_DEV void store_row_out(void* out, const Strides3& os, int b, int h, int64_t tok, const float* o, bool bf16,
                           int col0) {
  if (bf16) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(out) + (int64_t)b * os.b + (int64_t)h * os.h + tok * os.s +
                         col0;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      uint4 pk;
      uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 t = __floats2bfloat162_rn(o[v * 8 + 2 * j], o[v * 8 + 2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t*>(&t);
      }
      *reinterpret_cast<uint4*>(dst + v * 8) = pk;
    }
  } else {
    __half* dst = reinterpret_cast<__half*>(out) + (int64_t)b * os.b + (int64_t)h * os.h + tok * os.s + col0;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      uint4 pk;
      uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __half2 t = __floats2half2_rn(o[v * 8 + 2 * j], o[v * 8 + 2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t*>(&t);
      }
      *reinterpret_cast<uint4*>(dst + v * 8) = pk;
    }
  }
}

// 2^x on the FMA pipe (no SFU) for two lanes, x >= -126 after clamping: x = n + f with
// n = floor(x) (round-toward-minus-infinity add of 1.5 * 2^23) and f in [0, 1); 2^f by a
// degree-3 polynomial (relative error < 7.5e-5 on [0, 1); coefficients from a Lawson
// minimax fit of 2^f done for this kernel), then n added to the exponent field: the low
// bits of 1.5 * 2^23 + n shifted left by 23 are n << 23.  Used for part of the softmax
// exponentials so that the SFU and the FMA pipe share them.
#ifndef QF2_SAGE_EMU_MASK
#define QF2_SAGE_EMU_MASK 0
#endif
constexpr uint32_t kEmuMask = QF2_SAGE_EMU_MASK;   // bit c: chunk c of a row's 8 uses exp2_fma2
// the chunk (of 8 per row) after which a softmax warpgroup lets the other one start its exp
// pass (measured: 5, i.e. three quarters into the pass)
#ifndef QF2_SAGE_PP_CHUNK
#define QF2_SAGE_PP_CHUNK 5
#endif
constexpr int kPingPongChunk = QF2_SAGE_PP_CHUNK;
QF2_DEV float2 exp2_fma2(float2 x) {
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  float2 r;
  asm("{\n\t.reg .b64 rx, rm, rt, rn, rf, rp, rc;\n\t.reg .b32 px, py, tx, ty;\n\t"
      "mov.b64 rx, {%2, %3};\n\t"
      "mov.b64 rm, {0f4B400000, 0f4B400000};\n\t"
      "add.rm.f32x2 rt, rx, rm;\n\t"                       // 1.5 * 2^23 + floor(x)
      "sub.rn.f32x2 rn, rm, rt;\n\t"                       // -floor(x), exact
      "add.rn.f32x2 rf, rx, rn;\n\t"                       // f = x - floor(x), exact
      "mov.b64 rc, {0f3D9FCB2E, 0f3D9FCB2E};\n\t"
      "mov.b64 rp, {0f3E677E2C, 0f3E677E2C};\n\t"
      "fma.rn.f32x2 rp, rc, rf, rp;\n\t"
      "mov.b64 rc, {0f3F322228, 0f3F322228};\n\t"
      "fma.rn.f32x2 rp, rp, rf, rc;\n\t"
      "mov.b64 rc, {0f3F7FFB19, 0f3F7FFB19};\n\t"
      "fma.rn.f32x2 rp, rp, rf, rc;\n\t"                   // 2^f
      "mov.b64 {px, py}, rp;\n\tmov.b64 {tx, ty}, rt;\n\t"
      "shl.b32 tx, tx, 23;\n\tshl.b32 ty, ty, 23;\n\t"
      "add.s32 %0, px, tx;\n\tadd.s32 %1, py, ty;\n\t}"
      : "=r"(*reinterpret_cast<uint32_t*>(&r.x)), "=r"(*reinterpret_cast<uint32_t*>(&r.y))
      : "f"(x.x), "f"(x.y));
  return r;
}





// grid (ceil(max q tiles / 2) * nsplit, Hq, batch).  With nsplit > 1 a CTA walks the KV
// tiles [jb, jb + nkt) of its split and writes normalised partial rows (bf16) with their
// running max and row sum to the workspace; sage_combine_kernel merges the splits.
// KSTEPS = D / 32: the QK^T MMA K-steps (32 INT8 channels each).  PV keeps N = 128 (the V
// codes of channels >= D are 0) -- its MMA time is hidden behind the exp-bound softmax.
template <int KSTEPS>
__global__ void __launch_bounds__(kAttnThreads, 1) sage_attn_kernel(AttnParams P) {
  extern __shared__ uint8_t smem_raw[];
  const int nsplit = P.ws.nsplit;
  const int pair = blockIdx.x / nsplit, split = blockIdx.x - pair * nsplit, h = blockIdx.y, b = blockIdx.z;
  const SeqInfo sq = seq_q(P.g, b);
  const int64_t nqt = (sq.len + kTile - 1) / kTile;
  const int qt0 = 2 * pair;
  if (qt0 >= nqt) return;
  const int ntile = (qt0 + 1 < nqt) ? 2 : 1;  // Q tiles in this CTA
  const SeqInfo sk = seq_k(P.g, b);
  const int nkt_all = (int)((sk.len + kTile - 1) / kTile);
  const int per_split = (nkt_all + nsplit - 1) / nsplit;
  const int jb = min(nkt_all, split * per_split);
  const int nkt = min(nkt_all, jb + per_split) - jb;  // KV tiles of this CTA: [jb, jb + nkt)
  const int hk = h / (P.Hq / P.Hkv);

  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base + AttnSmem::q;
  uint8_t* sKV = base + AttnSmem::kv;
  uint8_t* sP = base + AttnSmem::p;
  float4* sKS = reinterpret_cast<float4*>(base + AttnSmem::kscale);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + AttnSmem::bars);
  uint64_t* bar_q = bars;
  uint64_t* bar_kv_full = bars + 1;
  uint64_t* bar_kv_empty = bar_kv_full + kStages;
  uint64_t* bar_s_full = bar_kv_empty + kStages;  // [2] per Q tile
  uint64_t* bar_s_empty = bar_s_full + 2;          // [2]
  uint64_t* bar_p_full = bar_s_empty + 2;          // [2 tiles]
  uint64_t* bar_o_done = bar_p_full + 2;           // [tile][P buffer]: PV_t(i) of P buffer i % kPBuf completed
  uint64_t* bar_pp = bar_o_done + 2 * kPBuf;       // [2 tiles]: softmax t is far enough into its exp pass
  uint64_t* bar_drain = bar_pp + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + AttnSmem::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + AttnSmem::misc + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < kStages; ++s) { mbar_init(bar_kv_full + s, 1); mbar_init(bar_kv_empty + s, 1); }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar_s_full + t, 1);
      mbar_init(bar_s_empty + t, 4);
      mbar_init(bar_p_full + t, 4);
      for (int bb = 0; bb < kPBuf; ++bb) mbar_init(bar_o_done + t * kPBuf + bb, 1);
      mbar_init(bar_pp + t, 4);
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

  const Workspace& ws = P.ws;
  auto fail = [&](int code) {
    atomicExch(ws.status, code);
    *abort_flag = 1;
  };

  // warp-uniform bounded wait: every lane agrees on the outcome, so .sync.aligned
  // instructions and elected issue that follow always see a converged warp
  auto wwait = [&](uint64_t* bar, uint32_t parity) -> bool {
    const bool w = mbar_wait(bar, parity, P.wait_clocks) && (*abort_flag == 0);
    return __all_sync(0xffffffffu, w);
  };

  if (warp < 4) {
    if (warp == 0 && nkt > 0) {
      // ------------------------------------------------------- producer --
      // the whole warp runs the loop (uniform addresses), lane 0 issues the copies
      const int64_t qslot = (int64_t)h * ws.tq + sq.tile0 + qt0;
      const int64_t kslot0 = (int64_t)hk * ws.tk + sk.tile0 + jb;
      if (lane == 0) {
        mbar_arrive_expect_tx(bar_q, ntile * kTileBytes + nkt * 16);
        bulk_g2s(sQ, ws.qc + qslot * kTileBytes, ntile * kTileBytes, bar_q);
        bulk_g2s(sKS, ws.ks + kslot0 * 4, nkt * 16, bar_q);
      }
      int issued = 0;
      for (int j = 0; j < nkt; ++j) {
        const int s = j % kStages, r = j / kStages;
        if (!wwait(bar_kv_empty + s, (r & 1) ^ 1)) { if (lane == 0) fail(kDevTimeoutProducer); break; }
        if (lane == 0 && jb + j != P.skip_kv) {
          mbar_arrive_expect_tx(bar_kv_full + s, 2 * kTileBytes);
          uint8_t* dK = sKV + s * 2 * kTileBytes;
          bulk_g2s(dK, ws.kc + (kslot0 + j) * kTileBytes, kTileBytes, bar_kv_full + s);
          bulk_g2s(dK + kTileBytes, ws.vc + (kslot0 + j) * kTileBytes, kTileBytes, bar_kv_full + s);
        }
        __syncwarp();
        issued = j + 1;
      }
      if (*abort_flag && lane == 0) {
        // let the copies already issued land before the CTA's shared memory goes away
        // (a load that was never issued only costs its bounded wait)
        mbar_wait(bar_q, 0, P.wait_clocks);
        for (int j = issued > kStages ? issued - kStages : 0; j < issued; ++j)
          mbar_wait(bar_kv_full + (j % kStages), (j / kStages) & 1, P.wait_clocks);
      }
    } else if (warp == 1 && nkt > 0) {
      // ------------------------------------------------------------ MMA --
      // converged warp: descriptors are warp-uniform, lane 0 issues and commits
      constexpr uint32_t idesc_qk = make_idesc(2, 1, 1, 0, 0, kTile, kTile);     // s8 x s8 -> s32
      // e4m3 x e4m3 -> f32; V tiles are token-major (MN-major B: 128-byte rows of channels,
      // 8-token swizzle atoms 1024 B apart, one 32-token K step = 4096 B)
      constexpr uint32_t idesc_pv = make_idesc(1, 0, 0, 0, 1, kTile, kHeadDim);
      bool ok = wwait(bar_q, 0);
      // Descriptors are built once; per stage / k-step only the 14-bit start-address
      // field moves (16-byte units: a stage is 2048, a 32-byte k-step is 2).
      const uint64_t dQ0 = sdesc_sw128_kmajor(smem_u32(sQ));
      const uint64_t dP0 = sdesc_sw128_kmajor(smem_u32(sP));
      const uint64_t dK0 = sdesc_sw128_kmajor(smem_u32(sKV));
      constexpr uint64_t kTileStep = kTileBytes >> 4, kStageStep = 2 * kTileBytes >> 4;
      auto issue_pv = [&](int i) -> bool {
        const uint32_t aV = smem_u32(sKV) + (uint32_t)(i % kStages) * 2 * kTileBytes + kTileBytes;
        for (int t = 0; t < ntile; ++t) {
          if (!wwait(bar_p_full + t, i & 1)) return false;
          tc_fence_after();
          const uint64_t dP = dP0 + (uint64_t)(t * kPBuf + i % kPBuf) * kTileStep;
          if (lane == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_f8f6f4(tmem + 256 + t * 128, dP + 2 * kk, sdesc_sw128_mnmajor(aV + kk * 4096, kTileBytes, 1024),
                         idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
            tc_commit(bar_o_done + t * kPBuf + i % kPBuf);
          }
          __syncwarp();
        }
        if (lane == 0) tc_commit(bar_kv_empty + (i % kStages));
        __syncwarp();
        return true;
      };
      for (int j = 0; ok && j < nkt; ++j) {
        const int s = j % kStages;
        if (!wwait(bar_kv_full + s, (j / kStages) & 1)) { ok = false; break; }
        const uint64_t dK = dK0 + (uint64_t)s * kStageStep;
        for (int t = 0; t < ntile && ok; ++t) {
          // S_t holds the softmax warps' fill of the magic bits (their arrive of phase j)
          if (!wwait(bar_s_empty + t, j & 1)) { ok = false; break; }
          tc_fence_after();
          const uint64_t dQ = dQ0 + (uint64_t)t * kTileStep;
          if (lane == 0) {
            // accumulate onto the fill: S = 0x4B400000 + q.k (int32) is the fp32 bit pattern
            // of 1.5 * 2^23 + q.k, the magic encoding the softmax reads as a float directly
#pragma unroll
            for (int kk = 0; kk < KSTEPS; ++kk) mma_i8(tmem + t * 128, dQ + 2 * kk, dK + 2 * kk, idesc_qk, 1u);
            tc_commit(bar_s_full + t);
          }
          __syncwarp();
        }
        if (ok && j > 0 && !issue_pv(j - 1)) ok = false;
      }
      if (ok) ok = issue_pv(nkt - 1);
      if (lane == 0) {
        if (!ok) fail(kDevTimeoutMma);
        // drain: wait until every MMA issued above has completed
        tc_commit(bar_drain);
        mbar_wait(bar_drain, 0);
      }
      __syncwarp();
    }
  } else {
    // -------------------------------------------------------- softmax --
    const int t = (warp >> 2) - 1;  // Q tile of this warpgroup
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * 128;
    const uint32_t tO = tmem + lane_off + 256 + t * 128;
    const bool active = t < ntile;
    const int qt = qt0 + t;
    const float* vsc = ws.vs + ((int64_t)b * P.Hkv + hk) * kHeadDim;
    bool ok = active && nkt > 0;
    float sqs = 0.f;
    if (ok) {
      const int64_t qslot = (int64_t)h * ws.tq + sq.tile0 + qt;
      sqs = ws.qs[qslot * 4 + (row >> 6)];
      ok = wwait(bar_q, 0);  // k scales are in smem once the Q tiles have landed
    }
    // S_t starts each KV tile filled with the magic bits 0x4B400000 (the QK MMA accumulates
    // onto it), so the int32 scores read back are already the fp32 encoding 1.5 * 2^23 + s
    // (|s| <= 128 * 127^2 < 2^22): no conversion per element.  The fill of tile j + 1 is
    // stored right after tile j is read, before S_t is handed back to the MMA warp.
    auto fill_s = [&]() {
#pragma unroll
      for (int c = 0; c < 16; ++c) tmem_fill8(tS + c * 8, (uint32_t)kMagicBits);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_s_empty + t);
    };
    if (ok) fill_s();
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; ok && j < nkt; ++j) {
      if (!wwait(bar_s_full + t, j & 1)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
      tmem_wait_ld();
      if (j + 1 < nkt) fill_s();
      float mf[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) mf[i] = __uint_as_float(s[i]);
      const int64_t rem = sk.len - (int64_t)(jb + j) * kTile;
      if (rem < kTile) {
        // ragged last tile: keys past the sequence end get -inf (below every magic-encoded
        // value in the max, and fma(-inf, sc > 0, c) = -inf gives P = 0 whatever the scales)
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= rem) mf[i] = -INFINITY;
      }
      // row max per 64-column half (one K scale each): 4 independent fmax3 chains
      float mq[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float m = fmax3(mf[c * 16], mf[c * 16 + 1], mf[c * 16 + 2]);
#pragma unroll
        for (int i = 3; i < 15; i += 2) m = fmax3(m, mf[c * 16 + i], mf[c * 16 + i + 1]);
        mq[c] = fmaxf(m, mf[c * 16 + 15]);
      }
      const float mx0 = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
      const float mx1 = fmaxf(fmaxf(mq[4], mq[5]), fmaxf(mq[6], mq[7]));
      const float4 ksc = sKS[j];
      const float sc0 = sqs * ksc.x, sc1 = sqs * ksc.y;
      const float m_tile = fmaxf((mx0 - kMagic) * sc0, (mx1 - kMagic) * sc1);
      const float m_new = fmaxf(m_run, m_tile);
      const bool rescale = __any_sync(0xffffffffu, m_new > m_run + kTau);
      float alpha = 1.0f;
      if (rescale) {
        alpha = fast_exp2(m_run - m_new);  // 0 on the first tile
        m_run = m_new;
        l_run *= alpha;
      }
      // P_fp8 = 2^(x - m_run + kPScaleLog2) with x = (mf - magic) * sc, as one fma on the
      // magic-encoded integer: fma(mf, sc, -(magic * sc + bias)).  The product is exact inside
      // the fma; the folded constant's rounding shifts a row half's exponents by at most
      // half an ulp of magic * sc (~1e-4 in log2 units for these scales), a common factor
      // of that half's P and row sum, far below the e4m3 rounding of P.
      const float bias = m_run - kPScaleLog2;
      const float c0 = -fmaf(kMagic, sc0, bias), c1 = -fmaf(kMagic, sc1, bias);
      const float2 cv0 = make_float2(c0, c0), cv1 = make_float2(c1, c1);
      const float2 sc0v = make_float2(sc0, sc0), sc1v = make_float2(sc1, sc1);
      // P buffer j % kPBuf was last read by PV_t(j - kPBuf): wait for it (phase
      // (j - kPBuf) / kPBuf of that buffer's barrier; its next phase needs this thread's P)
      const int pb = j % kPBuf;
      if (j >= kPBuf && !wwait(bar_o_done + t * kPBuf + pb, ((j - kPBuf) / kPBuf) & 1)) { ok = false; break; }
      if (ntile == 2) {  // ping-pong (see the arrive in the exp pass below)
        if (t == 1 && !wwait(bar_pp, j & 1)) { ok = false; break; }
        if (t == 0 && j >= 1 && !wwait(bar_pp + 1, (j - 1) & 1)) { ok = false; break; }
      }
      uint8_t* pdst = sP + (t * kPBuf + pb) * kTileBytes;
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int chunk = 0; chunk < 8; ++chunk) {
        const float2 scv = chunk < 4 ? sc0v : sc1v, cv = chunk < 4 ? cv0 : cv1;
        uint32_t w[4];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int i0 = chunk * 16 + q4 * 4;
          const float2 x01 = ffma2(make_float2(mf[i0], mf[i0 + 1]), scv, cv);
          const float2 x23 = ffma2(make_float2(mf[i0 + 2], mf[i0 + 3]), scv, cv);
          float2 p01, p23;
          if ((kEmuMask >> chunk) & 1u) {   // compile-time: this chunk's exps on the FMA pipe
            p01 = exp2_fma2(x01);
            p23 = exp2_fma2(x23);
          } else {
            p01 = make_float2(fast_exp2(x01.x), fast_exp2(x01.y));
            p23 = make_float2(fast_exp2(x23.x), fast_exp2(x23.y));
          }
          acc = fadd2(acc, fadd2(p01, p23));
          w[q4] = (uint32_t)f32x2_to_e4m3x2(p01.x, p01.y) | ((uint32_t)f32x2_to_e4m3x2(p23.x, p23.y) << 16);
        }
        *reinterpret_cast<uint4*>(pdst + swz(row, chunk)) = make_uint4(w[0], w[1], w[2], w[3]);
        // ping-pong of the two softmax warpgroups over the SFU: tile 1's exp pass of
        // iteration j starts when tile 0's is three quarters done, tile 0's of j + 1 when
        // tile 1's is (measured: the exp pass of one warpgroup alone does not fill the
        // SFU, two fully overlapped ones leave it idle during the max passes)
        if (ntile == 2 && chunk == kPingPongChunk) {
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_pp + t);
        }
      }
      l_run += acc.x + acc.y;
      if (rescale && j > 0) {
        // O holds sum_{i<j} P_i V_i against the old max once PV(j-1) has completed;
        // PV(j) is only issued after p_full(j) below
        if (kPBuf > 1 && !wwait(bar_o_done + t * kPBuf + (j - 1) % kPBuf, ((j - 1) / kPBuf) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
        tmem_wait_st();
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p_full + t);
    }
    if (active && nkt > 0 && !ok) fail(kDevTimeoutSoftmax);
    // ------------------------------------------------------- epilogue --
    if (active) {
      const int64_t r_tok = (int64_t)qt * kTile + row;
      if (ok && nkt > 0) {
        if (!wwait(bar_o_done + t * kPBuf + (nkt - 1) % kPBuf, ((nkt - 1) / kPBuf) & 1)) {
          fail(kDevTimeoutEpilogue);
          ok = false;
        }
        tc_fence_after();
      }
      const float inv_l = (ok && l_run > 0.f) ? 1.0f / l_run : 0.f;
#pragma unroll 1
      for (int c = 0; c < KSTEPS; ++c) {
        uint32_t o[32];
        if (ok && nkt > 0) {
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        float of[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) of[i] = __uint_as_float(o[i]) * vsc[c * 32 + i] * inv_l;
        if (r_tok >= sq.len) continue;
        if (nsplit == 1) {
          store_row_out(P.out, P.os, P.g.cu_q ? 0 : b, h, sq.tok0 + r_tok, of, P.out_bf16, c * 32);
        } else {
          const int64_t prow = (int64_t)split * ws.prows + ((int64_t)h * ws.tq + sq.tile0 + qt) * kTile + row;
          store_row_out(ws.part_o, Strides3{0, 0, kHeadDim}, 0, 0, prow, of, true, c * 32);
          if (c == 0) ws.part_ml[prow] = make_float2(m_run, ok ? l_run : 0.f);
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

// ---------------------------------------------------------------- combine --
// grid (tiles * 8, Hq, batch), 256 threads: 16 rows x 16 chunks of 8 channels.  Row r of
// split s holds o_s = O_s / l_s (bf16) with the running max m_s and row sum l_s of its
// base-2 softmax; the merged row is sum_s w_s o_s / sum_s w_s with w_s = l_s 2^(m_s - M).
__global__ void __launch_bounds__(256) sage_combine_kernel(AttnParams P) {
  const Workspace& ws = P.ws;
  const int b = blockIdx.z, h = blockIdx.y;
  const SeqInfo sq = seq_q(P.g, b);
  const int64_t r_tok = (int64_t)blockIdx.x * 16 + (threadIdx.x >> 4);
  if (r_tok >= sq.len) return;
  const int c8 = threadIdx.x & 15;
  if (c8 * 8 >= P.D) return;
  const int64_t prow = ((int64_t)h * ws.tq + sq.tile0) * kTile + r_tok;
  float m[kMaxSplits], w[kMaxSplits];
  float M = -INFINITY;
  for (int sp = 0; sp < ws.nsplit; ++sp) {
    const float2 ml = ws.part_ml[sp * ws.prows + prow];
    m[sp] = ml.y > 0.f ? ml.x : -INFINITY;
    w[sp] = ml.y;
    M = fmaxf(M, m[sp]);
  }
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (M > -INFINITY) {
    float W = 0.f;
    for (int sp = 0; sp < ws.nsplit; ++sp) {
      w[sp] = m[sp] > -INFINITY ? w[sp] * fast_exp2(m[sp] - M) : 0.f;
      W += w[sp];
    }
    const float invW = 1.0f / W;
    for (int sp = 0; sp < ws.nsplit; ++sp) {
      const uint4 raw = *reinterpret_cast<const uint4*>(ws.part_o + (sp * ws.prows + prow) * kHeadDim + c8 * 8);
      const float wn = w[sp] * invW;
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += wn * __bfloat162float(e[j]);
    }
  }
  uint4 pk;
  uint32_t* wd = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (P.out_bf16) {
      __nv_bfloat162 t = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
      wd[j] = *reinterpret_cast<uint32_t*>(&t);
    } else {
      __half2 t = __floats2half2_rn(acc[2 * j], acc[2 * j + 1]);
      wd[j] = *reinterpret_cast<uint32_t*>(&t);
    }
  }
  uint8_t* dst = reinterpret_cast<uint8_t*>(P.out) +
                 2 * ((int64_t)b * P.os.b + (int64_t)h * P.os.h + (sq.tok0 + r_tok) * P.os.s + c8 * 8);
  *reinterpret_cast<uint4*>(dst) = pk;
}

// ------------------------------------------------------------------ host --
struct Layout {
  int64_t off[12];
  int64_t tq, tk, nch;
  int64_t prows;
  int nsplit;
};

static int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Failure-injection settings of the attention launches (qf2_sage_fault_injection): the
// bound of every mbarrier wait, and a K/V tile whose load the producer never issues.
static std::atomic<long long> g_attn_wait_clocks{kWaitClocks};
static std::atomic<int> g_attn_skip_kv{-1};

// KV splits of the attention for a dense problem whose CTAs (pairs of Q tiles per head)
// fill few waves: each split walks a contiguous part of the K/V tiles and leaves
// normalised partial rows (bf16) with their running max and row sum; a combine kernel
// merges them.  Cost model in KV-tile iterations of one CTA (~2.1 us each), fitted to
// measured times at 3-24 heads and 4608 / 16896 tokens: waves x (tiles per split + a
// fixed 4 per CTA for its prologue and pipeline fill) + the partial rows' write and read
// (~135 KB per Q-tile pair and split, ~0.0105 iterations at HBM speed).  Varlen problems
// do not split.
static int attn_splits(int64_t batch, int64_t Hq, int64_t max_q, int64_t max_k, bool varlen) {
  if (varlen) return 1;
  int sms = 0;
  if (qf2_sm_count(&sms) != cudaSuccess || sms <= 0) sms = 148;
  const int64_t units = (((max_q + kTile - 1) / kTile + 1) / 2) * Hq * batch;
  const int64_t nkt = (max_k + kTile - 1) / kTile;
  if (units <= 0 || nkt < 4) return 1;
  constexpr double kCtaFixed = 4.0, kPartialPerUnit = 0.0105;
  auto cost = [&](int sp) {
    const int64_t per = (nkt + sp - 1) / sp;
    const double c = (double)((units * sp + sms - 1) / sms) * ((double)per + kCtaFixed);
    return sp > 1 ? c + kPartialPerUnit * (double)(units * sp) : c;
  };
  int best = 1;
  double best_c = cost(1);
  for (int sp = 2; sp <= kMaxSplits && (nkt + sp - 1) / sp >= 2; ++sp) {
    const double c = cost(sp);
    if (c < best_c - 1e-9) { best_c = c; best = sp; }
  }
  return best;
}

static Layout make_layout(int64_t batch, int64_t Hq, int64_t Hkv, int64_t total_q, int64_t total_k,
                          int64_t max_q, int64_t max_k, bool varlen) {
  Layout L;
  if (varlen) {
    L.tq = total_q / kTile + batch;
    L.tk = total_k / kTile + batch;
  } else {
    L.tq = batch * ((max_q + kTile - 1) / kTile);
    L.tk = batch * ((max_k + kTile - 1) / kTile);
  }
  L.nch = std::max<int64_t>(1, (max_k + kTile - 1) / kTile);
  L.nsplit = attn_splits(batch, Hq, max_q, max_k, varlen);
  L.prows = Hq * L.tq * kTile;
  const int64_t np = L.nsplit > 1 ? L.nsplit * L.prows : 0;
  int64_t o = 0;
  auto put = [&](int i, int64_t bytes) { L.off[i] = o; o = align_up(o + bytes, 1024); };
  put(0, 256);                                       // status word, Q tile counter at byte 16
  put(1, Hq * L.tq * kTileBytes);                    // q codes
  put(2, Hq * L.tq * 16);                            // q scales
  put(3, Hkv * L.tk * kTileBytes);                   // k codes
  put(4, Hkv * L.tk * 16);                           // k scales
  put(5, Hkv * L.tk * kTileBytes);                   // v codes (token-major tiles)
  put(6, batch * Hkv * kHeadDim * 4);                // v scales
  put(7, batch * Hkv * kHeadDim * 4);                // k mean
  put(8, batch * Hkv * kHeadDim * 4);                // v inverse scales (448 / amax)
  put(9, np * kHeadDim * 2);                         // split-KV partial rows (bf16)
  put(10, np * 8);                                   // split-KV running max and row sum
  L.off[11] = o;
  return L;
}

static Workspace bind_ws(void* w, const Layout& L) {
  uint8_t* p = reinterpret_cast<uint8_t*>(w);
  Workspace ws;
  ws.status = reinterpret_cast<int*>(p + L.off[0]);
  ws.qc = reinterpret_cast<int8_t*>(p + L.off[1]);
  ws.qs = reinterpret_cast<float*>(p + L.off[2]);
  ws.kc = reinterpret_cast<int8_t*>(p + L.off[3]);
  ws.ks = reinterpret_cast<float*>(p + L.off[4]);
  ws.vc = reinterpret_cast<uint8_t*>(p + L.off[5]);
  ws.vs = reinterpret_cast<float*>(p + L.off[6]);
  ws.kmean = reinterpret_cast<float*>(p + L.off[7]);
  ws.vinv = reinterpret_cast<float*>(p + L.off[8]);
  ws.part_o = reinterpret_cast<__nv_bfloat16*>(p + L.off[9]);
  ws.part_ml = reinterpret_cast<float2*>(p + L.off[10]);
  ws.prows = L.prows;
  ws.nsplit = L.nsplit;
  ws.tq = L.tq; ws.tk = L.tk; ws.nch = L.nch;
  return ws;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

struct Args {
  const void *q, *k, *v;
  void* out;
  Strides3 qs, ks, vs, os;
  const int32_t *cu_q, *cu_k;
  int64_t batch, Sq, Skv, total_q, total_k, max_q, max_k, Hq, Hkv, D;
  float sm_scale;
  int dtype;
  void* workspace;
  int64_t ws_bytes;
  cudaStream_t stream;
};

static int validate(const Args& a, bool need_out) {
  if (!a.q || !a.k || !a.v || !a.workspace || (need_out && !a.out)) return QF2_ERR_ARG;
  if (a.dtype != QF2_BF16 && a.dtype != QF2_F16) return QF2_ERR_DTYPE;
  if (!head_dim_ok(a.D)) return QF2_ERR_SHAPE;
  if (a.Hq <= 0 || a.Hkv <= 0 || a.Hq % a.Hkv != 0 || a.batch <= 0) return QF2_ERR_SHAPE;
  if (a.max_q < 0 || a.max_k < 0 || a.max_k > (int64_t)kMaxKvTiles * kTile) return QF2_ERR_SHAPE;
  if (a.Hq > 65535 || a.Hq + 2 * a.Hkv > 65535 || a.batch > 65535) return QF2_ERR_SHAPE;
  // the quantization grid is one-dimensional: batch * (Hq * q tiles + 2 * Hkv * kv tiles) CTAs
  if ((double)a.batch * ((double)a.Hq * (double)((a.max_q + kTile - 1) / kTile) +
                         2.0 * (double)a.Hkv * (double)((a.max_k + kTile - 1) / kTile)) > 2147483647.0)
    return QF2_ERR_SHAPE;
  if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || (need_out && !aligned16(a.out))) return QF2_ERR_ALIGN;
  const Strides3* ss[4] = {&a.qs, &a.ks, &a.vs, &a.os};
  for (int i = 0; i < (need_out ? 4 : 3); ++i) {
    if ((ss[i]->b % 8) || (ss[i]->h % 8) || (ss[i]->s % 8)) return QF2_ERR_ALIGN;
  }
  const bool varlen = a.cu_q != nullptr;
  const Layout L = make_layout(a.batch, a.Hq, a.Hkv, a.total_q, a.total_k, a.max_q, a.max_k, varlen);
  if (a.ws_bytes < L.off[11] || !aligned16(a.workspace) || (reinterpret_cast<uintptr_t>(a.workspace) & 1023))
    return QF2_ERR_WORKSPACE;
  return QF2_OK;
}

// Tensor map over q, k or v as {channels (D), tokens, heads, batch} with a 128 x 128 box
// and no swizzle (the consumers read whole 256-byte rows; for D < 128 the box's channels
// past D lie outside the tensor and arrive as zeros).  Varlen inputs have one batch entry
// whose stride is only a placeholder.
static bool make_prep_map(CUtensorMap* m, const void* base, const Strides3& st, int64_t tokens, int64_t H,
                          int64_t batch_ext, int dtype, int64_t D) {
  const uint64_t esz = 2;
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)tokens, (uint64_t)H, (uint64_t)batch_ext};
  const uint64_t sb = st.b != 0 ? (uint64_t)st.b * esz : (uint64_t)st.s * esz * (uint64_t)tokens;
  const uint64_t strides[3] = {(uint64_t)st.s * esz, (uint64_t)st.h * esz, sb};
  const uint32_t box[4] = {(uint32_t)kHeadDim, (uint32_t)kTile, 1, 1};
  return qf2_make_tmap_4d_noswizzle(m, dtype == QF2_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                                    base, dims, strides, box);
}


// Whether clusters of 16 prep CTAs (non-portable size) can run on the current device,
// cached per device; enables the size on first use.
template <typename T>
static bool prep_cluster16_ok() {
  static std::atomic<int> cache[64];  // 0 unknown, 1 yes, 2 no
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  int v = cache[dev & 63].load(std::memory_order_relaxed);
  if (v == 0) {
    v = 2;
    if (cudaFuncSetAttribute(sage_prep_kernel<T>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess &&
        cudaFuncSetAttribute(sage_prep_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, PrepSmem::total) ==
            cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(16);
      cfg.blockDim = dim3(kPrepThreads);
      cfg.dynamicSmemBytes = PrepSmem::total;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 16;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, sage_prep_kernel<T>, &cfg) == cudaSuccess && n >= 4) v = 1;
    }
    cudaGetLastError();  // a refused size leaves no sticky error behind
    cache[dev & 63].store(v, std::memory_order_relaxed);
  }
  return v == 1;
}

template <typename T>
static int launch_quant(const Args& a) {
  const bool varlen = a.cu_q != nullptr;
  const Layout L = make_layout(a.batch, a.Hq, a.Hkv, a.total_q, a.total_k, a.max_q, a.max_k, varlen);
  PrepArgs A;
  A.ws = bind_ws(a.workspace, L);
  A.g.cu_q = a.cu_q; A.g.cu_k = a.cu_k; A.g.Sq = a.Sq; A.g.Skv = a.Skv;
  A.g.tiles_q_dense = (a.Sq + kTile - 1) / kTile;
  A.g.tiles_k_dense = (a.Skv + kTile - 1) / kTile;
  A.batch = (int)a.batch; A.Hq = (int)a.Hq; A.Hkv = (int)a.Hkv;
  A.mtq = (a.max_q + kTile - 1) / kTile;
  const int64_t mtk = (a.max_k + kTile - 1) / kTile;
  A.qmul = (float)((double)a.sm_scale * 1.4426950408889634);
  A.varlen = varlen ? 1 : 0;
  const int64_t tok_q = varlen ? a.total_q : a.Sq, tok_k = varlen ? a.total_k : a.Skv;
  const int64_t bext = varlen ? 1 : a.batch;
  CUtensorMap mq, mk, mv;
  memset(&mq, 0, sizeof(mq));
  memset(&mk, 0, sizeof(mk));
  memset(&mv, 0, sizeof(mv));
  if (A.mtq > 0 && !make_prep_map(&mq, a.q, a.qs, tok_q, a.Hq, bext, a.dtype, a.D)) return QF2_ERR_ALIGN;
  if (mtk > 0 && (!make_prep_map(&mk, a.k, a.ks, tok_k, a.Hkv, bext, a.dtype, a.D) ||
                  !make_prep_map(&mv, a.v, a.vs, tok_k, a.Hkv, bext, a.dtype, a.D)))
    return QF2_ERR_ALIGN;
  int sms = 0;
  QF2_CUDA_CHECK(qf2_sm_count(&sms));
  static std::atomic<uint64_t> attr_done{0};
  QF2_CUDA_CHECK(qf2_set_smem_once(sage_prep_kernel<T>, PrepSmem::total, &attr_done));
  // One wave of CTAs, about two thirds of it with the K/V role (per element K/V read two
  // tensors and write two codes, Q one and one) in clusters of up to 8 CTAs (at most one
  // per tile of the longest sequence) that walk the kv heads; fewer heads in flight keep
  // phase 1's tiles in L2 for phase 2.  The other CTAs start on Q tiles, which the K/V
  // CTAs join when they are done.
  const int64_t slots = (int64_t)sms * kPrepCtasPerSm;
  const int64_t heads = a.batch * a.Hkv;
  int C = (int)std::min<int64_t>(kMaxCluster, std::max<int64_t>(1, mtk));
  // few kv heads (a head-parallel shard: 3 heads of 4608 tokens on 8 GPUs): clusters of 16
  // (a non-portable size, used where the device can place them) halve each K/V CTA's share
  // of its head, the critical path when every head fits the K/V role's CTA budget at 16
  // (with more heads, 16-CTA clusters would take them in two rounds: measured slower at
  // 24 heads, 53 against 42 µs)
  if (mtk >= 16 && heads * 16 * 3 <= slots * 2 && prep_cluster16_ok<T>()) C = 16;
  const int64_t n_cl = std::min(heads, std::max<int64_t>(1, std::llround((double)slots * 2.0 / 3.0 / C)));
  const int64_t n_kv = n_cl * C;
  const int64_t nq_tiles = a.batch * a.Hq * A.mtq;
  const int64_t grid = std::max(n_kv, std::min(slots / C * C, n_kv + (nq_tiles + C - 1) / C * C));
  A.csize = C;
  A.n_kv_ctas = (uint32_t)n_kv;
  A.q_next = reinterpret_cast<uint32_t*>(A.ws.status) + 4;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kPrepThreads);
  cfg.dynamicSmemBytes = PrepSmem::total;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QF2_CUDA_CHECK(cudaLaunchKernelEx(&cfg, sage_prep_kernel<T>, mq, mk, mv, A));
  return QF2_OK;
}

static int launch_attn(const Args& a) {
  const bool varlen = a.cu_q != nullptr;
  const Layout L = make_layout(a.batch, a.Hq, a.Hkv, a.total_q, a.total_k, a.max_q, a.max_k, varlen);
  AttnParams P;
  P.ws = bind_ws(a.workspace, L);
  P.g.cu_q = a.cu_q; P.g.cu_k = a.cu_k; P.g.Sq = a.Sq; P.g.Skv = a.Skv;
  P.g.tiles_q_dense = (a.Sq + kTile - 1) / kTile;
  P.g.tiles_k_dense = (a.Skv + kTile - 1) / kTile;
  P.out = a.out;
  P.os = a.os;
  P.Hq = (int)a.Hq; P.Hkv = (int)a.Hkv;
  P.out_bf16 = a.dtype == QF2_BF16;
  P.D = (int)a.D;
  P.wait_clocks = g_attn_wait_clocks.load(std::memory_order_relaxed);
  P.skip_kv = g_attn_skip_kv.load(std::memory_order_relaxed);
  const int64_t mqt = (a.max_q + kTile - 1) / kTile;
  if (mqt == 0) return QF2_OK;
  static std::atomic<uint64_t> attr_done[3];
  auto kern = a.D == 64 ? sage_attn_kernel<2> : a.D == 96 ? sage_attn_kernel<3> : sage_attn_kernel<4>;
  QF2_CUDA_CHECK(qf2_set_smem_once(kern, AttnSmem::alloc, &attr_done[a.D / 32 - 2]));
  kern<<<dim3((unsigned)(((mqt + 1) / 2) * P.ws.nsplit), (unsigned)a.Hq, (unsigned)a.batch), kAttnThreads,
         AttnSmem::alloc, a.stream>>>(P);
  QF2_LAUNCH_CHECK();
  if (P.ws.nsplit > 1) {
    sage_combine_kernel<<<dim3((unsigned)(mqt * (kTile / 16)), (unsigned)a.Hq, (unsigned)a.batch), 256, 0, a.stream>>>(P);
    QF2_LAUNCH_CHECK();
  }
  return QF2_OK;
}

static int run_attn_only(const Args& a) {
  const int st = validate(a, true);
  if (st != QF2_OK) return st;
  return launch_attn(a);
}

static int run(const Args& a, bool quant_only) {
  int st = validate(a, !quant_only);
  if (st != QF2_OK) return st;
  // the status word and the Q tile counter start every call at zero (stream-ordered,
  // no allocation)
  QF2_CUDA_CHECK(cudaMemsetAsync(a.workspace, 0, 32, a.stream));
  st = (a.dtype == QF2_BF16) ? launch_quant<__nv_bfloat16>(a) : launch_quant<__half>(a);
  if (st != QF2_OK || quant_only) return st;
  return launch_attn(a);
}

}  // namespace sage
}  // namespace qf2

using namespace qf2::sage;

static Strides3 s3(const int64_t* p) { return p ? Strides3{p[0], p[1], p[2]} : Strides3{0, 0, 0}; }
static Strides3 s2v(const int64_t* p) { return p ? Strides3{0, p[1], p[0]} : Strides3{0, 0, 0}; }

extern "C" int64_t qf2_sage_workspace_bytes(int64_t batch, int64_t Hq, int64_t Hkv, int64_t total_q, int64_t total_k,
                                            int64_t max_seqlen_q, int64_t max_seqlen_k, int64_t D) {
  if (!head_dim_ok(D)) return (int64_t)QF2_ERR_SHAPE;
  // dense callers pass total = batch * S; the varlen capacity bound covers both forms
  const Layout L = make_layout(batch, Hq, Hkv, total_q, total_k, max_seqlen_q, max_seqlen_k, true);
  const Layout Ld = make_layout(batch, Hq, Hkv, total_q, total_k, max_seqlen_q, max_seqlen_k, false);
  return std::max(L.off[11], Ld.off[11]);
}

extern "C" int qf2_sage_fault_injection(int64_t wait_limit_us, int skip_kv_tile) {
  // SM clocks per microsecond: the B200's 1965 MHz maximum rounded up, so the bound is at
  // least the requested time
  g_attn_wait_clocks.store(wait_limit_us > 0 ? wait_limit_us * 2000 : qf2::kWaitClocks, std::memory_order_relaxed);
  g_attn_skip_kv.store(skip_kv_tile >= 0 ? skip_kv_tile : -1, std::memory_order_relaxed);
  return QF2_OK;
}

extern "C" int qf2_sage_workspace_layout(int64_t batch, int64_t Hq, int64_t Hkv, int64_t total_q, int64_t total_k,
                                         int64_t max_seqlen_q, int64_t max_seqlen_k, int64_t D, int64_t* offsets) {
  if (!head_dim_ok(D)) return QF2_ERR_SHAPE;
  if (!offsets) return QF2_ERR_ARG;
  // total_q < 0 selects the dense layout (batch * ceil(S / 128) tiles per head)
  const bool varlen = total_q >= 0;
  const Layout L = make_layout(batch, Hq, Hkv, total_q, total_k, max_seqlen_q, max_seqlen_k, varlen);
  for (int i = 0; i < 12; ++i) offsets[i] = L.off[i];
  return QF2_OK;
}

extern "C" int qf2_sageattn(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                            const void* v, const int64_t* v_strides, void* out, const int64_t* out_strides, int64_t B,
                            int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D, float sm_scale, int dtype,
                            void* workspace, int64_t workspace_bytes, qf2_stream_t stream) {
  if (!q_strides || !k_strides || !v_strides || !out_strides) return QF2_ERR_ARG;
  Args a;
  a.q = q; a.k = k; a.v = v; a.out = out;
  a.qs = s3(q_strides); a.ks = s3(k_strides); a.vs = s3(v_strides); a.os = s3(out_strides);
  a.cu_q = nullptr; a.cu_k = nullptr;
  a.batch = B; a.Sq = Sq; a.Skv = Skv; a.total_q = B * Sq; a.total_k = B * Skv; a.max_q = Sq; a.max_k = Skv;
  a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.sm_scale = sm_scale; a.dtype = dtype;
  a.workspace = workspace; a.ws_bytes = workspace_bytes; a.stream = reinterpret_cast<cudaStream_t>(stream);
  return run(a, false);
}

extern "C" int qf2_sageattn_varlen(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                   const void* v, const int64_t* v_strides, void* out, const int64_t* out_strides,
                                   const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int64_t batch,
                                   int64_t total_q, int64_t total_k, int64_t max_seqlen_q, int64_t max_seqlen_k,
                                   int64_t Hq, int64_t Hkv, int64_t D, float sm_scale, int dtype, void* workspace,
                                   int64_t workspace_bytes, qf2_stream_t stream) {
  if (!q_strides || !k_strides || !v_strides || !out_strides || !cu_seqlens_q || !cu_seqlens_k) return QF2_ERR_ARG;
  Args a;
  a.q = q; a.k = k; a.v = v; a.out = out;
  a.qs = s2v(q_strides); a.ks = s2v(k_strides); a.vs = s2v(v_strides); a.os = s2v(out_strides);
  a.cu_q = cu_seqlens_q; a.cu_k = cu_seqlens_k;
  a.batch = batch; a.Sq = 0; a.Skv = 0; a.total_q = total_q; a.total_k = total_k;
  a.max_q = max_seqlen_q; a.max_k = max_seqlen_k;
  a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.sm_scale = sm_scale; a.dtype = dtype;
  a.workspace = workspace; a.ws_bytes = workspace_bytes; a.stream = reinterpret_cast<cudaStream_t>(stream);
  return run(a, false);
}

extern "C" int qf2_sage_quantize(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                 const void* v, const int64_t* v_strides, const int32_t* cu_seqlens_q,
                                 const int32_t* cu_seqlens_k, int64_t batch, int64_t Sq, int64_t Skv, int64_t total_q,
                                 int64_t total_k, int64_t max_seqlen_q, int64_t max_seqlen_k, int64_t Hq, int64_t Hkv,
                                 int64_t D, float sm_scale, int dtype, void* workspace, int64_t workspace_bytes,
                                 qf2_stream_t stream) {
  if (!q_strides || !k_strides || !v_strides) return QF2_ERR_ARG;
  const bool varlen = cu_seqlens_q != nullptr;
  if (varlen != (cu_seqlens_k != nullptr)) return QF2_ERR_ARG;
  Args a;
  a.q = q; a.k = k; a.v = v; a.out = nullptr;
  a.qs = varlen ? s2v(q_strides) : s3(q_strides);
  a.ks = varlen ? s2v(k_strides) : s3(k_strides);
  a.vs = varlen ? s2v(v_strides) : s3(v_strides);
  a.os = Strides3{0, 0, 0};
  a.cu_q = cu_seqlens_q; a.cu_k = cu_seqlens_k;
  a.batch = batch; a.Sq = Sq; a.Skv = Skv;
  a.total_q = varlen ? total_q : batch * Sq; a.total_k = varlen ? total_k : batch * Skv;
  a.max_q = varlen ? max_seqlen_q : Sq; a.max_k = varlen ? max_seqlen_k : Skv;
  a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.sm_scale = sm_scale; a.dtype = dtype;
  a.workspace = workspace; a.ws_bytes = workspace_bytes; a.stream = reinterpret_cast<cudaStream_t>(stream);
  return run(a, true);
}

extern "C" int qf2_sage_attn_quantized(void* out, const int64_t* out_strides, const int32_t* cu_seqlens_q,
                                       const int32_t* cu_seqlens_k, int64_t batch, int64_t Sq, int64_t Skv,
                                       int64_t total_q, int64_t total_k, int64_t max_seqlen_q, int64_t max_seqlen_k,
                                       int64_t Hq, int64_t Hkv, int64_t D, int dtype, void* workspace,
                                       int64_t workspace_bytes, qf2_stream_t stream) {
  if (!out_strides) return QF2_ERR_ARG;
  const bool varlen = cu_seqlens_q != nullptr;
  if (varlen != (cu_seqlens_k != nullptr)) return QF2_ERR_ARG;
  Args a;
  // q/k/v are not read by the attention stage; any aligned non-null value passes validation
  a.q = a.k = a.v = workspace;
  a.out = out;
  a.qs = a.ks = a.vs = Strides3{0, 0, 0};
  a.os = varlen ? s2v(out_strides) : s3(out_strides);
  a.cu_q = cu_seqlens_q; a.cu_k = cu_seqlens_k;
  a.batch = batch; a.Sq = Sq; a.Skv = Skv;
  a.total_q = varlen ? total_q : batch * Sq; a.total_k = varlen ? total_k : batch * Skv;
  a.max_q = varlen ? max_seqlen_q : Sq; a.max_k = varlen ? max_seqlen_k : Skv;
  a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.sm_scale = 1.0f; a.dtype = dtype;
  a.workspace = workspace; a.ws_bytes = workspace_bytes; a.stream = reinterpret_cast<cudaStream_t>(stream);
  return run_attn_only(a);
}

// --------------------------------------------- static-scratch entry point --
// Some callers cannot call cudaMalloc at all: programs that reserve every byte of
// device memory in their own pool at start-up, code that must not take the implicit
// device synchronization an allocation can cause, and thin foreign-language bindings
// that only hold the tensors they pass in.  qf2_sageattn_noalloc serves them by
// keeping the quantized codes and scales in the file-scope array below instead of a
// caller workspace.  Every GPU that loads this library holds the array until the
// process exits.
namespace {
constexpr int64_t kNoAllocScratchBytes = QF2_SAGE_NOALLOC_SCRATCH_BYTES;
__device__ __align__(256) uint8_t g_sage_noalloc_scratch[kNoAllocScratchBytes];

// The array's name is only a host-side stand-in; the device address comes from
// cudaGetSymbolAddress with the target device current.  It is looked up on every call
// (no cache), so a call after cudaDeviceReset, or under another driver context, never
// uses an address from a context that is gone.  The workspace starts at the first
// 1024-byte boundary inside the array.
int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return QF2_ERR_DEVICE;
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_sage_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    qf2_record_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol, "cudaGetSymbolAddress(noalloc scratch)");
    return QF2_ERR_LAUNCH;
  }
  *out = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
  return QF2_OK;
}
}  // namespace

extern "C" int qf2_sageattn_noalloc(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                    const void* v, const int64_t* v_strides, void* out, const int64_t* out_strides,
                                    int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D,
                                    float sm_scale, int dtype, qf2_stream_t stream) {
  if (!head_dim_ok(D)) return QF2_ERR_SHAPE;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq < 0 || Skv < 0) return QF2_ERR_SHAPE;
  const int64_t usable = kNoAllocScratchBytes - 1024;
  const Layout L = make_layout(B, Hq, Hkv, B * Sq, B * Skv, Sq, Skv, false);
  if (L.off[11] > usable) return QF2_ERR_WORKSPACE;
  void* base = nullptr;
  const int st = noalloc_scratch(&base);
  if (st != QF2_OK) return st;
  return qf2_sageattn(q, q_strides, k, k_strides, v, v_strides, out, out_strides, B, Hq, Hkv, Sq, Skv, D, sm_scale,
                      dtype, base, usable, stream);
}

extern "C" int qf2_sageattn_noalloc_status(qf2_stream_t stream) {
  void* base = nullptr;
  const int st = noalloc_scratch(&base);
  if (st != QF2_OK) return st;
  // the status word sits at the start of the workspace, as for the other entry points
  return qf2_workspace_status(base, stream);
}
