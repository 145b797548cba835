// Sage-style quantized attention for B200 (sm_100a).
//
// Replaces the third-party sageattention calls of the reference:
//   sageattn(q, k, v)                      src/models/flux/attn.py:39-41   (HND)
//   sageattn_varlen(q, k, v, cu_seqlens..) src/models/common/attn.py:109-120
//
// Pipeline (4 launches, all on the caller's stream):
//   1. sage_stats_kernel      per (seq, kv head, 512-token chunk): fp64 channel sums
//                             of K and channel amax of V -> partials
//   2. sage_finalize_kernel   per (seq, kv head): K token mean, V per-channel scale
//   3. sage_quant_kernel      per (128-token tile, head): Q and smoothed K to INT8 per
//                             64-token block, V^T to FP8 e4m3; codes written in the
//                             128-byte-swizzled K-major tile layout tcgen05 reads
//                             directly from shared memory (one 16 KB bulk copy per tile)
//   4. sage_attn_kernel       warp-specialised tcgen05 attention: 1 producer warp
//                             (bulk copies), 1 MMA warp (kind::i8 QK^T and kind::f8f6f4
//                             PV into TMEM), 4 softmax warps (TMEM -> registers, online
//                             base-2 softmax, P -> e4m3 into swizzled smem, O rescale,
//                             epilogue).
#include "qf2_common.cuh"

#include <algorithm>
#include <cmath>
#include <mutex>

namespace qf2 {
namespace sage {

constexpr int kTile = 128;          // tokens per tile (MMA M and N)
constexpr int kHeadDim = 128;       // D
constexpr int kTileBytes = 16384;   // 128 rows x 128 bytes of 8-bit codes
constexpr int kQuantBlock = 64;     // tokens per INT8 scale block
constexpr int kStatChunk = 512;     // tokens per stats partial (one CTA, 32 tokens per thread)
constexpr int kStages = 4;          // K/V smem ring depth
constexpr int kMaxKvTiles = 512;    // k-scale smem capacity (65536 tokens)
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
  double* ksum_part; float* vamax_part;
  int64_t tq, tk;   // tile slots per head
  int64_t nch;      // stats chunks per sequence
};

// ----------------------------------------------------------------- stats --
// grid (nch, Hkv, batch), 256 threads: thread = (row slot 0..15, 8-channel chunk 0..15)
template <typename T>
__global__ void __launch_bounds__(256, 3) sage_stats_kernel(const T* __restrict__ k, Strides3 ks_, const T* __restrict__ v,
                                                         Strides3 vs_, SeqGeom g, int Hkv, Workspace ws) {
  const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const SeqInfo si = seq_k(g, b);
  const int64_t t_begin = (int64_t)chunk * kStatChunk;
  const int slot = threadIdx.x >> 4, c8 = threadIdx.x & 15;
  double sum[8];
  float amax[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) { sum[j] = 0.0; amax[j] = 0.f; }
  if (t_begin < si.len) {
    const int64_t t_end = si.len < t_begin + kStatChunk ? si.len : t_begin + kStatChunk;
    const T* kb = k + (int64_t)b * ks_.b + (int64_t)h * ks_.h + c8 * 8;
    const T* vb = v + (int64_t)b * vs_.b + (int64_t)h * vs_.h + c8 * 8;
    // 4 tokens per batch, the next batch's 8 loads issued before this batch's arithmetic
    constexpr int kBatch = 4, kBatches = kStatChunk / (16 * kBatch);
    uint4 kc[kBatch], vc[kBatch], kn[kBatch], vn[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t t = t_begin + slot + u * 16;
      const bool in = t < t_end;
      kc[u] = in ? *reinterpret_cast<const uint4*>(kb + (si.tok0 + t) * ks_.s) : make_uint4(0, 0, 0, 0);
      vc[u] = in ? *reinterpret_cast<const uint4*>(vb + (si.tok0 + t) * vs_.s) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll 1
    for (int bt = 0; bt < kBatches; ++bt) {
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t t = t_begin + slot + ((bt + 1) * kBatch + u) * 16;
        const bool in = bt + 1 < kBatches && t < t_end;
        kn[u] = in ? *reinterpret_cast<const uint4*>(kb + (si.tok0 + t) * ks_.s) : make_uint4(0, 0, 0, 0);
        vn[u] = in ? *reinterpret_cast<const uint4*>(vb + (si.tok0 + t) * vs_.s) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const T* ke = reinterpret_cast<const T*>(&kc[u]);
        const T* ve = reinterpret_cast<const T*>(&vc[u]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          sum[j] += (double)to_f32(ke[j]);
          amax[j] = fmaxf(amax[j], fabsf(to_f32(ve[j])));
        }
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        kc[u] = kn[u];
        vc[u] = vn[u];
      }
    }
  }
  __shared__ double s_sum[16][kHeadDim];
  __shared__ float s_amax[16][kHeadDim];
#pragma unroll
  for (int j = 0; j < 8; ++j) { s_sum[slot][c8 * 8 + j] = sum[j]; s_amax[slot][c8 * 8 + j] = amax[j]; }
  __syncthreads();
  if (threadIdx.x < kHeadDim) {
    const int c = threadIdx.x;
    double acc = 0.0;
    float am = 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) { acc += s_sum[r][c]; am = fmaxf(am, s_amax[r][c]); }
    const int64_t o = (((int64_t)b * Hkv + h) * ws.nch + chunk) * kHeadDim + c;
    ws.ksum_part[o] = acc;
    ws.vamax_part[o] = am;
  }
}

// -------------------------------------------------------------- finalize --
// grid (Hkv, batch), 128 threads (one per channel)
__global__ void __launch_bounds__(128) sage_finalize_kernel(SeqGeom g, int Hkv, Workspace ws) {
  const int h = blockIdx.x, b = blockIdx.y, c = threadIdx.x;
  const SeqInfo si = seq_k(g, b);
  const int64_t nchunks = (si.len + kStatChunk - 1) / kStatChunk;
  const int64_t base = ((int64_t)b * Hkv + h) * ws.nch * kHeadDim + c;
  double acc = 0.0;
  float am = 0.f;
  for (int64_t i = 0; i < nchunks; ++i) {
    acc += ws.ksum_part[base + i * kHeadDim];
    am = fmaxf(am, ws.vamax_part[base + i * kHeadDim]);
  }
  const int64_t o = ((int64_t)b * Hkv + h) * kHeadDim + c;
  ws.kmean[o] = si.len > 0 ? (float)(acc / (double)si.len) : 0.f;
  ws.vs[o] = am > 0.f ? __fdiv_rn(am, 448.0f) : 1.0f;
  ws.vinv[o] = am > 0.f ? __fdiv_rn(448.0f, am) : 1.0f;
}

// ----------------------------------------------------------------- quant --
// Byte offset of (row, 16-byte chunk) in a 128x128-byte tile stored in the
// 128B-swizzle K-major layout: row r at r*128, chunk c at slot c ^ (r & 7).
QF2_DEV int swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

template <typename T>
QF2_DEV void unpack8(const uint4& raw, float* f) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = to_f32(e[j]);
}

// grid (max tiles, Hq + 2*Hkv, batch), 256 threads.
// Q/K tile: thread = (row slot 0..15, 8-channel chunk 0..15), rows slot + 16*i.
//   code = rint(x * (127 / amax_block)) with x = q * qmul or k - kmean (fp32).
// V tile: thread = (channel pair 0..63, 32-token group 0..3); writes rows of V^T.
//   code = e4m3(v * (448 / amax_channel)).
template <typename T>
__global__ void __launch_bounds__(256, 4) sage_quant_kernel(const T* __restrict__ q, Strides3 qs_, const T* __restrict__ k,
                                                         Strides3 ks_, const T* __restrict__ v, Strides3 vs_, SeqGeom g,
                                                         int Hq, int Hkv, float qmul, Workspace ws) {
  const int tile = blockIdx.x, job = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  __shared__ float s_red[2][8];

  if (job < Hq + Hkv) {
    const bool is_q = job < Hq;
    const int h = is_q ? job : job - Hq;
    const SeqInfo si = is_q ? seq_q(g, b) : seq_k(g, b);
    const int64_t ntiles = (si.len + kTile - 1) / kTile;
    if (tile >= ntiles) return;
    const T* src = is_q ? q : k;
    const Strides3 st = is_q ? qs_ : ks_;
    const int rg = tid >> 4, c8 = tid & 15;
    float sub[8];
    if (is_q) {
#pragma unroll
      for (int j = 0; j < 8; ++j) sub[j] = 0.f;
    } else {
      const float4* km = reinterpret_cast<const float4*>(ws.kmean + ((int64_t)b * Hkv + h) * kHeadDim + c8 * 8);
      const float4 a = km[0], c = km[1];
      sub[0] = a.x; sub[1] = a.y; sub[2] = a.z; sub[3] = a.w; sub[4] = c.x; sub[5] = c.y; sub[6] = c.z; sub[7] = c.w;
    }
    const T* base = src + (int64_t)b * st.b + (int64_t)h * st.h + (si.tok0 + (int64_t)tile * kTile) * st.s + c8 * 8;
    const int valid = (int)min((int64_t)kTile, si.len - (int64_t)tile * kTile);
    uint4 raw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = rg + 16 * i;
      raw[i] = r < valid ? *reinterpret_cast<const uint4*>(base + (int64_t)r * st.s) : make_uint4(0, 0, 0, 0);
    }
    auto xform = [&](float f, int j) { return is_q ? __fmul_rn(f, qmul) : __fsub_rn(f, sub[j]); };
    float am[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (rg + 16 * i < valid) {
        float f[8];
        unpack8<T>(raw[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) am[i >> 2] = fmaxf(am[i >> 2], fabsf(xform(f[j], j)));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      am[0] = fmaxf(am[0], __shfl_xor_sync(0xffffffffu, am[0], o));
      am[1] = fmaxf(am[1], __shfl_xor_sync(0xffffffffu, am[1], o));
    }
    if ((tid & 31) == 0) { s_red[0][tid >> 5] = am[0]; s_red[1][tid >> 5] = am[1]; }
    __syncthreads();
    float bm[2] = {0.f, 0.f};
#pragma unroll
    for (int w = 0; w < 8; ++w) { bm[0] = fmaxf(bm[0], s_red[0][w]); bm[1] = fmaxf(bm[1], s_red[1][w]); }
    const float inv[2] = {bm[0] > 0.f ? __fdiv_rn(127.0f, bm[0]) : 1.0f, bm[1] > 0.f ? __fdiv_rn(127.0f, bm[1]) : 1.0f};
    const int64_t slot = (int64_t)h * (is_q ? ws.tq : ws.tk) + si.tile0 + tile;
    int8_t* dst = (is_q ? ws.qc : ws.kc) + slot * kTileBytes;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = rg + 16 * i;
      uint32_t w[2] = {0u, 0u};
      if (r < valid) {
        float f[8];
        unpack8<T>(raw[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          int c = __float2int_rn(__fmul_rn(xform(f[j], j), inv[i >> 2]));
          c = max(-127, min(127, c));
          w[j >> 2] |= (uint32_t)(c & 0xff) << ((j & 3) * 8);
        }
      }
      *reinterpret_cast<uint2*>(dst + swz(r, c8 >> 1) + (c8 & 1) * 8) = make_uint2(w[0], w[1]);
    }
    if (tid == 0) {
      float* sc = (is_q ? ws.qs : ws.ks) + slot * 4;
      const float s0 = bm[0] > 0.f ? __fdiv_rn(bm[0], 127.0f) : 1.0f;
      const float s1 = bm[1] > 0.f ? __fdiv_rn(bm[1], 127.0f) : 1.0f;
      *reinterpret_cast<float4*>(sc) = make_float4(s0, s1, 0.f, 0.f);
    }
  } else {
    // ---- V: transpose to [d][token] and quantize to e4m3 per channel ----
    const int h = job - Hq - Hkv;
    const SeqInfo si = seq_k(g, b);
    const int64_t ntiles = (si.len + kTile - 1) / kTile;
    if (tile >= ntiles) return;
    const int dp = tid & 63, tg = tid >> 6;  // channel pair, 32-token group
    const float2 inv = *reinterpret_cast<const float2*>(ws.vinv + ((int64_t)b * Hkv + h) * kHeadDim + 2 * dp);
    const int valid = (int)min((int64_t)kTile, si.len - (int64_t)tile * kTile);
    const T* base = v + (int64_t)b * vs_.b + (int64_t)h * vs_.h + (si.tok0 + (int64_t)tile * kTile + tg * 32) * vs_.s +
                    2 * dp;
    uint32_t raw[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
      raw[i] = (tg * 32 + i < valid) ? *reinterpret_cast<const uint32_t*>(base + (int64_t)i * vs_.s) : 0u;
    uint32_t out0[8], out1[8];  // 32 bytes of V^T row per channel
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const T* e0 = reinterpret_cast<const T*>(&raw[i]);
      const T* e1 = reinterpret_cast<const T*>(&raw[i + 1]);
      const uint16_t p0 = f32x2_to_e4m3x2(__fmul_rn(to_f32(e0[0]), inv.x), __fmul_rn(to_f32(e1[0]), inv.x));
      const uint16_t p1 = f32x2_to_e4m3x2(__fmul_rn(to_f32(e0[1]), inv.y), __fmul_rn(to_f32(e1[1]), inv.y));
      if ((i & 2) == 0) {
        out0[i >> 2] = p0;
        out1[i >> 2] = p1;
      } else {
        out0[i >> 2] |= (uint32_t)p0 << 16;
        out1[i >> 2] |= (uint32_t)p1 << 16;
      }
    }
    const int64_t slot = (int64_t)h * ws.tk + si.tile0 + tile;
    uint8_t* dst = ws.vc + slot * kTileBytes;
    const int d0 = 2 * dp, d1 = 2 * dp + 1;
    *reinterpret_cast<uint4*>(dst + swz(d0, tg * 2)) = make_uint4(out0[0], out0[1], out0[2], out0[3]);
    *reinterpret_cast<uint4*>(dst + swz(d0, tg * 2 + 1)) = make_uint4(out0[4], out0[5], out0[6], out0[7]);
    *reinterpret_cast<uint4*>(dst + swz(d1, tg * 2)) = make_uint4(out1[0], out1[1], out1[2], out1[3]);
    *reinterpret_cast<uint4*>(dst + swz(d1, tg * 2 + 1)) = make_uint4(out1[4], out1[5], out1[6], out1[7]);
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
  static constexpr int p = kv + kStages * 2 * kTileBytes;       // one P tile per Q tile
  static constexpr int kscale = p + 2 * kTileBytes;             // up to kMaxKvTiles x 16 B
  static constexpr int bars = kscale + kMaxKvTiles * 16;
  static constexpr int nbars = 1 + 2 * kStages + 2 * 5 + 1;
  static constexpr int misc = bars + nbars * 8;
  static constexpr int total = misc + 64;
  static constexpr int alloc = total + 1024;  // slack for manual 1024-B alignment
};

struct AttnParams {
  Workspace ws;
  SeqGeom g;
  void* out;
  Strides3 os;
  int Hq, Hkv;
  int out_bf16;
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

// fma / add on two packed fp32 lanes (sm_100 f32x2 instructions)
QF2_DEV float2 ffma2(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}

QF2_DEV float2 fadd2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

QF2_DEV float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}


// grid (ceil(max q tiles / 2), Hq, batch)
__global__ void __launch_bounds__(kAttnThreads, 1) sage_attn_kernel(AttnParams P) {
  extern __shared__ uint8_t smem_raw[];
  const int pair = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const SeqInfo sq = seq_q(P.g, b);
  const int64_t nqt = (sq.len + kTile - 1) / kTile;
  const int qt0 = 2 * pair;
  if (qt0 >= nqt) return;
  const int ntile = (qt0 + 1 < nqt) ? 2 : 1;  // Q tiles in this CTA
  const SeqInfo sk = seq_k(P.g, b);
  const int nkt = (int)((sk.len + kTile - 1) / kTile);
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
  uint64_t* bar_o_done = bar_p_full + 2;           // [2 tiles]: PV_t(i) completed
  uint64_t* bar_pp = bar_o_done + 2;              // [2 tiles]: softmax t is far enough into its exp pass
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
      mbar_init(bar_o_done + t, 1);
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
    const bool w = mbar_wait(bar, parity) && (*abort_flag == 0);
    return __all_sync(0xffffffffu, w);
  };

  if (warp < 4) {
    if (warp == 0 && nkt > 0) {
      // ------------------------------------------------------- producer --
      // the whole warp runs the loop (uniform addresses), lane 0 issues the copies
      const int64_t qslot = (int64_t)h * ws.tq + sq.tile0 + qt0;
      const int64_t kslot0 = (int64_t)hk * ws.tk + sk.tile0;
      if (lane == 0) {
        mbar_arrive_expect_tx(bar_q, ntile * kTileBytes + nkt * 16);
        bulk_g2s(sQ, ws.qc + qslot * kTileBytes, ntile * kTileBytes, bar_q);
        bulk_g2s(sKS, ws.ks + kslot0 * 4, nkt * 16, bar_q);
      }
      int issued = 0;
      for (int j = 0; j < nkt; ++j) {
        const int s = j % kStages, r = j / kStages;
        if (!wwait(bar_kv_empty + s, (r & 1) ^ 1)) { if (lane == 0) fail(kDevTimeoutProducer); break; }
        if (lane == 0) {
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
        mbar_wait(bar_q, 0);
        for (int j = issued > kStages ? issued - kStages : 0; j < issued; ++j)
          mbar_wait(bar_kv_full + (j % kStages), (j / kStages) & 1);
      }
    } else if (warp == 1 && nkt > 0) {
      // ------------------------------------------------------------ MMA --
      // converged warp: descriptors are warp-uniform, lane 0 issues and commits
      constexpr uint32_t idesc_qk = make_idesc(2, 1, 1, 0, 0, kTile, kTile);     // s8 x s8 -> s32
      constexpr uint32_t idesc_pv = make_idesc(1, 0, 0, 0, 0, kTile, kHeadDim);  // e4m3 x e4m3 -> f32
      bool ok = wwait(bar_q, 0);
      // Descriptors are built once; per stage / k-step only the 14-bit start-address
      // field moves (16-byte units: a stage is 2048, a 32-byte k-step is 2).
      const uint64_t dQ0 = sdesc_sw128_kmajor(smem_u32(sQ));
      const uint64_t dP0 = sdesc_sw128_kmajor(smem_u32(sP));
      const uint64_t dK0 = sdesc_sw128_kmajor(smem_u32(sKV));
      constexpr uint64_t kTileStep = kTileBytes >> 4, kStageStep = 2 * kTileBytes >> 4;
      auto issue_pv = [&](int i) -> bool {
        const uint64_t dV = dK0 + (uint64_t)(i % kStages) * kStageStep + kTileStep;
        for (int t = 0; t < ntile; ++t) {
          if (!wwait(bar_p_full + t, i & 1)) return false;
          tc_fence_after();
          const uint64_t dP = dP0 + (uint64_t)t * kTileStep;
          if (lane == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_f8f6f4(tmem + 256 + t * 128, dP + 2 * kk, dV + 2 * kk, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
            tc_commit(bar_o_done + t);
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
          if (j > 0 && !wwait(bar_s_empty + t, (j - 1) & 1)) { ok = false; break; }
          tc_fence_after();
          const uint64_t dQ = dQ0 + (uint64_t)t * kTileStep;
          if (lane == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) mma_i8(tmem + t * 128, dQ + 2 * kk, dK + 2 * kk, idesc_qk, kk > 0 ? 1u : 0u);
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
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; ok && j < nkt; ++j) {
      if (!wwait(bar_s_full + t, j & 1)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_s_empty + t);

      // int32 -> fp32 exactly via the 1.5*2^23 magic constant (|s| < 2^22)
      float mf[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) mf[i] = __int_as_float((int)s[i] + kMagicBits);
      const int64_t rem = sk.len - (int64_t)j * kTile;
      if (rem < kTile) {
        // ragged last tile: 0.0 is below every magic-encoded value, so it acts as -inf
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= rem) mf[i] = 0.0f;
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
      // P_fp8 = 2^(x - m_run + kPScaleLog2), x = (mf - magic) * sc: exact subtraction, one fma
      const float bias = m_run - kPScaleLog2;
      const float2 nb = make_float2(-bias, -bias), nmag = make_float2(-kMagic, -kMagic);
      const float2 sc0v = make_float2(sc0, sc0), sc1v = make_float2(sc1, sc1);
      // P_t was last read by PV_t(j-1); its completion also orders the O rescale below
      if (j >= 1 && !wwait(bar_o_done + t, (j - 1) & 1)) { ok = false; break; }
      if (ntile == 2) {  // ping-pong (see the arrive in the exp pass below)
        if (t == 1 && !wwait(bar_pp, j & 1)) { ok = false; break; }
        if (t == 0 && j >= 1 && !wwait(bar_pp + 1, (j - 1) & 1)) { ok = false; break; }
      }
      uint8_t* pdst = sP + t * kTileBytes;
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int chunk = 0; chunk < 8; ++chunk) {
        const float2 scv = chunk < 4 ? sc0v : sc1v;
        uint32_t w[4];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int i0 = chunk * 16 + q4 * 4;
          const float2 x01 = ffma2(fadd2(make_float2(mf[i0], mf[i0 + 1]), nmag), scv, nb);
          const float2 x23 = ffma2(fadd2(make_float2(mf[i0 + 2], mf[i0 + 3]), nmag), scv, nb);
          const float2 p01 = make_float2(fast_exp2(x01.x), fast_exp2(x01.y));
          const float2 p23 = make_float2(fast_exp2(x23.x), fast_exp2(x23.y));
          acc = fadd2(acc, fadd2(p01, p23));
          w[q4] = (uint32_t)f32x2_to_e4m3x2(p01.x, p01.y) | ((uint32_t)f32x2_to_e4m3x2(p23.x, p23.y) << 16);
        }
        *reinterpret_cast<uint4*>(pdst + swz(row, chunk)) = make_uint4(w[0], w[1], w[2], w[3]);
        // ping-pong of the two softmax warpgroups over the SFU: tile 1's exp pass of
        // iteration j starts when tile 0's is three quarters done, tile 0's of j + 1 when
        // tile 1's is (measured: the exp pass of one warpgroup alone does not fill the
        // SFU, two fully overlapped ones leave it idle during the max passes)
        if (ntile == 2 && chunk == 5) {
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_pp + t);
        }
      }
      l_run += acc.x + acc.y;
      if (rescale && j > 0) {
        // O holds sum_{i<j} P_i V_i against the old max (PV(j-1) completed above);
        // PV(j) is only issued after p_full(j) below
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
        if (!wwait(bar_o_done + t, (nkt - 1) & 1)) {
          fail(kDevTimeoutEpilogue);
          ok = false;
        }
        tc_fence_after();
      }
      const float inv_l = (ok && l_run > 0.f) ? 1.0f / l_run : 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
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
        if (r_tok < sq.len) store_row_out(P.out, P.os, P.g.cu_q ? 0 : b, h, sq.tok0 + r_tok, of, P.out_bf16, c * 32);
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
struct Layout {
  int64_t off[12];
  int64_t tq, tk, nch;
};

static int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

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
  L.nch = std::max<int64_t>(1, (max_k + kStatChunk - 1) / kStatChunk);
  int64_t o = 0;
  auto put = [&](int i, int64_t bytes) { L.off[i] = o; o = align_up(o + bytes, 1024); };
  put(0, 256);                                       // status
  put(1, Hq * L.tq * kTileBytes);                    // q codes
  put(2, Hq * L.tq * 16);                            // q scales
  put(3, Hkv * L.tk * kTileBytes);                   // k codes
  put(4, Hkv * L.tk * 16);                           // k scales
  put(5, Hkv * L.tk * kTileBytes);                   // v codes (V^T tiles)
  put(6, batch * Hkv * kHeadDim * 4);                // v scales
  put(7, batch * Hkv * kHeadDim * 4);                // k mean
  put(8, batch * Hkv * kHeadDim * 4);                // v inverse scales (448 / amax)
  put(9, batch * Hkv * L.nch * kHeadDim * 8);        // k sum partials (fp64)
  put(10, batch * Hkv * L.nch * kHeadDim * 4);       // v amax partials
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
  ws.ksum_part = reinterpret_cast<double*>(p + L.off[9]);
  ws.vamax_part = reinterpret_cast<float*>(p + L.off[10]);
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
  if (a.D != kHeadDim) return QF2_ERR_SHAPE;
  if (a.Hq <= 0 || a.Hkv <= 0 || a.Hq % a.Hkv != 0 || a.batch <= 0) return QF2_ERR_SHAPE;
  if (a.max_q < 0 || a.max_k < 0 || a.max_k > (int64_t)kMaxKvTiles * kTile) return QF2_ERR_SHAPE;
  if (a.Hq > 65535 || a.Hq + 2 * a.Hkv > 65535 || a.batch > 65535) return QF2_ERR_SHAPE;
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

template <typename T>
static int launch_quant(const Args& a) {
  const bool varlen = a.cu_q != nullptr;
  const Layout L = make_layout(a.batch, a.Hq, a.Hkv, a.total_q, a.total_k, a.max_q, a.max_k, varlen);
  Workspace ws = bind_ws(a.workspace, L);
  SeqGeom g;
  g.cu_q = a.cu_q; g.cu_k = a.cu_k; g.Sq = a.Sq; g.Skv = a.Skv;
  g.tiles_q_dense = (a.Sq + kTile - 1) / kTile;
  g.tiles_k_dense = (a.Skv + kTile - 1) / kTile;
  const float qmul = (float)((double)a.sm_scale * 1.4426950408889634);
  const T* q = reinterpret_cast<const T*>(a.q);
  const T* k = reinterpret_cast<const T*>(a.k);
  const T* v = reinterpret_cast<const T*>(a.v);
  if (a.max_k > 0) {
    sage_stats_kernel<T><<<dim3((unsigned)L.nch, (unsigned)a.Hkv, (unsigned)a.batch), 256, 0, a.stream>>>(
        k, a.ks, v, a.vs, g, (int)a.Hkv, ws);
    QF2_LAUNCH_CHECK();
  }
  sage_finalize_kernel<<<dim3((unsigned)a.Hkv, (unsigned)a.batch), 128, 0, a.stream>>>(g, (int)a.Hkv, ws);
  QF2_LAUNCH_CHECK();
  const int64_t mt = std::max((a.max_q + kTile - 1) / kTile, (a.max_k + kTile - 1) / kTile);
  if (mt > 0) {
    sage_quant_kernel<T><<<dim3((unsigned)mt, (unsigned)(a.Hq + 2 * a.Hkv), (unsigned)a.batch), 256, 0, a.stream>>>(
        q, a.qs, k, a.ks, v, a.vs, g, (int)a.Hq, (int)a.Hkv, qmul, ws);
    QF2_LAUNCH_CHECK();
  }
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
  const int64_t mqt = (a.max_q + kTile - 1) / kTile;
  if (mqt == 0) return QF2_OK;
  static std::atomic<uint64_t> attr_done{0};
  QF2_CUDA_CHECK(qf2_set_smem_once(sage_attn_kernel, AttnSmem::alloc, &attr_done));
  sage_attn_kernel<<<dim3((unsigned)((mqt + 1) / 2), (unsigned)a.Hq, (unsigned)a.batch), kAttnThreads,
                     AttnSmem::alloc, a.stream>>>(P);
  QF2_LAUNCH_CHECK();
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
  // the status word starts every call at zero (stream-ordered, no allocation)
  QF2_CUDA_CHECK(cudaMemsetAsync(a.workspace, 0, sizeof(int), a.stream));
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
  if (D != kHeadDim) return (int64_t)QF2_ERR_SHAPE;
  // dense callers pass total = batch * S; the varlen capacity bound covers both forms
  const Layout L = make_layout(batch, Hq, Hkv, total_q, total_k, max_seqlen_q, max_seqlen_k, true);
  const Layout Ld = make_layout(batch, Hq, Hkv, total_q, total_k, max_seqlen_q, max_seqlen_k, false);
  return std::max(L.off[11], Ld.off[11]);
}

extern "C" int qf2_sage_workspace_layout(int64_t batch, int64_t Hq, int64_t Hkv, int64_t total_q, int64_t total_k,
                                         int64_t max_seqlen_q, int64_t max_seqlen_k, int64_t D, int64_t* offsets) {
  if (D != kHeadDim) return QF2_ERR_SHAPE;
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

std::mutex g_noalloc_mu;
constexpr int kMaxDevices = 64;
void* g_noalloc_addr[kMaxDevices] = {};

// The array's name is only a host-side stand-in; the device address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return QF2_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_sage_noalloc_scratch) != cudaSuccess || p == nullptr) return QF2_ERR_LAUNCH;
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return QF2_OK;
}
}  // namespace

extern "C" int qf2_sageattn_noalloc(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                    const void* v, const int64_t* v_strides, void* out, const int64_t* out_strides,
                                    int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Skv, int64_t D,
                                    float sm_scale, int dtype, qf2_stream_t stream) {
  if (D != kHeadDim) return QF2_ERR_SHAPE;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq < 0 || Skv < 0) return QF2_ERR_SHAPE;
  // the workspace starts at the first 1024-byte boundary inside the array
  const int64_t usable = kNoAllocScratchBytes - 1024;
  const Layout L = make_layout(B, Hq, Hkv, B * Sq, B * Skv, Sq, Skv, false);
  if (L.off[11] > usable) return QF2_ERR_WORKSPACE;
  void* base = nullptr;
  const int st = noalloc_scratch(&base);
  if (st != QF2_OK) return st;
  const uintptr_t a = (reinterpret_cast<uintptr_t>(base) + 1023) & ~uintptr_t(1023);
  return qf2_sageattn(q, q_strides, k, k_strides, v, v_strides, out, out_strides, B, Hq, Hkv, Sq, Skv, D, sm_scale,
                      dtype, reinterpret_cast<void*>(a), usable, stream);
}
