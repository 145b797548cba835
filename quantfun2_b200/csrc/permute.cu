// Chunk permutation copy (sm_100a): the layout changes around the head-parallel
// (Ulysses) all-to-all of the multi-GPU DiT step.  The reference runs on one GPU and has
// no counterpart; this replaces torch permute copies, which ran at ~1.1 TB/s on these
// six-dimensional views.
//
// Chunks of up to 4 KB go to copy_small_chunks_kernel (a warp per run of chunks); larger
// ones to copy_chunks_kernel (a CTA per 16 KB segment).
//
// A copy of n = d0*d1*d2*d3 chunks of `chunk` bytes: chunk (i0, i1, i2, i3) (i3 fastest)
// moves from src + sum_k i_k * src_stride[k] to dst + sum_k i_k * dst_stride[k].  Each
// CTA copies one 16 KB segment of one chunk with 16-byte vectors (4 per thread), so
// small chunks (a few heads of one token) and large ones (whole shards) both fill the
// GPU; the chunk's digits are decoded once per CTA.
#include "qf2_common.cuh"

#include <algorithm>

namespace qf2 {
namespace perm {

constexpr int kThreads = 256;
constexpr int kVecPerThread = 4;
constexpr int64_t kSegBytes = (int64_t)kThreads * kVecPerThread * 16;  // 16 KB

struct ChunkArgs {
  const uint8_t* src;
  uint8_t* dst;
  int64_t chunk;  // bytes per chunk (multiple of 16)
  int64_t segs;   // segments per chunk
  int64_t d[4];
  int64_t ss[4], ds[4];
};

__global__ void __launch_bounds__(kThreads) copy_chunks_kernel(ChunkArgs A) {
  const int64_t blk = blockIdx.x;
  const int64_t c = blk / A.segs, seg = blk - c * A.segs;
  int64_t rem = c, so = 0, dof = 0;
#pragma unroll
  for (int k = 3; k >= 0; --k) {
    const int64_t q = rem / A.d[k];
    const int64_t i = rem - q * A.d[k];
    so += i * A.ss[k];
    dof += i * A.ds[k];
    rem = q;
  }
  const uint4* s = reinterpret_cast<const uint4*>(A.src + so);
  uint4* d = reinterpret_cast<uint4*>(A.dst + dof);
  const int64_t nv = A.chunk >> 4;
  const int64_t v0 = seg * (kSegBytes >> 4) + threadIdx.x;
  uint4 r[kVecPerThread];
#pragma unroll
  for (int u = 0; u < kVecPerThread; ++u) {
    const int64_t v = v0 + u * kThreads;
    if (v < nv) r[u] = s[v];
  }
#pragma unroll
  for (int u = 0; u < kVecPerThread; ++u) {
    const int64_t v = v0 + u * kThreads;
    if (v < nv) d[v] = r[u];
  }
}

// Small chunks (at most kSmallMax bytes: a few heads of one token): a warp walks `per`
// consecutive chunks (4 to 16: enough warps for a few waves over the SMs, so copies of a
// few MB are not left to a fraction of the GPU), kUnroll at a time -- their addresses are
// decoded once per chunk (32-bit digit division), the lanes stride over the 16-byte
// vectors, and the loads of the kUnroll chunks are issued before their stores.
constexpr int64_t kSmallMax = 4096;
constexpr int kChunksPerWarpMax = 16;
constexpr int kUnroll = 4;

struct SmallArgs {
  const uint8_t* src;
  uint8_t* dst;
  uint32_t nv;     // 16-byte vectors per chunk
  uint32_t n;      // chunks
  uint32_t per;    // chunks per warp (a multiple of kUnroll)
  uint32_t d[4];
  int64_t ss[4], ds[4];
};

QF2_DEV void chunk_offsets(const SmallArgs& A, uint32_t c, int64_t& so, int64_t& dof) {
  so = 0;
  dof = 0;
#pragma unroll
  for (int k = 3; k >= 0; --k) {
    const uint32_t q = c / A.d[k];
    const uint32_t i = c - q * A.d[k];
    so += (int64_t)i * A.ss[k];
    dof += (int64_t)i * A.ds[k];
    c = q;
  }
}

__global__ void __launch_bounds__(kThreads) copy_small_chunks_kernel(SmallArgs A) {
  const int lane = threadIdx.x & 31;
  const uint32_t c0 = (blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5)) * A.per;
  for (uint32_t cb = c0; cb < c0 + A.per && cb < A.n; cb += kUnroll) {
    const uint4* s[kUnroll];
    uint4* d[kUnroll];
    bool live[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      live[u] = cb + u < A.n && cb + u < c0 + A.per;
      int64_t so = 0, dof = 0;
      if (live[u]) chunk_offsets(A, cb + u, so, dof);
      s[u] = reinterpret_cast<const uint4*>(A.src + so);
      d[u] = reinterpret_cast<uint4*>(A.dst + dof);
    }
    for (uint32_t v = lane; v < A.nv; v += 32) {
      uint4 r[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (live[u]) r[u] = s[u][v];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (live[u]) d[u][v] = r[u];
    }
  }
}

}  // namespace perm
}  // namespace qf2

using namespace qf2::perm;

extern "C" int qf2_copy_chunks(void* dst, const void* src, int64_t chunk_bytes, const int64_t* dims,
                               const int64_t* src_strides, const int64_t* dst_strides, qf2_stream_t stream) {
  if (!dst || !src || !dims || !src_strides || !dst_strides) return QF2_ERR_ARG;
  if (chunk_bytes <= 0 || (chunk_bytes & 15)) return QF2_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(dst) & 15) || (reinterpret_cast<uintptr_t>(src) & 15)) return QF2_ERR_ALIGN;
  ChunkArgs A;
  A.src = reinterpret_cast<const uint8_t*>(src);
  A.dst = reinterpret_cast<uint8_t*>(dst);
  A.chunk = chunk_bytes;
  A.segs = (chunk_bytes + kSegBytes - 1) / kSegBytes;
  int64_t n = 1;
  for (int k = 0; k < 4; ++k) {
    if (dims[k] <= 0) return dims[k] == 0 ? QF2_OK : QF2_ERR_SHAPE;
    if ((src_strides[k] & 15) || (dst_strides[k] & 15)) return QF2_ERR_ALIGN;
    A.d[k] = dims[k];
    A.ss[k] = src_strides[k];
    A.ds[k] = dst_strides[k];
    n *= dims[k];
  }
  if (chunk_bytes <= kSmallMax && n < 0x7fffffffll) {
    SmallArgs S;
    S.src = A.src;
    S.dst = A.dst;
    S.nv = (uint32_t)(chunk_bytes >> 4);
    S.n = (uint32_t)n;
    for (int k = 0; k < 4; ++k) {
      S.d[k] = (uint32_t)A.d[k];
      S.ss[k] = A.ss[k];
      S.ds[k] = A.ds[k];
    }
    // chunks per warp: 16, or fewer (down to kUnroll) until there are ~4 warps' worth of
    // work per resident warp slot (148 SMs x 64 warps)
    int sms = 148;
    QF2_CUDA_CHECK(qf2_sm_count(&sms));
    const int64_t want_warps = (int64_t)sms * 64 * 4;
    int64_t per = (n + want_warps - 1) / want_warps;
    per = std::min<int64_t>(kChunksPerWarpMax, std::max<int64_t>(kUnroll, (per + kUnroll - 1) / kUnroll * kUnroll));
    S.per = (uint32_t)per;
    const int64_t per_cta = (int64_t)(kThreads / 32) * per;
    copy_small_chunks_kernel<<<(unsigned)((n + per_cta - 1) / per_cta), kThreads, 0,
                               reinterpret_cast<cudaStream_t>(stream)>>>(S);
    QF2_LAUNCH_CHECK();
    return QF2_OK;
  }
  const int64_t blocks = n * A.segs;
  if (blocks > 2147483647ll) return QF2_ERR_SHAPE;
  copy_chunks_kernel<<<(unsigned)blocks, kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(A);
  QF2_LAUNCH_CHECK();
  return QF2_OK;
}
