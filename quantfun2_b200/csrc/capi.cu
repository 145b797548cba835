// Library-level entry points: version, status strings, device check and the
// workspace status word read-back used after bounded device waits.
#include "qf2_common.cuh"

#include <cstdio>

static thread_local char g_last_error[256] = "";

void qf2_record_cuda_error(cudaError_t e, const char* where) {
  snprintf(g_last_error, sizeof(g_last_error), "%s (%s) at %s", cudaGetErrorName(e), cudaGetErrorString(e), where);
}

extern "C" const char* qf2_last_error(void) { return g_last_error; }

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      return nullptr;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  return encode;
}

static bool make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                      const cuuint64_t* gdim, const cuuint64_t* gstr, const cuuint32_t* bdim,
                      CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tmap_encoder();
  if (encode == nullptr) return false;
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUresult r = encode(map, dtype, rank, const_cast<void*>(base), gdim, gstr, bdim, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool qf2_make_tmap_4d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[4],
                      const uint64_t strides_bytes[3], const uint32_t box[4]) {
  const cuuint64_t gdim[4] = {dims[0], dims[1], dims[2], dims[3]};
  const cuuint64_t gstr[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  const cuuint32_t bdim[4] = {box[0], box[1], box[2], box[3]};
  return make_tmap(map, dtype, 4, base, gdim, gstr, bdim);
}

bool qf2_make_tmap_4d_noswizzle(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[4],
                                const uint64_t strides_bytes[3], const uint32_t box[4]) {
  const cuuint64_t gdim[4] = {dims[0], dims[1], dims[2], dims[3]};
  const cuuint64_t gstr[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  const cuuint32_t bdim[4] = {box[0], box[1], box[2], box[3]};
  return make_tmap(map, dtype, 4, base, gdim, gstr, bdim, CU_TENSOR_MAP_SWIZZLE_NONE);
}

bool qf2_make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[2],
                      uint64_t stride_bytes, const uint32_t box[2]) {
  const cuuint64_t gdim[2] = {dims[0], dims[1]};
  const cuuint64_t gstr[1] = {stride_bytes};
  const cuuint32_t bdim[2] = {box[0], box[1]};
  return make_tmap(map, dtype, 2, base, gdim, gstr, bdim);
}

bool qf2_make_tmap_2d_noswizzle(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[2],
                                uint64_t stride_bytes, const uint32_t box[2]) {
  const cuuint64_t gdim[2] = {dims[0], dims[1]};
  const cuuint64_t gstr[1] = {stride_bytes};
  const cuuint32_t bdim[2] = {box[0], box[1]};
  return make_tmap(map, dtype, 2, base, gdim, gstr, bdim, CU_TENSOR_MAP_SWIZZLE_NONE);
}

bool qf2_make_tmap_2d_sw64(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[2],
                           uint64_t stride_bytes, const uint32_t box[2]) {
  const cuuint64_t gdim[2] = {dims[0], dims[1]};
  const cuuint64_t gstr[1] = {stride_bytes};
  const cuuint32_t bdim[2] = {box[0], box[1]};
  return make_tmap(map, dtype, 2, base, gdim, gstr, bdim, CU_TENSOR_MAP_SWIZZLE_64B);
}

extern "C" const char* qf2_version(void) { return "quantfun2-b200 0.1.0 (sm_100a)"; }

extern "C" const char* qf2_status_string(int status) {
  switch (status) {
    case QF2_OK: return "ok";
    case QF2_ERR_SHAPE: return "unsupported or inconsistent shape";
    case QF2_ERR_DTYPE: return "unsupported dtype";
    case QF2_ERR_LAUNCH: return "CUDA launch or runtime error";
    case QF2_ERR_TIMEOUT: return "a bounded device-side wait timed out";
    case QF2_ERR_ALIGN: return "pointer or stride alignment not met";
    case QF2_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case QF2_ERR_DEVICE: return "current device is not compute capability 10.0 (B200)";
    case QF2_ERR_ARG: return "invalid argument";
  }
  return "unknown status";
}

extern "C" int qf2_device_check(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return QF2_ERR_DEVICE;
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return QF2_ERR_DEVICE;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return QF2_ERR_DEVICE;
  return (major == 10 && minor == 0) ? QF2_OK : QF2_ERR_DEVICE;
}

extern "C" int qf2_workspace_status(void* workspace, qf2_stream_t stream) {
  if (!workspace) return QF2_ERR_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(st) != cudaSuccess) return QF2_ERR_LAUNCH;
  int word = 0;
  if (cudaMemcpy(&word, workspace, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return QF2_ERR_LAUNCH;
  if (word != 0) {
    const int zero = 0;
    cudaMemcpy(workspace, &zero, sizeof(int), cudaMemcpyHostToDevice);
    return word == qf2::kDevBadIndex ? QF2_ERR_ARG : QF2_ERR_TIMEOUT;
  }
  return QF2_OK;
}
