// Library-wide C ABI pieces: version, status strings, error bookkeeping, device check, and
// the 2-D tensor-map encoder the TMA-fed kernels share.
#include <cuda.h>

#include "otf_common.cuh"

namespace otf {

static thread_local int g_last_cuda_error = 0;

int set_cuda_error(cudaError_t e) {
  if (e == cudaSuccess) return OTF_OK;
  g_last_cuda_error = (int)e;
  return OTF_ERR_CUDA;
}

// The kernels are built for sm_100a only; refuse other devices up front
// instead of failing at launch with "no kernel image".
int check_device() {
  static thread_local int cached[64] = {};  // 0 unknown, 1 ok, 2 bad
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e);
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev] == 1 ? OTF_OK : OTF_ERR_DEVICE;
  int major = 0, minor = 0;
  e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e != cudaSuccess) return set_cuda_error(e);
  e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (e != cudaSuccess) return set_cuda_error(e);
  const bool ok = (major == 10 && minor == 0);
  if (dev >= 0 && dev < 64) cached[dev] = ok ? 1 : 2;
  return ok ? OTF_OK : OTF_ERR_DEVICE;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// A 2-D tiled tensor map over a row-major array of `rows` rows of `inner` elements of
// `elem_bytes` bytes, rows `row_bytes` apart, copied in boxes of box_inner x box_rows;
// reads past either extent come back as zeros.  cuTensorMapEncodeTiled is reached through
// the runtime's driver entry point, so the library does not link libcuda.  `map` points at
// a CUtensorMap (64-byte aligned, 128 bytes).
bool encode_tiled_2d(void* map, int elem_bytes, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                     uint32_t box_inner, uint32_t box_rows, bool swizzle128) {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    cudaGetLastError();
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  if (!fn) return false;
  const CUtensorMapDataType dt = elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_UINT32;
  const cuuint32_t es[2] = {1, 1};
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  return fn(static_cast<CUtensorMap*>(map), dt, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace otf

extern "C" OTF_API int otf_version(void) { return 100; }

extern "C" OTF_API const char* otf_status_string(int status) {
  switch (status) {
    case OTF_OK: return "ok";
    case OTF_ERR_INVALID: return "invalid argument (pointer, size, stride or alignment)";
    case OTF_ERR_UNSUPPORTED: return "unsupported shape or codebook";
    case OTF_ERR_CUDA: return "CUDA runtime error";
    case OTF_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    default: return "unknown status";
  }
}

extern "C" OTF_API int otf_last_cuda_error(void) { return otf::g_last_cuda_error; }
