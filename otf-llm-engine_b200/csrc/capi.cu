// Library-wide C ABI pieces: version, status strings, error bookkeeping, device check.
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
