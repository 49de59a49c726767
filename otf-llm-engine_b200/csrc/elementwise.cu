// Small fp16 decoder-step ops around the 2-bit linears: Llama RMSNorm and SiLU gate.
#include <algorithm>

#include "otf_common.cuh"

namespace otf {

int set_cuda_error(cudaError_t e);  // capi.cu
int check_device();                 // capi.cu

// One CTA per row: fp32 sum of squares, then out = w * fp16(x * rsqrt(mean + eps)).
__global__ void __launch_bounds__(256) k_rmsnorm(const uint16_t* x, int64_t ldx, const uint16_t* w, float eps,
                                                 uint16_t* out, int64_t ldo, int K) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[8];
  const uint16_t* xr = x + blockIdx.x * ldx;
  uint16_t* orow = out + blockIdx.x * ldo;
  float ss = 0.0f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = h2f(xr[k]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)K + eps);
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    __half v = __float2half_rn(h2f(xr[k]) * r);
    if (w) v = __hmul(__ushort_as_half(w[k]), v);
    orow[k] = __half_as_ushort(v);
  }
}

__global__ void k_silu_mul(const uint16_t* g, const uint16_t* u, uint16_t* out, int64_t n) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float gv = h2f(g[i]);
    const __half s = __float2half_rn(gv / (1.0f + expf(-gv)));
    out[i] = __half_as_ushort(__hmul(s, __ushort_as_half(u[i])));
  }
}

}  // namespace otf

using namespace otf;

extern "C" OTF_API int otf_rmsnorm(const void* x, int64_t ldx, const void* w, float eps, void* out, int64_t ldo,
                                   int64_t M, int64_t K, void* stream) {
  if (!x || !out || M <= 0 || K <= 0 || ldx < K || ldo < K) return OTF_ERR_INVALID;
  if (M > INT32_MAX || K > INT32_MAX) return OTF_ERR_UNSUPPORTED;
  int st = check_device();
  if (st != OTF_OK) return st;
  return set_cuda_error(launch_pdl(k_rmsnorm, dim3((unsigned)M), dim3(256), 0, static_cast<cudaStream_t>(stream), 1u,
                                   static_cast<const uint16_t*>(x), ldx, static_cast<const uint16_t*>(w), eps,
                                   static_cast<uint16_t*>(out), ldo, (int)K));
}

extern "C" OTF_API int otf_silu_mul(const void* g, const void* u, void* out, int64_t n, void* stream) {
  if (!g || !u || !out || n < 0) return OTF_ERR_INVALID;
  if (n == 0) return OTF_OK;
  int st = check_device();
  if (st != OTF_OK) return st;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
  return set_cuda_error(launch_pdl(k_silu_mul, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream), 1u,
                                   static_cast<const uint16_t*>(g), static_cast<const uint16_t*>(u),
                                   static_cast<uint16_t*>(out), n));
}
