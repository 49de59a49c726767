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

// The same op for rows of K = 8k halves on 16-byte boundaries (every Llama width): thread t
// holds the row's 16-byte pieces t, t + 256, ... (PER of them) in registers, all requested at
// once, and the weight's pieces are requested before the dependency wait, so a row costs one
// memory round trip instead of one per strided element.
template <int PER>
__global__ void __launch_bounds__(256) k_rmsnorm_v(const uint16_t* x, int64_t ldx, const uint16_t* w, float eps,
                                                   uint16_t* out, int64_t ldo, int K) {
  pdl_trigger();
  __shared__ float red[8];
  const int tid = threadIdx.x, nv = K >> 3;
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  uint4 wv[PER], xv[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int v = tid + i * 256;
    wv[i] = (w && v < nv) ? __ldg(reinterpret_cast<const uint4*>(w) + v) : z4;
  }
  pdl_wait();
  const uint4* xr = reinterpret_cast<const uint4*>(x + blockIdx.x * ldx);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int v = tid + i * 256;
    xv[i] = v < nv ? __ldg(xr + v) : z4;
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const __half2* h = reinterpret_cast<const __half2*>(&xv[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)K + eps);
  uint4* orow = reinterpret_cast<uint4*>(out + blockIdx.x * ldo);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int v = tid + i * 256;
    if (v >= nv) break;
    __half* e = reinterpret_cast<__half*>(&xv[i]);
    const __half* wh = reinterpret_cast<const __half*>(&wv[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      __half y = __float2half_rn(__half2float(e[j]) * r);
      if (w) y = __hmul(wh[j], y);
      e[j] = y;
    }
    orow[v] = xv[i];
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

// The same op on 16-byte pieces (n a multiple of 8, 16-byte aligned vectors): one piece of g
// and u per thread, both requested at once.
__global__ void k_silu_mul_v(const uint4* __restrict__ g, const uint4* __restrict__ u, uint4* __restrict__ out,
                             int64_t nv) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    uint4 gv = __ldg(g + i);
    const uint4 uv = __ldg(u + i);
    __half* e = reinterpret_cast<__half*>(&gv);
    const __half* uh = reinterpret_cast<const __half*>(&uv);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x = __half2float(e[j]);
      e[j] = __hmul(__float2half_rn(x / (1.0f + expf(-x))), uh[j]);
    }
    out[i] = gv;
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint16_t* xp = static_cast<const uint16_t*>(x);
  const uint16_t* wp = static_cast<const uint16_t*>(w);
  uint16_t* op = static_cast<uint16_t*>(out);
  const bool vec = K % 8 == 0 && ldx % 8 == 0 && ldo % 8 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(out) % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0;
  if (vec && K <= 2048)
    return set_cuda_error(launch_pdl(k_rmsnorm_v<1>, dim3((unsigned)M), dim3(256), 0, s, 1u, xp, ldx, wp, eps, op, ldo, (int)K));
  if (vec && K <= 4096)
    return set_cuda_error(launch_pdl(k_rmsnorm_v<2>, dim3((unsigned)M), dim3(256), 0, s, 1u, xp, ldx, wp, eps, op, ldo, (int)K));
  if (vec && K <= 8192)
    return set_cuda_error(launch_pdl(k_rmsnorm_v<4>, dim3((unsigned)M), dim3(256), 0, s, 1u, xp, ldx, wp, eps, op, ldo, (int)K));
  if (vec && K <= 16384)
    return set_cuda_error(launch_pdl(k_rmsnorm_v<8>, dim3((unsigned)M), dim3(256), 0, s, 1u, xp, ldx, wp, eps, op, ldo, (int)K));
  return set_cuda_error(launch_pdl(k_rmsnorm, dim3((unsigned)M), dim3(256), 0, s, 1u, xp, ldx, wp, eps, op, ldo, (int)K));
}

extern "C" OTF_API int otf_silu_mul(const void* g, const void* u, void* out, int64_t n, void* stream) {
  if (!g || !u || !out || n < 0) return OTF_ERR_INVALID;
  if (n == 0) return OTF_OK;
  int st = check_device();
  if (st != OTF_OK) return st;
  if (n % 8 == 0 && (reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(u) | reinterpret_cast<uintptr_t>(out)) % 16 == 0) {
    const int64_t nv = n / 8;
    const int vblocks = (int)std::min<int64_t>((nv + 255) / 256, 148 * 8);
    return set_cuda_error(launch_pdl(k_silu_mul_v, dim3(vblocks), dim3(256), 0, static_cast<cudaStream_t>(stream), 1u,
                                     static_cast<const uint4*>(g), static_cast<const uint4*>(u),
                                     static_cast<uint4*>(out), nv));
  }
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
  return set_cuda_error(launch_pdl(k_silu_mul, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream), 1u,
                                   static_cast<const uint16_t*>(g), static_cast<const uint16_t*>(u),
                                   static_cast<uint16_t*>(out), n));
}
