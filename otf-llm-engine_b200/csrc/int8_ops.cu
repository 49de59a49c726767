// INT8 shared-vocabulary LM head and embedding gather for B200 (sm_100a).
//
// The head streams int8 weight rows straight into the A operand of the integer
// tensor pipe (m16n8k32, s8 x s8 -> s32): no per-weight decode at all.  The
// activation is 16-bit fixed point per 16-value block, split into two s8 limbs in
// MMA columns 2t (hi) and 2t+1 (lo), so each thread's accumulator fragment holds
// its own block.  Replaces QuantizedLinearHead.forward
// (otf_llm/symmetric_2bit_engine.py:75-91) and QuantizedEmbedding.forward (:41-47).
#include <algorithm>

#include "otf_common.cuh"

namespace otf {

int set_cuda_error(cudaError_t e);  // capi.cu
int check_device();                 // capi.cu

constexpr int kHeadWarps = 8;
constexpr int kHeadSL = 24;  // bytes per (block, limb): 16 data + 8 pad (conflict-free lane map)
constexpr int kHeadSB = 48;  // bytes per 16-value block

struct HeadArgs {
  const uint16_t* x;
  const int8_t* w;
  int64_t ldw;
  const uint16_t* scales;
  float* out;
  int V, D;
};

__host__ __device__ inline int64_t head_smem_bytes(int D) {
  const int nb = D / 16;
  return align_up(align_up((int64_t)nb * kHeadSB, 16) + (int64_t)nb * 4, 16) + 16;
}

__device__ __forceinline__ float head_finish(float v, float s) {
  float r = v * s;
  if (isnan(r)) r = 0.0f;
  return fminf(fmaxf(r, -65504.0f), 65504.0f);
}

__global__ void __launch_bounds__(kHeadWarps * 32) k_i8_head_imma(const HeadArgs a) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = a.D / 16;
  const int nch = ceil_div(nb, 4);
  uint8_t* tbl = smem;
  float* metaF = reinterpret_cast<float*>(smem + align_up((int64_t)nb * kHeadSB, 16));
  uint8_t* zblk = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(metaF + nb), 16));

  // Activation table for the whole D (every CTA builds its own; rows amortise it).
  for (int it = threadIdx.x; it < 2 * nb; it += blockDim.x) {
    const int b = it >> 1, limb = it & 1;
    float xv[16];
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      xv[i] = h2f(a.x[b * 16 + i]);
      mx = fmaxf(mx, fabsf(xv[i]));
    }
    const int E = fixed_point_exp(mx);
    const float sc = ldexpf(1.0f, E);
    uint32_t wd[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      int hi, lo;
      split_limbs(__float2int_rn(__fmul_rn(xv[i], sc)), hi, lo);
      wd[i >> 2] |= (uint32_t)((limb == 0 ? hi : lo) & 0xff) << (8 * (i & 3));
    }
    uint2* dst = reinterpret_cast<uint2*>(tbl + b * kHeadSB + limb * kHeadSL);
    dst[0] = make_uint2(wd[0], wd[1]);
    dst[1] = make_uint2(wd[2], wd[3]);
    if (limb == 0) metaF[b] = ldexpf(1.0f, -E);
  }
  if (threadIdx.x < 4) reinterpret_cast<uint32_t*>(zblk)[threadIdx.x] = 0u;
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int ntiles = ceil_div(a.V, 16);
  for (int tile = blockIdx.x * kHeadWarps + warp; tile < ntiles; tile += gridDim.x * kHeadWarps) {
    const int rg = tile * 16 + g, rg8 = rg + 8;
    const bool vg = rg < a.V, vg8 = rg8 < a.V;
    const int8_t* pg = a.w + (int64_t)(vg ? rg : 0) * a.ldw;
    const int8_t* pg8 = a.w + (int64_t)(vg8 ? rg8 : 0) * a.ldw;
    float acc0 = 0.0f, acc1 = 0.0f;
    uint4 cw = make_uint4(0, 0, 0, 0), cw8 = make_uint4(0, 0, 0, 0);
    {
      const bool act = t < nb;
      ld_stream16_pred(cw, pg + 16 * t, act && vg);
      ld_stream16_pred(cw8, pg8 + 16 * t, act && vg8);
    }
    for (int c = 0; c < nch; ++c) {
      const int blk = 4 * c + t;
      const bool act = blk < nb;
      uint4 nw = make_uint4(0, 0, 0, 0), nw8 = make_uint4(0, 0, 0, 0);
      {
        const int blk2 = blk + 4;
        const bool act2 = blk2 < nb;
        ld_stream16_pred(nw, pg + 16 * (int64_t)blk2, act2 && vg);
        ld_stream16_pred(nw8, pg8 + 16 * (int64_t)blk2, act2 && vg8);
      }
      const int bblk = 4 * c + (g >> 1);
      const uint8_t* bp = ((g >> 1) == t && bblk < nb) ? (tbl + bblk * kHeadSB + (g & 1) * kHeadSL) : zblk;
      const uint2 b01 = *reinterpret_cast<const uint2*>(bp);
      const uint2 b23 = *reinterpret_cast<const uint2*>(bp + 8);
      int C[4] = {0, 0, 0, 0};
      mma_s8s8(C, cw.x, cw8.x, cw.y, cw8.y, b01.x, b01.y);
      mma_s8s8(C, cw.z, cw8.z, cw.w, cw8.w, b23.x, b23.y);
      if (act) {
        const float F = metaF[blk];
        acc0 = fmaf((float)(256 * C[0] + C[1]), F, acc0);
        acc1 = fmaf((float)(256 * C[2] + C[3]), F, acc1);
      }
      cw = nw;
      cw8 = nw8;
    }
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    if (t == 0) {
      if (vg) a.out[rg] = head_finish(acc0, h2f(a.scales[rg]));
      if (vg8) a.out[rg8] = head_finish(acc1, h2f(a.scales[rg8]));
    }
  }
}

// Portable head for any D / stride: one warp per vocabulary row.
__global__ void __launch_bounds__(256) k_i8_head_generic(const HeadArgs a) {
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= a.V) return;
  float acc = 0.0f;
  for (int d = lane; d < a.D; d += 32) acc = fmaf(h2f(a.x[d]), (float)a.w[(int64_t)row * a.ldw + d], acc);
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
  if (lane == 0) a.out[row] = head_finish(acc, h2f(a.scales[row]));
}

__global__ void k_i8_embed(const int64_t* ids, int n, const int8_t* w, int64_t ldw, const uint16_t* scales,
                           uint16_t* out, int64_t ldo, int64_t V, int D, int32_t* bad) {
  pdl_trigger();
  pdl_wait();
  const int tok = blockIdx.x;
  if (tok >= n) return;
  const int64_t id = ids[tok];
  uint16_t* o = out + (int64_t)tok * ldo;
  if (id < 0 || id >= V) {
    for (int d = threadIdx.x; d < D; d += blockDim.x) o[d] = 0;
    if (bad && threadIdx.x == 0) *bad = 1;
    return;
  }
  const __half s = __ushort_as_half(scales[id]);
  const int8_t* wr = w + id * ldw;
  for (int d = threadIdx.x; d < D; d += blockDim.x)
    o[d] = __half_as_ushort(__hmul(__int2half_rn((int)wr[d]), s));
}

}  // namespace otf

using namespace otf;

extern "C" OTF_API int otf_i8_head(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const void* scales,
                                   float* logits, int64_t ldl, int64_t M, int64_t V, int64_t D, void* stream) {
  if (!x || !w || !scales || !logits || M <= 0 || V <= 0 || D <= 0) return OTF_ERR_INVALID;
  if (ldx < D || ldw < D || ldl < V) return OTF_ERR_INVALID;
  if (V > INT32_MAX / 2 || D > (1 << 20)) return OTF_ERR_UNSUPPORTED;
  int st = check_device();
  if (st != OTF_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool fast = D % 16 == 0 && ldw % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
                    head_smem_bytes((int)D) <= 200 * 1024;
  if (fast) {
    static thread_local int configured_dev[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !configured_dev[dev]) {
      cudaError_t e = cudaFuncSetAttribute(k_i8_head_imma, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      if (e != cudaSuccess) return set_cuda_error(e);
      configured_dev[dev] = 1;
    }
  }
  int sms = 148;
  for (int64_t m = 0; m < M; ++m) {
    HeadArgs a;
    a.x = static_cast<const uint16_t*>(x) + m * ldx;
    a.w = w;
    a.ldw = ldw;
    a.scales = static_cast<const uint16_t*>(scales);
    a.out = logits + m * ldl;
    a.V = (int)V;
    a.D = (int)D;

    cudaError_t e = fast ? launch_pdl(k_i8_head_imma, dim3(std::max(1, std::min(ceil_div(ceil_div((int)V, 16), kHeadWarps),
                                                                               sms * 2))),
                                      dim3(kHeadWarps * 32), (size_t)head_smem_bytes((int)D), s, 1u, a)
                         : launch_pdl(k_i8_head_generic, dim3(ceil_div((int)V, 8)), dim3(256), 0, s, 1u, a);
    if (e != cudaSuccess) return set_cuda_error(e);
  }
  return OTF_OK;
}

extern "C" OTF_API int otf_i8_embed(const int64_t* ids, int64_t n, const int8_t* w, int64_t ldw, const void* scales,
                                    void* out, int64_t ldo, int64_t V, int64_t D, int32_t* bad_ids, void* stream) {
  if (!ids || !w || !scales || !out || n < 0 || V <= 0 || D <= 0 || ldw < D || ldo < D) return OTF_ERR_INVALID;
  if (n == 0) return OTF_OK;
  if (n > INT32_MAX || D > INT32_MAX) return OTF_ERR_UNSUPPORTED;
  int st = check_device();
  if (st != OTF_OK) return st;
  return set_cuda_error(launch_pdl(k_i8_embed, dim3((unsigned)n), dim3(128), 0, static_cast<cudaStream_t>(stream), 1u,
                                   ids, (int)n, w, ldw, static_cast<const uint16_t*>(scales),
                                   static_cast<uint16_t*>(out), ldo, V, (int)D, bad_ids));
}
