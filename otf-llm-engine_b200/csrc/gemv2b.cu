// 2-bit quantized linear layer for B200 (sm_100a): the decode GEMV and its portable companion.
//
// The decode kernel (k_gemv2b) runs the code/activation dot products on the
// integer tensor pipe with legacy warp MMA (m16n8k32, u8 x s8 -> s32):
//
//  * A operand = the packed code words themselves, masked in place.  A symmetric
//    (more generally "affine") codebook satisfies c(q) = c0 + (c1-c0)*l + (c2-c0)*h
//    for q = 2h + l, so every code contributes through its two bits.  One AND with
//    0x01010101<<2j keeps the l bit of code j of each byte (value l*4^j), one AND with
//    0x02020202<<2j keeps the h bit (value 2h*4^j).  Half an ALU op per weight, no shifts.
//  * B operand = the activation as 16-bit fixed point per 16W-code block, split into
//    two s8 limbs (hi, lo).  MMA column n = 2*t + limb, so each lane quad owns one
//    block and each thread's accumulator fragment holds its own block's hi/lo sums.
//  * Each class j (bit pair position) accumulates into its own int32 fragment; the
//    flush recombines 64*C0 + 16*C1 + 4*C2 + C3 (exact) and 256*hi + lo, converts once
//    and applies 2^-E, the group scale, c0*sum(x) and the optional zero point.
//
// Work split: persistent CTAs walk 16-row tiles; warp w of every CTA owns the same
// contiguous K slice (its chunks of 4 blocks) for every tile, so it quantises only its
// own slice of the activation table, once.  Each warp streams its (tile, chunk) items
// through a 4-deep register ring of code words and scales, folds its share of the fp16
// outlier anchors into its partial sums, and the eight K-partials of a tile meet in a
// double-buffered shared array behind one barrier per tile.
//
// Reference behaviour replaced: otf_llm/otf_triton_2bit_kernel.py:164-194 (dispatch,
// mask multiply, LUT path), :23-113 (warp GEMV), otf_llm/symmetric_2bit_engine.py:
// 214-235 (bias, outlier anchors, clamp), otf_llm/otf_2bit_quantizer.py:193-221.
#include <algorithm>

#include "otf_common.cuh"

namespace otf {

constexpr int kWarps = 8;      // warps per CTA (one K slice each)
constexpr int kRows = 16;      // rows per tile (the m16 of the MMA)
constexpr int kRing = 4;       // (tile, chunk) items in flight per warp
constexpr int kOutPerLane = 8; // prefetched anchor values per lane and row

struct LinearArgs {
  const uint16_t* x;
  int64_t ldx;
  const uint8_t* packed;
  int64_t ldp;
  const uint16_t* scales;
  int64_t lds;
  const uint16_t* zeros;
  int64_t ldz;
  const uint16_t* mask;
  const int64_t* oidx;
  int n_out;
  const uint16_t* ovals;
  int64_t ldo;
  const uint16_t* bias;
  const uint16_t* res;
  int64_t ldr;
  uint16_t* y;
  int64_t ldy;
  int M, N, K, G;
  float c0, c1, c2, c3;
  int clamp;
};

__host__ __device__ inline int64_t gemv_smem_bytes(int W, int K, int n_out) {
  const int SL = 32 * W + 8, SB = 2 * SL, nblk = K / (16 * W);
  int64_t off = align_up((int64_t)nblk * SB, 16);
  off += align_up((int64_t)K * 2, 16);     // staged activation x * mask (fp16)
  off += 3 * (int64_t)nblk * 4;            // F, T, S per block
  off += align_up(n_out, 4) * 4;           // anchor activations
  off += 2 * kWarps * kRows * 4;           // double-buffered K partials
  off = align_up(off, 16) + SL;            // zero block
  return align_up(off, 16);
}

template <int W>
struct Item {
  uint32_t wg[W], wg8[W];  // code words of rows g and g+8
  uint32_t s;              // scales of rows g (lo) and g+8 (hi), fp16 bits
  uint32_t z;              // zero points, same packing
};

__device__ __forceinline__ uint16_t ldg_u16(const uint16_t* p) { return __ldg(p); }

template <int W, bool ZEROS>
__global__ void __launch_bounds__(kWarps * 32, 2) k_gemv2b(const LinearArgs a) {
  constexpr int BLK = 16 * W, SL = 32 * W + 8, SB = 2 * SL;
  constexpr int LPB = 8 * W;          // table lanes per block
  constexpr int BPP = 32 / LPB;       // blocks per warp pass
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = a.K, N = a.N;
  const int nblk = K / BLK, nch = ceil_div(nblk, 4);
  uint8_t* tbl = smem;
  __half* xs = reinterpret_cast<__half*>(smem + align_up((int64_t)nblk * SB, 16));
  float* sF = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + align_up((int64_t)K * 2, 16));
  float* sT = sF + nblk;
  float* sS = sT + nblk;
  float* xo = sS + nblk;
  float* red = xo + align_up(a.n_out, 4);
  uint8_t* zblk = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(red + 2 * kWarps * kRows), 16));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int cb = warp * nch / kWarps, ce = (warp + 1) * nch / kWarps;  // my chunks [cb, ce)
  const int mych = ce - cb, ipt = mych > 0 ? mych : 1;                 // items per tile
  const int ob = warp * a.n_out / kWarps, oe = (warp + 1) * a.n_out / kWarps;
  const int ntiles = ceil_div(N, kRows);
  const int my_tiles = (int)blockIdx.x < ntiles ? ceil_div(ntiles - (int)blockIdx.x, (int)gridDim.x) : 0;
  const int nitems = my_tiles * ipt;
  const int grp_div = a.G / BLK;

  auto load_item = [&](Item<W>& r, int it) {
    bool ok = it < nitems;
    int tile = 0, c = 0;
    if (ok) {
      const int ci = it % ipt;
      tile = (int)blockIdx.x + (it / ipt) * (int)gridDim.x;
      c = cb + ci;
      ok = ci < mych;
    }
    const int blk = 4 * c + t;
    ok = ok && blk < nblk;
    const int rg = tile * kRows + g, rg8 = rg + 8;
    const bool og = ok && rg < N, og8 = ok && rg8 < N;
    const uint8_t* pg = a.packed + (int64_t)(og ? rg : 0) * a.ldp + (int64_t)blk * (BLK / 4);
    const uint8_t* pg8 = a.packed + (int64_t)(og8 ? rg8 : 0) * a.ldp + (int64_t)blk * (BLK / 4);
    if constexpr (W == 4) {
      const uint4 v = og ? ld_stream16(pg) : make_uint4(0, 0, 0, 0);
      const uint4 v8 = og8 ? ld_stream16(pg8) : make_uint4(0, 0, 0, 0);
      r.wg[0] = v.x; r.wg[1] = v.y; r.wg[2] = v.z; r.wg[3] = v.w;
      r.wg8[0] = v8.x; r.wg8[1] = v8.y; r.wg8[2] = v8.z; r.wg8[3] = v8.w;
    } else {
      const uint2 v = og ? ld_stream8(pg) : make_uint2(0, 0);
      const uint2 v8 = og8 ? ld_stream8(pg8) : make_uint2(0, 0);
      r.wg[0] = v.x; r.wg[1] = v.y;
      r.wg8[0] = v8.x; r.wg8[1] = v8.y;
    }
    const int grp = blk / grp_div;
    const uint32_t s0 = og ? ldg_u16(a.scales + (int64_t)rg * a.lds + grp) : 0u;
    const uint32_t s1 = og8 ? ldg_u16(a.scales + (int64_t)rg8 * a.lds + grp) : 0u;
    r.s = s0 | (s1 << 16);
    if constexpr (ZEROS) {
      const uint32_t z0 = og ? ldg_u16(a.zeros + (int64_t)rg * a.ldz + grp) : 0u;
      const uint32_t z1 = og8 ? ldg_u16(a.zeros + (int64_t)rg8 * a.ldz + grp) : 0u;
      r.z = z0 | (z1 << 16);
    } else {
      r.z = 0u;
    }
  };

  // 1. Put the first kRing items of weights in flight before anything else.
  Item<W> ring[kRing];
#pragma unroll
  for (int s = 0; s < kRing; ++s) load_item(ring[s], s);

  // 2. Anchor activations (index load, then value load) go in flight next.
  float xo_reg = 0.0f;
  if ((int)threadIdx.x < a.n_out) xo_reg = h2f(ldg_u16(a.x + __ldg(a.oidx + threadIdx.x)));

  // 3. Stage x * mask (fp16, as the reference multiplies) into shared memory: one
  //    batch of independent 16-byte loads per thread, so the latency is paid once.
  for (int v = threadIdx.x; v < K / 8; v += blockDim.x) {
    uint4 xv = __ldg(reinterpret_cast<const uint4*>(a.x) + v);
    if (a.mask) {
      const uint4 mv = __ldg(reinterpret_cast<const uint4*>(a.mask) + v);
      __half2* xh = reinterpret_cast<__half2*>(&xv);
      const __half2* mh = reinterpret_cast<const __half2*>(&mv);
#pragma unroll
      for (int i = 0; i < 4; ++i) xh[i] = __hmul2(xh[i], mh[i]);
    }
    reinterpret_cast<uint4*>(xs)[v] = xv;
  }
  __syncthreads();

  // 4. Quantise this warp's slice of the activation table (blocks [4cb, 4ce)).
  {
    const float bl = a.c1 - a.c0, bh = 0.5f * (a.c2 - a.c0);
    const float cmax = fmaxf(fabsf(bl), fabsf(bh));
    const int sub = lane / LPB, l = lane % LPB;
    const int limb = l / (4 * W), wq = (l % (4 * W)) / 4, j = l & 3;
    const int b_end = min(4 * ce, nblk);
    for (int b0 = 4 * cb; b0 < b_end; b0 += BPP) {
      const int b = b0 + sub;
      const bool on = b < b_end;
      float xv[4];
      float mx = 0.0f, sx = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float v = on ? __half2float(xs[b * BLK + 16 * wq + 4 * i + j]) : 0.0f;
        xv[i] = v;
        mx = fmaxf(mx, fabsf(v));
        sx += (limb == 0) ? v : 0.0f;
      }
#pragma unroll
      for (int o = LPB / 2; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        sx += __shfl_xor_sync(0xffffffffu, sx, o);
      }
      const int E = fixed_point_exp(mx * cmax);
      const float sc = ldexpf(1.0f, E);
      uint32_t wl = 0, wh = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        int hi, lo;
        split_limbs(__float2int_rn(__fmul_rn(__fmul_rn(xv[i], bl), sc)), hi, lo);
        wl |= (uint32_t)((limb == 0 ? hi : lo) & 0xff) << (8 * i);
        split_limbs(__float2int_rn(__fmul_rn(__fmul_rn(xv[i], bh), sc)), hi, lo);
        wh |= (uint32_t)((limb == 0 ? hi : lo) & 0xff) << (8 * i);
      }
      if (on) {
        *reinterpret_cast<uint2*>(tbl + b * SB + limb * SL + (wq * 4 + j) * 8) = make_uint2(wl, wh);
        if (l == 0) {
          sF[b] = ldexpf(1.0f, -E) * (1.0f / 64.0f);
          sT[b] = a.c0 * sx;
          sS[b] = sx;
        }
      }
    }
  }
  if ((int)threadIdx.x < a.n_out) xo[threadIdx.x] = xo_reg;
  for (int i = (int)blockDim.x + threadIdx.x; i < a.n_out; i += blockDim.x) xo[i] = h2f(a.x[a.oidx[i]]);
  for (int i = threadIdx.x; i < SL / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(zblk)[i] = 0u;
  __syncthreads();

  // 5. Stream items.  Per tile: chunks -> partials p0/p1 (rows g, g+8), anchors, flush.
  float p0 = 0.0f, p1 = 0.0f;
  float av0[kOutPerLane], av1[kOutPerLane];
  float ep = 0.0f;  // bias + residual of this lane's epilogue row (warps 0-1, lanes 0-7)
#pragma unroll
  for (int i = 0; i < kOutPerLane; ++i) av0[i] = av1[i] = 0.0f;

  for (int base = 0; base < nitems; base += kRing) {
#pragma unroll
    for (int s = 0; s < kRing; ++s) {
      const int it = base + s;
      if (it < nitems) {
        const int ci = it % ipt, tl = it / ipt;
        const int tile = (int)blockIdx.x + tl * (int)gridDim.x;
        const int rg = tile * kRows + g, rg8 = rg + 8;
        if (ci == 0) {
          // Anchor values of this tile for this warp's anchor columns, and the epilogue terms.
#pragma unroll
          for (int i = 0; i < kOutPerLane; ++i) {
            const int jo = ob + t + 4 * i;
            av0[i] = (jo < oe && rg < N) ? h2f(ldg_u16(a.ovals + (int64_t)rg * a.ldo + jo)) : 0.0f;
            av1[i] = (jo < oe && rg8 < N) ? h2f(ldg_u16(a.ovals + (int64_t)rg8 * a.ldo + jo)) : 0.0f;
          }
          if (warp < 2 && lane < 8) {
            const int r = tile * kRows + warp * 8 + lane;
            ep = 0.0f;
            if (r < N) {
              if (a.bias) ep += h2f(ldg_u16(a.bias + r));
              if (a.res) ep += h2f(ldg_u16(a.res + r));
            }
          }
        }
        if (ci < mych) {
          const int c = cb + ci;
          const int blk = 4 * c + t;
          const int bblk = 4 * c + (g >> 1);
          const uint8_t* bp = ((g >> 1) == t && bblk < nblk) ? (tbl + bblk * SB + (g & 1) * SL) : zblk;
          int C[4][4];
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int f = 0; f < 4; ++f) C[j][f] = 0;
#pragma unroll
          for (int w = 0; w < W; ++w) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint2 bb = *reinterpret_cast<const uint2*>(bp + (w * 4 + j) * 8);
              const uint32_t ml = 0x01010101u << (2 * j), mh = 0x02020202u << (2 * j);
              mma_u8s8(C[j], ring[s].wg[w] & ml, ring[s].wg8[w] & ml, ring[s].wg[w] & mh, ring[s].wg8[w] & mh,
                       bb.x, bb.y);
            }
          }
          if (blk < nblk) {
            int v[4];
#pragma unroll
            for (int f = 0; f < 4; ++f) v[f] = 64 * C[0][f] + 16 * C[1][f] + 4 * C[2][f] + C[3][f];
            const float F = sF[blk], T = sT[blk];
            const float sg = h2f((uint16_t)(ring[s].s & 0xffffu)), sg8 = h2f((uint16_t)(ring[s].s >> 16));
            p0 = fmaf(sg, fmaf((float)(256 * v[0] + v[1]), F, T), p0);
            p1 = fmaf(sg8, fmaf((float)(256 * v[2] + v[3]), F, T), p1);
            if constexpr (ZEROS) {
              const float S = sS[blk];
              p0 = fmaf(h2f((uint16_t)(ring[s].z & 0xffffu)), S, p0);
              p1 = fmaf(h2f((uint16_t)(ring[s].z >> 16)), S, p1);
            }
          }
        }
        load_item(ring[s], it + kRing);
        if (ci == ipt - 1) {
          // Tile flush: anchors, quad reduction, cross-warp exchange, epilogue.
#pragma unroll
          for (int i = 0; i < kOutPerLane; ++i) {
            const int jo = ob + t + 4 * i;
            if (jo < oe) {
              p0 = fmaf(xo[jo], av0[i], p0);
              p1 = fmaf(xo[jo], av1[i], p1);
            }
          }
          for (int jo = ob + t + 4 * kOutPerLane; jo < oe; jo += 4) {  // beyond the prefetched span
            if (rg < N) p0 = fmaf(xo[jo], h2f(ldg_u16(a.ovals + (int64_t)rg * a.ldo + jo)), p0);
            if (rg8 < N) p1 = fmaf(xo[jo], h2f(ldg_u16(a.ovals + (int64_t)rg8 * a.ldo + jo)), p1);
          }
          p0 += __shfl_xor_sync(0xffffffffu, p0, 1);
          p0 += __shfl_xor_sync(0xffffffffu, p0, 2);
          p1 += __shfl_xor_sync(0xffffffffu, p1, 1);
          p1 += __shfl_xor_sync(0xffffffffu, p1, 2);
          float* rb = red + (tl & 1) * (kWarps * kRows);
          if (t == 0) {
            rb[warp * kRows + g] = p0;
            rb[warp * kRows + g + 8] = p1;
          }
          p0 = p1 = 0.0f;
          __syncthreads();
          if (warp < 2 && lane < 8) {
            const int rl = warp * 8 + lane;
            const int r = tile * kRows + rl;
            if (r < N) {
              float yv = ep;
#pragma unroll
              for (int w = 0; w < kWarps; ++w) yv += rb[w * kRows + rl];
              if (a.clamp) yv = fminf(fmaxf(yv, -65504.0f), 65504.0f);
              a.y[r] = f2h(yv);
            }
          }
        }
      }
    }
  }
}

// Portable CUDA-core kernel: any M, any G dividing K with G % 4 == 0, any codebook.
// One warp per output row, lanes stride over packed bytes; MT activation rows per launch.
template <int MT>
__global__ void __launch_bounds__(256) k_linear_generic(const LinearArgs a, int m0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= a.N) return;
  const int mcount = min(MT, a.M - m0);
  float acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
  const uint8_t* pr = a.packed + (int64_t)row * a.ldp;
  for (int kb = lane; kb < a.K / 4; kb += 32) {
    const uint32_t byte = pr[kb];
    const int k = 4 * kb;
    const int grp = k / a.G;
    const float s = h2f(a.scales[(int64_t)row * a.lds + grp]);
    const float z = a.zeros ? h2f(a.zeros[(int64_t)row * a.ldz + grp]) : 0.0f;
    float w4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t q = (byte >> (2 * i)) & 3u;
      const float cv = (q & 2u) ? ((q & 1u) ? a.c3 : a.c2) : ((q & 1u) ? a.c1 : a.c0);
      w4[i] = fmaf(cv, s, z);
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m < mcount) {
        const uint16_t* xr = a.x + (int64_t)(m0 + m) * a.ldx + k;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          __half xh = __ushort_as_half(xr[i]);
          if (a.mask) xh = __hmul(xh, __ushort_as_half(a.mask[k + i]));
          acc[m] = fmaf(__half2float(xh), w4[i], acc[m]);
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], s);
  }
  for (int m = 0; m < mcount; ++m) {
    float o = 0.0f;
    const uint16_t* xr = a.x + (int64_t)(m0 + m) * a.ldx;
    for (int jo = lane; jo < a.n_out; jo += 32) o = fmaf(h2f(xr[a.oidx[jo]]), h2f(a.ovals[(int64_t)row * a.ldo + jo]), o);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) o += __shfl_xor_sync(0xffffffffu, o, s);
    if (lane == 0) {
      float yv = acc[m] + o;
      if (a.bias) yv += h2f(a.bias[row]);
      if (a.res) yv += h2f(a.res[(int64_t)(m0 + m) * a.ldr + row]);
      if (a.clamp) yv = fminf(fmaxf(yv, -65504.0f), 65504.0f);
      a.y[(int64_t)(m0 + m) * a.ldy + row] = f2h(yv);
    }
  }
}

// 2-bit code unpack: one thread per packed byte, four code bytes out.
__global__ void k_unpack_codes(const uint8_t* packed, int64_t ldp, int N, int K, uint8_t* codes, int64_t ldc) {
  const int64_t kb4 = K / 4;
  const int64_t total = (int64_t)N * kb4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / kb4, kb = i % kb4;
    const uint32_t b = packed[n * ldp + kb];
    uint8_t* o = codes + n * ldc + 4 * kb;
    o[0] = b & 3u;
    o[1] = (b >> 2) & 3u;
    o[2] = (b >> 4) & 3u;
    o[3] = (b >> 6) & 3u;
  }
}

// ---------------------------------------------------------------------------------------
// Host side.

int set_cuda_error(cudaError_t e);  // capi.cu
int check_device();                 // capi.cu

static int num_sms() {
  static thread_local int cached[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

template <int W, bool ZEROS>
static int launch_gemv(const LinearArgs& a, cudaStream_t st) {
  const int64_t smem = gemv_smem_bytes(W, a.K, a.n_out);
  static thread_local int configured_dev[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured_dev[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv2b<W, ZEROS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return set_cuda_error(e);
    configured_dev[dev] = 1;
  }
  const int ntiles = ceil_div(a.N, kRows);
  const int per_sm = smem <= 100 * 1024 ? 2 : 1;
  const int ctas = std::max(1, std::min(ntiles, per_sm * num_sms()));
  k_gemv2b<W, ZEROS><<<ctas, kWarps * 32, smem, st>>>(a);
  return set_cuda_error(cudaGetLastError());
}

static int launch_generic(const LinearArgs& a, cudaStream_t st) {
  const int ctas = ceil_div(a.N, 8);
  for (int m0 = 0; m0 < a.M; m0 += 4) {
    k_linear_generic<4><<<ctas, 256, 0, st>>>(a, m0);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(e);
  }
  return OTF_OK;
}

}  // namespace otf

using namespace otf;

extern "C" OTF_API int otf2b_linear(const void* x, int64_t ldx, const uint8_t* packed, int64_t ld_packed,
                                    const void* scales, int64_t ld_scales, const void* zeros, int64_t ld_zeros,
                                    const float* codebook, const void* mask, const int64_t* outlier_idx,
                                    int64_t n_outliers, const void* outlier_vals, int64_t ld_outlier_vals,
                                    const void* bias, const void* residual, int64_t ld_residual, void* y,
                                    int64_t ldy, int64_t M, int64_t N, int64_t K,
                                    int64_t group_size, uint32_t flags, void* stream) {
  if (!x || !packed || !scales || !codebook || !y) return OTF_ERR_INVALID;
  if (M <= 0 || N <= 0 || K <= 0 || group_size <= 0) return OTF_ERR_INVALID;
  if (K % 4 || group_size % 4 || K % group_size) return OTF_ERR_INVALID;
  if (N > (int64_t)INT32_MAX / 2 || K > (1 << 20) || M > (1 << 24)) return OTF_ERR_UNSUPPORTED;
  if (ld_packed < K / 4 || ld_scales < K / group_size || ldx < K || ldy < N) return OTF_ERR_INVALID;
  if (zeros && ld_zeros < K / group_size) return OTF_ERR_INVALID;
  if (residual && ld_residual < N) return OTF_ERR_INVALID;
  if (n_outliers < 0 || (n_outliers > 0 && (!outlier_idx || !outlier_vals || ld_outlier_vals < n_outliers)))
    return OTF_ERR_INVALID;
  if (n_outliers > 65536) return OTF_ERR_UNSUPPORTED;
  int st = check_device();
  if (st != OTF_OK) return st;

  LinearArgs a;
  a.x = static_cast<const uint16_t*>(x);
  a.ldx = ldx;
  a.packed = packed;
  a.ldp = ld_packed;
  a.scales = static_cast<const uint16_t*>(scales);
  a.lds = ld_scales;
  a.zeros = static_cast<const uint16_t*>(zeros);
  a.ldz = ld_zeros;
  a.mask = static_cast<const uint16_t*>(mask);
  a.oidx = n_outliers > 0 ? outlier_idx : nullptr;
  a.n_out = (int)n_outliers;
  a.ovals = static_cast<const uint16_t*>(outlier_vals);
  a.ldo = ld_outlier_vals;
  a.bias = static_cast<const uint16_t*>(bias);
  a.res = static_cast<const uint16_t*>(residual);
  a.ldr = ld_residual;
  a.y = static_cast<uint16_t*>(y);
  a.ldy = ldy;
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.G = (int)group_size;
  a.c0 = codebook[0];
  a.c1 = codebook[1];
  a.c2 = codebook[2];
  a.c3 = codebook[3];
  a.clamp = (flags & OTF_FLAG_CLAMP) ? 1 : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // The tensor-pipe path needs c3 - c2 == c1 - c0 (affine in the two code bits),
  // a block of 16W codes inside one scale group and aligned packed rows.
  const float lhs = a.c3 - a.c2, rhs = a.c1 - a.c0;
  const bool affine = fabsf(lhs - rhs) <= 1e-6f * fmaxf(1.0f, fabsf(rhs));
  const uintptr_t pa = reinterpret_cast<uintptr_t>(packed);
  const bool x_al = reinterpret_cast<uintptr_t>(x) % 16 == 0 && (!mask || reinterpret_cast<uintptr_t>(mask) % 16 == 0);
  const bool fast_ok = !(flags & OTF_FLAG_FORCE_GENERIC) && affine && M == 1 && x_al && K % 8 == 0;
  if (fast_ok && group_size % 64 == 0 && pa % 16 == 0 && ld_packed % 16 == 0 &&
      gemv_smem_bytes(4, a.K, a.n_out) <= 227 * 1024)
    return zeros ? launch_gemv<4, true>(a, s) : launch_gemv<4, false>(a, s);
  if (fast_ok && group_size % 32 == 0 && pa % 8 == 0 && ld_packed % 8 == 0 &&
      gemv_smem_bytes(2, a.K, a.n_out) <= 227 * 1024)
    return zeros ? launch_gemv<2, true>(a, s) : launch_gemv<2, false>(a, s);
  return launch_generic(a, s);
}

extern "C" OTF_API int otf2b_unpack_codes(const uint8_t* packed, int64_t ld_packed, int64_t N, int64_t K,
                                          uint8_t* codes, int64_t ld_codes, void* stream) {
  if (!packed || !codes || N <= 0 || K <= 0 || K % 4 || ld_packed < K / 4 || ld_codes < K) return OTF_ERR_INVALID;
  if (N > INT32_MAX || K > INT32_MAX) return OTF_ERR_UNSUPPORTED;
  int st = check_device();
  if (st != OTF_OK) return st;
  const int64_t total = N * (K / 4);
  const int blocks = (int)std::min<int64_t>(ceil_div((int)std::min<int64_t>(total, INT32_MAX), 256), 148 * 16);
  k_unpack_codes<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(packed, ld_packed, (int)N, (int)K, codes,
                                                                       ld_codes);
  return set_cuda_error(cudaGetLastError());
}
