// INT8 shared-vocabulary LM head and embedding gather for B200 (sm_100a).
//
// The head streams int8 weight rows straight into the A operand of the integer
// tensor pipe (m16n8k32, s8 x s8 -> s32): no per-weight decode at all.  The
// activation is 16-bit fixed point per 16-value block, split into two s8 limbs in
// MMA columns 2t (hi) and 2t+1 (lo), so each thread's accumulator fragment holds
// its own block.  Replaces QuantizedLinearHead.forward
// (otf_llm/symmetric_2bit_engine.py:75-91) and QuantizedEmbedding.forward (:41-47).
#include <cuda.h>

#include <algorithm>

#include "otf_common.cuh"

namespace otf {

int set_cuda_error(cudaError_t e);  // capi.cu
int check_device();                 // capi.cu
bool encode_tiled_2d(void* map, int elem_bytes, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                     uint32_t box_inner, uint32_t box_rows, bool swizzle128);  // capi.cu
int head_device_error(int clear);   // read (and optionally clear) the flag below

// Set when a bounded wait of the TMA-fed head gives up; read through otf_device_error.
__device__ int g_head_device_error;

constexpr int kHeadWarps = 8;
constexpr int kHeadSL = 24;  // bytes per (block, limb): 16 data + 8 pad (conflict-free lane map)
constexpr int kHeadSB = 48;  // bytes per 16-value block

struct HeadArgs {
  const uint16_t* x;
  const int8_t* w;
  int64_t ldw;
  const uint16_t* scales;
  float* out;                 // logits (may be null when only the argmax is wanted)
  unsigned long long* amax;   // packed (ordered logit, ~index) maximum, or null
  int V, D;
  int64_t ldx, ldl;           // row strides of x and of the logits (multi-row TMA head)
};

// Order-preserving 64-bit key of (logit, index): larger logit wins, then the smaller index
// (the first maximum, like torch.argmax).
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(~(uint32_t)idx);
}

__host__ __device__ inline int64_t head_smem_bytes(int D) {
  const int nb = D / 16;
  return align_up(align_up((int64_t)nb * kHeadSB, 16) + (int64_t)nb * 4, 16) + 16;
}

__device__ __forceinline__ float head_finish(float v, float s) {
  float r = v * s;
  if (isnan(r)) r = 0.0f;
  return fminf(fmaxf(r, -65504.0f), 65504.0f);
}

// Pipelined head: every warp streams its own stages of 16 rows x 128 weight bytes with
// cp.async (4 stages in flight, 144-byte row pitch so the consumers' 16-byte reads are
// bank-conflict-free), consumed as two block-diagonal MMA sets of four 16-value blocks.
constexpr int kHeadSlots = 4;
constexpr int kHeadChunk = 128;                     // weight bytes per row per stage
constexpr int kHeadPitch = kHeadChunk + 16;
constexpr int kHeadStage = 16 * kHeadPitch;

__host__ __device__ inline int64_t head_pipe_smem_bytes(int D) {
  return (int64_t)kHeadWarps * kHeadSlots * kHeadStage + head_smem_bytes(D);
}

__global__ void __launch_bounds__(kHeadWarps * 32) k_i8_head_imma(const HeadArgs a) {
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem[];
  const int nb = a.D / 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* const wst = smem + warp * kHeadSlots * kHeadStage;   // this warp's stages
  uint8_t* tbl = smem + (int64_t)kHeadWarps * kHeadSlots * kHeadStage;
  float* metaF = reinterpret_cast<float*>(tbl + align_up((int64_t)nb * kHeadSB, 16));
  uint8_t* zblk = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<uintptr_t>(metaF + nb), 16));

  // Work: warp gw of the grid takes the tiles [gw*T/W, (gw+1)*T/W) (balanced), every chunk of
  // the row in order.
  const int ntiles = ceil_div(a.V, 16);
  const int nch = ceil_div(a.D, kHeadChunk);
  const int nwarps = gridDim.x * kHeadWarps, gw = blockIdx.x * kHeadWarps + warp;
  const int t_beg = (int)(((int64_t)gw * ntiles) / nwarps), t_end = (int)(((int64_t)(gw + 1) * ntiles) / nwarps);
  const int nst = (t_end - t_beg) * nch;
  const int lr = lane >> 1, lh = lane & 1;
  const uint32_t cdst0 = smem_u32(wst) + lr * kHeadPitch + 64 * lh;
  int is_cc = 0, is_tile = t_beg;
  const int8_t* crow = a.w;
  bool row_ok = false;
  auto issue_tile = [&]() {
    const int r = is_tile * 16 + lr;
    row_ok = r < a.V;
    crow = a.w + (int64_t)(row_ok ? r : 0) * a.ldw + 64 * lh;
  };
  auto issue = [&](int slot) {
    const uint32_t so = (uint32_t)(slot * kHeadStage);
    const int cb = is_cc * kHeadChunk;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rem = row_ok ? a.D - cb - 64 * lh - 16 * i : 0;
      const uint32_t nbytes = (uint32_t)max(0, min(16, rem));
      cp_async16(cdst0 + so + 16 * i, nbytes ? reinterpret_cast<const void*>(crow + cb + 16 * i)
                                             : reinterpret_cast<const void*>(a.w), nbytes);
    }
    if (++is_cc == nch) {
      is_cc = 0;
      ++is_tile;
      issue_tile();
    }
  };
  issue_tile();
#pragma unroll
  for (int k = 0; k < kHeadSlots; ++k) {
    if (k < nst) issue(k);
    cp_async_commit();
  }

  pdl_wait();
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

  const int g = lane >> 2, t = lane & 3;
  const bool breal = (g >> 1) == t;
  float acc0 = 0.0f, acc1 = 0.0f;
  int cc = 0, tile = t_beg, s = 0;
  const uint8_t* st = wst;
  for (int k = 0; k < nst; ++k) {
    cp_async_wait<kHeadSlots - 1>();
    __syncwarp();
    const uint8_t* pa = st + g * kHeadPitch + 32 * t;
#pragma unroll
    for (int set = 0; set < 2; ++set) {
      const uint4 cw = *reinterpret_cast<const uint4*>(pa + 16 * set);
      const uint4 cw8 = *reinterpret_cast<const uint4*>(pa + 8 * kHeadPitch + 16 * set);
      const int blk = cc * 8 + 2 * t + set;        // my block (this quad's)
      const int bblk = cc * 8 + 2 * (g >> 1) + set;  // the block whose B rows this lane supplies
      const uint8_t* bp = (breal && bblk < nb) ? (tbl + bblk * kHeadSB + (g & 1) * kHeadSL) : zblk;
      const uint2 b01 = *reinterpret_cast<const uint2*>(bp);
      const uint2 b23 = *reinterpret_cast<const uint2*>(bp + 8);
      int C[4] = {0, 0, 0, 0};
      mma_s8s8(C, cw.x, cw8.x, cw.y, cw8.y, b01.x, b01.y);
      mma_s8s8(C, cw.z, cw8.z, cw.w, cw8.w, b23.x, b23.y);
      if (blk < nb) {
        const float F = metaF[blk];
        acc0 = fmaf((float)(256 * C[0] + C[1]), F, acc0);
        acc1 = fmaf((float)(256 * C[2] + C[3]), F, acc1);
      }
    }
    __syncwarp();
    if (k + kHeadSlots < nst) issue(s);
    cp_async_commit();
    if (++s == kHeadSlots) {
      s = 0;
      st = wst;
    } else {
      st += kHeadStage;
    }
    if (++cc == nch) {
      acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
      acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
      acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
      acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
      const int rg = tile * 16 + g, rg8 = rg + 8;
      const float l0 = rg < a.V ? head_finish(acc0, h2f(a.scales[rg])) : 0.0f;
      const float l1 = rg8 < a.V ? head_finish(acc1, h2f(a.scales[rg8])) : 0.0f;
      if (t == 0 && a.out) {
        if (rg < a.V) a.out[rg] = l0;
        if (rg8 < a.V) a.out[rg8] = l1;
      }
      if (a.amax) {
        unsigned long long key = 0ull;
        if (rg < a.V) key = argmax_key(l0, rg);
        if (rg8 < a.V) key = max(key, argmax_key(l1, rg8));
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
        if (lane == 0) atomicMax(a.amax, key);
      }
      acc0 = acc1 = 0.0f;
      cc = 0;
      ++tile;
    }
  }
  cp_async_wait<0>();
}

// TMA-fed head: one producer warp streams boxes of 64 vocabulary rows x 128 weight bytes
// (128-byte swizzle) into two rings, one per team of four consumer warps.  Team k takes the
// CTA's row quads k, k+2, ... with all their chunks in order; warp w of the team multiplies
// tile w (16 rows) of each box, both MMA sets, exactly as the copy-stage kernel does.  The
// producer alternates the teams' boxes and refills a slot once that team's four warps have
// consumed it.  Every wait is bounded (about a second; then the flag above is raised).
constexpr int kHTRows = 64;                          // rows per box
constexpr int kHTBoxBytes = kHTRows * kHeadChunk;    // 8 KB
constexpr int kHTConsumers = 8;                      // two teams of four
constexpr int kHTThreads = (kHTConsumers + 1) * 32;
constexpr int kHTSlots = 4;                          // ring slots per team (a power of two)

struct alignas(64) HeadTmaArgs {
  CUtensorMap wmap;  // int8 [V, D], 128 x 64 boxes, 128-byte swizzle
  HeadArgs a;
};

// One activation row's fixed-point table and block factors (the layout head_smem_bytes
// describes, without the zero block).
__host__ __device__ inline int64_t head_row_table_bytes(int D) {
  const int nb = D / 16;
  return align_up(align_up((int64_t)nb * kHeadSB, 16) + (int64_t)nb * 4, 16);
}

// R activation rows per launch share every weight box: R tables, then the zero block.
__host__ __device__ inline int64_t head_tma_smem_bytes(int D, int R) {
  return 1024 + 2 * kHTSlots * kHTBoxBytes + 128 + (int64_t)R * head_row_table_bytes(D) + 16;
}

__device__ __forceinline__ void head_wait_failed() { atomicExch(&g_head_device_error, 1); }

// R activation rows (x rows a.x + r * a.ldx) per launch: each weight box feeds every row's MMAs,
// so the weights stream once for R rows; each row's arithmetic (table, MMA sets, flush order,
// reduction) is the single-row kernel's, so its logits are bit-identical to a launch of its own.
template <int R>
__global__ void __launch_bounds__(kHTThreads, R <= 2 ? 2 : 1) k_i8_head_tma(const __grid_constant__ HeadTmaArgs p) {
  const HeadArgs& a = p.a;
  pdl_trigger();
  // Dynamic shared memory rounded up to the 1024-byte period of the swizzle (1 KB of slack).
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* const smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* const ring = smem;                                      // [team][slot] boxes
  const uint32_t full = smem_u32(smem + 2 * kHTSlots * kHTBoxBytes);
  const uint32_t empty = full + 8 * 2 * kHTSlots;
  uint8_t* const tbl = smem + 2 * kHTSlots * kHTBoxBytes + 128;
  const int nb = a.D / 16;
  const int64_t tstride = head_row_table_bytes(a.D);              // row rr's table at tbl + rr * tstride
  const int64_t moff = align_up((int64_t)nb * kHeadSB, 16);        // its block factors after the table
  uint8_t* const zblk = tbl + R * tstride;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nq = ceil_div(a.V, kHTRows), nch = ceil_div(a.D, kHeadChunk);
  const int q_beg = (int)((int64_t)blockIdx.x * nq / gridDim.x);
  const int q_end = (int)((int64_t)(blockIdx.x + 1) * nq / gridDim.x);
  const int nq0 = (q_end - q_beg + 1) / 2, nq1 = (q_end - q_beg) / 2;  // quads of teams 0 and 1
  if (tid == 0) {
    for (int i = 0; i < 2 * kHTSlots; ++i) {
      mbar_init(full + 8 * i, 1);
      mbar_init(empty + 8 * i, 4);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kHTConsumers) {
    // Producer (weights only: they do not depend on the previous kernel, so no PDL wait).
    if (lane == 0) {
      const int nbox[2] = {nq0 * nch, nq1 * nch};
      int i[2] = {0, 0}, q[2] = {q_beg, q_beg + 1}, c[2] = {0, 0};
      while (i[0] < nbox[0] || i[1] < nbox[1]) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (i[k] >= nbox[k]) continue;
          const int sl = k * kHTSlots + (i[k] & (kHTSlots - 1));
          if (i[k] >= kHTSlots && !mbar_wait_sleep(empty + 8 * sl, (uint32_t)((i[k] / kHTSlots) - 1) & 1u))
            head_wait_failed();
          mbar_arrive_expect_tx(full + 8 * sl, (uint32_t)kHTBoxBytes);
          tma_load_2d(smem_u32(ring + sl * kHTBoxBytes), &p.wmap, c[k] * kHeadChunk, q[k] * kHTRows, full + 8 * sl);
          ++i[k];
          if (++c[k] == nch) {
            c[k] = 0;
            q[k] += 2;
          }
        }
      }
    }
    return;
  }

  pdl_wait();
  // Activation tables for the whole D, one per row (every CTA builds its own; its vocabulary
  // rows amortise them).
  for (int it = tid; it < 2 * nb * R; it += kHTConsumers * 32) {
    const int rr = it / (2 * nb), b = (it >> 1) - rr * nb, limb = it & 1;
    const uint16_t* const xr = a.x + rr * a.ldx;
    uint8_t* const trow = tbl + rr * tstride;
    float* const metaF = reinterpret_cast<float*>(trow + moff);
    float xv[16];
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      xv[i] = h2f(xr[b * 16 + i]);
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
    uint2* dst = reinterpret_cast<uint2*>(trow + b * kHeadSB + limb * kHeadSL);
    dst[0] = make_uint2(wd[0], wd[1]);
    dst[1] = make_uint2(wd[2], wd[3]);
    if (limb == 0) metaF[b] = ldexpf(1.0f, -E);
  }
  if (tid < 4) reinterpret_cast<uint32_t*>(zblk)[tid] = 0u;
  named_barrier_sync(1, kHTConsumers * 32);

  const int team = warp >> 2, wt = warp & 3;
  const int g = lane >> 2, t = lane & 3;
  const bool breal = (g >> 1) == t;
  const int r = wt * 16 + g;                        // box row of this thread's first row
  int i = 0;                                        // this team's box count
  const int my_nq = team ? nq1 : nq0;
  for (int qi = 0; qi < my_nq; ++qi) {
    const int quad = q_beg + team + 2 * qi;
    float acc0[R], acc1[R];
#pragma unroll
    for (int rr = 0; rr < R; ++rr) acc0[rr] = acc1[rr] = 0.0f;
    for (int cc = 0; cc < nch; ++cc, ++i) {
      const int sl = team * kHTSlots + (i & (kHTSlots - 1));
      if (!mbar_wait_spin(full + 8 * sl, (uint32_t)(i / kHTSlots) & 1u)) head_wait_failed();
      const uint8_t* const box = ring + sl * kHTBoxBytes;
#pragma unroll
      for (int set = 0; set < 2; ++set) {
        // 16-byte piece 2t+set of rows r and r+8 (piece j of row r sits at j ^ (r & 7) = j ^ g).
        const uint8_t* pa = box + r * kHeadChunk + (((2 * t + set) ^ g) << 4);
        const uint4 cw = *reinterpret_cast<const uint4*>(pa);
        const uint4 cw8 = *reinterpret_cast<const uint4*>(pa + 8 * kHeadChunk);
        const int blk = cc * 8 + 2 * t + set;          // my block (this quad's)
        const int bblk = cc * 8 + 2 * (g >> 1) + set;  // the block whose B rows this lane supplies
        const bool bok = breal && bblk < nb;
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
          const uint8_t* const trow = tbl + rr * tstride;
          const uint8_t* bp = bok ? (trow + bblk * kHeadSB + (g & 1) * kHeadSL) : zblk;
          const uint2 b01 = *reinterpret_cast<const uint2*>(bp);
          const uint2 b23 = *reinterpret_cast<const uint2*>(bp + 8);
          int C[4] = {0, 0, 0, 0};
          mma_s8s8(C, cw.x, cw8.x, cw.y, cw8.y, b01.x, b01.y);
          mma_s8s8(C, cw.z, cw8.z, cw.w, cw8.w, b23.x, b23.y);
          if (blk < nb) {
            const float F = reinterpret_cast<const float*>(trow + moff)[blk];
            acc0[rr] = fmaf((float)(256 * C[0] + C[1]), F, acc0[rr]);
            acc1[rr] = fmaf((float)(256 * C[2] + C[3]), F, acc1[rr]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + 8 * sl);
    }
    const int rg = quad * kHTRows + r, rg8 = rg + 8;
    const float s0 = rg < a.V ? h2f(a.scales[rg]) : 0.0f, s8 = rg8 < a.V ? h2f(a.scales[rg8]) : 0.0f;
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      float v0 = acc0[rr], v1 = acc1[rr];
      v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
      v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
      v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
      v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
      const float l0 = rg < a.V ? head_finish(v0, s0) : 0.0f;
      const float l1 = rg8 < a.V ? head_finish(v1, s8) : 0.0f;
      float* const out = a.out ? a.out + rr * a.ldl : nullptr;
      if (t == 0 && out) {
        if (rg < a.V) out[rg] = l0;
        if (rg8 < a.V) out[rg8] = l1;
      }
      if (a.amax) {
        unsigned long long key = 0ull;
        if (rg < a.V) key = argmax_key(l0, rg);
        if (rg8 < a.V) key = max(key, argmax_key(l1, rg8));
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
        if (lane == 0) atomicMax(a.amax + rr, key);
      }
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
  if (lane == 0) {
    const float l = head_finish(acc, h2f(a.scales[row]));
    if (a.out) a.out[row] = l;
    if (a.amax) atomicMax(a.amax, argmax_key(l, row));
  }
}

// Packed maximum -> vocabulary index, in place.
__global__ void k_argmax_finish(unsigned long long* key, int64_t* idx, int M) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_trigger();
  pdl_wait();
  if (m < M) idx[m] = (int64_t)(~(uint32_t)(key[m] & 0xffffffffull));
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

// The same gather for rows of D = 16k bytes on 16-byte boundaries: thread t converts the row's
// 16-byte pieces t, t + 256, ... (at most 4), all requested together with the row's scale once
// the id is known, so a row costs two memory round trips (id, then row) instead of one per
// strided byte.
__global__ void __launch_bounds__(256) k_i8_embed_v(const int64_t* ids, int n, const int8_t* __restrict__ w,
                                                    int64_t ldw, const uint16_t* __restrict__ scales,
                                                    uint16_t* __restrict__ out, int64_t ldo, int64_t V, int D,
                                                    int32_t* bad) {
  pdl_trigger();
  pdl_wait();
  const int tok = blockIdx.x;
  if (tok >= n) return;
  const int64_t id = ids[tok];
  const int nv = D >> 4, tid = threadIdx.x;
  uint4* o = reinterpret_cast<uint4*>(out + (int64_t)tok * ldo);
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  if (id < 0 || id >= V) {
    for (int v = tid; v < nv; v += 256) o[2 * v] = o[2 * v + 1] = z4;
    if (bad && tid == 0) *bad = 1;
    return;
  }
  const uint4* wr = reinterpret_cast<const uint4*>(w + id * ldw);
  uint4 wv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) wv[i] = tid + i * 256 < nv ? __ldg(wr + tid + i * 256) : z4;
  const __half s = __ushort_as_half(__ldg(scales + id));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int v = tid + i * 256;
    if (v >= nv) break;
    const int8_t* b = reinterpret_cast<const int8_t*>(&wv[i]);
    uint4 r[2];
    __half* e = reinterpret_cast<__half*>(r);
#pragma unroll
    for (int j = 0; j < 16; ++j) e[j] = __hmul(__int2half_rn((int)b[j]), s);
    o[2 * v] = r[0];
    o[2 * v + 1] = r[1];
  }
}

}  // namespace otf

using namespace otf;

int otf::head_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, otf::g_head_device_error, sizeof(int)) != cudaSuccess) {
    set_cuda_error(cudaGetLastError());
    return -1;
  }
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(otf::g_head_device_error, &z, sizeof(int));
  }
  return v;
}

// Rows per launch of the TMA-fed head: the most (1, 2, 4 or 8, at most the rows left) whose
// activation tables fit in shared memory beside the weight rings.
static int head_tma_rows(int64_t left, int D) {
  int R = 8;
  while (R > 1 && (R > left || head_tma_smem_bytes(D, R) > 227 * 1024)) R >>= 1;
  return R;
}

template <int R>
static cudaError_t launch_head_tma(const HeadTmaArgs& p, int dev, int sms, cudaStream_t s) {
  static thread_local int configured_dev[64] = {};
  if (!configured_dev[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_i8_head_tma<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    configured_dev[dev] = 1;
  }
  const int64_t smem = head_tma_smem_bytes(p.a.D, R);
  const int per_sm = (R <= 2 && smem <= 113 * 1024) ? 2 : 1;
  const int ctas = std::max(1, std::min(ceil_div(p.a.V, kHTRows), per_sm * std::max(1, sms)));
  return launch_pdl(k_i8_head_tma<R>, dim3((unsigned)ctas), dim3(kHTThreads), (size_t)smem, s, 1u, p);
}

// The TMA-fed head for R rows (x rows a.x + r * a.ldx, logits a.out + r * a.ldl, keys
// a.amax + r) of 16-byte aligned int8 weights (D a multiple of 16); false if the layout does
// not qualify (the caller then runs the copy-stage kernel row by row).
static bool head_launch_tma(const HeadArgs& a, int R, cudaStream_t s, cudaError_t& err) {
  const int64_t smem = head_tma_smem_bytes(a.D, R);
  if (a.D % 16 || a.ldw % 16 || reinterpret_cast<uintptr_t>(a.w) % 16 || smem > 227 * 1024) return false;
  static thread_local int sms_of[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return false;
  if (!sms_of[dev]) cudaDeviceGetAttribute(&sms_of[dev], cudaDevAttrMultiProcessorCount, dev);
  static thread_local HeadTmaArgs p;  // 128-byte tensor map + arguments, kept off the stack
  if (!encode_tiled_2d(&p.wmap, 1, a.w, (uint64_t)a.D, (uint64_t)a.V, (uint64_t)a.ldw, (uint32_t)kHeadChunk,
                       (uint32_t)kHTRows, true))
    return false;
  p.a = a;
  switch (R) {
    case 1: err = launch_head_tma<1>(p, dev, sms_of[dev], s); break;
    case 2: err = launch_head_tma<2>(p, dev, sms_of[dev], s); break;
    case 4: err = launch_head_tma<4>(p, dev, sms_of[dev], s); break;
    default: err = launch_head_tma<8>(p, dev, sms_of[dev], s); break;
  }
  return true;
}

static int head_launch(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const void* scales, float* logits,
                       int64_t ldl, unsigned long long* keys, int64_t M, int64_t V, int64_t D, cudaStream_t s) {
  const bool fast = D % 16 == 0 && ldw % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
                    head_pipe_smem_bytes((int)D) <= 220 * 1024;
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
  for (int64_t m = 0; m < M;) {
    HeadArgs a;
    a.x = static_cast<const uint16_t*>(x) + m * ldx;
    a.w = w;
    a.ldw = ldw;
    a.scales = static_cast<const uint16_t*>(scales);
    a.out = logits ? logits + m * ldl : nullptr;
    a.amax = keys ? keys + m : nullptr;
    a.V = (int)V;
    a.D = (int)D;
    a.ldx = ldx;
    a.ldl = ldl;
    cudaError_t e = cudaSuccess;
    const int R = head_tma_rows(M - m, (int)D);
    if (head_launch_tma(a, R, s, e)) {
      if (e != cudaSuccess) return set_cuda_error(e);
      m += R;
      continue;
    }
    ++m;
    const int ctas_per_sm = head_pipe_smem_bytes((int)D) <= 110 * 1024 ? 2 : 1;
    e = fast ? launch_pdl(k_i8_head_imma,
                                      dim3(std::max(1, std::min(ceil_div(ceil_div((int)V, 16), kHeadWarps),
                                                                sms * ctas_per_sm))),
                                      dim3(kHeadWarps * 32), (size_t)head_pipe_smem_bytes((int)D), s, 1u, a)
                         : launch_pdl(k_i8_head_generic, dim3(ceil_div((int)V, 8)), dim3(256), 0, s, 1u, a);
    if (e != cudaSuccess) return set_cuda_error(e);
  }
  return OTF_OK;
}

extern "C" OTF_API int otf_i8_head(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const void* scales,
                                   float* logits, int64_t ldl, int64_t M, int64_t V, int64_t D, void* stream) {
  if (!x || !w || !scales || !logits || M <= 0 || V <= 0 || D <= 0) return OTF_ERR_INVALID;
  if (ldx < D || ldw < D || ldl < V) return OTF_ERR_INVALID;
  if (V > INT32_MAX / 2 || D > (1 << 20)) return OTF_ERR_UNSUPPORTED;
  int st = check_device();
  if (st != OTF_OK) return st;
  return head_launch(x, ldx, w, ldw, scales, logits, ldl, nullptr, M, V, D, static_cast<cudaStream_t>(stream));
}

extern "C" OTF_API int otf_i8_head_argmax(const void* x, int64_t ldx, const int8_t* w, int64_t ldw,
                                          const void* scales, float* logits, int64_t ldl, int64_t* argmax,
                                          int64_t M, int64_t V, int64_t D, void* stream) {
  if (!x || !w || !scales || !argmax || M <= 0 || V <= 0 || D <= 0) return OTF_ERR_INVALID;
  if (ldx < D || ldw < D || (logits && ldl < V)) return OTF_ERR_INVALID;
  if (V > INT32_MAX / 2 || D > (1 << 20) || M > INT32_MAX) return OTF_ERR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(argmax) % 8) return OTF_ERR_INVALID;
  int st = check_device();
  if (st != OTF_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The int64 output doubles as the packed-maximum scratch: cleared, reduced, converted.
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(argmax);
  cudaError_t e = cudaMemsetAsync(keys, 0, (size_t)M * sizeof(unsigned long long), s);
  if (e != cudaSuccess) return set_cuda_error(e);
  st = head_launch(x, ldx, w, ldw, scales, logits, ldl, keys, M, V, D, s);
  if (st != OTF_OK) return st;
  return set_cuda_error(launch_pdl(k_argmax_finish, dim3((unsigned)ceil_div((int)M, 128)), dim3(128), 0, s, 1u, keys,
                                   argmax, (int)M));
}

extern "C" OTF_API int otf_i8_embed(const int64_t* ids, int64_t n, const int8_t* w, int64_t ldw, const void* scales,
                                    void* out, int64_t ldo, int64_t V, int64_t D, int32_t* bad_ids, void* stream) {
  if (!ids || !w || !scales || !out || n < 0 || V <= 0 || D <= 0 || ldw < D || ldo < D) return OTF_ERR_INVALID;
  if (n == 0) return OTF_OK;
  if (n > INT32_MAX || D > INT32_MAX) return OTF_ERR_UNSUPPORTED;
  int st = check_device();
  if (st != OTF_OK) return st;
  if (D % 16 == 0 && D <= 4 * 256 * 16 && ldw % 16 == 0 && ldo % 8 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(out) % 16 == 0)
    return set_cuda_error(launch_pdl(k_i8_embed_v, dim3((unsigned)n), dim3(256), 0, static_cast<cudaStream_t>(stream),
                                     1u, ids, (int)n, w, ldw, static_cast<const uint16_t*>(scales),
                                     static_cast<uint16_t*>(out), ldo, V, (int)D, bad_ids));
  return set_cuda_error(launch_pdl(k_i8_embed, dim3((unsigned)n), dim3(128), 0, static_cast<cudaStream_t>(stream), 1u,
                                   ids, (int)n, w, ldw, static_cast<const uint16_t*>(scales),
                                   static_cast<uint16_t*>(out), ldo, V, (int)D, bad_ids));
}
