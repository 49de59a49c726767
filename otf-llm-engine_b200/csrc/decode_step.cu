// One batch-1 decode step of a Llama-shaped 2-bit decoder stack in a single persistent
// launch (otf2b_decode_step).
//
// Why: at batch 1 every projection of a 7B-class model is a few MB of codes, so a launch
// per projection (or per fused group) pays a fixed 4-5 us -- predecessor drain, activation
// staging, table build, cross-CTA reduction -- against under 2 us of HBM time.  Here one
// CTA per SM runs all 4 x n_layers stages of the step; stages are separated by a
// device-wide barrier (a counter in global memory, bounded polling), and the weight stream
// never stops at those barriers: every warp walks its own fixed list of weight items
// (16 rows x 512 codes + their scales) across all stages and layers and keeps kMSlots of
// them in flight in its private cp.async ring, so the next stage's codes land while the
// barrier, the activation staging and the table build run.
//
// Per stage a CTA serves one matrix (q, k or v; o; gate or up; down): the host splits the
// CTAs over a stage's matrices in proportion to their row tiles and each CTA takes a
// contiguous run of 16-row tiles.  Inside the CTA, the (tile, 512-code chunk) items of
// those tiles are dealt to the warps in contiguous runs; a warp accumulates its items of
// one tile in registers and leaves one partial per (tile, warp), which the epilogue adds in
// warp order (deterministic).  The dot products are the integer-MMA scheme of gemv2b.cu:
// the masked code words are the u8 A operand, the activation is 16-bit fixed point per
// block in two s8 limbs (the per-stage table, B), classes and limbs are folded exactly in
// int32 and scaled once per group.
//
// Stage inputs: q/k/v take RMSNorm(h), o takes the attention output (single position:
// query head j reads KV head j / (heads / kv_heads) of v), gate/up take RMSNorm(h1), down
// takes fp16(fp16(silu(g)) * u).  Epilogues add the fp16 anchor columns, bias and (o,
// down) the residual, clamp and store fp16.  The RMSNorm scale is computed by every CTA
// from the whole input vector it reads anyway, so it needs no extra exchange.
#include <cuda.h>

#include <algorithm>
#include <vector>

#include "otf_common.cuh"

namespace otf {

int set_cuda_error(cudaError_t e);  // capi.cu
int check_device();                 // capi.cu

constexpr int kMWarps = 16;                 // warps per CTA (one CTA per SM)
constexpr int kMThreads = kMWarps * 32;
constexpr int kMSlots = 3;                  // items in flight per warp
constexpr int kMCodeBytes = kRows * kChunk; // one item's codes: 16 rows x 128 bytes (TMA box, 128B swizzle)
constexpr int kMMaxTiles = 16;              // 16-row tiles per CTA per stage
constexpr int kMOvBytes = 8 * 1024;         // anchor weights staged per stage
constexpr int kMMaxOut = 256;               // anchor columns per matrix
constexpr uint32_t kMSpin = 1u << 21;       // barrier polls before giving up

__device__ int g_mk_device_error;           // set when a barrier wait gives up

struct MkArgs {
  const otf2b_decoder_layer* layers;        // device copy of the descriptors
  int n_layers, hidden, inter, qdim, kvdim, head_dim, rep, G;
  float c0, c1, c2, c3, eps;
  uint16_t *h, *q, *k, *v, *h1, *g, *u;     // activation vectors (h: in/out)
  unsigned* bar;                            // stage counter, zero at launch
  int nmat[4];                              // matrices per stage (3, 1, 2, 1)
  int split[4][4];                          // first CTA of each matrix; split[s][nmat] = CTAs
  int ntile[4][3];                          // 16-row tiles of each matrix
  int kstage[4];                            // K of each stage
  const CUtensorMap* maps;                  // per (layer, projection): codes map, scales map
  // shared-memory layout (bytes from the 1024-aligned base)
  int off_rs, off_bar, off_tbl, off_ft, off_part, off_ey, off_ov, off_xo, off_red, smem;
};
// Per-stage values the epilogue needs, parked in shared memory across the compute phase
// (keeps them out of the registers the MMA loop needs).
struct MkStageInfo {
  const uint16_t* ovals;
  const uint16_t* bias;
  const uint16_t* res;      // residual (o: h, down: h1) or null
  uint16_t* out;
  long long ldo;
  int t0, rows, n_out, ov_smem, nch, ntl;
};
// What a stage needs from its descriptor and its anchor weights, loaded one stage ahead
// (during the previous stage's epilogue and barrier) so the loads are off the critical path.
constexpr int kOvPer = kMOvBytes / 2 / kMThreads;   // anchor weights staged per thread
struct MkPre {
  const uint16_t* ovals;
  const uint16_t* bias;
  const uint16_t* nw;       // RMSNorm weight of the stage input (stages 0 and 2)
  long long ldo;
  int n_out, kcol, has_mask;
  uint16_t ov[kOvPer];
};
// Width (halves) of the scale box of one item: the item's 512/G groups, at least 16 bytes.
__host__ __device__ constexpr int mk_sbox(int G) { return kChunkCodes / G >= 8 ? kChunkCodes / G : 8; }

// The matrix / tile range a CTA serves in stage s.
struct MkWork {
  int m, t0, t1;
};
__device__ __forceinline__ MkWork mk_work(const MkArgs& a, int s, int cta) {
  MkWork w;
  int m = 0;
  while (m + 1 < a.nmat[s] && cta >= a.split[s][m + 1]) ++m;
  const int nc = a.split[s][m + 1] - a.split[s][m], lc = cta - a.split[s][m];
  const int T = a.ntile[s][m];
  w.m = m;
  w.t0 = (int)((int64_t)lc * T / nc);
  w.t1 = (int)((int64_t)(lc + 1) * T / nc);
  return w;
}
// Projection index inside otf2b_decoder_layer (q, k, v, o, gate, up, down) of matrix m of stage s.
__host__ __device__ __forceinline__ int mk_pidx(int s, int m) { return s == 0 ? m : (s == 1 ? 3 : (s == 2 ? 4 + m : 6)); }

__device__ __forceinline__ void mk_prefetch(const MkArgs& a, int l, int s, int tid, MkPre& p) {
  if (l >= a.n_layers) return;
  const MkWork wk = mk_work(a, s, blockIdx.x);
  const otf2b_proj& P = (&a.layers[l].q)[mk_pidx(s, wk.m)];
  p.n_out = (int)P.n_outliers;
  p.ovals = static_cast<const uint16_t*>(P.outlier_vals);
  p.ldo = P.ld_outlier_vals;
  p.bias = static_cast<const uint16_t*>(P.bias);
  p.has_mask = P.mask != nullptr;
  p.nw = static_cast<const uint16_t*>(s == 0 ? a.layers[l].input_norm : (s == 2 ? a.layers[l].post_norm : nullptr));
  const int rows = (wk.t1 - wk.t0) * kRows;
  p.kcol = (rows > 0 && tid < p.n_out) ? (int)__ldg(P.outlier_idx + tid) : 0;
  const bool ov_smem = p.n_out > 0 && rows * p.n_out * 2 <= kMOvBytes;
#pragma unroll
  for (int i = 0; i < kOvPer; ++i) {
    const int e = tid + i * kMThreads;
    p.ov[i] = 0;
    if (ov_smem && e < rows * p.n_out) {
      const int rr = e / p.n_out, j = e - rr * p.n_out;
      p.ov[i] = __ldg(p.ovals + ((int64_t)wk.t0 * kRows + rr) * p.ldo + j);
    }
  }
}

// Grid-wide stage barrier: every CTA adds one after its stage; waiting for target = (stages
// done) x CTAs.  Bounded: on time-out the error flag is raised and the CTA carries on.
__device__ __forceinline__ void mk_arrive(unsigned* bar) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
}
__device__ __forceinline__ void mk_wait(const unsigned* bar, unsigned target) {
  uint32_t i = 0;
  unsigned v;
  while (true) {
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
    if (v >= target) break;
    if (++i >= kMSpin) {
      atomicExch(&g_mk_device_error, 1);
      break;
    }
    __nanosleep(40);
  }
}

// A warp's walk over its weight items: stage by stage, layer by layer, the contiguous run
// [ibeg, iend) of its CTA's (tile, chunk) items.  The copy side runs kMSlots items ahead of
// the compute side over the same sequence.
struct MkCursor {
  int l, s;                 // layer, stage
  int i, iend;              // item, end of this warp's run in the stage
  int nch, t0;              // chunks per tile (K / 512, rounded up), first tile of the CTA
  int mi;                   // index of the stage matrix's codes map (scales map: mi + 1)
};

__device__ __forceinline__ bool mk_enter(const MkArgs& a, MkCursor& c, int warp) {
  // Move to the first stage at or after (c.l, c.s) in which this warp has items.
  while (c.l < a.n_layers) {
    const MkWork w = mk_work(a, c.s, blockIdx.x);
    const int K = a.kstage[c.s];
    const int nch = (K + kChunkCodes - 1) / kChunkCodes;
    const int I = (w.t1 - w.t0) * nch;
    const int ib = warp * I / kMWarps, ie = (warp + 1) * I / kMWarps;
    if (ib < ie) {
      const int mi = (c.l * 7 + mk_pidx(c.s, w.m)) * 2;
      c.i = ib;
      c.iend = ie;
      c.nch = nch;
      c.t0 = w.t0;
      c.mi = mi;
      return true;
    }
    if (++c.s == 4) {
      c.s = 0;
      ++c.l;
    }
  }
  return false;
}

__device__ __forceinline__ void mk_advance(const MkArgs& a, MkCursor& c, int warp) {
  if (++c.i < c.iend) return;
  if (++c.s == 4) {
    c.s = 0;
    ++c.l;
  }
  mk_enter(a, c, warp);
}

// Copy item c.i into its slot: one TMA box of codes (16 rows x 128 bytes, 128-byte
// swizzle) and one box of scales (16 rows x mk_sbox(G) groups starting at a 16-byte
// boundary), both completing on the slot's mbarrier.  Out-of-range parts (a ragged last
// chunk) arrive as zeros.  Issued by one lane.
template <int G>
__device__ __forceinline__ void mk_issue(const MkArgs& a, const MkCursor& c, uint32_t cdst, uint32_t sdst, uint32_t bar) {
  constexpr int SGR = kChunkCodes / G;
  constexpr int SBOX = mk_sbox(G);
  const int tl = c.t0 + c.i / c.nch, ch = c.i % c.nch;
  mbar_arrive_expect_tx(bar, (uint32_t)(kMCodeBytes + kRows * SBOX * 2));
  tma_load_2d(cdst, a.maps + c.mi, ch * kChunk, tl * kRows, bar);
  tma_load_2d(sdst, a.maps + c.mi + 1, ch * SGR / SBOX * SBOX, tl * kRows, bar);
}

// Eight stage-input values at k0 (k0 % 8 == 0) as raw loads: stage 0/2 read h/h1 and the
// RMSNorm weight, stage 1 the attention output (query head j reads KV head j / rep of v),
// stage 3 g and u.  mk_finish8 turns them into the fp16 stage input.
struct MkRaw {
  uint4 x, w;
};
// Vectors written by other CTAs earlier in the same launch are read through L2 only (the
// SM's L1 is not coherent with their stores).
__device__ __forceinline__ uint4 ld_cg16(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint16_t ld_cg_u16(const uint16_t* p) {
  uint16_t v;
  asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ MkRaw mk_load8(const MkArgs& a, int s, int k0, const uint16_t* nw) {
  MkRaw r;
  if (s == 0 || s == 2) {
    const uint16_t* src = s == 0 ? a.h : a.h1;
    r.x = ld_cg16(src + k0);
    r.w = nw ? __ldg(reinterpret_cast<const uint4*>(nw + k0)) : make_uint4(0x3c003c00u, 0x3c003c00u, 0x3c003c00u, 0x3c003c00u);
  } else if (s == 1) {
    const int hd = a.head_dim;
    const int kv = (k0 / hd) / a.rep;
    r.x = ld_cg16(a.v + kv * hd + k0 % hd);
    r.w = make_uint4(0, 0, 0, 0);
  } else {
    r.x = ld_cg16(a.g + k0);
    r.w = ld_cg16(a.u + k0);
  }
  return r;
}
__device__ __forceinline__ float mk_ssq8(const uint4& x) {
  const __half2* h = reinterpret_cast<const __half2*>(&x);
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
  }
  return ss;
}
// RMSNorm: w * fp16(x * r); SiLU gate: fp16(fp16(silu(g)) * u); attention: x as loaded.
__device__ __forceinline__ uint4 mk_finish8(int s, const MkRaw& r, float rs) {
  if (s == 1) return r.x;
  uint4 out;
  const __half* x = reinterpret_cast<const __half*>(&r.x);
  const __half* w = reinterpret_cast<const __half*>(&r.w);
  __half* o = reinterpret_cast<__half*>(&out);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (s == 3) {
      const float gv = __half2float(x[i]);
      o[i] = __hmul(__float2half_rn(gv / (1.0f + expf(-gv))), w[i]);
    } else {
      o[i] = __hmul(w[i], __float2half_rn(__half2float(x[i]) * rs));
    }
  }
  return out;
}

template <int G>
__global__ void __launch_bounds__(kMThreads, 1) k_decode_step(const __grid_constant__ MkArgs a) {
  constexpr int W = words_for(G);
  constexpr int BLK = 16 * W, SL = tbl_sl(W), SB = tbl_sb(W);
  constexpr int NBC = kChunkCodes / BLK;           // blocks per chunk
  constexpr int NBT = NBC / 4;                     // MMA sets per chunk
  constexpr int GSHIFT = G == 32 ? 0 : (G == 64 ? 0 : (G == 128 ? 1 : 2));  // log2(G / BLK)
  constexpr int SGR = kChunkCodes / G;
  constexpr int SBOX = mk_sbox(G);
  constexpr int kScaleBytes = kRows * SBOX * 2;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // 1024-aligned base: the 128-byte swizzle of the code boxes repeats every 1024 bytes.
  uint8_t* const smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  uint8_t* const rcodes = smem + warp * kMSlots * kMCodeBytes;            // this warp's code slots
  uint8_t* const rscales = smem + a.off_rs + warp * kMSlots * kScaleBytes;  // its scale slots
  const uint32_t rbar = smem_u32(smem + a.off_bar) + warp * kMSlots * 8;   // its slot mbarriers
  uint8_t* const tbl = smem + a.off_tbl;
  float2* const sFT = reinterpret_cast<float2*>(smem + a.off_ft);
  float* const part = reinterpret_cast<float*>(smem + a.off_part);
  uint16_t* const xs = reinterpret_cast<uint16_t*>(smem + a.off_part);  // stage input; dead before partials
  uint16_t* const ovs = reinterpret_cast<uint16_t*>(smem + a.off_ov);
  float* const xo = reinterpret_cast<float*>(smem + a.off_xo);
  float* const red = reinterpret_cast<float*>(smem + a.off_red);
  float* const eys = reinterpret_cast<float*>(smem + a.off_ey);   // row-side epilogue terms
  MkStageInfo* const sti = reinterpret_cast<MkStageInfo*>(smem + a.off_red + 64);
  uint8_t* const zblk = smem + a.off_red + 128 + 64;       // 128 zero bytes at 64 mod 128
  for (int i = tid; i < 32; i += kMThreads) reinterpret_cast<uint32_t*>(zblk)[i] = 0u;

  if (lane == 0) {
    for (int k = 0; k < kMSlots; ++k) mbar_init(rbar + 8 * k, 1);
    mbar_fence_init();
  }
  __syncwarp();
  // Copy side: fill the ring with this warp's first kMSlots items (they may belong to any
  // stage; nothing below waits for them before it needs them).
  MkCursor ic{};
  bool ihave = mk_enter(a, ic, warp);
#pragma unroll 1
  for (int k = 0; k < kMSlots; ++k) {
    if (ihave) {
      if (lane == 0) mk_issue<G>(a, ic, smem_u32(rcodes + k * kMCodeBytes), smem_u32(rscales + k * kScaleBytes), rbar + 8 * k);
      mk_advance(a, ic, warp);
      ihave = ic.l < a.n_layers;
    }
  }
  int slot = 0;
  uint32_t phase = 0u;  // bit k: parity of slot k's next completion

  const bool breal = (g >> 1) == t;
  const float bl = a.c1 - a.c0, bh = 0.5f * (a.c2 - a.c0);
  const float cmax = fmaxf(fabsf(bl), fabsf(bh));

  MkPre pre;
  mk_prefetch(a, 0, 0, tid, pre);
#pragma unroll 1
  for (int l = 0; l < a.n_layers; ++l) {
#pragma unroll 1
    for (int s = 0; s < 4; ++s) {
      const MkWork wk = mk_work(a, s, blockIdx.x);
      const int K = a.kstage[s];
      const int nch = (K + kChunkCodes - 1) / kChunkCodes;
      const int nblk = nch * NBC;                  // table blocks incl. the zero tail
      const int ntl = wk.t1 - wk.t0;
      const int n_out = pre.n_out;
      const int rows = ntl * kRows;
      const bool ov_smem = n_out > 0 && rows * n_out * 2 <= kMOvBytes;
      const uint16_t* ovals = pre.ovals;
      const uint16_t* nw = pre.nw;

      // Before the barrier: anchor weights of my rows (loaded one stage ahead).
      if (ov_smem) {
#pragma unroll
        for (int i = 0; i < kOvPer; ++i) {
          const int e = tid + i * kMThreads;
          if (e < rows * n_out) ovs[e] = pre.ov[i];
        }
      }
      const int kcol = pre.kcol;
      const bool zero_anchors = pre.has_mask != 0;
      if (tid == 0) {
        MkStageInfo si;
        si.ovals = ovals;
        si.bias = pre.bias;
        si.res = s == 1 ? a.h : (s == 3 ? a.h1 : nullptr);
        si.out = s == 0 ? (wk.m == 0 ? a.q : (wk.m == 1 ? a.k : a.v))
                        : (s == 1 ? a.h1 : (s == 2 ? (wk.m == 0 ? a.g : a.u) : a.h));
        si.ldo = pre.ldo;
        si.t0 = wk.t0;
        si.rows = rows;
        si.n_out = n_out;
        si.ov_smem = ov_smem ? 1 : 0;
        si.nch = nch;
        si.ntl = ntl;
        *sti = si;
      }

      // Wait until every CTA finished the previous stage.
      if (tid == 0) mk_wait(a.bar, (unsigned)(4 * l + s) * gridDim.x);
      __syncthreads();

      if (ntl > 0) {
        // Stage input into shared memory: every load of the stage issued at once (16 bytes
        // per thread and piece), RMSNorm's sum of squares over the whole vector.
        const int n8 = K / 8;
        constexpr int kU = 3;                      // pieces per thread (K <= 3 * 8 * 512)
        MkRaw raw[kU];
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < kU; ++i) {
          const int v = tid + i * kMThreads;
          if (v < n8) {
            raw[i] = mk_load8(a, s, 8 * v, nw);
            if (s == 0 || s == 2) ss += mk_ssq8(raw[i].x);
          }
        }
        float r = 1.0f;
        if (s == 0 || s == 2) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          if (lane == 0) red[warp] = ss;
          __syncthreads();
          float tot = 0.0f;
#pragma unroll
          for (int w = 0; w < kMWarps; ++w) tot += red[w];
          r = rsqrtf(tot / (float)K + a.eps);
        }
#pragma unroll
        for (int i = 0; i < kU; ++i) {
          const int v = tid + i * kMThreads;
          if (v < n8) reinterpret_cast<uint4*>(xs)[v] = mk_finish8(s, raw[i], r);
        }
        // Zero tail of the last chunk.
        for (int k = K + tid; k < nblk * BLK; k += kMThreads) xs[k] = 0;
        __syncthreads();
        // Anchor activations (unmasked); then the anchor columns leave the table's input
        // (the mask of a SymmetricOTF2BitLinear is exactly "not an anchor column").
        if (tid < n_out) {
          xo[tid] = h2f(xs[kcol]);
          if (zero_anchors) xs[kcol] = 0;
        }
        __syncthreads();
        // Table of the stage input: 4W lanes per block, lane (w, j) owns codes 16w+4i+j.
        constexpr int LPB = 4 * W;
        constexpr int BPP = 32 / LPB;
        const int sub = lane / LPB, ll = lane % LPB;
        const int wq = ll >> 2, j = ll & 3;
#pragma unroll 1
        for (int b0 = 0; b0 < nblk; b0 += BPP * kMWarps) {
          const int bi = b0 + warp * BPP + sub;
          const bool on = bi < nblk;
          float xv[4];
          float mx = 0.0f, sx = 0.0f;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float v = on ? h2f(xs[bi * BLK + 16 * wq + 4 * i + j]) : 0.0f;
            xv[i] = v;
            mx = fmaxf(mx, fabsf(v));
            sx += v;
          }
#pragma unroll
          for (int o = LPB / 2; o > 0; o >>= 1) {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            sx += __shfl_xor_sync(0xffffffffu, sx, o);
          }
          const int E = fixed_point_exp(mx * cmax);
          const float sc = exp2i(E);
          const float kl = bl * sc, kh = bh * sc;
          int hl[4], lo_l[4], hh[4], lo_h[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            split_limbs(rint_small(xv[i] * kl), hl[i], lo_l[i]);
            split_limbs(rint_small(xv[i] * kh), hh[i], lo_h[i]);
          }
          if (on) {
            uint8_t* e = tbl + bi * SB + (wq * 4 + j) * 8;
            *reinterpret_cast<uint2*>(e) =
                make_uint2(pack4(hl[0], hl[1], hl[2], hl[3]), pack4(hh[0], hh[1], hh[2], hh[3]));
            *reinterpret_cast<uint2*>(e + SL) =
                make_uint2(pack4(lo_l[0], lo_l[1], lo_l[2], lo_l[3]), pack4(lo_h[0], lo_h[1], lo_h[2], lo_h[3]));
            if (ll == 0) sFT[bi] = make_float2(exp2i(-E) * (1.0f / 64.0f), a.c0 * sx);
          }
        }
      }
      __syncthreads();  // table and anchor activations ready; the staged input is dead

      // My items of this stage, in the order the copy side issued them.
      {
        const int I = ntl * nch;
        const int ib = warp * I / kMWarps, ie = (warp + 1) * I / kMWarps;
        const uint8_t* bbase = breal ? (tbl + t * NBT * SB + (g & 1) * SL) : zblk;
        const int bstep = breal ? NBC * SB : 0;
        const int sstep = breal ? SB : 0;
        const int s_off = g * SBOX * 2 + 2 * ((t * NBT) >> GSHIFT);
        int C[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int f = 0; f < 4; ++f) C[j][f] = 0;
        uint32_t vprev[4] = {0u, 0u, 0u, 0u};
        float p0 = 0.0f, p1 = 0.0f;
#pragma unroll 1
        for (int it = ib; it < ie; ++it) {
          const int tl = it / nch, cc = it - tl * nch;
          if (!mbar_wait(rbar + 8 * slot, (phase >> slot) & 1u)) atomicExch(&g_mk_device_error, 1);
          phase ^= 1u << slot;
          const uint8_t* ca = rcodes + slot * kMCodeBytes;           // swizzled rows: unit u of row r at (u ^ (r & 7))
          const uint8_t* ps = rscales + slot * kScaleBytes + s_off + 2 * (cc * SGR % SBOX);
          const uint8_t* bp = bbase + cc * bstep;
          const float2* ft = sFT + cc * NBC + t * NBT;
#pragma unroll
          for (int set = 0; set < NBT; ++set) {
            uint32_t cw[W], cw8[W];
            if constexpr (W == 4) {
              const int off = (((2 * t + set) ^ g) << 4);
              const uint4 va = *reinterpret_cast<const uint4*>(ca + g * kChunk + off);
              const uint4 vc = *reinterpret_cast<const uint4*>(ca + (g + 8) * kChunk + off);
              cw[0] = va.x; cw[1] = va.y; cw[2] = va.z; cw[3] = va.w;
              cw8[0] = vc.x; cw8[1] = vc.y; cw8[2] = vc.z; cw8[3] = vc.w;
            } else {
              const int off = (((2 * t + (set >> 1)) ^ g) << 4) + 8 * (set & 1);
              const uint2 va = *reinterpret_cast<const uint2*>(ca + g * kChunk + off);
              const uint2 vc = *reinterpret_cast<const uint2*>(ca + (g + 8) * kChunk + off);
              cw[0] = va.x; cw[1] = va.y;
              cw8[0] = vc.x; cw8[1] = vc.y;
            }
            const uint8_t* bs = bp + set * sstep;
#pragma unroll
            for (int w = 0; w < W; ++w) {
#pragma unroll
              for (int jp = 0; jp < 4; jp += 2) {
                const uint4 bq = *reinterpret_cast<const uint4*>(bs + (w * 4 + jp) * 8);
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                  const int j = jp + hh;
                  const uint32_t b0 = hh ? bq.z : bq.x, b1 = hh ? bq.w : bq.y;
                  const uint32_t ml = 0x01010101u << (2 * j), mh = 0x02020202u << (2 * j);
                  mma_u8s8(C[j], cw[w] & ml, cw8[w] & ml, cw[w] & mh, cw8[w] & mh, b0, b1);
                }
              }
            }
            uint32_t v[4];
#pragma unroll
            for (int f = 0; f < 4; ++f) {
              const uint32_t vn =
                  4u * (4u * (4u * (uint32_t)C[0][f] + (uint32_t)C[1][f]) + (uint32_t)C[2][f]) + (uint32_t)C[3][f];
              v[f] = vn - vprev[f];
              vprev[f] = vn;
            }
            const int so = 2 * (set >> GSHIFT);
            const float sg = h2f(*reinterpret_cast<const uint16_t*>(ps + so));
            const float sg8 = h2f(*reinterpret_cast<const uint16_t*>(ps + 8 * SBOX * 2 + so));
            const float2 FT = ft[set];
            p0 = fmaf(sg, fmaf((float)(int)(v[0] * 256u + v[1]), FT.x, FT.y), p0);
            p1 = fmaf(sg8, fmaf((float)(int)(v[2] * 256u + v[3]), FT.x, FT.y), p1);
          }
          // The slot is consumed: refill it with the next item of this warp's walk.
          __syncwarp();
          if (ihave) {
            if (lane == 0)
              mk_issue<G>(a, ic, smem_u32(rcodes + slot * kMCodeBytes), smem_u32(rscales + slot * kScaleBytes),
                          rbar + 8 * slot);
            mk_advance(a, ic, warp);
            ihave = ic.l < a.n_layers;
          }
          if (++slot == kMSlots) slot = 0;
          // Last item of this tile in my run: leave the tile's partial for the epilogue.
          if (cc == nch - 1 || it == ie - 1) {
            p0 += __shfl_xor_sync(0xffffffffu, p0, 1);
            p0 += __shfl_xor_sync(0xffffffffu, p0, 2);
            p1 += __shfl_xor_sync(0xffffffffu, p1, 1);
            p1 += __shfl_xor_sync(0xffffffffu, p1, 2);
            if (t == 0) {
              float* pp = part + ((tl)*kMWarps + warp) * kRows;
              pp[g] = p0;
              pp[g + 8] = p1;
            }
            p0 = p1 = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
              for (int f = 0; f < 4; ++f) C[j][f] = 0;
#pragma unroll
            for (int f = 0; f < 4; ++f) vprev[f] = 0u;
          }
        }
      }
      // Next stage's descriptor values and anchor weights: loads issued now, used after the
      // epilogue and the barrier.
      mk_prefetch(a, s == 3 ? l + 1 : l, s == 3 ? 0 : s + 1, tid, pre);
      // Row-side terms of the epilogue (anchor dot, bias, residual), computed while other
      // warps may still be on their items.  Stage values come back from shared memory.
      {
        const volatile MkStageInfo* vi = sti;
        const int rows_ = vi->rows;
        if (tid < rows_) {
          const int n_out_ = vi->n_out;
          const int tlc = tid / kRows, rr = tid - tlc * kRows;
          const int64_t row = (int64_t)(vi->t0 + tlc) * kRows + rr;
          float ey = 0.0f;
          if (n_out_ > 0) {
            float d = 0.0f;
            if (vi->ov_smem) {
              const uint16_t* orow = ovs + tid * n_out_;
              for (int j = 0; j < n_out_; ++j) d = fmaf(xo[j], h2f(orow[j]), d);
            } else {
              const uint16_t* orow = vi->ovals + row * vi->ldo;
              for (int j = 0; j < n_out_; ++j) d = fmaf(xo[j], h2f(__ldg(orow + j)), d);
            }
            ey += d;
          }
          const uint16_t* bias = vi->bias;
          const uint16_t* res = vi->res;
          if (bias) ey += h2f(bias[row]);
          if (res) ey += h2f(ld_cg_u16(res + row));
          eys[tid] = ey;   // (the store waits for the loads, so their latency stays before the barrier)
        }
      }
      __syncthreads();  // every partial of the stage is in shared memory

      // Epilogue: one thread per row of my tiles; the partials of the warps whose item runs
      // touched the tile, in warp order.
      {
        const volatile MkStageInfo* vi = sti;
        const int rows_ = vi->rows;
        if (tid < rows_) {
          const int nch_ = vi->nch;
          const int tlc = tid / kRows, rr = tid - tlc * kRows;
          const int64_t row = (int64_t)(vi->t0 + tlc) * kRows + rr;
          const int I = vi->ntl * nch_;
          float y = 0.0f;
#pragma unroll
          for (int w = 0; w < kMWarps; ++w) {
            const int ib = w * I / kMWarps, ie = (w + 1) * I / kMWarps;
            const float pv = part[(tlc * kMWarps + w) * kRows + rr];
            if (ib < ie && ib < (tlc + 1) * nch_ && ie > tlc * nch_) y += pv;
          }
          y += eys[tid];
          y = fminf(fmaxf(y, -65504.0f), 65504.0f);
          vi->out[row] = f2h(y);
        }
      }
      __syncthreads();
      if (tid == 0) mk_arrive(a.bar);
    }
  }
}

}  // namespace otf

// ---------------------------------------------------------------------------------------
// Host side.

namespace {

struct MkLayout {
  int64_t ws_desc, ws_maps, ws_q, ws_k, ws_v, ws_h1, ws_g, ws_u, ws_total;
};

MkLayout mk_ws_layout(const otf2b_decode_dims& d) {
  MkLayout L;
  const int64_t qdim = d.heads * d.head_dim, kvdim = d.kv_heads * d.head_dim;
  int64_t off = 256;  // stage counter
  L.ws_desc = off;  off = otf::align_up(off + d.n_layers * (int64_t)sizeof(otf2b_decoder_layer), 256);
  L.ws_maps = off;  off = otf::align_up(off + d.n_layers * 14 * (int64_t)sizeof(CUtensorMap), 256);
  L.ws_q = off;     off = otf::align_up(off + qdim * 2, 256);
  L.ws_k = off;     off = otf::align_up(off + kvdim * 2, 256);
  L.ws_v = off;     off = otf::align_up(off + kvdim * 2, 256);
  L.ws_h1 = off;    off = otf::align_up(off + d.hidden * 2, 256);
  L.ws_g = off;     off = otf::align_up(off + d.intermediate * 2, 256);
  L.ws_u = off;     off = otf::align_up(off + d.intermediate * 2, 256);
  L.ws_total = off;
  return L;
}

bool dims_ok(const otf2b_decode_dims* d) {
  if (!d || d->n_layers <= 0 || d->hidden <= 0 || d->intermediate <= 0 || d->heads <= 0 || d->kv_heads <= 0 ||
      d->head_dim <= 0 || d->heads % d->kv_heads)
    return false;
  const int64_t G = d->group_size;
  if (!(G == 32 || G == 64 || G == 128 || G == 256)) return false;
  const int64_t qdim = d->heads * d->head_dim;
  if (d->hidden % G || d->intermediate % G || qdim % G) return false;
  if (d->hidden % otf::kRows || d->intermediate % otf::kRows || (d->kv_heads * d->head_dim) % otf::kRows ||
      qdim % otf::kRows)
    return false;
  // each thread stages at most three 8-value pieces of a stage input
  const int64_t kmax = 3 * 8 * otf::kMThreads;
  if (d->hidden > kmax || d->intermediate > kmax || qdim > kmax) return false;
  if (d->head_dim % 8) return false;
  const float lhs = d->codebook[3] - d->codebook[2], rhs = d->codebook[1] - d->codebook[0];
  return fabsf(lhs - rhs) <= 1e-6f * fmaxf(1.0f, fabsf(rhs));
}

int stage_k(const otf2b_decode_dims& d, int s) {
  return (int)(s == 1 ? d.heads * d.head_dim : (s == 3 ? d.intermediate : d.hidden));
}

// Shared memory of the kernel for these dimensions (0 if it does not fit).
struct MkSmem {
  int off_rs, off_bar, off_tbl, off_ft, off_part, off_ey, off_ov, off_xo, off_red, total;
};
MkSmem mk_smem(const otf2b_decode_dims& d) {
  MkSmem m;
  const int G = (int)d.group_size;
  const int W = otf::words_for(G), BLK = 16 * W, SB = otf::tbl_sb(W);
  int nblk = 0;
  for (int s = 0; s < 4; ++s) {
    const int nch = (stage_k(d, s) + otf::kChunkCodes - 1) / otf::kChunkCodes;
    nblk = std::max(nblk, nch * (otf::kChunkCodes / BLK));
  }
  const int64_t slots = (int64_t)otf::kMWarps * otf::kMSlots;
  int64_t off = slots * otf::kMCodeBytes;          // code slots at the 1024-aligned base
  m.off_rs = (int)off;   off += slots * otf::kRows * otf::mk_sbox(G) * 2;
  m.off_bar = (int)off;  off = otf::align_up(off + slots * 8, 128);
  m.off_tbl = (int)off;  off = otf::align_up(off + (int64_t)nblk * SB, 128);
  m.off_ft = (int)off;   off = otf::align_up(off + (int64_t)nblk * 8, 128);
  // partials of the compute phase share their bytes with the staged stage input
  const int64_t part_bytes = (int64_t)otf::kMMaxTiles * otf::kMWarps * otf::kRows * 4;
  const int64_t xs_bytes = (int64_t)nblk * BLK * 2;
  m.off_part = (int)off; off = otf::align_up(off + std::max(part_bytes, xs_bytes), 128);
  m.off_ey = (int)off;   off = otf::align_up(off + otf::kMThreads * 4, 128);
  m.off_ov = (int)off;   off = otf::align_up(off + otf::kMOvBytes, 128);
  m.off_xo = (int)off;   off = otf::align_up(off + otf::kMMaxOut * 4, 128);
  m.off_red = (int)off;  off = off + 384;
  off += 1024;                                     // room to align the base at run time
  m.total = off <= 227 * 1024 ? (int)off : 0;
  return m;
}

bool proj_ok(const otf2b_proj& p, int64_t N, int64_t K, int64_t G) {
  const auto al = [](const void* q, int n) { return reinterpret_cast<uintptr_t>(q) % n == 0; };
  if (!p.packed || !p.scales || p.N != N || p.K != K) return false;
  if (p.ld_packed < K / 4 || p.ld_packed % 16 || !al(p.packed, 16)) return false;
  // TMA boxes: 16-byte aligned bases and row strides
  if (p.ld_scales < K / G || (p.ld_scales * 2) % 16 || !al(p.scales, 16)) return false;
  if (p.mask && !al(p.mask, 2)) return false;
  if (p.n_outliers < 0 || p.n_outliers > otf::kMMaxOut) return false;
  if (p.n_outliers > 0 && (!p.outlier_idx || !p.outlier_vals || p.ld_outlier_vals < p.n_outliers)) return false;
  return true;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    cudaGetLastError();
  }
  return fn;
}

// The two maps of a projection: codes uint8 [N, K/4] with 16 x 128-byte boxes (128-byte
// swizzle), scales fp16 [N, K/G] with 16 x mk_sbox(G) boxes.  Reads past K come back as 0.
bool encode_proj(const otf2b_proj& p, int64_t G, CUtensorMap* maps) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const cuuint32_t es[2] = {1, 1};
  const cuuint64_t cd[2] = {(cuuint64_t)(p.K / 4), (cuuint64_t)p.N};
  const cuuint64_t cs[1] = {(cuuint64_t)p.ld_packed};
  const cuuint32_t cb[2] = {(cuuint32_t)otf::kChunk, (cuuint32_t)otf::kRows};
  if (enc(&maps[0], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(p.packed), cd, cs, cb, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  const cuuint64_t sd[2] = {(cuuint64_t)(p.K / G), (cuuint64_t)p.N};
  const cuuint64_t ss[1] = {(cuuint64_t)(p.ld_scales * 2)};
  const cuuint32_t sb[2] = {(cuuint32_t)otf::mk_sbox((int)G), (cuuint32_t)otf::kRows};
  return enc(&maps[1], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(p.scales), sd, ss, sb, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

namespace otf {
int mk_device_error(int clear);
}

int otf::mk_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, otf::g_mk_device_error, sizeof(int)) != cudaSuccess) {
    otf::set_cuda_error(cudaGetLastError());
    return -1;
  }
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(otf::g_mk_device_error, &z, sizeof(int));
  }
  return v;
}

extern "C" OTF_API int64_t otf2b_decode_workspace_bytes(const otf2b_decode_dims* dims) {
  if (!dims_ok(dims)) return -1;
  return mk_ws_layout(*dims).ws_total;
}

extern "C" OTF_API int otf2b_decode_prepare(const otf2b_decoder_layer* layers, const otf2b_decode_dims* dims,
                                            void* workspace, int64_t workspace_bytes) {
  if (!layers || !workspace || !dims_ok(dims)) return OTF_ERR_INVALID;
  const otf2b_decode_dims& d = *dims;
  const MkLayout L = mk_ws_layout(d);
  if (workspace_bytes < L.ws_total || reinterpret_cast<uintptr_t>(workspace) % 256) return OTF_ERR_INVALID;
  if (mk_smem(d).total == 0) return OTF_ERR_UNSUPPORTED;
  const int64_t G = d.group_size, qdim = d.heads * d.head_dim, kvdim = d.kv_heads * d.head_dim;
  for (int64_t l = 0; l < d.n_layers; ++l) {
    const otf2b_decoder_layer& y = layers[l];
    if (!proj_ok(y.q, qdim, d.hidden, G) || !proj_ok(y.k, kvdim, d.hidden, G) || !proj_ok(y.v, kvdim, d.hidden, G) ||
        !proj_ok(y.o, d.hidden, qdim, G) || !proj_ok(y.gate, d.intermediate, d.hidden, G) ||
        !proj_ok(y.up, d.intermediate, d.hidden, G) || !proj_ok(y.down, d.hidden, d.intermediate, G))
      return OTF_ERR_INVALID;
  }
  int st = otf::check_device();
  if (st != OTF_OK) return st;
  // The kernel zeroes the anchor columns of its staged input instead of multiplying by the
  // mask, so a mask must be exactly "1 except at the anchor columns"; the norms are read
  // 16 bytes at a time.
  std::vector<uint16_t> hm;
  std::vector<int64_t> hi;
  for (int64_t l = 0; l < d.n_layers; ++l) {
    const otf2b_decoder_layer& y = layers[l];
    if ((y.input_norm && reinterpret_cast<uintptr_t>(y.input_norm) % 16) ||
        (y.post_norm && reinterpret_cast<uintptr_t>(y.post_norm) % 16))
      return OTF_ERR_INVALID;
    for (const otf2b_proj* p : {&y.q, &y.k, &y.v, &y.o, &y.gate, &y.up, &y.down}) {
      if (!p->mask) continue;
      hm.resize((size_t)p->K);
      hi.resize((size_t)p->n_outliers);
      cudaError_t e = cudaMemcpy(hm.data(), p->mask, (size_t)p->K * 2, cudaMemcpyDeviceToHost);
      if (e == cudaSuccess && p->n_outliers > 0)
        e = cudaMemcpy(hi.data(), p->outlier_idx, (size_t)p->n_outliers * 8, cudaMemcpyDeviceToHost);
      if (e != cudaSuccess) return otf::set_cuda_error(e);
      std::vector<uint16_t> want((size_t)p->K, 0x3C00);
      for (int64_t j = 0; j < p->n_outliers; ++j) {
        if (hi[j] < 0 || hi[j] >= p->K) return OTF_ERR_INVALID;
        want[(size_t)hi[j]] = 0;
      }
      if (hm != want) return OTF_ERR_UNSUPPORTED;
    }
  }
  std::vector<CUtensorMap> maps((size_t)d.n_layers * 14);
  for (int64_t l = 0; l < d.n_layers; ++l) {
    const otf2b_proj* ps = &layers[l].q;
    for (int pi = 0; pi < 7; ++pi)
      if (!encode_proj(ps[pi], G, &maps[(size_t)(l * 7 + pi) * 2])) return OTF_ERR_UNSUPPORTED;
  }
  cudaError_t e = cudaMemcpy(static_cast<char*>(workspace) + L.ws_desc, layers,
                             (size_t)d.n_layers * sizeof(otf2b_decoder_layer), cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(static_cast<char*>(workspace) + L.ws_maps, maps.data(), maps.size() * sizeof(CUtensorMap),
                   cudaMemcpyHostToDevice);
  return otf::set_cuda_error(e);
}

extern "C" OTF_API int otf2b_decode_step(const otf2b_decode_dims* dims, void* h, void* workspace, void* stream) {
  if (!dims_ok(dims) || !h || !workspace || reinterpret_cast<uintptr_t>(h) % 16) return OTF_ERR_INVALID;
  const otf2b_decode_dims& d = *dims;
  const MkSmem sm = mk_smem(d);
  if (sm.total == 0) return OTF_ERR_UNSUPPORTED;
  int st = otf::check_device();
  if (st != OTF_OK) return st;
  int dev = 0, nsm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int G = (int)d.group_size;
  const void* kfn = G == 32 ? (const void*)otf::k_decode_step<32>
                    : G == 64 ? (const void*)otf::k_decode_step<64>
                              : G == 128 ? (const void*)otf::k_decode_step<128> : (const void*)otf::k_decode_step<256>;
  static thread_local int configured[64][4] = {};
  const int gi = G == 32 ? 0 : G == 64 ? 1 : G == 128 ? 2 : 3;
  if (dev >= 0 && dev < 64 && !configured[dev][gi]) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return otf::set_cuda_error(e);
    configured[dev][gi] = 1;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, otf::kMThreads, (size_t)sm.total) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    return OTF_ERR_UNSUPPORTED;
  }
  const int nc = nsm;  // one CTA per SM, all co-resident (cooperative launch)

  const MkLayout L = mk_ws_layout(d);
  char* ws = static_cast<char*>(workspace);
  otf::MkArgs a = {};
  a.layers = reinterpret_cast<const otf2b_decoder_layer*>(ws + L.ws_desc);
  a.maps = reinterpret_cast<const CUtensorMap*>(ws + L.ws_maps);
  a.n_layers = (int)d.n_layers;
  a.hidden = (int)d.hidden;
  a.inter = (int)d.intermediate;
  a.qdim = (int)(d.heads * d.head_dim);
  a.kvdim = (int)(d.kv_heads * d.head_dim);
  a.head_dim = (int)d.head_dim;
  a.rep = (int)(d.heads / d.kv_heads);
  a.G = G;
  a.c0 = d.codebook[0];
  a.c1 = d.codebook[1];
  a.c2 = d.codebook[2];
  a.c3 = d.codebook[3];
  a.eps = d.eps;
  a.h = static_cast<uint16_t*>(h);
  a.q = reinterpret_cast<uint16_t*>(ws + L.ws_q);
  a.k = reinterpret_cast<uint16_t*>(ws + L.ws_k);
  a.v = reinterpret_cast<uint16_t*>(ws + L.ws_v);
  a.h1 = reinterpret_cast<uint16_t*>(ws + L.ws_h1);
  a.g = reinterpret_cast<uint16_t*>(ws + L.ws_g);
  a.u = reinterpret_cast<uint16_t*>(ws + L.ws_u);
  a.bar = reinterpret_cast<unsigned*>(ws);
  // Stage matrices (rows) and the CTAs each gets, in proportion to its row tiles.
  const int64_t rows[4][3] = {{a.qdim, a.kvdim, a.kvdim}, {a.hidden, 0, 0}, {a.inter, a.inter, 0}, {a.hidden, 0, 0}};
  const int nmat[4] = {3, 1, 2, 1};
  for (int s = 0; s < 4; ++s) {
    a.nmat[s] = nmat[s];
    a.kstage[s] = stage_k(d, s);
    int64_t tot = 0;
    for (int m = 0; m < nmat[s]; ++m) {
      a.ntile[s][m] = (int)(rows[s][m] / otf::kRows);
      tot += a.ntile[s][m];
    }
    int cnt[3] = {0, 0, 0}, used = 0;
    for (int m = 0; m < nmat[s]; ++m) {
      cnt[m] = std::max(1, (int)((int64_t)nc * a.ntile[s][m] / tot));
      used += cnt[m];
    }
    // Hand out (or take back) the remainder from the matrix with the most tiles per CTA.
    while (used != nc) {
      int best = 0;
      for (int m = 1; m < nmat[s]; ++m)
        if ((int64_t)a.ntile[s][m] * cnt[best] > (int64_t)a.ntile[s][best] * cnt[m]) best = m;
      if (used < nc) {
        ++cnt[best];
        ++used;
      } else {
        int worst = -1;
        for (int m = 0; m < nmat[s]; ++m)
          if (cnt[m] > 1 && (worst < 0 || (int64_t)a.ntile[s][m] * cnt[worst] < (int64_t)a.ntile[s][worst] * cnt[m]))
            worst = m;
        if (worst < 0) return OTF_ERR_UNSUPPORTED;
        --cnt[worst];
        --used;
      }
    }
    int c0 = 0;
    for (int m = 0; m < nmat[s]; ++m) {
      a.split[s][m] = c0;
      c0 += cnt[m];
      if ((a.ntile[s][m] + cnt[m] - 1) / cnt[m] > otf::kMMaxTiles) return OTF_ERR_UNSUPPORTED;
    }
    a.split[s][nmat[s]] = c0;
  }
  a.off_rs = sm.off_rs;
  a.off_bar = sm.off_bar;
  a.off_tbl = sm.off_tbl;
  a.off_ft = sm.off_ft;
  a.off_part = sm.off_part;
  a.off_ey = sm.off_ey;
  a.off_ov = sm.off_ov;
  a.off_xo = sm.off_xo;
  a.off_red = sm.off_red;
  a.smem = sm.total;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(a.bar, 0, sizeof(unsigned), s);
  if (e != cudaSuccess) return otf::set_cuda_error(e);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)nc);
  cfg.blockDim = dim3(otf::kMThreads);
  cfg.dynamicSmemBytes = (size_t)sm.total;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (G == 32) e = cudaLaunchKernelEx(&cfg, otf::k_decode_step<32>, a);
  else if (G == 64) e = cudaLaunchKernelEx(&cfg, otf::k_decode_step<64>, a);
  else if (G == 128) e = cudaLaunchKernelEx(&cfg, otf::k_decode_step<128>, a);
  else e = cudaLaunchKernelEx(&cfg, otf::k_decode_step<256>, a);
  return otf::set_cuda_error(e);
}
