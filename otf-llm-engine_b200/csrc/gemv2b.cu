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
// Work split: a thread-block cluster of S CTAs covers one group of row tiles; CTA s of
// the cluster owns K slice s, so it quantises only that slice of the activation table.
// Each warp owns whole 16-row tiles inside its CTA's slice and pipelines its own stages
// of 16 rows x 128 code bytes (512 codes) plus their scales: every lane issues 16-byte
// cp.async copies into one of kSlots shared-memory slots (row pitch 144 bytes, so the
// consumers' 16-byte reads are bank-conflict-free), one commit group per stage, and the
// warp refills a slot as soon as it has consumed it.  No CTA barrier in the main loop.
// A stage is consumed as 8/W "sets": lane quad t takes blocks t*8/W + s, so each set is
// one block-diagonal MMA group over four blocks.  The S K-partials of every row meet
// once, over distributed shared memory, in the CTA that finishes the row (contiguous
// blocks of rows per CTA); its fused epilogue adds the fp16 outlier anchors (their
// weights arrive by one bulk copy issued at kernel entry), bias and residual, clamps and
// stores fp16.
//
// Every wait is bounded; a wait that gives up sets g_otf_device_error (read through
// otf_device_error) and the kernel runs to completion with wrong data instead of hanging.
//
// Reference behaviour replaced: otf_llm/otf_triton_2bit_kernel.py:164-194 (dispatch,
// mask multiply, LUT path), :23-113 (warp GEMV), otf_llm/symmetric_2bit_engine.py:
// 214-235 (bias, outlier anchors, clamp), otf_llm/otf_2bit_quantizer.py:193-221.
#include <cuda.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "otf_common.cuh"
#include "tp_ar.cuh"

namespace otf {

constexpr int kCWarps = 8;                  // warps per CTA (each pipelines its own stages)
constexpr int kThreads = kCWarps * 32;
constexpr int kCThreads = kCWarps * 32;
constexpr int kSlots = 3;                   // stages in flight per warp
constexpr int kMaxCluster = 8;              // K slices per cluster
#ifndef OTF_GEMV_MIN_CTAS
#define OTF_GEMV_MIN_CTAS 2
#endif
constexpr int kMinCtas = OTF_GEMV_MIN_CTAS;  // resident CTAs per SM the register budget targets
constexpr int kOvMax = 32 * 1024;           // largest anchor-weight block staged in shared memory

__device__ int g_otf_device_error;          // set when a bounded wait gives up

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
  int tiles_per_group;  // row tiles per cluster
  int xop;              // OTF_XOP_*: transform applied to x while staging it
  const uint16_t* xaux; // RMSNorm weight or the SiLU gate's second operand
  float eps;            // RMSNorm epsilon
  const ArPeers* ar;    // tensor-parallel peer table (device), or null
  int ar_mode;          // OTF_AR_*: produce rows into the peers' buffers / consume their sum as x
  int ar_buf;           // receive buffer 0 or 1
  uint16_t* ar_out;     // consumer: fp16 copy of the reduced x (written by cluster 0), or null
};

// A group of layers launched together (decode-step fusion: q/k/v or gate/up share an
// input and one launch).  Cluster c serves layer m with prefix[m] <= c < prefix[m+1].
constexpr int kMaxGroup = 4;
struct GroupParams {
  LinearArgs L[kMaxGroup];
  int n;
  int prefix[kMaxGroup + 1];
};


// Rows a CTA of the cluster finishes: tiles are dealt out in contiguous blocks of tpf.
__host__ __device__ inline int tiles_per_finisher(int tiles_per_group, int S) { return ceil_div(tiles_per_group, S); }

// One CTA's shared memory: per-warp pipeline stages (codes, scales, zero points), the
// CTA's slice of the activation table, the staged activation slice, per-block constants,
// the anchor activations, the anchor weights and per-row anchor sums of the rows this CTA
// finishes, the K-partials pushed to it and a few scalars.
struct GemvSmem {
  int64_t stages, tbl, xs, meta, xo, ov, afin, fin, zblk, nrm, bars, total;
  int stage_bytes, stage_scales, stage_zeros, ov_bytes;
};


__host__ __device__ inline GemvSmem gemv_smem_layout(int W, bool zeros, int K, int G, int S, int n_out, int64_t ldo,
                                                      int tiles_per_group) {
  const int BLK = 16 * W, SB = tbl_sb(W);
  const int nch = ceil_div(K, kChunkCodes);
  const int ch_slice = ceil_div(nch, S), blk_slice = ch_slice * (kChunkCodes / BLK);
  const int frows = tiles_per_finisher(tiles_per_group, S) * kRows;
  GemvSmem L;
  L.stage_scales = kRows * kPitch;
  L.stage_zeros = L.stage_scales + kRows * scale_pitch(G);
  L.stage_bytes = L.stage_zeros + (zeros ? kRows * scale_pitch(G) : 0);
  const int64_t ovb = n_out > 0 ? ((int64_t)(frows - 1) * ldo + n_out) * 2 + 32 : 0;
  L.ov_bytes = ovb <= kOvMax ? (int)align_up(ovb, 16) : 0;  // 0: anchors read from global memory
  int64_t off = 0;
  L.stages = off; off = align_up(off + (int64_t)kCWarps * kSlots * L.stage_bytes, 128);
  L.tbl = off;    off = align_up(off + (int64_t)blk_slice * SB, 128);
  L.zblk = off;   off = off + 64 + 128;  // zero block at offset 64 mod 128, 128 bytes long
  off = align_up(off, 16);
  L.xs = off;     off = align_up(off + (int64_t)blk_slice * BLK * 2, 16);
  L.meta = off;   off = align_up(off + 3 * (int64_t)blk_slice * 4, 16);
  L.xo = off;     off = align_up(off + (int64_t)n_out * 4, 16);
  L.ov = off;     off = align_up(off + L.ov_bytes, 16);
  L.afin = off;   off = align_up(off + (int64_t)frows * 4, 16);
  L.fin = off;    off = align_up(off + (int64_t)S * frows * 4, 16);
  L.nrm = off;    off = align_up(off + kMaxCluster * 4 + kCWarps * 4, 16);  // RMSNorm partial sums
  L.bars = off;   off = align_up(off + 8, 16);
  L.total = off;
  return L;
}


__device__ __forceinline__ uint16_t ldg_u16(const uint16_t* p) { return __ldg(p); }

__device__ __forceinline__ void report_wait_failure() { atomicExch(&g_otf_device_error, 1); }

// x transform while staging: x <- w * fp16(x * rsqrt(mean(x^2) + eps)) (Llama RMSNorm) or
// x <- fp16(fp16(silu(x)) * aux) (Llama SiLU gate), then the layer's mask multiply.
// aux_v is the auxiliary operand at this column (has_aux: whether the layer has one).
__device__ __forceinline__ __half xform_v(__half x, int xop, uint16_t aux_v, bool has_aux, float r) {
  if (xop == OTF_XOP_RMSNORM) {
    const __half v = __float2half_rn(__half2float(x) * r);
    return has_aux ? __hmul(__ushort_as_half(aux_v), v) : v;
  }
  if (xop == OTF_XOP_SILU_MUL) {
    const float gv = __half2float(x);
    return __hmul(__float2half_rn(gv / (1.0f + expf(-gv))), __ushort_as_half(aux_v));
  }
  return x;
}


// Where one CTA's activation side lives in shared memory and which slice of the layer it
// owns (the batch-1 kernel's single and grouped launches).
struct XSlice {
  uint8_t* tbl;          // fixed-point table of the K slice (the MMA's B fragments)
  __half* xs;            // staged x slice (fp16)
  float2* sFT;           // per block: (2^-E / 64, c0 * sum x)
  float* sS;             // per block: sum x (zero-point term)
  float* xo;             // x at the anchor columns
  float* afin_sum;       // anchor dot product of each row this CTA finishes
  float* fin;            // K-partials pushed to this CTA: [parts][fin_rows]
  uint8_t* zblk;         // zero block read by the lanes without a real B fragment
  float* nrm;            // RMSNorm partial sums exchanged across the cluster
  const uint8_t* ov;     // anchor weights of the finished rows in shared memory, or null
  uint32_t ov_bar;       // mbarrier of their bulk copy
  int kbeg, nbs, nbs_pad;  // first code of the K slice; real and padded blocks in it
  int S, rank, group;    // cluster size, rank in it, cluster group of the layer
  int frow0, nfin, fin_rows;  // rows this CTA finishes: [frow0, frow0 + nfin)
};

// Everything between the entry and the main loop that depends on the activation, run by the
// kCThreads threads that compute (thread i < nfin also owns finished row frow0 + i): bias,
// the PDL wait, residual, the tensor-parallel consumer's sum, the staged x slice with its
// transform and mask, the RMSNorm statistics over the cluster, the anchor activations, the
// fixed-point table and the anchor dot products.  Returns the row's bias + residual.
template <int W>
__device__ __forceinline__ float gemv_stage_x(const LinearArgs& a, const XSlice& c) {
  constexpr int BLK = 16 * W, SL = tbl_sl(W), SB = tbl_sb(W);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Epilogue inputs of the rows this CTA finishes: thread i takes row c.frow0 + i.
  const bool fin_ok = tid < c.nfin;
  const int frow = c.frow0 + tid;
  float ep = 0.0f;
  if (fin_ok && a.bias) ep += h2f(ldg_u16(a.bias + frow));
  // Anchor columns (independent of the predecessor): thread j < n_out holds column j.
  int kcol = 0;
  if (tid < a.n_out) kcol = (int)__ldg(a.oidx + tid);
  const bool norm = a.xop == OTF_XOP_RMSNORM;
  const bool ar_cons = a.ar_mode == OTF_AR_CONSUME;
  // Mask (and RMSNorm weight) of this thread's first 8-value piece of the slice: constants, so
  // they are requested before the wait and the staging passes below read registers.
  const uint4 kOnes4 = make_uint4(0x3c003c00u, 0x3c003c00u, 0x3c003c00u, 0x3c003c00u);
  uint4 w_pre = kOnes4, m_pre = kOnes4;
  if (tid < c.nbs * BLK / 8) {
    if (norm && a.xaux) w_pre = __ldg(reinterpret_cast<const uint4*>(a.xaux + c.kbeg) + tid);
    if (a.mask) m_pre = __ldg(reinterpret_cast<const uint4*>(a.mask + c.kbeg) + tid);
  }
  // Weights, scales and bias are in flight; from here on we read the predecessor's output.
  pdl_wait();
  if (fin_ok && a.res) ep += h2f(ldg_u16(a.res + frow));
  // Tensor-parallel consumer: x is the sum of every rank's rows in the receive buffer,
  // each word polled until it carries this exchange's tag (bounded per thread).
  const unsigned ar_tg = ar_cons ? ar_tag(a.ar, a.ar_buf) : 0u;
  uint32_t ar_budget = kArSpinLimit;
  int ar_err = 0;
  // x at this thread's anchor column (and the transform's second operand there), issued
  // together with the staging loads below.
  uint32_t x_k = 0u, xaux_k = 0u;
  if (ar_cons) {
    if (tid < a.n_out) x_k = ar_sum1(a.ar, a.ar_buf, kcol, ar_tg, ar_budget, ar_err);
  } else {
    ld_u16_pred(x_k, a.x + kcol, tid < a.n_out);
  }
  ld_u16_pred(xaux_k, a.xaux + kcol, tid < a.n_out && a.xaux != nullptr && a.xop != OTF_XOP_NONE);
  // Stage my slice of x (fp16); padded tail = 0.  The SiLU gate and the mask apply on the
  // way in; RMSNorm first needs the sum of squares of all K, then a second pass.  Every CTA
  // sums the squares of the whole vector itself (the extra reads hit L2 and travel with the
  // slice's), so no cluster exchange sits in the chain; the tensor-parallel consumer, whose x
  // is a sum over the ranks' buffers, combines its slices' partial sums across the cluster.
  const bool ssq_local = norm && !ar_cons;
  float ssq = 0.0f;
  if (ssq_local) {
    // The slice pieces this thread stages (v = t, t + 256) are requested first, then the whole
    // vector in the same fixed thread order in every CTA (pieces t, t + 256, ...), so all loads
    // are in flight together and every CTA sums the squares in one order (the same rnorm bits).
    const uint4* xsl = reinterpret_cast<const uint4*>(a.x + c.kbeg);
    const uint4* xall = reinterpret_cast<const uint4*>(a.x);
    const int nv = a.K / 8, nsl = c.nbs * BLK / 8;
    const uint4 z4 = make_uint4(0, 0, 0, 0);
    const uint4 s0 = tid < nsl ? __ldg(xsl + tid) : z4;
    const uint4 s1 = tid + kCThreads < nsl ? __ldg(xsl + tid + kCThreads) : z4;
    for (int v = tid; v < nv; v += 2 * kCThreads) {
      const uint4 x0 = __ldg(xall + v);
      const uint4 x1 = v + kCThreads < nv ? __ldg(xall + v + kCThreads) : z4;
      const __half2* h0 = reinterpret_cast<const __half2*>(&x0);
      const __half2* h1 = reinterpret_cast<const __half2*>(&x1);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h0[i]);
        ssq = fmaf(f.x, f.x, fmaf(f.y, f.y, ssq));
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h1[i]);
        ssq = fmaf(f.x, f.x, fmaf(f.y, f.y, ssq));
      }
    }
    uint4* xsd = reinterpret_cast<uint4*>(c.xs);
    if (tid < c.nbs_pad * BLK / 8) xsd[tid] = s0;
    if (tid + kCThreads < c.nbs_pad * BLK / 8) xsd[tid + kCThreads] = s1;
    for (int v = tid + 2 * kCThreads; v < c.nbs_pad * BLK / 8; v += kCThreads) xsd[v] = v < nsl ? __ldg(xsl + v) : z4;
  }
  if (!ssq_local) {
    const uint4* xsrc = reinterpret_cast<const uint4*>(a.x + c.kbeg);
    for (int v = tid; v < c.nbs_pad * BLK / 8; v += kCThreads) {
      uint4 xv = make_uint4(0, 0, 0, 0);
      if (v < c.nbs * BLK / 8) {
        if (ar_cons) {
          xv = ar_sum8(a.ar, a.ar_buf, (int64_t)c.kbeg + 8 * v, ar_tg, ar_budget, ar_err);
          if (a.ar_out && c.group == 0) reinterpret_cast<uint4*>(a.ar_out + c.kbeg)[v] = xv;
        } else {
          xv = __ldg(xsrc + v);
        }
        __half2* xh = reinterpret_cast<__half2*>(&xv);
        if (norm) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(xh[i]);
            ssq = fmaf(f.x, f.x, fmaf(f.y, f.y, ssq));
          }
        } else {
          if (a.xop == OTF_XOP_SILU_MUL) {
            const uint4 uv = __ldg(reinterpret_cast<const uint4*>(a.xaux + c.kbeg) + v);
            const __half* uh = reinterpret_cast<const __half*>(&uv);
            __half* e = reinterpret_cast<__half*>(&xv);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float gv = __half2float(e[i]);
              e[i] = __hmul(__float2half_rn(gv / (1.0f + expf(-gv))), uh[i]);
            }
          }
          if (a.mask) {
            const uint4 mv = v == tid ? m_pre : __ldg(reinterpret_cast<const uint4*>(a.mask + c.kbeg) + v);
            const __half2* mh = reinterpret_cast<const __half2*>(&mv);
#pragma unroll
            for (int i = 0; i < 4; ++i) xh[i] = __hmul2(xh[i], mh[i]);
          }
        }
      }
      reinterpret_cast<uint4*>(c.xs)[v] = xv;
    }
  }
  cluster_wait();  // every CTA of the cluster is running: peers' shared memory is live
  float rnorm = 1.0f;
  if (norm) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ssq += __shfl_xor_sync(0xffffffffu, ssq, o);
    if (lane == 0) c.nrm[kMaxCluster + warp] = ssq;
    float tot = 0.0f;
    if (ssq_local) {
      named_barrier_sync(1, kCThreads);
      for (int w = 0; w < kCWarps; ++w) tot += c.nrm[kMaxCluster + w];
    } else {
      named_barrier_sync(1, kCThreads);
      if (tid == 0) {
        float part = 0.0f;
        for (int w = 0; w < kCWarps; ++w) part += c.nrm[kMaxCluster + w];
        for (int q = 0; q < c.S; ++q) st_cluster_f32_plain(mapa_shared(smem_u32(c.nrm + c.rank), (uint32_t)q), part);
      }
      cluster_sync_all();
      for (int q = 0; q < c.S; ++q) tot += c.nrm[q];
    }
    rnorm = rsqrtf(tot / (float)a.K + a.eps);
    for (int v = tid; v < c.nbs * BLK / 8; v += kCThreads) {
      uint4 xv = reinterpret_cast<uint4*>(c.xs)[v];
      __half* e = reinterpret_cast<__half*>(&xv);
      uint4 wv = w_pre, mv = m_pre;                // ones where there is no weight / mask
      if (v != tid) {
        if (a.xaux) wv = __ldg(reinterpret_cast<const uint4*>(a.xaux + c.kbeg) + v);
        if (a.mask) mv = __ldg(reinterpret_cast<const uint4*>(a.mask + c.kbeg) + v);
      }
      const __half* wh = reinterpret_cast<const __half*>(&wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) e[i] = __hmul(wh[i], __float2half_rn(__half2float(e[i]) * rnorm));
      if (a.mask) {
        __half2* xh = reinterpret_cast<__half2*>(&xv);
        const __half2* mh = reinterpret_cast<const __half2*>(&mv);
#pragma unroll
        for (int i = 0; i < 4; ++i) xh[i] = __hmul2(xh[i], mh[i]);
      }
      reinterpret_cast<uint4*>(c.xs)[v] = xv;
    }
  }
  // Anchor activations: the transformed, unmasked x at the anchor columns.
  if (tid < a.n_out)
    c.xo[tid] = __half2float(xform_v(__ushort_as_half((uint16_t)x_k), a.xop, (uint16_t)xaux_k, a.xaux != nullptr, rnorm));
  for (int j = tid + kCThreads; j < a.n_out; j += kCThreads) {
    const int k = (int)__ldg(a.oidx + j);
    const uint16_t av = (a.xaux && a.xop != OTF_XOP_NONE) ? ldg_u16(a.xaux + k) : (uint16_t)0;
    c.xo[j] = __half2float(xform_v(__ushort_as_half(ldg_u16(a.x + k)), a.xop, av, a.xaux != nullptr, rnorm));
  }
  for (int i = tid; i < 32; i += kCThreads) reinterpret_cast<uint32_t*>(c.zblk)[i] = 0u;
  named_barrier_sync(1, kCThreads);  // the staged slice of x is complete
  if (ar_cons) {
    if (ar_err) report_wait_failure();
    if (tid == 0) ar_consumed(a.ar, a.ar_buf);  // every read of the buffer is done
  }
  // Quantise the table slice: 4W lanes per block, lane (w, j) owns codes 16w+4i+j.
  {
    constexpr int LPB = 4 * W;
    constexpr int BPP = 32 / LPB;
    const float bl = a.c1 - a.c0, bh = 0.5f * (a.c2 - a.c0);
    const float cmax = fmaxf(fabsf(bl), fabsf(bh));
    const int sub = lane / LPB, l = lane % LPB;
    const int wq = l >> 2, j = l & 3;
    for (int b0 = 0; b0 < c.nbs_pad; b0 += BPP * kCWarps) {
      const int bi = b0 + warp * BPP + sub;
      const bool on = bi < c.nbs_pad;
      float xv[4];
      float mx = 0.0f, sx = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float v = on ? __half2float(c.xs[bi * BLK + 16 * wq + 4 * i + j]) : 0.0f;
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
      int hl[4], ll[4], hh[4], lh[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        split_limbs(rint_small(xv[i] * kl), hl[i], ll[i]);
        split_limbs(rint_small(xv[i] * kh), hh[i], lh[i]);
      }
      if (on) {
        uint8_t* e = c.tbl + bi * SB + (wq * 4 + j) * 8;
        *reinterpret_cast<uint2*>(e) =
            make_uint2(pack4(hl[0], hl[1], hl[2], hl[3]), pack4(hh[0], hh[1], hh[2], hh[3]));
        *reinterpret_cast<uint2*>(e + SL) =
            make_uint2(pack4(ll[0], ll[1], ll[2], ll[3]), pack4(lh[0], lh[1], lh[2], lh[3]));
        if (l == 0) {
          c.sFT[bi] = make_float2(exp2i(-E) * (1.0f / 64.0f), a.c0 * sx);
          c.sS[bi] = sx;
        }
      }
    }
  }
  named_barrier_sync(1, kCThreads);
  // Anchor dot products of the rows this CTA finishes, one row per thread, from the
  // weights the bulk copy brought in (or from global memory when they did not fit).
  if (a.n_out > 0 && tid < c.nfin) {
    float d = 0.0f;
    if (c.ov) {
      if (!mbar_wait_spin(c.ov_bar, 0u)) report_wait_failure();
      const uint16_t* ovr = reinterpret_cast<const uint16_t*>(c.ov) + (int64_t)tid * a.ldo;
      for (int j = 0; j < a.n_out; ++j) d = fmaf(c.xo[j], h2f(ovr[j]), d);
    } else {
      const uint16_t* ovr = a.ovals + (int64_t)(c.frow0 + tid) * a.ldo;
      for (int j = 0; j < a.n_out; ++j) d = fmaf(c.xo[j], h2f(ldg_u16(ovr + j)), d);
    }
    c.afin_sum[tid] = d;
  }
  return ep;
}

// The finisher: after one cluster barrier (every K-partial has landed in its shared memory)
// thread i sums the parts of row frow0 + i in a fixed order, adds bias, residual and the
// anchor term, and stores fp16 (or hands the fp32 row to the tensor-parallel exchange).
__device__ __forceinline__ void gemv_finish(const LinearArgs& a, const XSlice& c, float ep, int parts) {
  const int tid = threadIdx.x;
  cluster_sync_all();
  const bool ar_prod = a.ar_mode == OTF_AR_PRODUCE;
  if (tid < c.nfin) {
    const int frow = c.frow0 + tid;
    float yv = ep + (a.n_out > 0 ? c.afin_sum[tid] : 0.0f);
    for (int q = 0; q < parts; ++q) yv += c.fin[q * c.fin_rows + tid];
    if (ar_prod) {
      // Tensor-parallel producer: the fp32 row goes to every rank (clamped after the sum).
      ar_put(a.ar, a.ar_buf, frow, yv, ar_tag(a.ar, a.ar_buf));
    } else {
      if (a.clamp) yv = fminf(fmaxf(yv, -65504.0f), 65504.0f);
      a.y[frow] = f2h(yv);
    }
  }
}

template <int G, bool ZEROS>
__device__ __forceinline__ void gemv_body(const LinearArgs& a, const int group) {
  constexpr int W = words_for(G);
  constexpr int BLK = 16 * W, SL = tbl_sl(W), SB = tbl_sb(W);
  constexpr int NBC = kChunkCodes / BLK;           // blocks per stage row (8 or 16)
  constexpr int NBT = NBC / 4;                     // blocks per lane quad = MMA sets per stage
  constexpr int GSHIFT = G == 32 ? 0 : (G == 64 ? 0 : (G == 128 ? 1 : 2));  // log2(G / BLK)
  constexpr int SGR = kChunkCodes / G;             // scale groups per stage row (2..16)
  constexpr int SPITCH = 2 * SGR + 4;              // bytes of scales per stage row (padded)
  static_assert(G == 32 || G == 64 || G == 128 || G == 256, "group size");
  constexpr int kStageScales = kRows * kPitch;     // stage layout: codes, scales, zero points
  constexpr int kStageZeros = kStageScales + kRows * SPITCH;
  constexpr int kStageBytes = kStageZeros + (ZEROS ? kRows * SPITCH : 0);
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = a.K, N = a.N;
  const int nblk = K / BLK, nch = ceil_div(K, kChunkCodes);
  uint32_t cs;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(cs));
  const int S = (int)cs;
  const int rank = (int)cluster_ctarank();
  const int ch_slice = ceil_div(nch, S);
  const int cbeg = min(rank * ch_slice, nch), cend = min(cbeg + ch_slice, nch);
  const int mych = cend - cbeg;                    // stages per tile in my slice
  const int blk0 = cbeg * NBC, blk1 = min(cend * NBC, nblk);
  const int kbeg = blk0 * BLK;
  const int nbs = blk1 - blk0;                     // real blocks in my slice
  const int nbs_pad = mych * NBC;
  const GemvSmem L = gemv_smem_layout(W, ZEROS, K, G, S, a.n_out, a.ldo, a.tiles_per_group);
  uint8_t* tbl = smem + L.tbl;
  __half* xs = reinterpret_cast<__half*>(smem + L.xs);
  float2* sFT = reinterpret_cast<float2*>(smem + L.meta);  // (2^-E/64, c0*sum x) per block
  float* sS = reinterpret_cast<float*>(smem + L.meta) + 2 * nbs_pad;
  float* xo = reinterpret_cast<float*>(smem + L.xo);
  float* afin_sum = reinterpret_cast<float*>(smem + L.afin);
  float* fin = reinterpret_cast<float*>(smem + L.fin);
  uint8_t* zblk = smem + L.zblk + 64;
  const uint32_t ov_bar = smem_u32(smem + L.bars);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ntiles = ceil_div(N, kRows);
  const int tile0 = group * a.tiles_per_group;
  const int gtiles = max(0, min(a.tiles_per_group, ntiles - tile0));
  const int tpf = tiles_per_finisher(a.tiles_per_group, S);
  const int fin_rows = tpf * kRows;
  const int ngrp = K / G;                          // scale groups per row

  // Programmatic dependent launch: let the next kernel in the stream start launching now
  // (no-op without the launch attribute).  Everything this kernel reads from its
  // predecessor's output comes after griddepcontrol.wait below.
  pdl_trigger();

  // Rows this CTA finishes: local rows [rank*fin_rows, +nfin) of the group.
  const int frow0 = tile0 * kRows + rank * fin_rows;
  const int nfin = max(0, min(min(fin_rows, gtiles * kRows - rank * fin_rows), N - frow0));
  // Anchor weights of those rows: one bulk copy of the contiguous byte range, widened to
  // 16-byte boundaries (the widening stays inside the 16-byte segments that hold the first
  // and last bytes, so it never leaves mapped memory).
  const bool ov_smem = a.n_out > 0 && L.ov_bytes > 0 && nfin > 0;
  uint32_t ov_skew = 0;
  if (ov_smem) {
    const uintptr_t lo = reinterpret_cast<uintptr_t>(a.ovals + (int64_t)frow0 * a.ldo);
    const uintptr_t hi = reinterpret_cast<uintptr_t>(a.ovals + (int64_t)(frow0 + nfin - 1) * a.ldo + a.n_out);
    const uintptr_t lo16 = lo & ~(uintptr_t)15, hi16 = (hi + 15) & ~(uintptr_t)15;
    ov_skew = (uint32_t)(lo - lo16);
    if (tid == 0) {
      mbar_init(ov_bar, 1);
      mbar_fence_init();
      mbar_arrive_expect_tx(ov_bar, (uint32_t)(hi16 - lo16));
      bulk_load(smem_u32(smem + L.ov), reinterpret_cast<const void*>(lo16), (uint32_t)(hi16 - lo16), ov_bar);
    }
  }
  cluster_arrive_relaxed();  // paired with cluster_wait() before the first DSMEM store

  // Stage k of warp w = (tile w + 8*(k / mych), chunk cbeg + k % mych).  Lane pair
  // (2r, 2r+1) copies row r of the stage: lane half h takes code bytes [64h, 64h+64) as four
  // 16-byte pieces and scale groups [h*SGR/2, (h+1)*SGR/2) as 4-byte pieces; one commit
  // group per stage.
  const int my_tiles = warp < gtiles ? ceil_div(gtiles - warp, kCWarps) : 0;
  const int nst = my_tiles * mych;
  uint8_t* const wstages = smem + L.stages + warp * kSlots * kStageBytes;
  const int kbytes = K / 4;
  const int lr = lane >> 1, lh = lane & 1;
  const uint32_t cdst0 = smem_u32(wstages) + lr * kPitch + 64 * lh;
  const uint32_t sdst0 = smem_u32(wstages + kStageScales) + lr * SPITCH + lh * SGR;
  const uint32_t zdst0 = smem_u32(wstages + kStageZeros) + lr * SPITCH + lh * SGR;
  // Issue cursor: chunk within the slice and tile, with the tile's row pointers.
  int is_cc = 0, is_tile = 0;
  const uint8_t* crow = a.packed;
  const uint16_t* srow = a.scales;
  const uint16_t* zrow = a.zeros;
  bool row_ok = false;
  auto issue_tile = [&]() {
    const int r = (tile0 + warp + kCWarps * is_tile) * kRows + lr;
    row_ok = r < N;
    const int64_t rr = row_ok ? r : 0;
    crow = a.packed + rr * a.ldp + 64 * lh;
    srow = a.scales + rr * a.lds + lh * (SGR / 2);
    if constexpr (ZEROS) zrow = a.zeros + rr * a.ldz + lh * (SGR / 2);
  };
  auto issue = [&](int slot) {
    const uint32_t so = (uint32_t)(slot * kStageBytes);
    const int ch = cbeg + is_cc;
    const int cb = ch * kChunk;                    // byte offset of the chunk in a row
    const int g0 = ch * SGR;                       // its first scale group
    if (row_ok && cb + kChunk <= kbytes) {         // whole chunk inside the row: no tail
#pragma unroll
      for (int i = 0; i < 4; ++i) cp_async16(cdst0 + so + 16 * i, crow + cb + 16 * i, 16u);
      if (G != 256 || lh == 0) {
#pragma unroll
        for (int i = 0; i < (SGR >= 4 ? SGR / 4 : 1); ++i) {
          cp_async4(sdst0 + so + 4 * i, srow + g0 + 2 * i, 4u);
          if constexpr (ZEROS) cp_async4(zdst0 + so + 4 * i, zrow + g0 + 2 * i, 4u);
        }
      }
    } else {                                       // ragged tail or a row past N: zero fill
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int rem = row_ok ? kbytes - cb - 64 * lh - 16 * i : 0;
        const uint32_t nb = (uint32_t)max(0, min(16, rem));
        cp_async16(cdst0 + so + 16 * i, nb ? crow + cb + 16 * i : a.packed, nb);
      }
      if (G != 256 || lh == 0) {
#pragma unroll
        for (int i = 0; i < (SGR >= 4 ? SGR / 4 : 1); ++i) {
          const int grp = g0 + lh * (SGR / 2) + 2 * i;
          const uint32_t nb = row_ok ? (uint32_t)max(0, min(2 * (ngrp - grp), 4)) : 0u;
          cp_async4(sdst0 + so + 4 * i, nb ? srow + g0 + 2 * i : a.scales, nb);
          if constexpr (ZEROS) cp_async4(zdst0 + so + 4 * i, nb ? zrow + g0 + 2 * i : a.zeros, nb);
        }
      }
    }
    if (++is_cc == mych) {
      is_cc = 0;
      ++is_tile;
      issue_tile();
    }
  };
  issue_tile();
#pragma unroll
  for (int k = 0; k < kSlots; ++k) {
    if (k < nst) issue(k);
    cp_async_commit();
  }

  const XSlice xc{tbl, xs, sFT, sS, xo, afin_sum, fin, zblk, reinterpret_cast<float*>(smem + L.nrm),
                  ov_smem ? smem + L.ov + ov_skew : nullptr, ov_bar, kbeg, nbs, nbs_pad, S, rank, group, frow0, nfin,
                  fin_rows};
  const float ep = gemv_stage_x<W>(a, xc);
  const int g = lane >> 2, t = lane & 3;
  {
    // Main loop: my tiles tl = warp + 8*i, their chunks in order, one stage each.  The MMA
    // accumulators run across a tile's stages; each set's contribution is the difference of
    // the folded sums before and after it (uint32 arithmetic), so no MMA starts from zero.
    const bool breal = (g >> 1) == t;
    const uint8_t* bbase = breal ? (tbl + t * NBT * SB + (g & 1) * SL) : zblk;
    const int bstep = breal ? NBC * SB : 0;         // next chunk
    const int sstep = breal ? SB : 0;               // next set
    const float inv_tpf = 1.0f / (float)tpf;
    // Per-thread offsets inside a stage: codes of row g (row g+8 is 8 pitches further) and
    // the scale of row g for the first set (later sets add 2*(set >> GSHIFT) bytes).
    const int a_off = g * kPitch + 32 * t;
    const int s_off = kStageScales + g * SPITCH + 2 * ((t * NBT) >> GSHIFT);
    const float2* ft0 = sFT + t * NBT;
    const float* sx0 = sS + t * NBT;
    int C[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int f = 0; f < 4; ++f) C[j][f] = 0;
    uint32_t vprev[4] = {0u, 0u, 0u, 0u};
    float p0 = 0.0f, p1 = 0.0f;
    int cc = 0, ct = 0;
    int s = 0;                                      // slot of stage k
    const uint8_t* st = wstages;                    // that slot's base
    for (int k = 0; k < nst; ++k) {
      cp_async_wait<kSlots - 1>();
      __syncwarp();
      const uint8_t* pa = st + a_off;
      const uint8_t* ps = st + s_off;
      const uint8_t* bp = bbase + cc * bstep;
      const float2* ft = ft0 + cc * NBC;
#pragma unroll
      for (int set = 0; set < NBT; ++set) {
        // Codes of rows g and g+8 in block t*NBT + set: W words each.
        uint32_t cw[W], cw8[W];
        if constexpr (W == 4) {
          const uint4 va = *reinterpret_cast<const uint4*>(pa + 16 * set);
          const uint4 vc = *reinterpret_cast<const uint4*>(pa + 8 * kPitch + 16 * set);
          cw[0] = va.x; cw[1] = va.y; cw[2] = va.z; cw[3] = va.w;
          cw8[0] = vc.x; cw8[1] = vc.y; cw8[2] = vc.z; cw8[3] = vc.w;
        } else {
          const uint2 va = *reinterpret_cast<const uint2*>(pa + 8 * set);
          const uint2 vc = *reinterpret_cast<const uint2*>(pa + 8 * kPitch + 8 * set);
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
            for (int h = 0; h < 2; ++h) {
              const int j = jp + h;
              const uint32_t b0 = h ? bq.z : bq.x, b1 = h ? bq.w : bq.y;
              const uint32_t ml = 0x01010101u << (2 * j), mh = 0x02020202u << (2 * j);
              mma_u8s8(C[j], cw[w] & ml, cw8[w] & ml, cw[w] & mh, cw8[w] & mh, b0, b1);
            }
          }
        }
        // Flush the set: fold the classes, take the difference, scale.
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
        const float sg8 = h2f(*reinterpret_cast<const uint16_t*>(ps + 8 * SPITCH + so));
        const float2 FT = ft[set];
        p0 = fmaf(sg, fmaf((float)(int)(v[0] * 256u + v[1]), FT.x, FT.y), p0);
        p1 = fmaf(sg8, fmaf((float)(int)(v[2] * 256u + v[3]), FT.x, FT.y), p1);
        if constexpr (ZEROS) {
          const float Sx = sx0[cc * NBC + set];
          const uint8_t* pz = ps + (kStageZeros - kStageScales);
          p0 = fmaf(h2f(*reinterpret_cast<const uint16_t*>(pz + so)), Sx, p0);
          p1 = fmaf(h2f(*reinterpret_cast<const uint16_t*>(pz + 8 * SPITCH + so)), Sx, p1);
        }
      }
      // Every lane has read the slot (its values fed the MMAs above): refill it.
      __syncwarp();
      if (k + kSlots < nst) issue(s);
      cp_async_commit();
      if (++s == kSlots) {
        s = 0;
        st = wstages;
      } else {
        st += kStageBytes;
      }
      if (++cc == mych) {
        // Tile done: reduce over the lane quad and push the K-partials of rows g, g+8 to the
        // CTA that finishes this tile (q = tl / tpf; exact in float for these sizes).
        const int tl = warp + kCWarps * ct;
        const int q = (int)(((float)tl + 0.5f) * inv_tpf);
        const int slot = (tl - q * tpf) * kRows + g;
        p0 += __shfl_xor_sync(0xffffffffu, p0, 1);
        p0 += __shfl_xor_sync(0xffffffffu, p0, 2);
        p1 += __shfl_xor_sync(0xffffffffu, p1, 1);
        p1 += __shfl_xor_sync(0xffffffffu, p1, 2);
        if (t == 0) {
          const uint32_t f0 = smem_u32(fin + rank * fin_rows + slot);
          st_cluster_f32_plain(mapa_shared(f0, (uint32_t)q), p0);
          st_cluster_f32_plain(mapa_shared(f0 + 8 * 4, (uint32_t)q), p1);
        }
        p0 = p1 = 0.0f;
        cc = 0;
        ++ct;
        // Restart the running sums per tile: a tile's sums stay far inside int32 (at most
        // 2^19 per MMA output times 8 MMAs per stage times K/4096 stages).
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int f = 0; f < 4; ++f) C[j][f] = 0;
#pragma unroll
        for (int f = 0; f < 4; ++f) vprev[f] = 0u;
      }
    }
    cp_async_wait<0>();
    // One cluster barrier: every partial has landed in its finisher's shared memory.
    gemv_finish(a, xc, ep, S);
  }
}

template <int G, bool ZEROS>
__global__ void __launch_bounds__(kThreads, kMinCtas) k_gemv2b(const __grid_constant__ LinearArgs a) {
  uint32_t cs;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(cs));
  gemv_body<G, ZEROS>(a, (int)(blockIdx.x / cs));
}

template <int G, bool ZEROS>
__global__ void __launch_bounds__(kThreads, kMinCtas) k_gemv2b_group(const __grid_constant__ GroupParams gp) {
  uint32_t cs;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(cs));
  const int cid = (int)(blockIdx.x / cs);
  int m = 0;
  while (m + 1 < gp.n && cid >= gp.prefix[m + 1]) ++m;
  gemv_body<G, ZEROS>(gp.L[m], cid - gp.prefix[m]);
}

// ---------------------------------------------------------------------------------------
// Batched decode (2 <= M <= 8 activation rows), same packed layout and work split.  The
// MMA's eight B columns are (batch row, limb) pairs -- four batch rows per column group,
// MB = 4*CG -- so B is dense: every lane reads a useful table fragment, and the four code
// words of one 64-code block fill the 32 k-slots of an MMA (lane quad t holds word t of the
// block, loaded with ldmatrix).  Each lane quad owns one batch row of the accumulators, so
// no cross-lane reduction is needed.  Group sizes of 64, 128 and 256 codes (a block never
// straddles a scale group); no fused input transforms.

// Table bytes of one 64-code block for one column group: 4 rows x 2 limbs x 4 quads x 32 bytes.
constexpr int kBatchTbl = 1024;

struct GemvBatchSmem {
  int64_t stages, tbl, meta, xo, ov, fin, bars, total;
  int stage_bytes, stage_scales, stage_zeros, ov_bytes;
};

__host__ __device__ inline GemvBatchSmem gemv_batch_smem_layout(int CG, bool zeros, int K, int G, int S, int n_out,
                                                                int64_t ldo, int tiles_per_group) {
  const int MB = 4 * CG;
  const int nch = ceil_div(K, kChunkCodes);
  const int ch_slice = ceil_div(nch, S), blk_slice = ch_slice * (kChunkCodes / 64);
  const int frows = tiles_per_finisher(tiles_per_group, S) * kRows;
  GemvBatchSmem L;
  L.stage_scales = kRows * kPitch;
  L.stage_zeros = L.stage_scales + kRows * scale_pitch(G);
  L.stage_bytes = L.stage_zeros + (zeros ? kRows * scale_pitch(G) : 0);
  const int64_t ovb = n_out > 0 ? ((int64_t)(frows - 1) * ldo + n_out) * 2 + 32 : 0;
  L.ov_bytes = ovb <= kOvMax ? (int)align_up(ovb, 16) : 0;
  int64_t off = 0;
  L.stages = off; off = align_up(off + (int64_t)kCWarps * kSlots * L.stage_bytes, 128);
  L.tbl = off;    off = align_up(off + (int64_t)blk_slice * CG * kBatchTbl, 128);
  L.meta = off;   off = align_up(off + (int64_t)blk_slice * MB * 12, 16);   // (F, T) and sum x per (block, row)
  L.xo = off;     off = align_up(off + (int64_t)MB * n_out * 4, 16);
  L.ov = off;     off = align_up(off + L.ov_bytes, 16);
  L.fin = off;    off = align_up(off + (int64_t)S * MB * frows * 4, 16);
  L.bars = off;   off = align_up(off + 8, 16);
  L.total = off;
  return L;
}

template <int G, bool ZEROS, int CG>
__device__ __forceinline__ void gemv_batch_body(const LinearArgs& a, const int group) {
  constexpr int BLK = 64;                          // codes per block (four 32-bit words per row)
  constexpr int NBC = kChunkCodes / BLK;           // 8 blocks per stage row
  constexpr int GSHIFT = G == 64 ? 0 : (G == 128 ? 1 : 2);
  constexpr int SGR = kChunkCodes / G;
  constexpr int SPITCH = 2 * SGR + 4;
  constexpr int MB = 4 * CG;
  constexpr int TBB = CG * kBatchTbl;              // table bytes per block
  static_assert(G == 64 || G == 128 || G == 256, "group size");
  constexpr int kStageScales = kRows * kPitch;
  constexpr int kStageZeros = kStageScales + kRows * SPITCH;
  constexpr int kStageBytes = kStageZeros + (ZEROS ? kRows * SPITCH : 0);
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = a.K, N = a.N, M = a.M;
  const int nblk = K / BLK, nch = ceil_div(K, kChunkCodes);
  uint32_t cs;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(cs));
  const int S = (int)cs;
  const int rank = (int)cluster_ctarank();
  const int ch_slice = ceil_div(nch, S);
  const int cbeg = min(rank * ch_slice, nch), cend = min(cbeg + ch_slice, nch);
  const int mych = cend - cbeg;
  const int blk0 = cbeg * NBC;
  const int kbeg = blk0 * BLK;
  const int nbs = min(cend * NBC, nblk) - blk0;
  const int nbs_pad = mych * NBC;
  const GemvBatchSmem L = gemv_batch_smem_layout(CG, ZEROS, K, G, S, a.n_out, a.ldo, a.tiles_per_group);
  uint8_t* tbl = smem + L.tbl;
  float2* sFT = reinterpret_cast<float2*>(smem + L.meta);          // [block][row]
  float* sS = reinterpret_cast<float*>(smem + L.meta) + 2 * nbs_pad * MB;
  float* xo = reinterpret_cast<float*>(smem + L.xo);               // [row][anchor]
  float* fin = reinterpret_cast<float*>(smem + L.fin);             // [source CTA][row][finished row]
  const uint32_t ov_bar = smem_u32(smem + L.bars);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ntiles = ceil_div(N, kRows);
  const int tile0 = group * a.tiles_per_group;
  const int gtiles = max(0, min(a.tiles_per_group, ntiles - tile0));
  const int tpf = tiles_per_finisher(a.tiles_per_group, S);
  const int fin_rows = tpf * kRows;
  const int ngrp = K / G;

  pdl_trigger();

  const int frow0 = (tile0 + rank * tpf) * kRows;
  const int nfin = max(0, min(min(fin_rows, gtiles * kRows - rank * fin_rows), N - frow0));
  const bool ov_smem = a.n_out > 0 && L.ov_bytes > 0 && nfin > 0;
  uint32_t ov_skew = 0;
  if (ov_smem) {
    const uintptr_t lo = reinterpret_cast<uintptr_t>(a.ovals + (int64_t)frow0 * a.ldo);
    const uintptr_t hi = reinterpret_cast<uintptr_t>(a.ovals + (int64_t)(frow0 + nfin - 1) * a.ldo + a.n_out);
    const uintptr_t lo16 = lo & ~(uintptr_t)15, hi16 = (hi + 15) & ~(uintptr_t)15;
    ov_skew = (uint32_t)(lo - lo16);
    if (tid == 0) {
      mbar_init(ov_bar, 1);
      mbar_fence_init();
      mbar_arrive_expect_tx(ov_bar, (uint32_t)(hi16 - lo16));
      bulk_load(smem_u32(smem + L.ov), reinterpret_cast<const void*>(lo16), (uint32_t)(hi16 - lo16), ov_bar);
    }
  }
  cluster_arrive_relaxed();

  // Stage pipeline: identical to the batch-1 kernel (tile w + 8*(k / mych), chunk k % mych).
  const int my_tiles = warp < gtiles ? ceil_div(gtiles - warp, kCWarps) : 0;
  const int nst = my_tiles * mych;
  uint8_t* const wstages = smem + L.stages + warp * kSlots * kStageBytes;
  const int kbytes = K / 4;
  const int lr = lane >> 1, lh = lane & 1;
  const uint32_t cdst0 = smem_u32(wstages) + lr * kPitch + 64 * lh;
  const uint32_t sdst0 = smem_u32(wstages + kStageScales) + lr * SPITCH + lh * SGR;
  const uint32_t zdst0 = smem_u32(wstages + kStageZeros) + lr * SPITCH + lh * SGR;
  int is_cc = 0, is_tile = 0;
  const uint8_t* crow = a.packed;
  const uint16_t* srow = a.scales;
  const uint16_t* zrow = a.zeros;
  bool row_ok = false;
  auto issue_tile = [&]() {
    const int r = (tile0 + warp + kCWarps * is_tile) * kRows + lr;
    row_ok = r < N;
    const int64_t rr = row_ok ? r : 0;
    crow = a.packed + rr * a.ldp + 64 * lh;
    srow = a.scales + rr * a.lds + lh * (SGR / 2);
    if constexpr (ZEROS) zrow = a.zeros + rr * a.ldz + lh * (SGR / 2);
  };
  auto issue = [&](int slot) {
    const uint32_t so = (uint32_t)(slot * kStageBytes);
    const int ch = cbeg + is_cc;
    const int cb = ch * kChunk;
    const int g0 = ch * SGR;
    if (row_ok && cb + kChunk <= kbytes) {
#pragma unroll
      for (int i = 0; i < 4; ++i) cp_async16(cdst0 + so + 16 * i, crow + cb + 16 * i, 16u);
      if (G != 256 || lh == 0) {
#pragma unroll
        for (int i = 0; i < (SGR >= 4 ? SGR / 4 : 1); ++i) {
          cp_async4(sdst0 + so + 4 * i, srow + g0 + 2 * i, 4u);
          if constexpr (ZEROS) cp_async4(zdst0 + so + 4 * i, zrow + g0 + 2 * i, 4u);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int rem = row_ok ? kbytes - cb - 64 * lh - 16 * i : 0;
        const uint32_t nb = (uint32_t)max(0, min(16, rem));
        cp_async16(cdst0 + so + 16 * i, nb ? crow + cb + 16 * i : a.packed, nb);
      }
      if (G != 256 || lh == 0) {
#pragma unroll
        for (int i = 0; i < (SGR >= 4 ? SGR / 4 : 1); ++i) {
          const int grp = g0 + lh * (SGR / 2) + 2 * i;
          const uint32_t nb = row_ok ? (uint32_t)max(0, min(2 * (ngrp - grp), 4)) : 0u;
          cp_async4(sdst0 + so + 4 * i, nb ? srow + g0 + 2 * i : a.scales, nb);
          if constexpr (ZEROS) cp_async4(zdst0 + so + 4 * i, nb ? zrow + g0 + 2 * i : a.zeros, nb);
        }
      }
    }
    if (++is_cc == mych) {
      is_cc = 0;
      ++is_tile;
      issue_tile();
    }
  };
  issue_tile();
#pragma unroll
  for (int k = 0; k < kSlots; ++k) {
    if (k < nst) issue(k);
    cp_async_commit();
  }

  const int g = lane >> 2, t = lane & 3;
  pdl_wait();
  // Anchor activations per batch row (unmasked x at the anchor columns).
  for (int i = tid; i < M * a.n_out; i += kCThreads) {
    const int m = i / a.n_out, j = i - m * a.n_out;
    xo[m * a.n_out + j] = h2f(ldg_u16(a.x + (int64_t)m * a.ldx + __ldg(a.oidx + j)));
  }
  // Table of the slice: for each (block, batch row), 16 lanes quantise the block's 64 codes
  // (lane (w, j) owns codes 16w + 4i + j) and write the fragment of lane (2*row4 + limb, w).
  {
    const float bl = a.c1 - a.c0, bh = 0.5f * (a.c2 - a.c0);
    const float cmax = fmaxf(fabsf(bl), fabsf(bh));
    const int sub = lane >> 4, l = lane & 15;
    const int wq = l >> 2, j = l & 3;
    const int npairs = nbs_pad * MB;
    for (int p0 = 0; p0 < npairs; p0 += 2 * kCWarps) {
      const int p = p0 + warp * 2 + sub;
      const int bi = p / MB, m = p - (p / MB) * MB;
      const bool live = p < npairs;
      const bool on = live && bi < nbs && m < M;
      float xv[4];
      float mx = 0.0f, sx = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = kbeg + bi * BLK + 16 * wq + 4 * i + j;
        float v = 0.0f;
        if (on) {
          __half xh = __ushort_as_half(ldg_u16(a.x + (int64_t)m * a.ldx + k));
          if (a.mask) xh = __hmul(xh, __ushort_as_half(ldg_u16(a.mask + k)));
          v = __half2float(xh);
        }
        xv[i] = v;
        mx = fmaxf(mx, fabsf(v));
        sx += v;
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        sx += __shfl_xor_sync(0xffffffffu, sx, o);
      }
      const int E = fixed_point_exp(mx * cmax);
      const float sc = exp2i(E);
      const float kl = bl * sc, kh = bh * sc;
      int hl[4], ll[4], hh[4], lh2[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        split_limbs(rint_small(xv[i] * kl), hl[i], ll[i]);
        split_limbs(rint_small(xv[i] * kh), hh[i], lh2[i]);
      }
      if (live) {
        const int cg = m >> 2, m4 = m & 3;
        uint8_t* base = tbl + bi * TBB + cg * kBatchTbl + ((j >> 1) * 16) + (j & 1) * 8;
#pragma unroll
        for (int limb = 0; limb < 2; ++limb) {
          const int gl = 2 * m4 + limb;                 // the lane row (g) that reads this entry
          uint8_t* e = base + (gl * 4 + wq) * 32;
          e = reinterpret_cast<uint8_t*>(reinterpret_cast<uintptr_t>(e) ^ (uintptr_t)(limb * 16));
          *reinterpret_cast<uint2*>(e) = limb == 0 ? make_uint2(pack4(hl[0], hl[1], hl[2], hl[3]), pack4(hh[0], hh[1], hh[2], hh[3]))
                                                   : make_uint2(pack4(ll[0], ll[1], ll[2], ll[3]), pack4(lh2[0], lh2[1], lh2[2], lh2[3]));
        }
        if (l == 0) {
          sFT[bi * MB + m] = make_float2(exp2i(-E) * (1.0f / 64.0f), a.c0 * sx);
          sS[bi * MB + m] = sx;
        }
      }
    }
  }
  named_barrier_sync(1, kCThreads);
  cluster_wait();

  // Main loop.  Running accumulators per column group; each block's contribution is the
  // difference of the folded sums (uint32 arithmetic).
  const uint32_t ldm_off = (uint32_t)((lane & 15) * kPitch + 16 * (lane >> 4));
  const int s_off = kStageScales + g * SPITCH;
  const int lane_tb = (g * 4 + t) * 32;            // my table fragment inside a block / group
  const int swz = (g & 1) * 16;
  const float inv_tpf = 1.0f / (float)tpf;
  int C[CG][4][4];
  uint32_t vprev[CG][4];
#pragma unroll
  for (int c = 0; c < CG; ++c)
#pragma unroll
    for (int f = 0; f < 4; ++f) {
      vprev[c][f] = 0u;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) C[c][jj][f] = 0;
    }
  float pr[CG][2];
#pragma unroll
  for (int c = 0; c < CG; ++c) pr[c][0] = pr[c][1] = 0.0f;
  int cc = 0, ct = 0;
  int s = 0;
  const uint8_t* st = wstages;
  for (int k = 0; k < nst; ++k) {
    cp_async_wait<kSlots - 1>();
    __syncwarp();
    const uint8_t* ps = st + s_off;
#pragma unroll
    for (int bp = 0; bp < NBC / 2; ++bp) {
      uint32_t r[4];
      ldmatrix_x4(smem_u32(st) + ldm_off + 32 * bp, r[0], r[1], r[2], r[3]);
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const int b = 2 * bp + hb;                 // block within the stage
        const uint32_t ra = r[2 * hb], rb = r[2 * hb + 1];
        const int lb = cc * NBC + b;               // block within the slice
        const int so = 2 * (b >> GSHIFT);
        const float sg = h2f(*reinterpret_cast<const uint16_t*>(ps + so));
        const float sg8 = h2f(*reinterpret_cast<const uint16_t*>(ps + 8 * SPITCH + so));
#pragma unroll
        for (int c = 0; c < CG; ++c) {
          const uint8_t* bb = tbl + lb * TBB + c * kBatchTbl + lane_tb;
          const uint4 bq0 = *reinterpret_cast<const uint4*>(bb + (0 ^ swz));
          const uint4 bq1 = *reinterpret_cast<const uint4*>(bb + (16 ^ swz));
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const uint4& bq = jj < 2 ? bq0 : bq1;
            const uint32_t b0 = (jj & 1) ? bq.z : bq.x, b1 = (jj & 1) ? bq.w : bq.y;
            const uint32_t ml = 0x01010101u << (2 * jj), mh = 0x02020202u << (2 * jj);
            mma_u8s8(C[c][jj], ra & ml, rb & ml, ra & mh, rb & mh, b0, b1);
          }
          uint32_t v[4];
#pragma unroll
          for (int f = 0; f < 4; ++f) {
            const uint32_t vn = 4u * (4u * (4u * (uint32_t)C[c][0][f] + (uint32_t)C[c][1][f]) + (uint32_t)C[c][2][f]) +
                                (uint32_t)C[c][3][f];
            v[f] = vn - vprev[c][f];
            vprev[c][f] = vn;
          }
          const float2 FT = sFT[lb * MB + 4 * c + t];
          pr[c][0] = fmaf(sg, fmaf((float)(int)(v[0] * 256u + v[1]), FT.x, FT.y), pr[c][0]);
          pr[c][1] = fmaf(sg8, fmaf((float)(int)(v[2] * 256u + v[3]), FT.x, FT.y), pr[c][1]);
          if constexpr (ZEROS) {
            const float Sx = sS[lb * MB + 4 * c + t];
            const uint8_t* pz = ps + (kStageZeros - kStageScales);
            pr[c][0] = fmaf(h2f(*reinterpret_cast<const uint16_t*>(pz + so)), Sx, pr[c][0]);
            pr[c][1] = fmaf(h2f(*reinterpret_cast<const uint16_t*>(pz + 8 * SPITCH + so)), Sx, pr[c][1]);
          }
        }
      }
    }
    __syncwarp();
    if (k + kSlots < nst) issue(s);
    cp_async_commit();
    if (++s == kSlots) {
      s = 0;
      st = wstages;
    } else {
      st += kStageBytes;
    }
    if (++cc == mych) {
      // Tile done: lane (g, t) holds batch row 4c + t of rows g, g+8; push them.
      const int tl = warp + kCWarps * ct;
      const int q = (int)(((float)tl + 0.5f) * inv_tpf);
      const int slot = (tl - q * tpf) * kRows + g;
#pragma unroll
      for (int c = 0; c < CG; ++c) {
        const int m = 4 * c + t;
        if (m < M) {
          const uint32_t f0 = smem_u32(fin + (rank * MB + m) * fin_rows + slot);
          st_cluster_f32_plain(mapa_shared(f0, (uint32_t)q), pr[c][0]);
          st_cluster_f32_plain(mapa_shared(f0 + 8 * 4, (uint32_t)q), pr[c][1]);
        }
        pr[c][0] = pr[c][1] = 0.0f;
      }
      cc = 0;
      ++ct;
#pragma unroll
      for (int c = 0; c < CG; ++c)
#pragma unroll
        for (int f = 0; f < 4; ++f) {
          vprev[c][f] = 0u;
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) C[c][jj][f] = 0;
        }
    }
  }
  cp_async_wait<0>();
  cluster_sync_all();
  if (ov_smem)
    if (!mbar_wait(ov_bar, 0u)) report_wait_failure();
  // Epilogue: (finished row, batch row) pairs.
  for (int i = tid; i < nfin * M; i += kCThreads) {
    const int m = i / nfin, rr = i - m * nfin;
    const int row = frow0 + rr;
    float yv = 0.0f;
    for (int q = 0; q < S; ++q) yv += fin[(q * MB + m) * fin_rows + rr];
    if (a.n_out > 0) {
      const float* xm = xo + m * a.n_out;
      float d = 0.0f;
      if (ov_smem) {
        const uint16_t* ovr = reinterpret_cast<const uint16_t*>(smem + L.ov + ov_skew) + (int64_t)rr * a.ldo;
        for (int jx = 0; jx < a.n_out; ++jx) d = fmaf(xm[jx], h2f(ovr[jx]), d);
      } else {
        const uint16_t* ovr = a.ovals + (int64_t)row * a.ldo;
        for (int jx = 0; jx < a.n_out; ++jx) d = fmaf(xm[jx], h2f(ldg_u16(ovr + jx)), d);
      }
      yv += d;
    }
    if (a.bias) yv += h2f(ldg_u16(a.bias + row));
    if (a.res) yv += h2f(ldg_u16(a.res + (int64_t)m * a.ldr + row));
    if (a.clamp) yv = fminf(fmaxf(yv, -65504.0f), 65504.0f);
    a.y[(int64_t)m * a.ldy + row] = f2h(yv);
  }
}

template <int G, bool ZEROS, int CG>
__global__ void __launch_bounds__(kThreads, kMinCtas) k_gemv2b_batch(const __grid_constant__ LinearArgs a) {
  uint32_t cs;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(cs));
  gemv_batch_body<G, ZEROS, CG>(a, (int)(blockIdx.x / cs));
}

// ---------------------------------------------------------------------------------------
// Batched and prefill shapes (M >= 16 activation rows) on the 5th-generation tensor cores:
// a real dense contraction, so the weights are dequantised to fp16 tiles in shared memory
// and multiplied by tcgen05.mma (kind::f16, fp32 accumulator in tensor memory).
//
// CTA = 128 weight rows (the MMA M) x NB activation rows (the MMA N), 128 threads.  Per
// 64-code K tile: cp.async brings the rows' 16 code bytes, the scale (and zero-point) pair,
// the mask slice and the x tile (x lands directly in the 128-byte-swizzled K-major B layout);
// thread r then dequantises row r -- W = fp16(c[q] * s) through a byte-permute table, the
// reference's own fp16 dequant (fp32 c*s + z for the asymmetric layout), times the mask --
// into the swizzled A tile; one thread issues four K=16 MMAs and commits them to the slot's
// mbarrier, so the tensor core runs while the next tile is dequantised.  The fp16 anchors are
// extra K tiles of the same accumulation: A = the anchor weights of the rows, B = x gathered
// at the anchor columns.  The epilogue reads the accumulator with tcgen05.ld and adds bias
// and residual.
constexpr int kTcMinRows = 32;    // activation rows from which a layer runs on the tcgen05 GEMM
namespace tc {
constexpr int kRowsT = 128;       // weight rows per CTA = MMA M
constexpr int kKT = 64;           // codes per K tile: one 128-byte row of fp16
constexpr int kSlotsT = 4;        // A/B tile slots
constexpr int kDistT = 2;         // copy prefetch distance (tiles)
constexpr int kThreadsT = 128;
}  // namespace tc

struct TcSmem {
  int64_t a, b, codes, scl, msk, sel, bars, tptr, total;
};

__host__ __device__ inline TcSmem tc_smem_layout(int nb) {
  TcSmem L;
  int64_t off = 0;
  L.a = off;     off += (int64_t)tc::kSlotsT * tc::kRowsT * 128;  // 16 KB per slot, 1024-aligned
  L.b = off;     off += (int64_t)tc::kSlotsT * nb * 128;          // nb rows x 128 B per slot
  L.codes = off; off += (int64_t)tc::kSlotsT * tc::kRowsT * 16;   // 16 code bytes per row
  L.scl = off;   off += (int64_t)tc::kSlotsT * tc::kRowsT * 8;    // scale pair and zero pair per row
  L.msk = off;   off += (int64_t)tc::kSlotsT * 128;               // 64 mask values
  L.sel = off;   off += 256 * 4;                                  // byte -> two permute selectors
  L.bars = off;  off += tc::kSlotsT * 8;
  L.tptr = off;  off += 16;
  L.total = off;
  return L;
}

// Byte-permute selector picking fp16 entries qa and qb of a 4-entry table held in two words.
__host__ __device__ constexpr uint32_t pair_selector(uint32_t qa, uint32_t qb) {
  return (2 * qa) | ((2 * qa + 1) << 4) | ((2 * qb) << 8) | ((2 * qb + 1) << 12);
}

template <int G, bool ZEROS, int NB>
__global__ void __launch_bounds__(tc::kThreadsT, 1) k_gemm2b_tc(const __grid_constant__ LinearArgs a) {
  using namespace tc;
  constexpr int NCOLS = NB < 32 ? 32 : NB;        // tensor-memory columns (power of two >= 32)
  // Instruction descriptor, kind::f16: D fp32, A and B fp16, both K-major, N = NB, M = 128.
  constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(kRowsT >> 4) << 24);
  static_assert(NB % 16 == 0 && NB >= 16 && NB <= 256, "MMA N");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The 128-byte swizzle is keyed to absolute shared-memory address bits: start the tiles on a
  // 1024-byte boundary (the launch adds 1 KB of slack).
  uint8_t* const smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const TcSmem L = tc_smem_layout(NB);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int N = a.N, K = a.K, M = a.M;
  // Split over K: a cluster of S CTAs (S in {1, 2, 4}) shares one 128-row tile; CTA q takes
  // K tiles [kt0, kt1) and the last CTA also the anchor tiles.
  uint32_t csz;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(csz));
  const int S = (int)csz;
  const int q = (int)cluster_ctarank();
  const int row0 = (int)(blockIdx.x / csz) * kRowsT, m0 = blockIdx.y * NB;
  const int nkt_all = ceil_div(K, kKT);
  const int kt0 = (int)(((int64_t)q * nkt_all) / S), kt1 = (int)(((int64_t)(q + 1) * nkt_all) / S);
  const int nkt = kt1 - kt0;                       // my K tiles (local index t -> tile kt0 + t)
  const int nat = (q == S - 1) ? ceil_div(a.n_out, kKT) : 0;  // anchor tiles
  const int ntiles = nkt + nat;
  const int ngrp = K / G;
  uint32_t* sel = reinterpret_cast<uint32_t*>(smem + L.sel);
  const uint32_t bars = smem_u32(smem + L.bars);

  pdl_trigger();
  for (int v = tid; v < 256; v += kThreadsT)
    sel[v] = pair_selector(v & 3, (v >> 2) & 3) | (pair_selector((v >> 4) & 3, (v >> 6) & 3) << 16);
  if (tid == 0) {
    for (int s = 0; s < kSlotsT; ++s) mbar_init(bars + 8 * s, 1);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(smem + L.tptr), NCOLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + L.tptr);
  pdl_wait();

  // Per-thread x-copy geometry (fixed for the whole K loop).
  const int xn0 = tid >> 3, xc = tid & 7;
  const uint32_t xdst0 = (uint32_t)(xn0 * 128 + ((xc ^ (xn0 & 7)) << 4));
  int64_t xoff[NB / 16];
  uint32_t xrows = 0;
#pragma unroll
  for (int j = 0; j < NB / 16; ++j) {
    const int m = m0 + xn0 + 16 * j;
    xrows |= (m < M ? 1u : 0u) << j;
    xoff[j] = (int64_t)(m < M ? m : 0) * a.ldx;
  }
  // Copies of K tile t (t < nkt) into slot t % 4.
  const int r = tid;                               // the weight row this thread dequantises
  const int grow = row0 + r;
  const bool rok = grow < N;
  auto issue = [&](int t) {
    const int slot = t & (kSlotsT - 1);
    const int tg = kt0 + t;                        // global K tile
    const int kb = tg * (kKT / 4);                 // code byte offset of the tile in a row
    const uint32_t ncb = rok ? (uint32_t)max(0, min(16, K / 4 - kb)) : 0u;
    cp_async16(smem_u32(smem + L.codes + (slot * kRowsT + r) * 16), ncb ? a.packed + (int64_t)grow * a.ldp + kb : a.packed,
               ncb);
    const int gp = ((tg * kKT) / G) & ~1;           // even group holding (or preceding) the tile's first group
    const uint32_t nsb = rok ? (uint32_t)max(0, min(4, 2 * (ngrp - gp))) : 0u;
    cp_async4(smem_u32(smem + L.scl + (slot * kRowsT + r) * 8), nsb ? a.scales + (int64_t)grow * a.lds + gp : a.scales,
              nsb);
    if constexpr (ZEROS)
      cp_async4(smem_u32(smem + L.scl + (slot * kRowsT + r) * 8 + 4),
                nsb ? a.zeros + (int64_t)grow * a.ldz + gp : a.zeros, nsb);
    if (a.mask && tid < 8) {
      const int k = tg * kKT + 8 * tid;
      const uint32_t nmb = (uint32_t)max(0, min(16, 2 * (K - k)));
      cp_async16(smem_u32(smem + L.msk + slot * 128 + 16 * tid), nmb ? a.mask + k : a.mask, nmb);
    }
    // x tile: NB rows x 8 pieces of 16 bytes, swizzled (piece c of row n at c ^ (n & 7)).
    // Thread (n0 = tid/8, c = tid%8) copies rows n0 + 16j: same swizzle, 2 KB apart.
    const uint32_t bdst = smem_u32(smem + L.b) + (uint32_t)(slot * NB * 128) + xdst0;
    const int kx = tg * kKT + 8 * xc;
    const uint32_t kbytes_x = (uint32_t)max(0, min(16, 2 * (K - kx)));
    const uint16_t* xs = a.x + kx;
#pragma unroll
    for (int j = 0; j < NB / 16; ++j) {
      const uint32_t nxb = ((xrows >> j) & 1u) ? kbytes_x : 0u;
      cp_async16(bdst + 2048u * j, nxb ? reinterpret_cast<const void*>(xs + xoff[j]) : reinterpret_cast<const void*>(a.x),
                 nxb);
    }
  };
  for (int t = 0; t < kDistT; ++t) {
    if (t < nkt) issue(t);
    cp_async_commit();
  }

  // fp16 codebook entries (the reference's dequant multiplies these by the fp16 scale).
  const __half cbh[4] = {__float2half_rn(a.c0), __float2half_rn(a.c1), __float2half_rn(a.c2), __float2half_rn(a.c3)};
  const uint32_t a_swz_row = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
  for (int t = 0; t < ntiles; ++t) {
    const int slot = t & (kSlotsT - 1);
    // Slot of tile t+2 was last read by the MMAs of tile t-2: wait for them, then refill it.
    if (t + kDistT < ntiles && t >= kDistT) {
      const int tp = t - kDistT;
      if (!mbar_wait(bars + 8 * (tp & (kSlotsT - 1)), (uint32_t)(tp >> 2) & 1u)) report_wait_failure();
    }
    if (t + kDistT < nkt) issue(t + kDistT);
    cp_async_commit();
    cp_async_wait<kDistT>();
    __syncthreads();
    uint8_t* aslot = smem + L.a + (int64_t)slot * kRowsT * 128;
    uint8_t* bslot = smem + L.b + (int64_t)slot * NB * 128;
    if (t < nkt) {
      // Dequantise row r of the tile: 64 codes -> 64 fp16 in 8 pieces of 16 bytes.
      const uint4 cw = *reinterpret_cast<const uint4*>(smem + L.codes + (slot * kRowsT + r) * 16);
      const uint32_t sp = *reinterpret_cast<const uint32_t*>(smem + L.scl + (slot * kRowsT + r) * 8);
      const uint32_t zp = ZEROS ? *reinterpret_cast<const uint32_t*>(smem + L.scl + (slot * kRowsT + r) * 8 + 4) : 0u;
      const int g_first = ((kt0 + t) * kKT) / G;
      uint32_t lut[2][2];                          // [scale group half][table word]
#pragma unroll
      for (int hsel = 0; hsel < (G == 32 ? 2 : 1); ++hsel) {
        // Codes [32*hsel, 32*hsel + 32) of the tile belong to group g_first + (G == 32 ? hsel : 0).
        const int gi = g_first + ((G == 32) ? hsel : 0);
        const uint16_t sb = (uint16_t)((gi & 1) ? (sp >> 16) : (sp & 0xFFFFu));
        __half e[4];
        if constexpr (ZEROS) {
          const uint16_t zb = (uint16_t)((gi & 1) ? (zp >> 16) : (zp & 0xFFFFu));
#pragma unroll
          for (int q = 0; q < 4; ++q)
            e[q] = __float2half_rn(fmaf(__half2float(cbh[q]), h2f(sb), h2f(zb)));
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) e[q] = __hmul(cbh[q], __ushort_as_half(sb));
        }
        lut[hsel][0] = (uint32_t)__half_as_ushort(e[0]) | ((uint32_t)__half_as_ushort(e[1]) << 16);
        lut[hsel][1] = (uint32_t)__half_as_ushort(e[2]) | ((uint32_t)__half_as_ushort(e[3]) << 16);
      }
      if constexpr (G != 32) {
        lut[1][0] = lut[0][0];
        lut[1][1] = lut[0][1];
      }
      const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
      for (int c = 0; c < 8; ++c) {                // piece c: code bytes 2c, 2c+1 -> 8 fp16
        const int hsel = c >> 2;
        uint32_t o[4];
#pragma unroll
        for (int bb = 0; bb < 2; ++bb) {
          const uint32_t byte = (words[c >> 1] >> (8 * (2 * (c & 1) + bb))) & 0xFFu;
          const uint32_t sv = sel[byte];
          o[2 * bb] = __byte_perm(lut[hsel][0], lut[hsel][1], sv & 0xFFFFu);
          o[2 * bb + 1] = __byte_perm(lut[hsel][0], lut[hsel][1], sv >> 16);
        }
        *reinterpret_cast<uint4*>(aslot + a_swz_row + ((c ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      // The mask (0 at the anchor columns, else 1) multiplies x: zero those columns of the x
      // tile (a handful per layer) instead of scaling every weight.
      if (a.mask && tid < kKT) {
        const __half mv = *reinterpret_cast<const __half*>(smem + L.msk + slot * 128 + 2 * tid);
        if (__half2float(mv) != 1.0f) {
          const int kc = tid >> 3, ke = tid & 7;
          for (int n = 0; n < NB; ++n) {
            __half* e = reinterpret_cast<__half*>(bslot + n * 128 + ((kc ^ (n & 7)) << 4)) + ke;
            *e = __hmul(*e, mv);
          }
        }
      }
    } else {
      // Anchor tile: A row r = the row's anchor weights [64*ta, 64*ta + 64), B row n = x of
      // activation row m0+n at those anchor columns; zeros past n_out.
      const int ta = t - nkt;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int j0 = ta * kKT + 8 * c + 2 * i;
          const uint32_t lo = (rok && j0 < a.n_out) ? ldg_u16(a.ovals + (int64_t)grow * a.ldo + j0) : 0u;
          const uint32_t hi = (rok && j0 + 1 < a.n_out) ? ldg_u16(a.ovals + (int64_t)grow * a.ldo + j0 + 1) : 0u;
          o[i] = lo | (hi << 16);
        }
        *reinterpret_cast<uint4*>(aslot + a_swz_row + ((c ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      for (int i = tid; i < NB * 8; i += kThreadsT) {
        const int n = i >> 3, c = i & 7;
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int j0 = ta * kKT + 8 * c + 2 * q;
          const bool mok = m0 + n < M;
          const uint32_t lo = (mok && j0 < a.n_out) ? ldg_u16(a.x + (int64_t)(m0 + n) * a.ldx + __ldg(a.oidx + j0)) : 0u;
          const uint32_t hi =
              (mok && j0 + 1 < a.n_out) ? ldg_u16(a.x + (int64_t)(m0 + n) * a.ldx + __ldg(a.oidx + j0 + 1)) : 0u;
          o[q] = lo | (hi << 16);
        }
        *reinterpret_cast<uint4*>(bslot + n * 128 + ((c ^ (n & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    // Generic-proxy stores (and landed copies) must be visible to the tensor core's reads.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before_sync();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after_sync();
      const uint32_t abase = smem_u32(aslot), bbase = smem_u32(bslot);
#pragma unroll
      for (int kk = 0; kk < kKT / 16; ++kk)
        tc_mma_f16(tmem, tc_desc_sw128(abase + 32 * kk), tc_desc_sw128(bbase + 32 * kk), kIdesc,
                   (t > 0 || kk > 0) ? 1u : 0u);
      tc_commit(bars + 8 * slot);
    }
  }
  cp_async_wait<0>();
  // The last commit covers every MMA: wait for it, then read the accumulator.
  if (ntiles > 0) {
    const int tl = ntiles - 1;
    if (!mbar_wait(bars + 8 * (tl & (kSlotsT - 1)), (uint32_t)(tl >> 2) & 1u)) report_wait_failure();
  }
  tc_fence_after_sync();
  // Warp w reads tensor-memory lanes 32w..32w+31 = weight rows row0 + 32w + lane.
  const int lrow = 32 * warp + lane;
  const int orow = row0 + lrow;
  auto finish = [&](int row, int m, float acc) {
    if (row < N && m < M) {
      float yv = acc;
      if (a.bias) yv += h2f(ldg_u16(a.bias + row));
      if (a.res) yv += h2f(ldg_u16(a.res + (int64_t)m * a.ldr + row));
      if (a.clamp) yv = fminf(fmaxf(yv, -65504.0f), 65504.0f);
      a.y[(int64_t)m * a.ldy + row] = f2h(yv);
    }
  };
  if (S == 1) {
#pragma unroll 1
    for (int c0 = 0; c0 < NB; c0 += 8) {
      uint32_t v[8];
      tmem_ld8(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 8; ++j) finish(orow, m0 + c0 + j, __uint_as_float(v[j]));
    }
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, NCOLS);
  } else {
    // Every CTA of the cluster is past its last MMA before any shared memory is reused.
    cluster_sync_all();
    // CTA o owns rows [o*128/S, (o+1)*128/S): warp w's 32 rows belong to CTA w*S/4.  Partials
    // land in the owner's (now idle) A-tile area as recv[source][owned row][column] fp32.
    const int rows_own = kRowsT / S;
    const int owner = warp * S / 4;
    float* recv = reinterpret_cast<float*>(smem + L.a);
#pragma unroll 1
    for (int c0 = 0; c0 < NB; c0 += 8) {
      uint32_t v[8];
      tmem_ld8(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, v);
      tmem_wait_ld();
      const uint32_t dst = smem_u32(recv + ((q * rows_own + (lrow - owner * rows_own)) * NB + c0));
      const uint32_t rdst = mapa_shared(dst, (uint32_t)owner);
      asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rdst), "r"(v[0]), "r"(v[1]), "r"(v[2]),
                   "r"(v[3]) : "memory");
      asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rdst + 16), "r"(v[4]), "r"(v[5]),
                   "r"(v[6]), "r"(v[7]) : "memory");
    }
    tc_fence_before_sync();
    cluster_sync_all();
    if (warp == 0) tmem_dealloc(tmem, NCOLS);
    // Owned rows: sum the S partials in rank order (deterministic), then the epilogue.
    for (int i = tid; i < rows_own * NB; i += kThreadsT) {
      const int rr = i / NB, c = i - rr * NB;
      float acc = 0.0f;
      for (int src = 0; src < S; ++src) acc += recv[(src * rows_own + rr) * NB + c];
      finish(row0 + q * rows_own + rr, m0 + c, acc);
    }
  }
}


// ---------------------------------------------------------------------------------------
// Batched and prefill shapes with the dequantised weights in tensor memory (k_gemm2b_tmem):
// the weight-only-quantised GEMM in its tcgen05 form, for symmetric layers with G = 32 or 64
// and 16-byte aligned code, scale and activation rows.
//
// CTA = 128 weight rows (MMA M) x NB activation rows (MMA N), eleven warps:
//  * warp 0 streams 512-code "super-stages" (128 rows x 128 code bytes, 128-byte swizzle, and
//    the rows' scales) into ring 1 with tensor copies, before the programmatic-dependent-launch
//    wait (weights do not depend on the previous kernel);
//  * warp 1 streams the x tile of each 64-code K tile (NB rows x 128 bytes, 128-byte swizzle:
//    the MMA's B operand as it lands) into ring 2;
//  * warps 3-10 dequantise: thread (quarter, half) turns 32 codes of row 32*quarter + lane into
//    fp16 -- W = fp16(c[q] * s) through a byte-permute table, the reference's own fp16 dequant,
//    times the mask where it is not 1 -- and stores them with tcgen05.st into the K tile's A
//    buffer in tensor memory (a warp reaches only its own 32 lanes: quarter = warp % 4);
//  * warp 2 issues the tile's four K=16 tcgen05.mma (A from tensor memory, B from shared
//    memory) and commits them to the slot's empty barrier, which frees the A buffer and the
//    x tile together.
// The fp32 accumulator is in tensor memory as well; the dequant warps read it back for the
// epilogue (bias, residual, clamp).  The fp16 anchors are extra K tiles of the same
// accumulation (A = the rows' anchor weights, B = x at the anchor columns).  Split K over a
// cluster of S CTAs as in k_gemm2b_tc, in whole super-stages.  Every wait is bounded.
namespace tm {
constexpr int kRowsW = 128;       // weight rows per CTA = MMA M
constexpr int kKT = 64;           // codes per K tile
constexpr int kSS = 8;            // K tiles per super-stage (one 128-byte row of codes)
constexpr int kNS1 = 3;           // super-stage slots
constexpr int kNA = 4;            // A buffers in tensor memory (K tiles in flight)
constexpr int kMaxNX = 16;        // x-tile slots in shared memory (the host sizes the ring)
constexpr int kWarps = 11;
constexpr int kThr = kWarps * 32;
constexpr int kDeq = 8;           // dequant warps 3..10
}  // namespace tm

struct alignas(64) TmParams {
  CUtensorMap cmap;  // codes uint8 [N, K/4]: 128 x 128 boxes, 128-byte swizzle
  CUtensorMap smap;  // scales fp16 [N, K/G]: (512/G) x 128 boxes
  CUtensorMap xmap;  // x fp16 [M, K]: 64 x NB boxes, 128-byte swizzle
  LinearArgs a;
};

// x-tile slots for NB activation rows: a 32 KB ring, between 4 and 16 slots.
__host__ __device__ constexpr int tm_nx(int nb) {
  return (32 * 1024) / (nb * 128) < 4 ? 4 : ((32 * 1024) / (nb * 128) > tm::kMaxNX ? tm::kMaxNX : (32 * 1024) / (nb * 128));
}

struct TmSmem {
  int64_t codes, xt, scl, sel, amask, bars, tptr, total;
};

// nkt_max: K tiles of the largest K slice of the cluster.
__host__ __device__ inline TmSmem tm_smem_layout(int nb, int G, int nkt_max) {
  TmSmem L;
  int64_t off = 0;
  const int nx = tm_nx(nb);
  L.codes = off; off += (int64_t)tm::kNS1 * tm::kRowsW * 128;                 // 16 KB per slot
  L.xt = off;    off += (int64_t)(nx > 4 ? nx : 4) * nb * 128;              // nb rows x 128 B per slot
  L.scl = off;   off = align_up(off + (int64_t)tm::kNS1 * tm::kRowsW * 2 * (tm::kSS * tm::kKT / G), 128);
  L.sel = off;   off += 256 * 16 * 4;                                        // selectors, 16 copies
  L.amask = off; off = align_up(off + (int64_t)nkt_max * 8, 16);            // columns whose mask is not 1
  L.bars = off;  off = align_up(off + (2 * tm::kNS1 + 2 * tm::kMaxNX + 2 * tm::kNA + 1) * 8, 16);
  L.tptr = off;  off += 16;
  L.total = off;
  return L;
}

template <int G, int NB>
__global__ void __launch_bounds__(tm::kThr, 2) k_gemm2b_tmem(const __grid_constant__ TmParams p) {
  using namespace tm;
  static_assert(G == 32 || G == 64, "group size");
  static_assert(NB % 16 == 0 && NB >= 16 && NB <= 256, "MMA N");
  // Independent fp32 accumulators: the MMAs into one accumulator form a dependent chain, so
  // consecutive K=16 steps go round-robin to NACC of them (summed in the epilogue).
  constexpr int NACC = NB <= 32 ? 4 : (NB <= 128 ? 2 : 1);
  constexpr int ACOL = NACC * NB;                             // first A-buffer column
  constexpr int NCOLS = ACOL + kNA * 32 <= 256 ? 256 : 512;  // accumulators + A buffers (power of two)
  constexpr int NX = tm_nx(NB);
  constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(kRowsW >> 4) << 24);
  constexpr int SROW = 2 * (kSS * kKT / G);                   // scale bytes per row per super-stage
  const LinearArgs& a = p.a;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The 128-byte swizzle is keyed to absolute shared-memory address bits (1 KB of slack).
  uint8_t* const smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int N = a.N, K = a.K, M = a.M;
  uint32_t csz;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(csz));
  const int S = (int)csz;
  const int q = (int)cluster_ctarank();
  const int row0 = (int)(blockIdx.x / csz) * kRowsW, m0 = blockIdx.y * NB;
  const int nkt_all = ceil_div(K, kKT), nss_all = ceil_div(nkt_all, kSS);
  const int ss0 = (q * nss_all) / S, ss1 = ((q + 1) * nss_all) / S;
  const int kt0 = ss0 * kSS, kt1 = min(ss1 * kSS, nkt_all);
  const int nkt = max(0, kt1 - kt0), nss = ss1 - ss0;
  const int nat = (q == S - 1) ? ceil_div(a.n_out, kKT) : 0;  // anchor tiles
  const int ntiles = nkt + nat;
  const TmSmem L = tm_smem_layout(NB, G, ceil_div(nss_all, S) * kSS);
  uint8_t* const codes = smem + L.codes;
  uint8_t* const xt = smem + L.xt;
  const uint8_t* const scl = smem + L.scl;
  uint32_t* const sel = reinterpret_cast<uint32_t*>(smem + L.sel);
  uint32_t* const amask = reinterpret_cast<uint32_t*>(smem + L.amask);
  const uint32_t full1 = smem_u32(smem + L.bars), empty1 = full1 + 8 * kNS1;
  const uint32_t xfull = empty1 + 8 * kNS1, xempty = xfull + 8 * kMaxNX;
  const uint32_t afull = xempty + 8 * kMaxNX, aempty = afull + 8 * kNA;
  const uint32_t done = aempty + 8 * kNA;

  pdl_trigger();
  // Selector table in 16 copies (entry v of copy c at word 16 v + c; lane l reads copy l % 16,
  // so a warp's lookups meet at most two to a bank): byte v of four codes -> the byte-permute
  // selectors of their two fp16 pairs.
  for (int i = tid; i < 256 * 16; i += kThr) {
    const int v = i >> 4;
    sel[i] = pair_selector(v & 3, (v >> 2) & 3) | (pair_selector((v >> 4) & 3, (v >> 6) & 3) << 16);
  }
  for (int i = tid; i < 2 * nkt; i += kThr) amask[i] = 0u;
  if (tid == 0) {
    for (int i = 0; i < kNS1; ++i) {
      mbar_init(full1 + 8 * i, 1);
      mbar_init(empty1 + 8 * i, kDeq);
    }
    for (int i = 0; i < NX; ++i) {
      mbar_init(xfull + 8 * i, 1);
      mbar_init(xempty + 8 * i, 1);
    }
    for (int i = 0; i < kNA; ++i) {
      mbar_init(afull + 8 * i, kDeq);
      mbar_init(aempty + 8 * i, 1);
    }
    mbar_init(done, 1);
    mbar_fence_init();
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(smem + L.tptr), NCOLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  // Columns of my K range whose mask is not 1 (the anchors): their weights get the mask value.
  if (a.mask)
    for (int k = kt0 * kKT + tid; k < min(kt1 * kKT, K); k += kThr)
      if (h2f(ldg_u16(a.mask + k)) != 1.0f) atomicOr(&amask[2 * (k / kKT - kt0) + ((k % kKT) >> 5)], 1u << (k & 31));
  __syncthreads();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + L.tptr);

  if (warp == 0) {
    // Ring 1: codes and scales of super-stage j into slot j % 2.
    if (lane == 0) {
      for (int j = 0; j < nss; ++j) {
        const int sl = j % kNS1;
        if (j >= kNS1 && !mbar_wait_sleep(empty1 + 8 * sl, (uint32_t)((j / kNS1) - 1) & 1u)) report_wait_failure();
        mbar_arrive_expect_tx(full1 + 8 * sl, (uint32_t)(kRowsW * 128 + kRowsW * SROW));
        tma_load_2d(smem_u32(codes + sl * kRowsW * 128), &p.cmap, (ss0 + j) * 128, row0, full1 + 8 * sl);
        tma_load_2d(smem_u32(scl + sl * kRowsW * SROW), &p.smap, (ss0 + j) * (kSS * kKT / G), row0, full1 + 8 * sl);
      }
    }
    __syncwarp();  // lanes 1-31 wait here, converged, for lane 0's loop (not at the CTA barrier)
  } else if (warp == 1) {
    // Ring 2: the x tile of K tile t into slot t % NX, once the MMAs of tile t - NX are done.
    if (lane == 0) {
      pdl_wait();  // x is the previous kernel's output
      int sl = 0;
      uint32_t ph = 0;
      for (int t = 0; t < nkt; ++t) {
        if (t >= NX && !mbar_wait_spin(xempty + 8 * sl, ph ^ 1u)) report_wait_failure();
        mbar_arrive_expect_tx(xfull + 8 * sl, (uint32_t)(NB * 128));
        tma_load_2d(smem_u32(xt + sl * NB * 128), &p.xmap, (kt0 + t) * kKT, m0, xfull + 8 * sl);
        if (++sl == NX) {
          sl = 0;
          ph ^= 1u;
        }
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    // MMA issue: K tile t = four K=16 steps, A from tensor memory, B from the x tile.
    if (lane == 0) {
      int xs = 0;
      uint32_t xph = 0;
      for (int t = 0; t < ntiles; ++t) {
        const int as = t & (kNA - 1);
        if (t < nkt && !mbar_wait_spin(xfull + 8 * xs, xph)) report_wait_failure();
        if (!mbar_wait_spin(afull + 8 * as, (uint32_t)(t / kNA) & 1u)) report_wait_failure();
        tc_fence_after_sync();
        const uint32_t bbase = smem_u32(xt + xs * NB * 128);
#pragma unroll
        for (int kk = 0; kk < kKT / 16; ++kk) {
          const int step = t * (kKT / 16) + kk;     // K=16 step index; accumulator step % NACC
          tc_mma_f16_ta(tmem + (uint32_t)((step % NACC) * NB), tmem + (uint32_t)(ACOL + 32 * as + 8 * kk),
                        tc_desc_sw128(bbase + 32 * kk), kIdesc, step >= NACC ? 1u : 0u);
        }
        tc_commit(xempty + 8 * xs);
        tc_commit(aempty + 8 * as);
        if (++xs == NX) {
          xs = 0;
          xph ^= 1u;
        }
      }
      tc_commit(done);
    }
    __syncwarp();
  } else {
    // Dequant warps.
    const int dq = warp - 3, h = dq >> 2, quarter = warp & 3;
    const int r = 32 * quarter + lane;             // the weight row of this thread
    const int grow = row0 + r;
    const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
    const __half2 cb01 = __halves2half2(__float2half_rn(a.c0), __float2half_rn(a.c1));
    const __half2 cb23 = __halves2half2(__float2half_rn(a.c2), __float2half_rn(a.c3));
    const uint32_t* const selr = sel + (lane & 15);
    // Software-pipelined: the tensor-memory store of tile t completes while tile t + 1 is
    // dequantised; its afull arrival follows the wait.
    int pend = -1;                                   // tile whose store is in flight
    auto publish = [&](int tp) {
      tmem_wait_st();
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(afull + 8 * (tp & (kNA - 1)));
    };
    for (int t = 0; t < nkt; ++t) {
      const int j = t >> 3, kt = t & (kSS - 1);
      const int s1 = j % kNS1, sl = t & (kNA - 1);
      if (kt == 0 && !mbar_wait_spin(full1 + 8 * s1, (uint32_t)(j / kNS1) & 1u)) report_wait_failure();
      // 32 codes: bytes [8h, 8h + 8) of 16-byte piece kt of row r (piece c at c ^ (r & 7)).
      const uint2 cw = *reinterpret_cast<const uint2*>(codes + s1 * kRowsW * 128 + r * 128 + ((kt ^ (r & 7)) << 4) +
                                                      8 * h);
      const int grp = G == 64 ? kt : 2 * kt + h;     // scale group within the super-stage
      const __half sh = *reinterpret_cast<const __half*>(scl + s1 * kRowsW * SROW + r * SROW + 2 * grp);
      const __half2 s2 = __halves2half2(sh, sh);
      const __half2 e01 = __hmul2(cb01, s2), e23 = __hmul2(cb23, s2);
      const uint32_t lut0 = *reinterpret_cast<const uint32_t*>(&e01), lut1 = *reinterpret_cast<const uint32_t*>(&e23);
      uint32_t o[16];
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        const uint32_t w = b < 4 ? cw.x : cw.y;
        const uint32_t sv = selr[((w >> (8 * (b & 3))) & 0xFFu) * 16];
        o[2 * b] = __byte_perm(lut0, lut1, sv & 0xFFFFu);
        o[2 * b + 1] = __byte_perm(lut0, lut1, sv >> 16);
      }
      const uint32_t mb = amask[2 * t + h];
      if (mb) {                                      // rare: anchor columns (mask 0) or other masks
        const uint16_t* mrow = a.mask + (kt0 + t) * kKT + 32 * h;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if ((mb >> (2 * i)) & 3u) {
            const __half2 m2 = __halves2half2(__ushort_as_half(ldg_u16(mrow + 2 * i)),
                                              __ushort_as_half(ldg_u16(mrow + 2 * i + 1)));
            __half2 v = *reinterpret_cast<const __half2*>(&o[i]);
            v = __hmul2(v, m2);
            o[i] = *reinterpret_cast<const uint32_t*>(&v);
          }
        }
      }
      if (kt == kSS - 1 || t == nkt - 1) {           // the super-stage's codes are all read
        __syncwarp();
        if (lane == 0) mbar_arrive(empty1 + 8 * s1);
      }
      if (pend >= 0) publish(pend);
      if (t >= kNA && !mbar_wait_spin(aempty + 8 * sl, (uint32_t)((t / kNA) - 1) & 1u)) report_wait_failure();
      tmem_st16(tmem + lane_base + (uint32_t)(ACOL + 32 * sl + 16 * h), o);
      pend = t;
    }
    if (pend >= 0) publish(pend);
    if (nat > 0) pdl_wait();
    for (int ta = 0; ta < nat; ++ta) {
      // Anchor tile: A = anchor weights [64 ta + 32 h, +32) of row r; B = x at those anchors.
      const int t = nkt + ta, sl = t & (kNA - 1), xs = t % NX;
      if (t >= kNA && !mbar_wait_spin(aempty + 8 * sl, (uint32_t)((t / kNA) - 1) & 1u)) report_wait_failure();
      if (t >= NX && !mbar_wait_spin(xempty + 8 * xs, (uint32_t)((t / NX) - 1) & 1u)) report_wait_failure();
      uint32_t o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j0 = ta * kKT + 32 * h + 2 * i;
        const uint32_t lo = (grow < N && j0 < a.n_out) ? ldg_u16(a.ovals + (int64_t)grow * a.ldo + j0) : 0u;
        const uint32_t hi = (grow < N && j0 + 1 < a.n_out) ? ldg_u16(a.ovals + (int64_t)grow * a.ldo + j0 + 1) : 0u;
        o[i] = lo | (hi << 16);
      }
      tmem_st16(tmem + lane_base + (uint32_t)(ACOL + 32 * sl + 16 * h), o);
      // x rows n < NB at anchors [64 ta, +64): 8 fp16 per 16-byte piece, 128-byte swizzle.
      for (int i = tid - 3 * 32; i < NB * 8; i += kDeq * 32) {
        const int n = i >> 3, c = i & 7;
        uint32_t v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j0 = ta * kKT + 8 * c + 2 * u;
          const bool mok = m0 + n < M;
          const uint32_t lo = (mok && j0 < a.n_out) ? ldg_u16(a.x + (int64_t)(m0 + n) * a.ldx + __ldg(a.oidx + j0)) : 0u;
          const uint32_t hi =
              (mok && j0 + 1 < a.n_out) ? ldg_u16(a.x + (int64_t)(m0 + n) * a.ldx + __ldg(a.oidx + j0 + 1)) : 0u;
          v[u] = lo | (hi << 16);
        }
        *reinterpret_cast<uint4*>(xt + xs * NB * 128 + n * 128 + ((c ^ (n & 7)) << 4)) = make_uint4(v[0], v[1], v[2], v[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tmem_wait_st();
      tc_fence_before_sync();
      named_barrier_sync(1, kDeq * 32);              // every x row of the tile is written
      if (lane == 0) mbar_arrive(afull + 8 * sl);
    }
  }

  // Epilogue: the dequant warps read the accumulator (their own 32 lanes, half the columns each).
  auto finish = [&](int row, int m, float acc) {
    if (row < N && m < M) {
      float yv = acc;
      if (a.bias) yv += h2f(ldg_u16(a.bias + row));
      if (a.res) yv += h2f(ldg_u16(a.res + (int64_t)m * a.ldr + row));
      if (a.clamp) yv = fminf(fmaxf(yv, -65504.0f), 65504.0f);
      a.y[(int64_t)m * a.ldy + row] = f2h(yv);
    }
  };
  const bool deq = warp >= 3;
  const int h = (warp - 3) >> 2, quarter = warp & 3;
  const int lrow = 32 * quarter + lane;
  // Columns c0..c0+7 of this thread's row, summed over the accumulators (0 without MMAs).
  auto acc_ld8 = [&](int c0, float (&acc)[8]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
#pragma unroll
    for (int u = 0; u < NACC; ++u) {
      uint32_t v[8];
      tmem_ld8(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(u * NB + c0), v);
      tmem_wait_ld();
      if (ntiles > 0)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += __uint_as_float(v[j]);
    }
  };
  pdl_wait();  // every thread that stores y or reads the residual waits for the previous kernel
  if (deq) {
    if (ntiles > 0 && !mbar_wait_spin(done, 0u)) report_wait_failure();
    tc_fence_after_sync();
  }
  if (S == 1) {
    if (deq) {
#pragma unroll 1
      for (int c0 = h * (NB / 2); c0 < (h + 1) * (NB / 2); c0 += 8) {
        float acc[8];
        acc_ld8(c0, acc);
#pragma unroll
        for (int j = 0; j < 8; ++j) finish(row0 + lrow, m0 + c0 + j, acc[j]);
      }
    }
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 2) tmem_dealloc(tmem, NCOLS);
  } else {
    // Every CTA of the cluster is past its last MMA before the x area is reused: partials of
    // row r go to CTA r / (128/S) as recv[source][owned row][column] fp32.
    cluster_sync_all();
    const int rows_own = kRowsW / S;
    float* recv = reinterpret_cast<float*>(xt);
    if (deq) {
      const int owner = lrow / rows_own;
#pragma unroll 1
      for (int c0 = h * (NB / 2); c0 < (h + 1) * (NB / 2); c0 += 8) {
        float acc[8];
        acc_ld8(c0, acc);
        uint32_t v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __float_as_uint(acc[j]);
        const uint32_t dst = smem_u32(recv + ((q * rows_own + (lrow - owner * rows_own)) * NB + c0));
        const uint32_t rdst = mapa_shared(dst, (uint32_t)owner);
        asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rdst), "r"(v[0]), "r"(v[1]), "r"(v[2]),
                     "r"(v[3]) : "memory");
        asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rdst + 16), "r"(v[4]), "r"(v[5]),
                     "r"(v[6]), "r"(v[7]) : "memory");
      }
    }
    tc_fence_before_sync();
    cluster_sync_all();
    if (warp == 2) tmem_dealloc(tmem, NCOLS);
    for (int i = tid; i < rows_own * NB; i += kThr) {
      const int rr = i / NB, c = i - rr * NB;
      float acc = 0.0f;
      for (int src = 0; src < S; ++src) acc += recv[(src * rows_own + rr) * NB + c];
      finish(row0 + q * rows_own + rr, m0 + c, acc);
    }
  }
}

// Portable CUDA-core kernel: any M, any G dividing K with G % 4 == 0, any codebook.
// One warp per output row, lanes stride over packed bytes; MT activation rows per launch.
template <int MT>
__global__ void __launch_bounds__(256) k_linear_generic(const LinearArgs a, int m0) {
  pdl_trigger();
  pdl_wait();
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
  pdl_trigger();
  pdl_wait();
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
const void* ar_device_table(const otf_ar* ar);  // tp_ar.cu
int64_t ar_max_elems(const otf_ar* ar);         // tp_ar.cu
int ar_device_error(int clear);                 // tp_ar.cu
int mk_device_error(int clear);                 // decode_step.cu
int attn_device_error(int clear);               // attention.cu
int head_device_error(int clear);               // int8_ops.cu

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

// Launch geometry of one layer: K slices per cluster (S) and row tiles per cluster.
struct GemvPlan {
  int S, groups, tpg;
  int64_t smem;
};

static int gemv_S(int K) {
  const int nch = ceil_div(K, kChunkCodes);
  int S = std::max(1, std::min(kMaxCluster, nch));
  while (S > 1 && ceil_div(nch, S) * (S - 1) >= nch) --S;  // every slice non-empty
  return S;
}

// Row groups for a layer given a budget of clusters: every warp holds at least one tile,
// and each CTA finishes at most one row per thread.
template <int G>
static GemvPlan gemv_plan(const LinearArgs& a, int S, int budget) {
  constexpr int W = words_for(G);
  GemvPlan p;
  p.S = S;
  const int ntiles = ceil_div(a.N, kRows);
  const int max_tpg = S * (kCThreads / kRows);
  const int min_groups = std::max(1, ceil_div(ntiles, max_tpg));
  int groups = std::max(min_groups, std::min(std::max(budget, 1), ceil_div(ntiles, kCWarps)));
  p.tpg = ceil_div(ntiles, groups);
  p.groups = ceil_div(ntiles, p.tpg);
  p.smem = gemv_smem_layout(W, a.zeros != nullptr, a.K, G, S, a.n_out, a.ldo, p.tpg).total;
  return p;
}

// Largest number of co-resident clusters of S CTAs of a kernel for a given dynamic shared
// memory size (cached: the occupancy query is a host call we do not want per launch).
static int max_active_clusters_of(const void* kernel, int S, int64_t smem, int threads = kThreads) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, int, int64_t, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t bucket = align_up(smem, 4096);
  const auto key = std::make_tuple(dev, kernel, S, bucket, threads);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)S, 1, 1);
  cfg.blockDim = dim3((unsigned)threads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)bucket;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int mc = 0;
  if (cudaOccupancyMaxActiveClusters(&mc, kernel, &cfg) != cudaSuccess || mc <= 0) mc = std::max(1, num_sms() / S);
  cudaGetLastError();
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = mc;
  return mc;
}

// Largest number of co-resident clusters of S CTAs for a given dynamic shared memory
// size (cached: the occupancy query is a host call we do not want per launch).
template <int G, bool ZEROS>
static int max_active_clusters(int S, int64_t smem) {
  return max_active_clusters_of(reinterpret_cast<const void*>(k_gemv2b<G, ZEROS>), S, smem);
}

template <int G, bool ZEROS>
static int configure_kernels() {
  static thread_local int configured_dev[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured_dev[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv2b<G, ZEROS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k_gemv2b_group<G, ZEROS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return set_cuda_error(e);
    configured_dev[dev] = 1;
  }
  return OTF_OK;
}

template <int G, bool ZEROS>
static int launch_gemv(LinearArgs a, cudaStream_t st) {
  int rc = configure_kernels<G, ZEROS>();
  if (rc != OTF_OK) return rc;
  const int S = gemv_S(a.K);
  // No more clusters than can be resident at once: a second wave would double the time.
  GemvPlan p = gemv_plan<G>(a, S, 1 << 20);
  for (int pass = 0; pass < 3; ++pass) {
    if (p.smem > 227 * 1024) return OTF_ERR_UNSUPPORTED;
    const GemvPlan q = gemv_plan<G>(a, S, max_active_clusters<G, ZEROS>(S, p.smem));
    if (q.groups == p.groups) break;
    p = q;
  }
  if (p.smem > 227 * 1024 || tiles_per_finisher(p.tpg, S) * kRows > kCThreads) return OTF_ERR_UNSUPPORTED;
  a.tiles_per_group = p.tpg;
  return set_cuda_error(launch_pdl(k_gemv2b<G, ZEROS>, dim3((unsigned)(p.groups * S)), dim3(kThreads),
                                   (size_t)p.smem, st, (unsigned)S, a));
}

// Layers with the same K, G and zero-point use launched as one grid: cluster budgets are
// split in proportion to each layer's row tiles so that the whole group is co-resident.
template <int G, bool ZEROS>
static int launch_gemv_group(LinearArgs* L, int n, cudaStream_t st) {
  int rc = configure_kernels<G, ZEROS>();
  if (rc != OTF_OK) return rc;
  static thread_local GroupParams gp;  // large: keep it off the host stack
  gp.n = n;
  const int S = gemv_S(L[0].K);
  int64_t smem_hi = 0;
  int tiles_total = 0;
  for (int m = 0; m < n; ++m) {
    tiles_total += ceil_div(L[m].N, kRows);
    smem_hi = std::max(smem_hi, gemv_plan<G>(L[m], S, 1 << 20).smem);
  }
  GemvPlan plans[kMaxGroup];
  int64_t smem = smem_hi;
  for (int pass = 0; pass < 3; ++pass) {
    if (smem > 227 * 1024) return OTF_ERR_UNSUPPORTED;
    const int mc = max_active_clusters<G, ZEROS>(S, smem);
    int64_t s2 = 0;
    for (int m = 0; m < n; ++m) {
      const int tiles = ceil_div(L[m].N, kRows);
      const int budget = std::max(1, (int)((int64_t)mc * tiles / std::max(tiles_total, 1)));
      plans[m] = gemv_plan<G>(L[m], S, budget);
      s2 = std::max(s2, plans[m].smem);
    }
    if (s2 == smem) break;
    smem = s2;
  }
  int clusters = 0;
  for (int m = 0; m < n; ++m) {
    if (tiles_per_finisher(plans[m].tpg, S) * kRows > kCThreads) return OTF_ERR_UNSUPPORTED;
    gp.L[m] = L[m];
    gp.L[m].tiles_per_group = plans[m].tpg;
    gp.prefix[m] = clusters;
    clusters += plans[m].groups;
  }
  gp.prefix[n] = clusters;
  if (smem > 227 * 1024) return OTF_ERR_UNSUPPORTED;
  return set_cuda_error(launch_pdl(k_gemv2b_group<G, ZEROS>, dim3((unsigned)(clusters * S)), dim3(kThreads),
                                   (size_t)smem, st, (unsigned)S, gp));
}

// Batched layers (2 <= M <= 4*CG): same geometry rules as the batch-1 launch.
template <int G, bool ZEROS, int CG>
static int launch_gemv_batch(LinearArgs a, cudaStream_t st) {
  static thread_local int configured_dev[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured_dev[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv2b_batch<G, ZEROS, CG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return set_cuda_error(e);
    configured_dev[dev] = 1;
  }
  const int S = gemv_S(a.K);
  const int ntiles = ceil_div(a.N, kRows);
  auto plan = [&](int budget, int& groups, int& tpg) {
    groups = std::max(1, std::min(std::max(budget, 1), ceil_div(ntiles, kCWarps)));
    tpg = ceil_div(ntiles, groups);
    groups = ceil_div(ntiles, tpg);
    return gemv_batch_smem_layout(CG, ZEROS, a.K, G, S, a.n_out, a.ldo, tpg).total;
  };
  int groups = 0, tpg = 0;
  int64_t smem = plan(1 << 20, groups, tpg);
  for (int pass = 0; pass < 3; ++pass) {
    if (smem > 227 * 1024) return OTF_ERR_UNSUPPORTED;
    int g2 = 0, t2 = 0;
    const int64_t s2 = plan(max_active_clusters_of(reinterpret_cast<const void*>(k_gemv2b_batch<G, ZEROS, CG>), S, smem),
                            g2, t2);
    if (g2 == groups) break;
    groups = g2;
    tpg = t2;
    smem = s2;
  }
  if (smem > 227 * 1024) return OTF_ERR_UNSUPPORTED;
  a.tiles_per_group = tpg;
  return set_cuda_error(launch_pdl(k_gemv2b_batch<G, ZEROS, CG>, dim3((unsigned)(groups * S)), dim3(kThreads),
                                   (size_t)smem, st, (unsigned)S, a));
}

template <int G, bool ZEROS, int NB>
static int launch_gemm_tc(const LinearArgs& a, cudaStream_t st) {
  const int64_t smem = tc_smem_layout(NB).total + 1024;
  static thread_local int configured_dev[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured_dev[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm2b_tc<G, ZEROS, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return set_cuda_error(e);
    configured_dev[dev] = 1;
  }
  // Split K over a cluster of S in {1, 2, 4} CTAs while the grid is under two CTAs per SM and
  // every CTA keeps at least 8 K tiles.
  const int rt = ceil_div(a.N, tc::kRowsT), bt = ceil_div(a.M, NB), nkt = ceil_div(a.K, tc::kKT);
  int S = 1;
  while (S < 4 && (int64_t)rt * bt * S * 2 <= 2 * num_sms() && nkt >= 16 * S) S *= 2;
  const dim3 grid((unsigned)(rt * S), (unsigned)bt);
  return set_cuda_error(launch_pdl(k_gemm2b_tc<G, ZEROS, NB>, grid, dim3(tc::kThreadsT), (size_t)smem, st,
                                   (unsigned)S, a));
}

bool encode_tiled_2d(void* map, int elem_bytes, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                     uint32_t box_inner, uint32_t box_rows, bool swizzle128);  // capi.cu

// The tensor-memory GEMM (k_gemm2b_tmem) for activation rows 9.. and the layers it takes:
// symmetric, G = 32 or 64, 16-byte aligned code, scale and activation rows (tensor copies).
constexpr int kTmMinRows = 9;
static bool tm_variant(const LinearArgs& a) {
  const auto al = [](const void* p, int n) { return reinterpret_cast<uintptr_t>(p) % n == 0; };
  return !a.zeros && (a.G == 32 || a.G == 64) && a.xop == OTF_XOP_NONE && al(a.packed, 16) && a.ldp % 16 == 0 &&
         al(a.scales, 16) && (a.lds * 2) % 16 == 0 && al(a.x, 16) && (a.ldx * 2) % 16 == 0 &&
         (!a.mask || al(a.mask, 2)) && a.K % 8 == 0;
}

template <int G, int NB>
static int launch_gemm_tmem(const LinearArgs& a, cudaStream_t st) {
  static thread_local int configured_dev[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured_dev[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm2b_tmem<G, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return set_cuda_error(e);
    configured_dev[dev] = 1;
  }
  // Split K over a cluster of S in {1, 2, 4} CTAs (whole super-stages) while the grid stays
  // within two CTAs per SM and every CTA keeps at least two super-stages.
  const int rt = ceil_div(a.N, tm::kRowsW), bt = ceil_div(a.M, NB);
  const int nss = ceil_div(ceil_div(a.K, tm::kKT), tm::kSS);
  int S = 1;
  while (S < 4 && (int64_t)rt * bt * S * 2 <= 2 * num_sms() && nss >= 4 * S) S *= 2;
  const int64_t smem = tm_smem_layout(NB, G, ceil_div(nss, S) * tm::kSS).total + 1024;
  if (smem > 227 * 1024) return OTF_ERR_UNSUPPORTED;
  static thread_local TmParams p;  // three tensor maps + arguments, kept off the stack
  if (!encode_tiled_2d(&p.cmap, 1, a.packed, (uint64_t)(a.K / 4), (uint64_t)a.N, (uint64_t)a.ldp, 128u,
                       (uint32_t)tm::kRowsW, true) ||
      !encode_tiled_2d(&p.smap, 2, a.scales, (uint64_t)(a.K / G), (uint64_t)a.N, (uint64_t)(a.lds * 2),
                       (uint32_t)(tm::kSS * tm::kKT / G), (uint32_t)tm::kRowsW, false) ||
      !encode_tiled_2d(&p.xmap, 2, a.x, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)(a.ldx * 2), (uint32_t)tm::kKT,
                       (uint32_t)NB, true))
    return OTF_ERR_UNSUPPORTED;
  p.a = a;
  const dim3 grid((unsigned)(rt * S), (unsigned)bt);
  return set_cuda_error(launch_pdl(k_gemm2b_tmem<G, NB>, grid, dim3(tm::kThr), (size_t)smem, st, (unsigned)S, p));
}

template <int G>
static int launch_tmem_g(const LinearArgs& a, cudaStream_t s) {
  if (a.M <= 16) return launch_gemm_tmem<G, 16>(a, s);
  if (a.M <= 32) return launch_gemm_tmem<G, 32>(a, s);
  if (a.M <= 64) return launch_gemm_tmem<G, 64>(a, s);
  if (a.M <= 128) return launch_gemm_tmem<G, 128>(a, s);
  return launch_gemm_tmem<G, 256>(a, s);
}

static int launch_tmem(const LinearArgs& a, cudaStream_t s) {
  switch (a.G) {
    case 32: return launch_tmem_g<32>(a, s);
    case 64: return launch_tmem_g<64>(a, s);
    default: return OTF_ERR_UNSUPPORTED;
  }
}

static int launch_generic(const LinearArgs& a, cudaStream_t st) {
  const int ctas = ceil_div(a.N, 8);
  for (int m0 = 0; m0 < a.M; m0 += 4) {
    cudaError_t e = launch_pdl(k_linear_generic<4>, dim3(ctas), dim3(256), 0, st, 1u, a, m0);
    if (e != cudaSuccess) return set_cuda_error(e);
  }
  return OTF_OK;
}

}  // namespace otf

using namespace otf;

// Validate one layer's arguments and fill LinearArgs; returns OTF_OK or an error code.
static int build_args(LinearArgs& a, const void* x, int64_t ldx, const uint8_t* packed, int64_t ld_packed,
                      const void* scales, int64_t ld_scales, const void* zeros, int64_t ld_zeros, const float* codebook,
                      const void* mask, const int64_t* outlier_idx, int64_t n_outliers, const void* outlier_vals,
                      int64_t ld_outlier_vals, const void* bias, const void* residual, int64_t ld_residual, void* y,
                      int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group_size, uint32_t flags) {
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
  a = LinearArgs{};
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
  a.xop = OTF_XOP_NONE;
  a.xaux = nullptr;
  a.eps = 0.0f;
  return OTF_OK;
}

// Which tensor-pipe variant serves these arguments: the group size (32, 64, 128, 256) or 0.
// It needs c3 - c2 == c1 - c0 (affine in the two code bits), batch 1, G a power-of-two
// multiple of the 16W-code block with at least two groups per 512-code stage, 16-byte
// aligned code rows, 4-byte aligned scale rows and 16-byte aligned activation vectors.
static int fast_variant(const LinearArgs& a, uint32_t flags) {
  const auto pow2 = [](int64_t v) { return v > 0 && (v & (v - 1)) == 0; };
  const float lhs = a.c3 - a.c2, rhs = a.c1 - a.c0;
  const bool affine = fabsf(lhs - rhs) <= 1e-6f * fmaxf(1.0f, fabsf(rhs));
  const auto al = [](const void* p, int n) { return reinterpret_cast<uintptr_t>(p) % n == 0; };
  const bool vec_ok = al(a.x, 16) && (!a.mask || al(a.mask, 16)) && (!a.xaux || al(a.xaux, 16)) && al(a.scales, 4) &&
                      a.lds % 2 == 0 && (!a.zeros || (al(a.zeros, 4) && a.ldz % 2 == 0)) && al(a.packed, 16) &&
                      a.ldp % 16 == 0 && a.K % 8 == 0;
  if ((flags & OTF_FLAG_FORCE_GENERIC) || !affine || a.M != 1 || !vec_ok || !pow2(a.G) || a.G > 256 || a.G < 32)
    return 0;
  return (a.G >= 32) ? a.G : 0;
}


// tcgen05 GEMM variant: the group size (32, 64, 128, 256) when the rows, vectors and strides are
// aligned for its copies (any codebook: the dequant is a table lookup), else 0.
static int tc_variant(const LinearArgs& a) {
  const auto pow2 = [](int64_t v) { return v > 0 && (v & (v - 1)) == 0; };
  const auto al = [](const void* p, int n) { return reinterpret_cast<uintptr_t>(p) % n == 0; };
  const bool ok = al(a.x, 16) && a.ldx % 8 == 0 && (!a.mask || al(a.mask, 16)) && al(a.packed, 16) &&
                  a.ldp % 16 == 0 && al(a.scales, 4) && a.lds % 2 == 0 &&
                  (!a.zeros || (al(a.zeros, 4) && a.ldz % 2 == 0)) && a.xop == OTF_XOP_NONE;
  if (!ok || !pow2(a.G) || a.G < 32 || a.G > 256) return 0;
  return a.G;
}

template <int G, bool ZEROS>
static int launch_tc_g(const LinearArgs& a, cudaStream_t s) {
  if (a.M <= 16) return launch_gemm_tc<G, ZEROS, 16>(a, s);
  if (a.M <= 32) return launch_gemm_tc<G, ZEROS, 32>(a, s);
  if (a.M <= 64) return launch_gemm_tc<G, ZEROS, 64>(a, s);
  return launch_gemm_tc<G, ZEROS, 128>(a, s);
}

static int launch_tc(const LinearArgs& a, int G, cudaStream_t s) {
  const bool z = a.zeros != nullptr;
  switch (G) {
    case 32: return z ? launch_tc_g<32, true>(a, s) : launch_tc_g<32, false>(a, s);
    case 64: return z ? launch_tc_g<64, true>(a, s) : launch_tc_g<64, false>(a, s);
    case 128: return z ? launch_tc_g<128, true>(a, s) : launch_tc_g<128, false>(a, s);
    case 256: return z ? launch_tc_g<256, true>(a, s) : launch_tc_g<256, false>(a, s);
    default: return OTF_ERR_UNSUPPORTED;
  }
}

// Batched tensor-pipe variant: the group size (64, 128, 256) when 2 <= M <= 8 and the layer
// otherwise qualifies for the tensor-pipe path (no fused input transform), else 0.
static int batch_variant(const LinearArgs& a, uint32_t flags) {
  if (a.M < 2 || a.M > 8 || a.G < 64 || a.xop != OTF_XOP_NONE) return 0;
  LinearArgs one = a;
  one.M = 1;
  const auto al = [](int64_t v, int n) { return v % n == 0; };
  if (!al(a.ldx * 2, 16)) return 0;  // every activation row 16-byte aligned
  return fast_variant(one, flags);
}

static int launch_batch(const LinearArgs& a, int G, cudaStream_t s) {
  const bool z = a.zeros != nullptr;
  const bool one = a.M <= 4;
  switch (G) {
    case 64:
      return z ? (one ? launch_gemv_batch<64, true, 1>(a, s) : launch_gemv_batch<64, true, 2>(a, s))
               : (one ? launch_gemv_batch<64, false, 1>(a, s) : launch_gemv_batch<64, false, 2>(a, s));
    case 128:
      return z ? (one ? launch_gemv_batch<128, true, 1>(a, s) : launch_gemv_batch<128, true, 2>(a, s))
               : (one ? launch_gemv_batch<128, false, 1>(a, s) : launch_gemv_batch<128, false, 2>(a, s));
    case 256:
      return z ? (one ? launch_gemv_batch<256, true, 1>(a, s) : launch_gemv_batch<256, true, 2>(a, s))
               : (one ? launch_gemv_batch<256, false, 1>(a, s) : launch_gemv_batch<256, false, 2>(a, s));
    default: return OTF_ERR_UNSUPPORTED;
  }
}

// One layer on the tensor-pipe kernel for group size G (from fast_variant); UNSUPPORTED if G is 0.
static int launch_fast(const LinearArgs& a, int G, cudaStream_t s) {
  const bool z = a.zeros != nullptr;
  switch (G) {
    case 32: return z ? launch_gemv<32, true>(a, s) : launch_gemv<32, false>(a, s);
    case 64: return z ? launch_gemv<64, true>(a, s) : launch_gemv<64, false>(a, s);
    case 128: return z ? launch_gemv<128, true>(a, s) : launch_gemv<128, false>(a, s);
    case 256: return z ? launch_gemv<256, true>(a, s) : launch_gemv<256, false>(a, s);
    default: return OTF_ERR_UNSUPPORTED;
  }
}

extern "C" OTF_API int otf2b_linear(const void* x, int64_t ldx, const uint8_t* packed, int64_t ld_packed,
                                    const void* scales, int64_t ld_scales, const void* zeros, int64_t ld_zeros,
                                    const float* codebook, const void* mask, const int64_t* outlier_idx,
                                    int64_t n_outliers, const void* outlier_vals, int64_t ld_outlier_vals,
                                    const void* bias, const void* residual, int64_t ld_residual, void* y,
                                    int64_t ldy, int64_t M, int64_t N, int64_t K,
                                    int64_t group_size, uint32_t flags, void* stream) {
  LinearArgs a;
  int st = build_args(a, x, ldx, packed, ld_packed, scales, ld_scales, zeros, ld_zeros, codebook, mask, outlier_idx,
                      n_outliers, outlier_vals, ld_outlier_vals, bias, residual, ld_residual, y, ldy, M, N, K,
                      group_size, flags);
  if (st != OTF_OK) return st;
  st = check_device();
  if (st != OTF_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = OTF_ERR_UNSUPPORTED;
  // Nine rows and more: the tensor-memory tcgen05 GEMM when the layer qualifies.
  if (a.M >= kTmMinRows && !(flags & OTF_FLAG_FORCE_GENERIC) && tm_variant(a)) rc = launch_tmem(a, s);
  const int Gt = (a.M >= kTcMinRows && !(flags & OTF_FLAG_FORCE_GENERIC)) ? tc_variant(a) : 0;
  if (rc != OTF_ERR_UNSUPPORTED) {
    // done
  } else if (Gt != 0) {
    rc = launch_tc(a, Gt, s);
  } else if (a.M == 1) {
    rc = launch_fast(a, fast_variant(a, flags), s);
  } else {
    // Batches of up to 8 rows on the batched tensor-pipe kernel; larger batches in slices of 8.
    LinearArgs probe = a;
    probe.M = std::min(a.M, 8);
    const int Gb = batch_variant(probe, flags);
    if (Gb != 0) {
      rc = OTF_OK;
      for (int m0 = 0; m0 < a.M && rc == OTF_OK; m0 += 8) {
        LinearArgs s8 = a;
        s8.M = std::min(8, a.M - m0);
        s8.x = a.x + (int64_t)m0 * a.ldx;
        s8.y = a.y + (int64_t)m0 * a.ldy;
        if (a.res) s8.res = a.res + (int64_t)m0 * a.ldr;
        rc = s8.M == 1 ? launch_fast(s8, fast_variant(s8, flags), s) : launch_batch(s8, Gb, s);
      }
    }
  }
  if (rc != OTF_ERR_UNSUPPORTED) return rc;
  return launch_generic(a, s);
}

extern "C" OTF_API int otf2b_gemm_mma(const void* x, int64_t ldx, const uint8_t* packed, int64_t ld_packed,
                                      const void* scales, int64_t ld_scales, const void* zeros, int64_t ld_zeros,
                                      const float* codebook, const void* mask, const int64_t* outlier_idx,
                                      int64_t n_outliers, const void* outlier_vals, int64_t ld_outlier_vals,
                                      const void* bias, const void* residual, int64_t ld_residual, void* y,
                                      int64_t ldy, int64_t M, int64_t N, int64_t K, int64_t group_size,
                                      uint32_t flags, void* stream) {
  LinearArgs a;
  int st = build_args(a, x, ldx, packed, ld_packed, scales, ld_scales, zeros, ld_zeros, codebook, mask, outlier_idx,
                      n_outliers, outlier_vals, ld_outlier_vals, bias, residual, ld_residual, y, ldy, M, N, K,
                      group_size, flags);
  if (st != OTF_OK) return st;
  st = check_device();
  if (st != OTF_OK) return st;
  if (tm_variant(a) && !(flags & OTF_FLAG_FORCE_GENERIC)) {
    const int rc = launch_tmem(a, static_cast<cudaStream_t>(stream));
    if (rc != OTF_ERR_UNSUPPORTED) return rc;
  }
  const int G = tc_variant(a);
  if (G == 0) return OTF_ERR_UNSUPPORTED;
  return launch_tc(a, G, static_cast<cudaStream_t>(stream));
}

extern "C" OTF_API int otf2b_linear_group(const otf2b_layer* layers, int n_layers, void* stream) {
  if (!layers || n_layers <= 0 || n_layers > kMaxGroup) return OTF_ERR_INVALID;
  LinearArgs L[kMaxGroup];
  for (int m = 0; m < n_layers; ++m) {
    const otf2b_layer& d = layers[m];
    int st = build_args(L[m], d.x, d.ldx, d.packed, d.ld_packed, d.scales, d.ld_scales, d.zeros, d.ld_zeros,
                        d.codebook, d.mask, d.outlier_idx, d.n_outliers, d.outlier_vals, d.ld_outlier_vals, d.bias,
                        d.residual, d.ld_residual, d.y, d.ldy, 1, d.N, d.K, d.group_size, d.flags);
    if (st != OTF_OK) return st;
    if (d.x_op < OTF_XOP_NONE || d.x_op > OTF_XOP_SILU_MUL) return OTF_ERR_INVALID;
    if (d.x_op == OTF_XOP_SILU_MUL && !d.x_aux) return OTF_ERR_INVALID;
    L[m].xop = d.x_op;
    L[m].xaux = static_cast<const uint16_t*>(d.x_aux);
    L[m].eps = d.eps;
    // Tensor-parallel exchange: one producing layer per launch; consuming layers share
    // their x, so all of them consume the same buffer.
    if (d.ar && d.ar_mode != OTF_AR_NONE) {
      const otf_ar* ar = static_cast<const otf_ar*>(d.ar);
      const void* tbl = ar_device_table(ar);
      if (!tbl || (d.ar_buf != 0 && d.ar_buf != 1)) return OTF_ERR_INVALID;
      if (d.ar_mode == OTF_AR_PRODUCE) {
        if (n_layers != 1 || d.N > ar_max_elems(ar)) return OTF_ERR_INVALID;
      } else if (d.ar_mode == OTF_AR_CONSUME) {
        if (d.K > ar_max_elems(ar) || d.x_op == OTF_XOP_SILU_MUL) return OTF_ERR_INVALID;
        if (d.n_outliers > kCThreads) return OTF_ERR_UNSUPPORTED;
        if (m == 0 && d.ar_out && reinterpret_cast<uintptr_t>(d.ar_out) % 16) return OTF_ERR_INVALID;
      } else {
        return OTF_ERR_INVALID;
      }
      L[m].ar = static_cast<const ArPeers*>(tbl);
      L[m].ar_mode = d.ar_mode;
      L[m].ar_buf = d.ar_buf;
      L[m].ar_out = m == 0 ? static_cast<uint16_t*>(d.ar_out) : nullptr;
    }
    if (m > 0 && (L[m].ar_mode != L[0].ar_mode || L[m].ar != L[0].ar || L[m].ar_buf != L[0].ar_buf))
      return OTF_ERR_INVALID;
  }
  int st = check_device();
  if (st != OTF_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // One grid needs one kernel variant and one cluster shape: same K, G and zero-point use.
  bool same = true;
  const int v0 = fast_variant(L[0], layers[0].flags);
  for (int m = 1; m < n_layers; ++m)
    same = same && L[m].K == L[0].K && L[m].G == L[0].G && (L[m].zeros != nullptr) == (L[0].zeros != nullptr) &&
           fast_variant(L[m], layers[m].flags) == v0;
  // The exchange needs the whole group in the one tensor-pipe grid (its consumer CTAs
  // count themselves to re-arm the buffer).
  if (L[0].ar_mode != OTF_AR_NONE && !(same && v0 != 0)) return OTF_ERR_UNSUPPORTED;
  if (same && v0 != 0) {
    const bool z = L[0].zeros != nullptr;
    switch (v0) {
      case 32: return z ? launch_gemv_group<32, true>(L, n_layers, s) : launch_gemv_group<32, false>(L, n_layers, s);
      case 64: return z ? launch_gemv_group<64, true>(L, n_layers, s) : launch_gemv_group<64, false>(L, n_layers, s);
      case 128: return z ? launch_gemv_group<128, true>(L, n_layers, s) : launch_gemv_group<128, false>(L, n_layers, s);
      case 256: return z ? launch_gemv_group<256, true>(L, n_layers, s) : launch_gemv_group<256, false>(L, n_layers, s);
      default: break;
    }
  }
  // Otherwise one launch per layer; transforms need the tensor-pipe kernel.
  for (int m = 0; m < n_layers; ++m) {
    const int v = fast_variant(L[m], layers[m].flags);
    int rc = OTF_ERR_UNSUPPORTED;
    if (v != 0) rc = launch_fast(L[m], v, s);
    else if (L[m].xop == OTF_XOP_NONE) rc = launch_generic(L[m], s);
    if (rc != OTF_OK) return rc;
  }
  return OTF_OK;
}

extern "C" OTF_API int otf2b_unpack_codes(const uint8_t* packed, int64_t ld_packed, int64_t N, int64_t K,
                                          uint8_t* codes, int64_t ld_codes, void* stream) {
  if (!packed || !codes || N <= 0 || K <= 0 || K % 4 || ld_packed < K / 4 || ld_codes < K) return OTF_ERR_INVALID;
  if (N > INT32_MAX || K > INT32_MAX) return OTF_ERR_UNSUPPORTED;
  int st = check_device();
  if (st != OTF_OK) return st;
  const int64_t total = N * (K / 4);
  const int blocks = (int)std::min<int64_t>(ceil_div((int)std::min<int64_t>(total, INT32_MAX), 256), 148 * 16);
  return set_cuda_error(launch_pdl(k_unpack_codes, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream), 1u,
                                   packed, ld_packed, (int)N, (int)K, codes, ld_codes));
}

extern "C" OTF_API int otf_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, otf::g_otf_device_error, sizeof(int)) != cudaSuccess) { set_cuda_error(cudaGetLastError()); return -1; }
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(otf::g_otf_device_error, &z, sizeof(int));
  }
  const int w = ar_device_error(clear);
  const int x = mk_device_error(clear);
  const int a = attn_device_error(clear);
  const int h = head_device_error(clear);
  if (w < 0 || x < 0 || a < 0 || h < 0) return -1;
  return v | w | x | a | h;
}
