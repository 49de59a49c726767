// Batch-1 decode attention around the 2-bit projections: rotary embedding + KV-cache write,
// split-KV attention over the cached positions, and the device-side position counter.
//
// These run between the q/k/v and o launches of a decoder layer when the decoder stack
// does real attention (a growing fp16 KV cache, grouped-query heads, RoPE).  The position
// of the token being decoded lives in device memory, so a whole token step -- embedding,
// every layer, final norm, head argmax, position advance -- replays as one CUDA graph.
//
// Reference behaviour replaced: the attention of HF's LlamaAttention that the reference
// runner keeps around its injected projections (otf_llm/run_symmetric_2bit.py:150-187):
// RoPE with rotate_half in the projections' dtype (fp16), repeat_kv for grouped heads,
// softmax(q k^T / sqrt(d)) v.  Here the dot products and the softmax run in fp32 (as the
// fused SDPA kernels do); RoPE rounds like HF's fp16 elementwise ops.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "otf_common.cuh"

namespace otf {

int set_cuda_error(cudaError_t e);  // capi.cu
int check_device();                 // capi.cu
int attn_device_error(int clear);   // read (and optionally clear) the flag below

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kAttnMaxRep = 8;       // query heads per KV head
constexpr int kAttnSplitPos = 64;    // cached positions per CTA (split-KV)

// Set when an attention launch saw a position outside [0, max_pos): such a launch writes
// nothing (no cache row, no output).  Read and cleared through otf_device_error.
__device__ int g_attn_device_error;

__device__ __forceinline__ void report_bad_position() {
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) atomicExch(&g_attn_device_error, 1);
}

// q (heads x D), k (kv_heads x D) rotated in place with cos/sin of position *pos; k and v
// copied into the caches at row *pos.  HF rotate_half form, fp16 arithmetic:
//   out[i]     = fp16(fp16(x[i] * c[i])         + fp16(-x[i + D/2] * s[i]))
//   out[i+D/2] = fp16(fp16(x[i + D/2] * c[i+D/2]) + fp16( x[i] * s[i+D/2]))
// cos_sin: fp16 [max_pos, 2, D] (cos row, then sin row; both halves duplicated as in HF).
__global__ void k_rope_kv(uint16_t* q, uint16_t* k, const uint16_t* v, const uint16_t* cos_sin, const int* pos,
                          uint16_t* kc, uint16_t* vc, int heads, int kv_heads, int D, int max_pos) {
  pdl_trigger();
  pdl_wait();
  const int p = *pos;
  if (p < 0 || p >= max_pos) {  // the host sized the cache; an out-of-range position writes nothing
    report_bad_position();
    return;
  }
  const int half = D / 2;
  const uint16_t* cs = cos_sin + (int64_t)p * 2 * D;
  const int nvec = (heads + kv_heads) * half;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < nvec; e += gridDim.x * blockDim.x) {
    const int hh = e / half, i = e - hh * half;
    uint16_t* x = hh < heads ? q + (int64_t)hh * D : k + (int64_t)(hh - heads) * D;
    const __half a = __ushort_as_half(x[i]), b = __ushort_as_half(x[i + half]);
    const __half c0 = __ushort_as_half(cs[i]), c1 = __ushort_as_half(cs[i + half]);
    const __half s0 = __ushort_as_half(cs[D + i]), s1 = __ushort_as_half(cs[D + i + half]);
    // _rn forms: each product and the sum round separately (no fused multiply-add), as the
    // separate fp16 tensor ops do
    const __half lo = __hadd_rn(__hmul_rn(a, c0), __hmul_rn(__hneg(b), s0));
    const __half hi = __hadd_rn(__hmul_rn(b, c1), __hmul_rn(a, s1));
    x[i] = __half_as_ushort(lo);
    x[i + half] = __half_as_ushort(hi);
    if (hh >= heads) {
      uint16_t* krow = kc + (int64_t)p * kv_heads * D + (int64_t)(hh - heads) * D;
      krow[i] = __half_as_ushort(lo);
      krow[i + half] = __half_as_ushort(hi);
    }
  }
  const int nv = kv_heads * D;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < nv; e += gridDim.x * blockDim.x)
    vc[(int64_t)p * nv + e] = v[e];
}

// Split-KV attention: CTA (g, sp) takes KV head g and cached positions [sp*64, sp*64+64) for
// the rep query heads of g; each warp walks a quarter of those positions with an online
// softmax per query head (lane l holds dims 4l..4l+3 when D = 128, 2l..2l+1 when D = 64).
// Partials (max, sum, acc) go to the workspace; the last CTA of head g (an atomic ticket,
// no waiting) merges them and writes fp16 out.
template <int D>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(const uint16_t* q, const uint16_t* kc, const uint16_t* vc,
                                                              const int* pos, uint16_t* out, float scale, int heads,
                                                              int kv_heads, int max_pos, float* ws, unsigned* tickets,
                                                              int max_split) {
  constexpr int PL = D / 32;  // dims per lane
  pdl_trigger();
  pdl_wait();
  const int rep = heads / kv_heads;
  const int g = blockIdx.x, sp = blockIdx.y;
  const int p = *pos;
  if (p < 0 || p >= max_pos) {  // out of range: write nothing, as the fused kernel does
    report_bad_position();
    return;
  }
  const int L = p + 1;
  const int nsplit = min((L + kAttnSplitPos - 1) / kAttnSplitPos, max_split);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float sm_m[kAttnWarps][kAttnMaxRep], sm_l[kAttnWarps][kAttnMaxRep];
  __shared__ float sm_acc[kAttnWarps][kAttnMaxRep][D];
  __shared__ unsigned s_last;
  if (sp >= nsplit) return;  // uniform per CTA: positions beyond the cache length
  const int per = (L + nsplit - 1) / nsplit;
  const int p0 = sp * per, p1 = min(L, p0 + per);
  // (loops over query heads run to kAttnMaxRep with a guard, so the arrays stay in registers)
  float qv[kAttnMaxRep][PL];
#pragma unroll
  for (int r = 0; r < kAttnMaxRep; ++r)
#pragma unroll
    for (int i = 0; i < PL; ++i) qv[r][i] = r < rep ? h2f(q[(int64_t)(g * rep + r) * D + lane * PL + i]) * scale : 0.0f;
  float m[kAttnMaxRep], l[kAttnMaxRep], acc[kAttnMaxRep][PL];
#pragma unroll
  for (int r = 0; r < kAttnMaxRep; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int i = 0; i < PL; ++i) acc[r][i] = 0.0f;
  }
  const int64_t stride = (int64_t)kv_heads * D;
  for (int p = p0 + warp; p < p1; p += kAttnWarps) {
    const uint16_t* kr = kc + p * stride + (int64_t)g * D + lane * PL;
    const uint16_t* vr = vc + p * stride + (int64_t)g * D + lane * PL;
    float kf[PL], vf[PL];
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      kf[i] = h2f(kr[i]);
      vf[i] = h2f(vr[i]);
    }
#pragma unroll
    for (int r = 0; r < kAttnMaxRep; ++r) {
      if (r >= rep) break;
      float d = 0.0f;
#pragma unroll
      for (int i = 0; i < PL; ++i) d = fmaf(qv[r][i], kf[i], d);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      const float mn = fmaxf(m[r], d);
      const float corr = __expf(m[r] - mn), w = __expf(d - mn);
      l[r] = l[r] * corr + w;
#pragma unroll
      for (int i = 0; i < PL; ++i) acc[r][i] = fmaf(acc[r][i], corr, w * vf[i]);
      m[r] = mn;
    }
  }
  // Merge the warps of this CTA.
#pragma unroll
  for (int r = 0; r < kAttnMaxRep; ++r) {
    if (r >= rep) break;
    if (lane == 0) {
      sm_m[warp][r] = m[r];
      sm_l[warp][r] = l[r];
    }
#pragma unroll
    for (int i = 0; i < PL; ++i) sm_acc[warp][r][lane * PL + i] = acc[r][i];
  }
  __syncthreads();
  float* part = ws + ((int64_t)g * max_split + sp) * kAttnMaxRep * (D + 2);
  for (int e = threadIdx.x; e < rep * D; e += kAttnThreads) {
    const int r = e / D, dd = e - r * D;
    float mm = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, sm_m[w][r]);
    float ll = 0.0f, aa = 0.0f;
    for (int w = 0; w < kAttnWarps; ++w) {
      const float c = sm_m[w][r] == -INFINITY ? 0.0f : __expf(sm_m[w][r] - mm);
      ll += sm_l[w][r] * c;
      aa += sm_acc[w][r][dd] * c;
    }
    part[r * (D + 2) + 2 + dd] = aa;
    if (dd == 0) {
      part[r * (D + 2)] = mm;
      part[r * (D + 2) + 1] = ll;
    }
  }
  // Last CTA of this KV head merges the splits (it reads partials the others published).
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(tickets + g, 1u) == (unsigned)nsplit - 1u) ? 1u : 0u;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int e = threadIdx.x; e < rep * D; e += kAttnThreads) {
    const int r = e / D, dd = e - r * D;
    float mm = -INFINITY;
    for (int s = 0; s < nsplit; ++s) mm = fmaxf(mm, __ldcg(ws + ((int64_t)g * max_split + s) * kAttnMaxRep * (D + 2) + r * (D + 2)));
    float ll = 0.0f, aa = 0.0f;
    for (int s = 0; s < nsplit; ++s) {
      const float* ps = ws + ((int64_t)g * max_split + s) * kAttnMaxRep * (D + 2) + r * (D + 2);
      const float ms = __ldcg(ps);
      const float c = ms == -INFINITY ? 0.0f : __expf(ms - mm);
      ll += __ldcg(ps + 1) * c;
      aa += __ldcg(ps + 2 + dd) * c;
    }
    out[(int64_t)(g * rep + r) * D + dd] = f2h(aa / ll);
  }
  if (threadIdx.x == 0) tickets[g] = 0u;  // re-armed for the next call
}

// RoPE, KV-cache write and split-KV attention in one launch.  Same split of the cached
// positions and the same partial/ticket merge as k_attn_decode, with three changes:
//  * every CTA rotates the query heads it needs in registers (the partner half of a head's
//    vector is 16 lanes away: one shuffle), so q is read unrotated;
//  * the CTA whose split holds the new position rotates that position's k, writes k and v to
//    the cache rows and makes them visible to its own warps with a CTA barrier (no other CTA
//    reads that row in this call);
//  * 8 warps per CTA, each issuing the loads of up to 4 cached positions before using them.
constexpr int kAttn2Warps = 8;
constexpr int kAttn2Threads = kAttn2Warps * 32;
constexpr int kAttn2Batch = 4;

template <int PL>
__device__ __forceinline__ void rope_lane(const uint16_t* x, const uint16_t* cs, int D, int lane, __half (&o)[PL]) {
  __half xv[PL];
#pragma unroll
  for (int i = 0; i < PL; ++i) xv[i] = __ushort_as_half(x[lane * PL + i]);
#pragma unroll
  for (int i = 0; i < PL; ++i) {
    const __half pv = __ushort_as_half((uint16_t)__shfl_xor_sync(0xffffffffu, (int)__half_as_ushort(xv[i]), 16));
    const int dim = lane * PL + i;
    const __half c = __ushort_as_half(cs[dim]), sn = __ushort_as_half(cs[D + dim]);
    const __half t = lane < 16 ? __hmul_rn(__hneg(pv), sn) : __hmul_rn(pv, sn);
    o[i] = __hadd_rn(__hmul_rn(xv[i], c), t);
  }
}

// Batched form: blockIdx.z is the sequence; each has its own q/k/v rows (row strides ldq /
// ldkv), caches (cache_stride elements apart), position pos[b], output row and workspace slice.
// REP > 0: the query heads per KV head fixed at compile time (the head loops unroll without
// early exits, so the heads' reductions interleave); REP = 0: any ratio up to kAttnMaxRep.
template <int D, int REP>
__global__ void __launch_bounds__(kAttn2Threads) k_attn_rope_decode(
    const uint16_t* q, const uint16_t* knew, const uint16_t* vnew, const uint16_t* cos_sin, const int* pos,
    uint16_t* kc, uint16_t* vc, uint16_t* out, float scale, int heads, int kv_heads, int max_pos, float* ws,
    unsigned* tickets, int max_split, int64_t ldq, int64_t ldkv, int64_t cache_stride, int64_t ldo,
    int64_t ws_stride) {
  constexpr int PL = D / 32;
  pdl_trigger();
  pdl_wait();
  {
    const int b = blockIdx.z;
    q += b * ldq;
    knew += b * ldkv;
    vnew += b * ldkv;
    kc += b * cache_stride;
    vc += b * cache_stride;
    out += b * ldo;
    ws += b * ws_stride;
    tickets += b * kv_heads;
    pos += b;
  }
  const int p = *pos;
  if (p < 0 || p >= max_pos) {  // the host sized the cache; out of range writes nothing
    report_bad_position();  // one thread of each sequence's first CTA
    return;
  }
  const int rep = REP > 0 ? REP : heads / kv_heads;
  const int g = blockIdx.x, sp = blockIdx.y;
  const int L = p + 1;
  const int nsplit = min((L + kAttnSplitPos - 1) / kAttnSplitPos, max_split);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float sm_m[kAttn2Warps][kAttnMaxRep], sm_l[kAttn2Warps][kAttnMaxRep];
  __shared__ float sm_acc[kAttn2Warps][kAttnMaxRep][D];
  __shared__ unsigned s_last;
  if (sp >= nsplit) return;  // uniform per CTA
  const int per = (L + nsplit - 1) / nsplit;
  const int p0 = sp * per, p1 = min(L, p0 + per);
  const uint16_t* cs = cos_sin + (int64_t)p * 2 * D;
  const int64_t stride = (int64_t)kv_heads * D;
  if (p1 == L && warp == 0) {
    __half kr[PL];
    rope_lane<PL>(knew + (int64_t)g * D, cs, D, lane, kr);
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      kc[p * stride + (int64_t)g * D + lane * PL + i] = __half_as_ushort(kr[i]);
      vc[p * stride + (int64_t)g * D + lane * PL + i] = vnew[(int64_t)g * D + lane * PL + i];
    }
  }
  __syncthreads();  // the new cache row is visible to this CTA's warps
  float qv[kAttnMaxRep][PL];
#pragma unroll
  for (int r = 0; r < kAttnMaxRep; ++r) {
    if (r < rep) {
      __half qr[PL];
      rope_lane<PL>(q + (int64_t)(g * rep + r) * D, cs, D, lane, qr);
#pragma unroll
      for (int i = 0; i < PL; ++i) qv[r][i] = __half2float(qr[i]) * scale;
    } else {
#pragma unroll
      for (int i = 0; i < PL; ++i) qv[r][i] = 0.0f;
    }
  }
  float m[kAttnMaxRep], l[kAttnMaxRep], acc[kAttnMaxRep][PL];
#pragma unroll
  for (int r = 0; r < kAttnMaxRep; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int i = 0; i < PL; ++i) acc[r][i] = 0.0f;
  }
  for (int base = p0 + warp; base < p1; base += kAttn2Warps * kAttn2Batch) {
    float kf[kAttn2Batch][PL], vf[kAttn2Batch][PL];
#pragma unroll
    for (int j = 0; j < kAttn2Batch; ++j) {
      const int pp = base + j * kAttn2Warps;
      const int pc = pp < p1 ? pp : p0;  // a valid row; its values are not used
      const uint16_t* kr = kc + pc * stride + (int64_t)g * D + lane * PL;
      const uint16_t* vr = vc + pc * stride + (int64_t)g * D + lane * PL;
#pragma unroll
      for (int i = 0; i < PL; ++i) {
        kf[j][i] = h2f(kr[i]);
        vf[j][i] = h2f(vr[i]);
      }
    }
#pragma unroll
    for (int j = 0; j < kAttn2Batch; ++j) {
      if (base + j * kAttn2Warps >= p1) break;
#pragma unroll
      for (int r = 0; r < (REP > 0 ? REP : kAttnMaxRep); ++r) {
        if (REP == 0 && r >= rep) break;
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < PL; ++i) d = fmaf(qv[r][i], kf[j][i], d);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        const float mn = fmaxf(m[r], d);
        const float corr = __expf(m[r] - mn), w = __expf(d - mn);
        l[r] = l[r] * corr + w;
#pragma unroll
        for (int i = 0; i < PL; ++i) acc[r][i] = fmaf(acc[r][i], corr, w * vf[j][i]);
        m[r] = mn;
      }
    }
  }
#pragma unroll
  for (int r = 0; r < (REP > 0 ? REP : kAttnMaxRep); ++r) {
    if (REP == 0 && r >= rep) break;
    if (lane == 0) {
      sm_m[warp][r] = m[r];
      sm_l[warp][r] = l[r];
    }
#pragma unroll
    for (int i = 0; i < PL; ++i) sm_acc[warp][r][lane * PL + i] = acc[r][i];
  }
  __syncthreads();
  float* part = ws + ((int64_t)g * max_split + sp) * kAttnMaxRep * (D + 2);
  for (int e = threadIdx.x; e < rep * D; e += kAttn2Threads) {
    const int r = e / D, dd = e - r * D;
    float mm = -INFINITY;
    for (int w = 0; w < kAttn2Warps; ++w) mm = fmaxf(mm, sm_m[w][r]);
    float ll = 0.0f, aa = 0.0f;
    for (int w = 0; w < kAttn2Warps; ++w) {
      const float c = sm_m[w][r] == -INFINITY ? 0.0f : __expf(sm_m[w][r] - mm);
      ll += sm_l[w][r] * c;
      aa += sm_acc[w][r][dd] * c;
    }
    if (nsplit == 1) {              // the whole cache in this CTA: no partials, no merge
      out[(int64_t)(g * rep + r) * D + dd] = f2h(aa / ll);
      continue;
    }
    part[r * (D + 2) + 2 + dd] = aa;
    if (dd == 0) {
      part[r * (D + 2)] = mm;
      part[r * (D + 2) + 1] = ll;
    }
  }
  if (nsplit == 1) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(tickets + g, 1u) == (unsigned)nsplit - 1u) ? 1u : 0u;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* pbase = ws + (int64_t)g * max_split * kAttnMaxRep * (D + 2);
  constexpr int kSmFloats = kAttn2Warps * kAttnMaxRep * D;
  if (2 * nsplit * rep + 2 * rep <= kSmFloats) {
    // The split maxima and sums of every head, loaded in parallel into shared memory (sm_acc
    // is free now); one thread per head forms the weights exp(m_s - max) and the total sum in
    // split order; every output element then loads its splits' partial sums together.
    float* pm = &sm_acc[0][0][0];   // [nsplit][rep]: maxima, then weights
    float* pl = pm + nsplit * rep;  // [nsplit][rep]: sums
    float* hl = pl + nsplit * rep;  // [rep]: total sum per head
    for (int i = threadIdx.x; i < nsplit * rep; i += kAttn2Threads) {
      const int s2 = i / rep, r = i - s2 * rep;
      const float* ps = pbase + ((int64_t)s2 * kAttnMaxRep + r) * (D + 2);
      pm[i] = __ldcg(ps);
      pl[i] = __ldcg(ps + 1);
    }
    __syncthreads();
    if (threadIdx.x < rep) {
      const int r = threadIdx.x;
      float mm = -INFINITY;
      for (int s2 = 0; s2 < nsplit; ++s2) mm = fmaxf(mm, pm[s2 * rep + r]);
      float ll = 0.0f;
      for (int s2 = 0; s2 < nsplit; ++s2) {
        const float ms = pm[s2 * rep + r];
        const float c = ms == -INFINITY ? 0.0f : __expf(ms - mm);
        ll += pl[s2 * rep + r] * c;
        pm[s2 * rep + r] = c;
      }
      hl[r] = ll;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < rep * D; e += kAttn2Threads) {
      const int r = e / D, dd = e - r * D;
      const float* pe = pbase + (int64_t)r * (D + 2) + 2 + dd;
      float aa = 0.0f;
#pragma unroll 8
      for (int s2 = 0; s2 < nsplit; ++s2) aa += __ldcg(pe + (int64_t)s2 * kAttnMaxRep * (D + 2)) * pm[s2 * rep + r];
      out[(int64_t)(g * rep + r) * D + dd] = f2h(aa / hl[r]);
    }
  } else {
    for (int e = threadIdx.x; e < rep * D; e += kAttn2Threads) {
      const int r = e / D, dd = e - r * D;
      const float* pb = pbase + r * (D + 2);
      float mm = -INFINITY;
      for (int s2 = 0; s2 < nsplit; ++s2) mm = fmaxf(mm, __ldcg(pb + (int64_t)s2 * kAttnMaxRep * (D + 2)));
      float ll = 0.0f, aa = 0.0f;
      for (int s2 = 0; s2 < nsplit; ++s2) {
        const float* ps = pb + (int64_t)s2 * kAttnMaxRep * (D + 2);
        const float ms = __ldcg(ps);
        const float c = ms == -INFINITY ? 0.0f : __expf(ms - mm);
        ll += __ldcg(ps + 1) * c;
        aa += __ldcg(ps + 2 + dd) * c;
      }
      out[(int64_t)(g * rep + r) * D + dd] = f2h(aa / ll);
    }
  }
  if (threadIdx.x == 0) tickets[g] = 0u;  // re-armed for the next call
}

// The same fused step with the split merge inside a thread-block cluster: the S CTAs of one KV
// head (S <= 16, one cluster, split index = cluster rank) each take a contiguous 1/S of the cached
// positions.  The query-head x dimension outputs are dealt to the S CTAs in contiguous runs; each
// CTA stores the weighted sums of every run into the run owner's shared memory over DSMEM and
// its (max, sum) per query head into every CTA's, and after one cluster barrier each CTA
// combines the S partials of its own run in rank order.  No global partials, fences or tickets
// sit in the chain, and no CTA receives more than its share.  Also: the query rows are requested
// together with the position (they do not depend on it), and each warp's first batch of cached
// rows before the rotations (the new position's row is never read from the cache in this call:
// its rotated k and its v reach this CTA's warps through shared memory).  Every CTA of a cluster
// runs the same path to the barrier (an empty range contributes max -inf, sum 0).
constexpr int kAttnClMax = 16;

template <int PL>
__device__ __forceinline__ void rope_vals(const uint16_t (&xr)[PL], const uint16_t* cs, int D, int lane, __half (&o)[PL]) {
#pragma unroll
  for (int i = 0; i < PL; ++i) {
    const __half xv = __ushort_as_half(xr[i]);
    const __half pv = __ushort_as_half((uint16_t)__shfl_xor_sync(0xffffffffu, (int)xr[i], 16));
    const int dim = lane * PL + i;
    const __half c = __ushort_as_half(cs[dim]), sn = __ushort_as_half(cs[D + dim]);
    const __half t = lane < 16 ? __hmul_rn(__hneg(pv), sn) : __hmul_rn(pv, sn);
    o[i] = __hadd_rn(__hmul_rn(xv, c), t);
  }
}

// Up to 4 query heads per KV head the kernel is compiled for two CTAs per SM (measured 4% faster
// on the 3B decode); with 8 it keeps its registers (one CTA per SM, no spills).
template <int D, int REP>
__global__ void __launch_bounds__(kAttn2Threads, REP <= 4 ? 2 : 1) k_attn_rope_decode_cl(
    const uint16_t* q, const uint16_t* knew, const uint16_t* vnew, const uint16_t* cos_sin, const int* pos,
    uint16_t* kc, uint16_t* vc, uint16_t* out, float scale, int kv_heads, int max_pos, int64_t ldq, int64_t ldkv,
    int64_t cache_stride, int64_t ldo) {
  constexpr int PL = D / 32;
  static_assert(REP >= 1 && REP <= kAttnMaxRep, "query heads per KV head");
  extern __shared__ __align__(16) float cl_part[];  // [S][chunk] values, then [S][REP][2] (max, sum)
  __shared__ float sm_m[kAttn2Warps][REP], sm_l[kAttn2Warps][REP];
  __shared__ float sm_acc[kAttn2Warps][REP][D];
  __shared__ float s_knew[D], s_vnew[D];
  pdl_trigger();
  cluster_arrive_relaxed();  // paired with cluster_wait() before the first DSMEM store
  pdl_wait();
  {
    const int b = blockIdx.z;
    q += b * ldq;
    knew += b * ldkv;
    vnew += b * ldkv;
    kc += b * cache_stride;
    vc += b * cache_stride;
    out += b * ldo;
    pos += b;
  }
  const int S = (int)gridDim.x, sp = (int)blockIdx.x, g = (int)blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint16_t qraw[REP][PL];
#pragma unroll
  for (int r = 0; r < REP; ++r)
#pragma unroll
    for (int i = 0; i < PL; ++i) qraw[r][i] = q[(int64_t)(g * REP + r) * D + lane * PL + i];
  const int p = *pos;
  if (p < 0 || p >= max_pos) {  // the same position for every CTA of the cluster: all leave here
    report_bad_position();  // one thread of each sequence's first CTA
    return;
  }
  const int L = p + 1;
  const int per = (L + S - 1) / S;
  const int p0 = min(L, sp * per), p1 = min(L, p0 + per);
  const uint16_t* cs = cos_sin + (int64_t)p * 2 * D;
  const int64_t stride = (int64_t)kv_heads * D;
  float kf[kAttn2Batch][PL], vf[kAttn2Batch][PL];
  auto load_batch = [&](int base) {
#pragma unroll
    for (int j = 0; j < kAttn2Batch; ++j) {
      const int pp = base + j * kAttn2Warps;
      const int pc = (pp < p1 && pp != p) ? pp : 0;  // row 0 always exists; its values are not used
      const uint16_t* kr = kc + pc * stride + (int64_t)g * D + lane * PL;
      const uint16_t* vr = vc + pc * stride + (int64_t)g * D + lane * PL;
#pragma unroll
      for (int i = 0; i < PL; ++i) {
        kf[j][i] = h2f(kr[i]);
        vf[j][i] = h2f(vr[i]);
      }
    }
  };
  load_batch(p0 + warp);
  if (p0 <= p && p < p1 && warp == 0) {
    __half kr[PL];
    rope_lane<PL>(knew + (int64_t)g * D, cs, D, lane, kr);
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const uint16_t vv = vnew[(int64_t)g * D + lane * PL + i];
      kc[p * stride + (int64_t)g * D + lane * PL + i] = __half_as_ushort(kr[i]);
      vc[p * stride + (int64_t)g * D + lane * PL + i] = vv;
      s_knew[lane * PL + i] = __half2float(kr[i]);
      s_vnew[lane * PL + i] = h2f(vv);
    }
  }
  __syncthreads();  // the new position's k and v are in shared memory
  float qv[REP][PL];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    __half qr[PL];
    rope_vals<PL>(qraw[r], cs, D, lane, qr);
#pragma unroll
    for (int i = 0; i < PL; ++i) qv[r][i] = __half2float(qr[i]) * scale;
  }
  float m[REP], l[REP], acc[REP][PL];
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int i = 0; i < PL; ++i) acc[r][i] = 0.0f;
  }
  for (int base = p0 + warp; base < p1; base += kAttn2Warps * kAttn2Batch) {
    if (base != p0 + warp) load_batch(base);
#pragma unroll
    for (int j = 0; j < kAttn2Batch; ++j) {
      const int pp = base + j * kAttn2Warps;
      if (pp >= p1) break;
      if (pp == p) {
#pragma unroll
        for (int i = 0; i < PL; ++i) {
          kf[j][i] = s_knew[lane * PL + i];
          vf[j][i] = s_vnew[lane * PL + i];
        }
      }
#pragma unroll
      for (int r = 0; r < REP; ++r) {
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < PL; ++i) d = fmaf(qv[r][i], kf[j][i], d);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        const float mn = fmaxf(m[r], d);
        const float corr = __expf(m[r] - mn), w = __expf(d - mn);
        l[r] = l[r] * corr + w;
#pragma unroll
        for (int i = 0; i < PL; ++i) acc[r][i] = fmaf(acc[r][i], corr, w * vf[j][i]);
        m[r] = mn;
      }
    }
  }
#pragma unroll
  for (int r = 0; r < REP; ++r) {
    if (lane == 0) {
      sm_m[warp][r] = m[r];
      sm_l[warp][r] = l[r];
    }
#pragma unroll
    for (int i = 0; i < PL; ++i) sm_acc[warp][r][lane * PL + i] = acc[r][i];
  }
  __syncthreads();
  cluster_wait();  // every CTA of the cluster is running: its peers' shared memory is live
  // The REP*D outputs are dealt to the S CTAs in contiguous runs of `chunk`: each CTA sends the
  // weighted sums of every run to the run's owner and its (max, sum) per head to every CTA, then
  // combines the S partials of its own run in rank order.
  constexpr int E = REP * D;
  const int chunk = (E + S - 1) / S;
  float* const recv = cl_part;               // [S][chunk]
  float* const mls = cl_part + S * chunk;    // [S][REP][2]
  const uint32_t recv0 = smem_u32(recv), mls0 = smem_u32(mls);
  for (int e = threadIdx.x; e < E; e += kAttn2Threads) {
    const int r = e / D, dd = e - r * D;
    float mm = -INFINITY;
    for (int w = 0; w < kAttn2Warps; ++w) mm = fmaxf(mm, sm_m[w][r]);
    float ll = 0.0f, aa = 0.0f;
    for (int w = 0; w < kAttn2Warps; ++w) {
      const float c = sm_m[w][r] == -INFINITY ? 0.0f : __expf(sm_m[w][r] - mm);
      ll += sm_l[w][r] * c;
      aa += sm_acc[w][r][dd] * c;
    }
    const int owner = e / chunk;
    st_cluster_f32_plain(mapa_shared(recv0 + (uint32_t)(sp * chunk + (e - owner * chunk)) * 4u, (uint32_t)owner), aa);
    if (dd == 0) {
      const uint32_t a = mls0 + (uint32_t)((sp * REP + r) * 2) * 4u;
      for (int q2 = 0; q2 < S; ++q2) {
        st_cluster_f32_plain(mapa_shared(a, (uint32_t)q2), mm);
        st_cluster_f32_plain(mapa_shared(a + 4u, (uint32_t)q2), ll);
      }
    }
  }
  cluster_sync_all();  // every partial has landed with its owner
  for (int el = threadIdx.x; el < chunk; el += kAttn2Threads) {
    const int e = sp * chunk + el;
    if (e >= E) break;
    const int r = e / D, dd = e - r * D;
    float mm = -INFINITY;
    for (int q2 = 0; q2 < S; ++q2) mm = fmaxf(mm, mls[(q2 * REP + r) * 2]);
    float ll = 0.0f, aa = 0.0f;
    for (int q2 = 0; q2 < S; ++q2) {
      const float ms = mls[(q2 * REP + r) * 2];
      const float c = ms == -INFINITY ? 0.0f : __expf(ms - mm);
      ll += mls[(q2 * REP + r) * 2 + 1] * c;
      aa += recv[q2 * chunk + el] * c;
    }
    out[(int64_t)(g * REP + r) * D + dd] = f2h(aa / ll);
  }
}

__global__ void k_pos_advance(int* pos, int n) {
  pdl_trigger();
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) pos[i] += 1;
}

// Prompt prefill, rows r = 0..P-1 (grid.y) at positions *pos + r: q and k of row r rotated in
// place (k_rope_kv's arithmetic), k and v copied into the caches at row *pos + r.  A row whose
// position falls outside [0, max_pos) writes nothing and raises the position flag.
__global__ void k_rope_kv_rows(uint16_t* q, int64_t ldq, uint16_t* k, const uint16_t* v, int64_t ldkv,
                               const uint16_t* cos_sin, const int* pos, uint16_t* kc, uint16_t* vc, int heads,
                               int kv_heads, int D, int max_pos) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.y, p0 = *pos;
  if (p0 < 0 || p0 >= max_pos || r >= max_pos - p0) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(&g_attn_device_error, 1);
    return;
  }
  const int p = p0 + r, half = D / 2;
  q += (int64_t)r * ldq;
  k += (int64_t)r * ldkv;
  v += (int64_t)r * ldkv;
  const uint16_t* cs = cos_sin + (int64_t)p * 2 * D;
  const int nvec = (heads + kv_heads) * half;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < nvec; e += gridDim.x * blockDim.x) {
    const int hh = e / half, i = e - hh * half;
    uint16_t* x = hh < heads ? q + (int64_t)hh * D : k + (int64_t)(hh - heads) * D;
    const __half a = __ushort_as_half(x[i]), b = __ushort_as_half(x[i + half]);
    const __half c0 = __ushort_as_half(cs[i]), c1 = __ushort_as_half(cs[i + half]);
    const __half s0 = __ushort_as_half(cs[D + i]), s1 = __ushort_as_half(cs[D + i + half]);
    const __half lo = __hadd_rn(__hmul_rn(a, c0), __hmul_rn(__hneg(b), s0));
    const __half hi = __hadd_rn(__hmul_rn(b, c1), __hmul_rn(a, s1));
    x[i] = __half_as_ushort(lo);
    x[i + half] = __half_as_ushort(hi);
    if (hh >= heads) {
      uint16_t* krow = kc + (int64_t)p * kv_heads * D + (int64_t)(hh - heads) * D;
      krow[i] = __half_as_ushort(lo);
      krow[i + half] = __half_as_ushort(hi);
    }
  }
  const int nv = kv_heads * D;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < nv; e += gridDim.x * blockDim.x)
    vc[(int64_t)p * nv + e] = v[e];
}

// Causal attention of prompt row r (grid.y; position p = *pos + r) over cache rows [0, p] for
// the query heads of KV head g (grid.x): the decode kernel's per-warp online softmax (fp32,
// the same dot-product and rescale arithmetic) with the positions dealt to 8 warps, merged in
// shared memory by one CTA, so no workspace.  The rows were written by k_rope_kv_rows.
constexpr int kPfWarps = 8;
template <int D>
__global__ void __launch_bounds__(kPfWarps * 32) k_attn_prefill(const uint16_t* q, int64_t ldq, const uint16_t* kc,
                                                                const uint16_t* vc, const int* pos, uint16_t* out,
                                                                int64_t ldo, float scale, int heads, int kv_heads,
                                                                int max_pos) {
  constexpr int PL = D / 32;
  pdl_trigger();
  pdl_wait();
  const int g = blockIdx.x, r = blockIdx.y, p0 = *pos;
  if (p0 < 0 || p0 >= max_pos || r >= max_pos - p0) return;  // flagged by k_rope_kv_rows
  const int p = p0 + r, rep = heads / kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float sm_m[kPfWarps][kAttnMaxRep], sm_l[kPfWarps][kAttnMaxRep];
  __shared__ float sm_acc[kPfWarps][kAttnMaxRep][D];
  q += (int64_t)r * ldq;
  out += (int64_t)r * ldo;
  float qv[kAttnMaxRep][PL];
#pragma unroll
  for (int h = 0; h < kAttnMaxRep; ++h)
#pragma unroll
    for (int i = 0; i < PL; ++i) qv[h][i] = h < rep ? h2f(q[(int64_t)(g * rep + h) * D + lane * PL + i]) * scale : 0.0f;
  float m[kAttnMaxRep], l[kAttnMaxRep], acc[kAttnMaxRep][PL];
#pragma unroll
  for (int h = 0; h < kAttnMaxRep; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int i = 0; i < PL; ++i) acc[h][i] = 0.0f;
  }
  const int64_t stride = (int64_t)kv_heads * D;
  // Warp w takes positions w, w + 8, w + 16, ... in that order; the k/v rows of the next
  // kPfBatch of them are requested together (raw fp16 pairs) before they are used.
  constexpr int kPfBatch = 4;
  for (int base = warp; base <= p; base += kPfBatch * kPfWarps) {
    uint32_t kraw[kPfBatch][PL / 2], vraw[kPfBatch][PL / 2];
#pragma unroll
    for (int j = 0; j < kPfBatch; ++j) {
      const int pp = base + j * kPfWarps;
      const uint32_t* kr = reinterpret_cast<const uint32_t*>(kc + (pp <= p ? pp : 0) * stride + (int64_t)g * D + lane * PL);
      const uint32_t* vr = reinterpret_cast<const uint32_t*>(vc + (pp <= p ? pp : 0) * stride + (int64_t)g * D + lane * PL);
#pragma unroll
      for (int i = 0; i < PL / 2; ++i) {
        kraw[j][i] = kr[i];
        vraw[j][i] = vr[i];
      }
    }
#pragma unroll
    for (int j = 0; j < kPfBatch; ++j) {
      if (base + j * kPfWarps > p) break;
      float kf[PL], vf[PL];
#pragma unroll
      for (int i = 0; i < PL / 2; ++i) {
        const float2 kk = __half22float2(*reinterpret_cast<const __half2*>(&kraw[j][i]));
        const float2 vv = __half22float2(*reinterpret_cast<const __half2*>(&vraw[j][i]));
        kf[2 * i] = kk.x;
        kf[2 * i + 1] = kk.y;
        vf[2 * i] = vv.x;
        vf[2 * i + 1] = vv.y;
      }
#pragma unroll
      for (int h = 0; h < kAttnMaxRep; ++h) {
        if (h >= rep) break;
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < PL; ++i) d = fmaf(qv[h][i], kf[i], d);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        const float mn = fmaxf(m[h], d);
        const float corr = __expf(m[h] - mn), w = __expf(d - mn);
        l[h] = l[h] * corr + w;
#pragma unroll
        for (int i = 0; i < PL; ++i) acc[h][i] = fmaf(acc[h][i], corr, w * vf[i]);
        m[h] = mn;
      }
    }
  }
#pragma unroll
  for (int h = 0; h < kAttnMaxRep; ++h) {
    if (h >= rep) break;
    if (lane == 0) {
      sm_m[warp][h] = m[h];
      sm_l[warp][h] = l[h];
    }
#pragma unroll
    for (int i = 0; i < PL; ++i) sm_acc[warp][h][lane * PL + i] = acc[h][i];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < rep * D; e += kPfWarps * 32) {
    const int h = e / D, dd = e - h * D;
    float mm = -INFINITY;
    for (int w = 0; w < kPfWarps; ++w) mm = fmaxf(mm, sm_m[w][h]);
    float ll = 0.0f, aa = 0.0f;
    for (int w = 0; w < kPfWarps; ++w) {
      const float c = sm_m[w][h] == -INFINITY ? 0.0f : __expf(sm_m[w][h] - mm);
      ll += sm_l[w][h] * c;
      aa += sm_acc[w][h][dd] * c;
    }
    out[(int64_t)(g * rep + h) * D + dd] = f2h(aa / ll);
  }
}

}  // namespace otf

namespace otf {
// The fused attention kernel for a query-per-KV-head ratio (compile-time for the common ones).
template <int D>
static decltype(&k_attn_rope_decode<D, 0>) attn2_kernel(int64_t rep) {
  switch (rep) {
    case 1: return k_attn_rope_decode<D, 1>;
    case 2: return k_attn_rope_decode<D, 2>;
    case 3: return k_attn_rope_decode<D, 3>;
    case 4: return k_attn_rope_decode<D, 4>;
    case 8: return k_attn_rope_decode<D, 8>;
    default: return k_attn_rope_decode<D, 0>;
  }
}
}  // namespace otf

namespace otf {
// The cluster form of the fused attention for the common query-per-KV-head ratios; null for
// the others (they keep the ticket-merge kernel).
template <int D>
static decltype(&k_attn_rope_decode_cl<D, 1>) attn_cl_kernel(int64_t rep) {
  switch (rep) {
    case 1: return k_attn_rope_decode_cl<D, 1>;
    case 2: return k_attn_rope_decode_cl<D, 2>;
    case 3: return k_attn_rope_decode_cl<D, 3>;
    case 4: return k_attn_rope_decode_cl<D, 4>;
    case 8: return k_attn_rope_decode_cl<D, 8>;
    default: return nullptr;
  }
}

// Launch the cluster form: grid (S, kv_heads, batch), clusters of S along x, S = the split count
// the ticket form would use at max_pos, at most 16 CTAs (a non-portable cluster size) for up to 4
// query heads per KV head and at most 8 for 8 (whose CTAs hold 150 registers a thread: one per
// SM).  Single sequences only: a batch keeps the ticket form, whose CTAs fill the GPU already.
// Returns false when the form does not apply (the caller launches the ticket form).
template <int D>
static bool launch_attn_cl(int64_t rep, cudaStream_t s, cudaError_t& err, const uint16_t* q, const uint16_t* kn,
                           const uint16_t* vn, const uint16_t* cs, const int* pp, uint16_t* kc, uint16_t* vc,
                           uint16_t* o, float scale, int kv_heads, int max_pos, int64_t batch, int64_t ldq,
                           int64_t ldkv, int64_t cache_stride, int64_t ldo) {
  auto* k = attn_cl_kernel<D>(rep);
  if (!k || batch != 1) return false;
  const int64_t cap = rep <= 4 ? kAttnClMax : 8;
  const int S = (int)std::max<int64_t>(1, std::min<int64_t>(cap, (max_pos + kAttnSplitPos - 1) / kAttnSplitPos));
  const int64_t chunk = (rep * D + S - 1) / S;
  const size_t dyn = (size_t)(S * chunk + S * rep * 2) * sizeof(float);
  // The shared-memory opt-in once per kernel, device and size (the first call is an eager one:
  // the decoders run warm-up steps before they capture a graph).
  {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int>, size_t> done;
    int dev = 0;
    err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return true;
    std::lock_guard<std::mutex> lock(mu);
    size_t& have = done[std::make_tuple(reinterpret_cast<const void*>(k), dev)];
    if (have < dyn) {
      err = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
      if (err != cudaSuccess) return true;
      err = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (err != cudaSuccess) return true;
      have = dyn;
    }
  }
  err = launch_pdl(k, dim3((unsigned)S, (unsigned)kv_heads, (unsigned)batch), dim3(kAttn2Threads), dyn, s,
                   (unsigned)S, q, kn, vn, cs, pp, kc, vc, o, scale, kv_heads, max_pos, ldq, ldkv, cache_stride, ldo);
  return true;
}
}  // namespace otf

using otf::check_device;
using otf::set_cuda_error;

extern "C" OTF_API int otf_rope_kv(void* q, void* k, const void* v, const void* cos_sin, const int32_t* pos,
                                   void* k_cache, void* v_cache, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                   int64_t max_pos, void* stream) {
  if (!q || !k || !v || !cos_sin || !pos || !k_cache || !v_cache) return OTF_ERR_INVALID;
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || head_dim <= 0 || head_dim % 2 || max_pos <= 0)
    return OTF_ERR_INVALID;
  int st = check_device();
  if (st != OTF_OK) return st;
  const int nvec = (int)((heads + kv_heads) * head_dim / 2);
  const int blocks = std::max(1, std::min(otf::ceil_div(std::max(nvec, (int)(kv_heads * head_dim)), 256), 148));
  return set_cuda_error(otf::launch_pdl(otf::k_rope_kv, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                                        1u, static_cast<uint16_t*>(q), static_cast<uint16_t*>(k),
                                        static_cast<const uint16_t*>(v), static_cast<const uint16_t*>(cos_sin),
                                        reinterpret_cast<const int*>(pos), static_cast<uint16_t*>(k_cache),
                                        static_cast<uint16_t*>(v_cache), (int)heads, (int)kv_heads, (int)head_dim,
                                        (int)max_pos));
}

extern "C" OTF_API int64_t otf_attn_workspace_bytes(int64_t kv_heads, int64_t head_dim, int64_t max_pos) {
  if (kv_heads <= 0 || head_dim <= 0 || max_pos <= 0) return -1;
  const int64_t max_split = (max_pos + otf::kAttnSplitPos - 1) / otf::kAttnSplitPos;
  return otf::align_up(kv_heads * 4, 256) + kv_heads * max_split * otf::kAttnMaxRep * (head_dim + 2) * 4;
}

extern "C" OTF_API int otf_attn_decode(const void* q, const void* k_cache, const void* v_cache, const int32_t* pos,
                                       void* out, float scale, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                       int64_t max_pos, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!q || !k_cache || !v_cache || !pos || !out || !workspace) return OTF_ERR_INVALID;
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || heads / kv_heads > otf::kAttnMaxRep || max_pos <= 0)
    return OTF_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return OTF_ERR_UNSUPPORTED;
  if (workspace_bytes < otf_attn_workspace_bytes(kv_heads, head_dim, max_pos)) return OTF_ERR_INVALID;
  int st = check_device();
  if (st != OTF_OK) return st;
  const int max_split = (int)((max_pos + otf::kAttnSplitPos - 1) / otf::kAttnSplitPos);
  unsigned* tickets = static_cast<unsigned*>(workspace);
  float* ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + otf::align_up(kv_heads * 4, 256));
  const dim3 grid((unsigned)kv_heads, (unsigned)max_split);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* qq = static_cast<const uint16_t*>(q);
  const auto* kc = static_cast<const uint16_t*>(k_cache);
  const auto* vc = static_cast<const uint16_t*>(v_cache);
  auto* o = static_cast<uint16_t*>(out);
  const int* pp = reinterpret_cast<const int*>(pos);
  cudaError_t e = head_dim == 128
                      ? otf::launch_pdl(otf::k_attn_decode<128>, grid, dim3(otf::kAttnThreads), 0, s, 1u, qq, kc, vc, pp, o,
                                        scale, (int)heads, (int)kv_heads, (int)max_pos, ws, tickets, max_split)
                      : otf::launch_pdl(otf::k_attn_decode<64>, grid, dim3(otf::kAttnThreads), 0, s, 1u, qq, kc, vc, pp, o,
                                        scale, (int)heads, (int)kv_heads, (int)max_pos, ws, tickets, max_split);
  return set_cuda_error(e);
}

extern "C" OTF_API int otf_attn_rope_decode(const void* q, const void* k, const void* v, const void* cos_sin,
                                            const int32_t* pos, void* k_cache, void* v_cache, void* out, float scale,
                                            int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t max_pos,
                                            void* workspace, int64_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !cos_sin || !pos || !k_cache || !v_cache || !out || !workspace) return OTF_ERR_INVALID;
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || heads / kv_heads > otf::kAttnMaxRep || max_pos <= 0)
    return OTF_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return OTF_ERR_UNSUPPORTED;
  if (workspace_bytes < otf_attn_workspace_bytes(kv_heads, head_dim, max_pos)) return OTF_ERR_INVALID;
  int st = check_device();
  if (st != OTF_OK) return st;
  const int max_split = (int)((max_pos + otf::kAttnSplitPos - 1) / otf::kAttnSplitPos);
  unsigned* tickets = static_cast<unsigned*>(workspace);
  float* ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + otf::align_up(kv_heads * 4, 256));
  const dim3 grid((unsigned)kv_heads, (unsigned)max_split);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* qq = static_cast<const uint16_t*>(q);
  const auto* kn = static_cast<const uint16_t*>(k);
  const auto* vn = static_cast<const uint16_t*>(v);
  const auto* cs = static_cast<const uint16_t*>(cos_sin);
  const int* pp = reinterpret_cast<const int*>(pos);
  auto* kc = static_cast<uint16_t*>(k_cache);
  auto* vc = static_cast<uint16_t*>(v_cache);
  auto* o = static_cast<uint16_t*>(out);
  const int64_t z = 0;
  cudaError_t e = cudaSuccess;
  if (head_dim == 128 ? otf::launch_attn_cl<128>(heads / kv_heads, s, e, qq, kn, vn, cs, pp, kc, vc, o, scale,
                                                 (int)kv_heads, (int)max_pos, 1, z, z, z, z)
                      : otf::launch_attn_cl<64>(heads / kv_heads, s, e, qq, kn, vn, cs, pp, kc, vc, o, scale,
                                                (int)kv_heads, (int)max_pos, 1, z, z, z, z))
    return set_cuda_error(e);
  e = head_dim == 128
                      ? otf::launch_pdl(otf::attn2_kernel<128>(heads / kv_heads), grid, dim3(otf::kAttn2Threads), 0, s, 1u, qq, kn,
                                        vn, cs, pp, kc, vc, o, scale, (int)heads, (int)kv_heads, (int)max_pos, ws,
                                        tickets, max_split, z, z, z, z, z)
                      : otf::launch_pdl(otf::attn2_kernel<64>(heads / kv_heads), grid, dim3(otf::kAttn2Threads), 0, s, 1u, qq, kn,
                                        vn, cs, pp, kc, vc, o, scale, (int)heads, (int)kv_heads, (int)max_pos, ws,
                                        tickets, max_split, z, z, z, z, z);
  return set_cuda_error(e);
}

extern "C" OTF_API int64_t otf_attn_workspace_bytes_batch(int64_t kv_heads, int64_t head_dim, int64_t max_pos,
                                                          int64_t batch) {
  if (kv_heads <= 0 || head_dim <= 0 || max_pos <= 0 || batch <= 0) return -1;
  const int64_t max_split = (max_pos + otf::kAttnSplitPos - 1) / otf::kAttnSplitPos;
  return otf::align_up(batch * kv_heads * 4, 256) +
         batch * kv_heads * max_split * otf::kAttnMaxRep * (head_dim + 2) * 4;
}

extern "C" OTF_API int otf_attn_rope_decode_batch(const void* q, int64_t ldq, const void* k, const void* v,
                                                  int64_t ldkv, const void* cos_sin, const int32_t* pos,
                                                  void* k_cache, void* v_cache, int64_t cache_stride, void* out,
                                                  int64_t ldo, float scale, int64_t heads, int64_t kv_heads,
                                                  int64_t head_dim, int64_t max_pos, int64_t batch, void* workspace,
                                                  int64_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !cos_sin || !pos || !k_cache || !v_cache || !out || !workspace) return OTF_ERR_INVALID;
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || heads / kv_heads > otf::kAttnMaxRep || max_pos <= 0)
    return OTF_ERR_INVALID;
  if (batch <= 0 || batch > 65535) return OTF_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return OTF_ERR_UNSUPPORTED;
  if (ldq < heads * head_dim || ldo < heads * head_dim || ldkv < kv_heads * head_dim ||
      cache_stride < max_pos * kv_heads * head_dim)
    return OTF_ERR_INVALID;
  if (workspace_bytes < otf_attn_workspace_bytes_batch(kv_heads, head_dim, max_pos, batch)) return OTF_ERR_INVALID;
  int st = check_device();
  if (st != OTF_OK) return st;
  const int max_split = (int)((max_pos + otf::kAttnSplitPos - 1) / otf::kAttnSplitPos);
  unsigned* tickets = static_cast<unsigned*>(workspace);
  float* ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + otf::align_up(batch * kv_heads * 4, 256));
  const int64_t ws_stride = kv_heads * max_split * otf::kAttnMaxRep * (head_dim + 2);
  const dim3 grid((unsigned)kv_heads, (unsigned)max_split, (unsigned)batch);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* qq = static_cast<const uint16_t*>(q);
  const auto* kn = static_cast<const uint16_t*>(k);
  const auto* vn = static_cast<const uint16_t*>(v);
  const auto* cs = static_cast<const uint16_t*>(cos_sin);
  const int* pp = reinterpret_cast<const int*>(pos);
  auto* kc = static_cast<uint16_t*>(k_cache);
  auto* vc = static_cast<uint16_t*>(v_cache);
  auto* o = static_cast<uint16_t*>(out);
  cudaError_t e = cudaSuccess;
  if (head_dim == 128 ? otf::launch_attn_cl<128>(heads / kv_heads, s, e, qq, kn, vn, cs, pp, kc, vc, o, scale,
                                                 (int)kv_heads, (int)max_pos, batch, ldq, ldkv, cache_stride, ldo)
                      : otf::launch_attn_cl<64>(heads / kv_heads, s, e, qq, kn, vn, cs, pp, kc, vc, o, scale,
                                                (int)kv_heads, (int)max_pos, batch, ldq, ldkv, cache_stride, ldo))
    return set_cuda_error(e);
  e = head_dim == 128
                      ? otf::launch_pdl(otf::attn2_kernel<128>(heads / kv_heads), grid, dim3(otf::kAttn2Threads), 0, s, 1u, qq, kn,
                                        vn, cs, pp, kc, vc, o, scale, (int)heads, (int)kv_heads, (int)max_pos, ws,
                                        tickets, max_split, ldq, ldkv, cache_stride, ldo, ws_stride)
                      : otf::launch_pdl(otf::attn2_kernel<64>(heads / kv_heads), grid, dim3(otf::kAttn2Threads), 0, s, 1u, qq, kn,
                                        vn, cs, pp, kc, vc, o, scale, (int)heads, (int)kv_heads, (int)max_pos, ws,
                                        tickets, max_split, ldq, ldkv, cache_stride, ldo, ws_stride);
  return set_cuda_error(e);
}

extern "C" OTF_API int otf_attn_prefill(void* q, int64_t ldq, void* k, const void* v, int64_t ldkv,
                                        const void* cos_sin, const int32_t* pos, void* k_cache, void* v_cache,
                                        void* out, int64_t ldo, float scale, int64_t heads, int64_t kv_heads,
                                        int64_t head_dim, int64_t max_pos, int64_t rows, void* stream) {
  if (!q || !k || !v || !cos_sin || !pos || !k_cache || !v_cache || !out) return OTF_ERR_INVALID;
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || heads / kv_heads > otf::kAttnMaxRep || max_pos <= 0)
    return OTF_ERR_INVALID;
  if (rows <= 0 || rows > max_pos || rows > 65535) return OTF_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return OTF_ERR_UNSUPPORTED;
  if (ldq < heads * head_dim || ldo < heads * head_dim || ldkv < kv_heads * head_dim) return OTF_ERR_INVALID;
  int st = check_device();
  if (st != OTF_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* qq = static_cast<uint16_t*>(q);
  auto* kc = static_cast<uint16_t*>(k_cache);
  auto* vc = static_cast<uint16_t*>(v_cache);
  const int* pp = reinterpret_cast<const int*>(pos);
  const int nvec = (int)((heads + kv_heads) * head_dim / 2);
  const dim3 rgrid((unsigned)std::max(1, std::min(otf::ceil_div(nvec, 256), 8)), (unsigned)rows);
  cudaError_t e = otf::launch_pdl(otf::k_rope_kv_rows, rgrid, dim3(256), 0, s, 1u, qq, ldq, static_cast<uint16_t*>(k),
                             static_cast<const uint16_t*>(v), ldkv, static_cast<const uint16_t*>(cos_sin), pp, kc, vc,
                             (int)heads, (int)kv_heads, (int)head_dim, (int)max_pos);
  if (e != cudaSuccess) return set_cuda_error(e);
  const dim3 agrid((unsigned)kv_heads, (unsigned)rows);
  e = head_dim == 128
          ? otf::launch_pdl(otf::k_attn_prefill<128>, agrid, dim3(otf::kPfWarps * 32), 0, s, 1u, (const uint16_t*)qq, ldq,
                       (const uint16_t*)kc, (const uint16_t*)vc, pp, static_cast<uint16_t*>(out), ldo, scale,
                       (int)heads, (int)kv_heads, (int)max_pos)
          : otf::launch_pdl(otf::k_attn_prefill<64>, agrid, dim3(otf::kPfWarps * 32), 0, s, 1u, (const uint16_t*)qq, ldq,
                       (const uint16_t*)kc, (const uint16_t*)vc, pp, static_cast<uint16_t*>(out), ldo, scale,
                       (int)heads, (int)kv_heads, (int)max_pos);
  return set_cuda_error(e);
}

int otf::attn_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, otf::g_attn_device_error, sizeof(int)) != cudaSuccess) {
    set_cuda_error(cudaGetLastError());
    return -1;
  }
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(otf::g_attn_device_error, &z, sizeof(int));
  }
  return v;
}

extern "C" OTF_API int otf_pos_advance(int32_t* pos, void* stream) {
  if (!pos) return OTF_ERR_INVALID;
  int st = check_device();
  if (st != OTF_OK) return st;
  return set_cuda_error(otf::launch_pdl(otf::k_pos_advance, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), 1u,
                                        reinterpret_cast<int*>(pos), 1));
}

extern "C" OTF_API int otf_pos_advance_batch(int32_t* pos, int64_t n, void* stream) {
  if (!pos || n <= 0 || n > (1 << 20)) return OTF_ERR_INVALID;
  int st = check_device();
  if (st != OTF_OK) return st;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148);
  return set_cuda_error(otf::launch_pdl(otf::k_pos_advance, dim3(blocks), dim3(256), 0,
                                        static_cast<cudaStream_t>(stream), 1u, reinterpret_cast<int*>(pos), (int)n));
}

// ---------------------------------------------------------------------------------------
// Decode attention without a caller-provided workspace.
//
// Some callers cannot allocate device memory for the split-KV partials: runtimes that
// hand a plugin only the tensors of the op (no allocator handle), code running under an
// allocator that forbids new allocations after warm-up, and hosts that must not call
// cudaMalloc at all.  For them the scratch lives in one fixed array that the library holds
// on every GPU that loads it, for as long as the process runs.

namespace otf {
constexpr int64_t kAttnScratchBytes = OTF_ATTN_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_attn_scratch[kAttnScratchBytes];
}  // namespace otf

// The current context, through the driver's cuCtxGetCurrent (looked up once from the runtime,
// so the library does not link libcuda).  Null if the lookup failed.
typedef int (*CtxGetCurrentFn)(void**);
static void* current_context() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  void* c = nullptr;
  if (fn && fn(&c) != 0) c = nullptr;
  return c;
}

// Device address of the scratch array in the current device's context (the array's
// host-side name is not a device address).  Looked up with cudaGetSymbolAddress on the
// first call in each context and cached per device together with that context, so a
// context torn down by cudaDeviceReset and created again is looked up afresh.
static int attn_scratch_ptr(unsigned char** out) {
  static std::mutex mu;
  static unsigned char* ptr[64] = {};
  static void* ctx[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e);
  if (dev < 0 || dev >= 64) return OTF_ERR_UNSUPPORTED;
  void* c = current_context();
  std::lock_guard<std::mutex> lk(mu);
  if (!ptr[dev] || c == nullptr || c != ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, otf::g_attn_scratch);
    if (e != cudaSuccess) return set_cuda_error(e);
    ptr[dev] = static_cast<unsigned char*>(p);
    ctx[dev] = c;
  }
  *out = ptr[dev];
  return OTF_OK;
}

extern "C" OTF_API int otf_attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                               const int32_t* pos, void* out, float scale, int64_t heads,
                                               int64_t kv_heads, int64_t head_dim, int64_t max_pos, void* stream) {
  if (!q || !k_cache || !v_cache || !pos || !out) return OTF_ERR_INVALID;
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || heads / kv_heads > otf::kAttnMaxRep || max_pos <= 0)
    return OTF_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return OTF_ERR_UNSUPPORTED;
  if (otf_attn_workspace_bytes(kv_heads, head_dim, max_pos) > otf::kAttnScratchBytes) return OTF_ERR_UNSUPPORTED;
  int st = check_device();
  if (st != OTF_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The scratch address belongs to the current device: the stream must be on that device.
  int cur = 0, sdev = 0;
  cudaError_t e = cudaGetDevice(&cur);
  if (e == cudaSuccess) e = cudaStreamGetDevice(s, &sdev);
  if (e != cudaSuccess) return set_cuda_error(e);
  if (sdev != cur) return OTF_ERR_INVALID;
  unsigned char* scratch = nullptr;
  st = attn_scratch_ptr(&scratch);
  if (st != OTF_OK) return st;
  // The per-head tickets must start at zero (a completed call leaves them there; clearing
  // them here keeps a call independent of how an earlier one ended).
  const int64_t tbytes = otf::align_up(kv_heads * 4, 256);
  e = cudaMemsetAsync(scratch, 0, (size_t)(kv_heads * 4), s);
  if (e != cudaSuccess) return set_cuda_error(e);
  const int max_split = (int)((max_pos + otf::kAttnSplitPos - 1) / otf::kAttnSplitPos);
  unsigned* tickets = reinterpret_cast<unsigned*>(scratch);
  float* ws = reinterpret_cast<float*>(scratch + tbytes);
  const dim3 grid((unsigned)kv_heads, (unsigned)max_split);
  const auto* qq = static_cast<const uint16_t*>(q);
  const auto* kc = static_cast<const uint16_t*>(k_cache);
  const auto* vc = static_cast<const uint16_t*>(v_cache);
  auto* o = static_cast<uint16_t*>(out);
  const int* pp = reinterpret_cast<const int*>(pos);
  e = head_dim == 128 ? otf::launch_pdl(otf::k_attn_decode<128>, grid, dim3(otf::kAttnThreads), 0, s, 1u, qq, kc, vc,
                                        pp, o, scale, (int)heads, (int)kv_heads, (int)max_pos, ws, tickets, max_split)
                      : otf::launch_pdl(otf::k_attn_decode<64>, grid, dim3(otf::kAttnThreads), 0, s, 1u, qq, kc, vc,
                                        pp, o, scale, (int)heads, (int)kv_heads, (int)max_pos, ws, tickets, max_split);
  return set_cuda_error(e);
}
