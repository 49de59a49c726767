// Device side of the tensor-parallel peer all-reduce (otf_ar_*): the peer table and the
// produce / receive / release steps that the GEMV kernels and the standalone push and
// finish kernels share.
//
// Every rank owns one receive region in its own HBM, mapped into every other rank's
// address space through CUDA IPC.  Buffer b of a region holds world slots of max_elems
// 8-byte words; the word for element k from rank s is (tag << 32) | fp32 bits.  One
// aligned 8-byte store is single-copy atomic, so a reader sees either the old word or the
// new one, never a mix: a producer needs no fence and no separate flag -- it stores its
// words into slot[my rank] of every rank's buffer over NVLink -- and a consumer polls the
// words it needs until their tags equal the use count it expects (bounded: once a
// thread's polling budget is spent it records an error and stops waiting).
//
// The tag of the n-th exchange through buffer b is n: each rank keeps epoch[b] (the
// exchanges through b it has consumed), producers write epoch[b] + 1, consumers expect
// epoch[b] + 1, and the last consumer CTA of a launch increments epoch[b].  Every rank
// runs the same sequence of exchanges, so the counts agree.  Reuse is safe because
// consecutive exchanges alternate buffers: a rank produces into buffer b again only after
// it consumed the exchange in between, which every rank produced only after finishing its
// own consumption of b (kernels on a stream complete in order, and every kernel here waits
// for its predecessor before it exits).
#pragma once

#include "otf_common.cuh"

namespace otf {

constexpr int kArWorld = OTF_AR_MAX_WORLD;
constexpr uint32_t kArSpinLimit = 1u << 20;   // polls per thread (about a second) before giving up

struct ArPeers {
  unsigned long long* data[2][kArWorld];  // rank r's slots of buffer b, as mapped in this process
  unsigned* epoch[2];                     // exchanges through buffer b this rank has consumed
  unsigned* done[2];                      // consumer CTAs of the running launch that finished reading
  int rank, world;
  long long max_elems;
};

// Tag of the exchange now running through buffer b (written by the previous consumer
// launch on this rank, so a plain load after the predecessor's completion sees it).
__device__ __forceinline__ unsigned ar_tag(const ArPeers* P, int b) {
  return *reinterpret_cast<const volatile unsigned*>(P->epoch[b]) + 1u;
}

__device__ __forceinline__ void st_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void ld_sys_v2u64(const unsigned long long* p, unsigned long long& a,
                                             unsigned long long& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ unsigned long long ld_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Store one produced row value into slot[my rank] of every rank's buffer b.
__device__ __forceinline__ void ar_put(const ArPeers* P, int b, int64_t row, float v, unsigned tag) {
  const int world = P->world;
  const int64_t off = (int64_t)P->rank * P->max_elems + row;
  const unsigned long long w = ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
#pragma unroll 1
  for (int r = 0; r < world; ++r) st_sys_u64(P->data[b][r] + off, w);
}

__device__ __forceinline__ float clamp_h(float v) { return fminf(fmaxf(v, -65504.0f), 65504.0f); }

// Poll two words until both carry `tag` (or the thread's budget runs out: then the error
// flag is raised through *err and the values are used as they are).
__device__ __forceinline__ void ar_recv2(const unsigned long long* p, unsigned tag, uint32_t& budget, int& err,
                                         float& v0, float& v1) {
  unsigned long long a, c;
  ld_sys_v2u64(p, a, c);
  while (((unsigned)(a >> 32) != tag || (unsigned)(c >> 32) != tag) && budget > 0) {
    --budget;
    __nanosleep(32);
    ld_sys_v2u64(p, a, c);
  }
  if (budget == 0 && ((unsigned)(a >> 32) != tag || (unsigned)(c >> 32) != tag)) err = 1;
  v0 = __uint_as_float((unsigned)a);
  v1 = __uint_as_float((unsigned)c);
}

// Sum over ranks (rank order) of 8 consecutive received values at k0 (k0 % 8 == 0),
// rounded to fp16 and clamped; returned as 8 packed halves.
__device__ __forceinline__ uint4 ar_sum8(const ArPeers* P, int b, int64_t k0, unsigned tag, uint32_t& budget,
                                         int& err) {
  const unsigned long long* base = P->data[b][P->rank] + k0;
  const int world = P->world;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
  for (int r = 0; r < world; ++r) {
    const unsigned long long* s = base + (int64_t)r * P->max_elems;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float v0, v1;
      ar_recv2(s + 2 * i, tag, budget, err, v0, v1);
      acc[2 * i] += v0;
      acc[2 * i + 1] += v1;
    }
  }
  uint4 out;
  uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    o[i] = (uint32_t)f2h(clamp_h(acc[2 * i])) | ((uint32_t)f2h(clamp_h(acc[2 * i + 1])) << 16);
  return out;
}

// The same for one value.
__device__ __forceinline__ uint16_t ar_sum1(const ArPeers* P, int b, int64_t k, unsigned tag, uint32_t& budget,
                                            int& err) {
  const unsigned long long* base = P->data[b][P->rank] + k;
  float acc = 0.0f;
#pragma unroll 1
  for (int r = 0; r < P->world; ++r) {
    const unsigned long long* s = base + (int64_t)r * P->max_elems;
    unsigned long long w = ld_sys_u64(s);
    while ((unsigned)(w >> 32) != tag && budget > 0) {
      --budget;
      __nanosleep(32);
      w = ld_sys_u64(s);
    }
    if ((unsigned)(w >> 32) != tag) err = 1;
    acc += __uint_as_float((unsigned)w);
  }
  return f2h(clamp_h(acc));
}

// One thread per consumer CTA, after all of the CTA's reads of buffer b: count the CTA;
// the last one of the launch advances the buffer's use count.
__device__ __forceinline__ void ar_consumed(const ArPeers* P, int b) {
  __threadfence();
  if (atomicAdd(P->done[b], 1u) == gridDim.x * gridDim.y * gridDim.z - 1u) {
    *reinterpret_cast<volatile unsigned*>(P->epoch[b]) += 1u;
    *reinterpret_cast<volatile unsigned*>(P->done[b]) = 0u;
    __threadfence();
  }
}

}  // namespace otf
