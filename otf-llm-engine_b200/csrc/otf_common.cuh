// Shared device helpers for the sm_100a quantized-decode kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <utility>

#include "otf_b200.h"

namespace otf {

// fp16 bit pattern <-> fp32.
__device__ __forceinline__ float h2f(uint16_t v) { return __half2float(__ushort_as_half(v)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Legacy warp-level integer MMA, m16n8k32, D = A(16x32) * B(32x8) + C, int32 accumulate.
// A is u8 (2-bit code slots) or s8 (INT8 weights); B is s8 (activation limbs).
__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Same MMA with a zero accumulator input (starts a fresh sum without zeroing registers).
__device__ __forceinline__ void mma_u8s8_z(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void st_cluster_f32_plain(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Streaming 16/8-byte loads of weights: read once, do not keep them in L1.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ld_stream8(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

// Predicated streaming loads into registers the caller zero-initialised: when the
// predicate is false the registers keep their zeros, and no instruction consumes the
// loaded value before its first real use (a select on a pending load would stall).
__device__ __forceinline__ void ld_stream16_pred(uint4& v, const void* p, bool pred) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t"
      "@q ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n\t}"
      : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w) : "l"(p), "r"((int)pred));
}
__device__ __forceinline__ void ld_stream8_pred(uint2& v, const void* p, bool pred) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %3, 0;\n\t"
      "@q ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n\t}"
      : "+r"(v.x), "+r"(v.y) : "l"(p), "r"((int)pred));
}
// 16-bit load (zero-extended into a 32-bit register), predicated the same way.
__device__ __forceinline__ void ld_u16_pred(uint32_t& v, const void* p, bool pred) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t"
      "@q ld.global.nc.u16 %0, [%1];\n\t}"
      : "+r"(v) : "l"(p), "r"((int)pred));
}

// mbarrier + TMA (bulk tensor copy) helpers.  Every wait is bounded: after
// kWaitLimit polls the waiter gives up, records the failure in g_otf_device_error
// and carries on, so a broken pipeline can never hang the GPU.
constexpr uint32_t kWaitLimit = 1u << 20;  // try_wait rounds of at most ~1 us each: about 1 s
__device__ __forceinline__ void mbar_init(uint32_t addr, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(addr), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t addr) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(addr) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(addr), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
  return ok != 0;
}
// try_wait with a 1 us suspend-time hint: the hardware parks the warp until the phase
// completes or the hint expires.  Returns false (and the caller records an error) if the
// phase has not completed after kWaitLimit rounds.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(addr), "r"(parity), "r"(1000u) : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint32_t addr, uint32_t parity) {
  if (mbar_test_wait(addr, parity)) return true;
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait_hint(addr, parity)) return true;
  return false;
}
// try_wait without a suspend-time hint (the thread is parked for a short system-defined
// time at most and released as soon as the phase completes); the wait is bounded by the
// global timer instead of a poll count: false after about one second.
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mbar_wait_spin(uint32_t addr, uint32_t parity) {
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(addr, parity)) return true;
    if (global_ns() - t0 > 1000000000ull) return false;
  }
}
// The same wait for a thread that is not on the critical path (a copy producer refilling
// slots): a short sleep between polls keeps it from taking issue slots from the warps that
// compute.
__device__ __forceinline__ bool mbar_wait_sleep(uint32_t addr, uint32_t parity) {
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    __nanosleep(64);
    if (mbar_try_wait(addr, parity)) return true;
    if (global_ns() - t0 > 1000000000ull) return false;
  }
}
// 2-D tiled bulk tensor load into this CTA's shared memory, completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(tmap), "r"(x), "r"(y), "r"(mbar) : "memory");
}
// 4-byte async copy global -> shared with zero fill: copies src_bytes (0..4) bytes,
// zero-fills the rest (src_bytes == 0 reads nothing).
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// Arrive on an mbarrier once all of this thread's prior cp.async copies have landed
// (the arrival counts toward the barrier's expected count).
__device__ __forceinline__ void cp_async_mbar_arrive(uint32_t mbar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(mbar) : "memory");
}
// 16-byte async copy global -> shared, cached in L2 only; src_bytes 0 zero-fills the
// destination without reading the source.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// Contiguous bulk copy global -> this CTA's shared memory (16-byte aligned addresses, size a
// multiple of 16), completing on an mbarrier.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(src), "r"(bytes), "r"(mbar) : "memory");
}
// Four 8x8 b16 matrices (8 rows of 16 bytes each; lane l gives the row address of matrix
// l / 8): lane (g, t) receives 32-bit word t of row g of each matrix, the mma.sync A layout.
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr) : "memory");
}
// 5th-generation tensor core (tcgen05) helpers, single-CTA forms.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, fp16 inputs, fp32 accumulate (kind::f16).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, fp16 inputs, fp32 accumulate: the A operand read from
// tensor memory (128 lanes = rows, K/2 32-bit columns of two fp16 each).
__device__ __forceinline__ void tc_mma_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// 32 TMEM lanes x 16 consecutive 32-bit columns from registers: thread t of the warp writes
// lane (base lane + t).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]) : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Arrive (once) on an mbarrier when every tcgen05 operation this thread issued so far completes.
__device__ __forceinline__ void tc_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar) : "memory");
}
// 32 TMEM lanes x 8 consecutive 32-bit columns: thread t of the warp gets lane (base lane + t).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle layout: rows of
// 128 bytes, 8-row groups 1024 bytes apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t tc_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Thread-block-cluster helpers (distributed shared memory).
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_v2(uint32_t addr, uint32_t a, uint32_t b) {
  asm volatile("st.shared::cluster.v2.u32 [%0], {%1, %2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Split cluster barrier: arrive on entry, wait before the first distributed-shared-memory
// access, so that every CTA of the cluster is known to be running when a peer's shared
// memory is touched (the arrive costs nothing; by the wait the peers have long started).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

// Geometry shared by the 2-bit GEMV kernels (gemv2b.cu) and the decode-step kernel
// (decode_step.cu): a stage is 16 rows x 128 code bytes (512 codes) staged at a 144-byte
// row pitch (the consumers' 16-byte reads are bank-conflict-free), followed by the rows'
// scales.
constexpr int kRows = 16;                   // rows per tile (the m16 of the MMA)
constexpr int kChunk = 128;                 // code bytes per row per stage (512 codes)
constexpr int kChunkCodes = 4 * kChunk;
constexpr int kPitch = kChunk + 16;         // shared-memory row pitch of a stage

// Table geometry for W words per block: limb row SL = 32W+16 bytes (hi row, then lo row),
// block stride SB a multiple of 128 so that every block's two real reads fall on the same
// two 16-byte bank groups, and the all-zero block read by the other lanes sits 64 bytes off
// them (no bank conflict between the real and the zero reads of one instruction).
__host__ __device__ constexpr int tbl_sl(int W) { return 32 * W + 16; }
__host__ __device__ constexpr int tbl_sb(int W) { return (2 * tbl_sl(W) + 127) / 128 * 128; }

// Bytes of scales per row of a stage: the stage's 512/G groups plus 4 bytes of padding
// (rows of a stage then start on distinct banks).
__host__ __device__ inline int scale_pitch(int G) { return 2 * (kChunkCodes / G) + 4; }

// Words per 16W-code block for group size G (the block never straddles a group).
__host__ __device__ constexpr int words_for(int G) { return G >= 64 ? 4 : 2; }

// 2^e as a float for -126 <= e <= 127 (exact).
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((e + 127) << 23); }

// Round-to-nearest-even of |v| < 2^22 via the 1.5*2^23 magic constant.
__device__ __forceinline__ int rint_small(float v) { return __float_as_int(v + 12582912.0f) - 0x4B400000; }

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  const uint32_t p01 = __byte_perm((uint32_t)a, (uint32_t)b, 0x0040);
  const uint32_t p23 = __byte_perm((uint32_t)c, (uint32_t)d, 0x0040);
  return __byte_perm(p01, p23, 0x5410);
}

// Choose the power-of-two exponent E for 16-bit fixed point so that
// maxabs * 2^E lies in [8192, 16384): |X| <= 16384 keeps both s8 limbs of X
// (X = 256*hi + lo, lo in [-128,127]) inside the s8 range.
__device__ __forceinline__ int fixed_point_exp(float maxabs) {
  if (!(maxabs > 0.0f)) return 0;
  int e;
  frexpf(maxabs, &e);  // maxabs = f * 2^e, f in [0.5, 1)
  return 14 - e;
}

// Split an integer |X| <= 16384 into s8 limbs: X = 256*hi + lo, lo in [-128,127].
__device__ __forceinline__ void split_limbs(int X, int& hi, int& lo) {
  hi = (X + 128) >> 8;
  lo = X - 256 * hi;
}

__host__ __device__ constexpr int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Programmatic dependent launch inside a kernel: pdl_trigger lets the next kernel in the
// stream begin launching; pdl_wait blocks until the previous kernel has completed and its
// memory is visible.  Both are no-ops when the launch carried no PDL attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

#ifndef __CUDACC_RTC__
// Launch with the programmatic-stream-serialization attribute (and optional cluster size),
// so a kernel may start while its predecessor drains; every kernel of this library reads
// predecessor outputs only after pdl_wait().
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              unsigned cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
#endif
__host__ __device__ constexpr int64_t align_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

}  // namespace otf
