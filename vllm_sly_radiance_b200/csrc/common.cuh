// Shared device helpers for the sm_100a kernels: mbarriers, TMA, tcgen05 (TMEM alloc, MMA,
// commit, loads), cluster/DSMEM access, fp8/fp4 conversions, bounded waits with an error word.
//
// Every spin-wait in this library is bounded: after its time limit it records an error code
// into the caller's status word (if any) and gives up, so a kernel never hangs a GPU.
//
// Status word (int32[4], one per device): [0] error code (0 = ok), [1] reserved, [2] mbarrier
// wait limit in microseconds, [3] peer-flag wait limit in microseconds.  A limit of 0 selects the
// compile-time default; the host sets them at run time (ops.kernels.set_wait_limits).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define DEVI __device__ __forceinline__

namespace rad {

constexpr uint64_t kWaitNs = 200ull * 1000ull * 1000ull;   // 200 ms wall-clock bound per mbarrier wait

// error codes written to status words
enum StatusCode : int {
  kOk = 0,
  kErrMbarTimeout = 1,
  kErrPeerTimeout = 2,
  kErrBounds = 3,
  kErrTmemAlloc = 4,
};

DEVI uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

DEVI bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
DEVI void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
DEVI void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
DEVI void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

DEVI void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
DEVI void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
DEVI bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
DEVI uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait limit of status-word slot `slot` (2: mbarrier, 3: peer flags), default when unset.
DEVI uint64_t wait_limit_ns(const int* status, int slot, uint64_t dflt) {
  if (status == nullptr) return dflt;
  const int us = reinterpret_cast<const volatile int*>(status)[slot];
  return us > 0 ? (uint64_t)us * 1000ull : dflt;
}

// Named-barrier sync of `nthreads` threads (barrier `id`) that ORs a per-thread flag: every
// participant gets the same answer, so a loop that leaves on it leaves in all of its warps
// together (a warp that left alone would strand the others at the next sync of the barrier).
DEVI bool bar_sync_or(int id, int nthreads, bool flag) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((int)flag), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// Bounded wait (200 ms of wall clock by default).  A warp whose partner warps wait on the
// preceding kernel (griddepcontrol.wait) waits on it too before its first bounded wait, so the
// bound never covers the preceding kernel's run time.  Returns false (and flags *err) on timeout.
DEVI bool mbar_wait(uint64_t* bar, uint32_t phase, int* err) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = wait_limit_ns(err, 2, kWaitNs);
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, phase)) return true;
    if (globaltimer_ns() - t0 > limit) break;
  }
  if (err) atomicExch(err, (int)kErrMbarTimeout);
  return false;
}

// ---------------------------------------------------------------------------------------------
// TMA
// ---------------------------------------------------------------------------------------------
DEVI void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(desc) : "memory");
}
DEVI void tma_load_2d(void* smem_dst, const void* desc, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(desc), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
DEVI void tma_load_2d_hint(void* smem_dst, const void* desc, uint64_t* bar, int c0, int c1,
                           uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(desc), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
// plain (untiled) bulk copy global -> shared, 16-byte aligned, size multiple of 16
DEVI void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
DEVI uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
DEVI uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------------------------
// Allocate `ncols` TMEM columns (power of two >= 32); the base address lands in *dst_smem.
// Must be executed by one full warp.
DEVI void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
DEVI void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
DEVI void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
DEVI void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DEVI void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (sm100 format): K-major tile with 128B swizzle, rows of
// 128 bytes, 8-row core groups 1024 bytes apart.
DEVI uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);          // start address  [0,14)
  d |= (uint64_t)(16 >> 4) << 16;                    // LBO (unused for swizzled K-major) [16,30)
  d |= (uint64_t)(1024 >> 4) << 32;                  // SBO = 8 rows * 128 B  [32,46)
  d |= (uint64_t)1 << 46;                            // version = 1 (sm100)   [46,48)
  d |= (uint64_t)2 << 61;                            // layout: SWIZZLE_128B  [61,64)
  return d;
}
// Non-swizzled descriptor for tcgen05.cp sources (scale-factor atoms).
DEVI uint64_t sdesc_plain(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// Block-scaled MMA, A and B from shared memory, D in TMEM, scale factors in TMEM.
DEVI void mma_mxf8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                       uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// Plain f16/bf16 MMA (kind::f16), fp32 accumulate.
DEVI void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// fp8 MMA (kind::f8f6f4), fp32 accumulate.
DEVI void mma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05 ops of this thread complete.
DEVI void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// Copy a 32-row x 128-bit smem block into TMEM, replicated into all four lane quarters.
DEVI void tmem_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// TMEM -> registers: 32 lanes x 32 bit, 16 consecutive columns per thread.
DEVI void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
DEVI void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
}
DEVI void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
DEVI void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}
DEVI void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------
// clusters / distributed shared memory
// ---------------------------------------------------------------------------------------------
DEVI uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
DEVI void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
DEVI void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
DEVI void cluster_sync() {
  cluster_arrive();
  cluster_wait();
}
// map a local shared address to the same offset in CTA `rank` of the cluster
DEVI uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
DEVI float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}

// ---------------------------------------------------------------------------------------------
// system-scope flags (peer memory) with bounded waits
// ---------------------------------------------------------------------------------------------
DEVI uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
DEVI void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// ---------------------------------------------------------------------------------------------
// GEMM -> all-reduce push (tensor parallel, NVLink peer memory).  Every rank owns one receive
// buffer, mapped into every peer:
//   [.. epoch u32 @ 64, done u32 @ 68 ..][data @ 256: two parity halves of half_words words]
//   half: world source slots x M rows x ld/2 flag-in-word ("LL") words: low 32 bits = two bf16,
//   high 32 bits = the sequence number of the call (epoch + 1) that wrote them
// A row-parallel GEMM stores each finished output tile as LL words into its own source slot of
// every peer's buffer; the receiving kernel polls its local words until they carry the current
// sequence, reduces them, and its last CTA advances the epoch.
// ---------------------------------------------------------------------------------------------
struct PushArgs {
  uint8_t* peer[8];
  int world;        // 0: no push (plain output)
  int rank;
  int64_t half_words;
  int ld;           // row length (output features)
};
constexpr int kPushEpochOff = 64;
constexpr int kPushDoneOff = 68;
constexpr int kPushDataOff = 256;
DEVI uint32_t push_seq(const PushArgs& pa) {
  return *reinterpret_cast<volatile const uint32_t*>(pa.peer[pa.rank] + kPushEpochOff) + 1u;
}
// source slot `src` (M rows x ld/2 words) of parity `par` in rank p's buffer
DEVI uint64_t* push_slot(const PushArgs& pa, int p, uint32_t par, int src, int M) {
  return reinterpret_cast<uint64_t*>(pa.peer[p] + kPushDataOff) + (int64_t)par * pa.half_words +
         (size_t)src * M * (pa.ld / 2);
}
DEVI void st_ll_pair(uint64_t* p, float lo, float hi, uint32_t seq) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  const uint32_t d = *reinterpret_cast<uint32_t*>(&h);
  asm volatile("st.volatile.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(d), "r"(seq) : "memory");
}

// spin until *p >= target (wrap-safe); false + error after `timeout_ns` of wall clock
DEVI bool wait_flag_geq(const uint32_t* p, uint32_t target, int* err, int code,
                        uint64_t timeout_ns = kWaitNs) {
  if ((int32_t)(ld_acquire_sys(p) - target) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = wait_limit_ns(err, 3, timeout_ns);
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if ((int32_t)(ld_acquire_sys(p) - target) >= 0) return true;
    if (globaltimer_ns() - t0 > limit) break;
  }
  if (err) atomicExch(err, code);
  return false;
}

// ---------------------------------------------------------------------------------------------
// numeric helpers
// ---------------------------------------------------------------------------------------------
DEVI float to_f(float x) { return x; }
DEVI float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> DEVI T from_f(float x);
template <> DEVI float from_f<float>(float x) { return x; }
template <> DEVI __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

DEVI float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// e4m3 RNE with saturation to +-448
DEVI uint8_t f32_to_e4m3(float x) {
  x = fminf(fmaxf(x, -448.f), 448.f);
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
DEVI float e4m3_to_f32(uint8_t v) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)v, __NV_E4M3);
  return __half2float(__half(h));
}
// two e4m3 from two floats, packed low = a
DEVI uint16_t f32x2_to_e4m3x2(float a, float b) {
  a = fminf(fmaxf(a, -448.f), 448.f);
  b = fminf(fmaxf(b, -448.f), 448.f);
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

DEVI float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}
DEVI float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}

}  // namespace rad

// ---------------------------------------------------------------------------------------------
// programmatic dependent launch (PDL)
// ---------------------------------------------------------------------------------------------
namespace rad {
// Block until the preceding kernel in the stream has completed and its writes are visible.
DEVI void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel in the stream to start its prologue (it still waits in pdl_wait()).
DEVI void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
}  // namespace rad

#ifndef __CUDACC_RTC__
#include <cuda_runtime.h>
#include <cstdlib>
#include <cstring>
namespace rad {
// RADIANCE_PDL=0 launches every kernel without programmatic dependencies (A/B switch)
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("RADIANCE_PDL");
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}
// Launch with the programmatic-stream-serialization attribute: the kernel may start while its
// predecessor drains; every kernel of this library calls pdl_wait() before reading the
// predecessor's outputs.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
}  // namespace rad
#endif
