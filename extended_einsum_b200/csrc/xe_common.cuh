// Shared device helpers for the sm_100a kernels: error recording, bounded
// mbarrier waits, tcgen05 (TMEM / UMMA) wrappers written as inline PTX.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/xe_b200.h"

#ifndef __CUDACC__
#error "xe_common.cuh is CUDA-only"
#endif

namespace xe {

// ---------------------------------------------------------------------------
// Device status word.  A bounded wait that runs out stores
// (XE_ERR_DEVICE_TIMEOUT << 16) | site here and the kernel winds down
// instead of trapping; the host reads it with xe_device_status().
__device__ int g_device_status = 0;

enum WaitSite : int {
  kSiteGemmFull = 1,
  kSiteGemmEmpty = 2,
  kSiteGemmAccFull = 3,
  kSiteGemmAccEmpty = 4,
  kSiteGemmDrain = 5,
  // finer sites, distinguished only by the wait-time counters below
  kSiteAStaged = 6,
  kSiteAShiftSlot = 7,
  kSiteAStage = 8,
  kSiteBStage = 9,
  kSiteMmaCorr = 10,
  kSiteMmaChunk = 11,
  kSiteMmaFull = 12,
  kSiteDrainChunk = 13,
  kSiteDrainShift = 14,
  kSiteProducer = 15,
  kNumSites = 16,
  kSiteSoftmax = 16,      // the prefetching row softmax (not among the wait-time counters)
  kSiteWaitProbe = 17,    // xe_wait_probe, the test kernel whose barrier may never complete
  kSiteDrainCopies = 18,  // wind-down: bulk copies still landing in shared memory
};

#ifdef XE_PROFILE
// Cycles spent in each wait site, summed over threads that waited, and in
// timed code segments (profiling builds only: compiled with -DXE_PROFILE).
__device__ unsigned long long g_wait_cycles[kNumSites];
__device__ unsigned long long g_segment_cycles[kNumSites];
#define XE_SEGMENT_BEGIN(name) const long long name##_t0 = clock64()
#define XE_SEGMENT_END(name, idx) atomicAdd(&::xe::g_segment_cycles[idx], (unsigned long long)(clock64() - name##_t0))
#else
#define XE_SEGMENT_BEGIN(name)
#define XE_SEGMENT_END(name, idx)
#endif

#ifdef XE_TRACE_TILES
// Per-tile event times (clock64) of CTA 0's first 64 tiles, trace builds only.
constexpr int kTraceTiles = 64, kTraceEvents = 16;
__device__ long long g_trace[kTraceTiles * kTraceEvents];
#define XE_TILE_TRACE(n, ev)                                                                                 \
  do {                                                                                                       \
    if (blockIdx.x == 0 && (int)(n) < ::xe::kTraceTiles) ::xe::g_trace[(n) * ::xe::kTraceEvents + (ev)] = clock64(); \
  } while (0)
#else
#define XE_TILE_TRACE(n, ev)
#endif

// About two seconds: far above any legitimate wait in these kernels.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

// The limit of the ordinary waits, per device (xe_set_wait_timeout_ns; kWaitTimeoutNs by default).
// Waits that guard the release of resources (tensor-core work or bulk copies still in flight
// when a CTA winds down) keep the fixed kWaitTimeoutNs, so that a short limit never frees TMEM
// or shared memory under an operation that has not finished.
__constant__ uint64_t g_wait_timeout_ns = kWaitTimeoutNs;

__device__ __forceinline__ void record_timeout(int site) {
  atomicCAS(&g_device_status, 0, (XE_ERR_DEVICE_TIMEOUT << 16) | site);
}

// Data-dependent index checks (a uint8 pixel value at or above the number of
// states): the access is clamped into bounds and the first offence recorded.
enum IndexSite : int { kSiteGatherState = 32, kSiteGemmGatherState = 33 };

__device__ __forceinline__ void record_bad_index(int site) {
  atomicCAS(&g_device_status, 0, (XE_ERR_INVALID_ARGUMENT << 16) | site);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false (and
// records the site) if it has not completed after kWaitTimeoutNs, or at once
// if another wait of this kernel launch already gave up (`abort` flag in
// shared memory), so that every role of the CTA winds down promptly.  Waits
// that guard the release of resources (outstanding tensor-core work before
// TMEM is freed) pass honor_abort = false and rely on the time limit alone.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int site, volatile int* abort,
                                          bool honor_abort = true) {
  const uint32_t addr = smem_u32(bar);
#ifdef XE_PROFILE
  // the first try_wait may itself suspend the thread for a while: count it too
  const long long c0 = clock64();
  if (mbar_try_wait(addr, parity)) {
    atomicAdd(&g_wait_cycles[site & (kNumSites - 1)], (unsigned long long)(clock64() - c0));
    return true;
  }
#else
  if (mbar_try_wait(addr, parity)) return true;
#endif
  const uint64_t limit = honor_abort ? g_wait_timeout_ns : uint64_t(kWaitTimeoutNs);
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(addr, parity)) {
#ifdef XE_PROFILE
      atomicAdd(&g_wait_cycles[site & (kNumSites - 1)], (unsigned long long)(clock64() - c0));
#endif
      return true;
    }
    if ((i & 255u) == 0) {
      if (honor_abort && *abort) return false;
      if (globaltimer_ns() - t0 > limit) {
        *abort = 1;
        record_timeout(site);
        return false;
      }
    }
  }
}

// The ring barriers a producer thread armed last (arrive.expect_tx + bulk copies), with the
// phase parity of that arming.  A CTA that winds down after an abort drains them before it
// exits: a bulk copy must not land in shared memory that the CTA no longer owns.  One bit per
// barrier of a ring of at most 32.  Kept in shared memory beside the abort flag (cleared with
// it), so that no role carries it in registers.
struct ArmedCopies {
  uint32_t armed, parity;

  __device__ __forceinline__ void note(int slot, uint32_t phase) {
    const uint32_t bit = 1u << slot;
    armed |= bit;
    parity = (parity & ~bit) | ((phase & 1u) << slot);
  }

  // Waits (fixed limit) until the last armed phase of each noted barrier has completed.
  __device__ __forceinline__ void drain(uint64_t* bars, volatile int* abort) const {
    for (uint32_t m = armed; m != 0u; m &= m - 1u) {
      const int slot = __ffs(m) - 1;
      mbar_wait(&bars[slot], (parity >> slot) & 1u, kSiteDrainCopies, abort, /*honor_abort=*/false);
    }
  }
};

// A wait by every lane of a warp whose next steps are warp-collective
// (tcgen05.ld / tcgen05.st are .sync.aligned): the lanes leave the spin loop at
// different times, so the warp is reconverged here, and a timeout seen by any
// lane is seen by all of them.  `pre_ok` carries the outcome of an earlier
// per-lane wait of the same step into this vote (a lane whose earlier wait ran
// out does not wait again: it set the abort flag, which ends the others' waits),
// so that a step takes one vote however many barriers it waits on.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int site, volatile int* abort,
                                               bool pre_ok = true) {
  const bool ok = pre_ok && mbar_wait(bar, parity, site, abort);
  return __all_sync(0xffffffffu, ok);
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (tensor core) reads.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, UMMA issue, commit, TMEM loads.
template <uint32_t kCols>
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem) {
  static_assert(kCols >= 32 && kCols <= 512 && (kCols & (kCols - 1)) == 0, "TMEM columns: power of two in [32,512]");
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "n"(kCols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

template <uint32_t kCols>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "n"(kCols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem], kind::tf32, one CTA.
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of the calling warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  __syncwarp();  // .sync.aligned: the whole warp, converged
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() {
  __syncwarp();
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors (every tile base is 1024-byte aligned).
//
// K-major tiles use the 128-byte swizzle (layout type 2): 128-byte rows,
// 16-byte chunk index XOR (row & 7), 8-row groups.  MN-major TF32 tiles must
// use the 128-byte swizzle with 32-byte atoms (layout type 1): 128-byte
// k-rows along MN, 32-byte chunk index XOR (k-row & 3), 4-row groups.
enum : uint32_t { kLayoutSW128Base32B = 1, kLayoutSW128 = 2 };

// Shared-memory matrix descriptor: start address, leading and stride byte
// offsets (16-byte units), descriptor version 1, layout type.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;  // version
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::tf32 with fp32 accumulation.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                       // D format: F32
         | (2u << 7)                     // A format: TF32
         | (2u << 10)                    // B format: TF32
         | ((a_mn_major ? 1u : 0u) << 15)  // A major
         | ((b_mn_major ? 1u : 0u) << 16)  // B major
         | ((uint32_t)(n >> 3) << 17)    // N / 8
         | ((uint32_t)(m >> 4) << 24);   // M / 16
}

// ---------------------------------------------------------------------------
// Scalar helpers
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Splits an fp32 value into hi + lo, both exactly representable in TF32 to
// within 2^-22 relative, for the three-pass (hi*hi + hi*lo + lo*hi) product.
__device__ __forceinline__ void split_tf32(float e, float& hi, float& lo) {
  hi = tf32_round(e);
  float rest = e - hi;
  // inf/nan carry all information in hi; keep lo finite so that the
  // correction products do not turn an overflow into NaN.
  lo = isfinite(hi) ? tf32_round(rest) : 0.0f;
}

__device__ __forceinline__ float4 ldg_nc_v4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float ldg_nc(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ void sts_v4(uint32_t saddr, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(saddr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ void stg_v4(float* p, float4 v) {
  asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

}  // namespace xe
