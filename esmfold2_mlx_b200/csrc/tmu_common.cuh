// Shared device helpers for the sm_100a triangle-multiplicative-update kernels.
//
// Everything here is hand-written inline PTX for Blackwell (sm_100a):
//   * mbarrier init / arrive / expect-tx / bounded parity wait,
//   * TMA tiled loads and stores (cp.async.bulk.tensor; every load fills only its own CTA),
//   * tcgen05: TMEM alloc/dealloc, kind::f16 MMA with fp32 accumulation in TMEM, commit to an
//     mbarrier, and 32x32b TMEM loads for the epilogues,
//   * shared-memory matrix descriptors for 128-byte-swizzled K-major and MN-major operands.
//
// Every spin-wait is bounded: after `timeout_ns` of %globaltimer time it records an error code
// and the wait site in the status word of the caller's workspace, raises a CTA-wide abort flag
// and returns false, so the kernel winds down (draining its own copies and MMAs with bounded
// waits) and exits with the status readable from the host.  Nothing here traps.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace tmu {

// ------------------------------------------------------------------------------------------
// status word (first bytes of the caller's workspace)
// ------------------------------------------------------------------------------------------
// The device status word (the first bytes of a TMU_STATUS_BYTES block).  code/site/block hold the
// first error of the current call: the first kernel of tmu_trimul / tmu_pair_block clears them.
// first_code/first_site hold the first error since the block was last cleared by
// tmu_reset_status, which no kernel clears, so one read covers a whole sequence of calls.
struct DeviceStatus {
  unsigned int code;   // 0 ok, else a TMU_STATUS_* value (tmu.h)
  unsigned int site;   // kernel-specific id of the wait that gave up
  unsigned int block;  // blockIdx.x of the first CTA that gave up
  unsigned int pad;
  unsigned int first_code;  // first error since tmu_reset_status
  unsigned int first_site;
  unsigned int trace_flag;  // set by the host to record this launch's span (below)
  unsigned int pad2;
  unsigned long long t_start;  // min over CTAs of the %globaltimer value after the dependency wait
  unsigned long long t_end;    // max over CTAs of the %globaltimer value at exit
};

// Record an error: the first one wins in both the per-call and the since-reset fields.
__device__ __forceinline__ void record_status(DeviceStatus* s, unsigned int code, unsigned int site) {
  if (atomicCAS(&s->code, 0u, code) == 0u) {
    s->site = site;
    s->block = blockIdx.x;
  }
  if (atomicCAS(&s->first_code, 0u, code) == 0u) s->first_site = site;
}

constexpr unsigned int kStatusDeviceTimeout = 6;  // TMU_ERR_DEVICE_TIMEOUT in tmu.h
constexpr unsigned int kStatusLayout = 9;         // TMU_ERR_SMEM_LAYOUT in tmu.h

struct WaitCtx {
  DeviceStatus* status;   // global
  volatile int* abort;    // shared, CTA-wide
  uint64_t timeout_ns;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void raise_abort(const WaitCtx& ctx, unsigned int site) {
  *ctx.abort = 1;
  record_status(ctx.status, kStatusDeviceTimeout, site);
  __threadfence();
}

// Launch-span trace, a measurement aid.  When the host sets trace_flag in a status block, every
// CTA of a kernel given that block records when it passes its dependency wait (min over CTAs)
// and when it finishes (max), so a chain of kernels launched with programmatic dependent launch
// can be timed kernel by kernel inside the chain (an event between two launches would break the
// chain).  One thread per CTA, the last one, takes the marks: it belongs to a warp that has no
// work at the start, so the flag's load never delays a producer.
__device__ __forceinline__ bool trace_enabled(const DeviceStatus* s) {
  return threadIdx.x == blockDim.x - 1 && *reinterpret_cast<const volatile unsigned int*>(&s->trace_flag) != 0u;
}

__device__ __forceinline__ void trace_mark_start(DeviceStatus* s, bool on) {
  if (on) atomicMin(&s->t_start, static_cast<unsigned long long>(globaltimer_ns()));
}

__device__ __forceinline__ void trace_mark_end(DeviceStatus* s, bool on) {
  if (on) atomicMax(&s->t_end, static_cast<unsigned long long>(globaltimer_ns()));
}

// ------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the phase completes
// or about `hint_ns` pass, instead of re-polling and taking issue slots from working warps.
__device__ __forceinline__ bool mbar_test_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

constexpr uint32_t kSuspendHintNs = 200000;  // 0.2 ms: one timer/abort check per sleep

// Wait until the phase with parity `parity` of `bar` has completed.  Bounded: returns false
// (after raising the abort) when `ctx.timeout_ns` elapses or another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const WaitCtx& ctx,
                                          unsigned int site) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_test_sleep(bar, parity, kSuspendHintNs)) return true;
    if (*ctx.abort) return false;
    if (globaltimer_ns() - t0 > ctx.timeout_ns) {
      raise_abort(ctx, site);
      return false;
    }
  }
}

// Bounded wait used while winding down after an abort: never raises, gives up silently.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_test_sleep(bar, parity, kSuspendHintNs)) {
    if (globaltimer_ns() - t0 > limit_ns) return;
  }
}

// Programmatic dependent launch.  A kernel launched with the programmatic-serialisation
// attribute may start while the previous kernel in the stream is still running; it must execute
// griddep_wait() before it touches anything that kernel writes or reads.  griddep_trigger() lets
// the next kernel start launching (its own griddep_wait still waits for this grid to finish).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void griddep_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// A group of warps waits for one or two mbarrier phases: one thread (`leader`) waits (bounded)
// and the group meets at named barrier `bar_id`, where the other warps park without issuing
// instructions.  The verdict goes through flags[count & 1] (count = this group's wait counter,
// advanced identically by every thread): a slow reader of wait k still finds wait k's verdict,
// because the leader writes that slot again only after every thread has reached wait k+1.
__device__ __forceinline__ bool group_wait(uint64_t* bar, uint32_t parity, uint64_t* bar2, uint32_t parity2,
                                           const WaitCtx& ctx, unsigned int site, bool leader, uint32_t bar_id,
                                           uint32_t nthreads, volatile int* flags, uint32_t& count) {
  volatile int* flag = flags + (count & 1);
  ++count;
  if (leader) {
    bool ok = mbar_wait(bar, parity, ctx, site);
    if (ok && bar2 != nullptr) ok = mbar_wait(bar2, parity2, ctx, site);
    *flag = ok ? 1 : 0;
  }
  named_bar_sync(bar_id, nthreads);
  return *flag != 0;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------------------------------
// TMA (tiled tensor copies).  Loads signal an mbarrier with complete_tx; stores use bulk groups.
// Every load fills only the issuing CTA's shared memory (no cluster-wide broadcast form).
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                             int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------------------------------------------
// tcgen05 / TMEM
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {  // whole warp
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, fp16 inputs, fp32 accumulation; issued by one thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when every previously issued tcgen05.mma of this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ------------------------------------------------------------------------------------------
// CTA pairs: a thread-block cluster of two CTAs on two SMs whose tensor-core MMAs span both
// (tcgen05 .cta_group::2, M = 256: each CTA holds half of A's rows and half of B's rows in its own
// shared memory at the same offsets, and half of D's rows in its own TMEM).  The MMAs are issued
// by one thread of the even CTA; completion reaches both CTAs through a multicast commit.  Only
// mbarrier signals and the paired MMAs cross between the two CTAs: no TMA load here uses
// cluster multicast.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of both CTAs: release this CTA's prior writes, wait for the other CTA.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The shared::cluster address of shared-memory object `p`'s offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}

// Arrive on an mbarrier of either CTA (a shared::cluster address), releasing this thread's prior
// writes at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// The same arrive for a hand-off whose data is this CTA's shared memory or tensor memory only:
// a release fence restricted to shared::cta accesses at cluster scope, then a relaxed arrive.
// Used for operands written for the paired MMA (after fence.proxy.async.shared::cta and a
// __syncwarp, so the release covers the warp's writes) and for accumulator slots handed back to
// it (after tcgen05.wait::ld and tcgen05.fence::before_thread_sync).  Unlike a full cluster-scope
// release it does not wait for the thread's global-memory traffic: at c_z = 256 the pair kernels
// measured K1P -8 % and K3P -17 % at L = 2048 against mbarrier.arrive.release.cluster.
__device__ __forceinline__ void mbar_arrive_cluster_smem(uint32_t cluster_bar) {
  asm volatile("fence.release.sync_restrict::shared::cta.cluster;" ::: "memory");
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

__device__ __forceinline__ bool mbar_test_sleep_cl(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// mbar_wait for a barrier that the other CTA of the pair arrives on (cluster-scope acquire).
__device__ __forceinline__ bool mbar_wait_cl(uint64_t* bar, uint32_t parity, const WaitCtx& ctx, unsigned int site) {
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_test_sleep_cl(bar, parity, kSuspendHintNs)) return true;
    if (*ctx.abort) return false;
    if (globaltimer_ns() - t0 > ctx.timeout_ns) {
      raise_abort(ctx, site);
      return false;
    }
  }
}

// group_wait whose first barrier the other CTA of the pair completes (cluster-scope acquire).
__device__ __forceinline__ bool group_wait_cl(uint64_t* bar, uint32_t parity, uint64_t* bar2, uint32_t parity2,
                                              const WaitCtx& ctx, unsigned int site, bool leader, uint32_t bar_id,
                                              uint32_t nthreads, volatile int* flags, uint32_t& count) {
  volatile int* flag = flags + (count & 1);
  ++count;
  if (leader) {
    bool ok = mbar_wait_cl(bar, parity, ctx, site);
    if (ok && bar2 != nullptr) ok = mbar_wait(bar2, parity2, ctx, site);
    *flag = ok ? 1 : 0;
  }
  named_bar_sync(bar_id, nthreads);
  return *flag != 0;
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {  // same warp in both CTAs
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {  // same warp in both CTAs
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// The paired MMA (issued by one thread of the even CTA): D (+)= A * B^T with M = 256.
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The paired MMA with its A operand in tensor memory: rows [0, 128) of A in this CTA's TMEM lanes,
// rows [128, 256) in the peer's at the same address, K along columns (two fp16 per 32-bit
// column, the lower K index in the low half; a K = 16 step spans 8 columns).  B from shared
// memory by descriptor as for umma_f16_pair.
__device__ __forceinline__ void umma_f16_pair_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 columns of 32-bit into tensor memory: thread t of the warp writes row (lane base
// + t), columns [col, col + 32) from r[0..31].  The warp may only touch its own lane quadrant.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Wait for this thread's outstanding tcgen05.st.
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrive once on the mbarrier at `bar`'s offset in every CTA of `cta_mask` when the paired MMAs
// issued so far by this thread complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}


// 32 lanes x 32 columns of 32-bit: thread t of the warp gets row (lane base + t), columns
// [col, col+32) in r[0..31].  The warp may only touch its own 32-lane TMEM quadrant.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Wait for this thread's outstanding tcgen05.ld; the registers are tied to the wait so the
// compiler cannot consume them before it.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// 32 lanes x 16 columns of 32-bit.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld16x2(uint32_t (&r)[16], uint32_t (&s)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(s[0]), "+r"(s[1]), "+r"(s[2]), "+r"(s[3]), "+r"(s[4]), "+r"(s[5]), "+r"(s[6]),
                 "+r"(s[7]), "+r"(s[8]), "+r"(s[9]), "+r"(s[10]), "+r"(s[11]), "+r"(s[12]), "+r"(s[13]),
                 "+r"(s[14]), "+r"(s[15])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

// One thread of a warp waits (bounded) and the whole warp gets its verdict; the __syncwarp
// orders the other lanes' later reads after lane 0's acquiring wait.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const WaitCtx& ctx, unsigned int site) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, ctx, site) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

__device__ __forceinline__ void tmem_wait_ld2(uint32_t (&r)[32], uint32_t (&s)[32]) {
  tmem_wait_ld(r);
  asm volatile(""
               : "+r"(s[0]), "+r"(s[1]), "+r"(s[2]), "+r"(s[3]), "+r"(s[4]), "+r"(s[5]), "+r"(s[6]), "+r"(s[7]),
                 "+r"(s[8]), "+r"(s[9]), "+r"(s[10]), "+r"(s[11]), "+r"(s[12]), "+r"(s[13]), "+r"(s[14]),
                 "+r"(s[15]), "+r"(s[16]), "+r"(s[17]), "+r"(s[18]), "+r"(s[19]), "+r"(s[20]), "+r"(s[21]),
                 "+r"(s[22]), "+r"(s[23]), "+r"(s[24]), "+r"(s[25]), "+r"(s[26]), "+r"(s[27]), "+r"(s[28]),
                 "+r"(s[29]), "+r"(s[30]), "+r"(s[31])
               :
               : "memory");
}

// ------------------------------------------------------------------------------------------
// UMMA descriptors
// ------------------------------------------------------------------------------------------
// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm100 version bits = 1.
//   K-major operand: rows of 128 B (64 fp16 of K), 8-row groups `sbo` bytes apart; `lbo` unused.
//   MN-major operand: rows of 128 B (64 fp16 of M/N) per k, 8-k groups `sbo` bytes apart,
//                     64-wide M/N groups `lbo` bytes apart.
// The tile base must be 1024-byte aligned; K steps inside a swizzle atom move the start address.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// A descriptor advanced by `bytes` within its operand.  The start-address field holds bits
// [4, 18) of the shared-memory address and shared-memory addresses stay below 2^18, so adding
// bytes >> 4 never carries out of the field: an MMA loop builds each operand's descriptor once
// and adds constants (a single thread issues the MMAs, and fewer instructions per MMA let it
// issue them faster: 64 instead of 75 cycles per N = 128 MMA measured in isolation).
__device__ __forceinline__ uint64_t sdesc_add(uint64_t d, uint32_t bytes) { return d + (bytes >> 4); }

// Instruction descriptor for kind::f16: fp16 A and B, fp32 D, M x N, operand majorness.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                                  // D format: f32
         | (0u << 7) | (0u << 10)                   // A, B format: f16
         | ((a_mn_major ? 1u : 0u) << 15)           // A major
         | ((b_mn_major ? 1u : 0u) << 16)           // B major
         | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

// The same for bf16 A and B (kind::f16 takes both operands in one format: f16 or bf16).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn_major, bool b_mn_major) {
  return idesc_f16_f32(M, N, a_mn_major, b_mn_major) | (1u << 7) | (1u << 10);
}

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` in a 128B-swizzled tile whose
// rows are 128 bytes and whose base is 1024-byte aligned.
__device__ __forceinline__ uint32_t sw128_off(uint32_t row, uint32_t chunk) {
  return row * 128u + (((chunk ^ (row & 7u)) & 7u) << 4);
}

// ------------------------------------------------------------------------------------------
// small numerics
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Sigmoid in fp32: 1 / (1 + 2^(-x log2 e)) with the hardware base-2 exponential and reciprocal
// (both ~1 ulp of fp32, far below the fp16 rounding that follows).  Saturates cleanly:
// 2^(+big) = inf gives 0, 2^(-big) = 0 gives 1.
__device__ __forceinline__ float sigmoid_f32(float x) {
  return rcp_approx(1.0f + ex2_approx(x * -1.4426950408889634f));
}

__device__ __forceinline__ float2 sigmoid_f32x2(float2 x) {
  const float2 t = __fmul2_rn(x, make_float2(-1.4426950408889634f, -1.4426950408889634f));
  const float2 d = __fadd2_rn(make_float2(ex2_approx(t.x), ex2_approx(t.y)), make_float2(1.0f, 1.0f));
  return make_float2(rcp_approx(d.x), rcp_approx(d.y));
}

// Four 8x8 b16 matrices between shared memory and registers (lanes 8j..8j+7 give the row
// addresses of matrix j, 16 contiguous bytes each; register j holds matrix j).  Without .trans
// lane t holds row t/4, columns 2(t%4) and 2(t%4)+1 (the lower column in the low half); with
// .trans it holds column t/4, rows 2(t%4) and 2(t%4)+1.
__device__ __forceinline__ void ldsm_x4_trans(uint32_t saddr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(saddr)
               : "memory");
}

__device__ __forceinline__ void stsm_x4(uint32_t saddr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(saddr), "r"(r0), "r"(r1),
               "r"(r2), "r"(r3)
               : "memory");
}

// cvt(h) + c with one rounding (the fp16 -> fp32 conversion is exact): sm_100's mixed-precision
// add, which saves the separate conversion instruction.
__device__ __forceinline__ float add_f16_f32(unsigned short h, float c) {
  float d;
  asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(d) : "h"(h), "f"(c));
  return d;
}

__device__ __forceinline__ void split_half2(uint32_t u, unsigned short& lo, unsigned short& hi) {
  asm("mov.b32 {%0, %1}, %2;" : "=h"(lo), "=h"(hi) : "r"(u));
}

// Round a pair of fp32 values to fp16 and back (the value an fp16 tensor would hold).
__device__ __forceinline__ float2 round_f16x2(float2 v) { return __half22float2(__floats2half2_rn(v.x, v.y)); }

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float2 unpack_half2(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}

// ------------------------------------------------------------------------------------------
// LayerNorm of one 128-channel fp16 row held in a K-major 128B-swizzled tile (two 64-channel
// atoms `atom_bytes` apart): fp32 statistics, y = (x - mean) * rstd * gamma + beta rounded once
// to fp16 and written to the same row of `dst` (which may be `src`).
// Statistics take one pass over the row as sums of (x - k) and (x - k)^2 around k = the row's
// first value (shifted data keeps the cancellation in E[d^2] - E[d]^2 to O(eps * ((mean - k)/std)^2)
// of fp32); the normalising pass re-reads shared memory, so the row is never held in registers.
// `par(k, g, b)` returns gamma/beta for channels 8k..8k+7.
// ------------------------------------------------------------------------------------------
template <typename Par>
__device__ __forceinline__ void ln_row128_sw128(const uint8_t* src, uint8_t* dst, int atom_bytes, int row, float eps,
                                                Par par) {
  const float k = __half2float(*reinterpret_cast<const __half*>(src + sw128_off(row, 0)));
  float2 s1 = make_float2(0.f, 0.f), s2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int c16 = 0; c16 < 16; ++c16) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + (c16 >> 3) * atom_bytes + sw128_off(row, c16 & 7));
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      unsigned short lo, hi;
      split_half2(u[e], lo, hi);
      const float2 d = make_float2(add_f16_f32(lo, -k), add_f16_f32(hi, -k));
      s1 = __fadd2_rn(s1, d);
      s2 = __ffma2_rn(d, d, s2);
    }
  }
  const float m1 = (s1.x + s1.y) * (1.0f / 128);
  const float var = fmaxf((s2.x + s2.y) * (1.0f / 128) - m1 * m1, 0.0f);
  const float mean = k + m1;
  const float rstd = rsqrtf(var + eps);
  const float2 r2 = make_float2(rstd, rstd);
  asm volatile("" ::: "memory");
#pragma unroll
  for (int c16 = 0; c16 < 16; ++c16) {
    const int off = (c16 >> 3) * atom_bytes + sw128_off(row, c16 & 7);
    const uint4 v = *reinterpret_cast<const uint4*>(src + off);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    float g[8], b[8];
    par(c16, g, b);
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      unsigned short lo, hi;
      split_half2(u[e], lo, hi);
      const float2 d = __fmul2_rn(make_float2(add_f16_f32(lo, -mean), add_f16_f32(hi, -mean)), r2);
      const float2 y = __ffma2_rn(d, make_float2(g[2 * e], g[2 * e + 1]), make_float2(b[2 * e], b[2 * e + 1]));
      o[e] = pack_half2(y.x, y.y);
    }
    *reinterpret_cast<uint4*>(dst + off) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ------------------------------------------------------------------------------------------
// LayerNorm of a 256-channel row (four 128B-swizzled atoms of `atom_bytes` each), split over two
// threads: thread `half` owns channels [128 half, 128 half + 128) = atoms 2 half, 2 half + 1.
// Each computes the shifted partial sums of its half (shift k = the row's channel 0, read by
// both), the caller adds the two halves, and each normalises its own half in place or to dst.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ float ln_row_shift(const uint8_t* src, int row) {
  return __half2float(*reinterpret_cast<const __half*>(src + sw128_off(row, 0)));
}

__device__ __forceinline__ float2 ln_half_sums(const uint8_t* src, int atom_bytes, int row, int half, float k) {
  const uint8_t* base = src + 2 * half * atom_bytes;
  float2 s1 = make_float2(0.f, 0.f), s2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int c16 = 0; c16 < 16; ++c16) {
    const uint4 v = *reinterpret_cast<const uint4*>(base + (c16 >> 3) * atom_bytes + sw128_off(row, c16 & 7));
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      unsigned short lo, hi;
      split_half2(u[e], lo, hi);
      const float2 d = make_float2(add_f16_f32(lo, -k), add_f16_f32(hi, -k));
      s1 = __fadd2_rn(s1, d);
      s2 = __ffma2_rn(d, d, s2);
    }
  }
  return make_float2(s1.x + s1.y, s2.x + s2.y);
}

// mean and 1/sqrt(var + eps) of a 256-channel row from the two halves' shifted sums
__device__ __forceinline__ float2 ln256_moments(float2 a, float2 b, float k, float eps) {
  const float m1 = (a.x + b.x) * (1.0f / 256);
  const float var = fmaxf((a.y + b.y) * (1.0f / 256) - m1 * m1, 0.0f);
  return make_float2(k + m1, rsqrtf(var + eps));
}

template <typename Par>
__device__ __forceinline__ void ln_half_apply(const uint8_t* src, uint8_t* dst, int atom_bytes, int row, int half,
                                              float mean, float rstd, Par par) {
  const float2 r2 = make_float2(rstd, rstd);
#pragma unroll
  for (int c16 = 0; c16 < 16; ++c16) {
    const int off = (2 * half + (c16 >> 3)) * atom_bytes + sw128_off(row, c16 & 7);
    const uint4 v = *reinterpret_cast<const uint4*>(src + off);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    float g[8], b[8];
    par(16 * half + c16, g, b);
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      unsigned short lo, hi;
      split_half2(u[e], lo, hi);
      const float2 d = __fmul2_rn(make_float2(add_f16_f32(lo, -mean), add_f16_f32(hi, -mean)), r2);
      const float2 y = __ffma2_rn(d, make_float2(g[2 * e], g[2 * e + 1]), make_float2(b[2 * e], b[2 * e + 1]));
      o[e] = pack_half2(y.x, y.y);
    }
    *reinterpret_cast<uint4*>(dst + off) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// The same split four ways: thread `part` owns the single atom `part` (channels [64 part,
// 64 part + 64)) of a 256-channel row; the caller adds the four partial sums.
__device__ __forceinline__ float2 ln_atom_sums(const uint8_t* src, int atom_bytes, int row, int part, float k) {
  const uint8_t* base = src + part * atom_bytes;
  float2 s1 = make_float2(0.f, 0.f), s2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int c16 = 0; c16 < 8; ++c16) {
    const uint4 v = *reinterpret_cast<const uint4*>(base + sw128_off(row, c16));
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      unsigned short lo, hi;
      split_half2(u[e], lo, hi);
      const float2 d = make_float2(add_f16_f32(lo, -k), add_f16_f32(hi, -k));
      s1 = __fadd2_rn(s1, d);
      s2 = __ffma2_rn(d, d, s2);
    }
  }
  return make_float2(s1.x + s1.y, s2.x + s2.y);
}

template <typename Par>
__device__ __forceinline__ void ln_atom_apply(const uint8_t* src, uint8_t* dst, int atom_bytes, int row, int part,
                                              float mean, float rstd, Par par) {
  const float2 r2 = make_float2(rstd, rstd);
#pragma unroll
  for (int c16 = 0; c16 < 8; ++c16) {
    const int off = part * atom_bytes + sw128_off(row, c16);
    const uint4 v = *reinterpret_cast<const uint4*>(src + off);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    float g[8], b[8];
    par(8 * part + c16, g, b);
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      unsigned short lo, hi;
      split_half2(u[e], lo, hi);
      const float2 d = __fmul2_rn(make_float2(add_f16_f32(lo, -mean), add_f16_f32(hi, -mean)), r2);
      const float2 y = __ffma2_rn(d, make_float2(g[2 * e], g[2 * e + 1]), make_float2(b[2 * e], b[2 * e + 1]));
      o[e] = pack_half2(y.x, y.y);
    }
    *reinterpret_cast<uint4*>(dst + off) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// LayerNorm of a 128-channel row (two 128B-swizzled atoms) by a lane pair (lanes 2r, 2r+1 of a
// warp): lane parity `half` owns the 16-byte chunks of that parity in both atoms (channels
// 8c..8c+7 for c = half, half+2, ..); the partial sums meet through one shuffle.  Interleaving
// by chunk keeps the pair's two accesses in different banks of the same 128-byte row.
template <typename Par>
__device__ __forceinline__ void ln_row128_pair_sw128(const uint8_t* src, uint8_t* dst, int atom_bytes, int row,
                                                     int half, float eps, Par par) {
  const float k = __half2float(*reinterpret_cast<const __half*>(src + sw128_off(row, 0)));
  float2 s1 = make_float2(0.f, 0.f), s2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c16 = 2 * i + half;  // chunk index over both atoms
    const uint4 v = *reinterpret_cast<const uint4*>(src + (c16 >> 3) * atom_bytes + sw128_off(row, c16 & 7));
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      unsigned short lo, hi;
      split_half2(u[e], lo, hi);
      const float2 d = make_float2(add_f16_f32(lo, -k), add_f16_f32(hi, -k));
      s1 = __fadd2_rn(s1, d);
      s2 = __ffma2_rn(d, d, s2);
    }
  }
  float t1 = s1.x + s1.y, t2 = s2.x + s2.y;
  t1 += __shfl_xor_sync(0xffffffffu, t1, 1);
  t2 += __shfl_xor_sync(0xffffffffu, t2, 1);
  const float m1 = t1 * (1.0f / 128);
  const float var = fmaxf(t2 * (1.0f / 128) - m1 * m1, 0.0f);
  const float mean = k + m1;
  const float2 r2 = make_float2(rsqrtf(var + eps), rsqrtf(var + eps));
  asm volatile("" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c16 = 2 * i + half;
    const int off = (c16 >> 3) * atom_bytes + sw128_off(row, c16 & 7);
    const uint4 v = *reinterpret_cast<const uint4*>(src + off);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    float g[8], b[8];
    par(c16, g, b);
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      unsigned short lo, hi;
      split_half2(u[e], lo, hi);
      const float2 d = __fmul2_rn(make_float2(add_f16_f32(lo, -mean), add_f16_f32(hi, -mean)), r2);
      const float2 y = __ffma2_rn(d, make_float2(g[2 * e], g[2 * e + 1]), make_float2(b[2 * e], b[2 * e + 1]));
      o[e] = pack_half2(y.x, y.y);
    }
    *reinterpret_cast<uint4*>(dst + off) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// gamma/beta from fp16 arrays in shared memory
struct LnParSmemHalf {
  const __half* g;
  const __half* b;
  __device__ __forceinline__ void operator()(int k, float (&gg)[8], float (&bb)[8]) const {
    const uint4 gw = reinterpret_cast<const uint4*>(g)[k], bw = reinterpret_cast<const uint4*>(b)[k];
    const uint32_t gu[4] = {gw.x, gw.y, gw.z, gw.w}, bu[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = unpack_half2(gu[e]), y = unpack_half2(bu[e]);
      gg[2 * e] = x.x; gg[2 * e + 1] = x.y;
      bb[2 * e] = y.x; bb[2 * e + 1] = y.y;
    }
  }
};

// gamma/beta from fp32 arrays in shared memory
struct LnParSmem {
  const float* g;
  const float* b;
  __device__ __forceinline__ void operator()(int k, float (&gg)[8], float (&bb)[8]) const {
    const float4 g0 = reinterpret_cast<const float4*>(g)[2 * k], g1 = reinterpret_cast<const float4*>(g)[2 * k + 1];
    const float4 b0 = reinterpret_cast<const float4*>(b)[2 * k], b1 = reinterpret_cast<const float4*>(b)[2 * k + 1];
    gg[0] = g0.x; gg[1] = g0.y; gg[2] = g0.z; gg[3] = g0.w; gg[4] = g1.x; gg[5] = g1.y; gg[6] = g1.z; gg[7] = g1.w;
    bb[0] = b0.x; bb[1] = b0.y; bb[2] = b0.z; bb[3] = b0.w; bb[4] = b1.x; bb[5] = b1.y; bb[6] = b1.z; bb[7] = b1.w;
  }
};

// gamma/beta from fp16 arrays in global memory (L1-cached broadcast loads)
struct LnParHalf {
  const __half* g;
  const __half* b;
  __device__ __forceinline__ void operator()(int k, float (&gg)[8], float (&bb)[8]) const {
    const uint4 gw = __ldg(reinterpret_cast<const uint4*>(g) + k), bw = __ldg(reinterpret_cast<const uint4*>(b) + k);
    const uint32_t gu[4] = {gw.x, gw.y, gw.z, gw.w}, bu[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = unpack_half2(gu[e]), y = unpack_half2(bu[e]);
      gg[2 * e] = x.x; gg[2 * e + 1] = x.y;
      bb[2 * e] = y.x; bb[2 * e + 1] = y.y;
    }
  }
};

}  // namespace tmu
