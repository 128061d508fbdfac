// Device-side primitives for the sm_100a kernels of this library: mbarriers with bounded
// waits, TMA tile loads, tcgen05 (TMEM allocation, UMMA issue/commit, TMEM loads) and the
// shared-memory / instruction descriptors the UMMA instructions consume.
//
// Every spin on an mbarrier is bounded by a wall-clock limit read from %globaltimer. A wait
// that runs out records a status word in device memory (read by the host through
// b2_device_status) and raises a per-CTA abort flag, so every role of the CTA leaves its loop
// and the CTA still frees its TMEM and exits. Nothing here traps.
#pragma once

#include <cstdint>
#include <utility>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace b2 {

// ---------------------------------------------------------------------------------------------
// Status word shared by all kernels of the library (one per device; lives until process exit).
// Encoding: (kernel_id << 16) | (site << 8) | reason. 0 = no error since the last read.
// ---------------------------------------------------------------------------------------------
enum : uint32_t {
  kKernelLayerNorm = 1,
  kKernelGemm = 2,
  kKernelAttention = 3,
  kKernelPeerBarrier = 4,
};
enum : uint32_t {
  kReasonTimeout = 1,
  kReasonAbortSeen = 2,
};

// Defined once: the library is a single translation unit (b200tx.cu includes every kernel).
__device__ uint32_t g_device_status = 0;

__device__ __forceinline__ void record_status(uint32_t kernel_id, uint32_t site, uint32_t reason) {
  atomicCAS(&g_device_status, 0u, (kernel_id << 16) | (site << 8) | reason);
}

// Bounded polling loops (several barriers serviced by one thread) count idle spins and read the
// SM-local clock only every kPollCheckSpins idle spins; kPollTimeoutCycles ~ 4 s at 2 GHz.
constexpr uint32_t kPollCheckSpins = 256;
constexpr long long kPollTimeoutCycles = 8000000000ll;

struct PollTimeout {
  long long start;
  uint32_t idle;
  __device__ __forceinline__ void reset() {
    idle = 0;
    start = clock64();
  }
  // Call on an iteration that made no progress; true when the loop has been idle too long.
  // Sleeps briefly so the polling warp does not take issue slots from the compute warps that
  // share its SM sub-partition.
  __device__ __forceinline__ bool expired() {
    __nanosleep(32);
    if (++idle < kPollCheckSpins) return false;
    idle = 0;
    return clock64() - start > kPollTimeoutCycles;
  }
};

// Limit for one mbarrier wait. Legitimate waits in these kernels are microseconds long
// (the longest is an epilogue waiting for one full K loop); 4 s means the pipeline is stuck.
constexpr uint64_t kWaitTimeoutNs = 4000000000ull;

// The limit the kernels apply, settable from the host (b2_set_wait_limit) so that a test can make
// a wait run out in milliseconds instead of seconds; kWaitTimeoutNs unless set.
__device__ uint64_t g_wait_limit_ns = kWaitTimeoutNs;
__device__ __forceinline__ uint64_t wait_limit_ns() { return *reinterpret_cast<volatile uint64_t*>(&g_wait_limit_ns); }

// Test-only fault selector (b2_test_set_fault): 0 = none; kFaultGemmWithholdStage = the GEMM
// producer of CTA 0 neither arms nor loads its first pipeline stage, so the MMA warp's wait for
// that stage runs out (bounded, status word, abort) the way a lost TMA arrival would.
constexpr uint32_t kFaultGemmWithholdStage = 1;
__device__ uint32_t g_test_fault = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait with cluster-scope acquire: for barriers that threads of another CTA of the cluster
// arrive on (their prior memory operations become visible to this thread).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Non-blocking probe with cluster-scope acquire (barriers that other CTAs of the cluster arrive on).
__device__ __forceinline__ bool mbar_test_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Non-blocking probe of the same condition (mbarrier.test_wait never suspends the thread, unlike
// try_wait, which may sleep for a hardware time slice when the phase is incomplete). For loops that
// poll several barriers and must react to whichever completes first.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits until the phase of `bar` with parity `parity` has completed. Returns false (after
// recording a status word and raising *abort) when the wait exceeds wait_limit_ns(), and false
// without recording when another role of the CTA already raised *abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint32_t kernel_id, uint32_t site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > wait_limit_ns()) {
        record_status(kernel_id, site, kReasonTimeout);
        *abort = 1;
        return false;
      }
    }
  }
}

// mbar_wait for a barrier arrived on from other CTAs of the cluster (cluster-scope acquire).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                  uint32_t kernel_id, uint32_t site) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((++spins & 63u) == 0) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > wait_limit_ns()) {
        record_status(kernel_id, site, kReasonTimeout);
        *abort = 1;
        return false;
      }
    }
  }
}

// Named barrier over `nthreads` threads (a multiple of 32) with id `id` (1..15; 0 is
// __syncthreads). The non-.aligned form, so lanes may arrive from divergent paths.
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Arrives on named barrier `id` (expected count `nthreads`) without waiting; pairs with
// named_barrier_sync calls of other warps that complete the count.
__device__ __forceinline__ void named_barrier_arrive(uint32_t id, uint32_t nthreads) {
  asm volatile("barrier.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------------------------
// TMA (no multicast anywhere in this library: every CTA loads its own tiles from local HBM).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of one box at element coordinates (x = inner, y = outer). x * elem_size must be
// a multiple of 16 bytes; callers only pass multiples of 64 bf16 elements.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 2-D tiled load for a CTA pair running 2-SM UMMA: the box lands in this CTA's shared memory and
// the transaction bytes are counted on `leader_bar`, a barrier in the pair's leader CTA (a
// shared::cluster address from cluster_map_to_rank). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t leader_bar,
                                                 int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}

// ---------------------------------------------------------------------------------------------
// Thread-block clusters
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map_to_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// All threads of all CTAs of the cluster (release/acquire).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Asynchronous 2 x 32-bit store into (possibly another CTA's) shared memory that counts its 8 bytes
// on that CTA's mbarrier `cluster_bar` (complete_tx): the data is visible to whoever observes the
// barrier's phase complete, with no fence on the sending side.
__device__ __forceinline__ void st_async_v2f32(uint32_t cluster_addr, float a, float b, uint32_t cluster_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(cluster_addr),
               "f"(a), "f"(b), "r"(cluster_bar)
               : "memory");
}
// mbarrier arrive on a barrier given by a shared::cluster address (possibly another CTA's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// ---------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads
// ---------------------------------------------------------------------------------------------
// Whole warp. Writes the TMEM base address to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  __syncwarp();
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  __syncwarp();
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  __syncwarp();
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Pair-wide TMEM allocation for 2-SM UMMA: warp `w` of both CTAs of the pair execute it, same slot.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
  __syncwarp();
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  __syncwarp();
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  __syncwarp();
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Per-thread register budget of the executing warpgroup (all 4 warps execute it). The budgets of
// all warpgroups must add up to at most the block's launch allocation.
template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, fp32 accumulate. Single thread.
__device__ __forceinline__ void umma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D (+)= A * B^T with A read from tensor memory (128 lanes = M rows; K packed two bf16 per 32-bit
// column, so a K = 16 step spans 8 columns) and B from shared memory.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 2-SM UMMA issued by the pair's leader: D (M=256 across both CTAs' TMEM) (+)= A * B^T, where each
// CTA supplies half of A's rows and half of B's rows from its own shared memory at the addresses
// the descriptors give.
__device__ __forceinline__ void umma_bf16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the barrier at the same offset in each CTA of `cta_mask` when every 2-SM UMMA
// issued so far by this thread is done.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 async operation issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Loads 32 consecutive fp32 columns of this thread's TMEM lane (32x32b shape: lane i of the warp
// reads lane (taddr.lane + i)) and waits for completion inside the same asm statement, so no use
// of the result can be scheduled before the wait.
//
// tcgen05.ld is .sync.aligned: the whole warp must execute it converged. Lanes leave the bounded
// mbarrier spin independently, so the warp is re-converged here first.
__device__ __forceinline__ void tmem_load_32cols(uint32_t taddr, float* v) {
  uint32_t r[32];
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// The two halves of tmem_load_32cols, so that the next chunk's load is in flight while the
// current one is processed: tmem_ld32_issue starts the load (the registers are not valid yet) and
// tmem_ld32_wait waits for every tcgen05.ld this thread has issued. The wait takes the registers
// as in-out operands, so no use of them can be scheduled before it.
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]) : : "memory");
}

// 64 consecutive fp32 columns of this thread's TMEM lane in one instruction (then wait).
__device__ __forceinline__ void tmem_load_64cols(uint32_t taddr, float* v) {
  uint32_t r[64];
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// 128 consecutive fp32 columns of this thread's TMEM lane in one instruction (then wait).
__device__ __forceinline__ void tmem_load_128cols(uint32_t taddr, float* v) {
  uint32_t r[128];
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,"
      "%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,"
      "%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,"
      "%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,"
      "%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]),
        "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]),
        "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]),
        "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]),
        "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]),
        "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]),
        "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]),
        "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]),
        "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]),
        "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
}

// Stores 32 fp32 values into 32 consecutive columns of this thread's TMEM lane and waits for the
// store to complete (tcgen05.st is .sync.aligned like tcgen05.ld).
// 16 columns of this warp's 32 TMEM lanes; completion is awaited separately (tmem_wait_st).
__device__ __forceinline__ void tmem_store_16cols_async(uint32_t taddr, const uint32_t* w) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(taddr),
      "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7]), "r"(w[8]),
      "r"(w[9]), "r"(w[10]), "r"(w[11]), "r"(w[12]), "r"(w[13]), "r"(w[14]), "r"(w[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 columns of this warp's 32 TMEM lanes without waiting (tmem_wait_st before reading them back).
__device__ __forceinline__ void tmem_store_32cols_async(uint32_t taddr, const float (&v)[32]) {
  __syncwarp();
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_store_32cols(uint32_t taddr, const float* v) {
  __syncwarp();
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;\n" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

// ---------------------------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------------------------
// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D (PTX ISA "Instruction descriptor"
// table for .kind::f16): c_format bits [4,6) = 1 (F32), a_format [7,10) = 1 (BF16),
// b_format [10,13) = 1 (BF16), a_major bit 15, b_major bit 16 (0 = K-major, 1 = MN-major),
// N>>3 at bits [17,23), M>>4 at bits [24,29).
__host__ __device__ constexpr uint32_t make_idesc_bf16_f32(uint32_t M, uint32_t N, uint32_t a_mn_major,
                                                          uint32_t b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (a_mn_major << 15) | (b_mn_major << 16) | ((N >> 3) << 17) |
         ((M >> 4) << 24);
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand (PTX ISA "Shared memory
// descriptor"): start address >> 4 in bits [0,14), leading byte offset >> 4 in [16,30), stride
// byte offset >> 4 in [32,46), the fixed version field 1 at bit 46, layout type 2 (SWIZZLE_128B)
// in bits [61,64). Base offset 0: every operand tile starts on a 1024-byte boundary.
//   K-major:  rows of 128 B (64 bf16 along K); SBO = byte distance between 8-row groups; LBO unused.
//   MN-major: rows of 128 B (64 bf16 along M/N) per K index; SBO = distance between 8-K groups,
//             LBO = distance between 64-wide M/N blocks.
__device__ __forceinline__ uint64_t make_sdesc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// ---------------------------------------------------------------------------------------------
// Programmatic dependent launch. Every kernel of the library is launched with programmatic
// stream serialization: it may start while the previous kernel on the stream is finishing, does
// its prologue (barrier init, TMEM allocation, descriptor prefetch: nothing that touches global
// data), then waits for the previous grid to complete and its memory to be visible before reading
// its inputs or writing its outputs, and at once allows the next kernel to launch. Without a
// programmatic predecessor the wait returns immediately.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait_previous_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_allow_next_grid() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------
// Cross-GPU memory operations (tensor parallel): system-scope ordering and atomics on memory that
// may belong to a peer GPU (mapped over NVLink).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
// fp32 atomic add of 4 values, system scope (the address may be a peer GPU's memory).
__device__ __forceinline__ void red_add_v4_sys(float* p, float a, float b, float c, float d) {
  asm volatile("red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// ---------------------------------------------------------------------------------------------
// Small numeric helpers
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float fast_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fast_exp2(float x);

// Exact (erf-based) GELU, the form torch.nn.functional.gelu(approximate="none") computes:
// 0.5 x (1 + erf(x / sqrt 2)). erf is evaluated with the rational formula 7.1.28 of Abramowitz &
// Stegun, Handbook of Mathematical Functions (after Hastings):
//   erf(z) = 1 - (1 + a1 z + a2 z^2 + a3 z^3 + a4 z^4 + a5 z^5 + a6 z^6)^-16,  z >= 0,
// whose absolute error is at most 3e-7 (the approximate reciprocal adds a few ulp of the
// 16th power), far below the bf16 rounding the result goes through; odd symmetry gives z < 0.
// One reciprocal and no exponential: the epilogue of the GELU GEMM issues half the
// special-function instructions of the rational-exponential form 7.1.26 and runs about 6% faster.
constexpr float kErfA1 = 0.0705230784f, kErfA2 = 0.0422820123f, kErfA3 = 0.0092705272f,
                kErfA4 = 0.0001520143f, kErfA5 = 0.0002765672f, kErfA6 = 0.0000430638f;

__device__ __forceinline__ float gelu_erf(float x) {
  const float z = fabsf(x) * 0.70710678118654752440f;
  float q = fmaf(z, kErfA6, kErfA5);
  q = fmaf(z, q, kErfA4);
  q = fmaf(z, q, kErfA3);
  q = fmaf(z, q, kErfA2);
  q = fmaf(z, q, kErfA1);
  q = fmaf(z, q, 1.0f);
  float r = fast_rcp(q);  // q >= 1; q = inf for huge |x| gives r = 0
  r *= r;
  r *= r;
  r *= r;
  r *= r;
  const float erf_abs = 1.0f - r;
  return 0.5f * x * (1.0f + copysignf(erf_abs, x));
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// a = a * m + d and b = b * m + d with one packed fp32x2 FMA (sm_100).
__device__ __forceinline__ void fma2_inplace(float& a, float& b, uint64_t m2, uint64_t d2) {
  uint64_t x;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
  asm("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(x) : "l"(m2), "l"(d2));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x));
}

__device__ __forceinline__ uint64_t splat2(float v) {
  uint64_t x;
  asm("mov.b64 %0, {%1, %1};" : "=l"(x) : "f"(v));
  return x;
}

__device__ __forceinline__ uint64_t pack2f(float a, float b) {
  uint64_t x;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
  return x;
}
__device__ __forceinline__ void unpack2f(uint64_t x, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x));
}
__device__ __forceinline__ uint64_t mul2f(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t add2f(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2f(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// gelu_erf of two values with packed fp32x2 multiplies and FMAs (one instruction for both values):
// the same Abramowitz & Stegun 7.1.28 evaluation, with erf(|z|) = fma(-r, 1, 1) on the packed
// pair and the final 0.5 x (1 + sign(x) erf(|z|)) as fma(0.5 x, s, 0.5 x) (one rounding fewer than
// the scalar form; both sit far below the bf16 rounding that follows).
__device__ __forceinline__ void gelu_erf2(float& a, float& b) {
  const uint64_t z = mul2f(pack2f(fabsf(a), fabsf(b)), splat2(0.70710678118654752440f));
  uint64_t q = fma2f(z, splat2(kErfA6), splat2(kErfA5));
  q = fma2f(z, q, splat2(kErfA4));
  q = fma2f(z, q, splat2(kErfA3));
  q = fma2f(z, q, splat2(kErfA2));
  q = fma2f(z, q, splat2(kErfA1));
  q = fma2f(z, q, splat2(1.0f));
  float q0, q1;
  unpack2f(q, q0, q1);
  uint64_t r = pack2f(fast_rcp(q0), fast_rcp(q1));
  r = mul2f(r, r);
  r = mul2f(r, r);
  r = mul2f(r, r);
  r = mul2f(r, r);
  float e0, e1;
  unpack2f(fma2f(r, splat2(-1.0f), splat2(1.0f)), e0, e1);
  const uint64_t h = mul2f(pack2f(a, b), splat2(0.5f));
  unpack2f(fma2f(h, pack2f(copysignf(e0, a), copysignf(e1, b)), h), a, b);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for two values on the FMA pipe instead of the exponential unit (MUFU, 16/clk/SM, which
// is what bounds a head_dim-64 softmax). Range reduction: n = rint(x) by the 1.5 * 2^23
// round-to-integer addition, f = x - n in [-1/2, 1/2] (both exact); 2^f by a cubic whose
// coefficients were fitted for minimax relative error over that interval (iteratively
// reweighted least squares): max relative error 7.5e-5, against bf16's half-ulp of 2^-9. The
// exponent n is added to the cubic's exponent field with one integer multiply-add (the low 9
// bits of the rounded float hold n). x is clamped below at -126 so the field cannot wrap
// (-inf gives a denormal-or-zero result, never NaN); x above 127 is outside the contract.
__device__ __forceinline__ void exp2_poly_x2(float x0, float x1, float& e0, float& e1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  x0 = fmaxf(x0, -126.0f);
  x1 = fmaxf(x1, -126.0f);
  uint64_t x, t, r, f, p;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(x0), "f"(x1));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(t) : "l"(x), "l"(splat2(kRound)));
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(t), "l"(splat2(kRound)));
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(f) : "l"(x), "l"(r));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(p) : "l"(f), "l"(splat2(0.05517132f)), "l"(splat2(0.24261054f)));
  asm("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(p) : "l"(f), "l"(splat2(0.69326099f)));
  asm("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(p) : "l"(f), "l"(splat2(0.99992811f)));
  float p0, p1, t0, t1;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(p0), "=f"(p1) : "l"(p));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(t0), "=f"(t1) : "l"(t));
  e0 = __int_as_float(__float_as_int(t0) * (1 << 23) + __float_as_int(p0));
  e1 = __int_as_float(__float_as_int(t1) * (1 << 23) + __float_as_int(p1));
}

}  // namespace b2

namespace b2 {

// Launches `kernel` with programmatic stream serialization (see pdl_wait_previous_grid).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

}  // namespace b2
