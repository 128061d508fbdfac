// Cross-GPU barrier over peer memory (NVLink P2P), for the tensor-parallel path whose
// reduce-scatter is fused into the GEMM epilogues (kEpiRs*) and whose all-gather is fused into the
// LayerNorm: ranks add their partial rows into the row owners' residuals and store LayerNorm rows
// into every rank's buffer, so they must agree on "every add into my rows has landed" (before the
// owner's LayerNorm reads them) and "every rank's LayerNorm rows have landed" (before the next
// GEMM reads them).
//
// Each rank owns a pad of kPadChannels x kMaxPeers uint32 flags in memory every peer can map.
// Slot [channel][src] of rank d's pad is written only by rank src and cleared only by rank d:
//   signal: CAS 0 -> 1 (release, system scope) on the destination's slot for this rank;
//   wait:   CAS 1 -> 0 (acquire, system scope) on this rank's slot for each source.
// The flags reset themselves, so the barrier needs no epoch and replays unchanged inside a CUDA
// graph. A signal that finds its slot still set waits until the peer has consumed the previous
// one. Both waits are bounded (wait_limit_ns()): on expiry the kernel records a status and returns.
#pragma once

#include "b2_common.cuh"

namespace b2 {

constexpr int kMaxPeers = 8;
constexpr int kPadChannels = 4;

struct PeerPads {
  uint32_t* pad[kMaxPeers];
};

__device__ __forceinline__ uint32_t atom_cas_release_sys(uint32_t* p, uint32_t cmp, uint32_t val) {
  uint32_t old;
  asm volatile("atom.release.sys.global.cas.b32 %0, [%1], %2, %3;" : "=r"(old) : "l"(p), "r"(cmp), "r"(val) : "memory");
  return old;
}
__device__ __forceinline__ uint32_t atom_cas_acquire_sys(uint32_t* p, uint32_t cmp, uint32_t val) {
  uint32_t old;
  asm volatile("atom.acquire.sys.global.cas.b32 %0, [%1], %2, %3;" : "=r"(old) : "l"(p), "r"(cmp), "r"(val) : "memory");
  return old;
}
__device__ __forceinline__ void fence_sc_sys() { asm volatile("fence.sc.sys;" ::: "memory"); }

// One block of kMaxPeers threads; thread r exchanges the flag pair with peer r.
__global__ void __launch_bounds__(kMaxPeers, 1) peer_barrier_kernel(PeerPads pads, int world, int rank, int channel) {
  pdl_wait_previous_grid();
  const int r = threadIdx.x;
  if (r < world && r != rank) {
    uint32_t* to_peer = pads.pad[r] + channel * kMaxPeers + rank;
    uint32_t* from_peer = pads.pad[rank] + channel * kMaxPeers + r;
    fence_sc_sys();  // this GPU's earlier writes (previous kernels, peer adds and stores) before the flag
    const uint64_t t0 = global_timer_ns();
    bool ok = true;
    while (atom_cas_release_sys(to_peer, 0u, 1u) != 0u) {
      if (global_timer_ns() - t0 > wait_limit_ns()) {
        record_status(kKernelPeerBarrier, 0, kReasonTimeout);
        ok = false;
        break;
      }
      __nanosleep(64);
    }
    if (ok) {
      while (atom_cas_acquire_sys(from_peer, 1u, 0u) != 1u) {
        if (global_timer_ns() - t0 > wait_limit_ns()) {
          record_status(kKernelPeerBarrier, 1, kReasonTimeout);
          break;
        }
        __nanosleep(64);
      }
    }
    fence_sc_sys();
  }
  __syncthreads();
}

static cudaError_t launch_peer_barrier(const PeerPads& pads, int world, int rank, int channel, cudaStream_t stream) {
  return launch_pdl(peer_barrier_kernel, dim3(1), dim3(kMaxPeers), 0, stream, pads, world, rank, channel);
}

}  // namespace b2
