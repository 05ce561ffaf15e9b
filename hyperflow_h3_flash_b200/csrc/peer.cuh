// Cross-GPU ordering for the fused Ulysses exchange.
//
// Each rank owns a small array of 32-bit flags per phase, one slot per source rank, in memory the other ranks have
// mapped (CUDA IPC).  A phase of step e is "rank i has finished writing (or reading) what the others wait for":
// rank i stores e into slot i of every rank's flags with a release at system scope, after its producing kernels
// (stream order puts them before the store).  A waiting rank spins on its own flags with acquire loads until every
// slot has reached e; the kernels queued after the wait then see the peers' data.
//
// Epochs only grow, and a slot is compared as (int32)(flag - e) >= 0, so a flag that is already past e (the peer is
// a step ahead) passes, and 2^31 steps wrap safely.  Every wait is bounded: past the time limit the kernel records
// CONVROT_ERR_TIMEOUT in the device error word and returns, and the stream carries on (the host sees the status on
// its next poll); nothing spins forever and nothing traps.
//
// These kernels wait on other GPUs only: the ranks of one exchange are always distinct devices.

#pragma once

#include <stdint.h>

#include "ptx.cuh"

namespace convrot {

struct PeerSlots {
  uint32_t* slot[kMaxChunks];  // flag this rank writes in rank j's array (its own slot there)
};

// One thread per rank: release-store the epoch into that rank's slot for this sender.
__global__ void peer_signal_kernel(const PeerSlots slots, int n, uint32_t epoch) {
  const int j = threadIdx.x;
  if (j < n) st_release_sys(select_chunk(slots.slot, j), epoch);
}

// One thread per source rank: acquire-load its slot until it reaches the epoch, or give up at the time limit.
__global__ void peer_wait_kernel(const uint32_t* flags, int n, uint32_t epoch, uint64_t limit_ns, int* error_word) {
  const int j = threadIdx.x;
  if (j >= n) return;
  const uint64_t start = globaltimer_ns();
  while (static_cast<int32_t>(ld_acquire_sys(flags + j) - epoch) < 0) {
    if (globaltimer_ns() - start > limit_ns) {
      if (error_word) atomicCAS(error_word, 0, 6 /* CONVROT_ERR_TIMEOUT */);
      return;
    }
    __nanosleep(200);
  }
}

}  // namespace convrot
