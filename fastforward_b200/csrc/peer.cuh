// Cross-GPU handshakes over peer-mapped memory (NVLink / NVSwitch), for the kernels that
// read the tensor-parallel ranks' partial results directly instead of after an NCCL
// collective.  Plain loads, stores and atomics on peer memory only (no multicast).
#pragma once
#include "common.cuh"

// Slot `slot` of every rank: rank `rank` adds 1 to flags[p][rank][slot] on every rank p,
// then waits until its own flags[rank][q][slot] has reached the number of its own calls for
// this slot, for every rank q.  Every rank makes the same sequence of calls per slot, so the
// counts advance in lockstep and need no reset.  Release pattern: an acq_rel fence at system
// scope, then relaxed adds; acquire pattern: relaxed polling, then the same fence.  One thread per
// CTA calls it, after the CTA's writes to publish (ordered before it by a CTA barrier);
// false when the bounded wait (2 s) gave up.
__device__ __forceinline__ void red_relaxed_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ bool peer_handshake(const ffb_peer_sync& s, int slot) {
  const uint32_t n = s.local[slot] + 1u;  // only this CTA's one thread touches its slot
  s.local[slot] = n;
  fence_acq_rel_sys();
  for (int p = 0; p < s.world; ++p) red_relaxed_sys_add(s.flags[p] + (size_t)s.rank * s.nslots + slot, 1u);
  const uint64_t t0 = global_timer_ns();
  bool ok = true;
  for (int q = 0; q < s.world && ok; ++q) {
    const uint32_t* f = s.flags[s.rank] + (size_t)q * s.nslots + slot;
    uint32_t polls = 0;
    while ((int)(ld_relaxed_sys_u32(f) - n) < 0) {
      if ((++polls & 255u) == 0 && global_timer_ns() - t0 > 2000000000ull) {
        ok = false;
        break;
      }
    }
  }
  fence_acq_rel_sys();
  return ok;
}
