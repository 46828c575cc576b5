// All-gather form of the weight-only GEMM kernels (qtts_w8a16_gemm_allgather):
// the GEMM's output block goes straight into every rank's gathered buffer over
// peer memory, with two flag phases per call instead of a separate collective.
//
// Per rank: a signal pad uint32[2 * world] (slot q of [0, world): rank q is
// ready to receive call e; slot q of [world, 2 * world): rank q's stores of
// call e are complete), and sync uint32[2] (CTA arrivals of the running call,
// epoch of the last completed call). Calls are numbered on the device (epoch =
// last + 1), so CUDA-graph replays advance them; signal values only grow, so
// nothing is ever reset between calls.
//
//  1. After the dependency wait (so this rank's previous readers of its
//     gathered buffer have finished), thread 0 of every CTA writes ready = e
//     into every rank's pad (the same value from each CTA, so no CTA's wait
//     depends on another CTA of its own grid having started).
//  2. Every CTA, before its first output store, waits until every rank is
//     ready for e; it then stores each output element into every rank's
//     buffer (plain peer stores over NVLink, no multicast).
//  3. After a CTA barrier, thread 0 of each CTA counts the CTA in with a
//     GPU-scope acquire-release atomic; the last CTA fences at system scope,
//     re-arms the count, records e as completed, writes done = e into every
//     rank's pad (release) and waits until every rank is done.
//     The grid completes only then, so whatever follows on the stream sees
//     the whole gathered output.
// Every wait is bounded by the kernel's wait limit; on expiry the kernel
// records QTTS_ERR_TIMEOUT and goes on (a lost rank cannot hang the GPU).
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace qtts {

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// The peer tables are constant for the lifetime of a call site: pull them into
// L1 at kernel start so the epilogue's loads of them hit.
__device__ __forceinline__ void ag_prefetch_tables(const SkinnyArgs& a) {
  for (int p = 0; p < a.world; p += 8) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(a.peer_out + p));
    asm volatile("prefetch.global.L1 [%0];" ::"l"(a.peer_sig + p));
  }
}

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Epoch of the running call. Read after the dependency wait: the previous
// call's last CTA wrote its epoch before that grid completed.
__device__ __forceinline__ uint32_t ag_epoch(const SkinnyArgs& a) {
  return *reinterpret_cast<const volatile uint32_t*>(a.sync + 1) + 1u;
}

// Phase 1: this rank can receive call `epoch` (thread 0 of each CTA). A
// relaxed store: it publishes no data of this rank, and the previous readers
// of the gathered buffer finished before the dependency wait returned.
__device__ __forceinline__ void ag_announce_ready(const SkinnyArgs& a, uint32_t epoch) {
  for (int p = 0; p < a.world; ++p) st_relaxed_sys(a.peer_sig[p] + a.rank, epoch);
}

// Bounded wait until slots [base, base + world) of this rank's pad all hold
// `epoch` or later.
__device__ __forceinline__ bool ag_wait_all(const SkinnyArgs& a, int base, uint32_t epoch) {
  const uint32_t* mine = a.peer_sig[a.rank] + base;
  const uint64_t t0 = globaltimer_ns();
  for (int q = 0; q < a.world; ++q) {
    while (static_cast<int32_t>(ld_acquire_sys(mine + q) - epoch) < 0) {
      if (globaltimer_ns() - t0 > a.wait_ns) return false;
      __nanosleep(64);
    }
  }
  return true;
}

// Phase 2 gate, called by every thread of a group of `nthreads` (named
// barrier `bar_id`) before its first output store: thread `leader` waits for
// every rank's ready flag. Returns false if the wait expired (the stores are
// then skipped).
__device__ __forceinline__ bool ag_gate_stores(const SkinnyArgs& a, uint32_t epoch, int* flag_smem, int bar_id,
                                               int nthreads, bool leader) {
  if (leader) {
    const bool ok = ag_wait_all(a, 0, epoch);
    if (!ok) record_status(QTTS_ERR_TIMEOUT);
    *reinterpret_cast<volatile int*>(flag_smem) = ok ? 1 : 0;
  }
  named_bar_sync(bar_id, nthreads);
  return *reinterpret_cast<volatile int*>(flag_smem) != 0;
}

// One output element: into the local output, or in the all-gather form (AG,
// a template parameter of the kernels so the plain form carries none of it)
// into every rank's gathered buffer (`pbase` + `off` elements from its base).
template <bool AG, typename XT>
__device__ __forceinline__ void put_out(const SkinnyArgs& a, XT* og, int64_t pbase, int64_t off, XT v) {
  if (!AG) {
    og[off] = v;
    return;
  }
  for (int p = 0; p < a.world; ++p) static_cast<XT*>(a.peer_out[p])[pbase + off] = v;
}

// Phase 3, called by every thread of the CTA at the very end of the kernel.
// `epoch` is only read in thread 0, which must have passed the dependency wait.
// Ordering chain: every thread's output stores -> CTA barrier -> thread 0's
// GPU-scope release (the arrival) -> the last arrival's acquire -> its
// system-scope fence, then the `done` stores -> the peer's system-scope acquire.
// One system-scope fence per call; the arrivals stay inside the GPU.
__device__ __forceinline__ void ag_finish(const SkinnyArgs& a, uint32_t epoch) {
  __syncthreads();
  if (threadIdx.x != 0) return;
  const unsigned total = gridDim.x * gridDim.y * gridDim.z;
  if (atom_add_acq_rel_gpu(a.sync, 1u) + 1u != total) return;
  // The last CTA of this rank: the count is re-armed for the next call, which
  // counts only after its dependency wait (this grid has completed by then).
  *reinterpret_cast<volatile uint32_t*>(a.sync) = 0u;
  *reinterpret_cast<volatile uint32_t*>(a.sync + 1) = epoch;
  fence_acq_rel_sys();  // one fence releases every rank's `done` below
  for (int p = 0; p < a.world; ++p) st_relaxed_sys(a.peer_sig[p] + a.world + a.rank, epoch);
  if (!ag_wait_all(a, a.world, epoch)) record_status(QTTS_ERR_TIMEOUT);
}

}  // namespace qtts
