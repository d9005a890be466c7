// Peer-memory (NVLink / NVSwitch) building blocks for kernels that do their own
// communication: system-scope release/acquire on 64-bit flags that live in a
// symmetric heap (same layout on every rank, peers mapped through CUDA IPC),
// bounded flag waits, and the proxy fence that lets TMA (async proxy) read data
// that peers wrote with ordinary stores.
//
// Protocol used by every fused op: flags are monotonic counters.  Call number
// e (an epoch, identical on all ranks because every rank issues the same ops
// in the same order) waits for `counter >= e * per_epoch_increments`, so no
// flag is ever reset and no reset can race with a fast peer's next call.
// Buffers are double-buffered by epoch parity; a writer for epoch e first
// waits until the reader has finished epoch e-2 on that parity.
//
// No cluster fan-out loads anywhere: remote bytes cross NVLink through st.global from
// the producing GPU into the consumer's memory, and the consumer's TMA reads
// only its own memory.
#pragma once
#include "p2p_args.h"
#include "ptx.cuh"

namespace b200 {

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_sys_add(uint64_t* p, uint64_t v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Order this thread's earlier generic-proxy global accesses before later
// async-proxy (TMA) accesses to global memory.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait until *flag >= target.  Returns false after recording `code`
// (and raising *abort_flag) when the budget runs out or an abort was raised.
__device__ __forceinline__ bool wait_flag_ge(const uint64_t* flag, uint64_t target, int* err, int code,
                                             volatile int* abort_flag = nullptr,
                                             uint64_t budget_ns = kWaitBudgetNs) {
  if (ld_acquire_sys(flag) >= target) return true;
  const uint64_t start = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    __nanosleep(64);
    if (ld_acquire_sys(flag) >= target) return true;
    if ((++spins & 15u) == 0) {
      if (abort_flag && *abort_flag) return false;
      if (globaltimer_ns() - start > budget_ns) {
        record_error(err, code);
        if (abort_flag) *abort_flag = 1;
        return false;
      }
    }
  }
}

// Number, parity and flag targets of the running call: from the kernel
// arguments (host-counted mode) or from the device op-state block.
struct P2PCall {
  int parity;
  uint64_t arrive_target;
  uint64_t reuse_target;
};

__device__ __forceinline__ P2PCall p2p_call(const P2PArgs& p) {
  if (p.epoch == nullptr) return P2PCall{p.parity, p.arrive_target, p.reuse_target};
  const uint64_t calls = __ldcg(p.epoch + kEpochCalls) + 1;
  P2PCall c;
  c.parity = int(calls & 1u);
  c.arrive_target = __ldcg(p.epoch + kEpochArrive) + p.arrive_inc;
  c.reuse_target = calls >= 3 ? __ldcg(p.epoch + kEpochDone + (calls - 2) % 4) : 0ull;
  return c;
}

// Thread 0 of every CTA of the call's last kernel, after the CTA's work: the
// last CTA to get here advances the op state (every CTA has read it by then).
__device__ __forceinline__ void p2p_epoch_finish(const P2PArgs& p) {
  if (p.epoch == nullptr) return;
  __threadfence();
  const unsigned long long n = gridDim.x * gridDim.y * gridDim.z;
  const unsigned long long prev =
      atomicAdd(reinterpret_cast<unsigned long long*>(p.epoch + kEpochFinish), 1ull);
  if (prev + 1 != n) return;
  __threadfence();
  volatile uint64_t* e = p.epoch;
  const uint64_t calls = e[kEpochCalls] + 1;
  e[kEpochDone + calls % 4] = e[kEpochDone + (calls - 1) % 4] + p.done_inc;
  e[kEpochArrive] = e[kEpochArrive] + p.arrive_inc;
  e[kEpochCalls] = calls;
  e[kEpochFinish] = 0;
  __threadfence();
}

}  // namespace b200
