// Device primitives shared by every sm_100a kernel of the runtime.
//
// The flag contract follows the reference (src/tile.cuh:15-30): the yield
// flag is a generation counter that publishes ONLY its value (claims go
// through atomics, timestamps are read by the host after the kernel ends),
// so loads and stores are relaxed.  Here the scope is .sys rather than
// .gpu because the flag may live in mapped pinned host memory (host-set
// injection without a copy engine in the path).  -1 is the stop sentinel
// (src/yield.cu:142,857).
//
// Every wait in device code is bounded: a spin that exceeds its limit
// reports through a status word and lets the kernel unwind instead of
// hanging the GPU.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace apk {

// Device-side status codes (first error wins; written with atomicCAS).
enum DeviceStatus : int {
  DEV_OK = 0,
  DEV_WAIT_TIMEOUT_FULL = 1,    // an mbarrier 'stage full' wait exceeded its limit
  DEV_WAIT_TIMEOUT_TMEM = 2,    // a TMEM / MMA completion wait exceeded its limit
  DEV_WAIT_TIMEOUT_SPIN = 3,    // a flag spin exceeded its limit
  DEV_BAD_CONFIG = 4,           // kernel launched with an inconsistent shape
};

__device__ __forceinline__ long long globaltimer_ns() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned smid() {
  unsigned id;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(id));
  return id;
}

__device__ __forceinline__ int flag_load(const int* f) {
  int v;
  asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}

__device__ __forceinline__ void flag_store(int* f, int v) {
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}

// Acknowledge to the host through mapped pinned memory: the store is
// followed by a system-scope fence so it is pushed out to host memory now
// rather than whenever the write path drains.
__device__ __forceinline__ void ack_host(int* p) {
  flag_store(p, 1);
  __threadfence_system();
}

__device__ __forceinline__ void store_sys_ll(long long* p, long long v) {
  asm volatile("st.relaxed.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void report_status(int* status, int code, int* abort_word) {
  atomicCAS(status, 0, code);
  if (abort_word) atomicExch(abort_word, 1);
}

// Raise the generation to gen unless it is already >= gen or is the stop
// sentinel (a CAS loop, so a late trigger can never overwrite -1).
__device__ __forceinline__ void flag_raise(int* flag, int gen) {
  int old = *reinterpret_cast<volatile int*>(flag);
  while (old >= 0 && old < gen) {
    const int prev = atomicCAS(flag, old, gen);
    if (prev == old) break;
    old = prev;
  }
}

// Completed-tile accounting for count-triggered events: the CTA whose
// completion makes the counter reach count_trig[k] fires event k.
template <class EV>
__device__ __forceinline__ void count_trigger(const EV& ev) {
  if (ev.count_trig == nullptr) return;
  const unsigned long long n = atomicAdd(ev.completed, 1ull) + 1;
  for (int k = 0; k < ev.n_count; ++k)
    if (ev.count_trig[k] == n) {
      ev.set_ns[k] = globaltimer_ns();
      __threadfence();
      flag_raise(ev.flag, k + 1);
    }
}

// Grouped raster of the output-tile grid: tiles are walked in groups of
// `group` tile-rows, column-major inside a group, so the CTAs resident at
// one time share a few A row-panels and B column-panels and the working set
// of a wave stays in L2 (a row-major walk sweeps all of B once per tile-row).
// The order changes nothing but which CTA computes which tile.
__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int group, int& tm, int& tn) {
  const int per_group = group * tiles_n;
  const int g = tile / per_group;
  const int first = g * group;
  const int rows = (tiles_m - first) < group ? (tiles_m - first) : group;
  const int local = tile - g * per_group;
  tm = first + local % rows;
  tn = local / rows;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete, giving up after
// limit_ns of globaltimer time.  Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// ---- TMA (no multicast anywhere in this runtime) ---------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tm) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* tm, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// ---- streamed operands ------------------------------------------------------
// Wait (bounded) until both readiness words are nonzero; the copies they
// announce were written by a copy engine, so order this thread's later
// async-proxy (TMA) reads after the acquire.  False on timeout.
__device__ __forceinline__ bool wait_ready2(const int* a, const int* b, long long limit_ns) {
  const long long t0 = globaltimer_ns();
  while (true) {
    int va, vb;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(va) : "l"(a) : "memory");
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(vb) : "l"(b) : "memory");
    if (va != 0 && vb != 0) break;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// ---- cluster launch control (sm_100) ---------------------------------------
// Ask the hardware to cancel one not-yet-launched CTA of this grid; the
// 16-byte answer lands in *resp and completes 16 transaction bytes on bar
// (the caller arms bar with expect_tx first).  One-CTA clusters: no
// multicast form.
__device__ __forceinline__ void clc_try_cancel(void* resp, uint64_t* bar) {
  asm volatile("clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];" ::"r"(
                   smem_u32(resp)),
               "r"(smem_u32(bar))
               : "memory");
}
// Decode an answer: true and the cancelled CTA's x index, or false (nothing
// left to take, or the hardware kept the CTA for its own scheduling).
__device__ __forceinline__ bool clc_query(const void* resp, unsigned* ctaid_x) {
  unsigned valid = 0, x = 0;
  asm volatile(
      "{ .reg .pred p; .reg .b128 r;\n\t"
      "ld.shared.b128 r, [%2];\n\t"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, r;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t"
      "@p clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %1, r;\n\t"
      "}"
      : "=r"(valid), "=r"(x)
      : "r"(smem_u32(resp))
      : "memory");
  // the next request writes resp through the async proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  *ctaid_x = x;
  return valid != 0;
}

// Claim a free bit of a resident-slot bitmap (nslots bits); -1 if none came
// free within limit_ns.  At most nslots CTAs of one kernel are resident, and a
// CTA returns its bit before it exits, so a starting CTA finds one.
__device__ __forceinline__ int slot_claim(unsigned* bits, int nslots, long long limit_ns) {
  const int W = (nslots + 31) / 32;
  const long long t0 = globaltimer_ns();
  while (true) {
    for (int w = 0; w < W; ++w) {
      const int valid = nslots - 32 * w < 32 ? nslots - 32 * w : 32;
      const unsigned full = valid == 32 ? ~0u : ((1u << valid) - 1u);
      unsigned cur = *reinterpret_cast<volatile unsigned*>(&bits[w]);
      while ((cur & full) != full) {
        const int b = __ffs(~cur) - 1;
        const unsigned old = atomicOr(&bits[w], 1u << b);
        if (!(old & (1u << b))) return 32 * w + b;
        cur = old;
      }
    }
    if (globaltimer_ns() - t0 > limit_ns) return -1;
  }
}
__device__ __forceinline__ void slot_release(unsigned* bits, int slot) {
  atomicAnd(&bits[slot >> 5], ~(1u << (slot & 31)));
}

}  // namespace apk
