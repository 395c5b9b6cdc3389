// Flag-visibility microbenchmark: how long a generation raised by one CTA
// takes to be seen by every resident CTA, with no tile work in the way.
//
// Replaces the reference's visibility_poll<LOADED> (src/yield.cu:227-293)
// and its driver (src/yield.cu:466-564).  Every CTA runs a known-length
// dependent FMA chain per iteration, optionally streams loads from a buffer
// far larger than L2 (so HBM, not L2, serves them: the "under load"
// variant), then thread 0 polls the flag and logs the first observation of
// each new generation.  CTA 0 also raises the flag on a schedule of
// globaltimer offsets and stores -1 after the last event, so the run ends
// without the host.  B200 shape: the grid and the dynamic shared memory of
// the kernel whose residency is being studied (full residency), and a
// wall-clock limit on every CTA's loop so the probe always ends.
#include "common.cuh"
#include "proto.h"

namespace apk {
namespace vis {

constexpr int NT = 256;
constexpr int LOADS = 4;  // float4 loads in flight per thread per iteration

template <bool LOADED>
__global__ void __launch_bounds__(NT) visibility_poll(const __grid_constant__ VisParams p) {
  extern __shared__ float pad[];  // residency parity: sized like the studied kernel's ring
  __shared__ int s_flag, s_last, s_next;
  __shared__ long long s_base;
  const int tid = threadIdx.x, cta = blockIdx.x;
  const long long t0 = globaltimer_ns();
  if (tid == 0) {
    s_flag = 0;
    s_last = 0;
    s_next = 0;
    s_base = t0;
    p.t_begin[cta] = t0;
  }
  pad[tid] = (float)tid;
  __syncthreads();
  float acc = 1.0f;
  long long it = 0;
  const unsigned long long g = (unsigned long long)cta * NT + tid;
  const unsigned long long stride = (unsigned long long)gridDim.x * NT;
  unsigned long long pos = g;
  while (true) {
#pragma unroll 1
    for (int i = 0; i < p.work_iters; ++i) acc = fmaf(acc, 1.0000001f, 1e-7f);
    if (LOADED) {
      // consecutive threads read consecutive float4 (coalesced), the grid
      // sweeps the buffer: every byte comes from HBM once per sweep
      // (the host sizes the buffer to at least 2 * LOADS * stride float4, so
      // one conditional subtraction keeps every index in range)
      float4 v[LOADS];
#pragma unroll
      for (int j = 0; j < LOADS; ++j) {
        unsigned long long idx = pos + (unsigned long long)j * stride;
        if (idx >= p.traffic_n4) idx -= p.traffic_n4;
        v[j] = __ldcs(p.traffic + idx);
      }
#pragma unroll
      for (int j = 0; j < LOADS; ++j) acc += v[j].x + v[j].y + v[j].z + v[j].w;
      pos += LOADS * stride;
      if (pos >= p.traffic_n4) pos -= p.traffic_n4;
    }
    __syncthreads();
    if (tid == 0) {
      int f = flag_load(p.flag);
      const long long now = globaltimer_ns();
      if (cta == 0) {
        const int nx = s_next;
        if (nx < p.n_events) {
          if (now >= s_base + p.sched_ns[nx]) {
            p.set_ns[nx] = now;
            flag_store(p.flag, nx + 1);
            s_next = nx + 1;
          }
        } else if (now >= s_base + p.sched_ns[p.n_events - 1] + p.tail_ns) {
          flag_store(p.flag, -1);
        }
      }
      if (now - t0 > p.limit_ns) {
        atomicCAS(p.status, 0, DEV_WAIT_TIMEOUT_SPIN);
        f = -1;
      }
      s_flag = f;
    }
    __syncthreads();
    const int f = s_flag, last = s_last;
    __syncthreads();
    if (f < 0) break;
    if (f > last) {
      if (tid == 0) {
        const long long o = globaltimer_ns();
        for (int e = last; e < f && e < p.n_events; ++e) p.obs_ns[(size_t)e * gridDim.x + cta] = o;
        s_last = f;
      }
      __syncthreads();
    }
    ++it;
  }
  if (tid == 0) {
    p.iters[cta] = it;
    p.t_end[cta] = globaltimer_ns();
  }
  p.sink[g] = acc + pad[(tid + 1) % NT];
}

cudaError_t launch(const VisParams& prm, int grid, int smem_bytes, bool loaded, cudaStream_t stream) {
  const void* k = loaded ? reinterpret_cast<const void*>(&visibility_poll<true>)
                         : reinterpret_cast<const void*>(&visibility_poll<false>);
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e != cudaSuccess) return e;
  void* args[] = {const_cast<VisParams*>(&prm)};
  return cudaLaunchKernel(k, dim3(grid), dim3(NT), args, smem_bytes, stream);
}

int threads() { return NT; }
int loads_per_iter() { return LOADS; }

}  // namespace vis
}  // namespace apk
