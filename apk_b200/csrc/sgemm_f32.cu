// fp32 CUDA-core persistent SGEMM with tile-boundary and per-stage yield.
//
// Replaces the reference's SIMT tile routine and its persistent drivers:
//   tile_gemm            src/tile.cuh:62-107      (64x64 tile, scalar loads)
//   persistent_gemm      src/persistent.cu:51-79  (fetch-add queue)
//   persistent_yield     src/yield.cu:95-204      (boundary poll, mini-queue)
//   persistent_midyield  src/midyield.cu:92-320   (per-stage checkpoint)
//
// B200 design:
//   * 128x128 output tile, 128 threads, 8x16 register micro-tile per thread
//     computed with packed fp32 FMAs (fma.rn.f32x2: two round-to-nearest
//     FMAs per instruction, so half the issue slots of scalar FFMA for the
//     same sums), 2 CTAs per SM, K-tile BK (32 by default) staged by TMA
//     into a STAGES-deep ring of
//     shared-memory slots, each guarded by one transaction mbarrier.  A
//     slot is loaded as a [128 rows][32 k] box with 128-byte swizzle (so
//     rows read as float4 along k are bank-conflict free) and B as a
//     [32 k][128 cols] box without swizzle (float4 along n).
//   * One elected thread (tid 0) issues TMA and polls the yield flag; the
//     poll result is made uniform for the CTA by __syncthreads_or at the
//     stage barrier the ring needs anyway (the barrier that frees the slot
//     about to be refilled), so per-stage polling adds one relaxed load per
//     stage and no extra barrier (the reference paid two barriers per site,
//     src/midyield.cu:197-219, and a 14% cost at 1 CTA/SM,
//     results/summary/tc_summary.csv:8-10).
//   * Yield = the reference's cooperative mini-queue (src/yield.cu:163-183):
//     every CTA that observes a new generation pops urgent work items until
//     the queue is empty; the first popper is the claimer.  Unlike the
//     reference, a mid-pipeline yield does NOT abandon the background tile
//     (src/midyield.cu:237-318): in-flight TMA stages are drained, the
//     register accumulators are spilled to a global checkpoint slab with
//     the K cursor, the urgent items run through the same ring, and the
//     accumulators are restored so the tile continues at the same K stage
//     with the same FMA order -- bitwise identical to an uninterrupted run.
//   * Disciplines: DRAIN (always wait for in-flight stages before the slots
//     are reused) and POISON (drain, then corrupt one staged urgent value:
//     the detector's positive control, src/midyield.cu:146-147).  The
//     reference's NAIVE discipline (no wait) is not built: with an mbarrier
//     ring it would alias two transaction counts on one barrier phase, a
//     protocol error rather than the data race it measured.
//   * Every mbarrier wait is bounded (wait_limit_ns); a timeout sets the
//     status word and the abort word and the CTA unwinds.
#include "common.cuh"
#include "proto.h"

namespace apk {
namespace f32 {

// Tile geometries.  NT = BM threads: warp w owns output rows 32w .. 32w+31;
// thread (w, lane) holds rows 32w + lane/8 + 4i (i < 8) and columns
// (lane%8)*4 + 32q + 0..3 (q < BN/32): an 8 x BN/8 register micro-tile.
// SUB: K depth of one A box (32: 128-byte rows with the 128-byte swizzle;
// 16: 64-byte rows with the 64-byte swizzle); BK: K depth of one ring slot
// (a multiple of SUB); S: ring slots; MINB: resident CTAs per SM the
// register budget is compiled for.
//   L32: 128x128 tiles, 32-deep slots, 3 slots (97 KB): 2 CTAs per SM
//   L64: 128x128 tiles, 64-deep slots, 2 slots (129 KB): 1 CTA per SM
//   M:   64x128 tiles (two warps), 16-deep slots, 4 slots (49 KB): 4 CTAs
//        per SM
//   S:   32x128 tiles (one warp), 16-deep slots, 2 slots (21 KB): 8 CTAs
//        per SM
// Every geometry keeps the 8x16 micro-tile and thus at most 2 x 128
// threads' worth of registers per SM (255 per thread): at 4 and 8 CTAs per
// SM the CTA shrinks to two warps or one.  (64x64 and 128x64 tiles with 8x8
// micro-tiles, tried first, spilled at the 128 registers a thread gets
// there: the kernel's control state takes about 100.)
// Yield sites are every poll_every slots: the K-tile (the K depth between
// two sites) over BK.
template <int BM_, int BN_, int SUB_, int BK_, int S_, int MINB_>
struct Geo {
  static constexpr int BM = BM_, BN = BN_, NT = BM_, SUB = SUB_, BK = BK_, S = S_, MINB = MINB_;
  static constexpr int NQ = BN / 32;  // float4 column groups per thread
  static constexpr int A_BYTES = BM * BK * 4, B_BYTES = BK * BN * 4;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SMEM_BYTES = S * STAGE_BYTES + 1024;
  static_assert(BK % SUB == 0 && (SUB == 32 || SUB == 16), "A boxes are 32 or 16 deep");
};
using GeoL32 = Geo<128, 128, 32, 32, 3, 2>;
using GeoL64 = Geo<128, 128, 32, 64, 2, 1>;
using GeoM = Geo<64, 128, 16, 16, 4, 4>;
using GeoS = Geo<32, 128, 16, 16, 2, 8>;
enum GeoId : int { GEO_L32 = F32_GEO_L32, GEO_L64 = F32_GEO_L64, GEO_M = F32_GEO_M, GEO_S = F32_GEO_S };

// Physical 16-byte chunk of logical chunk kc in A row 32w + ty + 4i: the
// 128-byte swizzle XORs the chunk with (row & 7) = ty + 4(i & 1); the
// 64-byte swizzle with ((row >> 1) & 3) = (ty >> 1) + 2(i & 1).
template <class GE>
__device__ __forceinline__ int a_chunk(int kc, int ty, int i) {
  if constexpr (GE::SUB == 32) return kc ^ (ty + 4 * (i & 1));
  else return kc ^ ((ty >> 1) + 2 * (i & 1));
}

// One k-pair kp of one SUB-deep A box: acc[i][j] += A[r_i][k] * B[k][c_j]
// for its two k in increasing order.  A is read two k at a time (float2 per
// row) and B one k at a time (BN/32 float4, each row segment one 128-byte
// wavefront).  The FMAs are packed in pairs of adjacent columns with
// __ffma2_rn: each lane of the pair is the same round-to-nearest FMA as
// fmaf, so every sum and its k order is exactly that of scalar FMAs, while
// one instruction carries two FMAs -- half the issue slots, which is what
// lets 8 warps per SM keep the FP32 pipe fed (the 8x8 scalar tiling at 16
// warps per SM was issue-bound at ~60% of the pipe).
template <class GE>
__device__ __forceinline__ void kpair(const float* __restrict__ Asub, const float* __restrict__ Bsub,
                                      float (&acc)[8][4 * GE::NQ], int arow0, int ty, int bcol, int kp) {
  const int kc = kp >> 1, half = kp & 1;
  float2 a[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    a[i] = *reinterpret_cast<const float2*>(Asub + (arow0 + 4 * i) * GE::SUB + (a_chunk<GE>(kc, ty, i) << 2) +
                                            2 * half);
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    const float* brow = Bsub + (kp * 2 + kk) * GE::BN + bcol;
    float4 b[GE::NQ];
#pragma unroll
    for (int q = 0; q < GE::NQ; ++q) b[q] = *reinterpret_cast<const float4*>(brow + 32 * q);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float av = kk == 0 ? a[i].x : a[i].y;
      const float2 ad = make_float2(av, av);
#pragma unroll
      for (int q = 0; q < GE::NQ; ++q) {
        float2 c0 = make_float2(acc[i][4 * q], acc[i][4 * q + 1]);
        float2 c1 = make_float2(acc[i][4 * q + 2], acc[i][4 * q + 3]);
        c0 = __ffma2_rn(ad, make_float2(b[q].x, b[q].y), c0);
        c1 = __ffma2_rn(ad, make_float2(b[q].z, b[q].w), c1);
        acc[i][4 * q] = c0.x;
        acc[i][4 * q + 1] = c0.y;
        acc[i][4 * q + 2] = c1.x;
        acc[i][4 * q + 3] = c1.y;
      }
    }
  }
}

// poll: when non-null (tid 0 of a background stage), the yield flag is
// loaded into pend two k-pairs before the end of the slot, so the value the
// next slot barrier publishes is a fraction of a slot old while the load
// latency still hides under the remaining FMAs.
template <class GE>
__device__ __forceinline__ void compute_stage(const float* __restrict__ As, const float* __restrict__ Bs,
                                              float (&acc)[8][4 * GE::NQ], int arow0, int ty, int bcol, bool poll,
                                              const int* flag, const int* const* flag_at, int& pend) {
  constexpr int KP = GE::SUB / 2;
#pragma unroll
  for (int sub = 0; sub < GE::BK / GE::SUB; ++sub) {
    const float* Asub = As + sub * (GE::BM * GE::SUB);
    const float* Bsub = Bs + sub * GE::SUB * GE::BN;
    // not unrolled: unrolled by two the loop ran faster in a mainloop probe
    // (56.4 against 52.1 TFLOP/s, operands resident in shared memory) but
    // with this kernel's control state it exceeds 255 registers and spills
#pragma unroll 1
    for (int kp = 0; kp < KP - 2; ++kp) kpair<GE>(Asub, Bsub, acc, arow0, ty, bcol, kp);
    // the poll sits between two loops, not behind a per-iteration branch
    // 4 or 8 CTAs per SM poll their flag copy, whose address the CTA keeps in
    // shared memory (flag_at), read only on this branch so that no register
    // holds it through the loop; at 1 or 2 the launch keeps one copy, the
    // flag itself (a kernel parameter, no register either)
    if (sub == GE::BK / GE::SUB - 1 && poll) pend = flag_load(GE::MINB >= 4 ? *flag_at : flag);
    // keeps the two loops apart when there is no poll (POLL_OFF), so that
    // variant is the polling code minus the load, not a re-fused loop whose
    // speed measured 39.7 or 42.1 TFLOP/s depending on the B200 it ran on
    asm volatile("" ::: "memory");
#pragma unroll 1
    for (int kp = KP - 2; kp < KP; ++kp) kpair<GE>(Asub, Bsub, acc, arow0, ty, bcol, kp);
  }
}

template <class GE>
__device__ __forceinline__ void issue_stage(uint8_t* smem, uint64_t* full, uint32_t seq, const CUtensorMap* tA,
                                            const CUtensorMap* tB, int row0, int col0, int k0) {
  const int slot = seq % GE::S;
  float* a = reinterpret_cast<float*>(smem + slot * GE::A_BYTES);
  float* b = reinterpret_cast<float*>(smem + GE::S * GE::A_BYTES + slot * GE::B_BYTES);
  mbar_arrive_expect_tx(&full[slot], GE::STAGE_BYTES);
#pragma unroll
  for (int sub = 0; sub < GE::BK / GE::SUB; ++sub)
    tma_load_2d(a + sub * GE::BM * GE::SUB, tA, k0 + sub * GE::SUB, row0, &full[slot]);
  tma_load_2d(b, tB, col0, k0, &full[slot]);
}

// Work distribution: SCHED_QUEUE = persistent grid of resident CTAs popping
// a global fetch-add counter (src/persistent.cu:51-79); SCHED_CLC = one CTA
// per task, each running CTA taking not-yet-launched CTAs' tasks with
// cluster launch control.  Under CLC the hardware may decline a request
// (e.g. while a higher-priority stream's kernel waits for an SM); the CTA
// then exits and frees its SM, and the grid's remaining CTAs launch later.
enum Sched : int { SCHED_QUEUE = 0, SCHED_CLC = 1 };
constexpr unsigned long long NO_TASK = ~0ull;

template <int POLL, int DISC, bool ORACLE, class GE, int SCHED>
__global__ void __launch_bounds__(GE::NT, GE::MINB) sgemm_persistent(const __grid_constant__ F32Params p) {
  constexpr int S = GE::S, BM = GE::BM, BN = GE::BN, NT = GE::NT, BK = GE::BK, NQ = GE::NQ, NJ = 4 * GE::NQ;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[S];
  __shared__ unsigned long long s_task;
  __shared__ int s_f, s_item;
  // CLC: the answer buffer and barrier of the one request kept in flight,
  // the task it will yield, and this CTA's resident slot
  __shared__ __align__(16) uint4 s_clcResp;
  __shared__ __align__(8) uint64_t s_clcBar;
  __shared__ unsigned long long s_clcNext;
  __shared__ int s_clcInFlight, s_slot;
  __shared__ const int* s_flag;  // the flag copy this CTA polls
  __shared__ uint32_t s_clcPhase;
  // Bookkeeping touched only by tid 0, or needed only across a job switch,
  // lives in shared memory: as per-thread locals it costs every thread
  // registers under the 2-CTA/SM cap (the reference hit the same,
  // src/yield.cu:106-110).
  __shared__ int s_lastSeen, s_nextEv, s_site, s_inflight;
  __shared__ long long s_gBase;
  __shared__ unsigned long long s_myTiles, s_bgTask;
  __shared__ int s_bgRow0, s_bgCol0, s_bgC, s_pending;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int ty = lane >> 3;
  const int arow0 = warp * 32 + ty;
  const int bcol = (lane & 7) * 4;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
    if constexpr (SCHED == SCHED_CLC) mbar_init(&s_clcBar, 1);
    fence_mbar_init();
    s_lastSeen = 0;
    s_nextEv = 0;
    s_gBase = 0;
    s_myTiles = 0;
    s_pending = 0;
    s_slot = (int)blockIdx.x;
    if constexpr (SCHED == SCHED_CLC) {
      s_slot = slot_claim(p.q.slot_bits, p.q.nslots, p.wait_limit_ns);
      s_clcNext = blockIdx.x;
      s_clcInFlight = 0;
      s_clcPhase = 0;
      // a CTA launched mid-run takes the generations raised before it as
      // seen: their urgent work was popped by the CTAs that observed them
      const int f0 = flag_load(p.ev.flag);
      s_lastSeen = f0 > 0 ? f0 : 0;
      if (s_slot == 0 && p.q.setter_state != nullptr) {
        s_nextEv = (int)p.q.setter_state[0];
        s_gBase = p.q.setter_state[1];
      }
    }
    tma_prefetch_desc(&p.tmA);
    tma_prefetch_desc(&p.tmB);
    tma_prefetch_desc(&p.tmAu);
    tma_prefetch_desc(&p.tmBu);
    if constexpr (GE::MINB >= 4) s_flag = flag_copy(p.ev, s_slot < 0 ? 0 : s_slot);
    atomicMin(p.q.start_min, (unsigned long long)globaltimer_ns());
  }
  __syncthreads();
  // per-CTA logs, counters and the checkpoint slab are indexed by cta(): the
  // block index, or the resident slot under CLC, kept in shared memory and
  // re-read where it is used (rare paths).  Read from the special register
  // instead, the polling queue variants compiled to ~20 more registers
  // (252 of 255) and ran 10% slower (41 against 45 TFLOP/s).
  auto cta = [&]() -> int { return *reinterpret_cast<volatile int*>(&s_slot); };
  auto grid = [&]() -> int {
    if constexpr (SCHED == SCHED_CLC) return p.q.nslots;
    else return (int)gridDim.x;
  };
  if constexpr (SCHED == SCHED_CLC) {
    if (s_slot < 0) {  // no slot came free (cannot happen while residency holds)
      if (tid == 0) report_status(p.ev.status, DEV_BAD_CONFIG, p.ev.abort_word);
      return;
    }
  }

  // CLC: hand out the task prefetched one request earlier and put the next
  // request in flight, so its latency hides under the coming tile (tid 0)
  auto clc_take = [&]() -> unsigned long long {
    if (s_clcInFlight) {
      s_clcInFlight = 0;
      if (!mbar_wait(&s_clcBar, s_clcPhase, p.wait_limit_ns)) {
        report_status(p.ev.status, DEV_WAIT_TIMEOUT_SPIN, p.ev.abort_word);
        s_clcNext = NO_TASK;
      } else {
        unsigned x = 0;
        s_clcNext = clc_query(&s_clcResp, &x) ? (unsigned long long)x : NO_TASK;
      }
      s_clcPhase ^= 1u;
    }
    const unsigned long long t = s_clcNext;
    s_clcNext = NO_TASK;
    if (t != NO_TASK) {
      mbar_arrive_expect_tx(&s_clcBar, 16);
      clc_try_cancel(&s_clcResp, &s_clcBar);
      s_clcInFlight = 1;
    }
    return t;
  };

  uint32_t P = 0, Q = 0;  // issued / consumed stage sequence numbers (uniform)
  bool bad = false;       // this thread saw a wait time out
  int pend = 0;           // tid 0: last flag value loaded inside a stage
  float acc[8][NJ];

  // Job state (uniform).  A job is a background tile or one urgent item;
  // both run through the single mainloop below.
  bool urgent = false;    // current job is an urgent item
  bool bg_active = false; // a background tile is in progress (maybe suspended)
  bool ckpt = false;      // background accumulators are in the slab
  int row0 = 0, col0 = 0, kst0 = 0, nk = 0, c = 0;
  int ev = 0, popE = 0, popF = 0;  // urgent queue range still to pop
  bool popped = false;             // this CTA ran an item of event popE

  auto setter = [&]() {  // device-set events (src/yield.cu:186-195), tid 0 of CTA 0
    const int nextEv = s_nextEv;
    if (cta() == 0 && p.ev.sched_ns != nullptr && nextEv < p.ev.n_sched) {
      const long long now = globaltimer_ns();
      if (s_gBase == 0) s_gBase = now;
      if (now >= s_gBase + p.ev.sched_ns[nextEv]) {
        p.ev.set_ns[nextEv] = now;
        // 1 or 2 CTAs per SM: the launch keeps one flag copy; the loop over
        // copies, compiled into those kernels, cost them 8% of their speed
        if constexpr (GE::MINB >= 4) flag_raise(p.ev, nextEv);  // never overwrites the -1 sentinel
        else atomicCAS(p.ev.flag, nextEv, nextEv + 1);
        s_nextEv = nextEv + 1;
      }
    }
  };

  auto drain = [&]() {  // wait out every issued-but-unconsumed stage
    while (Q != P) {
      if (!mbar_wait(&full[Q % S], (Q / S) & 1, p.wait_limit_ns)) bad = true;
      ++Q;
    }
  };

  auto prime = [&](int from) {  // issue stages [from, from + S-1) of the job
    int n = nk - from;
    n = n < S - 1 ? n : S - 1;
    if (tid == 0) {
      const CUtensorMap* tA = urgent ? &p.tmAu : &p.tmA;
      const CUtensorMap* tB = urgent ? &p.tmBu : &p.tmB;
      for (int s = 0; s < n; ++s) issue_stage<GE>(smem, full, P + s, tA, tB, row0, col0, (kst0 + from + s) * BK);
    }
    P += n;
  };

  // Observation of new generations at a poll site (tid 0 wrote s_f before
  // the barrier that brought every thread here).  Returns true = exit.
  auto observe = [&](int site) -> bool {
    const int f = s_f;
    const int anyBad = __syncthreads_or(bad);  // also: everyone has read s_f
    if (anyBad || f < 0) {
      drain();
      if (anyBad && tid == 0) report_status(p.ev.status, DEV_WAIT_TIMEOUT_FULL, p.ev.abort_word);
      return true;
    }
    if (tid == 0) {
      const long long g = globaltimer_ns();
      for (int e = s_lastSeen; e < f && e < p.ev.max_events; ++e) p.ev.obs_ns[(size_t)e * grid() + cta()] = g;
      s_item = s_lastSeen;
      s_lastSeen = f;
      s_site = site;
      s_inflight = (int)(P - Q);
    }
    __syncthreads();
    popE = s_item;
    popF = f < p.ev.max_events ? f : p.ev.max_events;
    popped = false;
    return false;
  };

  while (true) {
    // ======================= choose the next job ===========================
    if (popE < popF) {
      // cooperative urgent mini-queue (src/yield.cu:163-183)
      if (tid == 0) {
        const int it = atomicAdd(&p.ev.uq_next[popE], 1);
        if (it == 0) {
          p.ev.claim_ns[popE] = globaltimer_ns();
          p.ev.claim[popE] = cta() + 1;
          p.ev.claim_site[popE] = s_site;
          p.ev.inflight[popE] = s_inflight;
          if (p.ev.ack != nullptr) ack_host(&p.ev.ack[2 * popE]);
        }
        s_item = it;
      }
      __syncthreads();
      const int it = s_item;
      __syncthreads();
      if (it >= p.uitems) {
        if (popped && tid == 0) atomicMax(&p.ev.done_ns[popE], (unsigned long long)globaltimer_ns());
        ++popE;
        popped = false;
        continue;
      }
      if (!ckpt) {
        // checkpoint: drain in-flight stages, park the accumulators
        drain();
        if (bg_active) {
          float4* s4 = reinterpret_cast<float4*>(p.slab) + (size_t)cta() * (BM * BN / 4);
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int q = 0; q < NQ; ++q)
              s4[(i * NQ + q) * NT + tid] =
                  make_float4(acc[i][4 * q], acc[i][4 * q + 1], acc[i][4 * q + 2], acc[i][4 * q + 3]);
          if (tid == 0) {
            s_bgRow0 = row0;
            s_bgCol0 = col0;
            s_bgC = c;
            long long* hdr = p.slab_hdr + (size_t)cta() * 4;
            hdr[0] = (long long)s_bgTask;
            hdr[1] = c;
            hdr[2] = popE;
            hdr[3] = 1;
            atomicAdd(p.q.yields, 1ull);
          }
        }
        ckpt = true;
      }
      popped = true;
      urgent = true;
      ev = popE;
      const int t = it / p.usplit, ks = it % p.usplit;
      row0 = (t / p.utiles_n) * BM;
      col0 = (t % p.utiles_n) * BN;
      nk = p.unk;
      kst0 = ks * p.unk;
      c = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < NJ; ++j) acc[i][j] = 0.f;
      __syncthreads();  // the slot refilled first was read by the previous job
      prime(0);
    } else if (bg_active) {
      if (ckpt) {
        // resume the background tile from its checkpoint
        urgent = false;
        ckpt = false;
        row0 = s_bgRow0;
        col0 = s_bgCol0;
        c = s_bgC;
        kst0 = 0;
        nk = p.nk;
        const float4* s4 = reinterpret_cast<const float4*>(p.slab) + (size_t)cta() * (BM * BN / 4);
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int q = 0; q < NQ; ++q) {
            const float4 v = s4[(i * NQ + q) * NT + tid];
            acc[i][4 * q] = v.x;
            acc[i][4 * q + 1] = v.y;
            acc[i][4 * q + 2] = v.z;
            acc[i][4 * q + 3] = v.w;
          }
        __syncthreads();
        prime(c);
      }
      // else: no item was popped; the job continues with its stages in flight
    } else {
      // ---------------- tile boundary: pop a background task --------------
      // A task popped before a boundary yield is kept (s_pending) and run
      // after the urgent work, never dropped (src/yield.cu:197-202).
      ckpt = false;
      int fl = 0;
      bool yb = false;
      if (tid == 0) {
        if (!s_pending) {
          if constexpr (SCHED == SCHED_CLC) s_task = clc_take();
          else s_task = atomicAdd(p.q.next_task, 1ull);
        }
        s_pending = 0;
        const int ab = *reinterpret_cast<volatile int*>(p.ev.abort_word);
        fl = s_lastSeen;
        if (POLL == POLL_BOUNDARY) {
          setter();
          fl = flag_load(GE::MINB >= 4 ? s_flag : p.ev.flag);
        }
        if (ab) fl = -1;
        s_f = fl;
        yb = fl != s_lastSeen;
      }
      const int y = __syncthreads_or(yb || bad);
      const unsigned long long task = s_task;
      if (y) {
        if (observe(-1)) break;
        if (popE < popF) {
          if (tid == 0) s_pending = 1;  // run this task after the urgent work
          continue;                     // boundary yield: pipeline is empty
        }
      }
      if (task >= p.q.num_tasks) break;
      if (tid == 0) s_bgTask = task;
      const int tile = (int)(task % (unsigned long long)p.total_tiles);
      urgent = false;
      bg_active = true;
      {
        int tm, tn;
        if (p.st.order != nullptr)
          stream_tile(p.st, tile, p.tiles_n, tm, tn);
        else
          tile_coords(tile, p.total_tiles / p.tiles_n, p.tiles_n, 8, tm, tn);
        row0 = tm * BM;
        col0 = tn * BN;
      }
      kst0 = 0;
      nk = p.nk;
      c = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < NJ; ++j) acc[i][j] = 0.f;
      // streamed operands: the tile's A row panel and B column panel must
      // have landed before its first TMA load
      if (p.st.a_ready != nullptr && tid == 0 &&
          !wait_ready2(&p.st.a_ready[(row0 / BM) / p.st.panel_tm], &p.st.b_ready[(col0 / BN) / p.st.b_units],
                       p.wait_limit_ns)) {
        bad = true;
        report_status(p.ev.status, DEV_WAIT_TIMEOUT_SPIN, p.ev.abort_word);
      }
      prime(0);
    }

    // ============================ mainloop =================================
    bool yielded = false;
    for (; c < nk; ++c) {
      bool ys = false;
      if (POLL == POLL_STAGE && !urgent && tid == 0) {
        const int fs = pend;  // loaded near the end of the previous slot
        setter();
        s_f = fs;
        // a yield site every poll_every slots (one K-tile)
        ys = fs != s_lastSeen && (p.poll_every <= 1 || c % p.poll_every == 0);
      }
      // frees the slot refilled below (read by every thread one stage ago)
      const int y = __syncthreads_or(ys || bad);
      if (y) {
        yielded = true;
        break;
      }
      if (c + S - 1 < nk) {
        if (tid == 0)
          issue_stage<GE>(smem, full, P, urgent ? &p.tmAu : &p.tmA, urgent ? &p.tmBu : &p.tmB, row0, col0,
                          (kst0 + c + S - 1) * BK);
        ++P;
      }
      if (!mbar_wait(&full[Q % S], (Q / S) & 1, p.wait_limit_ns)) bad = true;
      const int slot = Q % S;
      const float* As = reinterpret_cast<const float*>(smem + slot * GE::A_BYTES);
      const float* Bs = reinterpret_cast<const float*>(smem + S * GE::A_BYTES + slot * GE::B_BYTES);
      if (DISC == DISC_POISON && urgent && c == 0) {
        // detector control: one wrong staged value in each urgent item
        if (tid == 0) {
          const_cast<float*>(Bs)[0] += 1.0f;
          fence_proxy_async_smem();
        }
        __syncthreads();
      }
      compute_stage<GE>(As, Bs, acc, arow0, ty, bcol, POLL == POLL_STAGE && !urgent && tid == 0, p.ev.flag, &s_flag,
                        pend);
      ++Q;
    }
    if (yielded) {
      if (observe(c)) break;
      continue;  // pop urgent items (or resume this tile if none are left)
    }

    // ============================ epilogue =================================
    if (!urgent) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float* crow = p.C + (size_t)(row0 + arow0 + 4 * i) * p.ldc + col0 + bcol;
#pragma unroll
        for (int q = 0; q < NQ; ++q)
          *reinterpret_cast<float4*>(crow + 32 * q) =
              make_float4(acc[i][4 * q], acc[i][4 * q + 1], acc[i][4 * q + 2], acc[i][4 * q + 3]);
      }
      bg_active = false;
      if (p.st.done != nullptr) __threadfence();  // the block's copy back reads these stores
      __syncthreads();  // the whole tile is stored before it counts as complete
      if (tid == 0) {
        ++s_myTiles;
        if (ORACLE && p.q.exec_count != nullptr) atomicAdd(&p.q.exec_count[s_bgTask], 1);
        count_trigger(p.ev);
        if (p.st.done != nullptr)
          stream_tile_done(p.st, p.total_tiles / p.tiles_n, p.tiles_n, row0 / BM, col0 / BN);
      }
    } else {
      float* Cu = p.Cu + (size_t)ev * p.cu_stride;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float* crow = Cu + (size_t)(row0 + arow0 + 4 * i) * p.ldcu + col0 + bcol;
        if (p.usplit == 1) {
#pragma unroll
          for (int q = 0; q < NQ; ++q)
            *reinterpret_cast<float4*>(crow + 32 * q) =
                make_float4(acc[i][4 * q], acc[i][4 * q + 1], acc[i][4 * q + 2], acc[i][4 * q + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < NJ; ++j) atomicAdd(crow + 32 * (j >> 2) + (j & 3), acc[i][j]);
        }
      }
      __syncthreads();  // whole item written before it is counted
      if (tid == 0) {
        if (ORACLE) atomicAdd(&p.ev.uexec[ev], 1);
        __threadfence();
        const int done = atomicAdd(&p.ev.udone_cnt[ev], 1) + 1;
        if (done == p.uitems && p.ev.ack != nullptr) ack_host(&p.ev.ack[2 * ev + 1]);
      }
      urgent = false;
    }
  }

  drain();
  if (tid == 0) {
    if (bad) report_status(p.ev.status, DEV_WAIT_TIMEOUT_FULL, p.ev.abort_word);
    if constexpr (SCHED == SCHED_CLC) {
      // a request still in flight (a stopped or aborted run) must land before
      // shared memory goes away; a task it took is dropped with the run
      if (s_clcInFlight) mbar_wait(&s_clcBar, s_clcPhase, p.wait_limit_ns);
      if (cta() == 0 && p.q.setter_state != nullptr) {
        p.q.setter_state[0] = s_nextEv;
        p.q.setter_state[1] = s_gBase;
      }
      atomicAdd(&p.q.tiles_done[cta()], s_myTiles);
    } else {
      p.q.tiles_done[cta()] = s_myTiles;
    }
    atomicMax(p.q.end_max, (unsigned long long)globaltimer_ns());
    atomicAdd(p.q.exited, 1);
    if constexpr (SCHED == SCHED_CLC) {
      __threadfence();
      slot_release(p.q.slot_bits, cta());  // last: the slot's logs are written
    }
  }
}

// Host-side dispatch over the template instantiations.  geo: GEO_L32,
// GEO_L64, GEO_M, GEO_S (the Geo aliases above).

template <int POLL, int DISC, bool ORACLE, class GE, int SCHED>
static const void* kernel_ptr() {
  return reinterpret_cast<const void*>(&sgemm_persistent<POLL, DISC, ORACLE, GE, SCHED>);
}

static const void* select_kernel(int poll, int disc, bool oracle, int geo, int sched) {
#define APK_SEL(PL, DS, OR, SC)                                                    \
  if (poll == PL && disc == DS && oracle == OR && sched == SC) {                  \
    if (geo == GEO_L32) return kernel_ptr<PL, DS, OR, GeoL32, SC>();             \
    if (geo == GEO_L64) return kernel_ptr<PL, DS, OR, GeoL64, SC>();             \
  }
  APK_SEL(POLL_OFF, DISC_DRAIN, false, SCHED_QUEUE)
  APK_SEL(POLL_OFF, DISC_DRAIN, true, SCHED_QUEUE)
  APK_SEL(POLL_BOUNDARY, DISC_DRAIN, false, SCHED_QUEUE)
  APK_SEL(POLL_BOUNDARY, DISC_DRAIN, true, SCHED_QUEUE)
  APK_SEL(POLL_BOUNDARY, DISC_POISON, false, SCHED_QUEUE)
  APK_SEL(POLL_STAGE, DISC_DRAIN, false, SCHED_QUEUE)
  APK_SEL(POLL_STAGE, DISC_DRAIN, true, SCHED_QUEUE)
  APK_SEL(POLL_STAGE, DISC_POISON, false, SCHED_QUEUE)
  APK_SEL(POLL_STAGE, DISC_POISON, true, SCHED_QUEUE)
  APK_SEL(POLL_OFF, DISC_DRAIN, false, SCHED_CLC)
  APK_SEL(POLL_OFF, DISC_DRAIN, true, SCHED_CLC)
  APK_SEL(POLL_BOUNDARY, DISC_DRAIN, false, SCHED_CLC)
  APK_SEL(POLL_BOUNDARY, DISC_DRAIN, true, SCHED_CLC)
  APK_SEL(POLL_STAGE, DISC_DRAIN, false, SCHED_CLC)
  APK_SEL(POLL_STAGE, DISC_DRAIN, true, SCHED_CLC)
#undef APK_SEL
  // the multi-CTA geometries (queue scheduler): the scaling surface's 4 and
  // 8 CTAs per SM
#define APK_SEL(PL, DS, OR)                                                    \
  if (poll == PL && disc == DS && oracle == OR && sched == SCHED_QUEUE) {      \
    if (geo == GEO_M) return kernel_ptr<PL, DS, OR, GeoM, SCHED_QUEUE>();      \
    if (geo == GEO_S) return kernel_ptr<PL, DS, OR, GeoS, SCHED_QUEUE>();      \
  }
  APK_SEL(POLL_OFF, DISC_DRAIN, false)
  APK_SEL(POLL_OFF, DISC_DRAIN, true)
  APK_SEL(POLL_BOUNDARY, DISC_DRAIN, false)
  APK_SEL(POLL_STAGE, DISC_DRAIN, false)
  APK_SEL(POLL_STAGE, DISC_DRAIN, true)
  APK_SEL(POLL_STAGE, DISC_POISON, false)
#undef APK_SEL
  return nullptr;
}

template <class GE>
static GeoInfo info_of() {
  return GeoInfo{GE::BM, GE::BN, GE::NT, GE::BK, GE::S, GE::SUB, GE::SMEM_BYTES};
}

GeoInfo geo_info(int geo) {
  switch (geo) {
    case GEO_L64: return info_of<GeoL64>();
    case GEO_M: return info_of<GeoM>();
    case GEO_S: return info_of<GeoS>();
    default: return info_of<GeoL32>();
  }
}
size_t params_bytes() { return sizeof(F32Params); }

cudaError_t prepare(int poll, int disc, bool oracle, int geo, int sched, int* max_ctas_per_sm) {
  const void* k = select_kernel(poll, disc, oracle, geo, sched);
  if (!k) return cudaErrorInvalidValue;
  const GeoInfo g = geo_info(geo);
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, g.smem_bytes);
  if (e != cudaSuccess) return e;
  // the whole unified L1 as shared memory, whatever grid an earlier launch used
  e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(max_ctas_per_sm, k, g.threads, g.smem_bytes);
}

cudaError_t launch(const F32Params& prm, int grid, int poll, int disc, bool oracle, int geo, int sched,
                   cudaStream_t stream) {
  const void* k = select_kernel(poll, disc, oracle, geo, sched);
  if (!k) return cudaErrorInvalidValue;
  const GeoInfo g = geo_info(geo);
  void* args[] = {const_cast<F32Params*>(&prm)};
  return cudaLaunchKernel(k, dim3(grid), dim3(g.threads), args, g.smem_bytes, stream);
}

}  // namespace f32
}  // namespace apk

// ===========================================================================
// Allocation-free entry point: apk_sgemm_f32_noalloc.
//
// For callers that cannot call cudaMalloc: a process whose device memory is
// owned by a pool it does not control, code running where an allocation
// would synchronize the device or is not allowed (a latency-critical serving
// loop after start-up, a library called from inside another framework's
// stream-ordered work).  The same persistent fp32 SGEMM drain runs with its
// scratch -- the work-queue counter, exit bookkeeping and per-CTA tile
// counters -- in the file-scope array below instead of memory from
// cudaMalloc.  The caller passes inputs and output; nothing is allocated or
// freed on this path.
//
// The array exists once per device that loads this library and lives until
// the process exits.  Its device address is obtained with
// cudaGetSymbolAddress at the first call on each device (with that device
// current); that first call should therefore come before any stream capture.
// Every call on one device shares that device's array and it keeps the last
// call's contents: the queue header is cleared on the caller's stream before
// each launch, so calls issued in order on one stream are independent, while
// calls that overlap on the same device (for example on two streams) race on
// the same scratch and must not be issued.  Calls on different devices use
// different instances of the array and do not interact.
//
// The device status word sits in the same header.  A kernel whose bounded
// wait ran out (2 s) records a code there and leaves C incomplete; since the
// call itself is asynchronous, apk_sgemm_f32_noalloc_status reads the word
// back after the caller's stream has drained (no allocation either).
// ===========================================================================
#include <cstdio>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "../../include/apk.h"

namespace apk {
namespace f32 {
namespace {

constexpr size_t kNoAllocScratchBytes = 16384;  // stated maximum
constexpr size_t kNoAllocHeaderBytes = 256;
// 2016 per-CTA counters.  The kernel fits at most 2 CTAs per SM (97 KB of
// shared memory each), so residency -- checked first -- stays far below this
// on a B200 (296); the size check guards parts with more than 1008 SMs.
constexpr int kNoAllocMaxGrid = (int)((kNoAllocScratchBytes - kNoAllocHeaderBytes) / sizeof(unsigned long long));
static_assert(kNoAllocMaxGrid >= 2 * 148, "the static scratch must cover a B200's full residency");

struct NoAllocHeader {
  unsigned long long next_task, start_min, end_max, yields;
  int exited, abort_word, status, flag;
  int never_set;  // a word no code path writes (the status path's self-test)
};
static_assert(sizeof(NoAllocHeader) <= kNoAllocHeaderBytes, "header must fit");

struct NoAllocDevice {
  bool ready = false;
  unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch
  int sms = 0;
  int max_ctas_per_sm = 0;
};

constexpr int kMaxDevices = 64;
NoAllocDevice g_noalloc_dev[kMaxDevices];
std::mutex g_noalloc_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_noalloc_encode = nullptr;

}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

}  // namespace f32
}  // namespace apk

namespace apk {
namespace f32 {
namespace {

// A bounded spin on a word nothing writes: it gives up after limit_ns and
// records DEV_WAIT_TIMEOUT_SPIN in the status word, exactly as a kernel
// whose mbarrier wait ran out does.
__global__ void noalloc_spin_kernel(const int* word, long long limit_ns, int* status) {
  if (threadIdx.x != 0) return;
  const long long t0 = globaltimer_ns();
  while (flag_load(word) != 1)
    if (globaltimer_ns() - t0 > limit_ns) {
      atomicCAS(status, 0, DEV_WAIT_TIMEOUT_SPIN);
      return;
    }
}

// One-time set-up on the current device (the scratch array's device
// address, the kernel's shared-memory attribute, the SM count).  Returns
// the device's record, or nullptr on a CUDA failure.
NoAllocDevice* noalloc_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  NoAllocDevice& d = g_noalloc_dev[dev];
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!d.ready) {
      // one-time set-up on this device (it is current): the scratch array's
      // device address, the kernel's shared-memory attribute, SM count
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return nullptr;
      int maxc = 0;
      if (prepare(POLL_OFF, DISC_DRAIN, false, GEO_L32, SCHED_QUEUE, &maxc) != cudaSuccess || maxc < 1) return nullptr;
      int sms = 0;
      if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return nullptr;
      if (!g_noalloc_encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
          return nullptr;
        g_noalloc_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
      }
      d.scratch = static_cast<unsigned char*>(ptr);
      d.sms = sms;
      d.max_ctas_per_sm = maxc;
      d.ready = true;
    }
  }
  return &d;
}

}  // namespace
}  // namespace f32
}  // namespace apk

extern "C" apk_status apk_sgemm_f32_noalloc(const float* A, const float* B, float* C, int M, int N, int K,
                                            int grid, void* stream) {
  using namespace apk;
  using namespace apk::f32;
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0 || M % 128 || N % 128 || K % 32) return APK_EINVAL;
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) | reinterpret_cast<uintptr_t>(C)) & 15)
    return APK_EINVAL;
  NoAllocDevice* dp = noalloc_device();
  if (dp == nullptr) return APK_ECUDA;
  NoAllocDevice& d = *dp;
  const int resident = d.sms * d.max_ctas_per_sm;
  if (grid <= 0) grid = resident;
  if (grid > resident) return APK_EINVAL;  // CTAs beyond residency never start
  if (grid > kNoAllocMaxGrid) {
    fprintf(stderr,
            "apk_sgemm_f32_noalloc: grid %d needs %zu bytes of scratch; the static array holds %zu (max grid %d)\n",
            grid, kNoAllocHeaderBytes + (size_t)grid * sizeof(unsigned long long), kNoAllocScratchBytes,
            kNoAllocMaxGrid);
    return APK_EINVAL;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  F32Params p;
  memset(&p, 0, sizeof p);
  auto enc = [&](CUtensorMap* tm, const void* base, long long rows, long long cols, int box_cols, int box_rows,
                 CUtensorMapSwizzle sw) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return g_noalloc_encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  };
  if (!enc(&p.tmA, A, M, K, 32, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !enc(&p.tmB, B, K, N, 128, 32, CU_TENSOR_MAP_SWIZZLE_NONE))
    return APK_ECUDA;
  p.tmAu = p.tmA;
  p.tmBu = p.tmB;
  p.C = C;
  p.ldc = N;
  p.tiles_n = N / 128;
  p.total_tiles = (M / 128) * (N / 128);
  p.nk = K / 32;
  p.poll_every = 1;
  p.wait_limit_ns = 2000000000LL;

  NoAllocHeader* h = reinterpret_cast<NoAllocHeader*>(d.scratch);
  p.ev.flag = &h->flag;
  p.ev.flag_lines = 1;
  p.ev.abort_word = &h->abort_word;
  p.ev.status = &h->status;
  p.q.next_task = &h->next_task;
  p.q.num_tasks = (unsigned long long)p.total_tiles;
  p.q.tiles_done = reinterpret_cast<unsigned long long*>(d.scratch + kNoAllocHeaderBytes);
  p.q.start_min = &h->start_min;
  p.q.end_max = &h->end_max;
  p.q.exited = &h->exited;
  p.q.yields = &h->yields;

  // what must start at zero: the queue header (the tile counters are
  // written, not accumulated); start_min starts at all-ones for atomicMin
  if (cudaMemsetAsync(d.scratch, 0, kNoAllocHeaderBytes, s) != cudaSuccess) return APK_ECUDA;
  if (cudaMemsetAsync(&h->start_min, 0xFF, sizeof(h->start_min), s) != cudaSuccess) return APK_ECUDA;
  if (launch(p, grid, POLL_OFF, DISC_DRAIN, false, GEO_L32, SCHED_QUEUE, s) != cudaSuccess) return APK_ECUDA;
  return APK_OK;
}

extern "C" apk_status apk_sgemm_f32_noalloc_status(void* stream, int* device_status) {
  using namespace apk::f32;
  if (!device_status) return APK_EINVAL;
  NoAllocDevice* d = noalloc_device();
  if (d == nullptr) return APK_ECUDA;
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return APK_ECUDA;
  const NoAllocHeader* h = reinterpret_cast<const NoAllocHeader*>(d->scratch);
  // a 4-byte copy into the caller's variable: no buffer is allocated
  if (cudaMemcpy(device_status, &h->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return APK_ECUDA;
  return APK_OK;
}

extern "C" apk_status apk_sgemm_f32_noalloc_selftest(long long limit_ns, void* stream) {
  using namespace apk;
  using namespace apk::f32;
  if (limit_ns <= 0 || limit_ns > 10000000000LL) return APK_EINVAL;
  NoAllocDevice* d = noalloc_device();
  if (d == nullptr) return APK_ECUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  NoAllocHeader* h = reinterpret_cast<NoAllocHeader*>(d->scratch);
  if (cudaMemsetAsync(d->scratch, 0, kNoAllocHeaderBytes, s) != cudaSuccess) return APK_ECUDA;
  noalloc_spin_kernel<<<1, 32, 0, s>>>(&h->never_set, limit_ns, &h->status);
  return cudaGetLastError() == cudaSuccess ? APK_OK : APK_ECUDA;
}
