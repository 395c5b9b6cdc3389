// bf16 tensor-core persistent GEMM (tcgen05 + TMEM + TMA) with tile-boundary
// and per-stage yield and an accumulator checkpoint in TMEM -> slab.
//
// Replaces the reference's wmma pipeline persistent_tc (src/tcyield.cu:91-356:
// 128x128 tile, 3-stage cp.async, wmma fragments, 8 warps that all compute
// and all take every checkpoint barrier) with a Blackwell design:
//
//   * output tile 256x256 ("wide" job: two M=128, N=256 tcgen05.mma
//     accumulators, each one 128-column half of the tile), K-tile 64,
//     3-stage TMA ring (64 KB per stage: A as two [128 rows][64 k] boxes and
//     B as four [64 k][64 n] boxes, all 128-byte swizzled; B is consumed
//     MN-major straight from the row-major [K][N] operand, no transpose).
//     A 256-wide tile moves a third fewer operand bytes from L2 into shared
//     memory per MMA than a 256x128 tile; with the ring's 192 KB unchanged
//     that took 8192^3 from 1178 to 1455 TFLOPS on one B200, bitwise equal.
//     A job whose tile ends 128 columns in (an output width that is an odd
//     multiple of 128) is "narrow": one accumulator, two B boxes.
//   * fp32 accumulators in TMEM (512 columns = two 256-column buffers).  A
//     narrow job takes one buffer and alternates, so its epilogue overlaps
//     the MMAs of the next narrow job; a wide job takes both, so its
//     epilogue (tcgen05.ld -> global stores, a few percent of a tile's
//     MMAs) runs before the next job's first MMA.
//   * warp roles: 0 producer (queue pops, TMA, urgent mini-queue pops),
//     1 MMA issuer (one thread issues tcgen05.mma / commit), 2-9 epilogue
//     (tcgen05.ld -> global; warp w may access TMEM lane quadrant w%4, so
//     two warps share each quadrant and take alternate 32-row blocks),
//     10 control (polls the yield flag, runs the device setter).  No
//     block-wide barrier per stage: the reference's per-stage checkpoint
//     barrier pair at 1 CTA/SM cost 14% (results/summary/tc_summary.csv:8-10).
//   * yield / checkpoint: the producer sees a new generation at a stage
//     boundary c (from the control warp), pops urgent work items
//     (src/yield.cu:163-183 mini-queue); if the background tile already has
//     c > 0 stages in the ring it first emits a SUSPEND control slot.  The
//     MMA warp consumes the in-flight stages in order (the "drain": TMA
//     stages are never cancelled), then on SUSPEND commits the accumulator
//     and the epilogue spills it with tcgen05.ld to the checkpoint slab.  The
//     urgent items flow through the same ring into the other TMEM buffer.
//     The background stage c is re-issued with a RESUME tag: the epilogue
//     restores the slab into a TMEM buffer with tcgen05.st and the MMAs
//     continue with accumulate=1 -- the same MMA sequence as an
//     uninterrupted run, so the resumed tile is bitwise identical.
//   * every mbarrier wait is bounded; a timeout raises a CTA abort flag and
//     the device status word, every role unwinds, outstanding MMAs and TMA
//     loads are waited for (bounded) and TMEM is freed before exit.
//   * geometries (class BG below): STD is everything above; the N
//     geometries serve 2, 4 and 8 resident CTAs per SM (the scaling
//     surface's cells): narrow jobs only (BM x 128 output tiles, one MMA of
//     M = 128, N = BM per 16-deep k-step), one TMEM buffer of BM columns
//     (256 / 128 / 64: the SM's 512 columns shared by 2 / 4 / 8 CTAs) and
//     four epilogue warps, one per TMEM lane quadrant.  The CTAs sharing an
//     SM overlap each other's epilogues with their MMAs.
#include <algorithm>
#include <string>

#include "../../include/apk.h"
#include "common.cuh"
#include "proto.h"
#include "tcgen05.cuh"

namespace apk {
namespace bf16 {

constexpr int BNH = 128;                         // columns of one accumulator (a narrow job)
constexpr int RING = 8;                          // epilogue job ring
constexpr int RASTER_GROUP = 8;                  // tile-rows per raster group
constexpr int S_MAX = 7;

// Kernel geometry.  BM: output tile rows (the MMA's N: one M=128, N=BM
// instruction per 128-column half and 16-deep k-step); NBUF: TMEM buffers of
// BM columns (STD: two, a wide 256x256 job takes both); EPI: epilogue warps;
// BK: K depth of a ring slot; S: slots; MINB: resident CTAs per SM; LDX:
// TMEM columns per epilogue load (x8 where registers are scarce).
//
// The TMA ring for a K-tile of BK (64 or 32): A as [<=128 rows][BK k] boxes
// (K-major: 128-byte swizzle for BK 64, 64-byte for BK 32, one row = one
// swizzle span) and B as [BK k][64 n] boxes (MN-major, 128-byte swizzle),
// four for a wide job, two for a narrow one.
template <int BM_, int NBUF_, int EPI_, int BK_, int S_, int MINB_, int LDX_>
struct BG {
  static constexpr int BM = BM_, NBUF = NBUF_, EPI = EPI_, BK = BK_, S = S_, MINB = MINB_, LDX = LDX_;
  static constexpr bool WIDE = NBUF == 2;        // 256-wide jobs (STD)
  static constexpr int BN = WIDE ? 256 : BNH;    // output tile columns
  static constexpr int CTRL_WARP = 2 + EPI;
  static constexpr int NT = 32 * (CTRL_WARP + 1);
  static constexpr int TMEM_COLS = NBUF * BM;
  static constexpr int BPH = BM / 32;            // 32-row epilogue blocks per 128-column half
  static constexpr int A_BOX_ROWS = BM < 128 ? BM : 128;
  static constexpr int A_HALF = A_BOX_ROWS * BK * 2;       // one A box
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_CHUNK = BK * 64 * 2;               // one [BK k][64 n] box
  static constexpr int B_BYTES = (WIDE ? 4 : 2) * B_CHUNK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // a narrow STD job loads A + 2 chunks
  static constexpr int SMEM_BYTES = S * STAGE_BYTES + 1024;
  static constexpr uint32_t A_LAYOUT = BK == 64 ? tc::LAYOUT_SW128 : tc::LAYOUT_SW64;
  static constexpr uint32_t A_SBO = BK * 2 * 8;  // 8 rows of one swizzle span
  static_assert(S <= S_MAX && BM % 64 == 0 && (EPI == 8 || EPI == 4) && (LDX == 32 || LDX == 8), "geometry");
};
// STD: the configs[2] / configs[4] kernel, one CTA per SM
using BgStd64 = BG<256, 2, 8, 64, 3, 1, 32>;
using BgStd32 = BG<256, 2, 8, 32, 7, 1, 32>;
// multi-CTA geometries: 2 CTAs (256x128 tiles, 96 KB), 4 (128x128, 48 KB),
// 8 (64x128, 24 KB); 224 threads x 4 or x 8 leave 72 or 32 registers a
// thread, so those two load TMEM eight columns at a time
using BgN256x64 = BG<256, 1, 4, 64, 2, 2, 32>;
using BgN256x32 = BG<256, 1, 4, 32, 4, 2, 32>;
using BgN128 = BG<128, 1, 4, 32, 3, 4, 8>;
using BgN64 = BG<64, 1, 4, 32, 2, 8, 8>;

// Each 128-column half of the C tile is computed transposed, D = C_half^T
// (128 x BM): the MMA's A operand is the half's [BK k][128 n] B columns
// (MN-major), its B operand the [BM m][BK k] A tile (K-major).  One M=128,
// N=256 instruction per half and 16-deep k-step reads 12 KB of shared memory
// per 2^19 MACs where two M=128, N=128 instructions (one per 128-row half)
// would read 16 KB.
template <class G>
__host__ __device__ constexpr uint32_t idesc() {
  return tc::idesc_bf16_f32(128, G::BM, /*A MN-major*/ true, /*B MN-major*/ false);
}
// A task tile with only 128 valid rows (m an odd multiple of 128) multiplies
// just those: N = 128, one A box per stage (9.5% of configs[4]'s MMA work
// went to rows no one stores).
constexpr uint32_t IDESC_HALF = tc::idesc_bf16_f32(128, 128, true, false);

enum : int { T_BG = 1, T_URG = 2, T_SUSPEND = 3, T_STOP = 4 };
enum : int { F_FIRST = 1, F_LAST = 2, F_RESUME = 4, F_WIDE = 8, F_HALF = 16 };
enum : int { E_STORE_C = 1, E_STORE_U = 2, E_SPILL = 3, E_RESTORE = 4, E_EXIT = 5 };

struct StageTag {
  int kind, flags, row0, col0, e, item;
  unsigned long long task;
};
struct EpiJob {
  int action, buf, wide, row0, col0, e, item;
  unsigned long long task;
};

template <int EPI>
struct __align__(16) Shared {
  StageTag tag[S_MAX];
  EpiJob epi[RING];
  uint64_t full[S_MAX], empty[S_MAX];
  uint64_t tfull[2], tempty[2], tres[2];
  uint64_t efull[RING], eempty[RING];
  uint64_t drain;
  // cluster launch control: the answer of the one request kept in flight,
  // its barrier, and this CTA's resident slot (the index of its logs,
  // counters and slab); under the queue scheduler slot = blockIdx.x
  uint4 clc_resp;
  uint64_t clc_bar;
  int slot;
  uint32_t tmem_base;
  int abort;      // CTA-local: some role's bounded wait gave up
  int gen;        // latest yield-flag value seen by the control warp (-1 stop)
  int prod_done;  // producer finished: the control warp may exit
  int consumed;   // stages consumed by the MMA warp (for the in-flight log)
  int epi_cnt[RING];
  double chk_part[RING][2][EPI];  // per-warp sum(c^2) of each 256x128 half of a task tile
  unsigned long long tiles;
};

__device__ __forceinline__ int vload(const int* p) { return *reinterpret_cast<const volatile int*>(p); }
__device__ __forceinline__ void vstore(int* p, int v) { *reinterpret_cast<volatile int*>(p) = v; }

// Bounded mbarrier wait that also gives up when another role aborted.
template <class SH>
__device__ __noinline__ bool bwait(uint64_t* bar, uint32_t parity, const F32Params& p, SH& sh) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = globaltimer_ns();
  int n = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (++n == 64) {
      n = 0;
      if (vload(&sh.abort)) return false;
      if (globaltimer_ns() - t0 > p.wait_limit_ns) {
        vstore(&sh.abort, 1);
        report_status(p.ev.status, DEV_WAIT_TIMEOUT_FULL, p.ev.abort_word);
        return false;
      }
    }
  }
}

// Wait without the abort shortcut (used while unwinding: outstanding async
// work must complete before smem / TMEM are released).
__device__ __noinline__ void bwait_unwind(uint64_t* bar, uint32_t parity, long long limit) {
  const long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > limit) return;
}

// Work distribution: SCH_QUEUE = persistent grid popping the global fetch-add
// counter; SCH_CLC = one CTA per task, each running CTA taking
// not-yet-launched CTAs' tasks with cluster launch control (one request in
// flight, issued one tile ahead); when the hardware declines a request (a
// higher-priority stream's kernel waits for SMs) the CTA exits at its next
// tile boundary and frees its SM.
enum : int { SCH_QUEUE = 0, SCH_CLC = 1 };
constexpr unsigned long long NO_TASK = ~0ull;

template <int POLL, int DISC, bool ORACLE, class G, int SCHED = SCH_QUEUE>
__global__ void __launch_bounds__(G::NT, G::MINB) gemm_bf16_persistent(const __grid_constant__ F32Params p) {
  constexpr bool CLC = SCHED == SCH_CLC;
  using R = G;
  constexpr int S = G::S, A_HALF = G::A_HALF, A_BYTES = G::A_BYTES, B_CHUNK = G::B_CHUNK, BK = G::BK;
  constexpr int STAGE_BYTES = G::STAGE_BYTES, BM = G::BM, BN = G::BN, EPI_WARPS = G::EPI;
  constexpr int CTRL_WARP = G::CTRL_WARP, BPH = G::BPH;
  constexpr uint32_t IDESC = idesc<G>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Shared<G::EPI> sh;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    if constexpr (CLC) {
      mbar_init(&sh.clc_bar, 1);
      sh.slot = slot_claim(p.q.slot_bits, p.q.nslots, p.wait_limit_ns);
    } else {
      sh.slot = (int)blockIdx.x;
    }
    for (int s = 0; s < S; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int b = 0; b < G::NBUF; ++b) {
      mbar_init(&sh.tfull[b], 1);
      mbar_init(&sh.tempty[b], EPI_WARPS);
      mbar_init(&sh.tres[b], EPI_WARPS);
    }
    for (int r = 0; r < RING; ++r) {
      mbar_init(&sh.efull[r], 1);
      mbar_init(&sh.eempty[r], EPI_WARPS);
      sh.epi_cnt[r] = 0;
    }
    mbar_init(&sh.drain, 1);
    fence_mbar_init();
    sh.abort = 0;
    sh.gen = 0;
    sh.prod_done = 0;
    sh.consumed = 0;
    sh.tiles = 0;
    tma_prefetch_desc(&p.tmA);
    tma_prefetch_desc(&p.tmB);
    tma_prefetch_desc(&p.tmAu);
    tma_prefetch_desc(&p.tmBu);
    tma_prefetch_desc(&p.tmAw);
    tma_prefetch_desc(&p.tmBw);
    atomicMin(p.q.start_min, (unsigned long long)globaltimer_ns());
  }
  if (warp == 1) {
    tc::tmem_alloc(&sh.tmem_base, G::TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  // per-CTA logs, counters and the slab are indexed by the resident slot
  const int cta = sh.slot;
  const int gridw = CLC ? p.q.nslots : (int)gridDim.x;

  if (warp == 0 && lane == 0) {
    // ================================ producer ================================
    uint32_t P = 0;
    int lastSeen = 0;
    bool ok = true;
    // One ring slot.  The tag (row0, col0 = output origin of the job; e, item,
    // task = epilogue bookkeeping) travels with the data; the A rows from ar0
    // and B columns from bc0 (256 of them, 128 for a narrow job) are loaded at
    // k offsets ak / bk.
    auto emit = [&](int kind, int flags, int row0, int col0, int e, int item, unsigned long long task,
                    const CUtensorMap* tA, const CUtensorMap* tB, int ar0, int bc0, int ak, int bk) -> bool {
      const int s = P % S;
      if (!bwait(&sh.empty[s], ((P / S) & 1) ^ 1, p, sh)) return false;
      StageTag& t = sh.tag[s];
      t.kind = kind;
      t.flags = flags;
      t.row0 = row0;
      t.col0 = col0;
      t.e = e;
      t.item = item;
      t.task = task;
      if (tA != nullptr) {
        const int nb_chunks = (flags & F_WIDE) ? 4 : 2;
        const bool half = (flags & F_HALF) != 0;
        mbar_arrive_expect_tx(&sh.full[s], (half ? A_HALF : A_BYTES) + nb_chunks * B_CHUNK);
        uint8_t* st = stages + s * STAGE_BYTES;
        // background jobs load A and the job's B chunks as one box each (the
        // per-box maps serve urgent items, half-row and narrow STD jobs)
        const bool bg = tA == &p.tmA;
        if (bg && !half) {
          tma_load_2d(st, &p.tmAw, ak, ar0, &sh.full[s]);
        } else {
          tma_load_2d(st, tA, ak, ar0, &sh.full[s]);
          if (BM > 128 && !half) tma_load_2d(st + A_HALF, tA, ak, ar0 + 128, &sh.full[s]);
        }
        if (bg && nb_chunks == (G::WIDE ? 4 : 2)) {
          tma_load_3d(st + A_BYTES, &p.tmBw, 0, bk, bc0 / 64, &sh.full[s]);
        } else {
          for (int b = 0; b < nb_chunks; ++b)
            tma_load_2d(st + A_BYTES + b * B_CHUNK, tB, bc0 + 64 * b, bk, &sh.full[s]);
        }
      } else {
        mbar_arrive(&sh.full[s]);  // control slot: no data
      }
      ++P;
      return true;
    };
    // Observe generation f at a poll site and pop urgent work items; a
    // SUSPEND slot precedes the first item when the background tile has
    // stages in the ring.  Returns items popped, or -1 when aborting.
    auto handle = [&](int f, int site, bool partial) -> int {
      const int fc = f < p.ev.max_events ? f : p.ev.max_events;
      const long long g = globaltimer_ns();
      for (int e = lastSeen; e < fc; ++e) p.ev.obs_ns[(size_t)e * gridw + cta] = g;
      const int old = lastSeen;
      lastSeen = f;
      int n = 0;
      for (int e = old; e < fc; ++e) {
        while (true) {
          const int it = atomicAdd(&p.ev.uq_next[e], 1);
          if (it >= p.uitems) break;
          if (it == 0) {
            p.ev.claim_ns[e] = globaltimer_ns();
            p.ev.claim[e] = cta + 1;
            p.ev.claim_site[e] = site;
            p.ev.inflight[e] = (int)(P - (uint32_t)vload(&sh.consumed));
            if (p.ev.ack != nullptr) ack_host(&p.ev.ack[2 * e]);
          }
          if (n == 0 && partial) {
            if (!emit(T_SUSPEND, 0, 0, 0, 0, 0, 0, nullptr, nullptr, 0, 0, 0, 0)) return -1;
            atomicAdd(p.q.yields, 1ull);
          }
          ++n;
          const int t = it / p.usplit, ks = it % p.usplit;
          const int r0 = (t / p.utiles_n) * BM, c0 = (t % p.utiles_n) * (p.narrow_all ? BNH : BN);
          const int wide = G::WIDE && !p.narrow_all && c0 + BN <= p.ldcu ? F_WIDE : 0;
          for (int c = 0; c < p.unk; ++c) {
            const int kk = (ks * p.unk + c) * BK;
            if (!emit(T_URG, (c == 0 ? F_FIRST : 0) | (c == p.unk - 1 ? F_LAST : 0) | wide, r0, c0, e, it, 0,
                      &p.tmAu, &p.tmBu, r0, c0, kk, kk))
              return -1;
          }
        }
      }
      return n;
    };

    // the queue is popped one task ahead: the atomic's round trip overlaps
    // the current tile's stage issue instead of stalling the ring at every
    // tile boundary (a popped task is kept across a yield and run after it)
    // CLC: the task of the request answered at this boundary, asked for one
    // tile earlier (the first is this CTA's own index)
    uint32_t clc_phase = 0;
    bool clc_inflight = false;
    auto clc_issue = [&]() {
      mbar_arrive_expect_tx(&sh.clc_bar, 16);
      clc_try_cancel(&sh.clc_resp, &sh.clc_bar);
      clc_inflight = true;
    };
    auto clc_answer = [&]() -> unsigned long long {
      clc_inflight = false;
      if (!mbar_wait(&sh.clc_bar, clc_phase, p.wait_limit_ns)) {
        report_status(p.ev.status, DEV_WAIT_TIMEOUT_SPIN, p.ev.abort_word);
        return NO_TASK;
      }
      clc_phase ^= 1u;
      unsigned x = 0;
      return clc_query(&sh.clc_resp, &x) ? (unsigned long long)x : NO_TASK;
    };
    if (CLC) {
      // a CTA launched mid-run takes the generations raised before it as
      // seen: their urgent work was popped by the CTAs that observed them
      const int f0 = flag_load(p.ev.flag);
      lastSeen = f0 > 0 ? f0 : 0;
      if (cta < 0) {  // no resident slot came free (cannot happen while residency holds)
        report_status(p.ev.status, DEV_BAD_CONFIG, p.ev.abort_word);
        ok = false;
      }
    }
    unsigned long long next_task = CLC ? (unsigned long long)blockIdx.x : atomicAdd(p.q.next_task, 1ull);
    if (CLC && ok) clc_issue();
    while (ok) {
      // ---- tile boundary: take the popped background task ----
      const unsigned long long task = next_task;
      if (CLC) {
        next_task = clc_inflight ? clc_answer() : NO_TASK;
        if (next_task != NO_TASK) clc_issue();
      } else if (task < p.q.num_tasks) {
        next_task = atomicAdd(p.q.next_task, 1ull);
      }
      int f = vload(&sh.gen);
      if (f < 0 || vload(&sh.abort)) break;
      if (POLL != POLL_OFF && f != lastSeen)
        if (handle(f, -1, false) < 0) {
          ok = false;
          break;
        }
      if (task >= p.q.num_tasks) break;
      // job geometry: output origin (row0, col0), operand origins, K steps,
      // width (wide = 256 columns, else 128)
      int row0, col0, ar0, bc0, ak0, bk0, nk, mvalid, wide;
      unsigned long long tag_task = task;
      if (p.task_mode) {
        // work entry: task, tile row, first 128-column block (even) of the tile
        const unsigned w = p.work[task];
        const TaskDesc td = p.tasks[w >> 12];
        const int tm = (w >> 6) & 63, tn = w & 63;
        row0 = td.c_row0 + tm * BM;
        col0 = td.c_col0 + tn * BNH;
        ar0 = td.a_row0 + tm * BM;
        bc0 = td.b_col0 + tn * BNH;
        ak0 = td.a_k0;
        bk0 = td.b_k0;
        nk = td.k / BK;
        mvalid = (td.m - tm * BM) < BM ? (td.m - tm * BM) : BM;
        wide = G::WIDE && !(td.flags & APK_TASK_NARROW) && (tn + 2) * BNH <= td.n ? F_WIDE : 0;
        // checksum / oracle index of the tile's first 256x128 half
        tag_task = (unsigned long long)(td.chk_base + (long long)tm * (td.n / BNH) + tn);
      } else {
        const int tile = (int)(task % (unsigned long long)p.total_tiles);
        int tm, tn;
        if (p.st.order != nullptr)
          stream_tile(p.st, tile, p.tiles_n, tm, tn);
        else
          tile_coords(tile, p.total_tiles / p.tiles_n, p.tiles_n, RASTER_GROUP, tm, tn);
        row0 = ar0 = tm * BM;
        col0 = bc0 = tn * (p.narrow_all ? BNH : BN);
        ak0 = bk0 = 0;
        nk = p.nk;
        mvalid = BM;
        wide = G::WIDE && !p.narrow_all && col0 + BN <= p.ldc ? F_WIDE : 0;
        // streamed operands: the A row panel and the B column panel(s) of
        // the tile must have landed before its first TMA load
        if (p.st.a_ready != nullptr) {
          const int* ar = &p.st.a_ready[tm / p.st.panel_tm];
          const int u = col0 / BNH;
          if (!wait_ready2(ar, &p.st.b_ready[u / p.st.b_units], p.wait_limit_ns) ||
              (wide && !wait_ready2(ar, &p.st.b_ready[(u + 1) / p.st.b_units], p.wait_limit_ns))) {
            vstore(&sh.abort, 1);
            report_status(p.ev.status, DEV_WAIT_TIMEOUT_SPIN, p.ev.abort_word);
            ok = false;
            break;
          }
        }
      }
      // a yield site every poll_every ring slots (one K-tile), counted down
      // rather than by a modulo with a run-time divisor on every slot.  The
      // producer is the critical path of the small tiles and of K-tile 32:
      // the issue loop only tests the site and leaves it when the
      // generation moved; the yield itself is handled outside it (inlined
      // inside, it cost 8-20% of the drain when nothing was raised)
      bool resume = false, skip = false;
      int to_site = 0, c = 0;
      const int fl0 = wide | (BM == 256 && mvalid <= BNH ? F_HALF : 0);
      while (ok && c < nk) {
        int fs = 0;
        bool hit = false;
        for (; c < nk; ++c) {
          const bool site = to_site == 0;
          to_site = site ? p.poll_every - 1 : to_site - 1;
          if (POLL == POLL_STAGE && site && !skip) {
            fs = vload(&sh.gen);
            if (__builtin_expect(fs != lastSeen, 0)) {
              hit = true;
              break;
            }
          }
          skip = false;
          const int flags = (c == 0 ? F_FIRST : 0) | (c == nk - 1 ? F_LAST : 0) | (resume ? F_RESUME : 0) | fl0;
          resume = false;
          // e carries the valid rows of the tile, task the oracle / checksum index
          if (!emit(T_BG, flags, row0, col0, mvalid, 0, tag_task, &p.tmA, &p.tmB, ar0, bc0, ak0 + c * BK,
                    bk0 + c * BK)) {
            ok = false;
            break;
          }
        }
        if (!hit) break;
        if (fs < 0) {
          ok = false;  // stop sentinel: abandon the tile
          break;
        }
        const int n = handle(fs, c, c > 0);
        if (n < 0) {
          ok = false;
          break;
        }
        resume = n > 0 && c > 0;
        // stage c is issued next without testing its site again: its
        // generation has just been handled
        to_site = 0;
        skip = true;
      }
    }
    emit(T_STOP, 0, 0, 0, 0, 0, 0, nullptr, nullptr, 0, 0, 0, 0);
    // a CLC answer still in flight (a stopped or aborted run) lands before
    // shared memory goes away; a task it took is dropped with the run
    if (CLC && clc_inflight) mbar_wait(&sh.clc_bar, clc_phase, p.wait_limit_ns);
    vstore(&sh.prod_done, 1);
    // TMA loads still in flight (only when unwinding) must land before exit.
    // Only the last S stages can be: an older one's slot was reused, so its
    // loads landed and its barrier has moved on; waiting on its parity could
    // match a later phase that never comes.  (The consumer publishes
    // `consumed` late -- after posting an epilogue job -- so it may lag P by
    // a whole ring.)
    for (uint32_t q = max((uint32_t)vload(&sh.consumed), P >= (uint32_t)S ? P - S : 0u); q < P; ++q)
      bwait_unwind(&sh.full[q % S], (q / S) & 1, p.wait_limit_ns);
  } else if (warp == 1 && lane == 0) {
    // ================================== MMA ===================================
    // TMEM buffer use: ub[b] counts the jobs that took buffer b (the
    // epilogue frees it with one tempty phase per job), rb[b] the restores
    // into it.  cur / cwide: buffer and width of the job being fed.
    // parked: the buffer holding a suspended narrow background job's
    // accumulator (park mode), -1 when none; while one is parked every other
    // job takes the other buffer.
    uint32_t Q = 0, X = 0, ub[2] = {0, 0}, rb[2] = {0, 0};
    int nb = 0, cur = 0, cwide = 0, parked = -1;
    const uint32_t tbase = sh.tmem_base;
    auto post = [&](int action, int buf, int wide, const StageTag& t) -> bool {
      const int sl = X % RING;
      if (!bwait(&sh.eempty[sl], ((X / RING) & 1) ^ 1, p, sh)) return false;
      EpiJob& j = sh.epi[sl];
      j.action = action;
      j.buf = buf;
      j.wide = wide;
      j.row0 = t.row0;
      j.col0 = t.col0;
      j.e = t.e;
      j.item = t.item;
      j.task = t.task;
      mbar_arrive(&sh.efull[sl]);
      ++X;
      return true;
    };
    while (true) {
      const int s = Q % S;
      if (!bwait(&sh.full[s], (Q / S) & 1, p, sh)) break;
      const StageTag t = sh.tag[s];
      if (t.kind == T_STOP) {
        post(E_EXIT, 0, 0, t);
        break;
      }
      if (t.kind == T_SUSPEND) {
        if (G::NBUF == 2 && p.park && !cwide) {
          // park: the accumulator stays in its buffer, nothing is spilled;
          // the stages consumed so far have all been committed in order, so
          // the resumed MMAs continue the same sequence
          parked = cur;
          nb = cur ^ 1;
          if (p.q.ckpt != nullptr) atomicAdd(&p.q.ckpt[4], 1ull);
        } else {
          if (!post(E_SPILL, cur, cwide, t)) break;
          tc::commit(&sh.tfull[cur]);
        }
        mbar_arrive(&sh.empty[s]);
        ++Q;
        vstore(&sh.consumed, (int)Q);
        continue;
      }
      if (G::NBUF == 2 && (t.flags & F_RESUME) && parked >= 0) {
        // resume the parked job in place: no buffer to take, nothing to restore
        cur = parked;
        cwide = 0;
        parked = -1;
        nb = cur ^ 1;
      } else if (t.flags & (F_FIRST | F_RESUME)) {
        // a narrow job takes the next buffer, a wide one both
        cwide = (G::WIDE && (t.flags & F_WIDE)) ? 1 : 0;
        cur = cwide ? 0 : nb;
        nb = (cwide || G::NBUF == 1 || parked >= 0) ? (parked >= 0 ? parked ^ 1 : 0) : nb ^ 1;
        bool ok = true;
        for (int b = cur; b <= (cwide ? 1 : cur) && ok; ++b) {
          ok = bwait(&sh.tempty[b], (ub[b] & 1) ^ 1, p, sh);
          ++ub[b];
        }
        if (!ok) break;
        tc::fence_after_sync();
        if (t.flags & F_RESUME) {
          if (!post(E_RESTORE, cur, cwide, t)) break;
          if (!bwait(&sh.tres[cur], rb[cur] & 1, p, sh)) break;
          ++rb[cur];
          tc::fence_after_sync();
        }
      }
      uint8_t* st = stages + s * STAGE_BYTES;
      if (DISC == DISC_POISON && t.kind == T_URG && (t.flags & F_FIRST)) {
        // detector control: one wrong staged B value (8.0) in each urgent item
        reinterpret_cast<uint16_t*>(st + A_BYTES)[0] = 0x4100;
        fence_proxy_async_smem();
      }
      const uint32_t sa = smem_u32(st), sb = smem_u32(st + A_BYTES);
      const uint32_t d0 = tbase + (uint32_t)cur * BM;
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        // MMA A = B tile rows kk*16.. (MN-major: 64-column chunks LBO apart,
        // 8-row groups SBO apart); MMA B = A tile, K-major, 32 B per k-step
        // inside the 128-byte swizzled rows, 8-row groups 1024 B apart.  The
        // second half of a wide tile reads B chunks 2-3 into buffer 1.
        const uint32_t acc = (kk > 0 || !(t.flags & F_FIRST)) ? 1u : 0u;
        const uint64_t bdesc = tc::smem_desc(sa + kk * 32, 16, R::A_SBO, R::A_LAYOUT);
        const uint32_t idesc = (t.flags & F_HALF) ? IDESC_HALF : IDESC;
        tc::mma_bf16(d0, tc::smem_desc(sb + kk * 2048, B_CHUNK, 1024, tc::LAYOUT_SW128), bdesc, idesc, acc);
        if (G::WIDE && cwide)
          tc::mma_bf16(d0 + BM, tc::smem_desc(sb + 2 * B_CHUNK + kk * 2048, B_CHUNK, 1024, tc::LAYOUT_SW128),
                       bdesc, idesc, acc);
      }
      tc::commit(&sh.empty[s]);  // frees the slot once these MMAs have read it
      if (t.flags & F_LAST) {
        if (!post(t.kind == T_BG ? E_STORE_C : E_STORE_U, cur, cwide, t)) break;
        tc::commit(&sh.tfull[cur]);
      }
      ++Q;
      vstore(&sh.consumed, (int)Q);
    }
    // no tcgen05.mma may still run when TMEM is released
    tc::commit(&sh.drain);
    bwait_unwind(&sh.drain, 0, p.wait_limit_ns);
  } else if (warp >= 2 && warp < CTRL_WARP) {
    // ================================ epilogue ================================
    // A 32-row block (32 TMEM columns of one quadrant) moves as 32 / LDX
    // units of LDX columns; with 8 epilogue warps the quadrant's two warps
    // take alternate blocks (GS = 2), with 4 one warp takes them all.
    constexpr int LDX = G::LDX, UPB = 32 / LDX, GS = EPI_WARPS / 4;
    const int q = warp & 3;          // TMEM lane quadrant this warp may access
    const int g = (warp - 2) >> 2;   // which of the quadrant's warps: blocks g, g + GS, ...
    const int ew = (warp - 2);       // epilogue warp index (checksum slot)
    uint32_t Y = 0, eb[2] = {0, 0};
    const uint32_t tbase = sh.tmem_base;
    float* slab = p.slab + (size_t)cta * (BM * BN);
    while (true) {
      const int sl = Y % RING;
      if (!bwait(&sh.efull[sl], (Y / RING) & 1, p, sh)) break;
      const EpiJob j = sh.epi[sl];
      if (j.action == E_EXIT) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.eempty[sl]);
        break;
      }
      // TMEM holds each 128-column half of the tile transposed: lane = C
      // column (32q + lane of this warp's quadrant, plus 128 in the second
      // half), column = C row.  Block bb = (hh, blk) covers C rows blk*32 ..
      // blk*32+31 of half hh, one register per row; a wide job's second half
      // sits in the next BM TMEM columns.
      const uint32_t tcol = tbase + ((uint32_t)(32 * q) << 16) + (uint32_t)j.buf * BM;
      const int nh = j.wide ? 2 : 1;
      const int lim = BPH * nh;  // blocks of the job
      auto slab_blk = [&](int hh, int blk) { return slab + (size_t)((hh * BPH + blk) * 4 + q) * 1024; };
      // unit u = block * UPB + sub: TMEM columns blk*32 + sub*LDX .. + LDX of half hh
      auto ucol = [&](int u) {
        const int bb = u / UPB;
        return tcol + (uint32_t)((bb / BPH) * BM + (bb % BPH) * 32 + (u % UPB) * LDX);
      };
      if (j.action == E_RESTORE) {
        const long long r0 = globaltimer_ns();
#pragma unroll 1
        for (int bb = g; bb < lim; bb += GS) {
#pragma unroll 1
          for (int sub = 0; sub < UPB; ++sub) {
            const float4* s4 = reinterpret_cast<const float4*>(slab_blk(bb / BPH, bb % BPH));
            uint32_t v[LDX];
#pragma unroll
            for (int i = 0; i < LDX / 4; ++i) {
              const float4 x = s4[(sub * (LDX / 4) + i) * 32 + lane];
              v[4 * i] = __float_as_uint(x.x);
              v[4 * i + 1] = __float_as_uint(x.y);
              v[4 * i + 2] = __float_as_uint(x.z);
              v[4 * i + 3] = __float_as_uint(x.w);
            }
            tc::st_32x32b<LDX>(ucol(bb * UPB + sub), v);
          }
        }
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sh.tres[j.buf]);
          if (p.q.ckpt != nullptr) {
            // this warp moved lim / GS blocks of 32 x 32 floats from the slab
            atomicAdd(&p.q.ckpt[2], (unsigned long long)(globaltimer_ns() - r0));
            atomicAdd(&p.q.ckpt[3], (unsigned long long)(lim / GS) * 4096);
          }
        }
      } else {
        if (!bwait(&sh.tfull[j.buf], eb[j.buf] & 1, p, sh)) break;
        ++eb[j.buf];
        tc::fence_after_sync();
        const long long s0 = globaltimer_ns();
        // task mode: this lane's sum(c^2) per half in a fixed order; fp32 per
        // lane (256 terms, ~1e-6 relative) keeps the double conversions off
        // the path that frees TMEM, the lanes and warps add up in double
        float csum[2] = {0.0f, 0.0f};
        // This warp's blocks bb = g, g+GS, ... (< lim); rows past the task's
        // m (a 128-row task in a 256-row tile) are neither stored nor summed.
        // Software-pipelined: the next unit's tcgen05.ld is issued before
        // the current unit's stores, and TMEM is released as soon as the
        // last unit is in registers, before its stores.
        constexpr int ULIM = 1 << 30;
        auto valid = [&](int bb) { return !(j.action == E_STORE_C && (bb % BPH) * 32 >= j.e); };
        auto next = [&](int u) {
          if (u % UPB != UPB - 1) return u + 1;
          int bb = u / UPB + GS;
          while (bb < lim && !valid(bb)) bb += GS;
          return bb < lim ? bb * UPB : ULIM;
        };
        auto consume = [&](int u, const uint32_t(&v)[LDX]) {
          const int bb = u / UPB, sub = u % UPB, hh = bb / BPH, blk = bb % BPH;
          if (j.action == E_SPILL) {
            float4* s4 = reinterpret_cast<float4*>(slab_blk(hh, blk));
#pragma unroll
            for (int i = 0; i < LDX / 4; ++i)
              s4[(sub * (LDX / 4) + i) * 32 + lane] =
                  make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                              __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
            return;
          }
          // register i -> C row blk*32 + sub*LDX + i, lane -> C column: each
          // store instruction writes one contiguous 128-byte row segment
          const int col = j.col0 + BNH * hh + 32 * q + lane;
          const int row = j.row0 + blk * 32 + sub * LDX;
          if (j.action == E_STORE_C) {
            float* dst = p.C + (size_t)row * p.ldc + col;
#pragma unroll
            for (int i = 0; i < LDX; ++i) dst[(size_t)i * p.ldc] = __uint_as_float(v[i]);
            if (p.task_mode) {
              // one running sum per half, blocks in order, rows in order
              float cs = hh == 0 ? csum[0] : csum[1];
#pragma unroll
              for (int i = 0; i < LDX; ++i) {
                const float x = __uint_as_float(v[i]);
                cs = fmaf(x, x, cs);
              }
              if (hh == 0) csum[0] = cs; else csum[1] = cs;
            }
          } else {
            float* dst = p.Cu + (size_t)j.e * p.cu_stride + (size_t)row * p.ldcu + col;
            if (p.usplit == 1) {
#pragma unroll
              for (int i = 0; i < LDX; ++i) dst[(size_t)i * p.ldcu] = __uint_as_float(v[i]);
            } else {
#pragma unroll
              for (int i = 0; i < LDX; ++i) atomicAdd(dst + (size_t)i * p.ldcu, __uint_as_float(v[i]));
            }
          }
        };
        bool released = false;
        auto release = [&]() {  // every tcgen05.ld of this warp has completed
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&sh.tempty[j.buf]);
            if (j.wide) mbar_arrive(&sh.tempty[1]);  // a wide job held both buffers (buf 0 and 1)
            if (j.action == E_SPILL && p.q.ckpt != nullptr) {
              // TMEM free again: this warp's lim / GS blocks are in registers
              atomicAdd(&p.q.ckpt[0], (unsigned long long)(globaltimer_ns() - s0));
              atomicAdd(&p.q.ckpt[1], (unsigned long long)(lim / GS) * 4096);
            }
          }
          released = true;
        };
        uint32_t va[LDX], vb[LDX];
        int bb0 = g;
        while (bb0 < lim && !valid(bb0)) bb0 += GS;
        int cur = bb0 < lim ? bb0 * UPB : ULIM;
        if (cur != ULIM) tc::ld_32x32b<LDX>(ucol(cur), va);
        while (cur != ULIM) {
          tc::wait_ld();
          int nxt = next(cur);
          if (nxt != ULIM) tc::ld_32x32b<LDX>(ucol(nxt), vb); else release();
          consume(cur, va);
          cur = nxt;
          if (cur == ULIM) break;
          tc::wait_ld();
          nxt = next(cur);
          if (nxt != ULIM) tc::ld_32x32b<LDX>(ucol(nxt), va); else release();
          consume(cur, vb);
          cur = nxt;
        }
        if (!released) release();  // no block of this warp had valid rows
        if (j.action != E_SPILL) {
          if (p.task_mode && j.action == E_STORE_C) {
            for (int hh = 0; hh < nh; ++hh) {
              double s = (double)csum[hh];
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
              if (lane == 0) sh.chk_part[sl][hh][ew] = s;
            }
          }
          // the tile's stores are complete and visible before it is counted;
          // the last of the epilogue warps to finish does the accounting
          __threadfence();
          __syncwarp();
          if (lane == 0 && atomicAdd(&sh.epi_cnt[sl], 1) == EPI_WARPS - 1) {
            sh.epi_cnt[sl] = 0;
            if (j.action == E_STORE_C) {
              if (p.task_mode) {
                // task mode counts and checksums each 256x128 half; the
                // partial sums are added in a fixed order
                for (int hh = 0; hh < nh; ++hh) {
                  ++sh.tiles;
                  if (ORACLE && p.q.exec_count != nullptr) atomicAdd(&p.q.exec_count[j.task + hh], 1);
                  double s = 0.0;
                  for (int w = 0; w < EPI_WARPS; ++w) s += sh.chk_part[sl][hh][w];
                  p.chk[j.task + hh] = s;
                }
              } else {
                ++sh.tiles;
                if (ORACLE && p.q.exec_count != nullptr) atomicAdd(&p.q.exec_count[j.task], 1);
                if (p.st.done != nullptr)  // every warp fenced its stores above
                  stream_tile_done(p.st, p.total_tiles / p.tiles_n, p.tiles_n, j.row0 / BM,
                                   j.col0 / (p.narrow_all ? BNH : BN));
              }
              count_trigger(p.ev);
            } else {
              if (ORACLE) atomicAdd(&p.ev.uexec[j.e], 1);
              atomicMax(&p.ev.done_ns[j.e], (unsigned long long)globaltimer_ns());
              const int done = atomicAdd(&p.ev.udone_cnt[j.e], 1) + 1;
              if (done == p.uitems && p.ev.ack != nullptr) ack_host(&p.ev.ack[2 * j.e + 1]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.eempty[sl]);
      ++Y;
    }
  } else if (warp == CTRL_WARP && lane == 0) {
    // ================================ control =================================
    // device setter: the CTA in slot 0 (under CLC its state passes from one
    // slot-0 holder to the next)
    int nextEv = 0;
    long long gBase = 0;
    if (CLC && cta == 0 && p.q.setter_state != nullptr) {
      nextEv = (int)p.q.setter_state[0];
      gBase = p.q.setter_state[1];
    }
    // one poller per CTA: with c CTAs per SM each polls every 64*c ns, so an
    // SM loads the flag at the same rate whatever c is (8 CTAs per SM polling
    // every 64 ns each cost a third of the drain: 1184 pollers on one line)
    unsigned nsm;
    asm volatile("mov.u32 %0, %%nsmid;" : "=r"(nsm));
    const int per_sm = nsm > 0 && gridw > (int)nsm ? gridw / (int)nsm : 1;
    const unsigned sleep_ns = 64u * (unsigned)per_sm;
    const int* flag = flag_copy(p.ev, cta);
    // the abort word is one line every CTA reads: every 16th pass (a stop
    // also writes -1 into every flag copy); once seen it holds
    unsigned pass = 0;
    bool aborted = false;
    while (!vload(&sh.prod_done) && !vload(&sh.abort)) {
      int f = POLL != POLL_OFF ? flag_load(flag) : 0;
      if ((++pass & 15) == 0 && *reinterpret_cast<volatile int*>(p.ev.abort_word)) aborted = true;
      if (aborted) f = -1;
      if (cta == 0 && p.ev.sched_ns != nullptr && nextEv < p.ev.n_sched) {
        const long long now = globaltimer_ns();
        if (gBase == 0) gBase = now;
        if (now >= gBase + p.ev.sched_ns[nextEv]) {
          p.ev.set_ns[nextEv] = now;
          flag_raise(p.ev, nextEv);
          ++nextEv;
        }
      }
      vstore(&sh.gen, f);
      __nanosleep(sleep_ns);
    }
    if (CLC && cta == 0 && p.q.setter_state != nullptr) {
      p.q.setter_state[0] = nextEv;
      p.q.setter_state[1] = gBase;
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(sh.tmem_base, G::TMEM_COLS);
  }
  if (tid == 0) {
    if (CLC) {
      if (cta >= 0) atomicAdd(&p.q.tiles_done[cta], sh.tiles);
    } else {
      p.q.tiles_done[cta] = sh.tiles;
    }
    atomicMax(p.q.end_max, (unsigned long long)globaltimer_ns());
    atomicAdd(p.q.exited, 1);
    if (CLC && cta >= 0) {
      __threadfence();
      slot_release(p.q.slot_bits, cta);  // last: the slot's logs are written
    }
  }
}

// ---------------------------------------------------------------------------

template <int POLL, int DISC, bool ORACLE, class G, int SCHED = SCH_QUEUE>
static const void* kernel_ptr() {
  return reinterpret_cast<const void*>(&gemm_bf16_persistent<POLL, DISC, ORACLE, G, SCHED>);
}

// geo: BF16_GEO_* (proto.h); sched: SCH_QUEUE or SCH_CLC (the one-CTA-per-SM
// geometries, drain discipline)
static const void* select_kernel(int poll, int disc, bool oracle, int geo, int sched) {
  if (sched == SCH_CLC) {
#define APK_SEL(PL, OR)                                                                          \
  if (poll == PL && disc == DISC_DRAIN && oracle == OR) {                                       \
    if (geo == BF16_GEO_STD64) return kernel_ptr<PL, DISC_DRAIN, OR, BgStd64, SCH_CLC>();       \
    if (geo == BF16_GEO_STD32) return kernel_ptr<PL, DISC_DRAIN, OR, BgStd32, SCH_CLC>();       \
  }
    APK_SEL(POLL_OFF, false)
    APK_SEL(POLL_OFF, true)
    APK_SEL(POLL_BOUNDARY, false)
    APK_SEL(POLL_STAGE, false)
    APK_SEL(POLL_STAGE, true)
#undef APK_SEL
    return nullptr;
  }
#define APK_SEL(PL, DS, OR)                                                 \
  if (poll == PL && disc == DS && oracle == OR) {                          \
    if (geo == BF16_GEO_STD64) return kernel_ptr<PL, DS, OR, BgStd64>();   \
    if (geo == BF16_GEO_STD32) return kernel_ptr<PL, DS, OR, BgStd32>();   \
  }
  APK_SEL(POLL_OFF, DISC_DRAIN, false)
  APK_SEL(POLL_OFF, DISC_DRAIN, true)
  APK_SEL(POLL_BOUNDARY, DISC_DRAIN, false)
  APK_SEL(POLL_BOUNDARY, DISC_DRAIN, true)
  APK_SEL(POLL_STAGE, DISC_DRAIN, false)
  APK_SEL(POLL_STAGE, DISC_DRAIN, true)
  APK_SEL(POLL_STAGE, DISC_POISON, false)
  APK_SEL(POLL_STAGE, DISC_POISON, true)
#undef APK_SEL
  // the multi-CTA geometries: the variants the scaling surface and its tests use
#define APK_SEL(PL, DS, OR)                                                    \
  if (poll == PL && disc == DS && oracle == OR) {                             \
    if (geo == BF16_GEO_N256x64) return kernel_ptr<PL, DS, OR, BgN256x64>();  \
    if (geo == BF16_GEO_N256x32) return kernel_ptr<PL, DS, OR, BgN256x32>();  \
    if (geo == BF16_GEO_N128) return kernel_ptr<PL, DS, OR, BgN128>();        \
    if (geo == BF16_GEO_N64) return kernel_ptr<PL, DS, OR, BgN64>();          \
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

template <class G>
static GeoInfo info_of() {
  return GeoInfo{G::BM, G::BN, G::NT, G::BK, G::S, G::BK, G::SMEM_BYTES};
}

GeoInfo geo_info(int geo) {
  switch (geo) {
    case BF16_GEO_STD32: return info_of<BgStd32>();
    case BF16_GEO_N256x64: return info_of<BgN256x64>();
    case BF16_GEO_N256x32: return info_of<BgN256x32>();
    case BF16_GEO_N128: return info_of<BgN128>();
    case BF16_GEO_N64: return info_of<BgN64>();
    default: return info_of<BgStd64>();
  }
}
static int tmem_cols(int geo) {
  switch (geo) {
    case BF16_GEO_N256x64: case BF16_GEO_N256x32: return BgN256x64::TMEM_COLS;
    case BF16_GEO_N128: return BgN128::TMEM_COLS;
    case BF16_GEO_N64: return BgN64::TMEM_COLS;
    default: return BgStd64::TMEM_COLS;
  }
}
int epi_warps(int geo) { return geo == BF16_GEO_STD64 || geo == BF16_GEO_STD32 ? BgStd64::EPI : BgN128::EPI; }
size_t params_bytes() { return sizeof(F32Params); }

cudaError_t prepare(int poll, int disc, bool oracle, int geo, int sched, int* max_ctas_per_sm) {
  const void* k = select_kernel(poll, disc, oracle, geo, sched);
  if (!k) return cudaErrorInvalidValue;
  const GeoInfo g = geo_info(geo);
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, g.smem_bytes);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  // Residency from the kernel's own resources.  The occupancy calculator
  // answers 1 for every kernel that allocates tensor memory (on B200 with
  // driver 580 even 32 threads and no shared memory gave 1), while the
  // hardware places 2, 4 and 8 of the multi-CTA geometries on one SM: in a
  // launch of that many CTAs per SM every CTA observed a device-set event
  // within 4 us of its raise.  So the count is computed here: shared memory
  // (with the per-CTA reservation), registers (allocated per warp in units of
  // 256), threads, and the CTA's share of the SM's 512 TMEM columns (an
  // allocation beyond them would wait for another CTA's release).
  cudaFuncAttributes fa;
  if ((e = cudaFuncGetAttributes(&fa, k)) != cudaSuccess) return e;
  int dev = 0, smem_sm = 0, smem_rsv = 0, thr_sm = 0, regs_sm = 0, blk_sm = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&smem_rsv, cudaDevAttrReservedSharedMemoryPerBlock, dev)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&thr_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&blk_sm, cudaDevAttrMaxBlocksPerMultiprocessor, dev)) != cudaSuccess)
    return e;
  const int warps = (g.threads + 31) / 32;
  const int regs_per_warp = ((fa.numRegs * 32 + 255) / 256) * 256;
  const int by_smem = smem_sm / (g.smem_bytes + (int)fa.sharedSizeBytes + smem_rsv);
  const int by_regs = regs_per_warp > 0 ? regs_sm / (regs_per_warp * warps) : blk_sm;
  const int by_threads = thr_sm / g.threads;
  const int tmem_cap = 512 / tmem_cols(geo);
  *max_ctas_per_sm = std::min(std::min(std::min(by_smem, by_regs), std::min(by_threads, blk_sm)), tmem_cap);
  return cudaSuccess;
}

cudaError_t launch(const F32Params& prm, int grid, int poll, int disc, bool oracle, int geo, int sched,
                   cudaStream_t stream) {
  const void* k = select_kernel(poll, disc, oracle, geo, sched);
  if (!k) return cudaErrorInvalidValue;
  const GeoInfo g = geo_info(geo);
  void* args[] = {const_cast<F32Params*>(&prm)};
  return cudaLaunchKernel(k, dim3(grid), dim3(g.threads), args, g.smem_bytes, stream);
}

}  // namespace bf16
}  // namespace apk
