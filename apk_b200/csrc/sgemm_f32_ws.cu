// fp32 CUDA-core persistent SGEMM, warp-specialized: the default fp32 kernel
// at full residency (queue scheduler, K-tile 32).
//
// Same work, protocol and results as sgemm_f32.cu (which stays for the
// cluster-launch-control scheduler, K-tile 64, one CTA per SM and reserved
// grids); replaces the same reference routines:
//   tile_gemm            src/tile.cuh:62-107      (64x64 tile, scalar loads)
//   persistent_gemm      src/persistent.cu:51-79  (fetch-add queue)
//   persistent_yield     src/yield.cu:95-204      (boundary poll, mini-queue)
//   persistent_midyield  src/midyield.cu:92-320   (per-stage checkpoint)
//
// B200 design:
//   * One 384-thread CTA per SM holds two independent workers ("groups"),
//     each computing 128x128 output tiles from its own 3-slot TMA ring:
//     four compute warps per group (8x16 micro-tile per thread, packed
//     fma.rn.f32x2, the same k order and rounding as scalar FMAs, so C is
//     bitwise the block-synchronous kernel's), one producer warp per group
//     (queue pops, TMA issue, urgent mini-queue, yield decisions), and one
//     control warp (flag poll, device setter).  A worker is what the rest
//     of the runtime calls a CTA: grid = 2 x SMs workers, and the event log,
//     tile counters and checkpoint slabs are indexed by worker.
//   * Warpgroup 0 (producers, control) gives registers back with
//     setmaxnreg.dec, warpgroups 1-2 (compute) take them with setmaxnreg.inc:
//     128 x 56 + 256 x 224 = 384 x 168, the launch's register total.  The
//     compute warps have no control state and no block barrier: the ring is
//     guarded by a full mbarrier (TMA bytes) and an empty mbarrier (four
//     warp arrivals) per slot, so the mainloop can run the k-pair loop
//     unrolled by two.
//   * Each ring slot carries a tag (job kind, stage index, flags, output
//     origin, event, item, task) written by the producer before it arms the
//     slot; the compute warps act on the tag.  Kinds: background stage,
//     urgent stage, SUSPEND (checkpoint), STOP.
//   * Yield: the control warp publishes the flag in shared memory; a
//     producer watches it while it waits for each ring slot (POLL_STAGE) or
//     polls it at tile boundaries (POLL_BOUNDARY), logs the observation and
//     pops urgent items
//     from the event's mini-queue (src/yield.cu:163-183; the first popper is
//     the claimer).  When its background tile has stages in flight it sets
//     the group's skip request: the compute warps stop accumulating the
//     background stages still in the ring (each warp keeps the count of K
//     stages it has accumulated), and at the SUSPEND slot spill the 128x128
//     accumulators with those cursors to the worker's checkpoint slab.  The
//     urgent items run through the same ring; then the producer re-issues
//     the background tile from the smallest cursor, the first slot flagged
//     RESUME: the warps restore their accumulators and skip stages they had
//     already accumulated, so every element sees the same K order as an
//     uninterrupted run -- bitwise identical.
//   * A new background tile is issued only after every stage of the
//     previous one was consumed, so in-flight background stages always
//     belong to one tile.
//   * Tile completion: each compute warp stores its 32 rows, fences, and
//     adds one to the slot's shared counter; the fourth does the accounting
//     (tile counters, oracle counts, stream acks, urgent done acks) and only
//     then are the slot's empty arrivals complete.  No named barrier: a warp
//     that gives up on a bounded wait cannot leave the others waiting.
//   * Every wait is bounded (wait_limit_ns); a timeout sets the status and
//     abort words and every role unwinds.
#include "common.cuh"
#include "proto.h"

namespace apk {
namespace f32ws {

constexpr int BM = 128, BN = 128, BK = 32, S = 3, G = 2;
constexpr int NT = 384;
constexpr int A_BYTES = BM * BK * 4, B_BYTES = BK * BN * 4, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = G * S * STAGE_BYTES + 1024;
constexpr int PROD_REGS = 56, COMP_REGS = 224, LAUNCH_REGS = 168;
static_assert(128 * PROD_REGS + 256 * COMP_REGS <= NT * LAUNCH_REGS, "setmaxnreg split exceeds the launch's registers");

enum : int { T_BG = 1, T_URG = 2, T_SUSPEND = 3, T_STOP = 4 };
// F_CHAIN: the first stage of a K slice after the first, whose accumulators
// start from the previous slice's (streamed runs); F_HANDOFF: the last
// stage of a K slice before the last, which leaves them there.
enum : int { F_FIRST = 1, F_LAST = 2, F_RESUME = 4, F_CHAIN = 8, F_HANDOFF = 16 };

struct Tag {
  int kind, flags, c, row0, col0, e, item, pad;
  unsigned long long task;
};

struct __align__(16) GroupShared {
  Tag tag[S];
  uint64_t full[S], empty[S];
  uint64_t spilled;      // 4 compute-warp arrivals per SUSPEND
  int cnt[S];            // compute warps done with the urgent item ending in the slot
  int bg_cnt;            // compute warps done with the background tile's epilogue
  int exit_cnt;          // compute warps that left
  int cur[4];            // K stages each compute warp had accumulated at SUSPEND
  int skip;              // producer: stop accumulating background stages
  int consumed;          // stages the group's warp 0 has finished (event log)
  unsigned long long tiles;
};

struct __align__(16) Shared {
  GroupShared g[G];
  int gen;        // latest flag value seen by the control warp (-1 = stop)
  int abort;      // CTA-local: some role's bounded wait gave up
  int prod_done;  // producers finished
};

__device__ __forceinline__ int vload(const int* p) { return *reinterpret_cast<const volatile int*>(p); }
__device__ __forceinline__ void vstore(int* p, int v) { *reinterpret_cast<volatile int*>(p) = v; }

// Bounded mbarrier wait that also gives up when another role aborted.
// (Inlined: called across setmaxnreg regions, out-of-line calls made ptxas
// take minutes per instantiation.)
__device__ __forceinline__ bool bwait(uint64_t* bar, uint32_t parity, const F32Params& p, Shared& sh) {
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

// Bounded wait for a global counter to reach target (acquire), giving up
// when another role aborted.
__device__ __forceinline__ bool wait_count(const int* c, int target, const F32Params& p, Shared& sh) {
  const long long t0 = globaltimer_ns();
  while (true) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
    if (v >= target) return true;
    if (vload(&sh.abort)) return false;
    if (globaltimer_ns() - t0 > p.wait_limit_ns) {
      vstore(&sh.abort, 1);
      report_status(p.ev.status, DEV_WAIT_TIMEOUT_SPIN, p.ev.abort_word);
      return false;
    }
  }
}

__device__ __forceinline__ void bwait_unwind(uint64_t* bar, uint32_t parity, long long limit) {
  const long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > limit) return;
}

// acc[i][j] += A[r_i][k] * B[k][c_j] for the two k of k-pair kp of a 32-deep
// slot; rows r_i = arow0 + 4i, columns c_j = bcol + 32(j/4) + j%4 (the same
// tiling and order as sgemm_f32.cu's kpair).
__device__ __forceinline__ void kpair(const float* __restrict__ As, const float* __restrict__ Bs,
                                      float (&acc)[8][16], int arow0, int ty, int bcol, int kp) {
  const int kc = kp >> 1, half = kp & 1;
  float2 a[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // 128-byte swizzle: row r's 16-byte chunk kc sits at chunk kc ^ (r & 7)
    const int sw = kc ^ (ty + 4 * (i & 1));
    a[i] = *reinterpret_cast<const float2*>(As + (arow0 + 4 * i) * 32 + (sw << 2) + 2 * half);
  }
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    const float* brow = Bs + (kp * 2 + kk) * BN + bcol;
    float4 b[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) b[q] = *reinterpret_cast<const float4*>(brow + 32 * q);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float av = kk == 0 ? a[i].x : a[i].y;
      const float2 ad = make_float2(av, av);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
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

// KS: the instantiation for streamed runs with K slices (F_CHAIN /
// F_HANDOFF).  The resident instantiations carry none of that code, which
// changes how the compiler schedules the mainloop (-5% measured).
template <int POLL, int DISC, bool ORACLE, bool KS>
__global__ void __launch_bounds__(NT, 1) sgemm_ws(const __grid_constant__ F32Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring_all = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Shared sh;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nworkers = gridDim.x * G;

  if (tid == 0) {
    for (int g = 0; g < G; ++g) {
      GroupShared& gs = sh.g[g];
      for (int s = 0; s < S; ++s) {
        mbar_init(&gs.full[s], 1);
        mbar_init(&gs.empty[s], 4);
        gs.cnt[s] = 0;
      }
      mbar_init(&gs.spilled, 4);
      gs.bg_cnt = 0;
      gs.exit_cnt = 0;
      gs.skip = 0;
      gs.consumed = 0;
      gs.tiles = 0;
    }
    fence_mbar_init();
    sh.gen = 0;
    sh.abort = 0;
    sh.prod_done = 0;
    tma_prefetch_desc(&p.tmA);
    tma_prefetch_desc(&p.tmB);
    tma_prefetch_desc(&p.tmAu);
    tma_prefetch_desc(&p.tmBu);
    atomicMin(p.q.start_min, (unsigned long long)globaltimer_ns());
  }
  __syncthreads();

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(PROD_REGS));
    if (warp < G && lane == 0) {
      // ============================== producer ==============================
      const int g = warp, worker = blockIdx.x * G + g;
      GroupShared& gs = sh.g[g];
      uint8_t* ring = ring_all + g * S * STAGE_BYTES;
      uint32_t P = 0, nsusp = 0;
      int lastSeen = 0;
      bool ok = true;
      // Arm the next slot with a tag and (for data slots) its TMA loads.
      auto emit = [&](int kind, int flags, int c, int row0, int col0, int e, int item, unsigned long long task,
                      const CUtensorMap* tA, const CUtensorMap* tB, int k0) -> bool {
        const int s = P % S;
        if (!bwait(&gs.empty[s], ((P / S) & 1) ^ 1, p, sh)) return false;
        Tag& t = gs.tag[s];
        t.kind = kind;
        t.flags = flags;
        t.c = c;
        t.row0 = row0;
        t.col0 = col0;
        t.e = e;
        t.item = item;
        t.task = task;
        if (tA != nullptr) {
          mbar_arrive_expect_tx(&gs.full[s], STAGE_BYTES);
          uint8_t* st = ring + s * A_BYTES;
          tma_load_2d(st, tA, k0, row0, &gs.full[s]);
          tma_load_2d(ring + S * A_BYTES + s * B_BYTES, tB, col0, k0, &gs.full[s]);
        } else {
          mbar_arrive(&gs.full[s]);  // control slot: no data
        }
        ++P;
        return true;
      };
      // Wait for an empty-barrier phase while watching the flag (POLL_STAGE):
      // returns 1 when the phase completed, 0 when a new generation (or the
      // stop sentinel) was published first, -1 on abort or timeout.
      // Observing during the waits makes the claim as early as the control
      // warp's publication, not a stage later.
      auto wait_watch = [&](uint64_t* bar, uint32_t par) -> int {
        const long long t0 = globaltimer_ns();
        int n = 0;
        while (true) {
          if (mbar_try_wait(bar, par)) return 1;
          if (POLL == POLL_STAGE && vload(&sh.gen) != lastSeen) return 0;
          if (++n == 64) {
            n = 0;
            if (vload(&sh.abort)) return -1;
            if (globaltimer_ns() - t0 > p.wait_limit_ns) {
              vstore(&sh.abort, 1);
              report_status(p.ev.status, DEV_WAIT_TIMEOUT_FULL, p.ev.abort_word);
              return -1;
            }
          }
        }
      };
      // Background tile in progress: its geometry and next stage to issue.
      unsigned long long bg_task = 0;
      int bg_row0 = 0, bg_col0 = 0, bg_c = 0, bg_nk = 0;
      int bg_k0 = 0;  // first K stage of the tile's slice
      int bg_xf = 0;  // F_CHAIN on its first stage / F_HANDOFF on its last (K slices)
      bool bg_open = false;  // the tile has stages issued and not all consumed
      // Observe generation f at a poll site and pop urgent work items; with
      // background stages in flight the first item is preceded by the skip
      // request and a SUSPEND slot, and the tile is later re-issued from the
      // warps' smallest cursor.  Returns items popped, or -1 on abort.
      auto handle = [&](int f, int site) -> int {
        const int fc = f < p.ev.max_events ? f : p.ev.max_events;
        const long long now = globaltimer_ns();
        for (int e = lastSeen; e < fc; ++e) p.ev.obs_ns[(size_t)e * nworkers + worker] = now;
        const int old = lastSeen;
        lastSeen = f;
        int n = 0;
        bool suspended = false;
        for (int e = old; e < fc; ++e) {
          while (true) {
            const int it = atomicAdd(&p.ev.uq_next[e], 1);
            if (it >= p.uitems) break;
            if (it == 0) {
              p.ev.claim_ns[e] = globaltimer_ns();
              p.ev.claim[e] = worker + 1;
              p.ev.claim_site[e] = site;
              p.ev.inflight[e] = (int)(P - (uint32_t)vload(&gs.consumed));
              if (p.ev.ack != nullptr) ack_host(&p.ev.ack[2 * e]);
            }
            if (n == 0 && bg_open && bg_c > 0) {
              // checkpoint the background tile: warps stop accumulating its
              // queued stages and spill at the SUSPEND slot
              vstore(&gs.skip, 1);
              long long* hdr = p.slab_hdr + (size_t)worker * 4;
              hdr[0] = (long long)bg_task;
              hdr[1] = bg_c;
              hdr[2] = e;
              hdr[3] = 1;
              atomicAdd(p.q.yields, 1ull);
              if (!emit(T_SUSPEND, 0, bg_c, bg_row0, bg_col0, e, 0, bg_task, nullptr, nullptr, 0)) return -1;
              suspended = true;
            }
            ++n;
            const int t = it / p.usplit, ks = it % p.usplit;
            const int r0 = (t / p.utiles_n) * BM, c0 = (t % p.utiles_n) * BN;
            for (int c = 0; c < p.unk; ++c) {
              const int flags = (c == 0 ? F_FIRST : 0) | (c == p.unk - 1 ? F_LAST : 0);
              if (!emit(T_URG, flags, c, r0, c0, e, it, 0, &p.tmAu, &p.tmBu, (ks * p.unk + c) * BK)) return -1;
            }
          }
        }
        if (suspended) {
          // resume from the stage every warp has accumulated
          if (!bwait(&gs.spilled, nsusp & 1, p, sh)) return -1;
          ++nsusp;
          int cmin = vload(&gs.cur[0]);
          for (int w = 1; w < 4; ++w) cmin = min(cmin, vload(&gs.cur[w]));
          bg_c = cmin;
          vstore(&gs.skip, 0);
          n = -2 - n;  // tells the caller to flag the next background stage RESUME
        }
        return n;
      };

      // Issue the open tile's stages bg_c .. bg_nk-1.  Under POLL_STAGE the
      // flag is watched while each yield site's slot frees (one every
      // poll_every slots); a yield there checkpoints the
      // tile and moves bg_c back to the warps' smallest cursor, and the next
      // stage issued carries RESUME.  False on stop or abort.
      auto emit_rest = [&](bool resume) -> bool {
        while (bg_c < bg_nk) {
          // a yield site every poll_every slots (one K-tile)
          if (POLL == POLL_STAGE && (p.poll_every <= 1 || bg_c % p.poll_every == 0)) {
            if (wait_watch(&gs.empty[P % S], ((P / S) & 1) ^ 1) < 0) return false;
            const int fs = vload(&sh.gen);
            if (fs < 0) return false;  // stop sentinel: abandon the tile
            if (fs != lastSeen) {
              const int n = handle(fs, bg_c);
              if (n == -1) return false;
              if (n <= -2) resume = true;
            }
          }
          const int flags = (bg_c == 0 ? F_FIRST | (bg_xf & F_CHAIN) : 0) |
                            (bg_c == bg_nk - 1 ? F_LAST | (bg_xf & F_HANDOFF) : 0) | (resume ? F_RESUME : 0);
          resume = false;
          if (!emit(T_BG, flags, bg_c, bg_row0, bg_col0, 0, 0, bg_task, &p.tmA, &p.tmB, (bg_k0 + bg_c) * BK))
            return false;
          ++bg_c;
        }
        return true;
      };
      // Wait until every stage of the open tile is consumed.  Under
      // POLL_STAGE the flag is still watched: a yield now suspends the tile
      // like one in mid-issue (its queued stages are skipped, not waited
      // for), the urgent items run, and the tile is re-issued from the
      // warps' cursors before the wait resumes.
      auto finish_tile = [&]() -> bool {
        while (bg_open && P > 0) {
          const uint32_t q = P - 1;
          const int r = wait_watch(&gs.empty[q % S], (q / S) & 1);
          if (r < 0) return false;
          if (r == 1) break;
          const int fs = vload(&sh.gen);
          if (fs < 0) return false;
          const int n = handle(fs, bg_c);
          if (n == -1) return false;
          // a tile the warps had already finished is not re-issued
          if (n <= -2 && !emit_rest(true)) return false;
        }
        bg_open = false;
        return true;
      };

      unsigned long long next_task = atomicAdd(p.q.next_task, 1ull);
      while (ok) {
        // ---- tile boundary: take the popped background task ----
        const unsigned long long task = next_task;
        if (task < p.q.num_tasks) next_task = atomicAdd(p.q.next_task, 1ull);
        if (!finish_tile()) break;  // the previous tile's stages are all consumed
        int f = vload(&sh.gen);
        if (POLL != POLL_OFF) {
          // at a boundary also read the flag itself: the control warp's copy
          // lags a store by up to a load's latency, and a bounded drain's
          // last tiles must not end unaware of a yield raised just before
          const int fg = flag_load(p.ev.flag);
          f = (fg < 0 || f < 0) ? -1 : max(f, fg);
        }
        if (f < 0 || vload(&sh.abort)) break;
        if (POLL != POLL_OFF && f != lastSeen && handle(f, -1) == -1) break;
        if (task >= p.q.num_tasks) break;
        const int ks = KS ? stream_ksplit(p.st) : 1;
        const int tile = (int)(task % (unsigned long long)(p.total_tiles * ks));
        int tm, tn, slice = 0;
        if (p.st.order != nullptr)
          stream_job(p.st, tile, p.tiles_n, tm, tn, slice);
        else
          tile_coords(tile, p.total_tiles / p.tiles_n, p.tiles_n, 8, tm, tn);
        // streamed operands: the slice of the tile's A row panel and B
        // column panel must have landed before its first TMA load
        if (p.st.a_ready != nullptr && !wait_ready2(&p.st.a_ready[(tm / p.st.panel_tm) * ks + slice],
                                                    &p.st.b_ready[(tn / p.st.b_units) * ks + slice], p.wait_limit_ns)) {
          vstore(&sh.abort, 1);
          report_status(p.ev.status, DEV_WAIT_TIMEOUT_SPIN, p.ev.abort_word);
          break;
        }
        // a later K slice starts from the accumulators its predecessor left:
        // every compute warp of that job has stored its share.  The
        // predecessor was popped earlier (the visit order lists every
        // slice-0 job first) and waits on nothing this worker does.
        if (KS && slice > 0 && !wait_count(&p.st.part_ready[tm * p.tiles_n + tn], 4 * slice, p, sh)) break;
        bg_task = task;
        bg_row0 = tm * BM;
        bg_col0 = tn * BN;
        bg_nk = p.nk / ks;
        bg_k0 = slice * bg_nk;
        bg_xf = (slice > 0 ? F_CHAIN : 0) | (slice < ks - 1 ? F_HANDOFF : 0);
        bg_c = 0;
        bg_open = true;
        ok = emit_rest(false);
      }
      emit(T_STOP, 0, 0, 0, 0, 0, 0, 0, nullptr, nullptr, 0);
      atomicAdd(&sh.prod_done, 1);
      // TMA loads still in flight (only when unwinding) must land before
      // exit; only the last S stages can be (an older slot was reused, its
      // barrier has moved on and its parity could match a later phase)
      for (uint32_t q = max((uint32_t)vload(&gs.consumed), P >= (uint32_t)S ? P - S : 0u); q < P; ++q)
        bwait_unwind(&gs.full[q % S], (q / S) & 1, p.wait_limit_ns);
    } else if (warp == G && lane == 0) {
      // ============================== control ===============================
      // one CTA per SM: the launch keeps one flag copy (ev.flag_lines == 1)
      int nextEv = 0;
      long long gBase = 0;
      while (vload(&sh.prod_done) < G && !vload(&sh.abort)) {
        int f = POLL != POLL_OFF ? flag_load(p.ev.flag) : 0;
        if (*reinterpret_cast<volatile int*>(p.ev.abort_word)) f = -1;
        // device-set events (src/yield.cu:186-195): worker 0's CTA
        if (blockIdx.x == 0 && p.ev.sched_ns != nullptr && nextEv < p.ev.n_sched) {
          const long long now = globaltimer_ns();
          if (gBase == 0) gBase = now;
          if (now >= gBase + p.ev.sched_ns[nextEv]) {
            p.ev.set_ns[nextEv] = now;
            atomicCAS(p.ev.flag, nextEv, nextEv + 1);  // never overwrites the -1 sentinel
            ++nextEv;
          }
        }
        vstore(&sh.gen, f);
        __nanosleep(64);
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(COMP_REGS));
    // ================================ compute =================================
    const int cw = warp - 4, g = cw >> 2, w = cw & 3, worker = blockIdx.x * G + g;
    const int gtid = w * 32 + lane;  // thread index inside the group
    GroupShared& gs = sh.g[g];
    const uint8_t* ring = ring_all + g * S * STAGE_BYTES;
    const int ty = lane >> 3, arow0 = w * 32 + ty, bcol = (lane & 7) * 4;
    float4* slab = reinterpret_cast<float4*>(p.slab) + (size_t)worker * 32 * 128;
    float acc[8][16];
    int cur = 0;           // K stages of the background tile accumulated by this warp
    bool bg_regs = false;  // acc holds the background tile (not an urgent item's)
    uint32_t Q = 0;
    while (true) {
      const int s = Q % S;
      if (!bwait(&gs.full[s], (Q / S) & 1, p, sh)) break;
      // only the fields the stage needs live in registers across the
      // mainloop; the epilogue re-reads the rest from the slot, which is not
      // released before it is done
      const int kind = vload(&gs.tag[s].kind), flags = vload(&gs.tag[s].flags), tc = vload(&gs.tag[s].c);
      if (kind == T_STOP) break;
      if (kind == T_SUSPEND) {
        // checkpoint: this thread's 128 accumulators and the warp's cursor.
        // A second yield before the tile resumed finds an urgent item's
        // values in acc: the slab already holds the tile, keep it.
        if (bg_regs) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int q = 0; q < 4; ++q)
              slab[(i * 4 + q) * 128 + gtid] =
                  make_float4(acc[i][4 * q], acc[i][4 * q + 1], acc[i][4 * q + 2], acc[i][4 * q + 3]);
          bg_regs = false;
        }
        __syncwarp();
        if (lane == 0) {
          vstore(&gs.cur[w], cur);
          mbar_arrive(&gs.spilled);
          mbar_arrive(&gs.empty[s]);
        }
        ++Q;
        continue;
      }
      bool compute = true;
      if (kind == T_BG) {
        if (flags & (KS ? F_RESUME | F_CHAIN : F_RESUME)) {
          // RESUME: the checkpointed accumulators; cur is this warp's own
          // cursor, kept across the urgent items (a re-issue from stage 0
          // also carries F_FIRST, which must not reset it).  CHAIN (first
          // stage of a later K slice): the previous slice's accumulators,
          // stored by another worker, so the loads skip L1.
          // (slab: one float4 per (i, q) and thread; hand-off block: the
          // C tile layout, row stride BN)
          const float4* src = slab + gtid;
          int si = 4 * 128, sq = 128;
          if (KS && !(flags & F_RESUME)) {
            cur = 0;
            const int tid = (vload(&gs.tag[s].row0) / BM) * p.tiles_n + vload(&gs.tag[s].col0) / BN;
            src = reinterpret_cast<const float4*>(p.st.part + (size_t)tid * (BM * BN) + arow0 * BN + bcol);
            si = 4 * BN / 4;
            sq = 32 / 4;
          }
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 v = KS ? __ldcg(&src[i * si + q * sq]) : src[i * si + q * sq];
              acc[i][4 * q] = v.x;
              acc[i][4 * q + 1] = v.y;
              acc[i][4 * q + 2] = v.z;
              acc[i][4 * q + 3] = v.w;
            }
          bg_regs = true;
        } else if (flags & F_FIRST) {
          cur = 0;
          bg_regs = true;
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[i][j] = 0.f;
        }
        // already accumulated before a checkpoint, or queued behind a yield
        compute = tc == cur && !vload(&gs.skip);
      } else if (flags & F_FIRST) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[i][j] = 0.f;
      }
      if (compute) {
        const float* As = reinterpret_cast<const float*>(ring + s * A_BYTES);
        const float* Bs = reinterpret_cast<const float*>(ring + S * A_BYTES + s * B_BYTES);
        // fully unrolled: 53.5 TFLOP/s a drain against 53.2 unrolled by 4, 52.2
        // by 2 and 49.0 not unrolled (that one spill-free, so the few bytes
        // the unrolled loops spill cost less than the ILP they buy)
#pragma unroll
        for (int kp = 0; kp < 16; ++kp) kpair(As, Bs, acc, arow0, ty, bcol, kp);
        if (DISC == DISC_POISON && kind == T_URG && (flags & F_FIRST) && bcol == 0) {
          // detector control: the item's first staged B value B[k0][c0] read
          // as B + 1 (src/midyield.cu:146-147), applied in registers
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = arow0 + 4 * i;
            acc[i][0] += As[r * 32 + (((0 ^ (r & 7))) << 2)];
          }
        }
        if (kind == T_BG) cur = tc + 1;
      }
      // a background stage is computed only in cursor order, so computing
      // the F_LAST one completes the tile (or its K slice)
      const bool done_tile = (flags & F_LAST) && (kind == T_URG || (compute && (KS || cur == p.nk)));
      if (done_tile) {
        const Tag& t = gs.tag[s];
        const int row0 = vload(&t.row0), col0 = vload(&t.col0), e = vload(&t.e);
        // ---- epilogue: this warp's 32 rows of the tile ----
        if (kind == T_BG && !KS) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float* crow = p.C + (size_t)(row0 + arow0 + 4 * i) * p.ldc + col0 + bcol;
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<float4*>(crow + 32 * q) =
                  make_float4(acc[i][4 * q], acc[i][4 * q + 1], acc[i][4 * q + 2], acc[i][4 * q + 3]);
          }
        } else if (kind == T_BG) {
          // the tile's C block, or for a K slice before the last the tile's
          // hand-off block (the same layout with a row stride of BN)
          float* cb = p.C + (size_t)row0 * p.ldc + col0;
          size_t ld = p.ldc;
          if (flags & F_HANDOFF) {
            cb = p.st.part + (size_t)((row0 / BM) * p.tiles_n + col0 / BN) * (BM * BN);
            ld = BN;
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float* crow = cb + (size_t)(arow0 + 4 * i) * ld + bcol;
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<float4*>(crow + 32 * q) =
                  make_float4(acc[i][4 * q], acc[i][4 * q + 1], acc[i][4 * q + 2], acc[i][4 * q + 3]);
          }
        } else {
          float* Cu = p.Cu + (size_t)e * p.cu_stride;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float* crow = Cu + (size_t)(row0 + arow0 + 4 * i) * p.ldcu + col0 + bcol;
            if (p.usplit == 1) {
#pragma unroll
              for (int q = 0; q < 4; ++q)
                *reinterpret_cast<float4*>(crow + 32 * q) =
                    make_float4(acc[i][4 * q], acc[i][4 * q + 1], acc[i][4 * q + 2], acc[i][4 * q + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) atomicAdd(crow + 32 * (j >> 2) + (j & 3), acc[i][j]);
            }
          }
        }
        __threadfence();  // the tile's stores are visible before it is counted
        __syncwarp();
        if (KS && lane == 0 && kind == T_BG && (flags & F_HANDOFF))
          atomicAdd(&p.st.part_ready[(row0 / BM) * p.tiles_n + col0 / BN], 1);  // this warp's share is out
        // the fourth warp to finish does the accounting.  A background tile
        // counts on the group's counter: a warp that skipped its last stage
        // behind a yield stores it after the resume, in another slot.  An
        // urgent item (never skipped) counts on its slot, which is not
        // refilled before all four warps have released it.
        int* cnt = kind == T_BG ? &gs.bg_cnt : &gs.cnt[s];
        if (lane == 0 && atomicAdd(cnt, 1) == 3) {
          *cnt = 0;
          if (kind == T_BG) {
            if (ORACLE && p.q.exec_count != nullptr) atomicAdd(&p.q.exec_count[t.task], 1);
            if (!KS || !(flags & F_HANDOFF)) {  // the tile is complete
              ++gs.tiles;
              count_trigger(p.ev);
              if (p.st.done != nullptr)
                stream_tile_done(p.st, p.total_tiles / p.tiles_n, p.tiles_n, row0 / BM, col0 / BN);
            }
          } else {
            if (ORACLE) atomicAdd(&p.ev.uexec[e], 1);
            atomicMax(&p.ev.done_ns[e], (unsigned long long)globaltimer_ns());
            const int done = atomicAdd(&p.ev.udone_cnt[e], 1) + 1;
            if (done == p.uitems && p.ev.ack != nullptr) ack_host(&p.ev.ack[2 * e + 1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&gs.empty[s]);
        if (w == 0) vstore(&gs.consumed, (int)(Q + 1));
      }
      ++Q;
    }
    // last warp of the group out reports the worker's totals
    __syncwarp();
    if (lane == 0 && atomicAdd(&gs.exit_cnt, 1) == 3) {
      __threadfence_block();
      p.q.tiles_done[worker] = *reinterpret_cast<volatile unsigned long long*>(&gs.tiles);
      atomicMax(p.q.end_max, (unsigned long long)globaltimer_ns());
      atomicAdd(p.q.exited, 1);
    }
  }
}

// Host-side dispatch.

template <int POLL, int DISC, bool ORACLE>
static const void* kernel_ptr(bool ks) {
  return ks ? reinterpret_cast<const void*>(&sgemm_ws<POLL, DISC, ORACLE, true>)
            : reinterpret_cast<const void*>(&sgemm_ws<POLL, DISC, ORACLE, false>);
}

static const void* select_kernel(int poll, int disc, bool oracle, bool ks) {
#define APK_SEL(PL, DS, OR) \
  if (poll == PL && disc == DS && oracle == OR) return kernel_ptr<PL, DS, OR>(ks);
  APK_SEL(POLL_OFF, DISC_DRAIN, false)
  APK_SEL(POLL_OFF, DISC_DRAIN, true)
  APK_SEL(POLL_BOUNDARY, DISC_DRAIN, false)
  APK_SEL(POLL_BOUNDARY, DISC_DRAIN, true)
  APK_SEL(POLL_BOUNDARY, DISC_POISON, false)
  APK_SEL(POLL_STAGE, DISC_DRAIN, false)
  APK_SEL(POLL_STAGE, DISC_DRAIN, true)
  APK_SEL(POLL_STAGE, DISC_POISON, false)
  APK_SEL(POLL_STAGE, DISC_POISON, true)
#undef APK_SEL
  return nullptr;
}

int smem_bytes() { return SMEM_BYTES; }
int threads() { return NT; }
int workers_per_cta() { return G; }
size_t params_bytes() { return sizeof(F32Params); }

// Sets the kernel up; *ok = 0 when it cannot run here (its launch register
// count below the setmaxnreg split, or not one CTA per SM).
cudaError_t prepare(int poll, int disc, bool oracle, int* ok) {
  *ok = 0;
  int good = 1;
  for (const bool ks : {false, true}) {  // resident and K-sliced streamed runs
    const void* k = select_kernel(poll, disc, oracle, ks);
    if (!k) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, k);
    if (e != cudaSuccess) return e;
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, NT, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    // setmaxnreg.inc waits for registers the block does not have if the
    // launch gave it fewer than the split assumes: never launch that
    if (!(fa.numRegs >= LAUNCH_REGS && occ == 1)) good = 0;
  }
  *ok = good;
  return cudaSuccess;
}

// workers = the runtime's grid (2 per CTA).  prm.st.ksplit > 1 selects the
// K-sliced instantiation.
cudaError_t launch(const F32Params& prm, int workers, int poll, int disc, bool oracle, cudaStream_t stream) {
  const void* k = select_kernel(poll, disc, oracle, prm.st.ksplit > 1);
  if (!k || workers % G != 0) return cudaErrorInvalidValue;
  void* args[] = {const_cast<F32Params*>(&prm)};
  return cudaLaunchKernel(k, dim3(workers / G), dim3(NT), args, SMEM_BYTES, stream);
}

}  // namespace f32ws
}  // namespace apk
