// bf16 tensor-core persistent GEMM on CTA pairs (tcgen05.mma.cta_group::2):
// the default bf16 kernel for a plain background GEMM whose N is a multiple
// of 256 (the configs[2] shape).  Same job protocol, yields, checkpoints and
// outputs as gemm_bf16.cu (which keeps task mode, 128-wide edges, K-tile 32
// and every other shape); replaces the same reference code
// (src/tcyield.cu:91-356).
//
// B200 design:
//   * A cluster of two CTAs on two SMs computes a 256 x 512 output tile:
//     two accumulators D_h (C columns [c0 + 256h, +256)), each one M=256,
//     N=256 cta_group::2 MMA per 16-deep k-step.  CTA r stages A rows
//     [r0 + 128r, +128) and the B columns [c0 + 256h + 128r, +128) of each
//     half, and holds in its TMEM the accumulator lanes of its own C
//     columns.  Per MMA each SM reads 8 KB of shared memory for 2^19 MACs
//     (the one-CTA kernel: 12 KB), and the pair shares one A row panel:
//     the ring moves 48 KB per CTA and stage instead of 64 KB.
//   * The leader (cluster rank 0) decides everything: its producer pops the
//     queue, polls, pops urgent items, issues its own TMA loads and forwards
//     each slot's tag to the peer's producer through distributed shared
//     memory; the peer issues the loads of its halves.  Both CTAs' loads
//     complete on the leader's full barrier (cta_group::2 TMA).  The
//     leader's MMA warp issues the pair MMAs, commits to the barriers of both
//     CTAs and posts every epilogue job to both CTAs' job rings.  Each CTA's
//     8 epilogue warps drain, store, spill and restore their own TMEM; the
//     TMEM-free, restore-done and job-slot-free barriers live in the leader
//     and count 16 arrivals (8 local, 8 remote).  The last of the 16 warps
//     to finish a tile does its accounting.
//   * Yield / checkpoint / resume exactly as in the one-CTA kernel: SUSPEND
//     slot, both CTAs spill their accumulator lanes to their own slabs,
//     urgent items run through the same ring, RESUME restores and the MMAs
//     continue with the same sequence -- bitwise identical to an
//     uninterrupted run.
//   * No TMA multicast: each CTA loads its own operands.  Every wait is
//     bounded; every role of both CTAs reaches the final cluster barriers,
//     where the pair waits for outstanding MMAs and loads before TMEM is
//     released (cta_group::2 dealloc by both CTAs) and the CTAs exit.
#include <string>

#include "../../include/apk.h"
#include "common.cuh"
#include "proto.h"
#include "tcgen05.cuh"

namespace apk {
namespace bf16pair {

constexpr int BM = 256, BN = 512, BK = 64;
constexpr int EPI_WARPS = 8;
constexpr int CTRL_WARP = 2 + EPI_WARPS;
constexpr int NT = 32 * (CTRL_WARP + 1);
constexpr int A_BYTES = 128 * BK * 2;         // this CTA's 128 A rows
constexpr int B_CHUNK = BK * 64 * 2;          // one [64 k][64 n] box
constexpr int RING = 8;
// Peer tag ring.  The leader stores stage P's tag in entry P % T after its
// wait for stage P-1's slot, i.e. after the MMAs of stage P-1-S completed;
// those needed the peer's loads of every data stage up to P-1-S, which the
// peer issues only after reading their tags in order -- so with T > S + 1
// the peer has read entry P % T's previous tag (P - T) without an explicit
// acknowledgment (a SUSPEND slot is always followed by urgent data stages).
// A release-ordered acknowledgment from the peer cost ~1400 cycles a stage
// and starved the ring.
//
// Ring geometry: S slots of A + NCH B chunks.  A plain run's 512-wide pair
// tiles take four chunks a slot (4 x 48 KB); task lists, whose pair jobs are
// at most 256 wide, take two (6 x 32 KB): a short task's stage holds half the
// MMA work of a wide one, and four slots of it did not cover the load
// latency (the task kernel streamed at two thirds of the one-CTA kernel's
// rate).
template <int S_, int NCH_>
struct PG {
  static constexpr int S = S_, NCH = NCH_, T = 4 * S_;
  static constexpr int STAGE_BYTES = A_BYTES + NCH_ * B_CHUNK;
  static constexpr int SMEM_BYTES = S_ * STAGE_BYTES + 1024;
};
using PgPlain = PG<4, 4>;
using PgTasks = PG<6, 2>;
constexpr int RASTER_GROUP = 8;
// D = C_cols^T: MMA A = the B columns (MN-major), MMA B = the A rows (K-major)
constexpr uint32_t IDESC = tc::idesc_bf16_f32(256, 256, true, false);
// a task tile with 128 valid rows: N = 128, each CTA staging 64 of them
constexpr uint32_t IDESC_HALF = tc::idesc_bf16_f32(256, 128, true, false);

enum : int { T_BG = 1, T_URG = 2, T_SUSPEND = 3, T_STOP = 4 };
enum : int { F_FIRST = 1, F_LAST = 2, F_RESUME = 4, F_WIDE = 8, F_HALF = 16 };
enum : int { E_STORE_C = 1, E_STORE_U = 2, E_SPILL = 3, E_RESTORE = 4, E_EXIT = 5 };

// row0 / col0: the job's output origin; e: the urgent event, or for a
// background job its valid rows; ncols: its valid columns (512 for a wide
// pair tile, 256, or 128 for a task tile whose n ends 128 columns in: the
// peer's half is computed but not stored)
struct StageTag {
  int kind, flags, row0, col0, e, item, k, ncols;
  unsigned long long task;
};
struct EpiJob {
  int action, buf, wide, row0, col0, e, item, ncols;
  unsigned long long task;
};

template <int S, int T>
struct __align__(16) Shared {
  StageTag tag[S];   // the leader's MMA reads the slot's tag here
  uint4 ptag[T];     // the peer's copy {kind | flags << 8, row0, col0, k}, stored by the leader
  EpiJob epi[RING];
  uint64_t full[S], empty[S], tagfull[T];
  uint64_t tfull[2], tempty[2], tres[2];
  uint64_t efull[RING], eempty[RING];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int gen;
  int prod_done;
  int consumed;
  int epi_cnt[RING];
  // task mode: this CTA's 8 epilogue warps' sum(c^2) partials of its 128
  // columns of a job and their count (the CTA's own accounting)
  double chk_part[RING][EPI_WARPS];
  int cta_cnt[RING];
  unsigned long long tiles;
  // the pair's resident slot (logs, counters and slabs of its two CTAs are
  // at 2 * slot + rank); under CLC the leader's cancellation answer
  int slot;
  uint4 clc_resp;
  uint64_t clc_bar;
};

__device__ __forceinline__ int vload(const int* p) { return *reinterpret_cast<const volatile int*>(p); }
__device__ __forceinline__ void vstore(int* p, int v) { *reinterpret_cast<volatile int*>(p) = v; }

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of this CTA's variable in CTA `rank`'s shared memory
__device__ __forceinline__ uint32_t mapa(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_u64(uint32_t addr, unsigned long long v) {
  asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(addr), "l"(v) : "memory");
}
// 16-byte store into the peer's shared memory that completes 16 transaction
// bytes on the peer's barrier: the leader does not wait for it
__device__ __forceinline__ void st_async_v4(uint32_t addr, uint4 v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned atom_add_cluster(uint32_t addr, unsigned v) {
  unsigned old;
  asm volatile("atom.shared::cluster.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(addr), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void atom_add_cluster_u64(uint32_t addr, unsigned long long v) {
  asm volatile("red.shared::cluster.add.u64 [%0], %1;" ::"r"(addr), "l"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's shared memory completing on a barrier of either
// CTA of the pair
__device__ __forceinline__ void tma_load_pair(void* dst, const CUtensorMap* tm, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t acc,
                                         uint32_t idesc = IDESC) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// one arrival on the barrier (either CTA) once this thread's pair MMAs completed
__device__ __forceinline__ void commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Bounded wait on a barrier of this CTA (remote arrivals: cluster-scope
// acquire); also gives up when another role of this CTA aborted.
template <class SH>
__device__ __forceinline__ bool bwait(uint64_t* bar, uint32_t parity, const F32Params& p, SH& sh) {
  if (try_wait_cluster(bar, parity)) return true;
  const long long t0 = globaltimer_ns();
  int n = 0;
  while (true) {
    if (try_wait_cluster(bar, parity)) return true;
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
__device__ __forceinline__ void bwait_unwind(uint64_t* bar, uint32_t parity, long long limit) {
  const long long t0 = globaltimer_ns();
  while (!try_wait_cluster(bar, parity))
    if (globaltimer_ns() - t0 > limit) return;
}

// SCHED: SCH_QUEUE (the atomic queue) or SCH_CLC (one cluster per task:
// the leader of each running pair cancels a not-yet-launched cluster with
// clusterlaunchcontrol.try_cancel, without multicast, and takes its task;
// the peer learns every task from the leader's stage tags as it does under
// the queue)
enum : int { SCH_QUEUE = 0, SCH_CLC = 1 };
constexpr unsigned long long NO_TASK = ~0ull;

template <int POLL, int DISC, bool ORACLE, class PGEO, int SCHED = SCH_QUEUE>
__global__ void __launch_bounds__(NT, 1) gemm_bf16_pair(const __grid_constant__ F32Params p) {
  constexpr bool CLC = SCHED == SCH_CLC;
  constexpr int S = PGEO::S, T = PGEO::T, NCH = PGEO::NCH, STAGE_BYTES = PGEO::STAGE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Shared<S, T> sh;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;

  if (tid == 0) {
    if constexpr (CLC) {
      // the leader claims the pair's slot (one bit per resident pair); the
      // peer reads it from the leader once the start-up cluster barrier has
      // shown both CTAs running
      if (leader) {
        mbar_init(&sh.clc_bar, 1);
        int sl = slot_claim(p.q.slot_bits, p.q.nslots / 2, p.wait_limit_ns);
        sh.abort = 0;
        if (sl < 0) {  // cannot happen while residency holds: stop the pair at once
          report_status(p.ev.status, DEV_BAD_CONFIG, p.ev.abort_word);
          sh.abort = 1;
          sl = 0;
        }
        sh.slot = sl;
      }
    } else {
      sh.slot = (int)blockIdx.x / 2;
    }
    for (int s = 0; s < S; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int t = 0; t < T; ++t) mbar_init(&sh.tagfull[t], 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.tfull[b], 1);
      mbar_init(&sh.tempty[b], 2 * EPI_WARPS);
      mbar_init(&sh.tres[b], 2 * EPI_WARPS);
    }
    for (int r = 0; r < RING; ++r) {
      mbar_init(&sh.efull[r], 1);
      mbar_init(&sh.eempty[r], 2 * EPI_WARPS);
      sh.epi_cnt[r] = 0;
      sh.cta_cnt[r] = 0;
    }
    mbar_init(&sh.drain, 1);
    fence_mbar_init();
    if (!CLC || !leader) sh.abort = 0;  // a leader that found no slot stops the pair
    sh.gen = 0;
    sh.prod_done = 0;
    sh.consumed = 0;
    sh.tiles = 0;
    tma_prefetch_desc(&p.tmA);
    tma_prefetch_desc(&p.tmB);
    tma_prefetch_desc(&p.tmAu);
    tma_prefetch_desc(&p.tmBu);
    atomicMin(p.q.start_min, (unsigned long long)globaltimer_ns());
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     smem_u32(&sh.tmem_base))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc::fence_before_sync();
  __syncthreads();
  __syncwarp();
  cluster_sync();  // both CTAs' barriers initialised before any remote access
  tc::fence_after_sync();
  if (CLC && !leader) {
    if (tid == 0) {
      uint32_t sl;
      asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(sl) : "r"(mapa(&sh.slot, 0)) : "memory");
      sh.slot = (int)sl;
    }
    __syncthreads();
  }
  // per-CTA logs, counters and the slab: index 2 * slot + rank (the block
  // index under the queue, where slot = cluster index)
  const int cta = 2 * sh.slot + (int)rank;
  const int gridw = CLC ? p.q.nslots : (int)gridDim.x;

  if (warp == 0 && lane == 0 && leader) {
    // ============================ leader producer ============================
    uint32_t P = 0;
    int lastSeen = 0;
    bool ok = true;
    // One slot: the job's output origin (row0, col0) and bookkeeping travel
    // with the tag; the leader loads A rows from ar0 and B columns from bc0
    // at k offsets ak / bk (they differ in task mode, where A, B and C are
    // windows of pools), the peer A rows from ar0 + 128 (+ 64 for a
    // 128-row task tile, whose N = 128 MMAs take 64 rows from each CTA).
    auto emit = [&](int kind, int flags, int row0, int col0, int e, int item, unsigned long long task,
                    const CUtensorMap* tA, const CUtensorMap* tB, int ar0, int bc0, int ak, int bk,
                    int ncols) -> bool {
      // first the peer's copy of the tag, into its tag ring: the peer then
      // issues its loads the moment its slot frees, in step with the
      // leader's own.  {kind | flags << 8 | (bk - ak) << 16, peer A row,
      // B column base, ak}
      const int ti = P % T;
      const int peer_ar0 = ar0 + ((flags & F_HALF) ? 64 : 128);
      st_async_v4(mapa(&sh.ptag[ti], 1),
                  make_uint4((uint32_t)kind | ((uint32_t)flags << 8) | ((uint32_t)(bk - ak) << 16),
                             (uint32_t)peer_ar0, (uint32_t)bc0, (uint32_t)ak),
                  mapa(&sh.tagfull[ti], 1));
      const int s = P % S;
      if (!bwait(&sh.empty[s], ((P / S) & 1) ^ 1, p, sh)) return false;
      StageTag& t = sh.tag[s];
      t.kind = kind;
      t.flags = flags;
      t.row0 = row0;
      t.col0 = col0;
      t.e = e;
      t.item = item;
      t.k = ak;
      t.ncols = ncols;
      t.task = task;
      if (tA != nullptr) {
        const int nb = (NCH == 4 && (flags & F_WIDE)) ? 4 : 2;
        mbar_arrive_expect_tx(&sh.full[s], 2 * (A_BYTES + nb * B_CHUNK));
        uint8_t* st = stages + s * STAGE_BYTES;
        const uint32_t fb = mapa(&sh.full[s], 0);
        tma_load_pair(st, tA, ak, ar0, fb);
        for (int b = 0; b < nb; ++b)
          tma_load_pair(st + A_BYTES + b * B_CHUNK, tB, bc0 + 256 * (b >> 1) + 64 * (b & 1), bk, fb);
      } else {
        mbar_arrive(&sh.full[s]);  // control slot: no data
      }
      ++P;
      return true;
    };
    // Observe generation f at a poll site and pop urgent work items (as in
    // the one-CTA kernel); the observation is logged for both CTAs.
    auto handle = [&](int f, int site, bool partial) -> int {
      const int fc = f < p.ev.max_events ? f : p.ev.max_events;
      const long long g = globaltimer_ns();
      for (int e = lastSeen; e < fc; ++e) {
        p.ev.obs_ns[(size_t)e * gridw + cta] = g;
        p.ev.obs_ns[(size_t)e * gridw + cta + 1] = g;
      }
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
            if (!emit(T_SUSPEND, 0, 0, 0, 0, 0, 0, nullptr, nullptr, 0, 0, 0, 0, 0)) return -1;
            atomicAdd(p.q.yields, 1ull);
          }
          ++n;
          const int t = it / p.usplit, ks = it % p.usplit;
          const int r0 = (t / p.utiles_n) * BM, c0 = (t % p.utiles_n) * BN;
          const int wide = c0 + BN <= p.ldcu ? F_WIDE : 0;
          for (int c = 0; c < p.unk; ++c) {
            const int kk = (ks * p.unk + c) * BK;
            if (!emit(T_URG, (c == 0 ? F_FIRST : 0) | (c == p.unk - 1 ? F_LAST : 0) | wide, r0, c0, e, it, 0,
                      &p.tmAu, &p.tmBu, r0, c0, kk, kk, wide ? 512 : 256))
              return -1;
          }
        }
      }
      return n;
    };

    // CLC: the task of the cluster cancelled by the request answered at this
    // boundary, asked for one tile earlier (the first is the pair's own)
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
      return clc_query(&sh.clc_resp, &x) ? (unsigned long long)(x / 2) : NO_TASK;
    };
    if (CLC) {
      // a pair launched mid-run takes the generations raised before it as
      // seen: their urgent work was popped by the pairs that observed them
      const int f0 = flag_load(p.ev.flag);
      lastSeen = f0 > 0 ? f0 : 0;
    }
    unsigned long long next_task = CLC ? (unsigned long long)(blockIdx.x / 2) : atomicAdd(p.q.next_task, 1ull);
    if (CLC && ok && !vload(&sh.abort)) clc_issue();
    while (ok) {
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
      // job geometry: output origin, operand origins and k offsets, K steps,
      // valid rows and columns, width (wide = 512 columns over two
      // accumulators, else 256 in one)
      int row0, col0, ar0, bc0, ak0 = 0, bk0 = 0, nk = p.nk, mvalid = BM, wide = 0, ncols;
      unsigned long long tag_task = task;
      int tm = 0, tn = 0;
      if (p.task_mode) {
        // work entry: task, tile row, first 128-column block of the tile;
        // every task tile is a 256x256 pair job (a tile whose n ends 128
        // columns in computes the peer's half without storing it)
        const unsigned w = p.work[task];
        const TaskDesc td = p.tasks[w >> 12];
        tm = (w >> 6) & 63;
        tn = w & 63;
        row0 = td.c_row0 + tm * BM;
        col0 = td.c_col0 + tn * 128;
        ar0 = td.a_row0 + tm * BM;
        bc0 = td.b_col0 + tn * 128;
        ak0 = td.a_k0;
        bk0 = td.b_k0;
        nk = td.k / BK;
        mvalid = (td.m - tm * BM) < BM ? (td.m - tm * BM) : BM;
        ncols = (tn + 2) * 128 <= td.n ? 256 : 128;
        // checksum / oracle index of the tile's first 256x128 half
        tag_task = (unsigned long long)(td.chk_base + (long long)tm * (td.n / 128) + tn);
      } else {
        const int tile = (int)(task % (unsigned long long)p.total_tiles);
        if (p.st.order != nullptr)
          stream_tile(p.st, tile, p.tiles_n, tm, tn);
        else
          tile_coords(tile, p.total_tiles / p.tiles_n, p.tiles_n, RASTER_GROUP, tm, tn);
        row0 = ar0 = tm * BM;
        col0 = bc0 = tn * BN;
        wide = col0 + BN <= p.ldc ? F_WIDE : 0;
        ncols = wide ? 512 : 256;
      }
      if (p.st.a_ready != nullptr) {
        // every 128-column B unit of the tile must have landed
        const int* ar = &p.st.a_ready[tm / p.st.panel_tm];
        const int u0 = col0 / 128, un = (wide ? 4 : 2);
        bool rdy = true;
        for (int u = u0; u < u0 + un && rdy; u += p.st.b_units)
          rdy = wait_ready2(ar, &p.st.b_ready[u / p.st.b_units], p.wait_limit_ns);
        if (rdy) rdy = wait_ready2(ar, &p.st.b_ready[(u0 + un - 1) / p.st.b_units], p.wait_limit_ns);
        if (!rdy) {
          vstore(&sh.abort, 1);
          report_status(p.ev.status, DEV_WAIT_TIMEOUT_SPIN, p.ev.abort_word);
          ok = false;
          break;
        }
      }
      bool resume = false;
      for (int c = 0; c < nk && ok; ++c) {
        // a yield site every poll_every ring slots (one K-tile)
        if (POLL == POLL_STAGE && (p.poll_every <= 1 || c % p.poll_every == 0)) {
          const int fs = vload(&sh.gen);
          if (fs < 0) {
            ok = false;
            break;
          }
          if (fs != lastSeen) {
            const int n = handle(fs, c, c > 0);
            if (n < 0) {
              ok = false;
              break;
            }
            if (n > 0 && c > 0) resume = true;
          }
        }
        const int flags = (c == 0 ? F_FIRST : 0) | (c == nk - 1 ? F_LAST : 0) | (resume ? F_RESUME : 0) | wide |
                          (mvalid <= 128 ? F_HALF : 0);
        resume = false;
        if (!emit(T_BG, flags, row0, col0, mvalid, 0, tag_task, &p.tmA, &p.tmB, ar0, bc0, ak0 + c * BK,
                  bk0 + c * BK, ncols))
          ok = false;
      }
    }
    emit(T_STOP, 0, 0, 0, 0, 0, 0, nullptr, nullptr, 0, 0, 0, 0, 0);
    // a CLC answer still in flight (a stopped or aborted run) lands before
    // shared memory goes away; a cluster it cancelled is dropped with the run
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
  } else if (warp == 0 && lane == 0) {
    // ============================= peer producer =============================
    // Follows the leader's tags; loads a slot's halves once the pair MMAs
    // that read the slot's previous use have completed (its empty barrier,
    // committed by the leader's MMA warp).
    uint32_t P = 0;
    while (true) {
      const int ti = P % T, s = P % S;
      // this entry's phase: our arrival plus the leader's 16-byte store
      mbar_arrive_expect_tx(&sh.tagfull[ti], 16);
      if (!bwait(&sh.tagfull[ti], (P / T) & 1, p, sh)) break;
      const uint4 w = sh.ptag[ti];
      StageTag t;
      t.kind = (int)(w.x & 0xFF);
      t.flags = (int)((w.x >> 8) & 0xFF);
      const int dk = (int)(int16_t)(w.x >> 16);  // B's k offset minus A's
      t.row0 = (int)w.y;                         // this CTA's first A row
      t.col0 = (int)w.z;                         // the job's B column base
      t.k = (int)w.w;
      if (t.kind == T_STOP) break;
      if (t.kind == T_BG || t.kind == T_URG) {
        if (!bwait(&sh.empty[s], ((P / S) & 1) ^ 1, p, sh)) break;
        const CUtensorMap* tA = t.kind == T_BG ? &p.tmA : &p.tmAu;
        const CUtensorMap* tB = t.kind == T_BG ? &p.tmB : &p.tmBu;
        if (t.kind == T_BG && (t.flags & F_FIRST) && p.st.a_ready != nullptr) {
          // the leader saw the panels land; order this CTA's loads after it
          const int u0 = t.col0 / 128;
          if (!wait_ready2(&p.st.a_ready[((t.row0 - 128) / BM) / p.st.panel_tm],
                           &p.st.b_ready[(u0 + ((t.flags & F_WIDE) ? 3 : 1)) / p.st.b_units], p.wait_limit_ns))
            break;
        }
        const int nb = (NCH == 4 && (t.flags & F_WIDE)) ? 4 : 2;
        uint8_t* st = stages + s * STAGE_BYTES;
        const uint32_t fb = mapa(&sh.full[s], 0);
        tma_load_pair(st, tA, t.k, t.row0, fb);
        for (int b = 0; b < nb; ++b)
          tma_load_pair(st + A_BYTES + b * B_CHUNK, tB, t.col0 + 256 * (b >> 1) + 128 + 64 * (b & 1), t.k + dk,
                        fb);
      }
      ++P;
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ================================== MMA ===================================
    uint32_t Q = 0, X = 0, ub[2] = {0, 0}, rb[2] = {0, 0};
    int nb = 0, cur = 0, cwide = 0;
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
      j.ncols = t.ncols;
      j.task = t.task;
      const uint32_t pj = mapa(&j, 1);
      st_cluster_u32(pj + offsetof(EpiJob, action), (uint32_t)action);
      st_cluster_u32(pj + offsetof(EpiJob, buf), (uint32_t)buf);
      st_cluster_u32(pj + offsetof(EpiJob, wide), (uint32_t)wide);
      st_cluster_u32(pj + offsetof(EpiJob, row0), (uint32_t)t.row0);
      st_cluster_u32(pj + offsetof(EpiJob, col0), (uint32_t)t.col0);
      st_cluster_u32(pj + offsetof(EpiJob, e), (uint32_t)t.e);
      st_cluster_u32(pj + offsetof(EpiJob, item), (uint32_t)t.item);
      st_cluster_u32(pj + offsetof(EpiJob, ncols), (uint32_t)t.ncols);
      st_cluster_u64(pj + offsetof(EpiJob, task), t.task);
      mbar_arrive(&sh.efull[sl]);
      arrive_cluster(mapa(&sh.efull[sl], 1));
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
        if (!post(E_SPILL, cur, cwide, t)) break;
        commit_pair(mapa(&sh.tfull[cur], 0));
        commit_pair(mapa(&sh.tfull[cur], 1));
        mbar_arrive(&sh.empty[s]);
        arrive_cluster(mapa(&sh.empty[s], 1));  // every use of a slot completes a phase in both CTAs
        ++Q;
        vstore(&sh.consumed, (int)Q);
        continue;
      }
      if (t.flags & (F_FIRST | F_RESUME)) {
        cwide = (NCH == 4 && (t.flags & F_WIDE)) ? 1 : 0;
        cur = cwide ? 0 : nb;
        nb = cwide ? 0 : nb ^ 1;
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
      const uint32_t d0 = tbase + (uint32_t)cur * 256;
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        const uint32_t acc = (kk > 0 || !(t.flags & F_FIRST)) ? 1u : 0u;
        const uint64_t bdesc = tc::smem_desc(sa + kk * 32, 16, 1024, tc::LAYOUT_SW128);
        mma_pair(d0, tc::smem_desc(sb + kk * 2048, B_CHUNK, 1024, tc::LAYOUT_SW128), bdesc, acc,
                 (t.flags & F_HALF) ? IDESC_HALF : IDESC);
        if (NCH == 4 && cwide)
          mma_pair(d0 + 256, tc::smem_desc(sb + 2 * B_CHUNK + kk * 2048, B_CHUNK, 1024, tc::LAYOUT_SW128), bdesc,
                   acc);
      }
      commit_pair(mapa(&sh.empty[s], 0));  // frees the slot (both CTAs' halves) once read
      commit_pair(mapa(&sh.empty[s], 1));
      if (t.flags & F_LAST) {
        if (!post(t.kind == T_BG ? E_STORE_C : E_STORE_U, cur, cwide, t)) break;
        commit_pair(mapa(&sh.tfull[cur], 0));
        commit_pair(mapa(&sh.tfull[cur], 1));
      }
      ++Q;
      vstore(&sh.consumed, (int)Q);
    }
    commit_pair(mapa(&sh.drain, 0));
    bwait_unwind(&sh.drain, 0, p.wait_limit_ns);
  } else if (warp >= 2 && warp < CTRL_WARP) {
    // =============================== epilogue ================================
    const int q = warp & 3;
    const int g = (warp - 2) >> 2;
    uint32_t Y = 0, eb[2] = {0, 0};
    const uint32_t tbase = sh.tmem_base;
    float* slab = p.slab + (size_t)cta * (256 * 256);
    // the leader's barriers and counters (this CTA's own when it leads)
    const uint32_t L_tempty0 = mapa(&sh.tempty[0], 0), L_tempty1 = mapa(&sh.tempty[1], 0);
    while (true) {
      const int sl = Y % RING;
      if (!bwait(&sh.efull[sl], (Y / RING) & 1, p, sh)) break;
      const EpiJob j = sh.epi[sl];
      const uint32_t L_eempty = mapa(&sh.eempty[sl], 0);
      if (j.action == E_EXIT) {
        __syncwarp();
        if (lane == 0) arrive_cluster(L_eempty);
        break;
      }
      // TMEM lane = this CTA's C column 128*rank + 32q + lane of each 256-wide
      // half, column = C row
      const uint32_t tcol = tbase + ((uint32_t)(32 * q) << 16) + (uint32_t)j.buf * 256;
      const int nh = j.wide ? 2 : 1;
      auto slab_blk = [&](int hh, int blk) { return slab + (size_t)((hh * 8 + blk) * 4 + q) * 1024; };
      if (j.action == E_RESTORE) {
        const long long r0 = globaltimer_ns();
#pragma unroll 1
        for (int bb = g; bb < 8 * nh; bb += 2) {
          const int hh = bb >> 3, blk = bb & 7;
          const float4* s4 = reinterpret_cast<const float4*>(slab_blk(hh, blk));
          uint32_t v[32];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 x = s4[i * 32 + lane];
            v[4 * i] = __float_as_uint(x.x);
            v[4 * i + 1] = __float_as_uint(x.y);
            v[4 * i + 2] = __float_as_uint(x.z);
            v[4 * i + 3] = __float_as_uint(x.w);
          }
          tc::st_32x32b_x32(tcol + hh * 256 + blk * 32, v);
        }
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          arrive_cluster(mapa(&sh.tres[j.buf], 0));
          if (p.q.ckpt != nullptr) {
            atomicAdd(&p.q.ckpt[2], (unsigned long long)(globaltimer_ns() - r0));
            atomicAdd(&p.q.ckpt[3], (unsigned long long)nh * 4 * 4096);
          }
        }
      } else {
        if (!bwait(&sh.tfull[j.buf], eb[j.buf] & 1, p, sh)) break;
        ++eb[j.buf];
        tc::fence_after_sync();
        const long long s0 = globaltimer_ns();
        const int lim = 8 * nh;
        // rows past the job's valid rows, and this CTA's columns when the
        // job's valid columns end before them, are neither stored nor summed
        const bool cols_ok = 128 * (int)rank < j.ncols;
        auto valid = [&](int bb) { return !(j.action == E_STORE_C && ((bb & 7) * 32 >= j.e || !cols_ok)); };
        auto next = [&](int bb) {
          bb += 2;
          while (bb < lim && !valid(bb)) bb += 2;
          return bb;
        };
        // task mode: this lane's sum(c^2) of its column, rows in order, in
        // fp32 (the same order and grouping as the one-CTA kernel)
        float csum = 0.0f;
        auto tload = [&](int bb, uint32_t(&v)[32]) { tc::ld_32x32b_x32(tcol + (bb >> 3) * 256 + (bb & 7) * 32, v); };
        auto consume = [&](int bb, const uint32_t(&v)[32]) {
          const int hh = bb >> 3, blk = bb & 7;
          if (j.action == E_SPILL) {
            float4* s4 = reinterpret_cast<float4*>(slab_blk(hh, blk));
#pragma unroll
            for (int i = 0; i < 8; ++i)
              s4[i * 32 + lane] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                              __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
            return;
          }
          const int col = j.col0 + 256 * hh + 128 * (int)rank + 32 * q + lane;
          if (j.action == E_STORE_C) {
            float* dst = p.C + (size_t)(j.row0 + blk * 32) * p.ldc + col;
#pragma unroll
            for (int i = 0; i < 32; ++i) dst[(size_t)i * p.ldc] = __uint_as_float(v[i]);
            if (p.task_mode) {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const float x = __uint_as_float(v[i]);
                csum = fmaf(x, x, csum);
              }
            }
          } else {
            float* dst = p.Cu + (size_t)j.e * p.cu_stride + (size_t)(j.row0 + blk * 32) * p.ldcu + col;
            if (p.usplit == 1) {
#pragma unroll
              for (int i = 0; i < 32; ++i) dst[(size_t)i * p.ldcu] = __uint_as_float(v[i]);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) atomicAdd(dst + (size_t)i * p.ldcu, __uint_as_float(v[i]));
            }
          }
        };
        bool released = false;
        auto release = [&]() {
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) {
            arrive_cluster(j.buf == 0 ? L_tempty0 : L_tempty1);
            if (j.wide) arrive_cluster(L_tempty1);
            if (j.action == E_SPILL && p.q.ckpt != nullptr) {
              atomicAdd(&p.q.ckpt[0], (unsigned long long)(globaltimer_ns() - s0));
              atomicAdd(&p.q.ckpt[1], (unsigned long long)nh * 4 * 4096);
            }
          }
          released = true;
        };
        uint32_t va[32], vb[32];
        int cur = valid(g) ? g : next(g);
        if (cur < lim) tload(cur, va);
        while (cur < lim) {
          tc::wait_ld();
          int nxt = next(cur);
          if (nxt < lim) tload(nxt, vb); else release();
          consume(cur, va);
          cur = nxt;
          if (cur >= lim) break;
          tc::wait_ld();
          nxt = next(cur);
          if (nxt < lim) tload(nxt, va); else release();
          consume(cur, vb);
          cur = nxt;
        }
        if (!released) release();  // no block of this warp had valid rows
        if (j.action != E_SPILL) {
          if (p.task_mode && j.action == E_STORE_C) {
            double sd = (double)csum;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sd += __shfl_xor_sync(0xffffffffu, sd, o);
            if (lane == 0) sh.chk_part[sl][warp - 2] = sd;
          }
          // the job's stores are visible before it is counted
          __threadfence();
          __syncwarp();
          if (p.task_mode && j.action == E_STORE_C && lane == 0 &&
              atomicAdd(&sh.cta_cnt[sl], 1) == EPI_WARPS - 1) {
            // task mode: the last of this CTA's 8 warps accounts for its
            // 128-column half (checksum in the fixed warp order)
            sh.cta_cnt[sl] = 0;
            if (cols_ok) {
              double sum = 0.0;
              for (int w = 0; w < EPI_WARPS; ++w) sum += sh.chk_part[sl][w];
              p.chk[j.task + rank] = sum;
              ++sh.tiles;
              if (ORACLE && p.q.exec_count != nullptr) atomicAdd(&p.q.exec_count[j.task + rank], 1);
            }
          }
          // the last of the pair's 16 epilogue warps does the job's accounting
          if (lane == 0 && atom_add_cluster(mapa(&sh.epi_cnt[sl], 0), 1u) == 2 * EPI_WARPS - 1) {
            st_cluster_u32(mapa(&sh.epi_cnt[sl], 0), 0u);
            if (j.action == E_STORE_C) {
              if (!p.task_mode) {
                atom_add_cluster_u64(mapa(&sh.tiles, 0), 1ull);
                if (ORACLE && p.q.exec_count != nullptr) atomicAdd(&p.q.exec_count[j.task], 1);
                if (p.st.done != nullptr)
                  stream_tile_done(p.st, p.total_tiles / p.tiles_n, p.tiles_n, j.row0 / BM, j.col0 / BN);
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
      if (lane == 0) arrive_cluster(L_eempty);
      ++Y;
    }
  } else if (warp == CTRL_WARP && lane == 0 && leader) {
    // ================================ control =================================
    // device setter: the leader in slot 0 (under CLC its state passes from
    // one slot-0 holder to the next)
    int nextEv = 0;
    long long gBase = 0;
    if (CLC && cta == 0 && p.q.setter_state != nullptr) {
      nextEv = (int)p.q.setter_state[0];
      gBase = p.q.setter_state[1];
    }
    const int* flag = flag_copy(p.ev, cta);
    // the abort word: every 16th pass (a stop also writes -1 into every
    // flag copy); once seen it holds
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
      __nanosleep(64);
    }
    if (CLC && cta == 0 && p.q.setter_state != nullptr) {
      p.q.setter_state[0] = nextEv;
      p.q.setter_state[1] = gBase;
    }
  }

  // Teardown: every role of both CTAs is done (MMAs drained by the leader,
  // loads landed); the pair meets, releases TMEM together, and meets again
  // so that no remote access reaches a CTA that has exited.
  tc::fence_before_sync();
  __syncthreads();
  __syncwarp();
  cluster_sync();
  if (warp == 1) {
    tc::fence_after_sync();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(sh.tmem_base) : "memory");
  }
  __syncthreads();
  __syncwarp();
  cluster_sync();
  if (tid == 0) {
    // task mode: each CTA counted its own 128-column halves
    const unsigned long long mine = (leader || p.task_mode) ? sh.tiles : 0ull;
    if (CLC) atomicAdd(&p.q.tiles_done[cta], mine);  // the slot's earlier holders counted theirs
    else p.q.tiles_done[cta] = mine;
    atomicMax(p.q.end_max, (unsigned long long)globaltimer_ns());
    atomicAdd(p.q.exited, 1);
    if (CLC && leader) {
      // last: both CTAs' logs are written (the cluster barrier above)
      __threadfence();
      slot_release(p.q.slot_bits, sh.slot);
    }
  }
}

// ---------------------------------------------------------------------------

template <int POLL, int DISC, bool ORACLE, class PGEO, int SCHED = SCH_QUEUE>
static const void* kernel_ptr() {
  return reinterpret_cast<const void*>(&gemm_bf16_pair<POLL, DISC, ORACLE, PGEO, SCHED>);
}

// tasks: the task-list ring geometry (PgTasks), else PgPlain; clc: cluster
// launch control (plain drains, drain discipline)
static const void* select_kernel(int poll, int disc, bool oracle, bool tasks, bool clc = false) {
  if (clc) {
    if (tasks || disc != DISC_DRAIN) return nullptr;
#define APK_SELC(PL, OR) \
  if (poll == PL && oracle == OR) return kernel_ptr<PL, DISC_DRAIN, OR, PgPlain, SCH_CLC>();
    APK_SELC(POLL_OFF, false)
    APK_SELC(POLL_OFF, true)
    APK_SELC(POLL_BOUNDARY, false)
    APK_SELC(POLL_BOUNDARY, true)
    APK_SELC(POLL_STAGE, false)
    APK_SELC(POLL_STAGE, true)
#undef APK_SELC
    return nullptr;
  }
#define APK_SEL(PL, DS, OR)                                                   \
  if (poll == PL && disc == DS && oracle == OR)                               \
    return tasks ? kernel_ptr<PL, DS, OR, PgTasks>() : kernel_ptr<PL, DS, OR, PgPlain>();
  APK_SEL(POLL_OFF, DISC_DRAIN, false)
  APK_SEL(POLL_OFF, DISC_DRAIN, true)
  APK_SEL(POLL_BOUNDARY, DISC_DRAIN, false)
  APK_SEL(POLL_BOUNDARY, DISC_DRAIN, true)
  APK_SEL(POLL_STAGE, DISC_DRAIN, false)
  APK_SEL(POLL_STAGE, DISC_DRAIN, true)
  APK_SEL(POLL_STAGE, DISC_POISON, false)
  APK_SEL(POLL_STAGE, DISC_POISON, true)
#undef APK_SEL
  return nullptr;
}

int smem_bytes(bool tasks) { return tasks ? PgTasks::SMEM_BYTES : PgPlain::SMEM_BYTES; }
int stages(bool tasks) { return tasks ? PgTasks::S : PgPlain::S; }
int threads() { return NT; }
int epi_warps() { return EPI_WARPS; }
size_t params_bytes() { return sizeof(F32Params); }

// *pairs = clusters of two that can be resident at once (0: the kernel does
// not run here).
// Both ring geometries are prepared: a context learns of a task list after
// it is created.  clc: the cluster-launch-control kernel instead (plain
// drains only).
cudaError_t prepare(int poll, int disc, bool oracle, int sms, int* pairs, bool clc) {
  *pairs = 0;
  const void* k = select_kernel(poll, disc, oracle, false, clc);
  const void* kt = clc ? k : select_kernel(poll, disc, oracle, true);
  if (!k || !kt) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, PgPlain::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kt, cudaFuncAttributeMaxDynamicSharedMemorySize, PgTasks::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kt, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(sms - (sms & 1));
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = PgPlain::SMEM_BYTES;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  e = cudaOccupancyMaxActiveClusters(pairs, k, &cfg);
  if (e != cudaSuccess) return e;
  int tpairs = 0;
  cfg.dynamicSmemBytes = PgTasks::SMEM_BYTES;
  e = cudaOccupancyMaxActiveClusters(&tpairs, kt, &cfg);
  if (tpairs < *pairs) *pairs = tpairs;
  return e;
}

// grid: CTAs (two per cluster); under CLC one cluster per task
cudaError_t launch(const F32Params& prm, int grid, int poll, int disc, bool oracle, bool clc, cudaStream_t stream) {
  const bool tasks = prm.task_mode != 0;
  const void* k = select_kernel(poll, disc, oracle, tasks, clc);
  if (!k || grid % 2) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = tasks ? PgTasks::SMEM_BYTES : PgPlain::SMEM_BYTES;
  cfg.stream = stream;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  void* args[] = {const_cast<F32Params*>(&prm)};
  return cudaLaunchKernelExC(&cfg, k, args);
}

}  // namespace bf16pair
}  // namespace apk
