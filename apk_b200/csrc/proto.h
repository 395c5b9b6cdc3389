// Device-memory protocol between the host runtime and the persistent
// kernels.  It restates the reference's kernel-argument "ABI"
// (src/yield.cu:95-102: nextTask fetch-add counter, generation flag,
// claim[] CAS array, uqNext[] urgent mini-queue, setGT/obsGT/uGT timestamp
// arrays, uEndMax) as two structs, plus what the reference does not have:
// a checkpoint slab, a device status word and a bounded-wait limit.
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace apk {

enum PollMode : int { POLL_OFF = 0, POLL_BOUNDARY = 1, POLL_STAGE = 2 };
enum Discipline : int { DISC_DRAIN = 0, DISC_POISON = 2 };

// Yield-event side of the protocol (src/yield.cu:95-102,148-195).
// The generation is kept in flag_lines copies, one per 128-byte line
// (flag + FLAG_STRIDE * i); the setter writes every copy and CTA c polls copy
// c % flag_lines.  1184 CTAs (8 per SM) polling one line every 512 ns cost
// the drain a fifth of its speed; spread over 32 lines, the cost is that of
// no flag load at all.
constexpr int FLAG_LINES = 32, FLAG_STRIDE = 32;

struct EventProto {
  int* flag;                   // generation counter; -1 = stop.  Device memory
                               // or mapped pinned host memory.
  int flag_lines;              // copies of it at flag + FLAG_STRIDE * i (1: flag only)
  int* abort_word;             // device memory; nonzero makes every CTA exit
  int* status;                 // device memory; first device-side error code
  const long long* sched_ns;   // device setter: cumulative offsets (nullptr = host sets)
  int n_sched;
  int max_events;
  long long* set_ns;           // [max_events] globaltimer at the device setter's store
  long long* obs_ns;           // [max_events * grid] per-CTA observation time
  int* claim;                  // [max_events] first popper's CTA index + 1
  int* claim_site;             // [max_events] stage index of the claim, -1 = tile boundary
  int* inflight;               // [max_events] TMA stages in flight when the claimer yielded
  long long* claim_ns;         // [max_events] globaltimer of the claim
  unsigned long long* done_ns; // [max_events] atomicMax of urgent item completion times
  int* uq_next;                // [max_events] urgent mini-queue pop counter
  int* udone_cnt;              // [max_events] finished urgent items
  int* ack;                    // mapped host memory [2*max_events]: claim ack, done ack
  int* uexec;                  // oracle: [max_events] urgent item executions
  // count-triggered events: event k fires when the completed-tile counter
  // reaches count_trig[k] (deterministic yields for verification runs)
  const unsigned long long* count_trig;
  int n_count;
  unsigned long long* completed;
};

// The copy of the generation CTA (or resident slot) c polls.
__device__ __forceinline__ const int* flag_copy(const EventProto& ev, int c) {
  return ev.flag + (ev.flag_lines > 1 ? FLAG_STRIDE * (c % ev.flag_lines) : 0);
}

// Device setter: raise the generation from `from` to from + 1 in every copy:
// plain stores to copies 1.. (a compare-and-swap per copy waited out each
// one's round trip: the last copy landed ~10 us late), then a compare-and-
// swap on copy 0, which never overwrites the -1 stop sentinel there.  A stop
// racing the raise can leave a later copy at the generation; every poller
// also reads the abort word, which the stop sets too.
__device__ __forceinline__ void flag_raise(const EventProto& ev, int from) {
  for (int i = 1; i < ev.flag_lines; ++i)
    asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(ev.flag + FLAG_STRIDE * i), "r"(from + 1) : "memory");
  atomicCAS(ev.flag, from, from + 1);
}

// Background work-queue side (src/persistent.cu:51-79 fetch-add queue).
struct QueueProto {
  unsigned long long* next_task;
  unsigned long long num_tasks;
  int* exec_count;               // oracle: [num_tasks] executions per task id
  unsigned long long* tiles_done;  // [grid] completed background tiles per CTA
  unsigned long long* start_min;   // atomicMin of CTA start globaltimer
  unsigned long long* end_max;     // atomicMax of CTA exit globaltimer
  int* exited;
  unsigned long long* yields;      // checkpoints taken (accumulator spills)
  // cluster launch control scheduler: one CTA per task; per-CTA logs,
  // counters and checkpoint slabs are indexed by a resident slot taken from
  // this bitmap at CTA start and returned at exit (CTAs come and go)
  unsigned* slot_bits;             // [(nslots + 31) / 32]
  int nslots;                      // resident CTAs (sms * ctas_per_sm)
  long long* setter_state;         // [2] device setter's next event and time base across slot-0 holders
  // checkpoint accounting (bf16): [0] spill ns, [1] spill bytes, [2] restore
  // ns, [3] restore bytes, each summed over the epilogue warps; a warp's time
  // runs from its first accumulator read to its last write (nullptr = off)
  unsigned long long* ckpt;
};

// Streamed operands (apk_gemm from host memory): A arrives in row panels of
// panel_tm tile rows and B in column panels of b_units 128-column units
// while the kernel runs, interleaved so that the count of computable tiles
// grows with the bytes copied; the kernel visits tiles in the order they
// become computable (order[]), starts one once its A row panel and B column
// panel(s) are flagged, and acknowledges each finished C block (a row panel
// by cb_tn tile columns) to the host for its copy back.
struct StreamProto {
  const int* a_ready;     // [n_panels] set by the copy stream after A panel p (nullptr = resident)
  const int* b_ready;     // [N / (128 * b_units)] after B column panel j
  int b_units;            // 128-column units per B column panel
  int panel_tm;           // tile rows per A row panel and per C block
  int n_panels;
  int cb_tn;              // tile columns per C block
  int n_cb;               // C blocks across
  const unsigned* order;  // [tiles] visit order as tm * tiles_n + tn (nullptr = grouped raster)
  unsigned* done;         // [n_panels * n_cb] finished tiles per C block
  int* ack;               // mapped host memory [n_panels * n_cb]: C block complete
  // K slices (warp-specialized fp32 kernel only; 0 or 1 = whole K).  With
  // ksplit = 2 the operands move as K halves: ready flags are indexed
  // panel * ksplit + slice, order[] entries are (tile * ksplit + slice), and
  // a tile runs as two chained jobs: slice 0 leaves its accumulators in
  // part[] and raises part_ready once per compute warp, slice 1 starts from
  // them.  Each element sees the same FMA sequence as an unsplit tile.
  int ksplit;
  float* part;            // [tiles][BM * BN] slice-0 accumulators, row-major per tile
  int* part_ready;        // [tiles] compute warps of slice 0 that stored theirs
};

// Count a finished background tile of a streamed run; the last tile of a C
// block acknowledges the block to the host.  The tile's stores are fenced.
__device__ __forceinline__ void stream_tile_done(const StreamProto& st, int tiles_m, int tiles_n, int tm, int tn) {
  const int pn = tm / st.panel_tm, cb = tn / st.cb_tn;
  const int rows = tiles_m - pn * st.panel_tm < st.panel_tm ? tiles_m - pn * st.panel_tm : st.panel_tm;
  const int cols = tiles_n - cb * st.cb_tn < st.cb_tn ? tiles_n - cb * st.cb_tn : st.cb_tn;
  const int b = pn * st.n_cb + cb;
  if (atomicAdd(&st.done[b], 1u) + 1u == (unsigned)(rows * cols)) {
    // the host reads the block with a copy engine once it sees the ack in
    // mapped host memory: a system-scope fence orders every tile's C stores
    // (each made visible at GPU scope before it was counted) before the ack,
    // and a second one pushes the ack out now
    __threadfence_system();
    *reinterpret_cast<volatile int*>(&st.ack[b]) = 1;
    __threadfence_system();
  }
}

// Tile coordinates of a streamed run's tile-visit slot.
__device__ __forceinline__ void stream_tile(const StreamProto& st, int tile, int tiles_n, int& tm, int& tn) {
  const int o = (int)st.order[tile];
  tm = o / tiles_n;
  tn = o - tm * tiles_n;
}

// K slices of a streamed run (1 unless the host split K).
__device__ __forceinline__ int stream_ksplit(const StreamProto& st) { return st.ksplit > 1 ? st.ksplit : 1; }

// Tile coordinates and K slice of a streamed run's visit slot.
__device__ __forceinline__ void stream_job(const StreamProto& st, int slot, int tiles_n, int& tm, int& tn,
                                           int& slice) {
  const int ks = stream_ksplit(st);
  const int o = (int)st.order[slot];
  slice = o % ks;
  const int t = o / ks;
  tm = t / tiles_n;
  tn = t - tm * tiles_n;
}

// One heterogeneous background task: C window = A window *
// B window, each a window of a shared operand pool (so the tensor maps are
// fixed).  Layout-identical to apk_task in include/apk.h.
struct TaskDesc {
  int m, n, k;
  int a_row0, a_k0;
  int b_k0, b_col0;
  int c_row0, c_col0;
  int flags;
  long long chk_base;  // checksum index of the task's tile (0,0); tile (tm,tn) at +tm*tiles_n+tn
};

// Kernel parameters (both kernels; the fp32 kernel ignores the task-mode
// fields).
struct F32Params {
  CUtensorMap tmA;   // background A [M][K]  (fp32: 128 rows x 32 k boxes; bf16: 128 x BK, swizzled)
  CUtensorMap tmB;   // background B [K][N]  (fp32: BK x 128 boxes; bf16: BK x 64, 128B swizzle)
  CUtensorMap tmAu;  // urgent A
  CUtensorMap tmBu;  // urgent B
  // bf16 one-CTA kernel, background jobs: A as one box of the tile's rows
  // (up to 256), B as one 3-D box {64 n, BK k, chunks} of the view
  // [N/64][K][64] (4 chunks for 256-wide jobs, else 2), so a ring slot takes
  // two TMA loads; the shared-memory layout is that of the per-box loads
  CUtensorMap tmAw;
  CUtensorMap tmBw;
  float* C;
  int ldc, tiles_n, total_tiles, nk;   // nk = K / BK (ring slots per tile)
  int poll_every;                      // ring slots per stage-level yield site:
                                       // the K-tile (depth between yield sites)
                                       // over the ring slot's K depth
  float* Cu;                           // urgent output, one slot per event
  long long cu_stride;                 // floats between event slots
  int ldcu, utiles_n, usplit, unk, uitems;  // unk = stages per urgent item
  float* slab;                         // [grid][16][256] float4 accumulator checkpoints
  long long* slab_hdr;                 // [grid][4]: task, stage cursor, event, valid
  // task mode (bf16): queue entries index `work` (task << 12 | tm << 6 | tn);
  // A/B/C maps cover the pools; each finished tile writes sum(c^2) to chk
  const unsigned* work;
  const TaskDesc* tasks;
  double* chk;
  int task_mode;
  // bf16 one-CTA kernel: narrow_all runs background and urgent work as
  // 256x128 jobs (each holds one of the two TMEM buffers); park keeps a
  // yielding background job's accumulator in its buffer (the urgent items
  // use the other one) instead of spilling it to the slab
  int narrow_all, park;
  long long wait_limit_ns;
  EventProto ev;
  QueueProto q;
  StreamProto st;
};

// A kernel geometry as the host sees it: output tile, threads per CTA, the
// K depth and count of the ring slots, the K depth of one A box, dynamic
// shared memory.  fp32 block-synchronous geometries (sgemm_f32.cu): L32 and
// L64 (128x128 tiles, 32- or 64-deep slots), M (64x128) and S (32x128) for
// 4 and 8 resident CTAs per SM.
struct GeoInfo {
  int tile_m, tile_n, threads, slot_k, stages, a_box_k, smem_bytes;
};
enum F32Geo : int { F32_GEO_L32 = 0, F32_GEO_L64 = 1, F32_GEO_M = 2, F32_GEO_S = 3 };
// bf16 one-CTA kernel geometries (gemm_bf16.cu): STD (256x256 tiles, one CTA
// per SM, 64- or 32-deep slots) and N256 / N128 / N64 (256x128, 128x128,
// 64x128 tiles for 2, 4 and 8 resident CTAs per SM).
enum BF16Geo : int {
  BF16_GEO_STD64 = 0, BF16_GEO_STD32 = 1, BF16_GEO_N256x64 = 2, BF16_GEO_N256x32 = 3, BF16_GEO_N128 = 4,
  BF16_GEO_N64 = 5
};

// Visibility microbenchmark parameters (the flag-notification probe of
// src/yield.cu:227-293, decoupled from tile work).
struct VisParams {
  int* flag;                  // generation word; CTA 0 raises it on schedule, -1 ends the run
  const long long* sched_ns;  // cumulative event offsets from CTA 0's start
  int n_events;
  long long* set_ns;          // [n_events] globaltimer of each raise
  long long* obs_ns;          // [n_events][grid] first observation per CTA
  long long* iters;           // [grid] polling iterations per CTA
  long long* t_begin;         // [grid] globaltimer at CTA start / end
  long long* t_end;
  int work_iters;             // dependent FMA chain per iteration (known cadence)
  const float4* traffic;      // loaded variant: streamed operand, far larger than L2
  unsigned long long traffic_n4;
  float* sink;                // [grid * threads] keeps the work live
  long long tail_ns;          // CTA 0 stores -1 this long after the last event
  long long limit_ns;         // every CTA leaves after this long, whatever the flag says
  int* status;                // DEV_WAIT_TIMEOUT_SPIN if a CTA hit limit_ns
};

}  // namespace apk
