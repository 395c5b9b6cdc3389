/*
 * apk.h -- C ABI of the B200 preemptible persistent-GEMM runtime (libapk.so).
 *
 * The reference (AyaanFaisal21/APK) has no library: its boundary is the
 * device-memory protocol between each binary's main() and its persistent
 * kernel, plus the binaries' --mode switches.  Each entry point below names
 * the reference code it replaces (paths relative to the reference root).
 *
 * Conventions
 *   - Every function returns apk_status; APK_OK == 0.  No exceptions cross
 *     the ABI.  apk_last_error() returns a message for the last failure.
 *   - Plain pointers and sizes only.  Buffers passed with APK_MEM_HOST are
 *     caller-owned host memory the runtime copies from/to; APK_MEM_DEVICE
 *     buffers are caller-owned device memory used in place.
 *   - One context per device per host thread.  apk_inject_urgent and
 *     apk_stop may be called from a second host thread while a launch runs.
 *   - Every device-side wait is bounded (apk_config.wait_limit_ns); a wait
 *     that runs out is reported as APK_EDEVICE, never as a hung GPU.
 *   - Matrices are row-major.  fp32: M, N multiples of 128, K a multiple of
 *     k_tile.  bf16: M a multiple of 256, N of 128, K of k_tile.
 */
#ifndef APK_H_
#define APK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define APK_ABI_VERSION 4
#define APK_TASKS_UNBOUNDED 0xFFFFFFFFFFFFFFFFull

typedef enum apk_status {
  APK_OK = 0,
  APK_EINVAL = 1,       /* bad argument (shape, null pointer, mode)          */
  APK_ECUDA = 2,        /* a CUDA call failed (message in apk_last_error)    */
  APK_ETIMEDOUT = 3,    /* apk_wait deadline passed; the kernel still runs   */
  APK_ESTATE = 4,       /* call not valid now (e.g. launch while running)    */
  APK_EDEVICE = 5,      /* the kernel reported an error (bounded wait ended) */
  APK_ENOMEM = 6,
  APK_EUNSUPPORTED = 7
} apk_status;

typedef enum apk_dtype { APK_F32 = 0, APK_BF16 = 1 } apk_dtype;

/* Poll sites: src/midyield.cu:89 / src/tcyield.cu:88 (OFF, BOUNDARY, STAGE). */
typedef enum apk_poll_mode {
  APK_POLL_OFF = 0,
  APK_POLL_BOUNDARY = 1,
  APK_POLL_STAGE = 2
} apk_poll_mode;

/* Disciplines: src/midyield.cu:90 (DRAIN, POISON; NAIVE is not built). */
typedef enum apk_discipline { APK_DISC_DRAIN = 0, APK_DISC_POISON = 2 } apk_discipline;

/* Who sets the yield flag.  DEVICE: CTA 0 at scheduled globaltimer offsets
 * (src/yield.cu:186-195, the reference's primary instrument).  HOST_MEMCPY
 * (default host path): the host copies the generation into device memory
 * with cudaMemcpyAsync on a high-priority control stream
 * (src/yield.cu:851-852).  HOST_MAPPED: the host stores it into mapped
 * pinned memory that every CTA polls across PCIe -- kept for measurement
 * only: with one poll per stage per CTA it costs most of the background
 * throughput. */
typedef enum apk_set_mode {
  APK_SET_DEVICE = 0,
  APK_SET_HOST_MAPPED = 1,
  APK_SET_HOST_MEMCPY = 2
} apk_set_mode;

typedef enum apk_mem_kind { APK_MEM_HOST = 0, APK_MEM_DEVICE = 1 } apk_mem_kind;

/* How background tasks reach CTAs.  QUEUE: a persistent grid of resident
 * CTAs popping a global fetch-add counter (src/persistent.cu:51-79).  CLC
 * (fp32 128x128 tiles, the one-CTA bf16 kernel with task lists included,
 * and the bf16 CTA pairs for plain drains; drain discipline, bounded
 * launches of < 2^30 tasks): one CTA -- or one cluster of two -- per task,
 * running CTAs take not-yet-launched ones' tasks through Blackwell cluster
 * launch control (on pairs the leader cancels a cluster and relays its
 * tile to the peer); when the hardware declines (a higher-priority
 * stream's kernel is waiting) CTAs exit and free their SMs, and the rest of
 * the grid launches later.  The cooperative yield works the same under
 * both. */
typedef enum apk_scheduler { APK_SCHED_QUEUE = 0, APK_SCHED_CLC = 1 } apk_scheduler;

/* fp32 kernel.  WARP_SPECIALIZED: one 384-thread CTA per SM runs two
 * 128x128 workers (compute warps fed by a TMA producer warp per worker, a
 * control warp for the flag); it serves the queue scheduler with exactly
 * two workers per SM (32-deep ring slots, a yield site every k_tile / 32
 * slots).  BLOCK_SYNC: 128-thread CTAs, one block barrier per stage; it
 * serves every configuration (CLC, one CTA per SM with 64-deep slots at
 * K-tile 64 or 128, 4 and 8 CTAs per SM, reduced grids).  AUTO picks WARP_SPECIALIZED where it applies.
 * Both compute every C element with the same FMA sequence: bitwise-equal
 * outputs.  In the warp-specialized kernel a "CTA" of the grid, the event
 * log, tile counters and checkpoint slabs is a worker. */
typedef enum apk_f32_kernel {
  APK_F32_AUTO = 0,
  APK_F32_WARP_SPECIALIZED = 1,
  APK_F32_BLOCK_SYNC = 2
} apk_f32_kernel;

/* bf16 kernel.  PAIR: clusters of two CTAs compute 256x512 output tiles
 * with cta_group::2 MMAs (each CTA stages half the operands and holds half
 * the accumulators); it serves a background GEMM with N a multiple of 256,
 * the urgent N a multiple of 256, K-tile 64 or 128, one CTA per SM, and --
 * when asked for by PAIR -- task lists (256x256 jobs, one accumulator per
 * CTA; slower there than SINGLE).  SINGLE: one CTA per 256x256 tile; serves
 * every shape, task mode and K-tile 32.  AUTO picks PAIR for a plain
 * background GEMM where it applies.  info.tile_n reports 512 for PAIR. */
typedef enum apk_bf16_kernel {
  APK_BF16_AUTO = 0,
  APK_BF16_PAIR = 1,
  APK_BF16_SINGLE = 2,
  /* (ABI 4) one CTA per SM, every background and urgent job 256x128 (one
   * of the two 256-column TMEM buffers each, so a job's epilogue overlaps
   * the next job's MMAs).  NARROW parks a yielding background job's
   * accumulator in its buffer while the urgent items use the other one:
   * nothing is spilled or restored.  NARROW_SPILL checkpoints it to the
   * slab like the other kernels (the comparison arm). */
  APK_BF16_NARROW = 3,
  APK_BF16_NARROW_SPILL = 4
} apk_bf16_kernel;

typedef struct apk_config {
  int device;
  apk_dtype dtype;
  int ctas_per_sm;          /* 0 = as many as fit (full residency).  fp32: 4
                               or 8 select 64x128 or 32x128 output tiles (a
                               CTA of two warps or one, 16-deep ring slots);
                               bf16: 2, 4 or 8 select 256x128, 128x128 or
                               64x128 tiles with one TMEM buffer each, so
                               that many CTAs fit on an SM                    */
  int grid;                 /* 0 = SMs * ctas_per_sm                          */
  int k_tile;               /* 32, 64 or 128: the K depth between two
                               stage-level yield sites (the pipeline stage);
                               0 = the dtype's default (fp32 32, bf16 64).
                               The ring moves it in slots of the kernel's own
                               depth (apk_device_info.slot_k)                 */
  apk_poll_mode poll;
  apk_discipline discipline;
  apk_set_mode set_mode;
  int max_events;           /* capacity of the event log                      */
  int oracle;               /* 1 = count executions per task and per event    */
  int urgent_split_k;       /* urgent items per urgent output tile            */
  long long wait_limit_ns;  /* bound on every device-side wait                */
  apk_scheduler scheduler;  /* (ABI 2) background work distribution           */
  apk_f32_kernel f32_kernel;/* (ABI 3) fp32 kernel choice                       */
  apk_bf16_kernel bf16_kernel;/* (ABI 3) bf16 kernel choice                     */
} apk_config;

/* Fill *cfg with the defaults (fp32, full residency, default k_tile, stage
 * polling, drain, host-set flag through cudaMemcpyAsync, 4096
 * events, urgent split-K 8, 2 s waits). */
void apk_config_default(apk_config* cfg);

typedef struct apk_ctx apk_ctx;

/* Replaces each binary's setup: device query, occupancy-derived grid and
 * control-array allocation (src/yield.cu:349-400, src/persistent.cu:110-151). */
apk_status apk_create(const apk_config* cfg, apk_ctx** out);
apk_status apk_destroy(apk_ctx* ctx);
const char* apk_last_error(const apk_ctx* ctx);

typedef struct apk_device_info {
  int sms;
  int grid;                 /* CTAs of the persistent kernel (warp-specialized
                               fp32: workers, two per 384-thread CTA)         */
  int ctas_per_sm;          /* resident CTAs per SM actually used             */
  int max_ctas_per_sm;      /* occupancy limit of the selected kernel         */
  int cc_major, cc_minor;
  int smem_per_cta;
  int threads_per_cta;
  int tile_m, tile_n, k_tile, stages; /* output tile (the unit of the queue and
                                         of the grid's per-CTA accounting):
                                         fp32 128x128; bf16 256x256 (the last
                                         tile of a row 128 wide when N is an
                                         odd multiple of 128), or 256x512 per
                                         CTA pair with the CTA-pair kernel    */
  char name[128];
  int slot_k;               /* (ABI 4) K depth of one ring slot; a stage-level
                               yield site comes every k_tile / slot_k slots  */
} apk_device_info;
apk_status apk_get_info(apk_ctx* ctx, apk_device_info* info);

/* Background GEMM C = A * B.  Replaces the operand set-up and upload of
 * src/persistent.cu:132-151 and src/yield.cu:367-396.  For APK_MEM_HOST the
 * runtime owns device copies; for APK_MEM_DEVICE it uses the caller's
 * buffers (C must stay valid until the launch ends). */
apk_status apk_set_background(apk_ctx* ctx, const void* A, const void* B, void* C, int M, int N,
                              int K, apk_mem_kind kind);

/* The urgent GEMM every event runs (the reference's urgent tile,
 * src/yield.cu:163-178 and src/urgent_baseline.cu:101-112, generalised to
 * an M x N x K GEMM split into work items).  Each event writes its own
 * output slot. */
apk_status apk_set_urgent(apk_ctx* ctx, const void* A, const void* B, int M, int N, int K,
                          apk_mem_kind kind);

/* Start the persistent kernel over num_tasks background tasks (task t
 * computes tile t mod tiles, src/urgent_baseline.cu:78-83), or until
 * apk_stop with APK_TASKS_UNBOUNDED.  Asynchronous.  Replaces the launch
 * and zero_all lambdas of src/yield.cu:400-443. */
apk_status apk_launch(apk_ctx* ctx, unsigned long long num_tasks);

/* Device-set schedule: cumulative offsets (ns) from CTA 0's first poll at
 * which CTA 0 bumps the generation (src/yield.cu:824-834).  Call before
 * apk_launch; n = 0 clears it. */
apk_status apk_schedule_device_events(apk_ctx* ctx, const long long* offsets_ns, int n);

/* Count-triggered device events: event k fires when the k-th count of
 * completed background tiles is reached (counts ascending).  The CTA that
 * completes that tile bumps the generation, so the yield lands at a
 * deterministic point of the drain -- e.g. "one yield after 50% of tiles
 * complete".  Needs set_mode DEVICE; replaces any time schedule; call
 * before apk_launch (n = 0 clears it).  No reference counterpart: the
 * reference fires only at scheduled times (src/yield.cu:186-195). */
apk_status apk_schedule_count_events(apk_ctx* ctx, const unsigned long long* counts, int n);

/* Host-set injection (src/yield.cu:845-856): bump the generation.  Returns
 * the event index and the host steady-clock time of the store. */
apk_status apk_inject_urgent(apk_ctx* ctx, int* event, long long* host_set_ns);

/* Spin (bounded) until the event's claim ack (which = 0) or done ack
 * (which = 1) arrives from the device through mapped memory; returns the
 * host steady-clock time it was seen. */
apk_status apk_wait_ack(apk_ctx* ctx, int event, int which, long long timeout_ns,
                        long long* host_seen_ns);

/* Stop sentinel -1 (src/yield.cu:857-858). */
apk_status apk_stop(apk_ctx* ctx);

/* Wait for the launch to end (src/yield.cu:859) with a deadline:
 * APK_ETIMEDOUT if it is still running, APK_EDEVICE if the kernel
 * reported an error. */
apk_status apk_wait(apk_ctx* ctx, long long timeout_ns);

/* Copy the background C to host memory (src/persistent.cu:216-219). */
apk_status apk_read_output(apk_ctx* ctx, void* C_host);

/* Copy event e's urgent output (M_u x N_u fp32) to host memory. */
apk_status apk_read_urgent_output(apk_ctx* ctx, int event, float* Cu_host);

/* Per-event log (src/yield.cu:862-878).  Every pointer may be NULL; each
 * non-NULL array holds max_events entries (obs_ns: max_events * grid). */
typedef struct apk_event_log {
  int n_injected;           /* host-set events injected in the last launch    */
  int n_fired;              /* device-set events fired in the last launch     */
  int grid;
  long long* set_ns;        /* globaltimer at the device setter's store       */
  long long* host_set_ns;   /* host steady clock at the host store            */
  long long* host_ack_ns;   /* host steady clock when the claim ack was seen  */
  long long* host_done_ns;  /* host steady clock when the done ack was seen   */
  long long* claim_ns;      /* globaltimer of the first successful pop        */
  long long* done_ns;       /* globaltimer of the last finished urgent item   */
  int* claimer;             /* CTA index + 1 of the first popper (0 = none)   */
  int* claim_site;          /* stage index of the claim; -1 = tile boundary   */
  int* inflight;            /* TMA stages in flight at the claimer's yield    */
  long long* obs_ns;        /* [event * grid + cta] observation time, 0=never */
} apk_event_log;
apk_status apk_read_events(apk_ctx* ctx, apk_event_log* log);

/* Exactly-once scheduler verdict inputs (src/yield.cu:576-667).
 * exec_counts: one int per background task id of the last bounded launch
 * -- in task mode one per global tile (checksum index, n_chk ints) --
 * (requires cfg.oracle); uexec_counts: max_events ints. */
apk_status apk_read_oracle(apk_ctx* ctx, int* exec_counts, int* uexec_counts);

typedef struct apk_run_stats {
  long long start_ns, end_ns;        /* first CTA start / last CTA exit       */
  unsigned long long tiles_done;     /* completed background tiles (task mode:
                                        256x128 halves of tiles)              */
  unsigned long long yields;         /* checkpoints (accumulator spills)      */
  double bg_flops;                   /* tiles_done * 2*M*N*K / tiles; task mode: prorated by 256x128 halves */
  double bg_tflops;                  /* bg_flops / (end - start)              */
  int exited;                        /* CTAs that exited                      */
  int device_status;                 /* 0 or the first device error code      */
  double launch_ms;                  /* CUDA events around the launch, on the
                                        stream that ran it                    */
  /* bf16 checkpoint traffic of the launch (0 for fp32): bytes spilled from
   * TMEM to the slab and restored from it, and the CTA wall time of those
   * spills / restores summed over checkpoints (spill: first tcgen05.ld to
   * TMEM free with the slab stores issued; restore: first slab load to
   * tcgen05.st complete).  bytes / ns = a CTA's checkpoint GB/s. */
  unsigned long long ckpt_spill_bytes, ckpt_restore_bytes;
  long long ckpt_spill_ns, ckpt_restore_ns;
  unsigned long long parks;          /* (ABI 4) bf16 NARROW: checkpoints kept in
                                        TMEM instead of spilled               */
} apk_run_stats;
apk_status apk_read_run_stats(apk_ctx* ctx, apk_run_stats* st);

/* One synchronous GEMM through the persistent kernel: upload (host
 * buffers), drain every tile once, download.  Replaces one pass of
 * src/persistent.cu:155-172.  From host buffers the copies overlap the
 * kernel (operand panels in, finished C blocks out); with the
 * warp-specialized fp32 kernel K is taken in two chained slices.  C is
 * bitwise equal to a resident drain of the same operands either way.
 * run_stats.tiles_done counts tiles, not slices. */
apk_status apk_gemm(apk_ctx* ctx, const void* A, const void* B, void* C, int M, int N, int K,
                    apk_mem_kind kind);

/* Copy ceiling of apk_gemm from host memory: the host buffers, device
 * buffers and copy streams of this context's last host-memory apk_gemm,
 * with no kernel.  out_ms[0]: A and B host->device; out_ms[1]: C
 * device->host; out_ms[2]: both at once on their two streams (medians of
 * reps, host clock around the stream synchronisations).  2*M*N*K /
 * out_ms[0] bounds what apk_gemm can reach from host memory.  No reference
 * counterpart (the reference times no transfer). */
apk_status apk_probe_copy(apk_ctx* ctx, const void* A, const void* B, void* C, int reps, double* out_ms);

/* ---- harness modes (the reference binaries' --mode switches) ---------- */

typedef struct apk_latency_config {
  int events;               /* injections                                    */
  long long period_ns;      /* one injection per period at a uniform offset  */
  unsigned seed;
  int warmup_events;        /* discarded (src/yield.cu:340,915)              */
  long long settle_ns;      /* background time before the first injection    */
  unsigned long long bg_tasks; /* 0: run until stopped after the last event;
                                  else a bounded launch of that many tasks
                                  that ends by itself (injection stops when
                                  it ends)                                    */
  int probe_reps;           /* host-set only: visibility-calibration reps
                               before the launch (0 = none: the claim /
                               last_obs / done fields are then NaN and only
                               the rt_* host round trips are reported)     */
  int poisson;              /* 0: one arrival at a uniform offset in every
                               period; 1: Poisson arrivals with
                               mean gap period_ns (configs[4], 2 kHz)      */
} apk_latency_config;

typedef struct apk_latency_result {
  int n;                    /* events counted                                */
  int anomalies;            /* events some CTA never observed                */
  int unclaimed;
  double claim_p50_us, claim_p99_us;        /* set -> urgent work claimed    */
  double last_obs_p50_us, last_obs_p99_us;  /* set -> last CTA observed      */
  double done_p50_us, done_p99_us;          /* set -> urgent work finished   */
  double rt_claim_p50_us, rt_claim_p99_us;  /* host set -> host sees claim   */
  double rt_done_p50_us, rt_done_p99_us;    /* host set -> host sees done    */
  double bg_tflops;         /* background throughput during the run          */
  double vis_offset_ns;     /* host->globaltimer offset used (host-set)      */
} apk_latency_result;

/* Latency mode (src/yield.cu:776-958): unbounded background launch,
 * injections, stop, per-event latencies with nearest-rank percentiles.
 * For host-set modes "set" is the host store mapped to globaltimer with the
 * visibility calibration of src/yield.cu:782-813; rt_* need no mapping. */
apk_status apk_run_latency(apk_ctx* ctx, const apk_latency_config* lc, apk_latency_result* out);

/* Host->device flag visibility calibration (src/yield.cu:782-813):
 * offsets (globaltimer at first device observation - host store time),
 * reps entries.  Needs an idle device. */
apk_status apk_probe_visibility(apk_ctx* ctx, int reps, long long* offsets_ns);

/* Flag-visibility microbenchmark (src/yield.cu:227-293 and its driver,
 * src/yield.cu:466-564): no tile work; every CTA of this context's grid (with
 * the studied kernel's shared memory, so the residency is the same) runs a
 * work_iters-long dependent FMA chain per iteration, optionally streams
 * loads from a traffic_bytes buffer far larger than L2 (loaded = 1: HBM
 * busy), and thread 0 polls the flag; CTA 0 raises it at uniform-random gaps
 * in [gap_min_ns, gap_max_ns] and ends the run itself.  Delays are
 * observation - raise on the device clock, over CTAs 1..grid-1 (CTA 0 sees
 * its own store). */
typedef struct apk_visibility_config {
  int events;
  long long gap_min_ns, gap_max_ns;
  unsigned seed;
  int warmup_events;          /* first events left out of the statistics  */
  int work_iters;             /* FMA chain per polling iteration          */
  int loaded;                 /* 1 = stream HBM traffic while polling     */
  long long traffic_bytes;    /* loaded buffer; 0 = 1 GiB                 */
} apk_visibility_config;

typedef struct apk_visibility_result {
  int n;                      /* events in the statistics                 */
  int unset, anomalies;       /* never raised / not seen by every CTA     */
  double cadence_ns;          /* median CTA's time per polling iteration  */
  /* per event: min / median / p95 / max delay across CTAs; then p50 over
   * events (and p99 of the max) */
  double dmin_p50_us, d50_p50_us, d95_p50_us, dmax_p50_us, dmax_p99_us;
  double hbm_gbs;             /* loaded: bytes streamed / run time        */
  int device_status;          /* DEV_WAIT_TIMEOUT_SPIN if a CTA hit its limit */
} apk_visibility_result;

/* set_ns (events) and obs_ns (events x grid) may be NULL; when given they
 * receive the raw matrix (0 = not observed), e.g. for an OBS1 dump. */
apk_status apk_run_visibility(apk_ctx* ctx, const apk_visibility_config* cfg, apk_visibility_result* out,
                              long long* set_ns, long long* obs_ns);

/* Failure-path self-test: launches the bounded flag spin of
 * apk_probe_visibility on a flag nothing sets, with the given limit.  The
 * kernel must give up, report DEV_WAIT_TIMEOUT_SPIN (3) through its status
 * word and exit; *device_status receives the code.  Returns APK_OK when the
 * spin ended and reported, leaving the context usable.  Replaces the
 * reference's unbounded spin_flag (src/yield.cu:208-214), which would hang
 * on a lost store. */
apk_status apk_selftest_wait_timeout(apk_ctx* ctx, long long limit_ns, int* device_status);

/* Overhead mode (src/yield.cu:670-711): ABAB-interleaved drains of
 * num_tasks tasks with polling as configured vs polling off, warmup pairs
 * discarded; median ms of each and the ratio. */
apk_status apk_run_overhead(apk_ctx* ctx, unsigned long long num_tasks, int reps, double* ms_poll,
                            double* ms_nopoll);

/* No-preemption baseline (src/urgent_baseline.cu:144-343, mode sat):
 * background drain of num_tasks with polling off; the urgent GEMM is a
 * separate kernel on a max-priority stream launched at U(0.2,0.8) of the
 * drain.  Per trial: host arrival -> urgent done (host clock, us). */
apk_status apk_run_baseline(apk_ctx* ctx, unsigned long long num_tasks, int trials, unsigned seed,
                            double* e2e_us);

/* Reserved-capacity arm (src/urgent_baseline.cu:152-175, --reserve R, and
 * the reserved side of scripts/pareto.sh): as apk_run_baseline, but the
 * background runs on grid - reserve CTAs, so `reserve` resident slots stay
 * free and the urgent kernel (one CTA per 128x128 urgent tile) starts in them
 * at once instead of waiting for the drain.  reserve = 0 is the baseline.
 * e2e_us: trials doubles, host arrival -> urgent done; *bg_tflops (may be
 * NULL): the background's rate with the slots held out. */
apk_status apk_run_reserved(apk_ctx* ctx, unsigned long long num_tasks, int reserve, int trials, unsigned seed,
                            double* e2e_us, double* bg_tflops);

/* ---- heterogeneous task queue (configs[4], bf16 contexts) -------------- */

/* One background GEMM task: C window = A window * B window, each a window
 * of a shared operand pool (so 2^20 tasks need no private matrices).
 * m, n multiples of 128 (an odd multiple of 128 rows runs half of its last
 * 256-row tile: the A pool must hold 128 rows past such a window), k a
 * multiple of 64; a_k0, b_k0, b_col0 and c_col0 multiples of 64 (TMA
 * alignment), row offsets free.  chk_base: index of the task's first tile
 * in the checksum array (tile (tm,tn) at chk_base + tm*ceil(n/128) + tn),
 * global across shards so a shard's checksums land where an unsharded run
 * puts them.  No reference counterpart: the reference queues identical
 * tiles of one GEMM (src/urgent_baseline.cu:78-83). */
typedef struct apk_task {
  int m, n, k;
  int a_row0, a_k0;
  int b_k0, b_col0;
  int c_row0, c_col0;
  int flags;                /* APK_TASK_* bits                                 */
  long long chk_base;
} apk_task;
/* task flags: SAMPLED marks a task whose output window no other task touches
 * (set by apk_gen_tasks for spot checks); NARROW runs the task as 256x128
 * tiles in the one-CTA kernel, each holding one of the two TMEM accumulator
 * buffers so its epilogue overlaps the next tile's MMAs, instead of 256x256
 * tiles that hold both (the CTA-pair kernel's 256x256 jobs already hold one
 * buffer each and ignore it). */
#define APK_TASK_SAMPLED 1
#define APK_TASK_NARROW 2

/* Operand pools of a bf16 context: A [a_rows][a_cols] bf16, B [b_rows][b_cols]
 * bf16, C [c_rows][c_cols] fp32 (task outputs land in their windows). */
apk_status apk_set_task_pool(apk_ctx* ctx, const void* A, int a_rows, int a_cols, const void* B, int b_rows,
                             int b_cols, int c_rows, int c_cols, apk_mem_kind kind);

/* Install n tasks (checked against the pools) and build the flat tile work
 * list the persistent queue drains; n_chk = size of the checksum array.
 * The next apk_launch(ctx, n_work) runs task mode (n_work from *n_work_out);
 * apk_set_background switches back. */
apk_status apk_set_tasks(apk_ctx* ctx, const apk_task* tasks, int n, long long n_chk,
                         unsigned long long* n_work_out);

/* Per-tile checksums sum(c^2) (float64, fixed summation order) of the last
 * task-mode launch; untouched entries read 0. */
apk_status apk_read_checksums(apk_ctx* ctx, double* chk, long long n);

/* Copy a window of the C pool to host memory (rows x cols fp32). */
apk_status apk_read_pool_window(apk_ctx* ctx, int row0, int col0, int rows, int cols, float* out);

/* configs[4] generator: n tasks, m and n log-uniform in [mn_lo, mn_hi]
 * rounded to multiples of 128, k log-uniform in [k_lo, k_hi] rounded to
 * multiples of 64, windows placed at seeded offsets inside the pools;
 * chk_base is the running tile count.  The first n_samples tasks get
 * disjoint C windows in rows [c_rows - 2048*ceil(n_samples/4), c_rows) so
 * their outputs survive the run; every other task writes rows below that.
 * Returns the total tile count (the checksum array size). */
long long apk_gen_tasks(unsigned long long seed, int n, int mn_lo, int mn_hi, int k_lo, int k_hi, int a_rows,
                        int a_cols, int b_rows, int b_cols, int c_rows, int c_cols, int n_samples,
                        apk_task* out);

/* Static LPT shard of tasks over world ranks by 2*m*n*k (ties by task id):
 * writes this rank's task indices to idx (ascending) and returns their
 * count.  Deterministic, disjoint, and the ranks' union is every task. */
int apk_shard_tasks(const apk_task* tasks, int n, int world, int rank, int* idx);

/* ---- allocation-free entry point --------------------------------------- */

/* C = A * B (fp32, row-major, device pointers, 16-byte aligned; M and N
 * multiples of 128, K a multiple of 32) through the persistent fp32 SGEMM
 * drain, for callers that cannot call cudaMalloc -- a process whose device
 * memory belongs to a pool it does not control, or code that must not
 * allocate (an allocation can synchronize the device) once it is serving.
 * No counterpart in the reference: the reference allocates every buffer
 * itself in each binary's main().
 *
 * Nothing is allocated or freed: the kernel's scratch (work-queue counter,
 * exit bookkeeping, per-CTA tile counters) lives in a file-scope device
 * array of 16 KB, which every GPU that loads this library holds until the
 * process exits.  That fixes the limit: grid (0 = one CTA per resident
 * slot, 296 on a B200) may be at most 2016 CTAs; a larger grid, a grid
 * beyond residency, or a bad shape returns APK_EINVAL.  The first call on a
 * device does a one-time set-up (the array's device address, the kernel's
 * shared-memory attribute) and should come before any stream capture.  The
 * call is asynchronous on `stream` (a cudaStream_t, NULL = the legacy
 * default stream).  Every call shares the array: calls issued in order on
 * one stream are independent (the queue header is cleared on that stream
 * first), calls that overlap on the same device (e.g. on two streams) race
 * and must not be made; each device has its own array.  A bounded device
 * wait that runs out (2 s) leaves C incomplete and is not visible in the
 * return code, which comes back before the kernel runs: read it with
 * apk_sgemm_f32_noalloc_status. */
apk_status apk_sgemm_f32_noalloc(const float* A, const float* B, float* C, int M, int N, int K, int grid,
                                 void* stream);

/* Device status of the last apk_sgemm_f32_noalloc call on the current
 * device: synchronizes `stream` (the call's stream), then copies the status
 * word out of the static scratch into *device_status -- 0, or the code of
 * the wait that ran out (3 = a spin, 1 = a pipeline-stage wait).  Allocates
 * nothing.  Calls overlapping on the device would overwrite the word; the
 * next apk_sgemm_f32_noalloc clears it.  No counterpart in the reference
 * (its waits are unbounded). */
apk_status apk_sgemm_f32_noalloc_status(void* stream, int* device_status);

/* Failure-path self-test of the status word above: queues on `stream` a
 * bounded spin on a scratch word nothing sets, which gives up after
 * limit_ns (at most 10 s) and records 3 (DEV_WAIT_TIMEOUT_SPIN) as a
 * timed-out GEMM would.  apk_sgemm_f32_noalloc_status then reports it; the
 * device stays usable.  Allocates nothing.  No counterpart in the reference. */
apk_status apk_sgemm_f32_noalloc_selftest(long long limit_ns, void* stream);

/* ---- data and memory helpers ----------------------------------------- */

/* The reference's generator: srand(seed), then A (nA values) and B (nB
 * values) as (float)(rand()/(double)RAND_MAX*2-1), src/persistent.cu:132-135,
 * restated from glibc's published TYPE_3 additive-feedback algorithm. */
void apk_fill_uniform(unsigned seed, float* A, size_t nA, float* B, size_t nB);

/* Seeded N(0,1) rounded to bf16 (RNE); counter-based, multi-threaded. */
void apk_fill_normal_bf16(unsigned long long seed, uint16_t* out, size_t n);

/* fp32 -> bf16 round-to-nearest-even. */
void apk_round_bf16(const float* in, uint16_t* out, size_t n);

/* Pinned host memory for APK_MEM_HOST buffers (fast copies). */
void* apk_host_alloc(size_t bytes);
void apk_host_free(void* p);

int apk_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* APK_H_ */
