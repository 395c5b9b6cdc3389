// Host runtime behind include/apk.h: one context per device owning the
// persistent kernel's control block, event log, checkpoint slab and
// operands.  Replaces the per-binary main() drivers of the reference
// (src/persistent.cu:96-264, src/urgent_baseline.cu:144-380,
// src/yield.cu:327-960, src/midyield.cu:348-793, src/tcyield.cu:384-842).
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include <cudaTypedefs.h>

#include "../../include/apk.h"
#include "common.cuh"
#include "proto.h"

namespace apk {
namespace f32 {
cudaError_t prepare(int poll, int disc, bool oracle, int geo, int sched, int* max_ctas_per_sm);
cudaError_t launch(const F32Params& prm, int grid, int poll, int disc, bool oracle, int geo, int sched,
                   cudaStream_t stream);
GeoInfo geo_info(int geo);
size_t params_bytes();
}  // namespace f32
namespace bf16pair {
cudaError_t prepare(int poll, int disc, bool oracle, int sms, int* pairs, bool clc);
cudaError_t launch(const F32Params& prm, int grid, int poll, int disc, bool oracle, bool clc, cudaStream_t stream);
int smem_bytes(bool tasks);
int stages(bool tasks);
int threads();
int epi_warps();
size_t params_bytes();
}  // namespace bf16pair
namespace f32ws {
cudaError_t prepare(int poll, int disc, bool oracle, int* ok);
cudaError_t launch(const F32Params& prm, int workers, int poll, int disc, bool oracle, cudaStream_t stream);
int smem_bytes();
int threads();
int workers_per_cta();
size_t params_bytes();
}  // namespace f32ws
namespace vis {
cudaError_t launch(const VisParams& prm, int grid, int smem_bytes, bool loaded, cudaStream_t stream);
int threads();
int loads_per_iter();
}  // namespace vis
namespace bf16 {
cudaError_t prepare(int poll, int disc, bool oracle, int geo, int sched, int* max_ctas_per_sm);
cudaError_t launch(const F32Params& prm, int grid, int poll, int disc, bool oracle, int geo, int sched,
                   cudaStream_t stream);
GeoInfo geo_info(int geo);
int epi_warps(int geo);
size_t params_bytes();
}  // namespace bf16
}  // namespace apk

using namespace apk;

namespace {

long long host_now_ns() {
  return std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

void spin_until_ns(long long t) {
  while (host_now_ns() < t) {
  }
}

// Device control block (one per launch target).
struct Ctrl {
  unsigned long long next_task;
  unsigned long long start_min;
  unsigned long long end_max;
  unsigned long long yields;
  unsigned long long completed;  // completed background tiles (count triggers)
  unsigned long long ckpt[5];    // checkpoint spill ns, bytes, restore ns, bytes; TMEM parks
  int exited;
  int abort_word;
  int status;
  int never_set; // a word no code path writes (failure-path self-test)
  // yield flag in device memory (DEVICE / HOST_MEMCPY modes): copy 0 of the
  // generation, copies 1..FLAG_LINES-1 on the lines that follow it
  alignas(128) int flag_dev;
  int flag_copies[FLAG_LINES * FLAG_STRIDE - 1];
};
static_assert(offsetof(Ctrl, flag_copies) + sizeof(int) * (FLAG_LINES * FLAG_STRIDE - 1) ==
                  offsetof(Ctrl, flag_dev) + sizeof(int) * FLAG_LINES * FLAG_STRIDE,
              "flag copies follow flag_dev line by line");

// Host-to-globaltimer visibility probe (src/yield.cu:208-214), bounded.
__global__ void spin_flag_kernel(const int* flag, int target, long long limit_ns, long long* out,
                                 int* status) {
  if (threadIdx.x != 0) return;
  const long long t0 = globaltimer_ns();
  while (true) {
    if (flag_load(flag) == target) {
      *out = globaltimer_ns();
      return;
    }
    if (globaltimer_ns() - t0 > limit_ns) {
      *out = 0;
      atomicCAS(status, 0, DEV_WAIT_TIMEOUT_SPIN);
      return;
    }
  }
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

}  // namespace

struct apk_ctx {
  apk_config cfg{};
  std::string err;
  int sms = 0, grid = 0, ctas_per_sm = 0, max_ctas_per_sm = 0;
  // fp32: the warp-specialized kernel (two workers per 384-thread CTA) can
  // run every poll variant this context launches; sync_only holds the
  // block-synchronous kernel for experiments that compare grids slot by slot
  bool ws_ok = false;
  bool sync_only = false;
  // geometry and ring: fp32 block-synchronous tile geometry (F32Geo), the K
  // depth of one ring slot and the slots per stage-level yield site
  int f32_geo = F32_GEO_L32;
  int bf16_geo = BF16_GEO_STD64;
  int slot_k = 32;
  int poll_every = 1;
  // bf16: the CTA-pair kernel can run every poll variant this context
  // launches with every SM in a pair
  bool pair_ok = false;
  int cc_major = 0, cc_minor = 0;
  char name[128] = {0};
  cudaStream_t kstream = nullptr, cstream = nullptr, ustream = nullptr;
  // streamed apk_gemm (host operands): copy-in and copy-back streams, the
  // readiness words the kernel waits on, per-panel tile counters, mapped
  // per-panel completion acks and a pinned 1 the readiness writes copy from
  cudaStream_t h2dstream = nullptr, d2hstream = nullptr;
  cudaEvent_t ev_reset = nullptr;
  int* d_ready = nullptr;
  unsigned* d_pdone = nullptr;
  int* h_pack = nullptr;
  int* d_pack_mapped = nullptr;
  int* h_one = nullptr;
  unsigned* d_order = nullptr;  // tile visit order of a streamed run
  unsigned* h_order = nullptr;
  int stream_cap = 0;       // capacity of d_ready (panels + column panels)
  int pack_cap = 0;         // capacity of d_pdone / h_pack (C blocks)
  int order_cap = 0;        // capacity of d_order / h_order (visit slots)
  float* d_part = nullptr;  // K-slice hand-off accumulators of a streamed run
  int* d_part_ready = nullptr;
  int part_cap = 0;         // capacity of d_part / d_part_ready (tiles)
  StreamProto st_cfg{};     // copied into the launch's parameters (zeros = resident operands)
  cudaEvent_t ev_start = nullptr, ev_done = nullptr;
  bool running = false;

  // background operands
  int M = 0, N = 0, K = 0;
  void *dA = nullptr, *dB = nullptr, *dC = nullptr;
  bool ownA = false, ownB = false, ownC = false;
  size_t capA = 0, capB = 0, capC = 0;
  // urgent operands
  int Mu = 0, Nu = 0, Ku = 0;
  void *dAu = nullptr, *dBu = nullptr;
  bool ownAu = false, ownBu = false;
  float* dCu = nullptr;  // (max_events + 1) slots
  size_t cu_slot = 0;
  // urgent output slots [0, cu_dirty) may hold values (fresh allocation or
  // the split-K sums of the previous launch's events); the device-set events
  // the last launch could raise
  int cu_dirty = 0;
  int dev_events_last = 0;

  // control
  Ctrl* d_ctrl = nullptr;   // main launch
  Ctrl* d_uctrl = nullptr;  // baseline urgent launch
  int* h_flag = nullptr;    // mapped pinned
  int* d_flag_mapped = nullptr;
  int* h_ack = nullptr;     // mapped pinned [2*max_events]
  int* d_ack_mapped = nullptr;
  int* h_gen = nullptr;     // pinned sources for HOST_MEMCPY stores [max_events + 2]
  // HOST_MEMCPY flag stores: pinned images of the FLAG_LINES flag lines
  // (4 KB each), reused in a ring once the copy that read them has run
  static constexpr int kFlagRing = 16;
  int* h_flag_ring = nullptr;
  cudaEvent_t flag_ring_ev[kFlagRing] = {};
  int flag_ring_next = 0;
  int flag_lines = 1;  // flag copies of the running launch

  // event log (device)
  long long *d_sched = nullptr, *d_set = nullptr, *d_obs = nullptr, *d_claim_ns = nullptr;
  unsigned long long* d_done = nullptr;
  int *d_claim = nullptr, *d_site = nullptr, *d_inflight = nullptr, *d_uq = nullptr,
      *d_udone = nullptr, *d_uexec = nullptr;
  int n_sched = 0;
  unsigned long long* d_count = nullptr;
  int n_count = 0;
  // event log (host)
  std::vector<long long> host_set, host_ack, host_done;
  std::atomic<int> n_injected{0};

  // checkpoint slab, per-CTA counters
  float* d_slab = nullptr;
  long long* d_slab_hdr = nullptr;
  unsigned* d_slot_bits = nullptr;    // CLC resident-slot bitmap
  long long* d_setter_state = nullptr;  // CLC: device setter state across slot-0 holders
  unsigned long long* d_tiles = nullptr;
  unsigned long long* d_utiles = nullptr;
  int* d_exec = nullptr;
  size_t exec_cap = 0;
  unsigned long long last_tasks = 0;
  int last_grid = 0;

  // task mode: operand pools, task table, flat work list
  bool task_mode = false;
  void *dApool = nullptr, *dBpool = nullptr;
  float* dCpool = nullptr;
  bool ownApool = false, ownBpool = false;
  int a_rows = 0, a_cols = 0, b_rows = 0, b_cols = 0, c_rows = 0, c_cols = 0;
  TaskDesc* d_tasks = nullptr;
  unsigned* d_work = nullptr;
  double* d_chk = nullptr;
  int n_tasks = 0;
  unsigned long long n_work = 0;
  unsigned long long n_halves = 0;  // 256x128 halves of all work tiles (the kernel's task-mode tile count)
  long long n_chk = 0;
  double task_flops = 0.0;  // sum of 2*m*n*k over installed tasks
  unsigned long long last_exec_n = 0;  // oracle counters of the last launch
};

namespace {

apk_status fail(apk_ctx* c, apk_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  return s;
}

#define APK_CU(call)                                                                   \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess)                                                             \
      return fail(ctx, APK_ECUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                  __FILE__, __LINE__);                                                 \
  } while (0)

apk_status ensure_encoder(apk_ctx* ctx) {
  if (g_encode) return APK_OK;
  cudaDriverEntryPointQueryResult q;
  void* fn = nullptr;
  APK_CU(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q));
  if (q != cudaDriverEntryPointSuccess || !fn)
    return fail(ctx, APK_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return APK_OK;
}

// 2-D row-major tensor map: rows x cols elements, box box_cols x box_rows.
apk_status make_tmap(apk_ctx* ctx, CUtensorMap* tm, const void* base, CUtensorMapDataType dt,
                     int esize, long long rows, long long cols, int box_cols, int box_rows,
                     CUtensorMapSwizzle sw) {
  if (ensure_encoder(ctx) != APK_OK) return APK_ECUDA;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * esize};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(tm, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(ctx, APK_ECUDA, "cuTensorMapEncodeTiled failed (%d) rows=%lld cols=%lld box=%dx%d",
                (int)r, rows, cols, box_cols, box_rows);
  return APK_OK;
}

// 3-D map of a row-major rows x cols matrix seen as [cols/64][rows][64]:
// box {64, box_rows, chunks} lands chunk-major in shared memory, each chunk
// the [box_rows][64] block a 2-D map with a 64-column box would load.
apk_status make_tmap_chunks(apk_ctx* ctx, CUtensorMap* tm, const void* base, CUtensorMapDataType dt, int esize,
                            long long rows, long long cols, int box_rows, int chunks, CUtensorMapSwizzle sw) {
  if (ensure_encoder(ctx) != APK_OK) return APK_ECUDA;
  if (cols % 64 != 0) return fail(ctx, APK_EINVAL, "chunked map: %lld columns not a multiple of 64", cols);
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(cols / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)cols * esize, (cuuint64_t)64 * esize};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)chunks};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(tm, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(ctx, APK_ECUDA, "cuTensorMapEncodeTiled (3-D) failed (%d) rows=%lld cols=%lld box=64x%dx%d",
                (int)r, rows, cols, box_rows, chunks);
  return APK_OK;
}

size_t esize_of(apk_dtype d) { return d == APK_BF16 ? 2 : 4; }

// Output tiles: fp32 128x128; bf16 256 rows by 256 columns, the last tile of
// a row 128 wide when the width is an odd multiple of 128.
bool use_pair(const apk_ctx* ctx);
// bf16 NARROW / NARROW_SPILL: 256x128 jobs in the one-CTA kernel
bool narrow_jobs(const apk_ctx* ctx) {
  return ctx->cfg.dtype == APK_BF16 &&
         (ctx->cfg.bf16_kernel == APK_BF16_NARROW || ctx->cfg.bf16_kernel == APK_BF16_NARROW_SPILL);
}
int tile_rows(const apk_ctx* ctx) {
  return ctx->cfg.dtype == APK_F32 ? f32::geo_info(ctx->f32_geo).tile_m : bf16::geo_info(ctx->bf16_geo).tile_m;
}
int tile_cols(const apk_ctx* ctx) {
  return ctx->cfg.dtype == APK_F32 ? f32::geo_info(ctx->f32_geo).tile_n
         : use_pair(ctx)           ? 512
         : narrow_jobs(ctx)        ? 128
                                   : bf16::geo_info(ctx->bf16_geo).tile_n;
}
int tiles_across(const apk_ctx* ctx, int n) { return (n + tile_cols(ctx) - 1) / tile_cols(ctx); }

apk_status upload(apk_ctx* ctx, void** dst, bool* own, size_t* cap, const void* src, size_t bytes,
                  apk_mem_kind kind) {
  if (kind == APK_MEM_DEVICE) {
    if (*own && *dst) cudaFree(*dst);
    *dst = const_cast<void*>(src);
    *own = false;
    *cap = 0;
    return APK_OK;
  }
  if (!*own || *cap < bytes) {
    if (*own && *dst) cudaFree(*dst);
    *dst = nullptr;
    APK_CU(cudaMalloc(dst, bytes));
    *own = true;
    *cap = bytes;
  }
  if (src) APK_CU(cudaMemcpyAsync(*dst, src, bytes, cudaMemcpyHostToDevice, ctx->kstream));
  return APK_OK;
}

int kernel_poll(const apk_ctx* c) { return (int)c->cfg.poll; }

apk_status prepare_kernel(apk_ctx* ctx, int poll) {
  int maxc = 0;
  cudaError_t e;
  if (ctx->cfg.dtype == APK_F32)
    e = f32::prepare(poll, ctx->cfg.discipline, ctx->cfg.oracle != 0, ctx->f32_geo, ctx->cfg.scheduler, &maxc);
  else
    e = bf16::prepare(poll, ctx->cfg.discipline, ctx->cfg.oracle != 0, ctx->bf16_geo, ctx->cfg.scheduler, &maxc);
  if (e != cudaSuccess)
    return fail(ctx, APK_EUNSUPPORTED, "kernel variant unavailable (dtype %d poll %d disc %d oracle %d k_tile %d): %s",
                ctx->cfg.dtype, poll, ctx->cfg.discipline, ctx->cfg.oracle, ctx->cfg.k_tile,
                cudaGetErrorString(e));
  if (maxc < 1) return fail(ctx, APK_EUNSUPPORTED, "kernel does not fit on an SM");
  ctx->max_ctas_per_sm = maxc;
  if (ctx->cfg.dtype == APK_F32 && ctx->cfg.scheduler == APK_SCHED_QUEUE && ctx->f32_geo == F32_GEO_L32) {
    int ok = 0;
    e = f32ws::prepare(poll, ctx->cfg.discipline, ctx->cfg.oracle != 0, &ok);
    if (e != cudaSuccess) ok = 0;
    ctx->ws_ok = ctx->ws_ok && ok;
  }
  if (ctx->cfg.dtype == APK_BF16 && ctx->bf16_geo == BF16_GEO_STD64) {
    int pairs = 0;
    e = bf16pair::prepare(poll, ctx->cfg.discipline, ctx->cfg.oracle != 0, ctx->sms, &pairs,
                          ctx->cfg.scheduler == APK_SCHED_CLC);
    if (e != cudaSuccess) pairs = 0;
    ctx->pair_ok = ctx->pair_ok && ctx->sms % 2 == 0 && 2 * pairs >= ctx->sms;
  }
  return APK_OK;
}

// The bf16 launch runs the CTA-pair kernel for a task list, or a plain
// background GEMM whose N is a multiple of 256, when the urgent N is one too,
// K-tile is 64 or 128, one CTA per SM over every SM; the one-CTA kernel runs
// everything else.
// (task lists included: every task tile is a 256x256 pair job, the
// peer's half of a tile whose n ends 128 columns in computed and not stored)
// Under cluster launch control the pairs run plain drains (one cluster per
// 256x512 tile); task lists then take the one-CTA kernel.
bool pair_capable(const apk_ctx* ctx) {
  return ctx->cfg.dtype == APK_BF16 && ctx->pair_ok &&
         (ctx->cfg.scheduler == APK_SCHED_QUEUE || (ctx->cfg.scheduler == APK_SCHED_CLC && !ctx->task_mode)) &&
         (ctx->cfg.bf16_kernel == APK_BF16_AUTO || ctx->cfg.bf16_kernel == APK_BF16_PAIR) &&
         ctx->bf16_geo == BF16_GEO_STD64 && ctx->grid == ctx->sms && ctx->Nu % 256 == 0;
}
// Task lists run on pairs only when asked for (APK_BF16_PAIR): their
// 256-wide pair jobs issue one MMA a k-step into one accumulator, and on
// 2^18 configs[4] tasks the pair kernel reached 760-800 TFLOP/s against
// 860-910 for the one-CTA kernel.
bool use_pair(const apk_ctx* ctx) {
  return pair_capable(ctx) &&
         (ctx->task_mode ? ctx->cfg.bf16_kernel == APK_BF16_PAIR : ctx->N % 256 == 0);
}

// The fp32 launch runs the warp-specialized kernel (one 384-thread CTA per
// SM, two 128x128 workers) at full residency of the default schedule: queue
// scheduler, K-tile 32, exactly two workers per SM.  Other grids (reserved
// slots, one CTA per SM), K-tile 64 and cluster launch control run the
// block-synchronous kernel.
bool use_ws(const apk_ctx* ctx) {
  return ctx->cfg.dtype == APK_F32 && ctx->ws_ok && !ctx->sync_only && ctx->cfg.f32_kernel != APK_F32_BLOCK_SYNC &&
         ctx->cfg.scheduler == APK_SCHED_QUEUE &&
         ctx->f32_geo == F32_GEO_L32 && ctx->grid == ctx->sms * f32ws::workers_per_cta();
}

}  // namespace

extern "C" {

int apk_abi_version(void) { return APK_ABI_VERSION; }

void apk_config_default(apk_config* c) {
  memset(c, 0, sizeof *c);
  c->device = 0;
  c->dtype = APK_F32;
  c->ctas_per_sm = 0;
  c->grid = 0;
  c->k_tile = 0;  // the dtype's default: fp32 32, bf16 64
  c->poll = APK_POLL_STAGE;
  c->discipline = APK_DISC_DRAIN;
  c->set_mode = APK_SET_HOST_MEMCPY;
  c->max_events = 4096;
  c->oracle = 0;
  c->urgent_split_k = 8;
  c->wait_limit_ns = 2000000000LL;
}

const char* apk_last_error(const apk_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

apk_status apk_create(const apk_config* cfg, apk_ctx** out) {
  if (!cfg || !out) return APK_EINVAL;
  *out = nullptr;
  apk_ctx* ctx = new apk_ctx();
  ctx->cfg = *cfg;
  apk_config& c = ctx->cfg;
  // every translation unit must agree on the kernel parameter block (objects
  // compiled against different copies of proto.h would read garbage pointers)
  if (f32::params_bytes() != sizeof(F32Params) || bf16::params_bytes() != sizeof(F32Params) ||
      f32ws::params_bytes() != sizeof(F32Params) || bf16pair::params_bytes() != sizeof(F32Params)) {
    fail(ctx, APK_EUNSUPPORTED, "kernel parameter layout mismatch (f32 %zu, bf16 %zu, runtime %zu bytes): rebuild",
         f32::params_bytes(), bf16::params_bytes(), sizeof(F32Params));
    *out = ctx;
    return APK_EUNSUPPORTED;
  }
  if (c.max_events < 1) c.max_events = 1;
  if (c.urgent_split_k < 1) c.urgent_split_k = 1;
  if (c.wait_limit_ns <= 0) c.wait_limit_ns = 2000000000LL;
  if (c.k_tile == 0) c.k_tile = c.dtype == APK_BF16 ? 64 : 32;
  if (c.k_tile != 32 && c.k_tile != 64 && c.k_tile != 128) {
    fail(ctx, APK_EINVAL, "k_tile must be 32, 64 or 128");
    *out = ctx;
    return APK_EINVAL;
  }
  // Geometry and ring.  The K-tile is the K depth between two stage-level
  // yield sites; each kernel moves it through ring slots of its own depth
  // (fp32 128x128 tiles: 32, or 64 at one CTA per SM; 64x128 and 32x128
  // tiles for 4 and 8 CTAs per SM: 16; bf16: 64, or 32 for K-tile 32) and
  // polls every k_tile / slot_k slots.
  if (c.dtype == APK_F32) {
    ctx->f32_geo = c.ctas_per_sm >= 8   ? F32_GEO_S
                   : c.ctas_per_sm >= 4 ? F32_GEO_M
                   : (c.ctas_per_sm == 1 && c.k_tile >= 64) ? F32_GEO_L64
                                                             : F32_GEO_L32;
    ctx->slot_k = f32::geo_info(ctx->f32_geo).slot_k;
  } else {
    const bool k32 = c.k_tile == 32;
    ctx->bf16_geo = c.ctas_per_sm >= 8   ? BF16_GEO_N64
                    : c.ctas_per_sm >= 4 ? BF16_GEO_N128
                    : c.ctas_per_sm >= 2 ? (k32 ? BF16_GEO_N256x32 : BF16_GEO_N256x64)
                                         : (k32 ? BF16_GEO_STD32 : BF16_GEO_STD64);
    ctx->slot_k = bf16::geo_info(ctx->bf16_geo).slot_k;
  }
  ctx->poll_every = c.k_tile / ctx->slot_k;
  if (c.discipline == APK_DISC_POISON && c.poll == APK_POLL_OFF) {
    fail(ctx, APK_EINVAL, "the poison discipline needs a poll mode");
    *out = ctx;
    return APK_EINVAL;
  }
  if (c.scheduler != APK_SCHED_QUEUE && c.scheduler != APK_SCHED_CLC) {
    fail(ctx, APK_EINVAL, "unknown scheduler %d", (int)c.scheduler);
    *out = ctx;
    return APK_EINVAL;
  }
  if (c.scheduler == APK_SCHED_CLC &&
      (c.discipline != APK_DISC_DRAIN || (c.dtype == APK_BF16 && c.ctas_per_sm > 1) ||
       (c.dtype == APK_F32 && c.ctas_per_sm > 2))) {
    fail(ctx, APK_EUNSUPPORTED,
         "the cluster-launch-control scheduler is built for the drain discipline and the 128x128 fp32 / one-CTA bf16 "
         "geometries");
    *out = ctx;
    return APK_EUNSUPPORTED;
  }
  *out = ctx;
  APK_CU(cudaSetDevice(c.device));
  cudaDeviceProp prop;
  APK_CU(cudaGetDeviceProperties(&prop, c.device));
  ctx->sms = prop.multiProcessorCount;
  ctx->cc_major = prop.major;
  ctx->cc_minor = prop.minor;
  snprintf(ctx->name, sizeof ctx->name, "%s", prop.name);
  if (prop.major != 10)
    return fail(ctx, APK_EUNSUPPORTED, "device %s is sm_%d%d; this build targets sm_100a", prop.name,
                prop.major, prop.minor);
  ctx->ws_ok = c.dtype == APK_F32;  // cleared by any variant the warp-specialized kernel lacks
  ctx->pair_ok = c.dtype == APK_BF16;  // likewise for the CTA-pair kernel
  apk_status s = prepare_kernel(ctx, kernel_poll(ctx));
  if (s != APK_OK) return s;
  // the POLL_OFF variant is used by the overhead and baseline modes
  if (c.poll != APK_POLL_OFF && c.discipline == APK_DISC_DRAIN) {
    const int keep = ctx->max_ctas_per_sm;
    s = prepare_kernel(ctx, APK_POLL_OFF);
    if (s != APK_OK) return s;
    ctx->max_ctas_per_sm = std::min(keep, ctx->max_ctas_per_sm);
  }
  ctx->ctas_per_sm = c.ctas_per_sm > 0 ? std::min(c.ctas_per_sm, ctx->max_ctas_per_sm) : ctx->max_ctas_per_sm;
  ctx->grid = c.grid > 0 ? c.grid : ctx->sms * ctx->ctas_per_sm;
  if (narrow_jobs(ctx) && ctx->bf16_geo != BF16_GEO_STD64 && ctx->bf16_geo != BF16_GEO_STD32)
    return fail(ctx, APK_EUNSUPPORTED, "the NARROW bf16 kernels run one CTA per SM (ctas_per_sm 0 or 1)");
  if (c.dtype == APK_BF16 && c.bf16_kernel == APK_BF16_PAIR && !use_pair(ctx))
    return fail(ctx, APK_EUNSUPPORTED,
                "the CTA-pair bf16 kernel needs K-tile 64, one CTA on each of an even number of SMs and "
                "every SM in a co-resident pair (grid %d, %d SMs)", ctx->grid, ctx->sms);
  if (c.dtype == APK_F32 && c.f32_kernel == APK_F32_WARP_SPECIALIZED && !use_ws(ctx))
    return fail(ctx, APK_EUNSUPPORTED,
                "the warp-specialized fp32 kernel needs the queue scheduler, 128x128 tiles on 32-deep slots and two workers per SM "
                "(grid %d, %d SMs)", ctx->grid, ctx->sms);
  if (ctx->grid > ctx->sms * ctx->max_ctas_per_sm)
    return fail(ctx, APK_EINVAL,
                "grid %d exceeds the %d resident slots; CTAs beyond residency would never "
                "observe a yield (src/yield.cu:815-822)",
                ctx->grid, ctx->sms * ctx->max_ctas_per_sm);

  int lo = 0, hi = 0;
  APK_CU(cudaDeviceGetStreamPriorityRange(&lo, &hi));
  APK_CU(cudaStreamCreateWithPriority(&ctx->kstream, cudaStreamNonBlocking, lo));
  APK_CU(cudaStreamCreateWithPriority(&ctx->cstream, cudaStreamNonBlocking, hi));
  APK_CU(cudaStreamCreateWithPriority(&ctx->ustream, cudaStreamNonBlocking, hi));
  APK_CU(cudaEventCreate(&ctx->ev_start));
  APK_CU(cudaEventCreate(&ctx->ev_done));

  const int E = c.max_events;
  const int G = ctx->grid;
  APK_CU(cudaMalloc(&ctx->d_ctrl, sizeof(Ctrl)));
  APK_CU(cudaMalloc(&ctx->d_uctrl, sizeof(Ctrl)));
  APK_CU(cudaHostAlloc(&ctx->h_flag, 64, cudaHostAllocMapped));
  APK_CU(cudaHostGetDevicePointer((void**)&ctx->d_flag_mapped, ctx->h_flag, 0));
  APK_CU(cudaHostAlloc(&ctx->h_ack, sizeof(int) * 2 * E, cudaHostAllocMapped));
  APK_CU(cudaHostGetDevicePointer((void**)&ctx->d_ack_mapped, ctx->h_ack, 0));
  APK_CU(cudaHostAlloc(&ctx->h_gen, sizeof(int) * (E + 2), cudaHostAllocDefault));
  APK_CU(cudaHostAlloc(&ctx->h_flag_ring, sizeof(int) * apk_ctx::kFlagRing * FLAG_LINES * FLAG_STRIDE,
                       cudaHostAllocDefault));
  memset(ctx->h_flag_ring, 0, sizeof(int) * apk_ctx::kFlagRing * FLAG_LINES * FLAG_STRIDE);
  for (int i = 0; i < apk_ctx::kFlagRing; ++i)
    APK_CU(cudaEventCreateWithFlags(&ctx->flag_ring_ev[i], cudaEventDisableTiming));
  memset(ctx->h_flag, 0, 64);
  memset(ctx->h_ack, 0, sizeof(int) * 2 * E);
  APK_CU(cudaMalloc(&ctx->d_sched, sizeof(long long) * E));
  APK_CU(cudaMalloc(&ctx->d_count, sizeof(unsigned long long) * E));
  APK_CU(cudaMalloc(&ctx->d_set, sizeof(long long) * E));
  APK_CU(cudaMalloc(&ctx->d_obs, sizeof(long long) * (size_t)E * G));
  APK_CU(cudaMalloc(&ctx->d_claim_ns, sizeof(long long) * E));
  APK_CU(cudaMalloc(&ctx->d_done, sizeof(unsigned long long) * E));
  APK_CU(cudaMalloc(&ctx->d_claim, sizeof(int) * E));
  APK_CU(cudaMalloc(&ctx->d_site, sizeof(int) * E));
  APK_CU(cudaMalloc(&ctx->d_inflight, sizeof(int) * E));
  APK_CU(cudaMalloc(&ctx->d_uq, sizeof(int) * E));
  APK_CU(cudaMalloc(&ctx->d_udone, sizeof(int) * E));
  APK_CU(cudaMalloc(&ctx->d_uexec, sizeof(int) * E));
  // checkpoint slab: fp32 128x128 fp32 accumulators (64 KB), bf16 256x256 (256 KB)
  const size_t slab_floats = (c.dtype == APK_F32 ? 128 * 128 : 256 * 256);
  APK_CU(cudaMalloc(&ctx->d_slab, sizeof(float) * slab_floats * G));
  APK_CU(cudaMalloc(&ctx->d_slab_hdr, sizeof(long long) * 4 * G));
  APK_CU(cudaMalloc(&ctx->d_slot_bits, sizeof(unsigned) * ((G + 31) / 32)));
  APK_CU(cudaMalloc(&ctx->d_setter_state, sizeof(long long) * 2));
  APK_CU(cudaMalloc(&ctx->d_tiles, sizeof(unsigned long long) * G));
  APK_CU(cudaMalloc(&ctx->d_utiles, sizeof(unsigned long long) * G));
  ctx->host_set.assign(E, 0);
  ctx->host_ack.assign(E, 0);
  ctx->host_done.assign(E, 0);
  return APK_OK;
}

apk_status apk_destroy(apk_ctx* ctx) {
  if (!ctx) return APK_OK;
  if (ctx->running) {
    apk_stop(ctx);
    apk_wait(ctx, 5000000000LL);
  }
  cudaSetDevice(ctx->cfg.device);
  auto F = [](void* p) {
    if (p) cudaFree(p);
  };
  if (ctx->ownA) F(ctx->dA);
  if (ctx->ownB) F(ctx->dB);
  if (ctx->ownC) F(ctx->dC);
  if (ctx->ownAu) F(ctx->dAu);
  if (ctx->ownBu) F(ctx->dBu);
  F(ctx->dCu);
  F(ctx->d_ctrl);
  F(ctx->d_uctrl);
  F(ctx->d_sched);
  F(ctx->d_count);
  F(ctx->d_set);
  F(ctx->d_obs);
  F(ctx->d_claim_ns);
  F(ctx->d_done);
  F(ctx->d_claim);
  F(ctx->d_site);
  F(ctx->d_inflight);
  F(ctx->d_uq);
  F(ctx->d_udone);
  F(ctx->d_uexec);
  F(ctx->d_slab);
  F(ctx->d_slab_hdr);
  F(ctx->d_slot_bits);
  F(ctx->d_setter_state);
  F(ctx->d_tiles);
  F(ctx->d_utiles);
  F(ctx->d_exec);
  if (ctx->ownApool) F(ctx->dApool);
  if (ctx->ownBpool) F(ctx->dBpool);
  F(ctx->dCpool);
  F(ctx->d_tasks);
  F(ctx->d_work);
  F(ctx->d_chk);
  if (ctx->h_flag) cudaFreeHost(ctx->h_flag);
  if (ctx->h_ack) cudaFreeHost(ctx->h_ack);
  if (ctx->h_gen) cudaFreeHost(ctx->h_gen);
  for (int i = 0; i < apk_ctx::kFlagRing; ++i)
    if (ctx->flag_ring_ev[i]) cudaEventDestroy(ctx->flag_ring_ev[i]);
  if (ctx->h_flag_ring) cudaFreeHost(ctx->h_flag_ring);
  if (ctx->kstream) cudaStreamDestroy(ctx->kstream);
  if (ctx->cstream) cudaStreamDestroy(ctx->cstream);
  if (ctx->ustream) cudaStreamDestroy(ctx->ustream);
  if (ctx->h2dstream) cudaStreamDestroy(ctx->h2dstream);
  if (ctx->d2hstream) cudaStreamDestroy(ctx->d2hstream);
  if (ctx->ev_reset) cudaEventDestroy(ctx->ev_reset);
  F(ctx->d_ready);
  F(ctx->d_pdone);
  F(ctx->d_order);
  F(ctx->d_part);
  F(ctx->d_part_ready);
  if (ctx->h_pack) cudaFreeHost(ctx->h_pack);
  if (ctx->h_order) cudaFreeHost(ctx->h_order);
  if (ctx->h_one) cudaFreeHost(ctx->h_one);
  if (ctx->ev_start) cudaEventDestroy(ctx->ev_start);
  if (ctx->ev_done) cudaEventDestroy(ctx->ev_done);
  delete ctx;
  return APK_OK;
}

apk_status apk_get_info(apk_ctx* ctx, apk_device_info* info) {
  if (!ctx || !info) return APK_EINVAL;
  memset(info, 0, sizeof *info);
  info->sms = ctx->sms;
  info->grid = ctx->grid;
  info->ctas_per_sm = ctx->ctas_per_sm;
  info->max_ctas_per_sm = ctx->max_ctas_per_sm;
  info->cc_major = ctx->cc_major;
  info->cc_minor = ctx->cc_minor;
  if (ctx->cfg.dtype == APK_F32 && use_ws(ctx)) {
    // grid and ctas_per_sm count workers (two per CTA)
    info->smem_per_cta = f32ws::smem_bytes();
    info->threads_per_cta = f32ws::threads();
    info->tile_m = 128;
    info->tile_n = 128;
    info->stages = f32::geo_info(F32_GEO_L32).stages;
  } else if (ctx->cfg.dtype == APK_F32) {
    const GeoInfo g = f32::geo_info(ctx->f32_geo);
    info->smem_per_cta = g.smem_bytes;
    info->threads_per_cta = g.threads;
    info->tile_m = g.tile_m;
    info->tile_n = g.tile_n;
    info->stages = g.stages;
  } else if (use_pair(ctx)) {
    info->smem_per_cta = bf16pair::smem_bytes(ctx->task_mode);
    info->threads_per_cta = bf16pair::threads();
    info->tile_m = 256;
    info->tile_n = 512;  // one tile per CTA pair
    info->stages = bf16pair::stages(ctx->task_mode);
  } else {
    const GeoInfo g = bf16::geo_info(ctx->bf16_geo);
    info->smem_per_cta = g.smem_bytes;
    info->threads_per_cta = g.threads;
    info->tile_m = g.tile_m;
    info->tile_n = tile_cols(ctx);  // 128 for the NARROW kernels' 256x128 jobs
    info->stages = g.stages;
  }
  info->k_tile = ctx->cfg.k_tile;
  info->slot_k = ctx->slot_k;
  snprintf(info->name, sizeof info->name, "%s", ctx->name);
  return APK_OK;
}

apk_status apk_set_background(apk_ctx* ctx, const void* A, const void* B, void* C, int M, int N,
                              int K, apk_mem_kind kind) {
  if (!ctx) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "set_background while a launch runs");
  if (M <= 0 || N <= 0 || K <= 0 || M % 128 || N % 128 || K % ctx->cfg.k_tile)
    return fail(ctx, APK_EINVAL, "shape %dx%dx%d: M and N must be multiples of 128, K of %d", M, N,
                K, ctx->cfg.k_tile);
  if (ctx->cfg.dtype == APK_BF16 && M % 256)
    return fail(ctx, APK_EINVAL, "bf16 background M must be a multiple of 256");
  if (kind == APK_MEM_DEVICE && (!A || !B || !C))
    return fail(ctx, APK_EINVAL, "device operands must be non-null");
  APK_CU(cudaSetDevice(ctx->cfg.device));
  const size_t es = esize_of(ctx->cfg.dtype);
  apk_status s;
  if ((s = upload(ctx, &ctx->dA, &ctx->ownA, &ctx->capA, A, es * M * K, kind)) != APK_OK) return s;
  if ((s = upload(ctx, &ctx->dB, &ctx->ownB, &ctx->capB, B, es * (size_t)K * N, kind)) != APK_OK) return s;
  if (kind == APK_MEM_DEVICE) {
    if (ctx->ownC && ctx->dC) cudaFree(ctx->dC);
    ctx->dC = C;
    ctx->ownC = false;
  } else {
    if ((s = upload(ctx, &ctx->dC, &ctx->ownC, &ctx->capC, nullptr, 4ull * M * N, APK_MEM_HOST)) != APK_OK)
      return s;
  }
  ctx->M = M;
  ctx->N = N;
  ctx->K = K;
  ctx->task_mode = false;
  APK_CU(cudaStreamSynchronize(ctx->kstream));
  return APK_OK;
}

apk_status apk_set_task_pool(apk_ctx* ctx, const void* A, int a_rows, int a_cols, const void* B, int b_rows,
                             int b_cols, int c_rows, int c_cols, apk_mem_kind kind) {
  if (!ctx || !A || !B) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "set_task_pool while a launch runs");
  if (ctx->cfg.dtype != APK_BF16) return fail(ctx, APK_EUNSUPPORTED, "task pools need a bf16 context");
  if (a_rows < 256 || b_rows < 64 || c_rows < 128 || a_cols % 64 || b_cols % 64 || c_cols % 64 || a_cols < 64 ||
      b_cols < 128 || c_cols < 128)
    return fail(ctx, APK_EINVAL, "pool dimensions out of range (columns multiples of 64)");
  APK_CU(cudaSetDevice(ctx->cfg.device));
  size_t capA = 0, capB = 0;
  apk_status s;
  if ((s = upload(ctx, &ctx->dApool, &ctx->ownApool, &capA, A, 2ull * a_rows * a_cols, kind)) != APK_OK) return s;
  if ((s = upload(ctx, &ctx->dBpool, &ctx->ownBpool, &capB, B, 2ull * b_rows * b_cols, kind)) != APK_OK) return s;
  if (ctx->dCpool) cudaFree(ctx->dCpool);
  ctx->dCpool = nullptr;
  APK_CU(cudaMalloc(&ctx->dCpool, 4ull * c_rows * c_cols));
  APK_CU(cudaMemsetAsync(ctx->dCpool, 0, 4ull * c_rows * c_cols, ctx->kstream));
  ctx->a_rows = a_rows;
  ctx->a_cols = a_cols;
  ctx->b_rows = b_rows;
  ctx->b_cols = b_cols;
  ctx->c_rows = c_rows;
  ctx->c_cols = c_cols;
  APK_CU(cudaStreamSynchronize(ctx->kstream));
  return APK_OK;
}

apk_status apk_set_tasks(apk_ctx* ctx, const apk_task* tasks, int n, long long n_chk,
                         unsigned long long* n_work_out) {
  if (!ctx || !tasks || n <= 0 || n_chk <= 0) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "set_tasks while a launch runs");
  if (!ctx->dApool) return fail(ctx, APK_ESTATE, "no task pool set");
  if (ctx->bf16_geo != BF16_GEO_STD64 && ctx->bf16_geo != BF16_GEO_STD32)
    return fail(ctx, APK_EUNSUPPORTED, "task mode runs the one-CTA-per-SM bf16 geometry (ctas_per_sm 0 or 1)");
  // a work-list entry packs task (20 bits), tile row and the tile's first
  // 128-column block (6 bits each); a tile is 256x256, or 256x128 where the
  // task's n ends 128 columns into it.  Checksums and oracle counters are
  // kept per 256x128 half (chk_base + tile_row * n/128 + block).
  if ((long long)n > (1ll << 20)) return fail(ctx, APK_EINVAL, "at most 2^20 tasks per context");
  static_assert(sizeof(apk_task) == sizeof(TaskDesc), "apk_task and TaskDesc must match");
  std::vector<unsigned> work;
  double flops = 0.0;
  unsigned long long halves = 0;
  for (int t = 0; t < n; ++t) {
    const apk_task& d = tasks[t];
    const int tiles_m = (d.m + 255) / 256, tiles_n = d.n / 128;
    if (d.m <= 0 || d.n <= 0 || d.k <= 0 || d.m % 128 || d.n % 128 || d.k % 64 || d.a_k0 % 64 || d.b_k0 % 64 ||
        d.b_col0 % 64 || d.c_col0 % 64 || d.a_row0 < 0 || d.a_k0 < 0 || d.b_k0 < 0 || d.b_col0 < 0 ||
        d.c_row0 < 0 || d.c_col0 < 0 || d.a_row0 + tiles_m * 256 > ctx->a_rows || d.a_k0 + d.k > ctx->a_cols ||
        d.b_k0 + d.k > ctx->b_rows || d.b_col0 + d.n > ctx->b_cols || d.c_row0 + d.m > ctx->c_rows ||
        d.c_col0 + d.n > ctx->c_cols || tiles_m > 63 || tiles_n > 63 || d.chk_base < 0 ||
        d.chk_base + (long long)tiles_m * tiles_n > n_chk)
      return fail(ctx, APK_EINVAL, "task %d does not fit the pools / checksum array", t);
    // 256x128 jobs for APK_TASK_NARROW tasks -- except on CTA pairs, whose
    // jobs are 256 wide
    const int step =
        ((d.flags & APK_TASK_NARROW) && !(pair_capable(ctx) && ctx->cfg.bf16_kernel == APK_BF16_PAIR)) ? 1 : 2;
    for (int tm = 0; tm < tiles_m; ++tm)
      for (int tn = 0; tn < tiles_n; tn += step)
        work.push_back(((unsigned)t << 12) | ((unsigned)tm << 6) | (unsigned)tn);
    flops += 2.0 * d.m * d.n * (double)d.k;
    halves += (unsigned long long)tiles_m * tiles_n;
  }
  APK_CU(cudaSetDevice(ctx->cfg.device));
  auto F = [](void* p) {
    if (p) cudaFree(p);
  };
  F(ctx->d_tasks);
  F(ctx->d_work);
  F(ctx->d_chk);
  ctx->d_tasks = nullptr;
  ctx->d_work = nullptr;
  ctx->d_chk = nullptr;
  APK_CU(cudaMalloc(&ctx->d_tasks, sizeof(TaskDesc) * n));
  APK_CU(cudaMalloc(&ctx->d_work, sizeof(unsigned) * work.size()));
  APK_CU(cudaMalloc(&ctx->d_chk, sizeof(double) * n_chk));
  APK_CU(cudaMemcpy(ctx->d_tasks, tasks, sizeof(TaskDesc) * n, cudaMemcpyHostToDevice));
  APK_CU(cudaMemcpy(ctx->d_work, work.data(), sizeof(unsigned) * work.size(), cudaMemcpyHostToDevice));
  ctx->n_tasks = n;
  ctx->n_work = work.size();
  ctx->n_halves = halves;
  ctx->n_chk = n_chk;
  ctx->task_flops = flops;
  ctx->task_mode = true;
  if (n_work_out) *n_work_out = ctx->n_work;
  return APK_OK;
}

apk_status apk_read_checksums(apk_ctx* ctx, double* chk, long long n) {
  if (!ctx || !chk || n <= 0) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "launch still running");
  if (!ctx->d_chk || n > ctx->n_chk) return fail(ctx, APK_EINVAL, "no checksum array of that size");
  APK_CU(cudaMemcpy(chk, ctx->d_chk, sizeof(double) * n, cudaMemcpyDeviceToHost));
  return APK_OK;
}

apk_status apk_read_pool_window(apk_ctx* ctx, int row0, int col0, int rows, int cols, float* out) {
  if (!ctx || !out || !ctx->dCpool || row0 < 0 || col0 < 0 || rows <= 0 || cols <= 0 ||
      row0 + rows > ctx->c_rows || col0 + cols > ctx->c_cols)
    return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "launch still running");
  APK_CU(cudaMemcpy2D(out, sizeof(float) * cols, ctx->dCpool + (size_t)row0 * ctx->c_cols + col0,
                      sizeof(float) * ctx->c_cols, sizeof(float) * cols, rows, cudaMemcpyDeviceToHost));
  return APK_OK;
}

apk_status apk_set_urgent(apk_ctx* ctx, const void* A, const void* B, int M, int N, int K,
                          apk_mem_kind kind) {
  if (!ctx) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "set_urgent while a launch runs");
  const int split = ctx->cfg.urgent_split_k;
  const int tm = ctx->cfg.dtype == APK_F32 ? 128 : 256;
  if (M <= 0 || N <= 0 || K <= 0 || M % tm || N % 128 || K % (ctx->slot_k * split))
    return fail(ctx, APK_EINVAL,
                "urgent shape %dx%dx%d: M a multiple of %d, N of 128, K of slot depth*split (%d)", M, N, K,
                tm, ctx->slot_k * split);
  APK_CU(cudaSetDevice(ctx->cfg.device));
  const size_t es = esize_of(ctx->cfg.dtype);
  size_t capAu = 0, capBu = 0;
  apk_status s;
  if ((s = upload(ctx, &ctx->dAu, &ctx->ownAu, &capAu, A, es * M * K, kind)) != APK_OK) return s;
  if ((s = upload(ctx, &ctx->dBu, &ctx->ownBu, &capBu, B, es * (size_t)K * N, kind)) != APK_OK) return s;
  if (ctx->dCu) cudaFree(ctx->dCu);
  ctx->cu_slot = (size_t)M * N;
  APK_CU(cudaMalloc(&ctx->dCu, sizeof(float) * ctx->cu_slot * (ctx->cfg.max_events + 1)));
  ctx->cu_dirty = ctx->cfg.max_events + 1;
  ctx->Mu = M;
  ctx->Nu = N;
  ctx->Ku = K;
  APK_CU(cudaStreamSynchronize(ctx->kstream));
  return APK_OK;
}

apk_status apk_schedule_device_events(apk_ctx* ctx, const long long* offsets_ns, int n) {
  if (!ctx) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "schedule while a launch runs");
  if (n < 0 || n > ctx->cfg.max_events) return fail(ctx, APK_EINVAL, "n=%d out of [0,max_events]", n);
  if (n > 0 && !offsets_ns) return fail(ctx, APK_EINVAL, "null schedule");
  if (n > 0) APK_CU(cudaMemcpy(ctx->d_sched, offsets_ns, sizeof(long long) * n, cudaMemcpyHostToDevice));
  ctx->n_sched = n;
  if (n > 0) ctx->n_count = 0;
  return APK_OK;
}

apk_status apk_schedule_count_events(apk_ctx* ctx, const unsigned long long* counts, int n) {
  if (!ctx) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "schedule while a launch runs");
  if (n < 0 || n > ctx->cfg.max_events) return fail(ctx, APK_EINVAL, "n=%d out of [0,max_events]", n);
  if (n > 0 && ctx->cfg.set_mode != APK_SET_DEVICE)
    return fail(ctx, APK_EINVAL, "count-triggered events need set_mode DEVICE");
  for (int k = 0; k < n; ++k)
    if (counts[k] == 0 || (k > 0 && counts[k] <= counts[k - 1]))
      return fail(ctx, APK_EINVAL, "counts must be positive and strictly ascending");
  if (n > 0)
    APK_CU(cudaMemcpy(ctx->d_count, counts, sizeof(unsigned long long) * n, cudaMemcpyHostToDevice));
  ctx->n_count = n;
  if (n > 0) ctx->n_sched = 0;
  return APK_OK;
}

}  // extern "C"

namespace {

// Fill the protocol structs for a launch of the main persistent kernel.
void fill_protos(apk_ctx* ctx, unsigned long long num_tasks, EventProto* ev, QueueProto* q,
                 int* flag_ptr) {
  Ctrl* cb = ctx->d_ctrl;
  memset(ev, 0, sizeof *ev);
  memset(q, 0, sizeof *q);
  ev->flag = flag_ptr;
  // the copies pay where 4 or 8 CTAs per SM poll (1184 pollers on one line
  // cost those drains a fifth of their speed); at 1 or 2 a single word is
  // polled and stored (a 4-byte copy lands ~1.5 us before a 4 KB one)
  ev->flag_lines = flag_ptr == &cb->flag_dev && ctx->ctas_per_sm >= 4 ? FLAG_LINES : 1;
  ctx->flag_lines = ev->flag_lines;
  ev->abort_word = &cb->abort_word;
  ev->status = &cb->status;
  ev->sched_ns = (ctx->cfg.set_mode == APK_SET_DEVICE && ctx->n_sched > 0) ? ctx->d_sched : nullptr;
  ev->n_sched = ctx->cfg.set_mode == APK_SET_DEVICE ? ctx->n_sched : 0;
  ev->max_events = ctx->cfg.max_events;
  ev->set_ns = ctx->d_set;
  ev->obs_ns = ctx->d_obs;
  ev->claim = ctx->d_claim;
  ev->claim_site = ctx->d_site;
  ev->inflight = ctx->d_inflight;
  ev->claim_ns = ctx->d_claim_ns;
  ev->done_ns = ctx->d_done;
  ev->uq_next = ctx->d_uq;
  ev->udone_cnt = ctx->d_udone;
  ev->ack = ctx->d_ack_mapped;
  ev->uexec = ctx->d_uexec;
  ev->count_trig = (ctx->cfg.set_mode == APK_SET_DEVICE && ctx->n_count > 0) ? ctx->d_count : nullptr;
  ev->n_count = ev->count_trig ? ctx->n_count : 0;
  ev->completed = &cb->completed;
  q->next_task = &cb->next_task;
  q->num_tasks = num_tasks;
  q->exec_count = ctx->d_exec;
  q->tiles_done = ctx->d_tiles;
  q->start_min = &cb->start_min;
  q->end_max = &cb->end_max;
  q->exited = &cb->exited;
  q->yields = &cb->yields;
  q->ckpt = cb->ckpt;
}

apk_status reset_logs(apk_ctx* ctx, unsigned long long num_tasks) {
  const int E = ctx->cfg.max_events, G = ctx->grid;
  cudaStream_t s = ctx->kstream;
  Ctrl init{};
  init.start_min = ~0ull;
  APK_CU(cudaMemcpyAsync(ctx->d_ctrl, &init, offsetof(Ctrl, flag_dev), cudaMemcpyHostToDevice, s));
  APK_CU(cudaMemsetAsync(&ctx->d_ctrl->flag_dev, 0, sizeof(int) * FLAG_LINES * FLAG_STRIDE, s));
  APK_CU(cudaMemsetAsync(ctx->d_set, 0, sizeof(long long) * E, s));
  APK_CU(cudaMemsetAsync(ctx->d_obs, 0, sizeof(long long) * (size_t)E * G, s));
  APK_CU(cudaMemsetAsync(ctx->d_claim_ns, 0, sizeof(long long) * E, s));
  APK_CU(cudaMemsetAsync(ctx->d_done, 0, sizeof(unsigned long long) * E, s));
  APK_CU(cudaMemsetAsync(ctx->d_claim, 0, sizeof(int) * E, s));
  APK_CU(cudaMemsetAsync(ctx->d_site, 0xFF, sizeof(int) * E, s));
  APK_CU(cudaMemsetAsync(ctx->d_inflight, 0, sizeof(int) * E, s));
  APK_CU(cudaMemsetAsync(ctx->d_uq, 0, sizeof(int) * E, s));
  APK_CU(cudaMemsetAsync(ctx->d_udone, 0, sizeof(int) * E, s));
  APK_CU(cudaMemsetAsync(ctx->d_uexec, 0, sizeof(int) * E, s));
  APK_CU(cudaMemsetAsync(ctx->d_tiles, 0, sizeof(unsigned long long) * G, s));
  APK_CU(cudaMemsetAsync(ctx->d_slab_hdr, 0, sizeof(long long) * 4 * G, s));
  // every urgent output slot starts the launch at zero (split-K items add
  // into it).  Only slots a previous launch could have written are cleared:
  // events it raised are bounded by the host injections (n_injected, reset
  // below) or by the device schedule it ran with.
  if (ctx->dCu) {
    const int used = std::min(E + 1, std::max({ctx->cu_dirty, ctx->n_injected.load(), ctx->dev_events_last}));
    if (used > 0) APK_CU(cudaMemsetAsync(ctx->dCu, 0, sizeof(float) * ctx->cu_slot * used, s));
    ctx->cu_dirty = 0;
  }
  ctx->dev_events_last = ctx->cfg.set_mode == APK_SET_DEVICE ? ctx->n_sched + ctx->n_count : 0;
  // verification launches pre-fill C with 0xFF bytes (NaN) so a tile that
  // never runs fails loudly (src/persistent.cu:156-160)
  if (ctx->cfg.oracle && ctx->dC && !ctx->task_mode)
    APK_CU(cudaMemsetAsync(ctx->dC, 0xFF, 4ull * ctx->M * ctx->N, s));
  if (ctx->task_mode) APK_CU(cudaMemsetAsync(ctx->d_chk, 0, sizeof(double) * ctx->n_chk, s));
  // oracle execution counters: one per queue entry, or in task mode one per
  // global tile (checksum index) so shards can be unioned
  const unsigned long long n_exec = ctx->task_mode ? (unsigned long long)ctx->n_chk : num_tasks;
  if (ctx->cfg.oracle && num_tasks != APK_TASKS_UNBOUNDED) {
    if (ctx->exec_cap < n_exec) {
      if (ctx->d_exec) cudaFree(ctx->d_exec);
      ctx->d_exec = nullptr;
      APK_CU(cudaMalloc(&ctx->d_exec, sizeof(int) * n_exec));
      ctx->exec_cap = n_exec;
    }
    APK_CU(cudaMemsetAsync(ctx->d_exec, 0, sizeof(int) * n_exec, s));
  }
  ctx->last_exec_n = n_exec;
  // host-side state
  std::atomic_thread_fence(std::memory_order_seq_cst);
  *reinterpret_cast<volatile int*>(ctx->h_flag) = 0;
  memset(ctx->h_ack, 0, sizeof(int) * 2 * E);
  std::atomic_thread_fence(std::memory_order_seq_cst);
  std::fill(ctx->host_set.begin(), ctx->host_set.end(), 0);
  std::fill(ctx->host_ack.begin(), ctx->host_ack.end(), 0);
  std::fill(ctx->host_done.begin(), ctx->host_done.end(), 0);
  ctx->n_injected = 0;
  return APK_OK;
}

apk_status launch_impl(apk_ctx* ctx, unsigned long long num_tasks, int poll, cudaStream_t stream,
                       bool record) {
  if (ctx->task_mode) {
    if (!ctx->dApool || !ctx->d_work) return fail(ctx, APK_ESTATE, "no tasks installed");
    if (num_tasks != APK_TASKS_UNBOUNDED && num_tasks > ctx->n_work)
      return fail(ctx, APK_EINVAL, "task mode drains at most the %llu work items", ctx->n_work);
    if (num_tasks == APK_TASKS_UNBOUNDED) return fail(ctx, APK_EINVAL, "task mode needs a bounded launch");
  } else if (!ctx->dA || !ctx->dB || !ctx->dC) {
    return fail(ctx, APK_ESTATE, "no background operands set");
  }
  if (!ctx->dAu && poll != APK_POLL_OFF) return fail(ctx, APK_ESTATE, "no urgent operands set");
  const bool clc = ctx->cfg.scheduler == APK_SCHED_CLC;
  if (clc && (num_tasks == APK_TASKS_UNBOUNDED || num_tasks > 0x3fffffffull))
    return fail(ctx, APK_EINVAL,
                "the CLC scheduler launches one CTA (a CTA pair) per task: a bounded launch of < 2^30 tasks");
  apk_status s = reset_logs(ctx, num_tasks);
  if (s != APK_OK) return s;
  int* flag = ctx->cfg.set_mode == APK_SET_HOST_MAPPED ? ctx->d_flag_mapped : &ctx->d_ctrl->flag_dev;
  EventProto ev;
  QueueProto q;
  fill_protos(ctx, num_tasks, &ev, &q, flag);
  if (clc) {
    APK_CU(cudaMemsetAsync(ctx->d_slot_bits, 0, sizeof(unsigned) * ((ctx->grid + 31) / 32), stream));
    APK_CU(cudaMemsetAsync(ctx->d_setter_state, 0, sizeof(long long) * 2, stream));
    q.slot_bits = ctx->d_slot_bits;
    q.setter_state = ctx->d_setter_state;
  }
  q.nslots = ctx->grid;
  if (!(ctx->cfg.oracle && num_tasks != APK_TASKS_UNBOUNDED)) q.exec_count = nullptr;
  ctx->last_tasks = num_tasks;
  ctx->last_grid = ctx->grid;
  cudaError_t e;
  if (record) APK_CU(cudaEventRecord(ctx->ev_start, stream));
  const bool f32 = ctx->cfg.dtype == APK_F32;
  const int bk = ctx->slot_k;  // K depth of one ring slot
  const int tm = tile_rows(ctx);
  F32Params p;
  memset(&p, 0, sizeof p);
  {
    // fp32: A as [tile rows][32 or 16 k] boxes (128B or 64B swizzle: one
    // swizzle span per row), B as [BK k][tile cols] boxes (no swizzle); the
    // warp-specialized kernel uses the 128x128 / 32 ones.  bf16: A as
    // [<=128 rows][BK k] boxes, one swizzle span per row (128B for BK 64,
    // 64B for BK 32), and B as [BK k][64 n] boxes, 128B swizzled (the
    // tcgen05 canonical K- / MN-major atoms).
    const CUtensorMapDataType dt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const int es = f32 ? 4 : 2;
    const GeoInfo fg = f32::geo_info(ctx->f32_geo);
    const int a_box_k = f32 ? fg.a_box_k : bk, b_box_n = f32 ? fg.tile_n : 64;
    const int a_box_m = f32 ? fg.tile_m : std::min(128, bf16::geo_info(ctx->bf16_geo).tile_m);
    const CUtensorMapSwizzle asw = (f32 ? a_box_k == 32 : bk == 64) ? CU_TENSOR_MAP_SWIZZLE_128B
                                                                    : CU_TENSOR_MAP_SWIZZLE_64B;
    const CUtensorMapSwizzle bsw = f32 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B;
    apk_status t;
    // task mode: the maps cover the operand pools, tasks are windows of them
    const bool tk = ctx->task_mode;
    const void* srcA = tk ? ctx->dApool : ctx->dA;
    const void* srcB = tk ? ctx->dBpool : ctx->dB;
    const long long ar = tk ? ctx->a_rows : ctx->M, ac = tk ? ctx->a_cols : ctx->K;
    const long long br = tk ? ctx->b_rows : ctx->K, bc = tk ? ctx->b_cols : ctx->N;
    if ((t = make_tmap(ctx, &p.tmA, srcA, dt, es, ar, ac, a_box_k, a_box_m, asw)) != APK_OK) return t;
    if ((t = make_tmap(ctx, &p.tmB, srcB, dt, es, br, bc, b_box_n, bk, bsw)) != APK_OK) return t;
    if (!f32) {
      const GeoInfo bg = bf16::geo_info(ctx->bf16_geo);
      const int chunks = bg.tile_n == 256 ? 4 : 2;
      if ((t = make_tmap(ctx, &p.tmAw, srcA, dt, es, ar, ac, bk, std::min(256, bg.tile_m), asw)) != APK_OK) return t;
      if ((t = make_tmap_chunks(ctx, &p.tmBw, srcB, dt, es, br, bc, bk, chunks, bsw)) != APK_OK) return t;
    }
    if (ctx->dAu) {
      if ((t = make_tmap(ctx, &p.tmAu, ctx->dAu, dt, es, ctx->Mu, ctx->Ku, a_box_k, a_box_m, asw)) != APK_OK)
        return t;
      if ((t = make_tmap(ctx, &p.tmBu, ctx->dBu, dt, es, ctx->Ku, ctx->Nu, b_box_n, bk, bsw)) != APK_OK) return t;
    } else {
      p.tmAu = p.tmA;
      p.tmBu = p.tmB;
    }
  }
  if (ctx->task_mode) {
    p.C = ctx->dCpool;
    p.ldc = ctx->c_cols;
    p.tiles_n = 1;
    p.total_tiles = 1;
    p.nk = 1;
    p.task_mode = 1;
    p.work = ctx->d_work;
    p.tasks = ctx->d_tasks;
    p.chk = ctx->d_chk;
  } else {
    p.C = reinterpret_cast<float*>(ctx->dC);
    p.ldc = ctx->N;
    p.tiles_n = tiles_across(ctx, ctx->N);
    p.total_tiles = (ctx->M / tm) * p.tiles_n;
    p.nk = ctx->K / bk;
  }
  p.Cu = ctx->dCu;
  p.cu_stride = (long long)ctx->cu_slot;
  p.ldcu = ctx->Nu;
  p.utiles_n = tiles_across(ctx, ctx->Nu);
  p.usplit = ctx->cfg.urgent_split_k;
  p.unk = ctx->Ku ? ctx->Ku / bk / p.usplit : 0;
  p.uitems = (ctx->Mu / tm) * p.utiles_n * p.usplit;
  p.poll_every = ctx->poll_every;
  p.narrow_all = narrow_jobs(ctx) ? 1 : 0;
  p.park = ctx->cfg.dtype == APK_BF16 && ctx->cfg.bf16_kernel == APK_BF16_NARROW ? 1 : 0;
  p.slab = ctx->d_slab;
  p.slab_hdr = ctx->d_slab_hdr;
  p.wait_limit_ns = ctx->cfg.wait_limit_ns;
  p.ev = ev;
  p.q = q;
  p.st = ctx->st_cfg;
  if (f32 && use_ws(ctx))
    e = f32ws::launch(p, ctx->grid, poll, ctx->cfg.discipline, ctx->cfg.oracle != 0, stream);
  else if (f32)
    e = f32::launch(p, ctx->cfg.scheduler == APK_SCHED_CLC ? (int)num_tasks : ctx->grid, poll,
                    ctx->cfg.discipline, ctx->cfg.oracle != 0, ctx->f32_geo, ctx->cfg.scheduler, stream);
  else if (use_pair(ctx))
    e = bf16pair::launch(p, clc ? 2 * (int)num_tasks : ctx->grid, poll, ctx->cfg.discipline, ctx->cfg.oracle != 0,
                         clc, stream);
  else
    e = bf16::launch(p, clc ? (int)num_tasks : ctx->grid, poll, ctx->cfg.discipline, ctx->cfg.oracle != 0,
                     ctx->bf16_geo, ctx->cfg.scheduler, stream);
  if (e != cudaSuccess) return fail(ctx, APK_ECUDA, "kernel launch failed: %s", cudaGetErrorString(e));
  if (record) APK_CU(cudaEventRecord(ctx->ev_done, stream));
  return APK_OK;
}

apk_status read_status(apk_ctx* ctx) {
  int status = 0;  // the word alone: the control block is ~4 KB with the flag lines
  APK_CU(cudaMemcpy(&status, &ctx->d_ctrl->status, sizeof status, cudaMemcpyDeviceToHost));
  if (status != 0)
    return fail(ctx, APK_EDEVICE, "device reported status %d (a bounded wait ran out)", status);
  return APK_OK;
}

// Copy schedule of a streamed apk_gemm.  A moves in row panels of panel_tm
// tile rows, B in column panels of b_units 128-column units.  After A panel
// 0, each next copy is the next A row panel or the next B column panel,
// whichever makes more tiles computable per byte copied; tiles are visited
// in the order they become computable (column-major within each step's new
// tiles).  The kernel pops tiles in that order and waits for each tile's
// panels, so no CTA waits behind a tile whose operands come later.
struct StreamPlan {
  std::vector<int> copies;       // >= 0: A row panel; < 0: B column panel -(j + 1)
  std::vector<unsigned> order;   // tile visit order, tm * tiles_n + tn
};

StreamPlan plan_stream(int tiles_m, int tiles_n, int panel_tm, int np, int nb, int tn_units, int n_units,
                       int b_units, double a_bytes_per_tile_row, double b_bytes_per_unit) {
  // the last B column panel tile column tn needs
  auto last_bpanel = [&](int tn) {
    const int last_unit = std::min(n_units, (tn + 1) * tn_units) - 1;
    return last_unit / b_units;
  };
  // tile columns computable once B panels 0 .. b-1 are in (monotone in b)
  std::vector<int> cols_ready(nb + 1, 0);
  for (int b = 0, tn = 0; b <= nb; ++b) {
    while (tn < tiles_n && last_bpanel(tn) < b) ++tn;
    cols_ready[b] = tn;
  }
  auto rows_ready = [&](int a) { return std::min(tiles_m, a * panel_tm); };
  StreamPlan pl;
  pl.order.reserve((size_t)tiles_m * tiles_n);
  int a = 0, b = 0;
  while (a < np || b < nb) {
    bool take_a;
    if (a == 0 || b == nb) {
      take_a = true;
    } else if (a == np) {
      take_a = false;
    } else {
      // new computable tiles per byte of each candidate copy
      const int ra = rows_ready(a), rn = rows_ready(a + 1) - ra;
      const int ca = cols_ready[b], cn = cols_ready[b + 1] - ca;
      const int units = std::min(n_units, (b + 1) * b_units) - b * b_units;
      const double ga = (double)rn * ca / (a_bytes_per_tile_row * rn);
      const double gb = (double)ra * cn / (b_bytes_per_unit * units);
      take_a = ga >= gb;
    }
    if (take_a) {
      const int r0 = rows_ready(a), r1 = rows_ready(a + 1);
      for (int tn = 0; tn < cols_ready[b]; ++tn)
        for (int tm = r0; tm < r1; ++tm) pl.order.push_back((unsigned)(tm * tiles_n + tn));
      pl.copies.push_back(a++);
    } else {
      for (int tn = cols_ready[b]; tn < cols_ready[b + 1]; ++tn)
        for (int tm = 0; tm < rows_ready(a); ++tm) pl.order.push_back((unsigned)(tm * tiles_n + tn));
      pl.copies.push_back(-(b++) - 1);
    }
  }
  return pl;
}

// apk_gemm from host memory with the transfers overlapped: on a copy stream
// the tile-visit order, then A row panels and B column panels in the order
// plan_stream picks, each followed by a 4-byte readiness write (copy engine,
// no SM); the kernel, launched at once, visits tiles in that order and
// starts a tile when its A and B panels are flagged; every finished C block
// (row panel x cb_tn tile columns) is acknowledged through mapped memory and
// copied back on a second stream while the rest still computes.
apk_status gemm_streamed(apk_ctx* ctx, const char* A, const char* B, float* C) {
  const int M = ctx->M, N = ctx->N, K = ctx->K;
  const size_t es = esize_of(ctx->cfg.dtype);
  const int TM = tile_rows(ctx), tiles_m = M / TM;
  const int TN = tile_cols(ctx), tiles_n = tiles_across(ctx, N), tn_units = TN / 128, n_units = N / 128;
  const int panel_tm = 8, np = (tiles_m + panel_tm - 1) / panel_tm;
  const int b_units = N % 512 == 0 ? 4 : 1;  // 128-column units per B panel
  const int nb = n_units / b_units;
  const int cb_tn = std::max(1, b_units / tn_units), n_cb = (tiles_n + cb_tn - 1) / cb_tn;
  const int nblk = np * n_cb, ntiles = tiles_m * tiles_n;
  // The warp-specialized fp32 kernel takes K in two chained slices: both
  // operands move as K halves, all slice-0 jobs first, so slice-0 tiles
  // compute while the second half is still being copied and the tiles the
  // last copies unlock need half a tile's time (4096^3: modelled 4.13 ->
  // 3.52 ms per call).  Other kernels, or an odd or short K, take whole K.
  const int nk = K / ctx->slot_k;
  const int ks = (ctx->cfg.dtype == APK_F32 && use_ws(ctx) && nk % 2 == 0 && nk >= 4) ? 2 : 1;
  const int kh = K / ks;  // K elements per slice
  const int nslots = ntiles * ks;
  if (!ctx->h2dstream) {
    APK_CU(cudaStreamCreateWithFlags(&ctx->h2dstream, cudaStreamNonBlocking));
    APK_CU(cudaStreamCreateWithFlags(&ctx->d2hstream, cudaStreamNonBlocking));
    APK_CU(cudaEventCreateWithFlags(&ctx->ev_reset, cudaEventDisableTiming));
    APK_CU(cudaHostAlloc(&ctx->h_one, sizeof(int), cudaHostAllocPortable));
    *ctx->h_one = 1;
  }
  if (ctx->stream_cap < (np + nb) * ks) {
    if (ctx->d_ready) cudaFree(ctx->d_ready);
    ctx->d_ready = nullptr;
    APK_CU(cudaMalloc(&ctx->d_ready, sizeof(int) * (np + nb) * ks));
    ctx->stream_cap = (np + nb) * ks;
  }
  if (ks > 1 && ctx->part_cap < ntiles) {
    if (ctx->d_part) cudaFree(ctx->d_part);
    if (ctx->d_part_ready) cudaFree(ctx->d_part_ready);
    ctx->d_part = nullptr;
    ctx->d_part_ready = nullptr;
    APK_CU(cudaMalloc(&ctx->d_part, sizeof(float) * (size_t)ntiles * TM * TN));
    APK_CU(cudaMalloc(&ctx->d_part_ready, sizeof(int) * ntiles));
    ctx->part_cap = ntiles;
  }
  if (ctx->pack_cap < nblk) {
    if (ctx->d_pdone) cudaFree(ctx->d_pdone);
    if (ctx->h_pack) cudaFreeHost(ctx->h_pack);
    ctx->d_pdone = nullptr;
    ctx->h_pack = nullptr;
    APK_CU(cudaMalloc(&ctx->d_pdone, sizeof(unsigned) * nblk));
    APK_CU(cudaHostAlloc(&ctx->h_pack, sizeof(int) * nblk, cudaHostAllocMapped | cudaHostAllocPortable));
    APK_CU(cudaHostGetDevicePointer(reinterpret_cast<void**>(&ctx->d_pack_mapped), ctx->h_pack, 0));
    ctx->pack_cap = nblk;
  }
  if (ctx->order_cap < nslots) {
    if (ctx->d_order) cudaFree(ctx->d_order);
    if (ctx->h_order) cudaFreeHost(ctx->h_order);
    ctx->d_order = nullptr;
    ctx->h_order = nullptr;
    APK_CU(cudaMalloc(&ctx->d_order, sizeof(unsigned) * nslots));
    APK_CU(cudaHostAlloc(&ctx->h_order, sizeof(unsigned) * nslots, cudaHostAllocPortable));
    ctx->order_cap = nslots;
  }
  const StreamPlan plan = plan_stream(tiles_m, tiles_n, panel_tm, np, nb, tn_units, n_units, b_units,
                                      (double)TM * kh * es, (double)128 * kh * es);
  if ((int)plan.order.size() != ntiles)
    return fail(ctx, APK_EINVAL, "stream plan covers %d of %d tiles", (int)plan.order.size(), ntiles);
  // the previous call's copies have completed (its streams were synchronised).
  // Slot order: every tile's slice 0, then every tile's slice 1, each in the
  // plan's order (a slice-1 job's predecessor is always popped before it).
  for (int h = 0; h < ks; ++h)
    for (int i = 0; i < ntiles; ++i) ctx->h_order[(size_t)h * ntiles + i] = plan.order[i] * ks + h;
  volatile int* ack = ctx->h_pack;
  for (int i = 0; i < nblk; ++i) ack[i] = 0;
  std::atomic_thread_fence(std::memory_order_seq_cst);
  cudaStream_t hs = ctx->h2dstream, ds = ctx->d2hstream;
  APK_CU(cudaMemsetAsync(ctx->d_ready, 0, sizeof(int) * (np + nb) * ks, hs));
  APK_CU(cudaMemsetAsync(ctx->d_pdone, 0, sizeof(unsigned) * nblk, hs));
  if (ks > 1) APK_CU(cudaMemsetAsync(ctx->d_part_ready, 0, sizeof(int) * ntiles, hs));
  APK_CU(cudaMemcpyAsync(ctx->d_order, ctx->h_order, sizeof(unsigned) * nslots, cudaMemcpyHostToDevice, hs));
  APK_CU(cudaEventRecord(ctx->ev_reset, hs));
  char* dA = static_cast<char*>(ctx->dA);
  char* dB = static_cast<char*>(ctx->dB);
  const size_t bw = (size_t)128 * b_units * es;  // bytes per B panel row
  for (int h = 0; h < ks; ++h) {
    const size_t ka = (size_t)h * kh * es;  // byte offset of the slice in an A row
    const size_t kb = (size_t)h * kh * N * es;  // byte offset of the slice's first B row
    for (const int c : plan.copies) {
      if (c >= 0) {
        const size_t r0 = (size_t)c * panel_tm * TM;
        const size_t rows = std::min((size_t)M - r0, (size_t)panel_tm * TM);
        if (ks == 1)
          APK_CU(cudaMemcpyAsync(dA + r0 * K * es, A + r0 * K * es, rows * K * es, cudaMemcpyHostToDevice, hs));
        else
          APK_CU(cudaMemcpy2DAsync(dA + r0 * K * es + ka, (size_t)K * es, A + r0 * K * es + ka, (size_t)K * es,
                                   (size_t)kh * es, rows, cudaMemcpyHostToDevice, hs));
        APK_CU(cudaMemcpyAsync(ctx->d_ready + c * ks + h, ctx->h_one, sizeof(int), cudaMemcpyHostToDevice, hs));
      } else {
        const int j = -c - 1;
        APK_CU(cudaMemcpy2DAsync(dB + kb + j * bw, (size_t)N * es, B + kb + j * bw, (size_t)N * es, bw, kh,
                                 cudaMemcpyHostToDevice, hs));
        APK_CU(cudaMemcpyAsync(ctx->d_ready + (np + j) * ks + h, ctx->h_one, sizeof(int), cudaMemcpyHostToDevice,
                               hs));
      }
    }
  }

  StreamProto st{};
  st.a_ready = ctx->d_ready;
  st.b_ready = ctx->d_ready + np * ks;  // flags are [panel * ks + slice]
  st.b_units = b_units;
  st.panel_tm = panel_tm;
  st.n_panels = np;
  st.cb_tn = cb_tn;
  st.n_cb = n_cb;
  st.order = ctx->d_order;
  st.done = ctx->d_pdone;
  st.ack = ctx->d_pack_mapped;
  st.ksplit = ks;
  st.part = ks > 1 ? ctx->d_part : nullptr;
  st.part_ready = ks > 1 ? ctx->d_part_ready : nullptr;
  ctx->st_cfg = st;
  APK_CU(cudaStreamWaitEvent(ctx->kstream, ctx->ev_reset, 0));
  const int poll = ctx->dAu ? (int)ctx->cfg.poll : APK_POLL_OFF;
  apk_status s = launch_impl(ctx, (unsigned long long)nslots, poll, ctx->kstream, true);
  ctx->st_cfg = StreamProto{};
  if (s != APK_OK) return s;
  ctx->running = true;
  // copy each C block back once the device has acknowledged it, in the
  // order they finish; if the kernel ends with a block unacknowledged (an
  // aborted run) stop waiting
  apk_status out = APK_OK;
  std::vector<char> sent(nblk, 0);
  float* dC = static_cast<float*>(ctx->dC);
  int left = nblk;
  bool ended = false;
  while (left > 0 && out == APK_OK) {
    bool any = false;
    for (int blk = 0; blk < nblk; ++blk) {
      if (sent[blk] || ack[blk] == 0) continue;
      const int pn = blk / n_cb, cb = blk % n_cb;
      const size_t r0 = (size_t)pn * panel_tm * TM;
      const size_t rows = std::min((size_t)M - r0, (size_t)panel_tm * TM);
      const size_t c0 = (size_t)cb * cb_tn * TN;
      const size_t cols = std::min((size_t)N - c0, (size_t)cb_tn * TN);
      APK_CU(cudaMemcpy2DAsync(C + r0 * N + c0, (size_t)N * sizeof(float), dC + r0 * N + c0,
                               (size_t)N * sizeof(float), cols * sizeof(float), rows, cudaMemcpyDeviceToHost, ds));
      sent[blk] = 1;
      --left;
      any = true;
    }
    if (!any) {
      if (ended) {
        for (int blk = 0; blk < nblk && out == APK_OK; ++blk)
          if (!sent[blk]) out = fail(ctx, APK_EDEVICE, "kernel ended without finishing C block %d", blk);
      } else {
        const cudaError_t q = cudaEventQuery(ctx->ev_done);
        if (q == cudaSuccess) {
          // one more scan sees every ack the finished kernel wrote
          std::atomic_thread_fence(std::memory_order_seq_cst);
          ended = true;
        } else if (q != cudaErrorNotReady) {
          // a sticky error (failed launch, faulted kernel): no further ack
          // will come and every later query fails the same way
          out = fail(ctx, APK_ECUDA, "streamed GEMM kernel failed: %s", cudaGetErrorString(q));
        }
      }
    }
  }
  APK_CU(cudaStreamSynchronize(ds));
  APK_CU(cudaStreamSynchronize(hs));
  APK_CU(cudaStreamSynchronize(ctx->kstream));
  ctx->running = false;
  const apk_status st2 = read_status(ctx);
  return out != APK_OK ? out : st2;
}

}  // namespace

extern "C" {

apk_status apk_launch(apk_ctx* ctx, unsigned long long num_tasks) {
  if (!ctx) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "a launch is already running");
  if (num_tasks == 0) return fail(ctx, APK_EINVAL, "num_tasks must be > 0");
  if (ctx->cfg.poll == APK_POLL_OFF && num_tasks == APK_TASKS_UNBOUNDED) {
    // POLL_OFF kernels still stop through the abort word at tile boundaries
  }
  APK_CU(cudaSetDevice(ctx->cfg.device));
  apk_status s = launch_impl(ctx, num_tasks, ctx->cfg.poll, ctx->kstream, true);
  if (s != APK_OK) return s;
  ctx->running = true;
  return APK_OK;
}

namespace {
// HOST_MEMCPY: the generation goes to every flag line in one contiguous
// copy-engine transfer of the 4 KB of lines (a 2-D copy of one word per
// line took ~4 us longer to land).  The pinned image comes from a ring;
// a slot is rewritten only after the copy that read it has run.
cudaError_t stage_flag_lines(apk_ctx* ctx, int value, int** src) {
  const int slot = ctx->flag_ring_next;
  ctx->flag_ring_next = (slot + 1) % apk_ctx::kFlagRing;
  cudaError_t e = cudaEventSynchronize(ctx->flag_ring_ev[slot]);
  if (e != cudaSuccess) return e;
  int* img = ctx->h_flag_ring + (size_t)slot * FLAG_LINES * FLAG_STRIDE;
  for (int i = 0; i < FLAG_LINES; ++i) img[i * FLAG_STRIDE] = value;
  *src = img;
  return cudaSuccess;
}
cudaError_t copy_flag_lines(apk_ctx* ctx, const int* src) {
  const size_t bytes = ctx->flag_lines > 1 ? sizeof(int) * FLAG_LINES * FLAG_STRIDE : sizeof(int);
  cudaError_t e = cudaMemcpyAsync(&ctx->d_ctrl->flag_dev, src, bytes, cudaMemcpyHostToDevice, ctx->cstream);
  if (e != cudaSuccess) return e;
  const int slot = (ctx->flag_ring_next + apk_ctx::kFlagRing - 1) % apk_ctx::kFlagRing;
  return cudaEventRecord(ctx->flag_ring_ev[slot], ctx->cstream);
}
}  // namespace

apk_status apk_inject_urgent(apk_ctx* ctx, int* event, long long* host_set_ns) {
  if (!ctx) return APK_EINVAL;
  if (ctx->cfg.set_mode == APK_SET_DEVICE)
    return fail(ctx, APK_EINVAL, "set_mode is DEVICE: events come from the device schedule");
  const int gen = ctx->n_injected.load() + 1;
  if (gen > ctx->cfg.max_events) return fail(ctx, APK_EINVAL, "event log full (%d)", ctx->cfg.max_events);
  long long t;
  if (ctx->cfg.set_mode == APK_SET_HOST_MAPPED) {
    t = host_now_ns();
    *reinterpret_cast<volatile int*>(ctx->h_flag) = gen;
    std::atomic_thread_fence(std::memory_order_seq_cst);
  } else {
    int* src = nullptr;
    APK_CU(stage_flag_lines(ctx, gen, &src));
    t = host_now_ns();
    APK_CU(copy_flag_lines(ctx, src));
  }
  ctx->host_set[gen - 1] = t;
  ctx->n_injected = gen;
  if (event) *event = gen - 1;
  if (host_set_ns) *host_set_ns = t;
  return APK_OK;
}

apk_status apk_wait_ack(apk_ctx* ctx, int event, int which, long long timeout_ns, long long* seen) {
  if (!ctx || event < 0 || event >= ctx->cfg.max_events || (which != 0 && which != 1)) return APK_EINVAL;
  volatile int* a = reinterpret_cast<volatile int*>(ctx->h_ack) + 2 * event + which;
  const long long t0 = host_now_ns();
  while (true) {
    if (*a != 0) {
      const long long t = host_now_ns();
      if (which == 0) ctx->host_ack[event] = t;
      else ctx->host_done[event] = t;
      if (seen) *seen = t;
      return APK_OK;
    }
    if (host_now_ns() - t0 > timeout_ns) return fail(ctx, APK_ETIMEDOUT, "ack %d of event %d not seen", which, event);
  }
}

apk_status apk_stop(apk_ctx* ctx) {
  if (!ctx) return APK_EINVAL;
  static const int kStop = -1, kOne = 1;
  ctx->h_gen[ctx->cfg.max_events + 1] = kStop;
  if (ctx->cfg.set_mode == APK_SET_HOST_MAPPED) {
    *reinterpret_cast<volatile int*>(ctx->h_flag) = kStop;
    std::atomic_thread_fence(std::memory_order_seq_cst);
  } else {
    int* src = nullptr;
    APK_CU(stage_flag_lines(ctx, kStop, &src));
    APK_CU(copy_flag_lines(ctx, src));
  }
  // the abort word also stops POLL_OFF kernels at their next tile boundary
  ctx->h_gen[0] = kOne;
  APK_CU(cudaMemcpyAsync(&ctx->d_ctrl->abort_word, &ctx->h_gen[0], sizeof(int), cudaMemcpyHostToDevice,
                         ctx->cstream));
  APK_CU(cudaStreamSynchronize(ctx->cstream));
  (void)kOne;
  return APK_OK;
}

apk_status apk_wait(apk_ctx* ctx, long long timeout_ns) {
  if (!ctx) return APK_EINVAL;
  if (!ctx->running) return APK_OK;
  const long long t0 = host_now_ns();
  while (true) {
    cudaError_t q = cudaEventQuery(ctx->ev_done);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) {
      ctx->running = false;
      return fail(ctx, APK_ECUDA, "kernel failed: %s", cudaGetErrorString(q));
    }
    const long long waited = host_now_ns() - t0;
    if (waited > timeout_ns) return fail(ctx, APK_ETIMEDOUT, "launch still running");
    // poll without sleeping for the first 2 ms (a sleep of 50 us ended short
    // launches up to ~60 us late), then yield the core between polls
    if (waited > 2000000) std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  ctx->running = false;
  APK_CU(cudaGetLastError());
  return read_status(ctx);
}

apk_status apk_read_output(apk_ctx* ctx, void* C_host) {
  if (!ctx || !C_host) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "launch still running");
  APK_CU(cudaMemcpy(C_host, ctx->dC, 4ull * ctx->M * ctx->N, cudaMemcpyDeviceToHost));
  return APK_OK;
}

apk_status apk_read_urgent_output(apk_ctx* ctx, int event, float* Cu_host) {
  if (!ctx || !Cu_host || event < 0 || event > ctx->cfg.max_events || !ctx->dCu) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "launch still running");
  APK_CU(cudaMemcpy(Cu_host, ctx->dCu + ctx->cu_slot * event, sizeof(float) * ctx->cu_slot,
                    cudaMemcpyDeviceToHost));
  return APK_OK;
}

apk_status apk_read_events(apk_ctx* ctx, apk_event_log* log) {
  if (!ctx || !log) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "launch still running");
  const int E = ctx->cfg.max_events;
  log->n_injected = ctx->n_injected;
  log->grid = ctx->last_grid;
  auto D = [&](void* dst, const void* src, size_t bytes) -> apk_status {
    if (dst) APK_CU(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
    return APK_OK;
  };
  apk_status s;
  if ((s = D(log->set_ns, ctx->d_set, sizeof(long long) * E)) != APK_OK) return s;
  if ((s = D(log->claim_ns, ctx->d_claim_ns, sizeof(long long) * E)) != APK_OK) return s;
  if ((s = D(log->done_ns, ctx->d_done, sizeof(long long) * E)) != APK_OK) return s;
  if ((s = D(log->claimer, ctx->d_claim, sizeof(int) * E)) != APK_OK) return s;
  if ((s = D(log->claim_site, ctx->d_site, sizeof(int) * E)) != APK_OK) return s;
  if ((s = D(log->inflight, ctx->d_inflight, sizeof(int) * E)) != APK_OK) return s;
  if ((s = D(log->obs_ns, ctx->d_obs, sizeof(long long) * (size_t)E * ctx->last_grid)) != APK_OK) return s;
  if (log->host_set_ns) memcpy(log->host_set_ns, ctx->host_set.data(), sizeof(long long) * E);
  if (log->host_ack_ns) memcpy(log->host_ack_ns, ctx->host_ack.data(), sizeof(long long) * E);
  if (log->host_done_ns) memcpy(log->host_done_ns, ctx->host_done.data(), sizeof(long long) * E);
  std::vector<long long> set(E);
  APK_CU(cudaMemcpy(set.data(), ctx->d_set, sizeof(long long) * E, cudaMemcpyDeviceToHost));
  log->n_fired = (int)std::count_if(set.begin(), set.end(), [](long long v) { return v != 0; });
  return APK_OK;
}

apk_status apk_read_oracle(apk_ctx* ctx, int* exec_counts, int* uexec_counts) {
  if (!ctx) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "launch still running");
  if (!ctx->cfg.oracle) return fail(ctx, APK_ESTATE, "context was created without oracle counters");
  if (exec_counts) {
    if (ctx->last_tasks == APK_TASKS_UNBOUNDED || !ctx->d_exec)
      return fail(ctx, APK_ESTATE, "per-task counts need a bounded launch");
    // one counter per queue entry, or per global tile in task mode
    APK_CU(cudaMemcpy(exec_counts, ctx->d_exec, sizeof(int) * ctx->last_exec_n, cudaMemcpyDeviceToHost));
  }
  if (uexec_counts)
    APK_CU(cudaMemcpy(uexec_counts, ctx->d_uexec, sizeof(int) * ctx->cfg.max_events, cudaMemcpyDeviceToHost));
  return APK_OK;
}

apk_status apk_read_run_stats(apk_ctx* ctx, apk_run_stats* st) {
  if (!ctx || !st) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "launch still running");
  Ctrl cb;  // the counters precede the flag lines
  APK_CU(cudaMemcpy(&cb, ctx->d_ctrl, offsetof(Ctrl, flag_dev), cudaMemcpyDeviceToHost));
  std::vector<unsigned long long> t(ctx->last_grid);
  APK_CU(cudaMemcpy(t.data(), ctx->d_tiles, sizeof(unsigned long long) * ctx->last_grid, cudaMemcpyDeviceToHost));
  memset(st, 0, sizeof *st);
  st->start_ns = (long long)cb.start_min;
  st->end_ns = (long long)cb.end_max;
  for (auto v : t) st->tiles_done += v;
  st->yields = cb.yields;
  if (ctx->cfg.dtype == APK_BF16) {
    // the epilogue warps of a CTA split a checkpoint evenly and run side by
    // side: their summed time / warps is the CTA's wall time
    st->ckpt_spill_bytes = cb.ckpt[1];
    st->ckpt_restore_bytes = cb.ckpt[3];
    // (the pair kernel: 16 warps over two CTAs spill side by side; bytes
    // cover the pair)
    const unsigned long long w =
        use_pair(ctx) ? 2ull * bf16pair::epi_warps() : (unsigned long long)bf16::epi_warps(ctx->bf16_geo);
    st->ckpt_spill_ns = (long long)(cb.ckpt[0] / w);
    st->ckpt_restore_ns = (long long)(cb.ckpt[2] / w);
    st->parks = cb.ckpt[4];
  }
  if (ctx->task_mode) {
    // tiles differ in size: a complete drain did every task's 2*m*n*k; a
    // partial one is prorated by the 256x128 halves it completed
    st->bg_flops = ctx->n_halves ? ctx->task_flops * (double)st->tiles_done / (double)ctx->n_halves : 0.0;
  } else {
    // the average tile (bf16 tiles at the right edge may be 128 wide)
    const double tiles = (double)(ctx->M / tile_rows(ctx)) * tiles_across(ctx, ctx->N);
    st->bg_flops = tiles > 0 ? 2.0 * ctx->M * ctx->N * (double)ctx->K / tiles * (double)st->tiles_done : 0.0;
  }
  const double dt = (double)(st->end_ns - st->start_ns) * 1e-9;
  st->bg_tflops = dt > 0 ? st->bg_flops / dt / 1e12 : 0.0;
  st->exited = cb.exited;
  st->device_status = cb.status;
  float ms = 0.f;
  if (cudaEventElapsedTime(&ms, ctx->ev_start, ctx->ev_done) == cudaSuccess) st->launch_ms = ms;
  else cudaGetLastError();
  return APK_OK;
}

apk_status apk_gemm(apk_ctx* ctx, const void* A, const void* B, void* C, int M, int N, int K,
                    apk_mem_kind kind) {
  if (!ctx || !A || !B || !C) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "a launch is already running");
  APK_CU(cudaSetDevice(ctx->cfg.device));
  if (M <= 0 || N <= 0 || K <= 0 || M % 128 || N % 128 || K % ctx->cfg.k_tile)
    return fail(ctx, APK_EINVAL, "shape %dx%dx%d not tile-aligned", M, N, K);
  if (ctx->cfg.dtype == APK_BF16 && M % 256) return fail(ctx, APK_EINVAL, "bf16 M must be a multiple of 256");
  const size_t es = esize_of(ctx->cfg.dtype);
  apk_status s;
  if (kind == APK_MEM_HOST && ctx->cfg.dtype == APK_F32 &&
      (ctx->f32_geo == F32_GEO_M || ctx->f32_geo == F32_GEO_S)) {
    // the 4- and 8-CTA-per-SM fp32 geometries are not streamed: whole
    // operands in, one resident drain, C out
    if ((s = upload(ctx, &ctx->dA, &ctx->ownA, &ctx->capA, A, es * M * K, kind)) != APK_OK) return s;
    if ((s = upload(ctx, &ctx->dB, &ctx->ownB, &ctx->capB, B, es * (size_t)K * N, kind)) != APK_OK) return s;
    if ((s = upload(ctx, &ctx->dC, &ctx->ownC, &ctx->capC, nullptr, 4ull * M * N, kind)) != APK_OK) return s;
    ctx->M = M;
    ctx->N = N;
    ctx->K = K;
    const unsigned long long tiles = (unsigned long long)(M / tile_rows(ctx)) * tiles_across(ctx, N);
    const int poll = ctx->dAu ? (int)ctx->cfg.poll : APK_POLL_OFF;
    if ((s = launch_impl(ctx, tiles, poll, ctx->kstream, true)) != APK_OK) return s;
    ctx->running = true;
    APK_CU(cudaMemcpyAsync(C, ctx->dC, 4ull * M * N, cudaMemcpyDeviceToHost, ctx->kstream));
    APK_CU(cudaStreamSynchronize(ctx->kstream));
    ctx->running = false;
    return read_status(ctx);
  }
  if (kind == APK_MEM_HOST) {
    // device buffers only: the operands stream in while the kernel runs
    if ((s = upload(ctx, &ctx->dA, &ctx->ownA, &ctx->capA, nullptr, es * M * K, kind)) != APK_OK) return s;
    if ((s = upload(ctx, &ctx->dB, &ctx->ownB, &ctx->capB, nullptr, es * (size_t)K * N, kind)) != APK_OK) return s;
    if ((s = upload(ctx, &ctx->dC, &ctx->ownC, &ctx->capC, nullptr, 4ull * M * N, kind)) != APK_OK) return s;
    ctx->M = M;
    ctx->N = N;
    ctx->K = K;
    return gemm_streamed(ctx, static_cast<const char*>(A), static_cast<const char*>(B), static_cast<float*>(C));
  } else {
    if (ctx->ownA && ctx->dA) cudaFree(ctx->dA);
    if (ctx->ownB && ctx->dB) cudaFree(ctx->dB);
    if (ctx->ownC && ctx->dC) cudaFree(ctx->dC);
    ctx->dA = const_cast<void*>(A);
    ctx->dB = const_cast<void*>(B);
    ctx->dC = C;
    ctx->ownA = ctx->ownB = ctx->ownC = false;
    ctx->capA = ctx->capB = ctx->capC = 0;
  }
  ctx->M = M;
  ctx->N = N;
  ctx->K = K;
  const unsigned long long tiles = (unsigned long long)(M / tile_rows(ctx)) * tiles_across(ctx, N);
  const int poll = ctx->dAu ? (int)ctx->cfg.poll : APK_POLL_OFF;
  if ((s = launch_impl(ctx, tiles, poll, ctx->kstream, true)) != APK_OK) return s;
  ctx->running = true;
  APK_CU(cudaStreamSynchronize(ctx->kstream));
  ctx->running = false;
  return read_status(ctx);
}

apk_status apk_probe_copy(apk_ctx* ctx, const void* A, const void* B, void* C, int reps, double* out_ms) {
  if (!ctx || !A || !B || !C || reps <= 0 || !out_ms) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "probe needs an idle device");
  const size_t es = esize_of(ctx->cfg.dtype);
  const size_t ab = es * ctx->M * ctx->K, bb = es * (size_t)ctx->K * ctx->N, cb = 4ull * ctx->M * ctx->N;
  if (!ctx->h2dstream || !ctx->ownA || !ctx->ownB || !ctx->ownC || ctx->capA < ab || ctx->capB < bb ||
      ctx->capC < cb)
    return fail(ctx, APK_ESTATE, "needs a previous apk_gemm from host memory on this context");
  APK_CU(cudaSetDevice(ctx->cfg.device));
  cudaStream_t hs = ctx->h2dstream, ds = ctx->d2hstream;
  std::vector<double> t[3];
  for (int r = 0; r < reps; ++r)
    for (int m = 0; m < 3; ++m) {  // 0: A and B in, 1: C out, 2: both at once
      const long long t0 = host_now_ns();
      if (m != 1) {
        APK_CU(cudaMemcpyAsync(ctx->dA, A, ab, cudaMemcpyHostToDevice, hs));
        APK_CU(cudaMemcpyAsync(ctx->dB, B, bb, cudaMemcpyHostToDevice, hs));
      }
      if (m != 0) APK_CU(cudaMemcpyAsync(C, ctx->dC, cb, cudaMemcpyDeviceToHost, ds));
      APK_CU(cudaStreamSynchronize(hs));
      APK_CU(cudaStreamSynchronize(ds));
      t[m].push_back((double)(host_now_ns() - t0) / 1e6);
    }
  for (int m = 0; m < 3; ++m) {
    std::sort(t[m].begin(), t[m].end());
    out_ms[m] = t[m][t[m].size() / 2];
  }
  return APK_OK;
}

// ------------------------------------------------------------------ harness

apk_status apk_probe_visibility(apk_ctx* ctx, int reps, long long* offsets_ns) {
  if (!ctx || reps <= 0 || !offsets_ns) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "probe needs an idle device");
  if (ctx->cfg.set_mode == APK_SET_DEVICE) return fail(ctx, APK_EINVAL, "no host-set path in DEVICE mode");
  APK_CU(cudaSetDevice(ctx->cfg.device));
  long long* d_out = nullptr;
  APK_CU(cudaMalloc(&d_out, sizeof(long long)));
  Ctrl init{};
  for (int r = 0; r < reps; ++r) {
    APK_CU(cudaMemcpy(ctx->d_ctrl, &init, sizeof init, cudaMemcpyHostToDevice));
    *reinterpret_cast<volatile int*>(ctx->h_flag) = 0;
    std::atomic_thread_fence(std::memory_order_seq_cst);
    const int* flag = ctx->cfg.set_mode == APK_SET_HOST_MAPPED ? ctx->d_flag_mapped : &ctx->d_ctrl->flag_dev;
    spin_flag_kernel<<<1, 32, 0, ctx->kstream>>>(flag, 1, 50000000LL, d_out, &ctx->d_ctrl->status);
    spin_until_ns(host_now_ns() + 200000);  // let the spin kernel start
    long long t;
    if (ctx->cfg.set_mode == APK_SET_HOST_MAPPED) {
      t = host_now_ns();
      *reinterpret_cast<volatile int*>(ctx->h_flag) = 1;
      std::atomic_thread_fence(std::memory_order_seq_cst);
    } else {
      ctx->h_gen[1] = 1;
      t = host_now_ns();
      APK_CU(cudaMemcpyAsync(&ctx->d_ctrl->flag_dev, &ctx->h_gen[1], sizeof(int), cudaMemcpyHostToDevice,
                             ctx->cstream));
    }
    APK_CU(cudaStreamSynchronize(ctx->kstream));
    long long g = 0;
    APK_CU(cudaMemcpy(&g, d_out, sizeof g, cudaMemcpyDeviceToHost));
    offsets_ns[r] = g ? g - t : 0;
  }
  *reinterpret_cast<volatile int*>(ctx->h_flag) = 0;
  cudaFree(d_out);
  // A rep whose spin gave up (the store never became visible within the
  // bound, e.g. when a tool serialises launches) reads 0 and is skipped by
  // callers; it is not an error of the runtime.
  Ctrl cb;
  APK_CU(cudaMemcpy(&cb, ctx->d_ctrl, sizeof cb, cudaMemcpyDeviceToHost));
  if (cb.status != 0 && cb.status != DEV_WAIT_TIMEOUT_SPIN)
    return fail(ctx, APK_EDEVICE, "device reported status %d", cb.status);
  return APK_OK;
}

apk_status apk_selftest_wait_timeout(apk_ctx* ctx, long long limit_ns, int* device_status) {
  if (!ctx || limit_ns <= 0 || !device_status) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "self-test needs an idle device");
  APK_CU(cudaSetDevice(ctx->cfg.device));
  Ctrl init{};
  APK_CU(cudaMemcpy(ctx->d_uctrl, &init, sizeof init, cudaMemcpyHostToDevice));
  long long* d_out = nullptr;
  APK_CU(cudaMalloc(&d_out, sizeof(long long)));
  spin_flag_kernel<<<1, 32, 0, ctx->kstream>>>(&ctx->d_uctrl->never_set, 1, limit_ns, d_out,
                                               &ctx->d_uctrl->status);
  APK_CU(cudaGetLastError());
  APK_CU(cudaStreamSynchronize(ctx->kstream));
  cudaFree(d_out);
  Ctrl cb;
  APK_CU(cudaMemcpy(&cb, ctx->d_uctrl, sizeof cb, cudaMemcpyDeviceToHost));
  *device_status = cb.status;
  return APK_OK;
}

static double pct(std::vector<double> v, double q) {  // nearest rank, src/yield.cu:322-325
  if (v.empty()) return NAN;
  std::sort(v.begin(), v.end());
  return v[std::min((size_t)(q * v.size()), v.size() - 1)];
}

apk_status apk_run_latency(apk_ctx* ctx, const apk_latency_config* lc, apk_latency_result* out) {
  if (!ctx || !lc || !out) return APK_EINVAL;
  if (lc->events <= 0 || lc->events > ctx->cfg.max_events || lc->period_ns <= 0)
    return fail(ctx, APK_EINVAL, "events must be in [1, max_events] and period > 0");
  if (ctx->cfg.poll == APK_POLL_OFF) return fail(ctx, APK_EINVAL, "latency mode needs polling");
  memset(out, 0, sizeof *out);
  const int E = lc->events;
  std::mt19937 rng(lc->seed);
  std::uniform_real_distribution<double> u01(0.0, 1.0);
  std::vector<long long> when(E);
  if (lc->poisson) {
    // exponential gaps with mean period_ns (inverse-CDF of a uniform draw)
    double t = (double)lc->settle_ns;
    for (int e = 0; e < E; ++e) {
      t += -std::log(1.0 - u01(rng)) * (double)lc->period_ns;
      when[e] = (long long)t;
    }
  } else {
    for (int e = 0; e < E; ++e)
      when[e] = lc->settle_ns + (long long)e * lc->period_ns + (long long)(u01(rng) * lc->period_ns);
  }
  apk_status s;
  double offset = 0.0;
  const bool host_set = ctx->cfg.set_mode != APK_SET_DEVICE;
  if (host_set) {
    offset = NAN;
    if (lc->probe_reps > 0) {
      std::vector<long long> offs(lc->probe_reps);
      if ((s = apk_probe_visibility(ctx, lc->probe_reps, offs.data())) != APK_OK) return s;
      std::vector<double> o;
      for (long long v : offs)
        if (v != 0) o.push_back((double)v);
      if (!o.empty()) offset = pct(o, 0.5);
    }
    if ((s = apk_schedule_device_events(ctx, nullptr, 0)) != APK_OK) return s;
  } else {
    if ((s = apk_schedule_device_events(ctx, when.data(), E)) != APK_OK) return s;
  }
  out->vis_offset_ns = offset;
  // Bounded launches (bg_tasks > 0) end by themselves: the host injects
  // while the kernel runs and stops injecting once it has ended, so the run
  // needs no host action to terminate (safe under tools that serialise
  // launches).  Unbounded launches end with the stop sentinel.
  const bool bounded = lc->bg_tasks > 0;
  if ((s = apk_launch(ctx, bounded ? lc->bg_tasks : APK_TASKS_UNBOUNDED)) != APK_OK) return s;
  const long long t0 = host_now_ns();
  auto ended = [&]() { return bounded && cudaEventQuery(ctx->ev_done) == cudaSuccess; };
  if (host_set) {
    for (int e = 0; e < E; ++e) {
      while (host_now_ns() < t0 + when[e] && !ended()) {
      }
      if (ended()) break;
      int ev;
      long long ts;
      if ((s = apk_inject_urgent(ctx, &ev, &ts)) != APK_OK) break;
      long long seen;
      if (apk_wait_ack(ctx, ev, 0, lc->period_ns / 2, &seen) != APK_OK) continue;
      apk_wait_ack(ctx, ev, 1, lc->period_ns / 2, &seen);
    }
  } else {
    const long long until = t0 + when[E - 1] + 20000000LL;
    while (host_now_ns() < until && !ended()) {
    }
  }
  apk_status st_stop = bounded ? APK_OK : apk_stop(ctx);
  apk_status st_wait = apk_wait(ctx, 30000000000LL);
  if (s != APK_OK) return s;
  if (st_stop != APK_OK) return st_stop;
  if (st_wait != APK_OK) return st_wait;

  const int G = ctx->last_grid;
  const int Ecap = ctx->cfg.max_events;
  std::vector<long long> set(Ecap), claim(Ecap), done(Ecap), obs((size_t)Ecap * G), hs(Ecap), ha(Ecap), hd(Ecap);
  std::vector<int> claimer(Ecap);
  apk_event_log log{};
  log.set_ns = set.data();
  log.claim_ns = claim.data();
  log.done_ns = done.data();
  log.obs_ns = obs.data();
  log.claimer = claimer.data();
  log.host_set_ns = hs.data();
  log.host_ack_ns = ha.data();
  log.host_done_ns = hd.data();
  if ((s = apk_read_events(ctx, &log)) != APK_OK) return s;
  std::vector<double> lc_claim, lc_last, lc_done, rt_claim, rt_done;
  for (int e = std::max(0, lc->warmup_events); e < E; ++e) {
    double setg;
    if (host_set) {
      if (hs[e] == 0) continue;
      setg = (double)hs[e] + offset;
      if (ha[e]) rt_claim.push_back((ha[e] - hs[e]) / 1e3);
      if (hd[e]) rt_done.push_back((hd[e] - hs[e]) / 1e3);
    } else {
      if (set[e] == 0) continue;
      setg = (double)set[e];
    }
    ++out->n;
    if (claimer[e] == 0) {
      ++out->unclaimed;
      continue;
    }
    const bool have_set = !std::isnan(setg);  // host-set without calibration: NaN
    if (have_set) lc_claim.push_back((claim[e] - setg) / 1e3);
    if (have_set && done[e]) lc_done.push_back((done[e] - setg) / 1e3);
    long long hi = 0;
    int seen = 0;
    for (int b = 0; b < G; ++b) {
      const long long o = obs[(size_t)e * G + b];
      if (!o) continue;
      ++seen;
      hi = std::max(hi, o);
    }
    if (seen < G) ++out->anomalies;
    else if (have_set) lc_last.push_back((hi - setg) / 1e3);
  }
  out->claim_p50_us = pct(lc_claim, 0.5);
  out->claim_p99_us = pct(lc_claim, 0.99);
  out->last_obs_p50_us = pct(lc_last, 0.5);
  out->last_obs_p99_us = pct(lc_last, 0.99);
  out->done_p50_us = pct(lc_done, 0.5);
  out->done_p99_us = pct(lc_done, 0.99);
  out->rt_claim_p50_us = pct(rt_claim, 0.5);
  out->rt_claim_p99_us = pct(rt_claim, 0.99);
  out->rt_done_p50_us = pct(rt_done, 0.5);
  out->rt_done_p99_us = pct(rt_done, 0.99);
  apk_run_stats rs;
  if ((s = apk_read_run_stats(ctx, &rs)) != APK_OK) return s;
  out->bg_tflops = rs.bg_tflops;
  return APK_OK;
}

apk_status apk_run_overhead(apk_ctx* ctx, unsigned long long num_tasks, int reps, double* ms_poll,
                            double* ms_nopoll) {
  if (!ctx || reps <= 0 || num_tasks == 0 || num_tasks == APK_TASKS_UNBOUNDED) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "a launch is already running");
  APK_CU(cudaSetDevice(ctx->cfg.device));
  const int warm = 2;
  std::vector<double> on, off;
  for (int r = 0; r < 2 * (reps + warm); ++r) {
    // alternate which variant leads each pair (src/yield.cu:674-677)
    const bool poll = ((r / 2) % 2 == 0) ? (r % 2 == 0) : (r % 2 == 1);
    apk_status s = launch_impl(ctx, num_tasks, poll ? (int)ctx->cfg.poll : APK_POLL_OFF, ctx->kstream, true);
    if (s != APK_OK) return s;
    APK_CU(cudaEventSynchronize(ctx->ev_done));
    if ((s = read_status(ctx)) != APK_OK) return s;
    float ms = 0;
    APK_CU(cudaEventElapsedTime(&ms, ctx->ev_start, ctx->ev_done));
    if (r >= 2 * warm) (poll ? on : off).push_back(ms);
  }
  *ms_poll = pct(on, 0.5);
  *ms_nopoll = pct(off, 0.5);
  return APK_OK;
}

namespace {
apk_status run_reserved_impl(apk_ctx* ctx, unsigned long long num_tasks, int reserve, int trials, unsigned seed,
                             double* e2e_us, double* bg_tflops, bool slot_grid);
}

apk_status apk_run_reserved(apk_ctx* ctx, unsigned long long num_tasks, int reserve, int trials, unsigned seed,
                            double* e2e_us, double* bg_tflops) {
  return run_reserved_impl(ctx, num_tasks, reserve, trials, seed, e2e_us, bg_tflops, true);
}

apk_status apk_run_baseline(apk_ctx* ctx, unsigned long long num_tasks, int trials, unsigned seed,
                            double* e2e_us) {
  // the no-preemption baseline runs the context's own background kernel
  return run_reserved_impl(ctx, num_tasks, 0, trials, seed, e2e_us, nullptr, false);
}

namespace {
// slot_grid: run the block-synchronous kernel for every reserve (0
// included), whose resident CTA slots (two per SM) can be held out one at a
// time; the warp-specialized kernel's workers come two per SM-filling CTA.
apk_status run_reserved_impl(apk_ctx* ctx, unsigned long long num_tasks, int reserve, int trials, unsigned seed,
                             double* e2e_us, double* bg_tflops, bool slot_grid) {
  if (!ctx || trials <= 0 || !e2e_us || num_tasks == 0 || num_tasks == APK_TASKS_UNBOUNDED) return APK_EINVAL;
  if (reserve < 0 || reserve >= ctx->grid)
    return fail(ctx, APK_EINVAL, "reserve %d must leave at least one of the %d background CTAs", reserve, ctx->grid);
  // a CLC grid occupies every slot the hardware gives it: nothing to hold out
  if (ctx->cfg.scheduler == APK_SCHED_CLC && reserve != 0)
    return fail(ctx, APK_EINVAL, "with the CLC scheduler the urgent kernel takes SMs the hardware frees; reserve must be 0");
  if (ctx->running) return fail(ctx, APK_ESTATE, "a launch is already running");
  if (ctx->cfg.dtype != APK_F32) return fail(ctx, APK_EUNSUPPORTED, "baseline mode is fp32 only");
  if (!ctx->dAu) return fail(ctx, APK_ESTATE, "no urgent operands set");
  APK_CU(cudaSetDevice(ctx->cfg.device));
  // urgent kernel: the same tile code as a non-persistent launch over the
  // urgent GEMM's tiles on a max-priority stream (src/urgent_baseline.cu:101-112)
  F32Params up;
  memset(&up, 0, sizeof up);
  const int bk = 32;  // the urgent kernel runs the 128x128 tiles with 32-deep slots
  apk_status t;
  if ((t = make_tmap(ctx, &up.tmA, ctx->dAu, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ctx->Mu, ctx->Ku, 32, 128,
                     CU_TENSOR_MAP_SWIZZLE_128B)) != APK_OK)
    return t;
  if ((t = make_tmap(ctx, &up.tmB, ctx->dBu, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ctx->Ku, ctx->Nu, 128, bk,
                     CU_TENSOR_MAP_SWIZZLE_NONE)) != APK_OK)
    return t;
  up.tmAu = up.tmA;
  up.tmBu = up.tmB;
  const int utiles = (ctx->Mu / 128) * (ctx->Nu / 128);
  up.C = ctx->dCu + ctx->cu_slot * ctx->cfg.max_events;  // spare slot
  up.ldc = ctx->Nu;
  up.tiles_n = ctx->Nu / 128;
  up.total_tiles = utiles;
  up.nk = ctx->Ku / bk;
  up.poll_every = 1;
  up.Cu = up.C;
  up.ldcu = ctx->Nu;
  up.usplit = 1;
  up.utiles_n = up.tiles_n;
  up.wait_limit_ns = ctx->cfg.wait_limit_ns;
  up.slab = ctx->d_slab;
  up.slab_hdr = ctx->d_slab_hdr;
  Ctrl* ub = ctx->d_uctrl;
  up.ev.flag = &ub->flag_dev;
  up.ev.flag_lines = 1;
  up.ev.abort_word = &ub->abort_word;
  up.ev.status = &ub->status;
  up.ev.max_events = 0;
  up.q.next_task = &ub->next_task;
  up.q.num_tasks = (unsigned long long)utiles;
  up.q.tiles_done = ctx->d_utiles;
  up.q.start_min = &ub->start_min;
  up.q.end_max = &ub->end_max;
  up.q.exited = &ub->exited;
  up.q.yields = &ub->yields;

  // the background holds grid - reserve resident slots; the rest stay free
  // for the urgent launch (restored on every return path)
  struct GridGuard {
    apk_ctx* c;
    int keep;
    ~GridGuard() {
      c->grid = keep;
      c->sync_only = false;
    }
  } guard{ctx, ctx->grid};
  ctx->sync_only = slot_grid;
  ctx->grid -= reserve;

  // drain estimate, background alone (device timeline)
  apk_status s = launch_impl(ctx, num_tasks, APK_POLL_OFF, ctx->kstream, true);
  if (s != APK_OK) return s;
  APK_CU(cudaEventSynchronize(ctx->ev_done));
  float drain_ms = 0;
  APK_CU(cudaEventElapsedTime(&drain_ms, ctx->ev_start, ctx->ev_done));
  if (bg_tflops)
    *bg_tflops = drain_ms > 0 ? 2.0 * 128.0 * 128.0 * ctx->K * (double)num_tasks / (drain_ms * 1e-3) / 1e12 : 0.0;
  std::mt19937 rng(seed);
  std::uniform_real_distribution<double> frac(0.2, 0.8);
  Ctrl init{};
  init.start_min = ~0ull;
  for (int tr = 0; tr < trials; ++tr) {
    APK_CU(cudaMemcpy(ub, &init, sizeof init, cudaMemcpyHostToDevice));
    APK_CU(cudaDeviceSynchronize());
    const double delay_ns = frac(rng) * drain_ms * 1e6;
    if ((s = launch_impl(ctx, num_tasks, APK_POLL_OFF, ctx->kstream, true)) != APK_OK) return s;
    const long long t0 = host_now_ns();
    spin_until_ns(t0 + (long long)delay_ns);
    const long long ta = host_now_ns();
    cudaError_t e = f32::launch(up, utiles, APK_POLL_OFF, APK_DISC_DRAIN, false, F32_GEO_L32, APK_SCHED_QUEUE,
                                ctx->ustream);
    if (e != cudaSuccess) return fail(ctx, APK_ECUDA, "urgent launch failed: %s", cudaGetErrorString(e));
    APK_CU(cudaStreamSynchronize(ctx->ustream));
    const long long td = host_now_ns();
    APK_CU(cudaStreamSynchronize(ctx->kstream));
    e2e_us[tr] = (td - ta) / 1e3;
  }
  return read_status(ctx);
}

}  // namespace

apk_status apk_run_visibility(apk_ctx* ctx, const apk_visibility_config* vc, apk_visibility_result* out,
                              long long* set_out, long long* obs_out) {
  if (!ctx || !vc || !out) return APK_EINVAL;
  if (ctx->running) return fail(ctx, APK_ESTATE, "a launch is already running");
  if (vc->events <= 0 || vc->gap_min_ns <= 0 || vc->gap_max_ns < vc->gap_min_ns || vc->work_iters < 0 ||
      vc->warmup_events < 0 || vc->traffic_bytes < 0)
    return fail(ctx, APK_EINVAL, "visibility: events > 0, 0 < gap_min <= gap_max, work_iters >= 0");
  APK_CU(cudaSetDevice(ctx->cfg.device));
  memset(out, 0, sizeof *out);
  const int E = vc->events, G = ctx->grid, NT = vis::threads();
  const unsigned long long stride = (unsigned long long)G * NT;
  unsigned long long n4 = (unsigned long long)(vc->traffic_bytes ? vc->traffic_bytes : (1ll << 30)) / 16;
  const unsigned long long min_n4 = 2ull * vis::loads_per_iter() * stride;
  if (n4 < min_n4) n4 = min_n4;
  // the studied kernel's shared memory per CTA keeps the residency the same
  const int smem = std::max(4 * NT, ctx->cfg.dtype == APK_F32 ? f32::geo_info(ctx->f32_geo).smem_bytes
                                                               : bf16::geo_info(ctx->bf16_geo).smem_bytes);
  std::mt19937 rng(vc->seed);
  std::uniform_real_distribution<double> gap((double)vc->gap_min_ns, (double)vc->gap_max_ns);
  std::vector<long long> sched(E);
  long long acc = 0;
  for (int e = 0; e < E; ++e) sched[e] = (acc += (long long)gap(rng));

  struct Bufs {
    void* p[10] = {};
    ~Bufs() {
      for (void* q : p)
        if (q) cudaFree(q);
    }
  } b;
  int *d_flag, *d_status;
  long long *d_sched, *d_set, *d_obs, *d_iters, *d_t0, *d_t1;
  float* d_sink;
  float4* d_traffic = nullptr;
  APK_CU(cudaMalloc(&d_flag, sizeof(int)));
  b.p[0] = d_flag;
  APK_CU(cudaMalloc(&d_status, sizeof(int)));
  b.p[1] = d_status;
  APK_CU(cudaMalloc(&d_sched, sizeof(long long) * E));
  b.p[2] = d_sched;
  APK_CU(cudaMalloc(&d_set, sizeof(long long) * E));
  b.p[3] = d_set;
  APK_CU(cudaMalloc(&d_obs, sizeof(long long) * (size_t)E * G));
  b.p[4] = d_obs;
  APK_CU(cudaMalloc(&d_iters, sizeof(long long) * G));
  b.p[5] = d_iters;
  APK_CU(cudaMalloc(&d_t0, sizeof(long long) * G));
  b.p[6] = d_t0;
  APK_CU(cudaMalloc(&d_t1, sizeof(long long) * G));
  b.p[7] = d_t1;
  APK_CU(cudaMalloc(&d_sink, sizeof(float) * stride));
  b.p[8] = d_sink;
  if (vc->loaded) {
    APK_CU(cudaMalloc(&d_traffic, 16 * n4));
    b.p[9] = d_traffic;
    APK_CU(cudaMemset(d_traffic, 0, 16 * n4));
  }
  APK_CU(cudaMemset(d_flag, 0, sizeof(int)));
  APK_CU(cudaMemset(d_status, 0, sizeof(int)));
  APK_CU(cudaMemset(d_set, 0, sizeof(long long) * E));
  APK_CU(cudaMemset(d_obs, 0, sizeof(long long) * (size_t)E * G));
  APK_CU(cudaMemcpy(d_sched, sched.data(), sizeof(long long) * E, cudaMemcpyHostToDevice));
  APK_CU(cudaDeviceSynchronize());

  VisParams p;
  memset(&p, 0, sizeof p);
  p.flag = d_flag;
  p.sched_ns = d_sched;
  p.n_events = E;
  p.set_ns = d_set;
  p.obs_ns = d_obs;
  p.iters = d_iters;
  p.t_begin = d_t0;
  p.t_end = d_t1;
  p.work_iters = vc->work_iters;
  p.traffic = d_traffic;
  p.traffic_n4 = n4;
  p.sink = d_sink;
  p.tail_ns = 2000000;  // 2 ms after the last raise, as src/yield.cu:262-264
  p.limit_ns = sched[E - 1] + p.tail_ns + 2000000000LL;
  p.status = d_status;
  cudaError_t e = vis::launch(p, G, smem, vc->loaded != 0, ctx->kstream);
  if (e != cudaSuccess) return fail(ctx, APK_ECUDA, "visibility launch failed: %s", cudaGetErrorString(e));
  APK_CU(cudaStreamSynchronize(ctx->kstream));

  std::vector<long long> set(E), obs((size_t)E * G), iters(G), t0(G), t1(G);
  int status = 0;
  APK_CU(cudaMemcpy(set.data(), d_set, sizeof(long long) * E, cudaMemcpyDeviceToHost));
  APK_CU(cudaMemcpy(obs.data(), d_obs, sizeof(long long) * (size_t)E * G, cudaMemcpyDeviceToHost));
  APK_CU(cudaMemcpy(iters.data(), d_iters, sizeof(long long) * G, cudaMemcpyDeviceToHost));
  APK_CU(cudaMemcpy(t0.data(), d_t0, sizeof(long long) * G, cudaMemcpyDeviceToHost));
  APK_CU(cudaMemcpy(t1.data(), d_t1, sizeof(long long) * G, cudaMemcpyDeviceToHost));
  APK_CU(cudaMemcpy(&status, d_status, sizeof(int), cudaMemcpyDeviceToHost));
  if (set_out) memcpy(set_out, set.data(), sizeof(long long) * E);
  if (obs_out) memcpy(obs_out, obs.data(), sizeof(long long) * (size_t)E * G);

  std::vector<double> dmin, d50, d95, dmax, cad;
  for (int e2 = 0; e2 < E; ++e2) {
    if (set[e2] == 0) {
      ++out->unset;
      continue;
    }
    std::vector<double> d;
    bool complete = true;
    for (int c = 1; c < G; ++c) {  // CTA 0 raised the flag itself
      const long long o = obs[(size_t)e2 * G + c];
      if (o == 0) {
        complete = false;
        break;
      }
      d.push_back((o - set[e2]) / 1e3);
    }
    if (!complete || d.empty()) {
      ++out->anomalies;
      continue;
    }
    if (e2 < vc->warmup_events) continue;
    std::sort(d.begin(), d.end());
    dmin.push_back(d.front());
    d50.push_back(pct(d, 0.5));
    d95.push_back(pct(d, 0.95));
    dmax.push_back(d.back());
  }
  long long tmin = t0[0], tmax = t1[0], total_iters = 0;
  for (int c = 0; c < G; ++c) {
    if (iters[c] > 0) cad.push_back((double)(t1[c] - t0[c]) / (double)iters[c]);
    tmin = std::min(tmin, t0[c]);
    tmax = std::max(tmax, t1[c]);
    total_iters += iters[c];
  }
  out->n = (int)dmax.size();
  out->cadence_ns = cad.empty() ? 0.0 : pct(cad, 0.5);
  out->dmin_p50_us = pct(dmin, 0.5);
  out->d50_p50_us = pct(d50, 0.5);
  out->d95_p50_us = pct(d95, 0.5);
  out->dmax_p50_us = pct(dmax, 0.5);
  out->dmax_p99_us = pct(dmax, 0.99);
  if (vc->loaded && tmax > tmin)
    out->hbm_gbs = (double)total_iters * NT * vis::loads_per_iter() * 16.0 / (double)(tmax - tmin);
  out->device_status = status;
  if (status != 0) return fail(ctx, APK_EDEVICE, "visibility probe: a CTA reached its time limit (status %d)", status);
  return APK_OK;
}

void* apk_host_alloc(size_t bytes) {
  void* p = nullptr;
  if (cudaHostAlloc(&p, bytes, cudaHostAllocPortable) != cudaSuccess) return nullptr;
  return p;
}

void apk_host_free(void* p) {
  if (p) cudaFreeHost(p);
}

}  // extern "C"
