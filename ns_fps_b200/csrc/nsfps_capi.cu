// nsfps_capi.cu -- host side of the engine: the C ABI declared in
// include/nsfps.h, SpaceRange arithmetic, per-device workspaces and streams,
// and the orchestration of setup -> plan -> sampling loop -> epilogue.
//
// SpaceRange arithmetic restates make_range / make_uniform_range /
// compute_bbox of the reference (src/yuezu_fps.cpp:7-161, :643-670) in
// host float arithmetic (SSE, round-to-nearest, no contraction: this file is
// compiled with -fmad=false and the host compiler's default
// -ffp-contract=off for ISO C++ is forced by -Xcompiler -ffp-contract=off).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "nsfps.h"
#include "nsfps_internal.cuh"
#include "nsfps_kernels.h"

namespace nsfps {

// ------------------------------------------------------------------ errors
namespace {
thread_local std::string g_err;
thread_local nsfps_profile g_prof;
std::atomic<int> g_profiling{0};
// NSFPS_STEP_LOOP=1 in the environment selects the per-step loop even for
// direct ranges (both loops return identical samples).
std::atomic<int> g_force_steps{-1};
// nsfps_set_test_hooks: wait limit, withheld list / proposal, failed
// workspace request
constexpr long long kDefaultWaitNs = 2000000000ll;
std::atomic<long long> g_wait_ns{kDefaultWaitNs};
std::atomic<int> g_hold_cta{-1};
std::atomic<uint32_t> g_hold_step{0};
std::atomic<int> g_fail_alloc{-1};
}  // namespace

int set_error(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

void clear_error() { g_err.clear(); }

#define NSFPS_CUDA(call)                                                      \
  do {                                                                        \
    cudaError_t e_ = (call);                                                  \
    if (e_ != cudaSuccess)                                                    \
      return set_error(e_ == cudaErrorMemoryAllocation ? NSFPS_ERR_OOM        \
                                                       : NSFPS_ERR_CUDA,     \
                       "%s failed: %s", #call, cudaGetErrorString(e_));      \
  } while (0)

// ------------------------------------------------------------- SpaceRange
namespace {

// src/yuezu_fps.cpp:45-50
uint32_t calc_bits(uint32_t blocks) {
  uint32_t bits = 0;
  while (bits < 32 && (1u << bits) < blocks) ++bits;
  return bits ? bits : 1;
}

// src/yuezu_fps.cpp:69-97: x->y->z over the common bits, then the remaining
// bits of x, y, z in that order.
void bit_positions(const uint32_t bits[3], uint8_t pos[3][kMaxAxisBits]) {
  uint32_t bit = 0, np[3] = {0, 0, 0};
  const uint32_t common = std::min({bits[0], bits[1], bits[2]});
  const uint32_t maxb = std::max({bits[0], bits[1], bits[2]});
  for (uint32_t i = 0; i < common; ++i)
    for (int a = 0; a < 3; ++a) pos[a][np[a]++] = (uint8_t)bit++;
  for (uint32_t i = common; i < maxb; ++i)
    for (int a = 0; a < 3; ++a)
      if (i < bits[a]) pos[a][np[a]++] = (uint8_t)bit++;
}

uint32_t spread(uint32_t v, uint32_t bits, const uint8_t *pos) {
  uint32_t code = 0;
  for (uint32_t k = 0; k < bits; ++k)
    if (v & (1u << k)) code |= 1u << pos[k];
  return code;
}

int check_range(const nsfps_range &r) {
  const uint32_t b[3] = {r.x_blocks, r.y_blocks, r.z_blocks};
  for (int a = 0; a < 3; ++a) {
    if (b[a] == 0)
      return set_error(NSFPS_ERR_ARG, "SpaceRange block counts must be >= 1 (got %u x %u x %u)",
                       r.x_blocks, r.y_blocks, r.z_blocks);
    if (b[a] > NSFPS_MAX_BLOCKS_PER_AXIS)
      return set_error(NSFPS_ERR_UNSUPPORTED,
                       "SpaceRange block count %u exceeds this engine's limit of %u per axis",
                       b[a], NSFPS_MAX_BLOCKS_PER_AXIS);
  }
  return NSFPS_OK;
}

}  // namespace

int range_to_dev(const nsfps_range &r, RangeDev *out, const char **why) {
  (void)why;
  int rc = check_range(r);
  if (rc) return rc;
  std::memset(out, 0, sizeof(*out));
  const float mn[3] = {r.min_x, r.min_y, r.min_z};
  const float mx[3] = {r.max_x, r.max_y, r.max_z};
  const uint32_t b[3] = {r.x_blocks, r.y_blocks, r.z_blocks};
  for (int a = 0; a < 3; ++a) {
    volatile float span = mx[a] - mn[a];
    volatile float bs = span / (float)b[a];
    out->mn[a] = mn[a];
    out->hi[a] = mx[a] - NSFPS_BOUNDARY_EPS;
    out->inv_bs[a] = 1.0f / bs;
    out->bsz[a] = bs;  // block_size_*() = (max - min) / blocks
    out->blocks[a] = b[a];
    out->bits[a] = calc_bits(b[a]);
  }
  out->total = b[0] * b[1] * b[2];
  out->total_bits = out->bits[0] + out->bits[1] + out->bits[2];
  uint8_t pos[3][kMaxAxisBits] = {};
  bit_positions(out->bits, pos);
  std::memcpy(out->pos, pos, sizeof(pos));
  const uint32_t maxcode = spread(b[0] - 1, out->bits[0], pos[0]) |
                           spread(b[1] - 1, out->bits[1], pos[1]) |
                           spread(b[2] - 1, out->bits[2], pos[2]);
  out->direct = maxcode < out->total ? 1u : 0u;
  return NSFPS_OK;
}

// The ratio whose ceiling is the reference's cube half-width
// (src/yuezu_fps.cpp:566-570): std::sqrt on a float, then a float division,
// both correctly rounded on the host (sqrtss / divss).
static inline float cube_ratio(float D, float bs) { return std::sqrt(D) / bs; }

// Largest finite float D >= 0 for which `pred` holds, for a predicate that is
// true at 0 and monotone (true, then false) in D.
template <class F>
static float max_true(F pred) {
  uint32_t lo = 0, hi = 0x7f7fffffu;  // bit patterns of 0 and FLT_MAX
  float f;
  std::memcpy(&f, &hi, 4);
  if (pred(f)) return f;
  while (hi - lo > 1) {  // pred(lo) true, pred(hi) false
    const uint32_t mid = lo + (hi - lo) / 2;
    std::memcpy(&f, &mid, 4);
    if (pred(f)) lo = mid; else hi = mid;
  }
  std::memcpy(&f, &lo, 4);
  return f;
}

// For a positive finite block size the cube half-width is monotone in the
// distance D, so it can be read from thresholds instead of being recomputed:
// table a holds, for n = 0 .. blocks-2, the largest D with
// ceil(sqrt(D) / bs) <= n (a half-width of blocks-1 or more covers the whole
// axis), and ovf[a] the largest D whose ratio still converts to int.  The
// device then needs no IEEE division or square root per iteration.
void cube_thresholds(RangeDev &r, std::vector<float> &pool) {
  r.fast_cube = 1;
  for (int a = 0; a < 3; ++a)
    if (!(r.bsz[a] > 0.0f) || !std::isfinite(r.bsz[a])) r.fast_cube = 0;
  if (!r.fast_cube) return;
  for (int a = 0; a < 3; ++a) {
    const float bs = r.bsz[a];
    r.tab_off[a] = (uint32_t)pool.size();
    for (uint32_t n = 0; n + 1 < r.blocks[a]; ++n)
      pool.push_back(max_true([&](float D) { return cube_ratio(D, bs) <= (float)n; }));
    r.ovf[a] = max_true([&](float D) { return cube_ratio(D, bs) < 2147483648.0f; });
  }
}

int range_info(const nsfps_range &r, nsfps_range_info *info) {
  RangeDev d;
  int rc = range_to_dev(r, &d, nullptr);
  if (rc) return rc;
  for (int a = 0; a < 3; ++a) {
    info->inv_bs[a] = d.inv_bs[a];
    info->block_size[a] = d.bsz[a];
    info->bits[a] = d.bits[a];
  }
  info->total_bits = d.total_bits;
  info->total_blocks = (uint64_t)r.x_blocks * r.y_blocks * r.z_blocks;
  return NSFPS_OK;
}

// ------------------------------------------------------- device contexts
namespace {

// The setup pipeline of one call shape (its SetupArgs: sizes and workspace
// pointers), captured once as a CUDA graph and replayed by later calls of
// the same shape: one launch instead of ~25 small ones.
struct SetupGraph {
  SetupArgs args;
  cudaGraphExec_t exec = nullptr;
  uint32_t launches = 0;
  uint64_t used = 0;
};
constexpr size_t kSetupGraphs = 8;

struct DeviceCtx {
  std::mutex mu;
  int device = -1;
  cudaStream_t stream = nullptr;
  cudaStream_t capture = nullptr;  // private stream the setup graphs are captured on
  void *ws = nullptr;
  size_t ws_bytes = 0;
  cudaEvent_t ev[4] = {};
  bool ready = false;
  bool fixed = false;  // the workspace is the static scratch array: never (re)allocated
  bool small_ready = false;  // small_setup_prepare ran on this device
  std::vector<SetupGraph> graphs;
  uint64_t graph_clock = 0;
  // host staging of a call's small uploads and downloads: pinned (one
  // asynchronous copy each way), or a plain vector for the static context,
  // which allocates nothing on the device side
  void *pin = nullptr;
  size_t pin_bytes = 0;
  std::vector<unsigned char> pageable;
};

// Host staging area of at least `bytes` for ctx (pinned unless the context is
// the static one); nullptr when it cannot be had.
unsigned char *staging(DeviceCtx *ctx, size_t bytes) {
  if (ctx->fixed) {
    if (ctx->pageable.size() < bytes) ctx->pageable.resize(bytes);
    return ctx->pageable.data();
  }
  if (ctx->pin_bytes < bytes) {
    if (ctx->pin) {
      cudaStreamSynchronize(ctx->stream);
      cudaFreeHost(ctx->pin);
      ctx->pin = nullptr;
      ctx->pin_bytes = 0;
    }
    const size_t want = std::max<size_t>(bytes + bytes / 2, 64 << 10);
    if (cudaMallocHost(&ctx->pin, want) != cudaSuccess) {
      cudaGetLastError();
      ctx->pin = nullptr;
      return nullptr;
    }
    ctx->pin_bytes = want;
  }
  return (unsigned char *)ctx->pin;
}

void drop_setup_graphs(DeviceCtx *ctx) {
  for (SetupGraph &g : ctx->graphs)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  ctx->graphs.clear();
}

// Runs the setup pipeline on `st`, from a cached graph of this shape when
// there is one (captured now when there is not).  The static context never
// captures: instantiating a graph may allocate.
cudaError_t run_setup_cached(DeviceCtx *ctx, const SetupArgs &sa, cudaStream_t st,
                             uint32_t &launches) {
  if (sa.small_rounds && !ctx->small_ready) {
    const cudaError_t e = small_setup_prepare();
    if (e != cudaSuccess) return e;
    ctx->small_ready = true;
  }
  if (ctx->fixed) return run_setup(sa, st, launches);
  SetupGraph *hit = nullptr;
  for (SetupGraph &g : ctx->graphs)
    if (std::memcmp(&g.args, &sa, sizeof(SetupArgs)) == 0) hit = &g;
  if (!hit) {
    cudaError_t e = cudaSuccess;
    if (!ctx->capture) e = cudaStreamCreateWithFlags(&ctx->capture, cudaStreamNonBlocking);
    cudaGraph_t graph = nullptr;
    uint32_t l = 0;
    if (e == cudaSuccess) e = cudaStreamBeginCapture(ctx->capture, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
      const cudaError_t er = run_setup(sa, ctx->capture, l);
      e = cudaStreamEndCapture(ctx->capture, &graph);
      if (e == cudaSuccess) e = er;
    }
    cudaGraphExec_t exec = nullptr;
    if (e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
    if (graph) cudaGraphDestroy(graph);
    if (e != cudaSuccess) {  // no graph: launch the pipeline directly
      cudaGetLastError();
      return run_setup(sa, st, launches);
    }
    if (ctx->graphs.size() >= kSetupGraphs) {  // evict the least recently used
      size_t old = 0;
      for (size_t i = 1; i < ctx->graphs.size(); ++i)
        if (ctx->graphs[i].used < ctx->graphs[old].used) old = i;
      cudaGraphExecDestroy(ctx->graphs[old].exec);
      ctx->graphs.erase(ctx->graphs.begin() + (long)old);
    }
    SetupGraph g;
    g.args = sa;
    g.exec = exec;
    g.launches = l;
    ctx->graphs.push_back(g);
    hit = &ctx->graphs.back();
  }
  hit->used = ++ctx->graph_clock;
  launches += hit->launches;
  return cudaGraphLaunch(hit->exec, st);
}

constexpr int kMaxDevices = 64;
DeviceCtx g_ctx[kMaxDevices];
std::mutex g_ctx_mu;

void read_env_once() {
  int expected = -1;
  const char *v = std::getenv("NSFPS_STEP_LOOP");
  g_force_steps.compare_exchange_strong(expected, (v && v[0] == '1') ? 1 : 0);
}

int get_ctx(int device, DeviceCtx **out) {
  read_env_once();
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0)
    return set_error(NSFPS_ERR_CUDA, "no CUDA device available (%s)",
                     e == cudaSuccess ? "0 devices" : cudaGetErrorString(e));
  if (device < 0 || device >= count || device >= kMaxDevices)
    return set_error(NSFPS_ERR_ARG, "device %d out of range (0..%d)", device, count - 1);
  DeviceCtx *c = &g_ctx[device];
  std::lock_guard<std::mutex> lk(g_ctx_mu);
  if (!c->ready) {
    NSFPS_CUDA(cudaSetDevice(device));
    NSFPS_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    for (auto &ev : c->ev) NSFPS_CUDA(cudaEventCreate(&ev));
    c->device = device;
    c->ready = true;
  }
  *out = c;
  return NSFPS_OK;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Carves typed sub-buffers out of one allocation.
struct Carver {
  char *base;
  size_t off = 0;
  explicit Carver(void *b) : base((char *)b) {}
  template <class T>
  T *take(size_t count) {
    off = align_up(off, 256);
    T *p = (T *)(base ? base + off : nullptr);
    off += sizeof(T) * std::max<size_t>(count, 1);
    return p;
  }
};

// One GPU job: clouds packed back to back.
struct Job {
  uint32_t n = 0;                 // total points
  uint32_t B = 0;                 // clouds
  uint32_t k = 0;
  std::vector<uint32_t> poff;     // B + 1
  std::vector<uint32_t> rid;      // B
  std::vector<uint32_t> boff;     // B
  std::vector<RangeDev> ranges;
  std::vector<float> tabs;        // cube half-width thresholds of all ranges
  uint64_t total_buckets = 0;
  bool any_hashed = false;
};

struct Buffers {
  unsigned char *params;  // poff | rid | boff | ranges | tabs | cand, uploaded as one copy
  unsigned char *ctrl;    // scalars | stats | plan | out_count, downloaded as one copy
  float *xyz;
  uint32_t *keys0, *vals0, *keys1, *vals1, *hist, *partial, *perm, *tmp0, *tmp1;
  float4 *pts, *leaf_lo, *leaf_hi;
  float *leaf_md;
  uint32_t *leaf_start, *leaf_pre, *loff, *poff, *rid, *boff, *scalars, *plan, *cand;
  RangeDev *ranges;
  float *tabs;
  uint32_t *out_rank, *out_count;
  uint64_t *out;
  unsigned long long *stats;
  uint4 *glist;
  uint32_t *gbar;
};

// CTAs per cloud the setup plans for: cluster sizes (one thread-block
// cluster per cloud) first, then for one cloud the grid-wide sizes (one cloud
// over co-resident CTAs), for a batch the other sizes of CTA groups
// (groups of co-resident CTAs, each sampling its share of the clouds).
constexpr uint32_t kSingleCand[] = {1, 2, 4, 8, 16, 32, 64, 128};
constexpr uint32_t kBatchCand[] = {1, 2, 4, 8, 16, 6, 10, 12, 14};
constexpr int kNumSingle = 8, kNumBatch = 9;
static_assert(kNumSingle <= kMaxCand && kNumBatch <= kMaxCand, "plan capacity");
constexpr int kNumCluster = 5;
constexpr uint32_t kMaxGridP = 128;
// CTAs a grid-wide launch may hold (list buffers and counters are sized for it)
constexpr uint32_t kMaxGridCtas = 256;
// CTAs of the grid-wide loop of a small single cloud launched without a plan
// round trip (run_job)
constexpr uint32_t kDirectP = 64;
// Points from which one cloud runs on the grid-wide loop even when it fits a
// cluster.
constexpr uint32_t kGridMinPoints = NSFPS_GRID_MIN_POINTS;

// Byte offsets of a job's small per-call inputs inside the params block, and
// of the counters and results inside the control block.
struct ParamLayout {
  size_t poff, rid, boff, ranges, tabs, cand, bytes;
};
ParamLayout param_layout(const Job &j) {
  ParamLayout L{};
  size_t o = 0;
  auto put = [&](size_t sz) {
    const size_t at = o;
    o = align_up(o + std::max<size_t>(sz, 1), 16);
    return at;
  };
  L.poff = put(4 * ((size_t)j.B + 1));
  L.rid = put(4 * (size_t)j.B);
  L.boff = put(4 * (size_t)j.B);
  L.ranges = put(sizeof(RangeDev) * j.ranges.size());
  L.tabs = put(sizeof(float) * j.tabs.size());
  L.cand = put(4 * (size_t)kMaxCand);
  L.bytes = o;
  return L;
}
constexpr size_t kCtrlScalars = 0;                                   // kScalarCount uint32
constexpr size_t kCtrlStats = 32;                                    // 4 x uint64
constexpr size_t kCtrlPlan = 64;                                     // 3 * kMaxCand uint32
constexpr size_t kCtrlCount = kCtrlPlan + 4 * 3 * kMaxCand;          // B uint32
static_assert(4 * kScalarCount <= kCtrlStats, "control block layout");
size_t ctrl_bytes(const Job &j) { return kCtrlCount + 4 * (size_t)j.B; }

size_t carve(Carver &c, const Job &j, bool own_xyz, bool own_out, Buffers &b) {
  const size_t n = j.n;
  const size_t tiles = radix_tiles(j.n);
  const size_t scan_len = std::max(n, 256 * tiles);
  b.xyz = own_xyz ? c.take<float>(3 * n) : nullptr;
  b.keys0 = c.take<uint32_t>(n);
  b.vals0 = c.take<uint32_t>(n);
  b.keys1 = c.take<uint32_t>(n);
  b.vals1 = c.take<uint32_t>(n);
  b.hist = c.take<uint32_t>(256 * tiles + 1);
  b.partial = c.take<uint32_t>((scan_len + 4095) / 4096 + 2);
  b.pts = c.take<float4>(n);
  b.perm = c.take<uint32_t>(n);
  b.tmp0 = c.take<uint32_t>(n);
  b.tmp1 = c.take<uint32_t>(n);
  b.leaf_start = c.take<uint32_t>(n + 1);
  b.leaf_lo = c.take<float4>(n);
  b.leaf_hi = c.take<float4>(n);
  b.leaf_md = c.take<float>(n);
  b.leaf_pre = j.any_hashed ? c.take<uint32_t>(n * kMaxPreimages) : nullptr;
  b.loff = c.take<uint32_t>(j.B + 1);
  const ParamLayout L = param_layout(j);
  b.params = c.take<unsigned char>(L.bytes);
  b.poff = (uint32_t *)(b.params ? b.params + L.poff : nullptr);
  b.rid = (uint32_t *)(b.params ? b.params + L.rid : nullptr);
  b.boff = (uint32_t *)(b.params ? b.params + L.boff : nullptr);
  b.ranges = (RangeDev *)(b.params ? b.params + L.ranges : nullptr);
  b.tabs = (float *)(b.params ? b.params + L.tabs : nullptr);
  b.cand = (uint32_t *)(b.params ? b.params + L.cand : nullptr);
  b.ctrl = c.take<unsigned char>(ctrl_bytes(j));
  b.scalars = (uint32_t *)(b.ctrl ? b.ctrl + kCtrlScalars : nullptr);
  b.stats = (unsigned long long *)(b.ctrl ? b.ctrl + kCtrlStats : nullptr);
  b.plan = (uint32_t *)(b.ctrl ? b.ctrl + kCtrlPlan : nullptr);
  b.out_count = (uint32_t *)(b.ctrl ? b.ctrl + kCtrlCount : nullptr);
  b.out_rank = c.take<uint32_t>((size_t)j.B * j.k);
  b.out = own_out ? c.take<uint64_t>((size_t)j.B * j.k) : nullptr;
  // grid-wide lists and counters: one cloud over 64 or 128 CTAs, or groups of
  // at most 16 CTAs over at most kMaxGridCtas
  const size_t glist_bytes =
      j.B == 1 ? std::max(rounds_grid_list_bytes(64, 1), rounds_grid_list_bytes(128, 1))
               : rounds_group_list_bytes(kMaxGridCtas);
  b.glist = c.take<uint4>(glist_bytes / 16);
  b.gbar = c.take<uint32_t>(kMaxGridCtas);
  return align_up(c.off, 256);
}

int ensure_ws(DeviceCtx *ctx, size_t bytes) {
  if (!ctx->fixed) {
    int want = ctx->device;
    if (g_fail_alloc.load() == want && g_fail_alloc.compare_exchange_strong(want, -1))
      return set_error(NSFPS_ERR_OOM,
                       "workspace allocation on device %d failed (injected by "
                       "nsfps_set_test_hooks)", ctx->device);
  }
  if (ctx->ws_bytes >= bytes) return NSFPS_OK;
  if (ctx->fixed)
    return set_error(NSFPS_ERR_UNSUPPORTED, "needs %zu bytes of scratch, the fixed array holds %zu",
                     bytes, ctx->ws_bytes);
  if (ctx->ws) {
    cudaStreamSynchronize(ctx->stream);
    drop_setup_graphs(ctx);  // they point into the old workspace
    cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
  }
  const size_t want = align_up(bytes + bytes / 4, 1 << 20);
  cudaError_t e = cudaMalloc(&ctx->ws, want);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(NSFPS_ERR_OOM, "cudaMalloc of %zu bytes failed: %s", want,
                     cudaGetErrorString(e));
  }
  ctx->ws_bytes = want;
  return NSFPS_OK;
}

// The derived range and its cube threshold tables, cached per range: the
// tables take one bisection over float bit patterns per block boundary
// (15-50 us per call on the bench configs), and callers repeat their ranges.
struct RangeCacheEntry {
  nsfps_range key;
  RangeDev dev;               // tab_off relative to `tabs`
  std::vector<float> tabs;
  uint64_t used = 0;
};
constexpr size_t kRangeCache = 32;
std::mutex g_range_mu;
std::vector<RangeCacheEntry> g_range_cache;
uint64_t g_range_clock = 0;

// range_to_dev + cube_thresholds of r, appending its tables to `pool`.
int range_with_tables(const nsfps_range &r, RangeDev &out, std::vector<float> &pool) {
  {
    std::lock_guard<std::mutex> lk(g_range_mu);
    for (RangeCacheEntry &e : g_range_cache)
      if (std::memcmp(&e.key, &r, sizeof(nsfps_range)) == 0) {
        e.used = ++g_range_clock;
        out = e.dev;
        const uint32_t base = (uint32_t)pool.size();
        for (int a = 0; a < 3; ++a) out.tab_off[a] += base;
        pool.insert(pool.end(), e.tabs.begin(), e.tabs.end());
        return NSFPS_OK;
      }
  }
  RangeCacheEntry e;
  e.key = r;
  int rc = range_to_dev(r, &e.dev, nullptr);
  if (rc) return rc;
  cube_thresholds(e.dev, e.tabs);  // tab_off relative to e.tabs
  out = e.dev;
  const uint32_t base = (uint32_t)pool.size();
  for (int a = 0; a < 3; ++a) out.tab_off[a] += base;
  pool.insert(pool.end(), e.tabs.begin(), e.tabs.end());
  std::lock_guard<std::mutex> lk(g_range_mu);
  if (g_range_cache.size() >= kRangeCache) {  // evict the least recently used
    size_t old = 0;
    for (size_t i = 1; i < g_range_cache.size(); ++i)
      if (g_range_cache[i].used < g_range_cache[old].used) old = i;
    g_range_cache.erase(g_range_cache.begin() + (long)old);
  }
  e.used = ++g_range_clock;
  g_range_cache.push_back(std::move(e));
  return NSFPS_OK;
}

// Build a job from `count` clouds with point counts n[i]; ranges resolved.
int build_job(const uint64_t *n, uint64_t count, uint64_t k,
              const std::vector<nsfps_range> &ranges, const std::vector<uint32_t> &rid,
              Job &j) {
  uint64_t tot = 0;
  j.B = (uint32_t)count;
  j.k = (uint32_t)k;
  j.poff.assign(count + 1, 0);
  for (uint64_t i = 0; i < count; ++i) {
    j.poff[i] = (uint32_t)tot;
    tot += n[i];
  }
  if (tot >= (1ull << 31))
    return set_error(NSFPS_ERR_UNSUPPORTED, "too many points in one call (%llu >= 2^31)",
                     (unsigned long long)tot);
  if (k >= (1ull << 31))
    return set_error(NSFPS_ERR_UNSUPPORTED, "sample_count too large");
  j.poff[count] = (uint32_t)tot;
  j.n = (uint32_t)tot;
  j.ranges.resize(ranges.size());
  for (size_t r = 0; r < ranges.size(); ++r) {
    int rc = range_with_tables(ranges[r], j.ranges[r], j.tabs);
    if (rc) return rc;
    if (!j.ranges[r].direct) j.any_hashed = true;
  }
  if (j.tabs.empty()) j.tabs.push_back(0.0f);
  j.rid = rid;
  j.boff.assign(count, 0);
  uint64_t b = 0;
  for (uint64_t i = 0; i < count; ++i) {
    j.boff[i] = (uint32_t)b;
    b += j.ranges[rid[i]].total;
    if (b > 0xffffffffull)
      return set_error(NSFPS_ERR_UNSUPPORTED,
                       "total number of buckets over the batch exceeds 2^32");
  }
  j.total_buckets = b;
  return NSFPS_OK;
}

// The fused setup of small clouds (one CTA per cloud, two launches) when
// every cloud has 1 .. kSmallCloudMax points, every range at most
// kSmallMaxBuckets buckets, the candidate CTA counts sum to at most 512 and
// the batch fills at most two waves of CTAs; its sort's register rounds, else
// 0.
// NSFPS_SMALL_SETUP=0 keeps the multi-launch pipeline.
int small_setup(const Job &j, const uint32_t *cand, int ncand) {
  static const bool off = [] {
    const char *v = std::getenv("NSFPS_SMALL_SETUP");
    return v && v[0] == '0';
  }();
  if (off || j.B == 0 || j.B > 296) return 0;
  uint32_t mx = 0;
  for (uint32_t c = 0; c < j.B; ++c) {
    const uint32_t nc = j.poff[c + 1] - j.poff[c];
    if (nc == 0) return 0;
    mx = std::max(mx, nc);
  }
  if (mx > kSmallCloudMax) return 0;
  for (const RangeDev &r : j.ranges)
    if (r.total > kSmallMaxBuckets) return 0;
  uint32_t sum = 0;  // the plan's per-CTA sums: at most 512 entries
  for (int i = 0; i < ncand; ++i) sum += cand[i];
  if (sum > 512u) return 0;
  return small_setup_rounds(mx);
}

// Runs the whole pipeline for a job whose points are at d_xyz (device).
// Writes B*k uint64 results to d_out and the B lengths to lens (host).
int run_job(DeviceCtx *ctx, cudaStream_t st, const Job &j, const float *h_xyz_packed,
            const float *const *h_clouds, const float *d_xyz_in, uint64_t *d_out_user,
            std::vector<uint32_t> &lens, const uint64_t **h_out) {
  const bool own_xyz = d_xyz_in == nullptr;
  const bool own_out = d_out_user == nullptr;
  Buffers b{};
  Carver dry(nullptr);
  const size_t need = carve(dry, j, own_xyz, own_out, b);
  int rc = ensure_ws(ctx, need);
  if (rc) return rc;
  Carver c(ctx->ws);
  carve(c, j, own_xyz, own_out, b);
  const bool prof = g_profiling.load() != 0;
  uint32_t launches = 0;

  if (prof) NSFPS_CUDA(cudaEventRecord(ctx->ev[0], st));
  const float *d_xyz = d_xyz_in;
  if (own_xyz) {
    if (h_xyz_packed) {
      NSFPS_CUDA(cudaMemcpyAsync(b.xyz, h_xyz_packed, sizeof(float) * 3 * (size_t)j.n,
                                 cudaMemcpyHostToDevice, st));
    } else {
      for (uint32_t i = 0; i < j.B; ++i) {
        const size_t cnt = j.poff[i + 1] - j.poff[i];
        NSFPS_CUDA(cudaMemcpyAsync(b.xyz + 3 * (size_t)j.poff[i], h_clouds[i],
                                   sizeof(float) * 3 * cnt, cudaMemcpyHostToDevice, st));
      }
    }
    d_xyz = b.xyz;
  }
  // the call's small inputs, staged on the host and uploaded as one copy
  const uint32_t *cand = j.B == 1 ? kSingleCand : kBatchCand;
  const int ncand = j.B == 1 ? kNumSingle : kNumBatch;
  const ParamLayout L = param_layout(j);
  const size_t cbytes = ctrl_bytes(j);
  // (with host results: they come back behind the control block, so one
  // pinned buffer takes both and the copy runs asynchronously)
  const size_t res_off = align_up(cbytes, 256);
  const size_t res_bytes = h_out ? sizeof(uint64_t) * j.B * (size_t)j.k : 0;
  const size_t sbytes = std::max(L.bytes, res_off + res_bytes);
  unsigned char *hs = staging(ctx, sbytes);
  if (!hs) return set_error(NSFPS_ERR_OOM, "host staging buffer of %zu bytes unavailable",
                            sbytes);
  std::memcpy(hs + L.poff, j.poff.data(), 4 * ((size_t)j.B + 1));
  std::memcpy(hs + L.rid, j.rid.data(), 4 * (size_t)j.B);
  std::memcpy(hs + L.boff, j.boff.data(), 4 * (size_t)j.B);
  std::memcpy(hs + L.ranges, j.ranges.data(), sizeof(RangeDev) * j.ranges.size());
  std::memcpy(hs + L.tabs, j.tabs.data(), sizeof(float) * j.tabs.size());
  std::memcpy(hs + L.cand, cand, sizeof(uint32_t) * ncand);
  NSFPS_CUDA(cudaMemcpyAsync(b.params, hs, L.bytes, cudaMemcpyHostToDevice, st));
  NSFPS_CUDA(cudaMemsetAsync(b.stats, 0, 4 * sizeof(unsigned long long), st));

  uint32_t hplan[3 * kMaxCand] = {};
  uint32_t hscal[kScalarCount] = {};
  uint32_t max_tab = 0;
  for (const RangeDev &r : j.ranges)
    if (r.fast_cube)
      max_tab = std::max(max_tab, r.blocks[0] + r.blocks[1] + r.blocks[2] - 3);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device);
  // A single small cloud whose worst case -- every leaf a single point --
  // still gives each worker thread at most one leaf of a 64-CTA grid (and
  // fits shared memory) is launched right behind its setup with that worst
  // case as its plan: the layout is the one the data would get, and the call
  // makes no round trip to the host for the plan.
  int direct = -1;
  if (j.B == 1 && !j.any_hashed && !g_force_steps.load() && b.glist &&
      j.n >= kGridMinPoints && (uint32_t)sms >= kDirectP &&
      rounds_grid_candidates_per_cta(kDirectP) > 0) {
    const uint32_t lmax = (j.n + kDirectP - 1) / kDirectP;
    const uint32_t pmax = std::min<uint32_t>(j.n, (uint32_t)kLeafSize * lmax);
    for (int i = 0; i < ncand; ++i)
      if (cand[i] == kDirectP && rounds_leaves_per_thread(lmax) == 1 && pmax <= 65535 &&
          rounds_smem_bytes(pmax, lmax, max_tab) <= (size_t)rounds_max_smem(kDirectP)) {
        direct = i;
        hplan[3 * i] = pmax;
        hplan[3 * i + 1] = lmax;
      }
  }
  SetupArgs sa;
  std::memset(&sa, 0, sizeof(sa));  // compared bytewise by the graph cache
  sa.n = j.n;
  sa.B = j.B;
  sa.max_key = (uint32_t)(j.total_buckets - 1);
  sa.xyz = d_xyz;
  sa.poff = b.poff;
  sa.rid = b.rid;
  sa.ranges = b.ranges;
  sa.boff = b.boff;
  sa.keys0 = b.keys0; sa.vals0 = b.vals0; sa.keys1 = b.keys1; sa.vals1 = b.vals1;
  sa.hist = b.hist;
  sa.partial = b.partial;
  sa.pts = b.pts;
  sa.perm = b.perm;
  sa.tmp0 = b.tmp0; sa.tmp1 = b.tmp1;
  sa.leaf_start = b.leaf_start;
  sa.leaf_lo = b.leaf_lo; sa.leaf_hi = b.leaf_hi; sa.leaf_md = b.leaf_md;
  sa.leaf_pre = b.leaf_pre;
  sa.loff = b.loff;
  sa.scalars = b.scalars;
  sa.cand = b.cand;
  sa.cand_host = cand;
  sa.ncand = direct >= 0 ? 0 : ncand;  // a direct launch reads no plan
  sa.plan = b.plan;
  sa.small_rounds = small_setup(j, cand, ncand);
  NSFPS_CUDA(run_setup_cached(ctx, sa, st, launches));

  if (direct < 0) {
    // scalars, stats and plan come back as one copy (the staging buffer's
    // upload was issued before on the same stream, so it has been read)
    NSFPS_CUDA(cudaMemcpyAsync(hs, b.ctrl, kCtrlCount, cudaMemcpyDeviceToHost, st));
    if (prof) NSFPS_CUDA(cudaEventRecord(ctx->ev[1], st));
    NSFPS_CUDA(cudaStreamSynchronize(st));
    std::memcpy(hscal, hs + kCtrlScalars, sizeof(hscal));
    std::memcpy(hplan, hs + kCtrlPlan, sizeof(uint32_t) * 3 * ncand);
  } else if (prof) {
    NSFPS_CUDA(cudaEventRecord(ctx->ev[1], st));
  }

  // CTAs per cloud: the smallest count whose largest part fits in shared
  // memory; then, while every cloud still gets its own SMs, keep doubling it:
  // for the round loop up to the cluster limit (fewer leaves per worker warp,
  // the same steps), for the per-step loop until each thread owns a single
  // leaf (more CTAs also mean more proposals per step there).
  const int max_smem = loop_max_smem();
  // direct ranges use the round-based loop, hashed ranges the per-step one;
  // so do parts with more leaves than the round-based loop's threads can own
  bool rounds = !j.any_hashed && !g_force_steps.load();
  auto fits = [&](int i, int &m, size_t &bytes) {
    const uint32_t pts = hplan[3 * i], leaves = hplan[3 * i + 1], extra = hplan[3 * i + 2];
    const uint32_t P = cand[i];
    bytes = rounds ? rounds_smem_bytes(pts, leaves, max_tab)
                   : loop_smem_bytes(pts, leaves, extra, max_tab);
    const int cap = rounds ? rounds_max_smem(P) : max_smem;
    m = rounds ? rounds_leaves_per_thread(leaves) : loop_leaves_per_thread(leaves);
    return m > 0 && bytes <= (size_t)cap && pts <= 65535;
  };
  int pi = -1, m_sel = 0;
  size_t bytes_sel = 0;
  auto select = [&]() {
    pi = -1;
    for (int i = 0; i < kNumCluster; ++i) {
      int m;
      size_t bytes;
      if (!fits(i, m, bytes)) continue;
      if (pi < 0) {
        pi = i; m_sel = m; bytes_sel = bytes;
        continue;
      }
      if ((!rounds && m_sel == 1) || (uint64_t)j.B * cand[i] > (uint64_t)sms) break;
      pi = i; m_sel = m; bytes_sel = bytes;
    }
  };
  bool grid = false;
  uint32_t groups = 1;
  if (direct >= 0) {
    pi = direct;
    m_sel = 1;
    bytes_sel = rounds_smem_bytes(hplan[3 * direct], hplan[3 * direct + 1], max_tab);
    grid = true;
  } else {
    select();
    if (pi < 0 && rounds) {
      rounds = false;
      select();
    }
    // A single cloud too large for a cluster takes the grid-wide round loop
    // over P co-resident CTAs (one per SM), the smallest P that fits.  So does
    // a single cloud of kGridMinPoints or more that fits a cluster: over more
    // CTAs its parts are smaller (lighter workers, shorter lists) and each round
    // replays more candidates, so it runs faster.
    if (j.B == 1 && !j.any_hashed && !g_force_steps.load() && b.glist &&
        (pi < 0 || j.n >= kGridMinPoints)) {
      for (int i = kNumCluster; i < kNumSingle && !grid; ++i) {
        const uint32_t P = cand[i];
        // one cloud: 64 or 128 CTAs (32 with 8 candidates each was slower on
        // c2, 4.89 against 4.16 ms at 64)
        if (P > (uint32_t)sms || P > kMaxGridP || (P != 64u && P != 128u)) continue;
        const bool was_rounds = rounds;
        rounds = true;
        int m;
        size_t bytes;
        if (fits(i, m, bytes)) {
          pi = i; m_sel = m; bytes_sel = bytes; grid = true;
        } else {
          rounds = was_rounds;
        }
      }
    }
    // A batch whose clouds fit the round loop: the layout that keeps the most
    // clouds running at once.  A cluster must fit one GPC, so at one CTA per
    // SM the device holds only some clusters (7 of 16 CTAs on B200, 112 of
    // 148 SMs); groups of co-resident CTAs (the grid-wide loop, one group per
    // cloud in turn) have no such limit.
    if (j.B > 1 && rounds && pi >= 0 && !g_force_steps.load()) {
      const uint32_t Pc = cand[pi];
      int force = -1;  // NSFPS_BATCH_GROUP_CTAS: 0 = clusters, P = groups of P CTAs
      if (const char *v = std::getenv("NSFPS_BATCH_GROUP_CTAS")) force = std::atoi(v);
      const int cap =
          force < 0 ? rounds_cluster_capacity(Pc, m_sel, std::max<size_t>(bytes_sel, 16)) : 0;
      const uint32_t conc_c = cap > 0 ? std::min<uint32_t>(j.B, (uint32_t)cap * 1u) : j.B;
      int gi = -1;
      if (force > 0) {
        for (int i = 0; i < kNumBatch; ++i)
          if (cand[i] == (uint32_t)force) gi = i;
      } else if (force < 0 && conc_c < j.B && Pc >= 2) {
        gi = pi;  // the same CTAs per cloud, more clouds at once
      }
      if (gi >= 0) {
        int m;
        size_t bytes;
        const uint32_t P = cand[gi];
        if (P <= (uint32_t)sms && rounds_grid_candidates_per_cta(P) > 0 && fits(gi, m, bytes)) {
          pi = gi; m_sel = m; bytes_sel = bytes; grid = true;
          groups = std::min<uint32_t>(j.B, std::min<uint32_t>((uint32_t)sms, kMaxGridCtas) / P);
        } else if (force > 0) {
          return set_error(NSFPS_ERR_UNSUPPORTED, "NSFPS_BATCH_GROUP_CTAS=%d does not fit", force);
        }
      }
    }
  }
  if (pi < 0)
    return set_error(NSFPS_ERR_UNSUPPORTED,
                     "cloud too large for the shared-memory-resident sampler "
                     "(largest cloud part needs more than %d bytes at %u CTAs)",
                     max_smem, j.B == 1 ? std::min<uint32_t>(kMaxGridP, (uint32_t)sms) : 16u);
  LoopPlan plan{};
  plan.mode = grid ? 1 : 0;
  plan.rounds = rounds ? 1 : 0;
  plan.P = cand[pi];
  plan.leaves_per_thread = m_sel;
  plan.direct = !j.any_hashed;
  plan.smem_bytes = std::max<size_t>(bytes_sel, 16);

  LoopArgs la{};
  la.B = j.B;
  la.k = j.k;
  la.P = plan.P;
  la.max_pts = hplan[3 * pi];
  la.max_leaves = hplan[3 * pi + 1];
  la.max_extra = hplan[3 * pi + 2];
  la.max_tab = max_tab;
  la.pts = b.pts;
  la.leaf_start = b.leaf_start;
  la.leaf_lo = b.leaf_lo;
  la.leaf_hi = b.leaf_hi;
  la.leaf_md = b.leaf_md;
  la.leaf_pre = b.leaf_pre;
  la.loff = b.loff;
  la.poff = b.poff;
  la.rid = b.rid;
  la.ranges = b.ranges;
  la.tabs = b.tabs;
  la.out_rank = b.out_rank;
  la.out_count = b.out_count;
  la.scalars = b.scalars;
  la.stats = b.stats;
  la.groups = grid ? groups : 0;
  la.glist = b.glist;
  la.gbar = b.gbar;
  la.timeout_ns = g_wait_ns.load();
  la.hold_cta = g_hold_cta.load();
  la.hold_step = g_hold_step.load();
  if (prof) NSFPS_CUDA(cudaEventRecord(ctx->ev[2], st));
  NSFPS_CUDA(plan.rounds ? run_rounds(la, plan, st, launches) : run_loop(la, plan, st, launches));
  if (prof) NSFPS_CUDA(cudaEventRecord(ctx->ev[3], st));
  uint64_t *d_out = own_out ? b.out : d_out_user;
  NSFPS_CUDA(run_epilogue(b.out_rank, b.out_count, b.perm, b.poff, j.B, j.k, d_out, st,
                          launches));
  lens.assign(j.B, 0);
  unsigned long long hstats[4] = {};
  NSFPS_CUDA(cudaMemcpyAsync(hs, b.ctrl, cbytes, cudaMemcpyDeviceToHost, st));
  if (h_out) {
    NSFPS_CUDA(cudaMemcpyAsync(hs + res_off, d_out, res_bytes, cudaMemcpyDeviceToHost, st));
    *h_out = reinterpret_cast<const uint64_t *>(hs + res_off);
  }
  NSFPS_CUDA(cudaStreamSynchronize(st));
  std::memcpy(hscal, hs + kCtrlScalars, sizeof(hscal));
  std::memcpy(hstats, hs + kCtrlStats, sizeof(hstats));
  std::memcpy(lens.data(), hs + kCtrlCount, 4 * (size_t)j.B);
  if (hscal[kScalarStatus] & kStatusTimeout)
    return set_error(NSFPS_ERR_TIMEOUT, "sampling kernel: a bounded wait timed out");
  if (hscal[kScalarStatus] & kStatusBadPlan)
    return set_error(NSFPS_ERR_CUDA, "sampling kernel: partition exceeded its plan");

  if (prof) {
    nsfps_profile p{};
    float ms = 0;
    cudaEventElapsedTime(&ms, ctx->ev[0], ctx->ev[1]);
    p.setup_ms = ms;
    cudaEventElapsedTime(&ms, ctx->ev[2], ctx->ev[3]);
    p.loop_ms = ms;
    cudaEventElapsedTime(&ms, ctx->ev[0], ctx->ev[3]);
    p.total_ms = ms;
    p.launches = launches;
    p.ctas_per_cloud = plan.P;
    p.mode = plan.rounds ? (plan.mode == 1 ? 3u : 2u) : (uint32_t)plan.mode;
    p.leaves = hscal[kScalarLeaves];
    p.ref_points_updated = hstats[0];
    p.points_evaluated = hstats[1];
    uint64_t iters = 0;
    for (uint32_t l : lens) iters += l;
    p.iterations = iters;
    g_prof = p;
  }
  return NSFPS_OK;
}

int check_points(const float *xyz, uint64_t n) {
  if (n && !xyz) return set_error(NSFPS_ERR_ARG, "points pointer is NULL");
  return NSFPS_OK;
}

// compute_bbox (src/yuezu_fps.cpp:648-670), std::min/std::max semantics.
nsfps_range bbox_of(const float *xyz, uint64_t n, uint32_t xb, uint32_t yb, uint32_t zb) {
  nsfps_range r{};
  if (n == 0) {
    r = {0, 1, 0, 1, 0, 1, 1, 1, 1};
    return r;
  }
  float mn[3] = {xyz[0], xyz[1], xyz[2]}, mx[3] = {xyz[0], xyz[1], xyz[2]};
  for (uint64_t i = 0; i < n; ++i)
    for (int a = 0; a < 3; ++a) {
      const float v = xyz[3 * i + a];
      mn[a] = (v < mn[a]) ? v : mn[a];
      mx[a] = (mx[a] < v) ? v : mx[a];
    }
  const float eps = NSFPS_BOUNDARY_EPS;
  r.min_x = mn[0] - eps; r.max_x = mx[0] + eps;
  r.min_y = mn[1] - eps; r.max_y = mx[1] + eps;
  r.min_z = mn[2] - eps; r.max_z = mx[2] + eps;
  r.x_blocks = xb; r.y_blocks = yb; r.z_blocks = zb;
  return r;
}

// compute_bbox(cloud, xb, yb, zb) of `count` device-resident clouds (the
// reference's fps(range=None) and fps_with_bbox paths, src/yuezu_fps.cpp:
// 643-670), with the reduction on the device and the same float arithmetic
// as bbox_of after it.
int device_bboxes(DeviceCtx *ctx, cudaStream_t st, const float *d_xyz, const uint64_t *offsets,
                  uint64_t count, const uint32_t blocks[3], std::vector<nsfps_range> &rs) {
  const size_t off_bytes = align_up(sizeof(uint32_t) * (count + 1), 256);
  int rc = ensure_ws(ctx, off_bytes + sizeof(float) * 6 * count);
  if (rc) return rc;
  uint32_t *d_poff = (uint32_t *)ctx->ws;
  float *d_box = (float *)((char *)ctx->ws + off_bytes);
  std::vector<uint32_t> hpoff(count + 1);
  for (uint64_t i = 0; i <= count; ++i) {
    if (offsets[i] - offsets[0] >= (1ull << 31))
      return set_error(NSFPS_ERR_UNSUPPORTED, "too many points in one call");
    hpoff[i] = (uint32_t)(offsets[i] - offsets[0]);
  }
  std::vector<float> hbox(6 * count);
  uint32_t launches = 0;
  NSFPS_CUDA(cudaMemcpyAsync(d_poff, hpoff.data(), sizeof(uint32_t) * (count + 1),
                             cudaMemcpyHostToDevice, st));
  uint32_t max_cloud = 0;
  for (uint64_t i = 0; i < count; ++i) max_cloud = std::max(max_cloud, hpoff[i + 1] - hpoff[i]);
  NSFPS_CUDA(run_cloud_bbox(d_xyz, d_poff, (uint32_t)count, max_cloud, d_box, st, launches));
  NSFPS_CUDA(cudaMemcpyAsync(hbox.data(), d_box, sizeof(float) * 6 * count,
                             cudaMemcpyDeviceToHost, st));
  NSFPS_CUDA(cudaStreamSynchronize(st));
  const float eps = NSFPS_BOUNDARY_EPS;
  rs.resize(count);
  for (uint64_t c = 0; c < count; ++c) {
    const float *b = &hbox[6 * c];
    nsfps_range &r = rs[c];
    r.min_x = b[0] - eps; r.max_x = b[3] + eps;
    r.min_y = b[1] - eps; r.max_y = b[4] + eps;
    r.min_z = b[2] - eps; r.max_z = b[5] + eps;
    r.x_blocks = blocks[0];
    r.y_blocks = blocks[1];
    r.z_blocks = blocks[2];
  }
  return NSFPS_OK;
}

// Clouds handled without the GPU, exactly as yuezu_fps's early returns
// (src/yuezu_fps.cpp:678-688): n == 0 or k == 0 -> [], k >= n -> 0..n-1.
bool trivial(uint64_t n, uint64_t k) { return n == 0 || k == 0 || k >= n; }

void fill_trivial(uint64_t n, uint64_t k, uint64_t *out, uint64_t *len) {
  if (n == 0 || k == 0) { *len = 0; return; }
  for (uint64_t i = 0; i < n; ++i) out[i] = i;
  *len = n;
}

// ---- grouping after sampling

// offsets[0..count] (host, non-decreasing) relative to offsets[0], as uint32.
int rel_offsets(const uint64_t *offsets, uint64_t count, const char *what,
                std::vector<uint32_t> &out) {
  out.resize(count + 1);
  for (uint64_t i = 0; i <= count; ++i) {
    if (i < count && offsets[i + 1] < offsets[i])
      return set_error(NSFPS_ERR_ARG, "%s must not decrease", what);
    if (offsets[i] - offsets[0] >= (1ull << 31))
      return set_error(NSFPS_ERR_UNSUPPORTED, "too many entries in %s (>= 2^31)", what);
    out[i] = (uint32_t)(offsets[i] - offsets[0]);
  }
  return NSFPS_OK;
}

struct GroupBuffers {
  uint32_t *poff, *coff, *cbase, *keys0, *vals0, *keys1, *vals1, *hist, *partial, *cstart;
  uint32_t *box;
  GroupGrid *grids;
  float4 *pts;
};

size_t carve_group(Carver &c, uint32_t B, uint32_t n, uint32_t cells, GroupBuffers &b) {
  const size_t tiles = radix_tiles(n);
  const size_t scan_len = std::max<size_t>(256 * tiles, (size_t)cells + 1);
  b.poff = c.take<uint32_t>(B + 1);
  b.coff = c.take<uint32_t>(B + 1);
  b.cbase = c.take<uint32_t>(B + 1);
  b.box = c.take<uint32_t>(6 * (size_t)B);
  b.grids = c.take<GroupGrid>(B);
  b.keys0 = c.take<uint32_t>(n);
  b.vals0 = c.take<uint32_t>(n);
  b.keys1 = c.take<uint32_t>(n);
  b.vals1 = c.take<uint32_t>(n);
  b.hist = c.take<uint32_t>(256 * tiles + 1);
  b.partial = c.take<uint32_t>((scan_len + 4095) / 4096 + 2);
  b.cstart = c.take<uint32_t>((size_t)cells + 1);
  b.pts = c.take<float4>(n);
  return align_up(c.off, 256);
}

// Cells a cloud of nc points may use: up to 16 per point (so that cells
// stay about one radius wide in sparse clouds), at least 4096, at most 2^22.
uint32_t group_cell_cap(uint32_t nc) {
  const uint64_t want = std::max<uint64_t>(4096u, 16ull * nc);
  return (uint32_t)std::min<uint64_t>(want, 1u << 22);
}

// Ball query of packed device-resident clouds (poff / coff: host offsets)
// on stream st; returns after the stream has drained.
int ball_query_on(DeviceCtx *ctx, cudaStream_t st, const float *d_xyz,
                  const std::vector<uint32_t> &poff, const float *d_centers,
                  const std::vector<uint32_t> &coff, float radius, uint32_t S, int64_t *d_idx,
                  uint32_t *d_hits) {
  const uint32_t B = (uint32_t)(poff.size() - 1);
  const uint32_t n = poff[B], m = coff[B];
  if (m == 0) return NSFPS_OK;
  const float rr = std::fabs(radius);
  if (!(rr > 0.0f)) {
    // radius 0 or NaN: d2 < r2 holds for no point; every slot is index 0
    NSFPS_CUDA(cudaMemsetAsync(d_idx, 0, sizeof(int64_t) * (size_t)m * S, st));
    if (d_hits) NSFPS_CUDA(cudaMemsetAsync(d_hits, 0, sizeof(uint32_t) * (size_t)m, st));
    NSFPS_CUDA(cudaStreamSynchronize(st));
    return NSFPS_OK;
  }
  std::vector<uint32_t> cbase(B + 1);
  uint64_t cells = 0;
  for (uint32_t c = 0; c < B; ++c) {
    cbase[c] = (uint32_t)cells;
    cells += group_cell_cap(poff[c + 1] - poff[c]);
    if (cells >= (1ull << 31))
      return set_error(NSFPS_ERR_UNSUPPORTED, "too many clouds in one ball query");
  }
  cbase[B] = (uint32_t)cells;
  GroupBuffers b{};
  Carver dry(nullptr);
  const size_t need = carve_group(dry, B, n, (uint32_t)cells, b);
  int rc = ensure_ws(ctx, need);
  if (rc) return rc;
  Carver cv(ctx->ws);
  carve_group(cv, B, n, (uint32_t)cells, b);
  NSFPS_CUDA(cudaMemcpyAsync(b.poff, poff.data(), 4 * (B + 1), cudaMemcpyHostToDevice, st));
  NSFPS_CUDA(cudaMemcpyAsync(b.coff, coff.data(), 4 * (B + 1), cudaMemcpyHostToDevice, st));
  NSFPS_CUDA(cudaMemcpyAsync(b.cbase, cbase.data(), 4 * (B + 1), cudaMemcpyHostToDevice, st));
  GroupArgs a{};
  a.n = n; a.B = B; a.m = m; a.S = S;
  a.max_cloud = 0;
  for (uint32_t c = 0; c < B; ++c) a.max_cloud = std::max(a.max_cloud, poff[c + 1] - poff[c]);
  a.cells = (uint32_t)cells;
  a.r2 = radius * radius;
  a.h_min = 1.01 * (double)rr;
  a.xyz = d_xyz; a.centers = d_centers;
  a.poff = b.poff; a.coff = b.coff; a.cbase = b.cbase;
  a.box = b.box; a.grids = b.grids;
  a.keys0 = b.keys0; a.vals0 = b.vals0; a.keys1 = b.keys1; a.vals1 = b.vals1;
  a.hist = b.hist; a.partial = b.partial; a.cstart = b.cstart; a.pts = b.pts;
  a.out_idx = d_idx; a.out_hits = d_hits;
  uint32_t launches = 0;
  const bool prof = g_profiling.load() != 0;
  if (prof) NSFPS_CUDA(cudaEventRecord(ctx->ev[0], st));
  NSFPS_CUDA(run_ball_query(a, st, launches, prof ? ctx->ev[1] : nullptr,
                            prof ? ctx->ev[2] : nullptr));
  NSFPS_CUDA(cudaStreamSynchronize(st));
  if (prof) {
    // setup = grid build (box, cells, sort, cell starts); loop = query kernel
    g_prof = nsfps_profile{};
    cudaEventElapsedTime(&g_prof.setup_ms, ctx->ev[0], ctx->ev[1]);
    cudaEventElapsedTime(&g_prof.loop_ms, ctx->ev[1], ctx->ev[2]);
    cudaEventElapsedTime(&g_prof.total_ms, ctx->ev[0], ctx->ev[2]);
    g_prof.launches = launches;
    g_prof.mode = 4;
  }
  return NSFPS_OK;
}

// Gather (ctr == nullptr) or relative grouping of device-resident clouds:
// the index check's flag comes back through the workspace.
int gather_on(DeviceCtx *ctx, cudaStream_t st, const float *d_xyz,
              const std::vector<uint32_t> &poff, const float *d_centers,
              const std::vector<uint32_t> &ioff, uint32_t S, const int64_t *d_idx, float *d_out) {
  const uint32_t B = (uint32_t)(poff.size() - 1);
  const uint32_t m = ioff[B];
  if (m == 0) return NSFPS_OK;
  const size_t off_bytes = align_up(sizeof(uint32_t) * (B + 1), 256);
  int rc = ensure_ws(ctx, 2 * off_bytes + 256);
  if (rc) return rc;
  uint32_t *d_poff = (uint32_t *)ctx->ws;
  uint32_t *d_ioff = (uint32_t *)((char *)ctx->ws + off_bytes);
  uint32_t *d_err = (uint32_t *)((char *)ctx->ws + 2 * off_bytes);
  NSFPS_CUDA(cudaMemcpyAsync(d_poff, poff.data(), 4 * (B + 1), cudaMemcpyHostToDevice, st));
  NSFPS_CUDA(cudaMemcpyAsync(d_ioff, ioff.data(), 4 * (B + 1), cudaMemcpyHostToDevice, st));
  NSFPS_CUDA(cudaMemsetAsync(d_err, 0, sizeof(uint32_t), st));
  uint32_t launches = 0;
  if (d_centers)
    NSFPS_CUDA(run_group_points(d_xyz, d_poff, d_centers, d_ioff, B, m, S, d_idx, d_out, d_err, st,
                                launches));
  else
    NSFPS_CUDA(run_gather_points(d_xyz, d_poff, d_idx, d_ioff, B, m, d_out, d_err, st, launches));
  uint32_t herr = 0;
  NSFPS_CUDA(cudaMemcpyAsync(&herr, d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
  NSFPS_CUDA(cudaStreamSynchronize(st));
  if (herr)
    return set_error(NSFPS_ERR_ARG, "an index lies outside its cloud (its output is NaN)");
  return NSFPS_OK;
}

// Batched host-memory path on one device.
int batched_on_device(int device, const float *const *clouds, const uint64_t *n,
                      const std::vector<uint64_t> &idx, uint64_t k,
                      const std::vector<nsfps_range> &ranges,
                      const std::vector<uint32_t> &rid_all, uint64_t *const *out,
                      uint64_t *out_len) {
  std::vector<uint64_t> gpu_idx;
  for (uint64_t i : idx)
    if (!trivial(n[i], k)) gpu_idx.push_back(i);
  if (gpu_idx.empty()) return NSFPS_OK;
  DeviceCtx *ctx = nullptr;
  int rc = get_ctx(device, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  NSFPS_CUDA(cudaSetDevice(device));
  std::vector<uint64_t> gn;
  std::vector<const float *> gc;
  std::vector<uint32_t> grid;
  for (uint64_t i : gpu_idx) {
    gn.push_back(n[i]);
    gc.push_back(clouds[i]);
    grid.push_back(rid_all[i]);
  }
  Job j;
  rc = build_job(gn.data(), gn.size(), k, ranges, grid, j);
  if (rc) return rc;
  std::vector<uint32_t> lens;
  // the results stay in the device's staging buffer until the next call,
  // which the device lock held here keeps out
  const uint64_t *hout = nullptr;
  rc = run_job(ctx, ctx->stream, j, nullptr, gc.data(), nullptr, nullptr, lens, &hout);
  if (rc == NSFPS_ERR_UNSUPPORTED && gpu_idx.size() > 1) {
    // a cloud too large to share the device with the others: one job per
    // cloud (a single cloud may use the grid-wide loop)
    for (size_t c = 0; c < gpu_idx.size(); ++c) {
      Job j1;
      rc = build_job(&gn[c], 1, k, ranges, std::vector<uint32_t>(1, grid[c]), j1);
      if (rc) return rc;
      rc = run_job(ctx, ctx->stream, j1, nullptr, &gc[c], nullptr, nullptr, lens, &hout);
      if (rc) return rc;
      const uint64_t i = gpu_idx[c];
      std::memcpy(out[i], hout, sizeof(uint64_t) * lens[0]);
      out_len[i] = lens[0];
    }
    return NSFPS_OK;
  }
  if (rc) return rc;
  for (size_t c = 0; c < gpu_idx.size(); ++c) {
    const uint64_t i = gpu_idx[c];
    std::memcpy(out[i], hout + c * (size_t)k, sizeof(uint64_t) * lens[c]);
    out_len[i] = lens[c];
  }
  return NSFPS_OK;
}

// Per-device contexts whose workspace is the fixed scratch array of
// nsfps_static.cu: set up once per device (address and events) with that
// device current; never grown, never freed.
DeviceCtx g_static_ctx[kMaxDevices];

int get_static_ctx(int device, DeviceCtx **out) {
  if (device < 0 || device >= kMaxDevices)
    return set_error(NSFPS_ERR_ARG, "device %d out of range", device);
  DeviceCtx *c = &g_static_ctx[device];
  std::lock_guard<std::mutex> lk(g_ctx_mu);
  if (!c->ready) {
    void *p = nullptr;
    size_t bytes = 0;
    NSFPS_CUDA(static_scratch_address(&p, &bytes));
    if (!p || bytes < NSFPS_STATIC_SCRATCH_BYTES)
      return set_error(NSFPS_ERR_CUDA, "static scratch array unavailable");
    for (auto &ev : c->ev) NSFPS_CUDA(cudaEventCreate(&ev));
    c->ws = p;
    c->ws_bytes = bytes;
    c->device = device;
    c->fixed = true;
    c->ready = true;
  }
  *out = c;
  return NSFPS_OK;
}

}  // namespace
}  // namespace nsfps

// ======================================================================= C ABI
using namespace nsfps;

extern "C" {

const char *nsfps_last_error(void) { return g_err.c_str(); }

int nsfps_version(void) { return 100; }

int nsfps_device_count(int *count) {
  clear_error();
  if (!count) return set_error(NSFPS_ERR_ARG, "count is NULL");
  int c = 0;
  cudaError_t e = cudaGetDeviceCount(&c);
  if (e != cudaSuccess) {
    cudaGetLastError();
    *count = 0;
    return set_error(NSFPS_ERR_CUDA, "cudaGetDeviceCount: %s", cudaGetErrorString(e));
  }
  *count = c;
  return NSFPS_OK;
}

int nsfps_make_range(float min_x, float max_x, float min_y, float max_y, float min_z,
                     float max_z, uint32_t x_blocks, uint32_t y_blocks, uint32_t z_blocks,
                     nsfps_range *out) {
  clear_error();
  if (!out) return set_error(NSFPS_ERR_ARG, "out is NULL");
  *out = {min_x, max_x, min_y, max_y, min_z, max_z, x_blocks, y_blocks, z_blocks};
  return NSFPS_OK;
}

int nsfps_make_uniform_range(float min_x, float max_x, float min_y, float max_y,
                             float min_z, float max_z, uint32_t blocks_per_dim,
                             nsfps_range *out) {
  return nsfps_make_range(min_x, max_x, min_y, max_y, min_z, max_z, blocks_per_dim,
                          blocks_per_dim, blocks_per_dim, out);
}

int nsfps_range_get_info(const nsfps_range *r, nsfps_range_info *info) {
  clear_error();
  if (!r || !info) return set_error(NSFPS_ERR_ARG, "NULL argument");
  return range_info(*r, info);
}

int nsfps_range_get_lut(const nsfps_range *r, int axis, uint32_t *lut, uint64_t cap,
                        uint64_t *len) {
  clear_error();
  if (!r || !len || axis < 0 || axis > 2) return set_error(NSFPS_ERR_ARG, "bad argument");
  RangeDev d;
  int rc = range_to_dev(*r, &d, nullptr);
  if (rc) return rc;
  const uint64_t cnt = 1ull << d.bits[axis];
  *len = cnt;
  if (lut)
    for (uint64_t v = 0; v < cnt && v < cap; ++v)
      lut[v] = spread((uint32_t)v, d.bits[axis], d.pos[axis]);
  return NSFPS_OK;
}

int nsfps_compute_bbox(const float *xyz, uint64_t n, uint32_t x_blocks, uint32_t y_blocks,
                       uint32_t z_blocks, nsfps_range *out) {
  clear_error();
  if (!out) return set_error(NSFPS_ERR_ARG, "out is NULL");
  int rc = check_points(xyz, n);
  if (rc) return rc;
  *out = bbox_of(xyz, n, x_blocks, y_blocks, z_blocks);
  return NSFPS_OK;
}

int nsfps_fps_batched(const float *const *clouds, const uint64_t *n, uint64_t count,
                      uint64_t k, const nsfps_range *ranges, int per_cloud_ranges,
                      uint64_t *const *out, uint64_t *out_len, const int *devices,
                      int ndev) {
  clear_error();
  if (count == 0) return NSFPS_OK;
  if (!clouds || !n || !out || !out_len) return set_error(NSFPS_ERR_ARG, "NULL argument");
  if (ndev < 1) return set_error(NSFPS_ERR_ARG, "ndev must be >= 1");
  for (uint64_t i = 0; i < count; ++i) {
    int rc = check_points(clouds[i], n[i]);
    if (rc) return rc;
    if (!out[i] && n[i] && k) return set_error(NSFPS_ERR_ARG, "out[%llu] is NULL",
                                               (unsigned long long)i);
  }
  std::vector<nsfps_range> rs;
  std::vector<uint32_t> rid(count, 0);
  if (!ranges) {
    for (uint64_t i = 0; i < count; ++i) {
      rs.push_back(bbox_of(clouds[i], n[i], NSFPS_DEFAULT_X_BLOCKS, NSFPS_DEFAULT_Y_BLOCKS,
                           NSFPS_DEFAULT_Z_BLOCKS));
      rid[i] = (uint32_t)i;
    }
  } else if (per_cloud_ranges) {
    rs.assign(ranges, ranges + count);
    for (uint64_t i = 0; i < count; ++i) rid[i] = (uint32_t)i;
  } else {
    rs.push_back(ranges[0]);
  }
  for (auto &r : rs) {
    RangeDev d;
    int rc = range_to_dev(r, &d, nullptr);
    if (rc) return rc;
  }
  // An inverted range (max < min) gives a negative block size, so the
  // reference's cube list reserve() throws on the first sampling step; reject
  // it for every cloud that would reach that step.
  for (uint64_t i = 0; i < count; ++i) {
    if (trivial(n[i], k) || k < 2) continue;
    const nsfps_range &r = rs[rid[i]];
    if (r.max_x < r.min_x || r.max_y < r.min_y || r.max_z < r.min_z)
      return set_error(NSFPS_ERR_ARG,
                       "SpaceRange max must not be below min (got x [%g, %g], y [%g, %g], "
                       "z [%g, %g])", r.min_x, r.max_x, r.min_y, r.max_y, r.min_z, r.max_z);
  }
  // the reference's early returns (src/yuezu_fps.cpp:678-688) need no GPU;
  // the other clouds go whole, round-robin, to the devices (one host thread
  // per device)
  std::vector<std::vector<uint64_t>> share(ndev);
  uint64_t ngpu = 0;
  for (uint64_t i = 0; i < count; ++i) {
    if (trivial(n[i], k)) fill_trivial(n[i], k, out[i], &out_len[i]);
    else share[ngpu++ % ndev].push_back(i);
  }
  std::vector<int> rcs(ndev, NSFPS_OK);
  std::vector<std::string> errs(ndev);
  auto work = [&](int d) {
    const int dev = devices ? devices[d] : d;
    rcs[d] = batched_on_device(dev, clouds, n, share[d], k, rs, rid, out, out_len);
    if (rcs[d]) errs[d] = g_err;
  };
  if (ndev == 1) {
    work(0);
  } else {
    std::vector<std::thread> th;
    for (int d = 0; d < ndev; ++d) th.emplace_back(work, d);
    for (auto &t : th) t.join();
  }
  for (int d = 0; d < ndev; ++d)
    if (rcs[d]) return set_error(rcs[d], "device %d: %s", devices ? devices[d] : d,
                                 errs[d].c_str());
  return NSFPS_OK;
}

int nsfps_fps(const float *xyz, uint64_t n, uint64_t k, const nsfps_range *range,
              uint64_t *out, uint64_t *out_len, int device) {
  clear_error();
  if (!out_len) return set_error(NSFPS_ERR_ARG, "out_len is NULL");
  int rc = check_points(xyz, n);
  if (rc) return rc;
  if (!out && n && k) return set_error(NSFPS_ERR_ARG, "out is NULL");
  const float *clouds[1] = {xyz};
  uint64_t *outs[1] = {out};
  return nsfps_fps_batched(clouds, &n, 1, k, range, 0, outs, out_len, &device, 1);
}

int nsfps_fps_with_bbox(const float *xyz, uint64_t n, uint64_t k, uint32_t x_blocks,
                        uint32_t y_blocks, uint32_t z_blocks, uint64_t *out,
                        uint64_t *out_len, int device) {
  clear_error();
  int rc = check_points(xyz, n);
  if (rc) return rc;
  nsfps_range r = bbox_of(xyz, n, x_blocks, y_blocks, z_blocks);
  return nsfps_fps(xyz, n, k, &r, out, out_len, device);
}

}  // extern "C"

namespace nsfps {
namespace {
// nsfps_fps_device / nsfps_fps_device_with_bbox: ranges == NULL selects each
// cloud's bounding box with bbox_blocks, reduced on the device.
int fps_device_impl(const float *d_xyz, const uint64_t *offsets, uint64_t count, uint64_t k,
                    const nsfps_range *ranges, int per_cloud_ranges, const uint32_t bbox_blocks[3],
                    uint64_t *d_out, uint64_t *out_len, void *stream) {
  if (count == 0) return NSFPS_OK;
  if (!offsets || !out_len || !d_out || !d_xyz)
    return set_error(NSFPS_ERR_ARG, "NULL argument");
  int dev = 0;
  NSFPS_CUDA(cudaGetDevice(&dev));
  DeviceCtx *ctx = nullptr;
  int rc = get_ctx(dev, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  cudaStream_t user = (cudaStream_t)stream;
  std::vector<uint64_t> n(count);
  for (uint64_t i = 0; i < count; ++i) {
    if (offsets[i + 1] < offsets[i]) return set_error(NSFPS_ERR_ARG, "offsets must not decrease");
    n[i] = offsets[i + 1] - offsets[i];
  }
  // clouds needing no sampling loop are answered here; the others run as one job
  bool all_gpu = true;
  for (uint64_t i = 0; i < count; ++i) if (trivial(n[i], k)) all_gpu = false;
  if (!all_gpu)
    return set_error(NSFPS_ERR_UNSUPPORTED,
                     "nsfps_fps_device needs 0 < k < n for every cloud");
  if (offsets[0] != 0) d_xyz += 3 * offsets[0];
  std::vector<nsfps_range> rs;
  std::vector<uint32_t> rid(count, 0);
  if (!ranges) {
    rc = device_bboxes(ctx, user, d_xyz, offsets, count, bbox_blocks, rs);
    if (rc) return rc;
    for (uint64_t i = 0; i < count; ++i) rid[i] = (uint32_t)i;
  } else if (per_cloud_ranges) {
    rs.assign(ranges, ranges + count);
    for (uint64_t i = 0; i < count; ++i) rid[i] = (uint32_t)i;
  } else {
    rs.push_back(ranges[0]);
  }
  Job j;
  rc = build_job(n.data(), count, k, rs, rid, j);
  if (rc) return rc;
  // all work is issued on the caller's stream
  std::vector<uint32_t> lens;
  rc = run_job(ctx, user, j, nullptr, nullptr, d_xyz, d_out, lens, nullptr);
  if (rc) return rc;
  for (uint64_t i = 0; i < count; ++i) out_len[i] = lens[i];
  return NSFPS_OK;
}
}  // namespace
}  // namespace nsfps

extern "C" {

int nsfps_fps_device(const float *d_xyz, const uint64_t *offsets, uint64_t count,
                     uint64_t k, const nsfps_range *ranges, int per_cloud_ranges,
                     uint64_t *d_out, uint64_t *out_len, void *stream) {
  clear_error();
  const uint32_t blocks[3] = {NSFPS_DEFAULT_X_BLOCKS, NSFPS_DEFAULT_Y_BLOCKS,
                              NSFPS_DEFAULT_Z_BLOCKS};
  return fps_device_impl(d_xyz, offsets, count, k, ranges, per_cloud_ranges, blocks, d_out,
                         out_len, stream);
}

int nsfps_fps_device_with_bbox(const float *d_xyz, const uint64_t *offsets, uint64_t count,
                               uint64_t k, uint32_t x_blocks, uint32_t y_blocks,
                               uint32_t z_blocks, uint64_t *d_out, uint64_t *out_len,
                               void *stream) {
  clear_error();
  const uint32_t blocks[3] = {x_blocks, y_blocks, z_blocks};
  return fps_device_impl(d_xyz, offsets, count, k, nullptr, 0, blocks, d_out, out_len, stream);
}

int nsfps_fps_device_static(const float *d_xyz, uint64_t n, uint64_t k,
                            const nsfps_range *range, uint64_t *d_out, uint64_t *out_len,
                            void *stream) {
  clear_error();
  if (!d_xyz || !range || !d_out || !out_len) return set_error(NSFPS_ERR_ARG, "NULL argument");
  if (n > NSFPS_STATIC_MAX_POINTS)
    return set_error(NSFPS_ERR_ARG,
                     "nsfps_fps_device_static: %llu points exceed NSFPS_STATIC_MAX_POINTS (%u), "
                     "the capacity of its fixed scratch array",
                     (unsigned long long)n, NSFPS_STATIC_MAX_POINTS);
  if (trivial(n, k))
    return set_error(NSFPS_ERR_UNSUPPORTED, "nsfps_fps_device_static needs 0 < k < n");
  const nsfps_range &r = *range;
  if (k >= 2 && (r.max_x < r.min_x || r.max_y < r.min_y || r.max_z < r.min_z))
    return set_error(NSFPS_ERR_ARG, "SpaceRange max must not be below min");
  int dev = 0;
  NSFPS_CUDA(cudaGetDevice(&dev));
  std::vector<nsfps_range> rs(1, *range);
  std::vector<uint32_t> rid(1, 0);
  Job j;
  int rc = build_job(&n, 1, k, rs, rid, j);
  if (rc) return rc;
  Buffers b{};
  Carver dry(nullptr);
  const size_t need = carve(dry, j, false, false, b);
  if (need > NSFPS_STATIC_SCRATCH_BYTES)
    return set_error(NSFPS_ERR_UNSUPPORTED,
                     "nsfps_fps_device_static: needs %zu bytes of scratch, the fixed array "
                     "holds %u", need, NSFPS_STATIC_SCRATCH_BYTES);
  DeviceCtx *ctx = nullptr;
  rc = get_static_ctx(dev, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  // the workspace already holds `need` bytes, so run_job allocates nothing
  std::vector<uint32_t> lens;
  rc = run_job(ctx, (cudaStream_t)stream, j, nullptr, nullptr, d_xyz, d_out, lens, nullptr);
  if (rc) {
    // an error may leave work queued on `stream` that still uses the array:
    // drain it before the lock lets the next call in
    cudaStreamSynchronize((cudaStream_t)stream);
    return rc;
  }
  *out_len = lens[0];
  return NSFPS_OK;
}

int nsfps_ball_query_device(const float *d_xyz, const uint64_t *point_offsets,
                            const float *d_centers, const uint64_t *center_offsets,
                            uint64_t count, float radius, uint32_t nsample, int64_t *d_idx,
                            uint32_t *d_hits, void *stream) {
  clear_error();
  if (count == 0) return NSFPS_OK;
  if (!point_offsets || !center_offsets) return set_error(NSFPS_ERR_ARG, "NULL offsets");
  if (nsample == 0 || nsample > NSFPS_MAX_NSAMPLE)
    return set_error(NSFPS_ERR_ARG, "nsample must be in 1..%u", NSFPS_MAX_NSAMPLE);
  std::vector<uint32_t> poff, coff;
  int rc = rel_offsets(point_offsets, count, "point_offsets", poff);
  if (rc) return rc;
  rc = rel_offsets(center_offsets, count, "center_offsets", coff);
  if (rc) return rc;
  if ((poff[count] && !d_xyz) || (coff[count] && (!d_centers || !d_idx)))
    return set_error(NSFPS_ERR_ARG, "NULL argument");
  int dev = 0;
  NSFPS_CUDA(cudaGetDevice(&dev));
  DeviceCtx *ctx = nullptr;
  rc = get_ctx(dev, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (d_xyz) d_xyz += 3 * point_offsets[0];
  if (d_centers) d_centers += 3 * center_offsets[0];
  return ball_query_on(ctx, (cudaStream_t)stream, d_xyz, poff, d_centers, coff, radius, nsample,
                       d_idx, d_hits);
}

int nsfps_ball_query(const float *xyz, uint64_t n, const float *centers, uint64_t m,
                     float radius, uint32_t nsample, int64_t *idx, uint32_t *hits, int device) {
  clear_error();
  if (nsample == 0 || nsample > NSFPS_MAX_NSAMPLE)
    return set_error(NSFPS_ERR_ARG, "nsample must be in 1..%u", NSFPS_MAX_NSAMPLE);
  if (m == 0) return NSFPS_OK;
  if ((n && !xyz) || !centers || !idx) return set_error(NSFPS_ERR_ARG, "NULL argument");
  if (n >= (1ull << 31) || m >= (1ull << 31))
    return set_error(NSFPS_ERR_UNSUPPORTED, "too many points or centres (>= 2^31)");
  DeviceCtx *ctx = nullptr;
  int rc = get_ctx(device, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  NSFPS_CUDA(cudaSetDevice(device));
  cudaStream_t st = ctx->stream;
  const size_t bx = sizeof(float) * 3 * std::max<uint64_t>(n, 1);
  const size_t bc = sizeof(float) * 3 * m, bi = sizeof(int64_t) * m * nsample,
               bh = sizeof(uint32_t) * m;
  void *io = nullptr;
  NSFPS_CUDA(cudaMallocAsync(&io, align_up(bx, 256) + align_up(bc, 256) + align_up(bi, 256) + bh, st));
  char *p = (char *)io;
  float *d_xyz = (float *)p;
  float *d_c = (float *)(p + align_up(bx, 256));
  int64_t *d_idx = (int64_t *)(p + align_up(bx, 256) + align_up(bc, 256));
  uint32_t *d_hits = (uint32_t *)(p + align_up(bx, 256) + align_up(bc, 256) + align_up(bi, 256));
  std::vector<uint32_t> poff = {0u, (uint32_t)n}, coff = {0u, (uint32_t)m};
  rc = NSFPS_OK;
  cudaError_t e = cudaSuccess;
  if (n) e = cudaMemcpyAsync(d_xyz, xyz, sizeof(float) * 3 * n, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(d_c, centers, bc, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) {
    rc = set_error(NSFPS_ERR_CUDA, "copy to the device failed: %s", cudaGetErrorString(e));
  } else {
    rc = ball_query_on(ctx, st, d_xyz, poff, d_c, coff, radius, nsample, d_idx, d_hits);
  }
  if (rc == NSFPS_OK) {
    e = cudaMemcpyAsync(idx, d_idx, bi, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && hits) e = cudaMemcpyAsync(hits, d_hits, bh, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess)
      rc = set_error(NSFPS_ERR_CUDA, "copy to the host failed: %s", cudaGetErrorString(e));
  }
  cudaFreeAsync(io, st);
  cudaStreamSynchronize(st);
  return rc;
}

int nsfps_gather_points_device(const float *d_xyz, const uint64_t *point_offsets,
                               const int64_t *d_idx, const uint64_t *idx_offsets, uint64_t count,
                               float *d_out, void *stream) {
  clear_error();
  if (count == 0) return NSFPS_OK;
  if (!point_offsets || !idx_offsets) return set_error(NSFPS_ERR_ARG, "NULL offsets");
  std::vector<uint32_t> poff, ioff;
  int rc = rel_offsets(point_offsets, count, "point_offsets", poff);
  if (rc) return rc;
  rc = rel_offsets(idx_offsets, count, "idx_offsets", ioff);
  if (rc) return rc;
  if (ioff[count] && (!d_xyz || !d_idx || !d_out)) return set_error(NSFPS_ERR_ARG, "NULL argument");
  int dev = 0;
  NSFPS_CUDA(cudaGetDevice(&dev));
  DeviceCtx *ctx = nullptr;
  rc = get_ctx(dev, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (d_xyz) d_xyz += 3 * point_offsets[0];
  return gather_on(ctx, (cudaStream_t)stream, d_xyz, poff, nullptr, ioff, 1, d_idx, d_out);
}

int nsfps_group_points_device(const float *d_xyz, const uint64_t *point_offsets,
                              const float *d_centers, const uint64_t *center_offsets,
                              uint64_t count, uint32_t nsample, const int64_t *d_idx,
                              float *d_out, void *stream) {
  clear_error();
  if (count == 0) return NSFPS_OK;
  if (!point_offsets || !center_offsets) return set_error(NSFPS_ERR_ARG, "NULL offsets");
  if (nsample == 0 || nsample > NSFPS_MAX_NSAMPLE)
    return set_error(NSFPS_ERR_ARG, "nsample must be in 1..%u", NSFPS_MAX_NSAMPLE);
  std::vector<uint32_t> poff, coff;
  int rc = rel_offsets(point_offsets, count, "point_offsets", poff);
  if (rc) return rc;
  rc = rel_offsets(center_offsets, count, "center_offsets", coff);
  if (rc) return rc;
  if (coff[count] && (!d_xyz || !d_centers || !d_idx || !d_out))
    return set_error(NSFPS_ERR_ARG, "NULL argument");
  int dev = 0;
  NSFPS_CUDA(cudaGetDevice(&dev));
  DeviceCtx *ctx = nullptr;
  rc = get_ctx(dev, &ctx);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (d_xyz) d_xyz += 3 * point_offsets[0];
  if (d_centers) d_centers += 3 * center_offsets[0];
  return gather_on(ctx, (cudaStream_t)stream, d_xyz, poff, d_centers, coff, nsample, d_idx,
                   d_out);
}

int nsfps_set_test_hooks(const nsfps_test_hooks *h) {
  clear_error();
  if (!h) {
    g_wait_ns.store(kDefaultWaitNs);
    g_hold_cta.store(-1);
    g_hold_step.store(0);
    g_fail_alloc.store(-1);
    return NSFPS_OK;
  }
  if (h->wait_limit_ns > (uint64_t)kDefaultWaitNs * 30)
    return set_error(NSFPS_ERR_ARG, "wait_limit_ns above 60 s");
  g_wait_ns.store(h->wait_limit_ns ? (long long)h->wait_limit_ns : kDefaultWaitNs);
  g_hold_cta.store(h->withhold_cta < 0 ? -1 : h->withhold_cta);
  g_hold_step.store(h->withhold_step);
  g_fail_alloc.store(h->fail_alloc_device < 0 ? -1 : h->fail_alloc_device);
  return NSFPS_OK;
}

int nsfps_set_profiling(int enable) {
  g_profiling.store(enable ? 1 : 0);
  return NSFPS_OK;
}

int nsfps_last_profile(nsfps_profile *out) {
  if (!out) return set_error(NSFPS_ERR_ARG, "out is NULL");
  *out = g_prof;
  return NSFPS_OK;
}

}  // extern "C"
