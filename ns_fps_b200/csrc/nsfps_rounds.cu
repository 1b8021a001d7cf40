// nsfps_rounds.cu -- the sampling loop in exchange rounds (grids whose
// buckets are their cells).
//
// Placement is the one of nsfps_loop.cu: the leaves of a cloud are dealt
// round-robin to its P CTAs (one thread-block cluster); a CTA keeps its
// leaves' points in shared memory for the whole loop and every thread keeps
// its leaves' cell, box, count and current maximum in registers.
//
// Rounds.  The reference takes one sample per step: the global farthest point
// (largest distance, smallest sorted position), then min(old, d) over every
// point of the buckets in the sample's cell cube (src/yuezu_fps.cpp:703-722).
// Exchanging per-CTA maxima every step costs one cluster round trip per
// sample.  Instead, at the start of a round every CTA publishes its T
// farthest points (exact coordinates, distance, position, cell) and the key
// of its (T+1)-th farthest point, its bound B.  Every point a CTA did not
// list has a key below its B, and keys only decrease.  So as long as the
// best listed candidate beats B* = max over CTAs of B, it is the reference's
// next sample: every CTA can replay the reference's step on the P*T
// candidates alone -- pick the winner, build its cell cube, apply min(old, d)
// to the candidates inside the cube, with the same arithmetic as the leaves --
// and decide sample after sample without any communication.  The round ends
// when the best candidate no longer beats B* (or k samples / the queue is
// reached); then every CTA applies the round's samples, in order, to its own
// leaves and publishes new lists.  Each CTA replays the same deterministic
// sequence, so all agree on every sample and on when to stop.
//
// A round, per CTA:
//   1. top-(T+1) points: each worker warp picks its T+1 best leaves by leaf
//      maximum; warp 0 merges them to the CTA's T+1 best leaves (the T+1
//      best points lie in those leaves), gathers their points and selects
//      the T+1 best;
//   2. a bulk copy of the T candidates and the bound into every CTA of the
//      cluster, then a wait (mbarrier) for all P lists; in the grid-wide
//      variant, lists in global memory and an arrival counter;
//   3. the two replay warps (0, 1) replay steps on the candidates, queueing
//      each decided sample (point, distance, cube, position) in shared
//      memory;
//   4. at the same time the worker warps (2..7, which own all the leaves)
//      apply the queued samples to their leaves, in order, as they appear
//      (release/acquire on a shared counter).
//
// Received lists rotate over two buffers (a CTA publishes round r+1 only
// after it has every round-r list); waits are bounded by %globaltimer.
#include <type_traits>

#include "nsfps_device.cuh"

namespace nsfps {

namespace {

// Warps 0..kReplay-1 replay the steps, each on its share of the candidates;
// the other warps own the leaves.  A build-time choice (1, 2 or 4).
#ifndef NSFPS_REPLAY_WARPS
#define NSFPS_REPLAY_WARPS 2
#endif
constexpr int kReplay = NSFPS_REPLAY_WARPS;
// Threads per CTA of this kernel (a build-time choice, a multiple of 32 up
// to 512); above 256 a thread owns at most 4 leaves (registers).
#ifndef NSFPS_ROUND_THREADS
#define NSFPS_ROUND_THREADS 256
#endif
constexpr int kRoundThreads = NSFPS_ROUND_THREADS;
constexpr int kMaxLeavesPerThread = kRoundThreads > 256 ? 4 : 8;
constexpr int kWarps = kRoundThreads / 32;
// Optionally the replay warps' partners on their SM sub-partitions (warp
// r + 4 shares its scheduler with warp r) stay idle.
#ifndef NSFPS_IDLE_PARTNER
#define NSFPS_IDLE_PARTNER 0
#endif
constexpr int kIdle = NSFPS_IDLE_PARTNER ? kReplay : 0;
constexpr int kWorkers = kRoundThreads - 32 * (kReplay + kIdle);  // leaf-owning threads
static_assert(kIdle == 0 || (kRoundThreads == 256 && kReplay <= 2), "idle partners: 8 warps");

// Index of a leaf-owning warp among the workers; -1 for replay and idle warps.
__device__ __forceinline__ int worker_index(int warp) {
  if (warp < kReplay) return -1;
  if (kIdle && warp >= 4 && warp < 4 + kIdle) return -1;
  return warp - kReplay - ((kIdle && warp >= 4 + kIdle) ? kIdle : 0);
}
// Candidates each CTA of a cluster or a batch group publishes per round
// (build-time choices): NSFPS_ROUND_T for parts of fewer than
// kBigPartPoints points per CTA; for larger parts NSFPS_ROUND_T_FEW when a
// cloud has at most 4 CTAs, NSFPS_ROUND_T_BIG when it has more.  Few
// candidates end a round early; many make every step and list dearer.  On
// B200, 8 / 12 / 16 per CTA gave a batch of 32 clouds of 16,384 points at 4
// CTAs each 3.373 / 3.252 / 3.225 ms per loop and 72 scans in groups of 16
// CTAs 54.05 / 51.91 / 53.14 ms, while parts of 600 to 1,250 points per CTA
// ran 1.5 to 4.6 % slower at 12 or 16 than at 8.
#ifndef NSFPS_ROUND_T
#define NSFPS_ROUND_T 8
#endif
#ifndef NSFPS_ROUND_T_BIG
#define NSFPS_ROUND_T_BIG 12
#endif
#ifndef NSFPS_ROUND_T_FEW
#define NSFPS_ROUND_T_FEW 16
#endif
constexpr int kRoundT = NSFPS_ROUND_T;
constexpr int kRoundTBig = NSFPS_ROUND_T_BIG;
constexpr int kRoundTFew = NSFPS_ROUND_T_FEW;
constexpr uint32_t kBigPartPoints = 2048;
// candidates per CTA of a large part of a cloud over P <= 16 CTAs
__host__ __device__ constexpr int big_t(uint32_t P) { return P <= 4u ? kRoundTFew : kRoundTBig; }
constexpr int kMaxPartT = (kRoundT > kRoundTBig ? kRoundT : kRoundTBig) > kRoundTFew
                              ? (kRoundT > kRoundTBig ? kRoundT : kRoundTBig)
                              : kRoundTFew;
// Candidates per round, at most (P * T): the kernel's template parameter CAP,
// 256 in a cluster and in the 64-CTA grid, 512 in the 128-CTA grid.
constexpr int kClusterCap = kRoundT * 16 > 256 ? kRoundT * 16 : 256;
// Received lists rotate over two buffers: a CTA publishes round r+2 only
// after it has every round r+1 list, so after every CTA compacted round r.
constexpr int kListBufs = 2;
// Bits of the candidate slot in a replay key, for a capacity.
__host__ __device__ constexpr int cap_slot_bits(int cap) { return cap > 256 ? 9 : 8; }
constexpr int kQueue = 512;                    // samples decided per round, at most
constexpr int kBatch = 1;                      // samples a worker applies together
// Steps decided per replay iteration, at most (see the replay loop).
#ifndef NSFPS_SPEC_STEPS
#define NSFPS_SPEC_STEPS 1
#endif
constexpr int kSpec = NSFPS_SPEC_STEPS;
static_assert((kBatch & (kBatch - 1)) == 0, "kBatch is a power of two");
static_assert(kReplay == 1 || kReplay == 2 || kReplay == 4, "1, 2 or 4 replay warps");
static_assert(kWorkers >= 64, "at least two leaf-owning warps");
// Slots of 32 leaves per CTA, at most (kMaxLeavesPerThread * kWorkers / 32).
constexpr int kMaxSlots = 64;
static_assert(kMaxLeavesPerThread * kWorkers / 32 <= kMaxSlots, "slot mask holds every slot");
// Parts of at least this many leaves per worker thread publish each sample
// with the mask of the slots its cube reaches (see the kernel).
constexpr int kMaskMinM = 4;

struct __align__(16) Cand {
  float x, y, z, d;
  uint32_t pos, cell, pad0, pad1;
};

struct Sample {
  float4 q;  // x, y, z, distance
  uint4 c;   // cube x, y, z, sorted position
};
// A queued sample with the mask of the slots its cube reaches (bit j: slot
// j), for parts of kMaskMinM or more leaves per worker thread.
struct MaskedSample {
  float4 q;
  uint4 c;
  uint32_t hit[2];
  uint32_t pad[2];
};

// One CTA's published list: its T farthest points and its bound.  Copied as
// one block into every CTA of the cluster.
template <int T>
struct __align__(16) CtaList {
  Cand c[T];
  unsigned long long bound;
  unsigned long long pad;
};

template <int T, int CAP>
struct RoundCtl {
  CtaList<T> list[kListBufs][kMaxClusterP];  // received lists, by source CTA
  CtaList<T> stage;                      // this CTA's list, copied out from here
  Cand live[CAP];                        // the round's candidates that beat B*
  uint32_t nlive[kReplay];
  unsigned long long mbar[kListBufs];
  unsigned long long wkey[kWarps][T + 1];   // per-warp best leaves
  uint32_t wleaf[kWarps][T + 1];
  uint32_t mleaf[T + 1];                    // the CTA's T+1 best leaves
  unsigned long long xkey[2][kReplay][kSpec];  // per replay warp best keys, by parity
  uint32_t scan[33];
  uint2 sbox[kMaxSlots];  // slot-mask parts: per slot, packed lowest and highest cell
  uint32_t timed_out;  // warp 0's list wait gave up (read by the other replay warps)
  uint32_t produced;  // samples of this round queued so far (release/acquire)
  uint32_t done;      // the round's last sample is queued
  uint32_t first;     // sample index of the round's first sample
  uint32_t finished;
};

// Key of a point in the reference's order: larger distance first, then the
// smaller sorted position.  0 = no point.
__device__ __forceinline__ unsigned long long pkey(float d, uint32_t pos) {
  return ((unsigned long long)dkey(d) << 32) | (unsigned long long)(0xffffffffu - pos);
}

// In-register maximum of N keys (a tree; the array is overwritten).
template <int N>
__device__ __forceinline__ unsigned long long tree_max64(unsigned long long (&k)[N]) {
#pragma unroll
  for (int st = 1; st < N; st <<= 1)
#pragma unroll
    for (int c = 0; c + st < N; c += 2 * st) k[c] = k[c] > k[c + st] ? k[c] : k[c + st];
  return k[0];
}

// Largest 64-bit key over the warp (no owner lane needed).
__device__ __forceinline__ unsigned long long warp_max64_key(unsigned long long k) {
  const uint32_t hi = (uint32_t)(k >> 32), lo = (uint32_t)k;
  const uint32_t mh = __reduce_max_sync(kFull, hi);
  const uint32_t ml = __reduce_max_sync(kFull, hi == mh ? lo : 0u);
  return ((unsigned long long)mh << 32) | ml;
}

__device__ __forceinline__ unsigned long long max64(unsigned long long a, unsigned long long b) {
  return a > b ? a : b;
}

// True when the cube (axes packed lo | width << 16) holds no cell of the box
// [lo, hi] (packed like cells).  Empty cubes (kNoCell) miss every box.
__device__ __forceinline__ bool cube_misses(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t lo,
                                            uint32_t hi) {
  const uint32_t x0 = c0 & 0xffffu, y0 = c1 & 0xffffu, z0 = c2 & 0xffffu;
  return x0 > (hi & 1023u) || x0 + (c0 >> 16) < (lo & 1023u) ||
         y0 > ((hi >> 10) & 1023u) || y0 + (c1 >> 16) < ((lo >> 10) & 1023u) ||
         z0 > (hi >> 20) || z0 + (c2 >> 16) < (lo >> 20);
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// A candidate from a list in shared memory, or from the global list buffer
// (read at L2, past this SM's L1: the slot was rewritten by another SM).
template <bool GRID>
__device__ __forceinline__ Cand load_cand(const Cand *p) {
  if (!GRID) return *p;
  const uint4 *q = reinterpret_cast<const uint4 *>(p);
  const uint4 v0 = __ldcg(q), v1 = __ldcg(q + 1);
  Cand c;
  c.x = __uint_as_float(v0.x); c.y = __uint_as_float(v0.y); c.z = __uint_as_float(v0.z);
  c.d = __uint_as_float(v0.w);
  c.pos = v1.x; c.cell = v1.y; c.pad0 = v1.z; c.pad1 = v1.w;
  return c;
}

// Barrier of the replay warps alone (barrier 0 is __syncthreads).
__device__ __forceinline__ void replay_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(32 * kReplay) : "memory");
}

// Replay keys: the distance key above ((2^(32-S) - 1 - cloud-relative sorted
// position) << S | candidate slot), S = kSlotBits.  Ordered like pkey()
// inside one cloud (positions are unique, so the slot never decides), and the
// winner's slot and position read straight out of the key.  One cloud spans
// at most 128 CTAs of fewer than 65536 points, so the position fits in
// 32 - S >= 23 bits.
template <int S>
__device__ __forceinline__ uint32_t replay_lo(uint32_t rel_pos, uint32_t slot) {
  return ((((1u << (32 - S)) - 1u) - rel_pos) << S) | slot;
}

// GRID: the cloud's P CTAs are co-resident but not one cluster; the lists go
// through global memory (a.glist, by round parity) and a barrier over the P
// CTAs (an arrival counter in a.gbar) replaces the cluster copies and
// mbarriers.  The grid holds G groups of P CTAs (G = gridDim.x / P, all
// co-resident: a cooperative launch); group g samples clouds g, g + G,
// g + 2G, ... one after the other, each with its own list buffers and
// counter, so a batch fills every SM whatever clusters the GPU could hold.
// Without GRID, one cluster of P CTAs samples one cloud.
template <int M, int T, bool GRID, int CAP, bool BATCH = false>
__global__ void __launch_bounds__(kRoundThreads, 1)
fps_rounds_cluster(const LoopArgs a) {
  static_assert(!BATCH || GRID, "batch groups exchange through global memory");
  constexpr int THREADS = kRoundThreads;
  constexpr int kMaxCands = CAP;
  static_assert(kMaxCands <= 512, "at most 512 candidates (9-bit slots)");
  constexpr int kSlotBits = cap_slot_bits(CAP);
  constexpr int kCandPerLane = kMaxCands / (32 * kReplay);
  extern __shared__ float4 smem[];
  __shared__ RoundCtl<T, CAP> ctl;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t P = a.P;
  const uint32_t group = blockIdx.x / P;
  const uint32_t crank = blockIdx.x % P;  // == %cluster_ctarank
  const uint32_t NC = P * T;              // candidates per round
  // the group's list buffers (2 * P lists, by round parity) and arrival counter
  constexpr int kListWords = (int)(sizeof(CtaList<T>) / 16);
  uint4 *const glist = BATCH ? a.glist + (size_t)group * 2u * P * kListWords : a.glist;
  uint32_t *const gbar = BATCH ? a.gbar + group : a.gbar;

  float4 *s_pts = smem;
  float4 *s_lo = s_pts + a.max_pts;    // (lo.xyz, start | count << 16)
  float4 *s_hi = s_lo + a.max_leaves;  // (hi.xyz, cell)
  uint32_t *s_gst = reinterpret_cast<uint32_t *>(s_hi + a.max_leaves);  // global sorted start
  float *s_tab = reinterpret_cast<float *>(s_gst + ((a.max_leaves + 3u) & ~3u));
  constexpr bool kMask = M >= kMaskMinM;  // see the slot layout below
  using SampleT = std::conditional_t<kMask, MaskedSample, Sample>;
  SampleT *s_samp = reinterpret_cast<SampleT *>(s_tab + ((a.max_tab + 3u) & ~3u));

  uint32_t u_ref = 0, u_eval = 0;
  bool timed_out = false, bad_any = false;
  const long long tmo = a.timeout_ns;
  const int half = lane >> 4, j16 = lane & 15;
  // rounds this group ran on its earlier clouds: the list slot and counter
  // target of a round continue across the group's clouds
  uint32_t round_base = 0;
  for (uint32_t cloud = group;;) {
  const RangeDev &Rg = a.ranges[a.rid[cloud]];
  const uint32_t n0 = Rg.blocks[0] - 1, n1 = Rg.blocks[1] - 1, n2 = Rg.blocks[2] - 1;
  const bool fast = Rg.fast_cube != 0;
  const uint32_t l0 = a.loff[cloud], l1 = a.loff[cloud + 1];
  uint32_t nl = (l1 - l0 > crank) ? (l1 - l0 - crank + P - 1) / P : 0u;
  bool bad = nl > a.max_leaves || nl > (uint32_t)(M * kWorkers) ||
             (fast && n0 + n1 + n2 > a.max_tab) || NC > (uint32_t)kMaxCands;
  if (bad) nl = 0;
  auto gleaf = [&](uint32_t i) { return l0 + crank + P * i; };

  // ---- prologue: leaves, points and cube thresholds into shared memory
  if (fast && !bad)
    for (uint32_t i = tid; i < n0 + n1 + n2; i += THREADS) {
      const uint32_t src = i < n0 ? Rg.tab_off[0] + i
                                  : (i < n0 + n1 ? Rg.tab_off[1] + (i - n0)
                                                 : Rg.tab_off[2] + (i - n0 - n1));
      s_tab[i] = a.tabs[src];
    }
  uint32_t pts_base = 0;
  for (uint32_t base = 0; base < nl; base += THREADS) {
    const uint32_t i = base + tid;
    uint32_t cntl = 0, g = 0;
    float4 lo = make_float4(0, 0, 0, 0), hi = lo;
    if (i < nl) {
      g = gleaf(i);
      lo = a.leaf_lo[g];
      hi = a.leaf_hi[g];
      cntl = __float_as_uint(lo.w) & 0xffu;
    }
    uint32_t tot = 0;
    const uint32_t ex = block_excl_sum<THREADS>(cntl, ctl.scan, tot);
    if (i < nl) {
      const uint32_t lstart = pts_base + ex;
      if (lstart + cntl <= a.max_pts && lstart < 65536u) {
        s_lo[i] = make_float4(lo.x, lo.y, lo.z, __uint_as_float(lstart | (cntl << 16)));
        const uint32_t gs = a.leaf_start[g];
        for (uint32_t j = 0; j < cntl; ++j) s_pts[lstart + j] = a.pts[gs + j];
      }
      s_hi[i] = hi;  // hi.w = cell
      s_gst[i] = a.leaf_start[g];
    }
    pts_base += tot;
  }
  if (pts_base > a.max_pts || pts_base > 65536u) {  // never with a correct plan
    bad = true;
    nl = 0;
  }
  __syncthreads();

  AxisK ax[3];
#pragma unroll
  for (int d = 0; d < 3; ++d) {
    ax[d].mn = Rg.mn[d];
    ax[d].hi = Rg.hi[d];
    ax[d].inv = Rg.inv_bs[d];
    ax[d].ovf = Rg.ovf[d];
    ax[d].bsz = Rg.bsz[d];
    ax[d].blocks = (int)Rg.blocks[d];
  }
  ax[0].tab = s_tab;
  ax[1].tab = s_tab + n0;
  ax[2].tab = s_tab + n0 + n1;
  // Axes of at most 64 thresholds are held across the replay warp's lanes
  // (entries lane and lane + 32): the cube half-width n_a is the number of
  // thresholds below D (they increase with n), one ballot per 32 entries.
  const bool regtab = fast && n0 <= 64u && n1 <= 64u && n2 <= 64u;
  float rt[3][2];
#pragma unroll
  for (int d = 0; d < 3; ++d) {
    const uint32_t top = d == 0 ? n0 : (d == 1 ? n1 : n2);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t i = (uint32_t)lane + 32u * h;
      rt[d][h] = (regtab && i < top) ? ax[d].tab[i] : __int_as_float(0x7f800000);
    }
  }

  // per owned leaf, in registers.  The replay warps own no leaf.  The local
  // leaves (Morton order) form slots of 32 consecutive leaves.
  //  * Parts of fewer than kMaskMinM leaves per worker thread: worker warp w
  //    (kReplay..) owns the `span` consecutive local leaves from
  //    (w - kReplay) * span, a spatially compact run; its lane's m-th leaf is
  //    leaf m * 32 + lane of the run.  Each worker tests every sample's cube
  //    against its run's cell box and its slots' boxes.
  //  * Larger parts (kMask): slot j belongs to worker warp j % W as its
  //    (j / W)-th, so a sample's cube (a few consecutive slots) spreads its
  //    leaf updates over the worker warps, and the replay warps test the
  //    cube against every slot's box once, publishing the mask of the slots
  //    it reaches with the sample; a worker skips a sample that reaches none
  //    of its slots after one load.  Measured on parts of 6 leaves per
  //    thread (c4, c5) this trims the workers' backlog at each round's end;
  //    on small parts the replay warps' extra test costs more than it saves.
  constexpr uint32_t kWorkerWarps = (uint32_t)kWorkers / 32u;
  const uint32_t span = (nl + kWorkerWarps - 1u) / kWorkerWarps;
  const int widx = worker_index(warp);
  const uint32_t wbase = widx >= 0 ? (uint32_t)widx * span : 0u;
  auto lidx = [&](int m, uint32_t ln) {
    return kMask ? ((uint32_t)m * kWorkerWarps + (uint32_t)(widx >= 0 ? widx : 0)) * 32u + ln
                 : wbase + (uint32_t)m * 32u + ln;
  };
  auto owned = [&](int m, uint32_t ln) {
    if (kMask) return widx >= 0 && lidx(m, ln) < nl;
    const uint32_t r = (uint32_t)m * 32u + ln;
    return widx >= 0 && r < span && wbase + r < nl;
  };
  const uint32_t nslots = (nl + 31u) / 32u;
  uint32_t cell[M], cnt[M], gst[M], gpos[M], sbox_lo[M], sbox_hi[M];
  uint32_t lsc[M];  // shared-memory start | count << 16
  float lmax[M], bx0[M], by0[M], bz0[M], bx1[M], by1[M], bz1[M];
  uint32_t wx0 = 1023u, wy0 = 1023u, wz0 = 1023u, wx1 = 0u, wy1 = 0u, wz1 = 0u;
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const uint32_t i = lidx(m, (uint32_t)lane);
    if (owned(m, lane)) {
      const uint32_t g = gleaf(i);
      const float4 lo = a.leaf_lo[g], hi = a.leaf_hi[g];
      const uint32_t w = __float_as_uint(lo.w);
      const uint32_t slot = (w >> 8) & 0xffu;
      cell[m] = __float_as_uint(hi.w);
      cnt[m] = w & 0xffu;
      lsc[m] = (__float_as_uint(s_lo[i].w) & 0xffffu) | (cnt[m] << 16);
      gst[m] = a.leaf_start[g];
      lmax[m] = a.leaf_md[g];
      gpos[m] = gst[m] + slot;
      bx0[m] = lo.x; by0[m] = lo.y; bz0[m] = lo.z;
      bx1[m] = hi.x; by1[m] = hi.y; bz1[m] = hi.z;
    } else {
      cell[m] = 0xffffffffu;  // z field 4095: outside every cube
      cnt[m] = 0;
      lsc[m] = 0u;
      gst[m] = 0;
      lmax[m] = -1.0f;
      gpos[m] = 0xffffffffu;
      bx0[m] = by0[m] = bz0[m] = 0.0f;
      bx1[m] = by1[m] = bz1[m] = 0.0f;
    }
    uint32_t x0 = 1023u, y0 = 1023u, z0 = 1023u, x1 = 0u, y1 = 0u, z1 = 0u;
    if (owned(m, lane)) {
      x0 = x1 = cell[m] & 1023u;
      y0 = y1 = (cell[m] >> 10) & 1023u;
      z0 = z1 = cell[m] >> 20;
    }
    x0 = __reduce_min_sync(kFull, x0); y0 = __reduce_min_sync(kFull, y0);
    z0 = __reduce_min_sync(kFull, z0); x1 = __reduce_max_sync(kFull, x1);
    y1 = __reduce_max_sync(kFull, y1); z1 = __reduce_max_sync(kFull, z1);
    sbox_lo[m] = pack_cell(x0, y0, z0);
    sbox_hi[m] = pack_cell(x1, y1, z1);
    if (kMask && widx >= 0 && lane == 0) {
      const uint32_t j = (uint32_t)m * kWorkerWarps + (uint32_t)widx;
      if (j < nslots) ctl.sbox[j] = make_uint2(sbox_lo[m], sbox_hi[m]);
    }
    wx0 = min(wx0, x0); wy0 = min(wy0, y0); wz0 = min(wz0, z0);
    wx1 = max(wx1, x1); wy1 = max(wy1, y1); wz1 = max(wz1, z1);
  }
  const uint32_t wbox_lo = pack_cell(wx0, wy0, wz0), wbox_hi = pack_cell(wx1, wy1, wz1);

  const uint32_t tx_bytes = P * (uint32_t)sizeof(CtaList<T>);
  if (tid == 0) {
    if (!BATCH) {  // (a batch group re-enters here per cloud; it uses no mbarrier)
      for (int b = 0; b < kListBufs; ++b) mbar_init(smem_u32(&ctl.mbar[b]), 1);
      fence_mbar_init();
      for (int b = 0; b < kListBufs; ++b) mbar_arm(smem_u32(&ctl.mbar[b]), tx_bytes);
    }
    ctl.finished = 0;
  }
  __syncthreads();
  if (!BATCH) cluster_sync_all();  // every CTA's mbarriers are armed before any remote write

  // kMask: every replay lane holds the cell boxes of slots lane and 32 + lane
  // (unpacked: x0, x1, y0, y1, z0, z1), for the mask words 0 and 1
  uint32_t rsb[2][6];
  bool rs_ok[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t j = 32u * (uint32_t)h + (uint32_t)lane;
    rs_ok[h] = kMask && warp < kReplay && j < nslots;
    const uint2 bx = rs_ok[h] ? ctl.sbox[j] : make_uint2(0u, 0u);
    rsb[h][0] = bx.x & 1023u; rsb[h][1] = bx.y & 1023u;
    rsb[h][2] = (bx.x >> 10) & 1023u; rsb[h][3] = (bx.y >> 10) & 1023u;
    rsb[h][4] = bx.x >> 20; rsb[h][5] = bx.y >> 20;
  }

  uint32_t it = 1;           // next sample index (sample 0 is point 0)

  // ---- apply queued samples s0 .. s0+nb-1 (nb <= kBatch) to this worker's
  // leaves.  Each point takes min(old, d) over the samples whose cube holds its
  // cell -- the reference's per-step updates, whose result does not depend on
  // their order.  A sample whose cube misses the warp's cell box, or a slot's,
  // is skipped for all of it; a leaf is skipped for a sample when the
  // sample's distance to the leaf box is not below the leaf maximum from
  // before the batch (no smaller than the current one, so the skip is exact).
  auto apply = [&](uint32_t s0, uint32_t nb) {
    float qx[kBatch], qy[kBatch], qz[kBatch];
    uint32_t c0[kBatch], c1[kBatch], c2[kBatch];
    uint32_t live = 0u;
    // slots whose cell box the cubes reach (uniform over the warp)
    uint32_t act[M];
#pragma unroll
    for (int m = 0; m < M; ++m) act[m] = 0u;
    if constexpr (kMask) {
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const bool on = (uint32_t)j < nb;
        const uint2 hw = on ? *reinterpret_cast<const uint2 *>(s_samp[s0 + j].hit) : make_uint2(0u, 0u);
        const unsigned long long mine = (((unsigned long long)hw.y << 32) | hw.x) >> widx;
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const uint32_t b = (uint32_t)(mine >> ((uint32_t)m * kWorkerWarps)) & 1u;
          act[m] |= b << j;
          live |= b << j;
        }
      }
      if (live == 0u) return;
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const bool on = (uint32_t)j < nb && (!kMask || ((live >> j) & 1u) != 0u);
      const float4 q = on ? s_samp[s0 + j].q : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      const uint4 cb = on ? s_samp[s0 + j].c : make_uint4(kNoCell, kNoCell, kNoCell, 0u);
      qx[j] = q.x; qy[j] = q.y; qz[j] = q.z;
      c0[j] = cb.x; c1[j] = cb.y; c2[j] = cb.z;
      if (!kMask) live |= cube_misses(cb.x, cb.y, cb.z, wbox_lo, wbox_hi) ? 0u : (1u << j);
    }
    if (!kMask) {
      if (live == 0u) return;
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
          act[m] |= (((live >> j) & 1u) &&
                     !cube_misses(c0[j], c1[j], c2[j], sbox_lo[m], sbox_hi[m])) ? (1u << j) : 0u;
    }
    uint32_t needb[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
      needb[m] = 0u;
      if (act[m] == 0u) continue;
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const bool hit = ((act[m] >> j) & 1u) && in_box(cell[m], c0[j], c1[j], c2[j]);
        // distance from the sample to the leaf box, per axis (0 inside)
        const float gx = fmaxf(fmaxf(__fsub_rn(bx0[m], qx[j]), __fsub_rn(qx[j], bx1[m])), 0.0f);
        const float gy = fmaxf(fmaxf(__fsub_rn(by0[m], qy[j]), __fsub_rn(qy[j], by1[m])), 0.0f);
        const float gz = fmaxf(fmaxf(__fsub_rn(bz0[m], qz[j]), __fsub_rn(qz[j], bz1[m])), 0.0f);
        const float lbd =
            __fadd_rn(__fadd_rn(__fmul_rn(gx, gx), __fmul_rn(gy, gy)), __fmul_rn(gz, gz));
        const bool need = hit && lbd < lmax[m];
        u_ref += hit ? cnt[m] : 0u;
        needb[m] |= need ? (1u << j) : 0u;
      }
    }
    uint32_t mk[M];
#pragma unroll
    for (int m = 0; m < M; ++m) mk[m] = __ballot_sync(kFull, needb[m] != 0u);
#pragma unroll
    for (int m = 0; m < M; ++m) {
      uint32_t mask = mk[m];
      while (mask) {
        const int la = __ffs(mask) - 1;
        mask &= mask - 1;
        int lb2 = -1;
        if (mask) {
          lb2 = __ffs(mask) - 1;
          mask &= mask - 1;
        }
        // half-warp h updates leaf la (h = 0) or lb2 (h = 1), a point per
        // lane; the owner's start, count and sample bits come in one shuffle
        const int src = half ? lb2 : la;
        const uint32_t word =
            __shfl_sync(kFull, lsc[m] | (needb[m] << 24), src < 0 ? la : src);
        const uint32_t start = word & 0xffffu, c = (word >> 16) & 0xffu, nbits = word >> 24;
        const bool on = src >= 0 && (uint32_t)j16 < c;
        const uint32_t pi = start + (on ? (uint32_t)j16 : 0u);  // inside the leaf
        // points evaluated: one per lane of the pass and sample it takes (the
        // count in the leaf tests above cost the c3 / c4 / c5 loops 5-7 %)
        if constexpr (kBatch == 1) u_eval += on ? 1u : 0u;
        else u_eval += on ? (uint32_t)__popc(nbits) : 0u;
        const float4 p = s_pts[pi];
        float w = p.w;
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const float d = sqdist(p.x, p.y, p.z, qx[j], qy[j], qz[j]);
          w = (((nbits >> j) & 1u) && d < w) ? d : w;
        }
        if (on && w < p.w) s_pts[pi].w = w;
        const uint32_t key = on ? dkey(w) : 0u;
        const uint32_t kA = __reduce_max_sync(kFull, half ? 0u : key);
        const uint32_t kB = __reduce_max_sync(kFull, half ? key : 0u);
        const uint32_t fA = __ffs(__ballot_sync(kFull, !half && key == kA)) - 1;
        const uint32_t fB = __ffs(__ballot_sync(kFull, half && key == kB)) - 17;
        if (lane == la) {
          lmax[m] = __uint_as_float(kA - 1u);
          gpos[m] = gst[m] + fA;
        }
        if (lane == lb2) {
          lmax[m] = __uint_as_float(kB - 1u);
          gpos[m] = gst[m] + fB;
        }
      }
    }
  };

  uint32_t out_n = 0, out_first = 0;  // the round's samples (worker warps)
  uint32_t round = 0;
  for (;; ++round) {
    const uint32_t buf = round & (kListBufs - 1);
    // the group's round (list slot, counter target), numbered on across a
    // batch group's clouds
    const uint32_t grnd = BATCH ? round_base + round : round;

    // ---- 1a. each worker warp: its T+1 best leaves by leaf maximum, in
    // order (keys are unique: every leaf has its own sorted position)
    if (widx >= 0) {
      unsigned long long lk[M];
      int rk[M];
#pragma unroll
      for (int m = 0; m < M; ++m) {
        lk[m] = pkey(lmax[m], gpos[m]);  // 0 for a leaf this lane does not own
        rk[m] = -1;
      }
      if (lane <= T) ctl.wkey[widx][lane] = 0ull;
#pragma unroll 1
      for (int t = 0; t <= T; ++t) {
        unsigned long long tk[M];
#pragma unroll
        for (int m = 0; m < M; ++m) tk[m] = lk[m];
        const unsigned long long wk = warp_max64_key(tree_max64(tk));
        if (wk == 0ull) break;
#pragma unroll
        for (int m = 0; m < M; ++m)
          if (lk[m] == wk) { lk[m] = 0ull; rk[m] = t; }
      }
      __syncwarp();
#pragma unroll
      for (int m = 0; m < M; ++m)
        if (rk[m] >= 0) {
          ctl.wkey[widx][rk[m]] = pkey(lmax[m], gpos[m]);
          ctl.wleaf[widx][rk[m]] = lidx(m, (uint32_t)lane);
        }
    } else if (warp == 0 && lane == 0) {
      ctl.produced = 0u;
      ctl.done = 0u;
      ctl.first = it;
    }
    __syncthreads();

    // ---- 1b/2/3. warp 0: list and exchange; the replay warps: replay; the
    // workers apply the samples as they are queued
    if (warp < kReplay) {
      if (warp == 0) {
        // merge the worker warps' lists ((W - kReplay) * (T+1) entries)
        constexpr int NE = (kWorkers / 32) * (T + 1);
        constexpr int E = (NE + 31) / 32;
        unsigned long long ek[E];
        uint32_t el[E];
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int idx = lane + 32 * e;
          ek[e] = idx < NE ? ctl.wkey[idx / (T + 1)][idx % (T + 1)] : 0ull;
          el[e] = idx < NE ? ctl.wleaf[idx / (T + 1)][idx % (T + 1)] : 0u;
        }
        int er[E];
#pragma unroll
        for (int e = 0; e < E; ++e) er[e] = -1;
        uint32_t nleaf = 0;
#pragma unroll 1
        for (int t = 0; t <= T; ++t) {
          unsigned long long tk[E];
#pragma unroll
          for (int e = 0; e < E; ++e) tk[e] = ek[e];
          const unsigned long long wk = warp_max64_key(tree_max64(tk));
          if (wk == 0ull) break;
#pragma unroll
          for (int e = 0; e < E; ++e)
            if (ek[e] == wk) { ek[e] = 0ull; er[e] = t; }
          ++nleaf;
        }
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (er[e] >= 0) ctl.mleaf[er[e]] = el[e];
        __syncwarp();
        // gather the points of those leaves; half-warp h takes leaf 2r + h
        constexpr int G = (T + 2) / 2;  // points held per lane
        unsigned long long gk[G];
        float4 gp[G];
        uint32_t gc[G], gq[G];
#pragma unroll
        for (int r = 0; r < G; ++r) {
          const uint32_t li = 2u * r + (uint32_t)half;
          gk[r] = 0ull;
          gp[r] = make_float4(0, 0, 0, -1.0f);
          gc[r] = 0u;
          gq[r] = 0xffffffffu;
          if (li < nleaf) {
            const uint32_t leaf = ctl.mleaf[li];
            const uint32_t lw = __float_as_uint(s_lo[leaf].w);
            const uint32_t start = lw & 0xffffu, c = lw >> 16;
            if ((uint32_t)j16 < c) {
              gp[r] = s_pts[start + j16];
              gc[r] = __float_as_uint(s_hi[leaf].w);
              // sorted position: the leaf's global start + slot
              gq[r] = s_gst[leaf] + (uint32_t)j16;
              gk[r] = pkey(gp[r].w, gq[r]);
            }
          }
        }
        // the T+1 best points: the first T are the list, the next is the bound
        unsigned long long bound = 0ull;
        int gr[G];
#pragma unroll
        for (int r = 0; r < G; ++r) gr[r] = -1;
        uint32_t nsel = 0;
#pragma unroll 1
        for (int t = 0; t <= T; ++t) {
          unsigned long long tk[G];
#pragma unroll
          for (int r = 0; r < G; ++r) tk[r] = gk[r];
          const unsigned long long wk = warp_max64_key(tree_max64(tk));
          if (t == T) { bound = wk; break; }
          if (wk == 0ull) break;
#pragma unroll
          for (int r = 0; r < G; ++r)
            if (gk[r] == wk) { gk[r] = 0ull; gr[r] = t; }
          ++nsel;
        }
        // stage the list (after the previous round's copies have read it),
        // then copy it into every CTA's list[buf][crank]
        if (!GRID && (uint32_t)lane < P) bulk_wait_read_all();
        __syncwarp();
#pragma unroll
        for (int r = 0; r < G; ++r)
          if (gr[r] >= 0) {
            Cand cd;
            cd.x = gp[r].x; cd.y = gp[r].y; cd.z = gp[r].z; cd.d = gp[r].w;
            cd.pos = gq[r]; cd.cell = gc[r]; cd.pad0 = cd.pad1 = 0u;
            ctl.stage.c[gr[r]] = cd;
          }
        if ((uint32_t)lane >= nsel && lane < T) {
          Cand cd;
          cd.x = cd.y = cd.z = 0.0f;
          cd.d = -1.0f;
          cd.pos = 0xffffffffu;
          cd.cell = 0xffffffffu;
          cd.pad0 = cd.pad1 = 0u;
          ctl.stage.c[lane] = cd;
        }
        if (lane == 0) {
          ctl.stage.bound = bound;
          ctl.stage.pad = 0ull;
        }
        // test hook: one CTA of cloud 0 keeps this round's list to itself
        const bool hold = cloud == 0u && (int)crank == a.hold_cta && round == a.hold_step;
        if (!GRID) {
          fence_proxy_async_smem();
          __syncwarp();
          if ((uint32_t)lane < P && !hold) {
            const uint32_t ra = mapa(smem_u32(&ctl.list[buf][crank]), lane);
            const uint32_t rm = mapa(smem_u32(&ctl.mbar[buf]), lane);
            bulk_copy_to_cluster(ra, smem_u32(&ctl.stage), (uint32_t)sizeof(CtaList<T>), rm);
            bulk_commit();
          }

          // ---- wait for every CTA's list (bounded)
          const uint32_t mb = smem_u32(&ctl.mbar[buf]);
          const uint32_t parity = (round / kListBufs) & 1u;
          unsigned long long deadline = 0;
          uint32_t polls = 0;
          for (;;) {
            const bool ok = mbar_try_wait(mb, parity, 20000u);
            if (__all_sync(kFull, ok)) break;
            if ((++polls & 255u) == 0) {
              const unsigned long long now = globaltimer();
              if (deadline == 0) deadline = now + (unsigned long long)tmo;
              if (__shfl_sync(kFull, now > deadline ? 1 : 0, 0)) { timed_out = true; break; }
            }
          }
          // re-arm for round + kListBufs, only once this phase completed: a
          // phase that never completed has no arrival left to take, and an
          // arrive there is undefined
          if (lane == 0 && !timed_out) mbar_arm(mb, tx_bytes);
        } else {
          // ---- publish to global memory, then the group's barrier (bounded).
          // Slot (grnd & 1) is rewritten two rounds later, after every CTA of
          // the group passed the next barrier, so after every CTA read it;
          // the group's rounds are numbered on across its clouds.
          __syncwarp();
          constexpr int kWords = (int)(sizeof(CtaList<T>) / 16);
          const uint4 *src = reinterpret_cast<const uint4 *>(&ctl.stage);
          uint4 *dst = glist + ((size_t)(grnd & 1u) * P + crank) * kWords;
          if (!hold)
            for (int w = lane; w < kWords; w += 32) __stcg(dst + w, src[w]);
          __syncwarp();  // lane 0's release below covers every lane's stores
          if (lane == 0) {
            const uint32_t target = (grnd + 1u) * P;
            if (!hold) red_release_gpu_add(gbar, 1u);
            unsigned long long deadline = 0;
            uint32_t polls = 0;
            while (ld_acquire_gpu(gbar) < target) {
              if (polls >= 64u) __nanosleep(64);  // the first polls without backoff
              if ((++polls & 255u) == 0) {
                const unsigned long long now = globaltimer();
                if (deadline == 0) deadline = now + (unsigned long long)tmo;
                if (now > deadline) { timed_out = true; break; }
              }
            }
          }
          timed_out = __shfl_sync(kFull, timed_out ? 1 : 0, 0) != 0;
        }
        if (lane == 0) ctl.timed_out = timed_out ? 1u : 0u;
      }
      // every list is in and the timeout flag is set
      if (kReplay > 1) replay_sync(); else __syncwarp();

      // ---- 3. replay steps on the candidates
      uint32_t n = 0;
      bool finished = ctl.timed_out != 0u;
      if (!finished) {
        const uint32_t pbase = a.poff[cloud];
        // B* = the largest bound, in the replay key's encoding
        const CtaList<T> *lists =
            GRID ? reinterpret_cast<const CtaList<T> *>(glist) + (size_t)(grnd & 1u) * P
                 : ctl.list[buf];
        // this lane's candidates, loaded together with the bounds (one
        // round trip to L2 in the grid-wide loop)
        Cand lc[kCandPerLane];
#pragma unroll
        for (int c = 0; c < kCandPerLane; ++c) {
          const uint32_t idx = (uint32_t)(warp * 32 * kCandPerLane + 32 * c + lane);
          lc[c].d = -1.0f;
          if (idx < NC) lc[c] = load_cand<GRID>(&lists[idx / T].c[idx % T]);
        }
        unsigned long long bl = 0ull;
        for (uint32_t i = (uint32_t)lane; i < P; i += 32u) {
          unsigned long long b = GRID ? __ldcg(&lists[i].bound) : lists[i].bound;
          if (b != 0ull)
            b = (b & 0xffffffff00000000ull) | replay_lo<kSlotBits>((0xffffffffu - (uint32_t)b) - pbase, 0u);
          bl = max64(bl, b);
        }
        const unsigned long long bstar = warp_max64_key(bl);
        // Only candidates that beat B* can be chosen this round (keys only
        // decrease): compact them into ctl.live, so the steps touch no other.
        uint32_t nl_w = 0, lslot[kCandPerLane];
        bool lv[kCandPerLane];
#pragma unroll
        for (int c = 0; c < kCandPerLane; ++c) {
          lv[c] = lc[c].d >= 0.0f &&
                  (((unsigned long long)dkey(lc[c].d) << 32) | replay_lo<kSlotBits>(lc[c].pos - pbase, 0u)) > bstar;
          const uint32_t bm = __ballot_sync(kFull, lv[c]);
          lslot[c] = nl_w + __popc(bm & lanemask_lt());
          nl_w += __popc(bm);
        }
        if (lane == 0) ctl.nlive[warp] = nl_w;
        if (kReplay > 1) replay_sync(); else __syncwarp();
        uint32_t L = 0, off = 0;
#pragma unroll
        for (int w = 0; w < kReplay; ++w) {
          const uint32_t v = ctl.nlive[w];
          off += w < warp ? v : 0u;
          L += v;
        }
#pragma unroll
        for (int c = 0; c < kCandPerLane; ++c)
          if (lv[c]) ctl.live[off + lslot[c]] = lc[c];
        if (kReplay > 1) replay_sync(); else __syncwarp();
        // live candidate i sits in lane i % 32 of warp (i / 32) % kReplay, row
        // i / (32 * kReplay); rows past L are empty on every warp
        // per candidate: coordinates, its distance as a key (dkey: for the
        // non-negative distances here, integer order is float order, so
        // min(old, d) is an integer min), the low key word, its cell split
        // into axes (no candidate: key 0, cell outside every cube)
        float cx[kCandPerLane], cy[kCandPerLane], cz[kCandPerLane];
        uint32_t ck[kCandPerLane], clo[kCandPerLane];
        uint32_t gx[kCandPerLane], gy[kCandPerLane], gz[kCandPerLane];
#pragma unroll
        for (int c = 0; c < kCandPerLane; ++c) {
          const uint32_t idx = (uint32_t)(32 * kReplay * c + 32 * warp + lane);
          cx[c] = cy[c] = cz[c] = 0.0f;
          ck[c] = 0u;
          clo[c] = 0u;
          gx[c] = gy[c] = gz[c] = 0xffffu;
          if (idx < L) {
            const Cand cd = ctl.live[idx];
            cx[c] = cd.x; cy[c] = cd.y; cz[c] = cd.z;
            ck[c] = dkey(cd.d);
            clo[c] = replay_lo<kSlotBits>(cd.pos - pbase, idx);
            gx[c] = cd.cell & 1023u; gy[c] = (cd.cell >> 10) & 1023u; gz[c] = cd.cell >> 20;
          }
        }
        const uint32_t rows = (L + 32u * kReplay - 1u) / (32u * kReplay);
        // candidate pairs (rows 2h, 2h + 1) packed for the f32x2 distances
        constexpr int kPairs = kCandPerLane / 2 > 0 ? kCandPerLane / 2 : 1;
        unsigned long long px2[kPairs], py2[kPairs], pz2[kPairs];
#pragma unroll
        for (int h = 0; h < kPairs; ++h) {
          const int c0 = 2 * h, c1 = 2 * h + 1 < kCandPerLane ? 2 * h + 1 : 2 * h;
          px2[h] = f2pack(cx[c0], cx[c1]);
          py2[h] = f2pack(cy[c0], cy[c1]);
          pz2[h] = f2pack(cz[c0], cz[c1]);
        }

        // Each iteration takes the kSpec best candidates W0 > W1 > ... and
        // decides the longest prefix of them that are the reference's next
        // steps: Wj (j >= 1) is, when it beats B*, has a positive distance and
        // lies outside the cubes of W0..Wj-1 (all non-empty).  Then none of
        // those steps changes Wj's distance while each drops its own winner's
        // to 0, so after them Wj is the largest key, exactly as in the
        // reference; the candidates' updates commute (min).
        uint32_t iter = 0;
        // the loop, with the cube source fixed (no branch on it per step)
        auto replay = [&](auto use_regtab, auto nrows, auto wide_axes) {
          constexpr bool kRegTab = decltype(use_regtab)::value;
          constexpr bool kWide = decltype(wide_axes)::value;  // an axis has > 32 thresholds
          constexpr int R = decltype(nrows)::value;  // candidate rows in use
          for (;;) {
            unsigned long long wt[kSpec];  // this warp's best keys, in order
            if (kSpec == 1) {
              // the largest distance key, then among its holders the largest
              // low word: two 32-bit trees around the two warp reductions
              uint32_t th[R];
#pragma unroll
              for (int c = 0; c < R; ++c) th[c] = ck[c];
#pragma unroll
              for (int st = 1; st < R; st <<= 1)
#pragma unroll
                for (int c = 0; c + st < R; c += 2 * st) th[c] = max(th[c], th[c + st]);
              const uint32_t mh = __reduce_max_sync(kFull, th[0]);
              uint32_t tl[R];
#pragma unroll
              for (int c = 0; c < R; ++c) tl[c] = ck[c] == mh ? clo[c] : 0u;
#pragma unroll
              for (int st = 1; st < R; st <<= 1)
#pragma unroll
                for (int c = 0; c + st < R; c += 2 * st) tl[c] = max(tl[c], tl[c + st]);
              wt[0] = ((unsigned long long)mh << 32) | __reduce_max_sync(kFull, tl[0]);
            } else {
              unsigned long long kk[kCandPerLane];
#pragma unroll
              for (int c = 0; c < kCandPerLane; ++c)
                kk[c] = c < R ? (((unsigned long long)ck[c] << 32) | clo[c]) : 0ull;
#pragma unroll
              for (int j = 0; j < kSpec; ++j) {
                unsigned long long tk[kCandPerLane];
#pragma unroll
                for (int c = 0; c < kCandPerLane; ++c) tk[c] = kk[c];
                wt[j] = warp_max64_key(tree_max64(tk));
#pragma unroll
                for (int c = 0; c < kCandPerLane; ++c) kk[c] = kk[c] == wt[j] ? 0ull : kk[c];
              }
            }
            if (kReplay > 1) {  // the best over the replay warps
              const uint32_t par = iter & 1u;
              // every lane stores the same keys: no divergent branch
#pragma unroll
              for (int j = 0; j < kSpec; ++j) ctl.xkey[par][warp][j] = wt[j];
              replay_sync();
              unsigned long long all[kReplay * kSpec];
#pragma unroll
              for (int w = 0; w < kReplay; ++w)
#pragma unroll
                for (int j = 0; j < kSpec; ++j) all[w * kSpec + j] = ctl.xkey[par][w][j];
#pragma unroll
              for (int j = 0; j < kSpec; ++j) {
                unsigned long long tk[kReplay * kSpec];
#pragma unroll
                for (int e = 0; e < kReplay * kSpec; ++e) tk[e] = all[e];
                wt[j] = tree_max64(tk);
#pragma unroll
                for (int e = 0; e < kReplay * kSpec; ++e) all[e] = all[e] == wt[j] ? 0ull : all[e];
              }
            }
            ++iter;
            float wd[kSpec];
#pragma unroll
            for (int j = 0; j < kSpec; ++j)
              wd[j] = __uint_as_float((uint32_t)(wt[j] >> 32) - 1u);  // current distance
            // stop when some unlisted point may win (not certain), or when the
            // best distance is 0 (src/yuezu_fps.cpp:705-706)
            // one exit test per step: k samples taken, the queue full, some
            // unlisted point may win (not certain), or the best distance is 0
            // (src/yuezu_fps.cpp:705-706); only the first and the last end
            // the sampling
            const bool more = it < a.k && n < (uint32_t)kQueue;
            if (!(more && wt[0] > bstar && wd[0] > 0.0f)) {
              finished = it >= a.k || (more && wt[0] > bstar);
              break;
            }
            float wx[kSpec], wy[kSpec], wz[kSpec];
            uint32_t wcell[kSpec], wcube[kSpec][3];
#pragma unroll
            for (int j = 0; j < kSpec; ++j) {
              const Cand &qcd = ctl.live[(uint32_t)wt[j] & ((1u << kSlotBits) - 1u)];
              const float4 qv = *reinterpret_cast<const float4 *>(&qcd.x);
              wx[j] = qv.x; wy[j] = qv.y; wz[j] = qv.z;
              wcell[j] = qcd.cell;
            }
#pragma unroll
            for (int j = 0; j < kSpec; ++j) {
              const float qd = wd[j];
              const uint32_t qc[3] = {wcell[j] & 1023u, (wcell[j] >> 10) & 1023u, wcell[j] >> 20};
              if (kRegTab) {
                const bool empty = qd > ax[0].ovf || qd > ax[1].ovf || qd > ax[2].ovf;
#pragma unroll
                for (int d = 0; d < 3; ++d) {
                  int nh = __popc(__ballot_sync(kFull, qd > rt[d][0]));
                  if (kWide) nh += __popc(__ballot_sync(kFull, qd > rt[d][1]));  // entries 32..63
                  const int top = ax[d].blocks - 1;
                  const int l = (int)qc[d] - nh > 0 ? (int)qc[d] - nh : 0;
                  const int h = (int)qc[d] + nh < top ? (int)qc[d] + nh : top;
                  wcube[j][d] = empty ? kNoCell : ((uint32_t)l | ((uint32_t)(h - l) << 16));
                }
              } else {
                cube_of(ax, fast, qc, qd, wcube[j]);
              }
            }
            // the accepted prefix W0 .. W(m-1)
            uint32_t m = 1;
            bool ok = true;
#pragma unroll
            for (int j = 1; j < kSpec; ++j) {
              ok = ok && wt[j] > bstar && wd[j] > 0.0f && it + (uint32_t)j < a.k &&
                   n + (uint32_t)j < (uint32_t)kQueue;
#pragma unroll
              for (int i = 0; i < j; ++i)
                ok = ok && wcube[i][0] != kNoCell &&
                     !in_box(wcell[j], wcube[i][0], wcube[i][1], wcube[i][2]);
              m += ok ? 1u : 0u;
            }
            {  // queue the samples (every lane of every replay warp stores the same values)
#pragma unroll
              for (int j = 0; j < kSpec; ++j)
                if ((uint32_t)j < m) {
                  SampleT sm;
                  sm.q = make_float4(wx[j], wy[j], wz[j], wd[j]);
                  sm.c = make_uint4(wcube[j][0], wcube[j][1], wcube[j][2],
                                    pbase + (((1u << (32 - kSlotBits)) - 1u) - ((uint32_t)wt[j] >> kSlotBits)));
                  if constexpr (kMask) {  // the slots whose cell box the cube reaches
                    uint32_t cl[3], ch[3];  // the cube's cell range (empty: lo 0xffff)
#pragma unroll
                    for (int d = 0; d < 3; ++d) {
                      cl[d] = wcube[j][d] & 0xffffu;
                      ch[d] = cl[d] + (wcube[j][d] >> 16);
                    }
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                      sm.hit[h] = __ballot_sync(
                          kFull, rs_ok[h] && cl[0] <= rsb[h][1] && ch[0] >= rsb[h][0] &&
                                     cl[1] <= rsb[h][3] && ch[1] >= rsb[h][2] &&
                                     cl[2] <= rsb[h][5] && ch[2] >= rsb[h][4]);
                    sm.pad[0] = sm.pad[1] = 0u;
                  }
                  s_samp[n + j] = sm;
                }
              st_release_cta_if(warp == 0 && lane == 0, &ctl.produced, n + m);  // workers may apply them
            }
#pragma unroll
            for (int j = 0; j < kSpec; ++j)
              if ((uint32_t)j < m) {
                // the candidates' distances to the sample, two at a time
                // (sm_100 f32x2, bit-identical to sqdist())
                float pd[R];
                if (R >= 2) {
                  const unsigned long long qx2 = f2pack(wx[j], wx[j]), qy2 = f2pack(wy[j], wy[j]),
                                           qz2 = f2pack(wz[j], wz[j]);
#pragma unroll
                  for (int h = 0; h < R / 2; ++h)
                    f2unpack(sqdist_x2(px2[h], py2[h], pz2[h], qx2, qy2, qz2), pd[2 * h],
                             pd[2 * h + 1]);
                  if (R & 1)  // an odd last row
                    pd[R - 1] = sqdist(cx[R - 1], cy[R - 1], cz[R - 1], wx[j], wy[j], wz[j]);
                } else {
                  pd[0] = sqdist(cx[0], cy[0], cz[0], wx[j], wy[j], wz[j]);
                }
#pragma unroll
                for (int c = 0; c < R; ++c) {  // branch-free per candidate
                  // distances are never negative: the key is the bits + 1
                  const uint32_t dk = __float_as_uint(pd[c]) + 1u;
                  const bool in = (gx[c] - (wcube[j][0] & 0xffffu)) <= (wcube[j][0] >> 16) &&
                                  (gy[c] - (wcube[j][1] & 0xffffu)) <= (wcube[j][1] >> 16) &&
                                  (gz[c] - (wcube[j][2] & 0xffffu)) <= (wcube[j][2] >> 16);
                  ck[c] = in ? min(ck[c], dk) : ck[c];
                }
              }
            n += m;
            it += m;
          }
        };
        // rows (and whether an axis has more than 32 thresholds) fixed per
        // round: the steps touch only the rows in use, with no branch on them
        using std::integral_constant;
        const bool wide = n0 > 32u || n1 > 32u || n2 > 32u;
        auto replay_rows = [&](auto wide_axes) {
          if (!regtab) {
            replay(std::false_type{}, integral_constant<int, kCandPerLane>{}, wide_axes);
          } else if (!GRID && rows <= 1) {
            // the grid-wide kernels run one-row rounds on the two-row loop:
            // one replay copy less keeps more of their code in the
            // instruction cache (c2 4.141 -> 4.107 ms, c4 26.57 -> 26.28 ms)
            if constexpr (!GRID) replay(std::true_type{}, integral_constant<int, 1>{}, wide_axes);
          } else if (rows <= 2 || kCandPerLane == 2) {
            replay(std::true_type{}, integral_constant<int, (kCandPerLane >= 2 ? 2 : kCandPerLane)>{},
                   wide_axes);
          } else if (rows <= 4 || kCandPerLane == 4) {
            replay(std::true_type{}, integral_constant<int, (kCandPerLane >= 4 ? 4 : kCandPerLane)>{},
                   wide_axes);
          } else {
            replay(std::true_type{}, integral_constant<int, kCandPerLane>{}, wide_axes);
          }
        };
        if (wide) replay_rows(std::true_type{}); else replay_rows(std::false_type{});
        if (it >= a.k) finished = true;
      }
      if (warp == 0 && lane == 0) {
        st_release_cta(&ctl.produced, n);
        ctl.finished = finished ? 1u : 0u;
        st_release_cta(&ctl.done, 1u);
      }
    } else if (widx >= 0) {
      uint32_t s = 0;
      unsigned long long deadline = 0;
      uint32_t polls = 0;
      for (;;) {
        const uint32_t p = ld_acquire_cta(&ctl.produced);
        if (s < p) {
#pragma unroll 1
          for (; s < p; s += kBatch) apply(s, min(p - s, (uint32_t)kBatch));
          s = p;
          continue;
        }
        if (ld_acquire_cta(&ctl.done)) {
          if (s >= ld_acquire_cta(&ctl.produced)) {
            out_n = s;
            out_first = ctl.first;
            break;
          }
          continue;
        }
        __nanosleep(32);
        if ((++polls & 1023u) == 0) {  // bounded: warp 0 itself waits with a limit
          const unsigned long long now = globaltimer();
          if (deadline == 0) deadline = now + 2ull * (unsigned long long)tmo;
          if (now > deadline) { timed_out = true; break; }
        }
      }
    }
    __syncthreads();  // every sample of the round applied
    // CTA 0's workers write the round's samples out while warp 0 starts the
    // next round; s_samp is rewritten only after the next round's first
    // barrier, and the counts were read before this one
    if (crank == 0 && widx >= 0)
      for (uint32_t s2 = (uint32_t)(widx * 32 + lane); s2 < out_n; s2 += (uint32_t)kWorkers)
        a.out_rank[(uint64_t)cloud * a.k + out_first + s2] = s_samp[s2].c.w;
    if (ctl.finished) break;
  }
  // ---- this cloud's epilogue
  if (warp == 0 && lane == 0 && crank == 0) a.out_count[cloud] = it;
  bad_any = bad_any || bad;
  if (!BATCH) break;  // one cloud per cluster / per single-cloud grid
  round_base += round + 1u;
  cloud += gridDim.x / P;
  // a group whose wait ran out stops (its other CTAs' next waits run out too)
  if (__syncthreads_or(timed_out ? 1 : 0) || cloud >= a.B) break;
  }  // clouds

  // ---- epilogue
  if (lane == 0) {
    const uint32_t status = (timed_out ? kStatusTimeout : 0u) | (bad_any ? kStatusBadPlan : 0u);
    if (status) atomicOr(a.scalars + kScalarStatus, status);
  }
  {
    unsigned long long r64 = u_ref, e64 = u_eval;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      r64 += __shfl_xor_sync(kFull, r64, o);
      e64 += __shfl_xor_sync(kFull, e64, o);
    }
    if (lane == 0 && a.stats) {
      atomicAdd(&a.stats[0], r64);
      atomicAdd(&a.stats[1], e64);
    }
  }
  // ---- exit.  Normally every CTA ends in the same round, and every remote
  // write of that round was awaited.  After a wait ran out that no longer
  // holds: a late CTA may still copy its list into this one.  So no CTA of a
  // cluster leaves while another may still write its shared memory: warp 0's
  // copies have read their source, then a cluster barrier, which every CTA
  // reaches because every wait above is bounded.  A CTA issues each copy
  // before at least one complete list wait or replay of its own, so the
  // copies have landed by the time the last CTA arrives.
  if (!GRID) {
    if (warp == 0 && (uint32_t)lane < P) bulk_wait_read_all();
    __syncwarp();
    cluster_sync_all();
  }
}

template <int M, int T, bool GRID, int CAP, bool BATCH = false>
cudaError_t launch_rounds(const LoopArgs &a, size_t smem, cudaStream_t st) {
  auto kern = fps_rounds_cluster<M, T, GRID, CAP, BATCH>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
  if (err) return err;
  if (!GRID && a.P > 8) {
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (err) return err;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((BATCH ? a.groups : a.B) * a.P, 1, 1);
  cfg.blockDim = dim3(kRoundThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (GRID) {  // every CTA co-resident (the groups' barriers need it), or no launch
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  } else {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.P;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int T, bool GRID, int CAP, bool BATCH = false>
cudaError_t launch_rounds_m(const LoopArgs &a, int m, size_t smem, cudaStream_t st) {
  switch (m) {
    case 1: return launch_rounds<1, T, GRID, CAP, BATCH>(a, smem, st);
    case 2: return launch_rounds<2, T, GRID, CAP, BATCH>(a, smem, st);
    case 3: return launch_rounds<3, T, GRID, CAP, BATCH>(a, smem, st);
    case 4: return launch_rounds<4, T, GRID, CAP, BATCH>(a, smem, st);
    case 6: return kMaxLeavesPerThread >= 6
                       ? launch_rounds<(kMaxLeavesPerThread >= 6 ? 6 : 1), T, GRID, CAP, BATCH>(a, smem, st)
                       : cudaErrorInvalidValue;
    case 8: return kMaxLeavesPerThread >= 8
                       ? launch_rounds<(kMaxLeavesPerThread >= 8 ? 8 : 1), T, GRID, CAP, BATCH>(a, smem, st)
                       : cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

// Grid-wide rounds over P = 64 or 128 CTAs publish 5 or 4 candidates per
// CTA (320 or 512 in all).  The round lasts while the best candidate beats
// the largest CTA bound; more candidates per CTA lower that bound but cost
// every step more work: on c2 (P = 64) 4 / 5 / 6 / 7 / 8 per CTA gave 4.218 /
// 4.050 / 4.087 / 4.070 / 4.186 ms (bit-identical samples), on c4 (P = 128) 4
// per CTA gave 28.4 ms against 32.2 for 2.
// Groups of at most 16 CTAs (batches) publish as a cluster does (at most
// big_t(P) each).
constexpr int grid_t(uint32_t P) {
  return P == 64u ? 5 : (P == 128u ? 4 : (P <= 16u ? big_t(P) : 0));
}
constexpr int grid_cap(uint32_t P) { return P == 64u || P == 128u ? (int)P * grid_t(P) : kClusterCap; }
static_assert(16 * kRoundT <= kClusterCap && 16 * kRoundTBig <= kClusterCap &&
                  4 * kRoundTFew <= kClusterCap,
              "parts of up to 16 CTAs fit the cluster capacity");

}  // namespace

int rounds_candidates_per_cta(uint32_t P, uint32_t pts) {
  return pts >= kBigPartPoints ? big_t(P) : kRoundT;
}

int rounds_leaves_per_thread(uint32_t leaves) {
  static const int ms[] = {1, 2, 3, 4, 6, 8};
  for (int m : ms)
    if (m <= kMaxLeavesPerThread && (uint32_t)m * kWorkers >= leaves) return m;
  return 0;
}

size_t rounds_smem_bytes(uint32_t pts, uint32_t leaves, uint32_t tab) {
  return (size_t)pts * 16 + (size_t)leaves * 32 + (size_t)((leaves + 3) & ~3u) * 4 +
         (size_t)((tab + 3) & ~3u) * 4 +
         (size_t)kQueue * sizeof(MaskedSample);
}

int rounds_max_smem(uint32_t P) {
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  // the grid-wide loop (P > one cluster) keeps smaller lists in shared memory
  const int ctl = P == 64u    ? (int)sizeof(RoundCtl<grid_t(64), grid_cap(64)>)
                  : P == 128u ? (int)sizeof(RoundCtl<grid_t(128), grid_cap(128)>)
                              : (int)sizeof(RoundCtl<kMaxPartT, kClusterCap>);
  return optin - ctl - 1024;
}

int rounds_grid_candidates_per_cta(uint32_t P) {
  return grid_t(P);
}

size_t rounds_grid_list_bytes(uint32_t P, uint32_t groups) {
  const size_t list = P == 64u    ? sizeof(CtaList<grid_t(64)>)
                      : P == 128u ? sizeof(CtaList<grid_t(128)>)
                                  : sizeof(CtaList<kMaxPartT>);
  return grid_t(P) ? (size_t)groups * 2 * P * list : 0;
}

size_t rounds_group_list_bytes(uint32_t ctas) {
  return (size_t)2 * ctas * sizeof(CtaList<kMaxPartT>);
}

template <int T>
const void *cluster_kernel(int m) {
  switch (m) {
    case 1: return (const void *)fps_rounds_cluster<1, T, false, kClusterCap>;
    case 2: return (const void *)fps_rounds_cluster<2, T, false, kClusterCap>;
    case 3: return (const void *)fps_rounds_cluster<3, T, false, kClusterCap>;
    case 4: return (const void *)fps_rounds_cluster<4, T, false, kClusterCap>;
    case 6: return (const void *)fps_rounds_cluster<6, T, false, kClusterCap>;
    case 8: return (const void *)fps_rounds_cluster<8, T, false, kClusterCap>;
    default: return nullptr;
  }
}

int rounds_cluster_capacity(uint32_t P, int m, size_t smem) {
  // clusters of P CTAs of the round kernel the device holds at once (a
  // cluster must fit one GPC: on B200 7 clusters of 16 CTAs at one CTA per SM)
  if (P == 0 || P > (uint32_t)kMaxClusterP) return 0;
  // (the instance of the larger lists: its static shared memory bounds the others)
  const void *kern = P <= 4u ? cluster_kernel<kRoundTFew>(m) : cluster_kernel<kRoundTBig>(m);
  if (!kern) return 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ||
      (P > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1))) {
    cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P, 1, 1);
  cfg.blockDim = dim3(kRoundThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = P;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

cudaError_t run_rounds(const LoopArgs &a, const LoopPlan &plan, cudaStream_t st,
                       uint32_t &launches) {
  if (!plan.direct) return cudaErrorInvalidValue;
  cudaError_t err;
  if (plan.mode == 1) {
    if (!a.glist || !a.gbar || rounds_grid_candidates_per_cta(a.P) == 0) return cudaErrorInvalidValue;
    const int m = plan.leaves_per_thread;
    if (a.B == 1 && (a.P == 64u || a.P == 128u)) {  // one cloud over 64 or 128 CTAs
      if ((err = cudaMemsetAsync(a.gbar, 0, sizeof(uint32_t), st))) return err;
      err = a.P == 64u ? launch_rounds_m<grid_t(64), true, grid_cap(64)>(a, m, plan.smem_bytes, st)
                       : launch_rounds_m<grid_t(128), true, grid_cap(128)>(a, m, plan.smem_bytes, st);
    } else {  // a batch over groups of P CTAs
      if (a.groups == 0 || a.groups > a.B || a.P > 16u) return cudaErrorInvalidValue;
      if ((err = cudaMemsetAsync(a.gbar, 0, sizeof(uint32_t) * a.groups, st))) return err;
      const int t = rounds_candidates_per_cta(a.P, a.max_pts);
      err = t == kRoundTFew ? launch_rounds_m<kRoundTFew, true, kClusterCap, true>(a, m, plan.smem_bytes, st)
            : t == kRoundTBig ? launch_rounds_m<kRoundTBig, true, kClusterCap, true>(a, m, plan.smem_bytes, st)
                              : launch_rounds_m<kRoundT, true, kClusterCap, true>(a, m, plan.smem_bytes, st);
    }
  } else {
    if (a.P > (uint32_t)kMaxClusterP) return cudaErrorInvalidValue;
    const int m = plan.leaves_per_thread;
    const int t = rounds_candidates_per_cta(a.P, a.max_pts);
    err = t == kRoundTFew ? launch_rounds_m<kRoundTFew, false, kClusterCap>(a, m, plan.smem_bytes, st)
          : t == kRoundTBig ? launch_rounds_m<kRoundTBig, false, kClusterCap>(a, m, plan.smem_bytes, st)
                            : launch_rounds_m<kRoundT, false, kClusterCap>(a, m, plan.smem_bytes, st);
  }
  launches += 1;
  return err;
}

}  // namespace nsfps
