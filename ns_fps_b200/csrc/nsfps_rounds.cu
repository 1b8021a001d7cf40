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
//   1. top-(T+1) points: each warp picks its T+1 best leaves by leaf maximum;
//      warp 0 merges them to the CTA's T+1 best leaves (the T+1 best points
//      lie in those leaves), gathers their points and selects the T+1 best;
//   2. st.async the T candidates and the bound to every CTA; wait (mbarrier)
//      for all P lists;
//   3. warp 0 replays steps on the candidates, queueing each decided sample
//      (point, distance, cube, position) in shared memory;
//   4. at the same time the worker warps (1..7, which own all the leaves)
//      apply the queued samples to their leaves, in order, as they appear
//      (release/acquire on a shared counter).
//
// Buffers rotate over four rounds (a CTA publishes round r+1 only after it
// has every round-r list), waits are bounded by %globaltimer.
#include "nsfps_device.cuh"

namespace nsfps {

namespace {

constexpr int kWarps = kLoopThreads / 32;
constexpr int kWorkers = kLoopThreads - 32;    // warps 1.. own the leaves
constexpr int kMaxCands = 256;                 // P * T
constexpr int kCandPerLane = kMaxCands / 32;   // 8
constexpr int kQueue = 512;                    // samples decided per round, at most

struct Cand {
  float x, y, z, d;
  uint32_t pos, cell, pad0, pad1;
};

struct Sample {
  float4 q;  // x, y, z, distance
  uint4 c;   // cube x, y, z, sorted position
};

template <int T>
struct RoundCtl {
  Cand cand[kBufs][kMaxCands];
  unsigned long long bound[kBufs][kMaxClusterP];
  unsigned long long mbar[kBufs];
  unsigned long long wkey[kWarps][T + 1];   // per-warp best leaves
  uint32_t wleaf[kWarps][T + 1];
  uint32_t mleaf[T + 1];                    // the CTA's T+1 best leaves
  uint32_t scan[33];
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

// Largest 64-bit key over the warp; returns the lane holding it (lowest lane
// among equal keys) and the key.
__device__ __forceinline__ unsigned long long warp_max64(unsigned long long k, int &who) {
  const uint32_t hi = (uint32_t)(k >> 32), lo = (uint32_t)k;
  const uint32_t mh = __reduce_max_sync(kFull, hi);
  const uint32_t ml = __reduce_max_sync(kFull, hi == mh ? lo : 0u);
  who = __ffs(__ballot_sync(kFull, hi == mh && lo == ml)) - 1;
  return ((unsigned long long)mh << 32) | ml;
}

template <int M, int T>
__global__ void __launch_bounds__(kLoopThreads, 1)
fps_rounds_cluster(const LoopArgs a) {
  constexpr int THREADS = kLoopThreads;
  constexpr int W = kWarps;
  extern __shared__ float4 smem[];
  __shared__ RoundCtl<T> ctl;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t P = a.P;
  const uint32_t cloud = blockIdx.x / P;
  const uint32_t crank = blockIdx.x % P;  // == %cluster_ctarank
  const uint32_t NC = P * T;              // candidates per round

  float4 *s_pts = smem;
  float4 *s_lo = s_pts + a.max_pts;    // (lo.xyz, start | count << 16)
  float4 *s_hi = s_lo + a.max_leaves;  // (hi.xyz, cell)
  float *s_tab = reinterpret_cast<float *>(s_hi + a.max_leaves);
  Sample *s_samp = reinterpret_cast<Sample *>(s_tab + ((a.max_tab + 3u) & ~3u));

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

  // per owned leaf, in registers.  Warp 0 replays the steps and owns no
  // leaf; worker warp w (1..7) owns local leaves m * 224 + (w - 1) * 32 + lane.
  uint32_t cell[M], cnt[M], gst[M], lst[M], gpos[M], lpos[M], sbox_lo[M], sbox_hi[M];
  float lmax[M], bx0[M], by0[M], bz0[M], bx1[M], by1[M], bz1[M];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const uint32_t i = (uint32_t)m * kWorkers + (uint32_t)(warp - 1) * 32 + (uint32_t)lane;
    if (warp > 0 && i < nl) {
      const uint32_t g = gleaf(i);
      const float4 lo = a.leaf_lo[g], hi = a.leaf_hi[g];
      const uint32_t w = __float_as_uint(lo.w);
      const uint32_t slot = (w >> 8) & 0xffu;
      cell[m] = __float_as_uint(hi.w);
      cnt[m] = w & 0xffu;
      gst[m] = a.leaf_start[g];
      lst[m] = __float_as_uint(s_lo[i].w) & 0xffffu;
      lmax[m] = a.leaf_md[g];
      gpos[m] = gst[m] + slot;
      lpos[m] = lst[m] + slot;
      bx0[m] = lo.x; by0[m] = lo.y; bz0[m] = lo.z;
      bx1[m] = hi.x; by1[m] = hi.y; bz1[m] = hi.z;
    } else {
      cell[m] = 0xffffffffu;  // z field 4095: outside every cube
      cnt[m] = 0;
      gst[m] = lst[m] = 0;
      lmax[m] = -1.0f;
      gpos[m] = lpos[m] = 0xffffffffu;
      bx0[m] = by0[m] = bz0[m] = 0.0f;
      bx1[m] = by1[m] = bz1[m] = 0.0f;
    }
    uint32_t x0 = 1023u, y0 = 1023u, z0 = 1023u, x1 = 0u, y1 = 0u, z1 = 0u;
    if (warp > 0 && i < nl) {
      x0 = x1 = cell[m] & 1023u;
      y0 = y1 = (cell[m] >> 10) & 1023u;
      z0 = z1 = cell[m] >> 20;
    }
    x0 = __reduce_min_sync(kFull, x0); y0 = __reduce_min_sync(kFull, y0);
    z0 = __reduce_min_sync(kFull, z0); x1 = __reduce_max_sync(kFull, x1);
    y1 = __reduce_max_sync(kFull, y1); z1 = __reduce_max_sync(kFull, z1);
    sbox_lo[m] = pack_cell(x0, y0, z0);
    sbox_hi[m] = pack_cell(x1, y1, z1);
  }

  const uint32_t tx_bytes = P * (uint32_t)(T * sizeof(Cand) + sizeof(unsigned long long));
  if (tid == 0) {
    for (int b = 0; b < kBufs; ++b) mbar_init(smem_u32(&ctl.mbar[b]), 1);
    fence_mbar_init();
    for (int b = 0; b < kBufs; ++b) mbar_arm(smem_u32(&ctl.mbar[b]), tx_bytes);
    ctl.finished = 0;
  }
  __syncthreads();
  cluster_sync_all();  // every CTA's mbarriers are armed before any remote write

  uint32_t u_ref = 0, u_eval = 0;
  uint32_t it = 1;           // next sample index (sample 0 is point 0)
  bool timed_out = false;
  const long long tmo = a.timeout_ns;
  const int half = lane >> 4, j16 = lane & 15;

  // ---- apply queued sample s to this worker's leaves
  auto apply = [&](uint32_t s) {
      const float4 q = s_samp[s].q;
    const uint4 cb = s_samp[s].c;
    bool need[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
      need[m] = false;
      const uint32_t cxl = cb.x & 0xffffu, cyl = cb.y & 0xffffu, czl = cb.z & 0xffffu;
      const uint32_t cxh = cxl + (cb.x >> 16), cyh = cyl + (cb.y >> 16), czh = czl + (cb.z >> 16);
      const uint32_t sl = sbox_lo[m], sh = sbox_hi[m];
      if (cxl > (sh & 1023u) || (sl & 1023u) > cxh || cyl > ((sh >> 10) & 1023u) ||
          ((sl >> 10) & 1023u) > cyh || czl > (sh >> 20) || (sl >> 20) > czh)
        continue;
      const bool hit = in_box(cell[m], cb.x, cb.y, cb.z);
      const float gx = q.x < bx0[m] ? __fsub_rn(bx0[m], q.x)
                                    : (q.x > bx1[m] ? __fsub_rn(q.x, bx1[m]) : 0.0f);
      const float gy = q.y < by0[m] ? __fsub_rn(by0[m], q.y)
                                    : (q.y > by1[m] ? __fsub_rn(q.y, by1[m]) : 0.0f);
      const float gz = q.z < bz0[m] ? __fsub_rn(bz0[m], q.z)
                                    : (q.z > bz1[m] ? __fsub_rn(q.z, bz1[m]) : 0.0f);
      const float lbd =
          __fadd_rn(__fadd_rn(__fmul_rn(gx, gx), __fmul_rn(gy, gy)), __fmul_rn(gz, gz));
      need[m] = hit && lbd < lmax[m];
      u_ref += hit ? cnt[m] : 0u;
      u_eval += need[m] ? cnt[m] : 0u;
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      uint32_t mask = __ballot_sync(kFull, need[m]);
      while (mask) {
        const int la = __ffs(mask) - 1;
        mask &= mask - 1;
        int lb2 = -1;
        if (mask) {
          lb2 = __ffs(mask) - 1;
          mask &= mask - 1;
        }
        const int src = half ? lb2 : la;
        uint32_t key = 0u;
        if (src >= 0) {
          const uint32_t l = (uint32_t)m * kWorkers + (uint32_t)(warp - 1) * 32 + (uint32_t)src;
          const uint32_t lw = __float_as_uint(s_lo[l].w);
          const uint32_t start = lw & 0xffffu, c = lw >> 16;
          if ((uint32_t)j16 < c) {
            float4 p = s_pts[start + j16];
            const float d = sqdist(p.x, p.y, p.z, q.x, q.y, q.z);
            if (d < p.w) { p.w = d; s_pts[start + j16].w = d; }
            key = dkey(p.w);
          }
        }
        const uint32_t kA = __reduce_max_sync(kFull, half ? 0u : key);
        const uint32_t kB = __reduce_max_sync(kFull, half ? key : 0u);
        const uint32_t fA = __ffs(__ballot_sync(kFull, !half && key == kA)) - 1;
        const uint32_t fB = __ffs(__ballot_sync(kFull, half && key == kB)) - 17;
        if (lane == la) {
          lmax[m] = __uint_as_float(kA - 1u);
          lpos[m] = lst[m] + fA;
          gpos[m] = gst[m] + fA;
        }
        if (lane == lb2) {
          lmax[m] = __uint_as_float(kB - 1u);
          lpos[m] = lst[m] + fB;
          gpos[m] = gst[m] + fB;
        }
      }
    }
      };

  for (uint32_t round = 0;; ++round) {
    const uint32_t buf = round & (kBufs - 1);

    // ---- 1a. each worker warp: its T+1 best leaves by leaf maximum
    if (warp > 0) {
      uint32_t taken = 0u;
#pragma unroll 1
      for (int t = 0; t <= T; ++t) {
        unsigned long long best = 0ull;
        int bm = 0;
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const unsigned long long k = ((taken >> m) & 1u) ? 0ull : pkey(lmax[m], gpos[m]);
          if (k > best) { best = k; bm = m; }
        }
        int who;
        const unsigned long long wk = warp_max64(best, who);
        const int wm = __shfl_sync(kFull, bm, who);
        if (lane == who && wk != 0ull) taken |= 1u << wm;
        if (lane == 0) {
          ctl.wkey[warp][t] = wk;
          ctl.wleaf[warp][t] = (uint32_t)wm * kWorkers + (uint32_t)(warp - 1) * 32 + (uint32_t)who;
        }
      }
    } else if (lane == 0) {
      ctl.produced = 0u;
      ctl.done = 0u;
      ctl.first = it;
    }
    __syncthreads();

    // ---- 1b/2/3. warp 0: list, exchange, replay; the workers apply the
    // samples as they are queued
    if (warp == 0) {
      // merge the worker warps' lists ((W - 1) * (T+1) entries)
      constexpr int NE = (W - 1) * (T + 1);
      constexpr int E = (NE + 31) / 32;
      unsigned long long ek[E];
      uint32_t el[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int idx = lane + 32 * e;
        ek[e] = idx < NE ? ctl.wkey[1 + idx / (T + 1)][idx % (T + 1)] : 0ull;
        el[e] = idx < NE ? ctl.wleaf[1 + idx / (T + 1)][idx % (T + 1)] : 0u;
      }
      uint32_t nleaf = 0;
#pragma unroll 1
      for (int t = 0; t <= T; ++t) {
        unsigned long long best = 0ull;
        int be = 0;
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (ek[e] > best) { best = ek[e]; be = e; }
        int who;
        const unsigned long long wk = warp_max64(best, who);
        if (wk == 0ull) break;
        uint32_t lsel = 0u;
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (e == be) lsel = el[e];
        const uint32_t wl = __shfl_sync(kFull, lsel, who);
        if (lane == who) {
#pragma unroll
          for (int e = 0; e < E; ++e)
            if (e == be) ek[e] = 0ull;
        }
        if (lane == 0) ctl.mleaf[t] = wl;
        ++nleaf;
      }
      __syncwarp();
      // gather the points of those leaves; half-warp h takes leaf 2r + h
      constexpr int G = (T + 2) / 2;  // points held per lane
      unsigned long long gk[G];
      float4 gp[G];
      uint32_t gc[G];
#pragma unroll
      for (int r = 0; r < G; ++r) {
        const uint32_t li = 2u * r + (uint32_t)half;
        gk[r] = 0ull;
        gp[r] = make_float4(0, 0, 0, -1.0f);
        gc[r] = 0u;
        if (li < nleaf) {
          const uint32_t leaf = ctl.mleaf[li];
          const uint32_t lw = __float_as_uint(s_lo[leaf].w);
          const uint32_t start = lw & 0xffffu, c = lw >> 16;
          if ((uint32_t)j16 < c) {
            gp[r] = s_pts[start + j16];
            gc[r] = __float_as_uint(s_hi[leaf].w);
            // sorted position: the leaf's global start + slot
            const uint32_t gstart = a.leaf_start[gleaf(leaf)];
            gk[r] = pkey(gp[r].w, gstart + j16);
          }
        }
      }
      // the T+1 best points: the first T are the list, the next is the bound
      unsigned long long bound = 0ull;
#pragma unroll 1
      for (int t = 0; t <= T; ++t) {
        unsigned long long best = 0ull;
        int br = 0;
#pragma unroll
        for (int r = 0; r < G; ++r)
          if (gk[r] > best) { best = gk[r]; br = r; }
        int who;
        const unsigned long long wk = warp_max64(best, who);
        if (t == T) { bound = wk; break; }
        float4 p = make_float4(0, 0, 0, -1.0f);
        uint32_t c = 0u;
#pragma unroll
        for (int r = 0; r < G; ++r)
          if (r == br) { p = gp[r]; c = gc[r]; }
        p.x = __shfl_sync(kFull, p.x, who);
        p.y = __shfl_sync(kFull, p.y, who);
        p.z = __shfl_sync(kFull, p.z, who);
        p.w = __shfl_sync(kFull, p.w, who);
        c = __shfl_sync(kFull, c, who);
        if (lane == who) {
#pragma unroll
          for (int r = 0; r < G; ++r)
            if (r == br) gk[r] = 0ull;
        }
        // candidate t of this CTA: to every CTA's cand[buf][crank * T + t]
        Cand cd;
        if (wk == 0ull) {
          cd.x = cd.y = cd.z = 0.0f;
          cd.d = -1.0f;
          cd.pos = 0xffffffffu;
          cd.cell = 0xffffffffu;
        } else {
          cd.x = p.x; cd.y = p.y; cd.z = p.z; cd.d = p.w;
          cd.pos = 0xffffffffu - (uint32_t)wk;
          cd.cell = c;
        }
        if ((uint32_t)lane < P) {
          const uint32_t ra = mapa(smem_u32(&ctl.cand[buf][crank * T + t]), lane);
          const uint32_t rm = mapa(smem_u32(&ctl.mbar[buf]), lane);
          st_async_v4(ra, make_uint4(__float_as_uint(cd.x), __float_as_uint(cd.y),
                                     __float_as_uint(cd.z), __float_as_uint(cd.d)), rm);
          st_async_v4(ra + 16, make_uint4(cd.pos, cd.cell, 0u, 0u), rm);
        }
      }
      if ((uint32_t)lane < P) {
        const uint32_t ra = mapa(smem_u32(&ctl.bound[buf][crank]), lane);
        const uint32_t rm = mapa(smem_u32(&ctl.mbar[buf]), lane);
        st_async_v2(ra, (uint32_t)bound, (uint32_t)(bound >> 32), rm);
      }

      // ---- wait for every CTA's list (bounded)
      const uint32_t mb = smem_u32(&ctl.mbar[buf]);
      const uint32_t parity = (round / kBufs) & 1u;
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
      if (lane == 0) mbar_arm(mb, tx_bytes);  // for round + kBufs

      // ---- 3. replay steps on the candidates
      uint32_t n = 0;
      bool finished = timed_out;
      if (!timed_out) {
        float cx[kCandPerLane], cy[kCandPerLane], cz[kCandPerLane], cdd[kCandPerLane];
        uint32_t cpos[kCandPerLane], ccell[kCandPerLane];
#pragma unroll
        for (int c = 0; c < kCandPerLane; ++c) {
          const uint32_t idx = (uint32_t)(lane + 32 * c);
          if (idx < NC) {
            const Cand cd = ctl.cand[buf][idx];
            cx[c] = cd.x; cy[c] = cd.y; cz[c] = cd.z; cdd[c] = cd.d;
            cpos[c] = cd.pos; ccell[c] = cd.cell;
          } else {
            cx[c] = cy[c] = cz[c] = 0.0f; cdd[c] = -1.0f;
            cpos[c] = 0xffffffffu; ccell[c] = 0xffffffffu;
          }
        }
        // B* = the largest bound
        unsigned long long bl = 0ull;
        if ((uint32_t)lane < P) bl = ctl.bound[buf][lane];
        int who;
        const unsigned long long bstar = warp_max64(bl, who);

        while (it < a.k && n < (uint32_t)kQueue) {
          unsigned long long best = 0ull;
          int bc = 0;
#pragma unroll
          for (int c = 0; c < kCandPerLane; ++c) {
            const unsigned long long k = pkey(cdd[c], cpos[c]);
            if (cdd[c] >= 0.0f && k > best) { best = k; bc = c; }
          }
          const unsigned long long wk = warp_max64(best, who);
          if (wk <= bstar) break;  // not certain: some unlisted point may win
          float qx = 0.0f, qy = 0.0f, qz = 0.0f, qd = 0.0f;
          uint32_t qcell = 0u;
#pragma unroll
          for (int c = 0; c < kCandPerLane; ++c)
            if (c == bc) { qx = cx[c]; qy = cy[c]; qz = cz[c]; qd = cdd[c]; qcell = ccell[c]; }
          qx = __shfl_sync(kFull, qx, who);
          qy = __shfl_sync(kFull, qy, who);
          qz = __shfl_sync(kFull, qz, who);
          qd = __shfl_sync(kFull, qd, who);
          qcell = __shfl_sync(kFull, qcell, who);
          if (!(qd > 0.0f)) {  // src/yuezu_fps.cpp:705-706
            finished = true;
            break;
          }
          const uint32_t qpos = 0xffffffffu - (uint32_t)wk;
          const uint32_t qc[3] = {qcell & 1023u, (qcell >> 10) & 1023u, qcell >> 20};
          uint32_t cube[3];
          cube_of(ax, fast, qc, qd, cube);
          if (lane == 0) {
            Sample sm;
            sm.q = make_float4(qx, qy, qz, qd);
            sm.c = make_uint4(cube[0], cube[1], cube[2], qpos);
            s_samp[n] = sm;
            st_release_cta(&ctl.produced, n + 1);  // the workers may apply it now
          }
#pragma unroll
          for (int c = 0; c < kCandPerLane; ++c)
            if (in_box(ccell[c], cube[0], cube[1], cube[2])) {
              const float d = sqdist(cx[c], cy[c], cz[c], qx, qy, qz);
              if (d < cdd[c]) cdd[c] = d;
            }
          ++n;
          ++it;
        }
        if (it >= a.k) finished = true;
      }
      if (lane == 0) {
        ctl.finished = finished ? 1u : 0u;
        st_release_cta(&ctl.done, 1u);
      }
    }
 else {
      uint32_t s = 0;
      unsigned long long deadline = 0;
      uint32_t polls = 0;
      for (;;) {
        const uint32_t p = ld_acquire_cta(&ctl.produced);
        if (s < p) {
#pragma unroll 1
          for (; s < p; ++s) apply(s);
          continue;
        }
        if (ld_acquire_cta(&ctl.done)) {
          if (s >= ld_acquire_cta(&ctl.produced)) break;
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
    if (crank == 0) {  // the round's samples, written once the round is over
      const uint32_t nq = ctl.produced, f = ctl.first;
      for (uint32_t s2 = tid; s2 < nq; s2 += THREADS)
        a.out_rank[(uint64_t)cloud * a.k + f + s2] = s_samp[s2].c.w;
      __syncthreads();  // s_samp is rewritten by the next round
    }
    if (ctl.finished) break;
  }

  // ---- epilogue
  if (lane == 0) {
    const uint32_t status = (timed_out ? kStatusTimeout : 0u) | (bad ? kStatusBadPlan : 0u);
    if (status) atomicOr(a.scalars + kScalarStatus, status);
    if (warp == 0 && crank == 0) a.out_count[cloud] = it;
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
  // All CTAs replay the same steps, so they end in the same round; every
  // remote write of that round was awaited, so no final cluster barrier.
}

template <int M, int T>
cudaError_t launch_rounds(const LoopArgs &a, size_t smem, cudaStream_t st) {
  auto kern = fps_rounds_cluster<M, T>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
  if (err) return err;
  if (a.P > 8) {
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (err) return err;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.B * a.P, 1, 1);
  cfg.blockDim = dim3(kLoopThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.P;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int T>
cudaError_t launch_rounds_m(const LoopArgs &a, int m, size_t smem, cudaStream_t st) {
  switch (m) {
    case 1: return launch_rounds<1, T>(a, smem, st);
    case 2: return launch_rounds<2, T>(a, smem, st);
    case 3: return launch_rounds<3, T>(a, smem, st);
    case 4: return launch_rounds<4, T>(a, smem, st);
    case 6: return launch_rounds<6, T>(a, smem, st);
    case 8: return launch_rounds<8, T>(a, smem, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int rounds_candidates_per_cta(uint32_t) { return 16; }

int rounds_leaves_per_thread(uint32_t leaves) {
  static const int ms[] = {1, 2, 3, 4, 6, 8};
  for (int m : ms)
    if ((uint32_t)m * kWorkers >= leaves) return m;
  return 0;
}

size_t rounds_smem_bytes(uint32_t pts, uint32_t leaves, uint32_t tab) {
  return (size_t)pts * 16 + (size_t)leaves * 32 + (size_t)((tab + 3) & ~3u) * 4 +
         (size_t)kQueue * sizeof(Sample);
}

int rounds_max_smem(uint32_t P) {
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  (void)P;
  return optin - (int)sizeof(RoundCtl<16>) - 1024;
}

cudaError_t run_rounds(const LoopArgs &a, const LoopPlan &plan, cudaStream_t st,
                       uint32_t &launches) {
  if (a.P > (uint32_t)kMaxClusterP || !plan.direct) return cudaErrorInvalidValue;
  const cudaError_t err = launch_rounds_m<16>(a, plan.leaves_per_thread, plan.smem_bytes, st);
  launches += 1;
  return err;
}

}  // namespace nsfps
