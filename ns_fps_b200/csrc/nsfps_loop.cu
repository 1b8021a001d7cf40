// nsfps_loop.cu -- the persistent farthest-point-sampling kernel.
//
// Data placement.  The leaves of a cloud (runs of <= 16 sorted points of one
// bucket) are dealt round-robin to its P CTAs (leaf l -> CTA l % P), so the
// leaves of one cell -- which are consecutive -- land on different CTAs and a
// step's work spreads over them; inside a CTA, warp w's slot m holds 32
// consecutive local leaves (a compact region), so one cell-box test per slot
// skips most of a warp's leaves.  A CTA keeps, for the whole sampling loop, its
// leaves' points in shared memory as float4 (x, y, z, current min distance)
// and each leaf's (local start, count); every thread keeps in registers, per
// owned leaf (up to M), the cell, bounding box, count, current maximum
// distance and where the first point holding it sits (global sorted
// position, for ties, and shared-memory index).
//
// Agents.  Every warp is an independent agent over the leaves of its 32
// threads: the warps of all P CTAs (A = 8 P agents) each publish a proposal
// every step, and every warp picks the step's winner from all A proposals.
// There is no block-wide barrier and no block-wide reduction in the loop, so
// one step costs one exchange latency plus one warp's worth of work.
//
// One step (the body of the reference's loop, src/yuezu_fps.cpp:703-722):
//   1. wait for the A proposals of the step and pick the winner: largest
//      distance, ties to the smallest sorted position -- the root of the
//      reference's 16-ary cache tree (:549-558);
//   2. stop when that distance is <= 0 (:705-706); one warp of CTA 0 records
//      the winner's sorted position;
//   3. every thread tests its leaves against the winner's cell cube: a leaf is
//      selected iff one of the cells mapping to its bucket is in the cube (the
//      reference updates every leaf of those buckets, :495-513); a selected
//      leaf whose bounding-box lower bound (computed with the same rounding as
//      the distances, so it never exceeds any point's distance) is >= its
//      current max cannot change and is skipped;
//   4. the warp updates its remaining selected leaves together, two leaves
//      per pass (16 lanes per leaf, one point per lane): min(old, d)
//      (:234-265) and a new leaf max (first slot wins ties);
//   5. per-thread best -> warp best (redux.sync); the warp turns its farthest
//      point into the next step's proposal -- the point, its distance, the
//      cell cube of get_morton_codes_in_range (:560-597) it would induce as a
//      sample, and its sorted position -- and writes it to every CTA.
//
// Exchange (P <= 16 CTAs of one thread-block cluster).  A proposal is two
// st.async writes into each CTA's shared memory that complete transaction
// bytes on that CTA's mbarrier; warps wait on their own CTA's mbarrier
// (acquire).  Four slot buffers rotate with the step.  A buffer is rewritten,
// and its barrier re-armed, only after every warp has consumed it: a warp
// writes step i+1 only after it received every warp's step i, so a write for
// step i+4 causally follows three complete exchange rounds after every step-i
// write was issued; with two buffers one round would separate them, and
// nothing in the memory model orders one agent's writes to different CTAs.
//
// No wait is unbounded: a wait gives up after a time limit and sets a status
// bit; since every warp waits on the same phase, all of them give up.
#include <cfloat>

#include "nsfps_device.cuh"

namespace nsfps {

namespace {

constexpr int kWarpsPerCta = kLoopThreads / 32;
constexpr int kMaxAgents = kMaxClusterP * kWarpsPerCta;  // 128
// A proposal: an agent's farthest point (x, y, z, dist) and, for that point
// as the next sample, the packed cell cube and its sorted position.  The
// (distance key, position) pair is also written to a compact array, which
// the winner search scans without shared-memory bank conflicts.
struct Proposal {
  float4 q;
  uint4 c;  // cube x, cube y, cube z, global sorted position
};

struct SharedCtl {
  Proposal slot[kBufs][kMaxAgents];
  uint2 key[kBufs][kMaxAgents];  // (dkey(dist), global sorted position)
  unsigned long long mbar[kBufs];
  uint32_t scan[33];
};
constexpr uint32_t kProposalBytes = (uint32_t)(sizeof(Proposal) + sizeof(uint2));

template <int M, bool DIRECT>
__global__ void __launch_bounds__(kLoopThreads, 1)
fps_loop_cluster(const LoopArgs a) {
  constexpr int THREADS = kLoopThreads;
  constexpr int W = kWarpsPerCta;
  extern __shared__ float4 smem[];
  __shared__ SharedCtl ctl;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t P = a.P;
  const uint32_t A = P * W;  // agents
  const uint32_t cloud = blockIdx.x / P;
  const uint32_t crank = blockIdx.x % P;  // == %cluster_ctarank (cluster = P along x)

  float4 *s_pts = smem;
  float4 *s_lo = s_pts + a.max_pts;  // (lo.xyz, start | count << 16)
  float4 *s_hi = s_lo + a.max_leaves;  // (hi.xyz, npre << 24 | extra offset)
  uint32_t *s_pre = reinterpret_cast<uint32_t *>(s_hi + a.max_leaves);
  float *s_tab = reinterpret_cast<float *>(s_pre + a.max_extra);

  const RangeDev &Rg = a.ranges[a.rid[cloud]];
  const uint32_t n0 = Rg.blocks[0] - 1, n1 = Rg.blocks[1] - 1, n2 = Rg.blocks[2] - 1;
  const bool fast = Rg.fast_cube != 0;
  const uint32_t l0 = a.loff[cloud], l1 = a.loff[cloud + 1];
  // this CTA's leaves: l0 + crank + P * i for local index i < nl
  uint32_t nl = (l1 - l0 > crank) ? (l1 - l0 - crank + P - 1) / P : 0u;
  bool bad = nl > a.max_leaves || nl > (uint32_t)(M * THREADS) ||
             (fast && n0 + n1 + n2 > a.max_tab) || A > (uint32_t)kMaxAgents;
  if (bad) nl = 0;
  auto gleaf = [&](uint32_t i) { return l0 + crank + P * i; };

  // ---- prologue: leaves, their points and the cube thresholds into shared
  // memory (local point starts by a block scan of the leaf sizes)
  if (fast && !bad)
    for (uint32_t i = tid; i < n0 + n1 + n2; i += THREADS) {
      const uint32_t src = i < n0 ? Rg.tab_off[0] + i
                                  : (i < n0 + n1 ? Rg.tab_off[1] + (i - n0)
                                                 : Rg.tab_off[2] + (i - n0 - n1));
      s_tab[i] = a.tabs[src];
    }
  uint32_t pts_base = 0, extra_base = 0;
  for (uint32_t base = 0; base < nl; base += THREADS) {
    const uint32_t i = base + tid;
    uint32_t cntl = 0, npre = 1, g = 0;
    float4 lo = make_float4(0, 0, 0, 0), hi = lo;
    if (i < nl) {
      g = gleaf(i);
      lo = a.leaf_lo[g];
      hi = a.leaf_hi[g];
      cntl = __float_as_uint(lo.w) & 0xffu;
      npre = __float_as_uint(lo.w) >> 16;
    }
    uint32_t tot_pts = 0, tot_pre = 0, ex_pre = 0;
    const uint32_t ex_pts = block_excl_sum<THREADS>(cntl, ctl.scan, tot_pts);
    if (!DIRECT)
      ex_pre = block_excl_sum<THREADS>(i < nl && npre > 1 ? npre - 1 : 0, ctl.scan, tot_pre);
    if (i < nl) {
      const uint32_t lstart = pts_base + ex_pts;
      const uint32_t off = extra_base + ex_pre;
      if (lstart + cntl <= a.max_pts && lstart < 65536u) {
        s_lo[i] = make_float4(lo.x, lo.y, lo.z, __uint_as_float(lstart | (cntl << 16)));
        const uint32_t gs = a.leaf_start[g];
        for (uint32_t j = 0; j < cntl; ++j) s_pts[lstart + j] = a.pts[gs + j];
      }
      s_hi[i] = make_float4(hi.x, hi.y, hi.z, __uint_as_float((npre << 24) | (off & 0xffffffu)));
      if (!DIRECT && npre > 1 && off + npre - 1 <= a.max_extra)
        for (uint32_t j = 0; j + 1 < npre; ++j)
          s_pre[off + j] = a.leaf_pre[(uint64_t)g * kMaxPreimages + j];
    }
    pts_base += tot_pts;
    extra_base += tot_pre;
  }
  if (pts_base > a.max_pts || pts_base > 65536u || (!DIRECT && extra_base > a.max_extra)) {
    bad = true;  // never with a correct plan
    nl = 0;
  }
  __syncthreads();

  // range fields of the publishing path, in registers
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

  // per owned leaf (local index m * 256 + warp * 32 + lane), in registers;
  // per warp and slot m, the box of cells of the slot's 32 leaves (sbox_lo /
  // sbox_hi, packed like cells) lets a warp skip a slot with one test
  uint32_t cell[M], cnt[M], gst[M], lst[M], gpos[M], lpos[M], sbox_lo[M], sbox_hi[M];
  float lmax[M], bx0[M], by0[M], bz0[M], bx1[M], by1[M], bz1[M];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const uint32_t i = (uint32_t)m * THREADS + (uint32_t)warp * 32 + (uint32_t)lane;
    if (i < nl) {
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
    // cell box of this lane's leaf (every preimage cell for hashed ranges)
    uint32_t x0 = 1023u, y0 = 1023u, z0 = 1023u, x1 = 0u, y1 = 0u, z1 = 0u;
    if (i < nl) {
      const uint32_t c0 = cell[m];
      x0 = x1 = c0 & 1023u;
      y0 = y1 = (c0 >> 10) & 1023u;
      z0 = z1 = c0 >> 20;
      if (!DIRECT) {
        const uint32_t hw = __float_as_uint(s_hi[i].w);
        const uint32_t npre = hw >> 24, off = hw & 0xffffffu;
        for (uint32_t j = 0; j + 1 < npre; ++j) {
          const uint32_t c1 = s_pre[off + j];
          x0 = min(x0, c1 & 1023u); x1 = max(x1, c1 & 1023u);
          y0 = min(y0, (c1 >> 10) & 1023u); y1 = max(y1, (c1 >> 10) & 1023u);
          z0 = min(z0, c1 >> 20); z1 = max(z1, c1 >> 20);
        }
      }
    }
    x0 = __reduce_min_sync(kFull, x0); y0 = __reduce_min_sync(kFull, y0);
    z0 = __reduce_min_sync(kFull, z0); x1 = __reduce_max_sync(kFull, x1);
    y1 = __reduce_max_sync(kFull, y1); z1 = __reduce_max_sync(kFull, z1);
    sbox_lo[m] = pack_cell(x0, y0, z0);
    sbox_hi[m] = pack_cell(x1, y1, z1);
  }

  const uint32_t tx_bytes = kProposalBytes * A;
  if (tid == 0) {
    for (int b = 0; b < kBufs; ++b) mbar_init(smem_u32(&ctl.mbar[b]), 1);
    fence_mbar_init();
    for (int b = 0; b < kBufs; ++b) mbar_arm(smem_u32(&ctl.mbar[b]), tx_bytes);
  }
  __syncthreads();
  cluster_sync_all();  // every CTA's mbarriers are armed before any remote write

  // cluster addresses of this agent's slot 0 and of barrier 0 in CTA `lane`
  const uint32_t agent = crank * W + warp;
  const uint32_t r_slot0 = mapa(smem_u32(&ctl.slot[0][agent]), (uint32_t)lane < P ? lane : 0);
  const uint32_t r_key0 = mapa(smem_u32(&ctl.key[0][agent]), (uint32_t)lane < P ? lane : 0);
  const uint32_t r_mbar0 = mapa(smem_u32(&ctl.mbar[0]), (uint32_t)lane < P ? lane : 0);

  uint32_t u_ref = 0, u_eval = 0;
  uint32_t len = 1;
  bool timed_out = false;

  // ---- this warp's farthest point -> proposal for `step`, written into
  // slot[step % kBufs][agent] of every CTA of the cluster
  // The proposal of the previous step, re-sent unchanged when none of the
  // warp's leaves changed since (the common case: a step touches few leaves).
  uint4 qv = make_uint4(0u, 0u, 0u, __float_as_uint(-1.0f));
  uint4 cv = make_uint4(kNoCell, kNoCell, kNoCell, 0u);
  uint32_t kmax = 0u, gmin = 0xffffffffu;
  bool dirty = true;
  auto propose = [&](uint32_t step) {
    if (dirty) {
      float bd = -1.0f;
      uint32_t bg = 0xffffffffu, bl = 0u, bc = 0u;
#pragma unroll
      for (int m = 0; m < M; ++m)
        if (lmax[m] > bd || (lmax[m] == bd && gpos[m] < bg)) {
          bd = lmax[m];
          bg = gpos[m];
          bl = lpos[m];
          bc = cell[m];
        }
      const uint32_t key = dkey(bd);
      kmax = __reduce_max_sync(kFull, key);
      gmin = __reduce_min_sync(kFull, key == kmax ? bg : 0xffffffffu);
      qv = make_uint4(0u, 0u, 0u, __float_as_uint(-1.0f));
      cv = make_uint4(kNoCell, kNoCell, kNoCell, gmin);
      if (kmax != 0) {
        const uint32_t wl = __ffs(__ballot_sync(kFull, key == kmax && bg == gmin)) - 1;
        const float4 p = s_pts[__shfl_sync(kFull, bl, wl)];
        uint32_t qc[3];
        if (DIRECT) {  // the point's cell is its leaf's cell
          const uint32_t c = __shfl_sync(kFull, bc, wl);
          qc[0] = c & 1023u;
          qc[1] = (c >> 10) & 1023u;
          qc[2] = c >> 20;
        } else {
          qc[0] = cell_axis(p.x, ax[0].mn, ax[0].hi, ax[0].inv, (uint32_t)ax[0].blocks);
          qc[1] = cell_axis(p.y, ax[1].mn, ax[1].hi, ax[1].inv, (uint32_t)ax[1].blocks);
          qc[2] = cell_axis(p.z, ax[2].mn, ax[2].hi, ax[2].inv, (uint32_t)ax[2].blocks);
        }
        uint32_t cube[3];
        cube_of(ax, fast, qc, p.w, cube);
        qv = make_uint4(__float_as_uint(p.x), __float_as_uint(p.y), __float_as_uint(p.z),
                        __float_as_uint(p.w));
        cv = make_uint4(cube[0], cube[1], cube[2], gmin);
      }
      dirty = false;
    }
    // test hook: one CTA of cloud 0 withholds its agents' proposals of a step
    const bool hold = cloud == 0u && (int)crank == a.hold_cta && step == a.hold_step;
    if ((uint32_t)lane < P && !hold) {
      const uint32_t b = step & (kBufs - 1);
      const uint32_t rs = r_slot0 + b * (uint32_t)sizeof(ctl.slot[0]);
      const uint32_t rk = r_key0 + b * (uint32_t)sizeof(ctl.key[0]);
      const uint32_t rm = r_mbar0 + b * (uint32_t)sizeof(ctl.mbar[0]);
      st_async_v4(rs, qv, rm);
      st_async_v4(rs + 16, cv, rm);
      st_async_v2(rk, kmax, gmin, rm);
    }
  };

  if (a.k > 1) propose(1);

  const long long tmo = a.timeout_ns;
  const int half = lane >> 4, j16 = lane & 15;
  for (uint32_t it = 1; it < a.k; ++it) {
    // mbar[b] serves the steps it with it % kBufs == b (steps start at 1);
    // its phase for step it is (it - 1) / kBufs
    const uint32_t buf = it & (kBufs - 1), parity = ((it - 1) / kBufs) & 1u;
    const uint32_t mb = smem_u32(&ctl.mbar[buf]);
    {  // bounded wait, warp-uniform outcome
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
    }
    if (timed_out) break;
    // re-arm this buffer for step it + kBufs: its writers need this CTA's
    // step it + 1 proposals first, and warp 0 writes its own only after this
    if (tid == 0) mbar_arm(mb, tx_bytes);

    // ---- winner among the A proposals: largest distance, smallest position
    uint32_t bkey = 0, brank = 0xffffffffu, bidx = 0;
#pragma unroll
    for (int t = 0; t < kMaxAgents / 32; ++t) {
      const uint32_t idx = (uint32_t)(lane + 32 * t);
      if (idx < A) {
        const uint2 kr = ctl.key[buf][idx];
        if (kr.x > bkey || (kr.x == bkey && kr.y < brank)) { bkey = kr.x; brank = kr.y; bidx = idx; }
      }
    }
    const uint32_t kmax = __reduce_max_sync(kFull, bkey);
    const uint32_t rmin = __reduce_min_sync(kFull, bkey == kmax ? brank : 0xffffffffu);
    const uint32_t wl = __ffs(__ballot_sync(kFull, bkey == kmax && brank == rmin)) - 1;
    const uint32_t widx = __shfl_sync(kFull, bidx, wl);
    const float4 q = ctl.slot[buf][widx].q;
    const uint4 cb = ctl.slot[buf][widx].c;
    // every warp of every CTA reads the same proposals, so all stop together
    if (!(q.w > 0.0f)) break;
    if (crank == 0 && tid == 0) a.out_rank[(uint64_t)cloud * a.k + it] = cb.w;

    // ---- (a) which owned leaves may change: selected by the cube and not
    // provably unchanged by the bounding-box bound
    bool need[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
      need[m] = false;
      // the whole slot first: does its cell box meet the cube?  (uniform)
      const uint32_t cxl = cb.x & 0xffffu, cyl = cb.y & 0xffffu, czl = cb.z & 0xffffu;
      const uint32_t cxh = cxl + (cb.x >> 16), cyh = cyl + (cb.y >> 16), czh = czl + (cb.z >> 16);
      const uint32_t sl = sbox_lo[m], sh = sbox_hi[m];
      if (cxl > (sh & 1023u) || (sl & 1023u) > cxh || cyl > ((sh >> 10) & 1023u) ||
          ((sl >> 10) & 1023u) > cyh || czl > (sh >> 20) || (sl >> 20) > czh)
        continue;
      bool hit = in_box(cell[m], cb.x, cb.y, cb.z);
      if (!DIRECT && !hit && cnt[m]) {
        const uint32_t hw =
            __float_as_uint(s_hi[(uint32_t)m * THREADS + (uint32_t)warp * 32 + (uint32_t)lane].w);
        const uint32_t npre = hw >> 24, off = hw & 0xffffffu;
        for (uint32_t j = 0; j + 1 < npre; ++j)
          hit = hit || in_box(s_pre[off + j], cb.x, cb.y, cb.z);
      }
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
    }
    // ---- (b) the warp updates the selected leaves together, two at a time:
    // half-warp h takes one leaf, lane j of the half its point j; each half's
    // new maximum is a redux over its lanes, its first position a ballot
#pragma unroll
    for (int m = 0; m < M; ++m) {
      uint32_t mask = __ballot_sync(kFull, need[m]);
      dirty = dirty || mask != 0u;
      while (mask) {
        const int la = __ffs(mask) - 1;
        mask &= mask - 1;
        int lb2 = -1;
        if (mask) {
          lb2 = __ffs(mask) - 1;
          mask &= mask - 1;
        }
        const int src = half ? lb2 : la;
        uint32_t key = 0u;  // dkey of the point's new distance; 0 = no point
        if (src >= 0) {
          const uint32_t l = (uint32_t)m * THREADS + (uint32_t)warp * 32 + (uint32_t)src;
          const uint32_t lw = __float_as_uint(s_lo[l].w);
          const uint32_t start = lw & 0xffffu, c = lw >> 16;
          if ((uint32_t)j16 < c) {
            ++u_eval;  // points evaluated, counted here rather than in the leaf tests
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
        // first slot holding the maximum; a leaf's points are consecutive
        // both in shared memory and in the sorted order
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
    len = it + 1;
    if (it + 1 < a.k) propose(it + 1);
  }

  // ---- epilogue
  if (lane == 0) {
    uint32_t status = (timed_out ? kStatusTimeout : 0u) | (bad ? kStatusBadPlan : 0u);
    if (status) atomicOr(a.scalars + kScalarStatus, status);
  }
  if (crank == 0 && tid == 0) a.out_count[cloud] = len;
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
  // ---- exit.  Normally every remote write into this CTA's shared memory
  // belongs to a step every warp here has waited for (all agents stop at the
  // same step and nobody writes past it).  After a wait ran out that no
  // longer holds: a late agent may still write its proposals here.  So no
  // CTA leaves before every CTA of the cluster is done writing: a cluster
  // barrier, which every CTA reaches because every wait above is bounded.
  // An agent writes a step's proposals before waiting (bounded) for that
  // step, so they have landed by the time the last CTA arrives.
  cluster_sync_all();
}

__global__ void epilogue_kernel(const uint32_t *__restrict__ out_rank,
                                const uint32_t *__restrict__ out_count,
                                const uint32_t *__restrict__ perm,
                                const uint32_t *__restrict__ poff, uint32_t B,
                                uint32_t k, uint64_t *__restrict__ out) {
  const uint64_t total = (uint64_t)B * k;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t c = (uint32_t)(t / k), i = (uint32_t)(t % k);
    if (i >= out_count[c]) continue;
    out[t] = i == 0 ? 0ull : (uint64_t)(perm[out_rank[t]] - poff[c]);
  }
}

template <int M, bool DIRECT>
cudaError_t launch_cluster(const LoopArgs &a, size_t smem, cudaStream_t st) {
  auto kern = fps_loop_cluster<M, DIRECT>;
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

template <bool DIRECT>
cudaError_t launch_m(const LoopArgs &a, int m, size_t smem, cudaStream_t st) {
  switch (m) {
    case 1: return launch_cluster<1, DIRECT>(a, smem, st);
    case 2: return launch_cluster<2, DIRECT>(a, smem, st);
    case 3: return launch_cluster<3, DIRECT>(a, smem, st);
    case 4: return launch_cluster<4, DIRECT>(a, smem, st);
    case 6: return launch_cluster<6, DIRECT>(a, smem, st);
    case 8: return launch_cluster<8, DIRECT>(a, smem, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

size_t loop_smem_bytes(uint32_t pts, uint32_t leaves, uint32_t extra, uint32_t tab) {
  return (size_t)pts * 16 + (size_t)leaves * 32 + (size_t)extra * 4 + (size_t)tab * 4;
}

int loop_max_smem() {
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return optin - (int)sizeof(SharedCtl) - 1024;
}

int loop_leaves_per_thread(uint32_t leaves) {
  static const int ms[] = {1, 2, 3, 4, 6, 8};
  for (int m : ms)
    if ((uint32_t)m * kLoopThreads >= leaves) return m;
  return 0;
}

cudaError_t run_loop(const LoopArgs &a, const LoopPlan &plan, cudaStream_t st,
                     uint32_t &launches) {
  if (plan.mode != 0 || a.P > (uint32_t)kMaxClusterP) return cudaErrorInvalidValue;
  const cudaError_t err = plan.direct
                              ? launch_m<true>(a, plan.leaves_per_thread, plan.smem_bytes, st)
                              : launch_m<false>(a, plan.leaves_per_thread, plan.smem_bytes, st);
  launches += 1;
  return err;
}

cudaError_t run_epilogue(const uint32_t *out_rank, const uint32_t *out_count,
                         const uint32_t *perm, const uint32_t *poff, uint32_t B,
                         uint32_t k, uint64_t *out, cudaStream_t st,
                         uint32_t &launches) {
  const uint64_t total = (uint64_t)B * k;
  uint32_t blocks = (uint32_t)((total + 255) / 256);
  if (blocks > 4096) blocks = 4096;
  if (blocks == 0) return cudaSuccess;
  epilogue_kernel<<<blocks, 256, 0, st>>>(out_rank, out_count, perm, poff, B, k, out);
  launches += 1;
  return cudaGetLastError();
}

}  // namespace nsfps
