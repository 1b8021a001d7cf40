// nsfps_group.cu -- grouping after sampling, the step that follows FPS in
// PointNet++-style pipelines: the ball query around the sampled centres, the
// gather of the sampled points, and the grouped coordinates relative to each
// centre.  satreeby/ns_fps stops at the sample indices (src/yuezu_fps.cpp:676-730);
// these operators have no counterpart there.
//
// Ball query semantics (PointNet++ query_ball_point): for centre j, the first
// `nsample` points k of its cloud in index order with d2 < radius * radius,
// where d2 = (dx*dx + dy*dy) + dz*dz and dx = x_k - cx, each operation fp32
// rounded to nearest without contraction (the sampler's distance form,
// src/yuezu_fps.cpp:205-209).  Unfilled slots repeat the first hit; a centre
// without hits gets index 0 in every slot.  Indices are within the cloud.
//
// Grid.  Per cloud: the box of its finite points, split into cells at least
// 1.01 r wide on every axis (at most 4096 per axis, and a cap on the cloud's
// cell count).  Cell coordinates are computed in double, so the rounding of
// the cell arithmetic is far below the 1 % margin: a hit lies within
// r (1 + 2^-22) of the centre on each axis, hence in a cell at most one away
// from the centre's on each axis, and the 27 neighbouring cells hold every
// hit.  Points with a non-finite coordinate can never be hits and lie in no
// cell.
//
// Order.  A stable sort by cell keeps each cell's points in index order, so
// only the first `nsample` hits of a cell can be among the centre's first
// `nsample`; the query keeps those per cell in shared memory and merges the
// (at most 27) sorted lists with warp-wide minima.
#include <algorithm>
#include <cmath>

#include "nsfps_kernels.h"

namespace nsfps {

namespace {

constexpr uint32_t kFull = 0xffffffffu;
constexpr uint32_t kNone = 0xffffffffu;
constexpr uint32_t kAxisCells = 4096u;

__device__ __forceinline__ uint32_t offset_owner(const uint32_t *__restrict__ off, uint32_t B,
                                                 uint32_t i) {
  // largest c < B with off[c] <= i
  uint32_t lo = 0, hi = B;
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) >> 1;
    if (off[mid] <= i) lo = mid; else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ bool finite3(float x, float y, float z) {
  return isfinite(x) && isfinite(y) && isfinite(z);
}

// Float <-> unsigned integer with the same order (non-NaN floats), so that
// atomicMin / atomicMax on the integers give float minima / maxima.
__device__ __forceinline__ uint32_t ordered_bits(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float ordered_float(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

// Box of each cloud's finite points as ordered integers: enc[3c + a] = min,
// enc[3B + 3c + a] = max (set to 0xffffffff / 0 beforehand).  Grid
// (slices, B): slice x of cloud c reduces its share and merges atomically.
__global__ void __launch_bounds__(256)
group_bbox(const float *__restrict__ xyz, const uint32_t *__restrict__ poff, uint32_t B,
           uint32_t *__restrict__ enc) {
  for (uint32_t c = blockIdx.y; c < B; c += gridDim.y) {
    const uint32_t s = poff[c], e = poff[c + 1];
    const uint32_t per = (e - s + gridDim.x - 1) / gridDim.x;
    const uint32_t b0 = s + blockIdx.x * per, b1 = min(e, b0 + per);
    uint32_t mn[3] = {kNone, kNone, kNone}, mx[3] = {0u, 0u, 0u};
    for (uint32_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) {
      const float x = xyz[3 * (size_t)i], y = xyz[3 * (size_t)i + 1], z = xyz[3 * (size_t)i + 2];
      if (!finite3(x, y, z)) continue;
      const uint32_t o[3] = {ordered_bits(x), ordered_bits(y), ordered_bits(z)};
#pragma unroll
      for (int a = 0; a < 3; ++a) { mn[a] = min(mn[a], o[a]); mx[a] = max(mx[a], o[a]); }
    }
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      mn[a] = __reduce_min_sync(kFull, mn[a]);
      mx[a] = __reduce_max_sync(kFull, mx[a]);
    }
    if ((threadIdx.x & 31u) == 0)
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        if (mn[a] != kNone) atomicMin(&enc[3 * (size_t)c + a], mn[a]);
        if (mx[a] != 0u) atomicMax(&enc[3 * (size_t)B + 3 * (size_t)c + a], mx[a]);
      }
  }
}

// Cell layout of each cloud: cells at least h_min wide per axis, at most
// kAxisCells per axis and cbase[c + 1] - cbase[c] (>= 1) in all.
__global__ void group_grid(const uint32_t *__restrict__ enc, const uint32_t *__restrict__ cbase,
                           uint32_t B, double h_min, GroupGrid *__restrict__ grids) {
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= B) return;
  const uint64_t cap = cbase[c + 1] - cbase[c];
  // no finite point: a 0-extent box at the origin
  const bool any = enc[3 * (size_t)c] != kNone;
  uint32_t g[3];
  double ext[3];
  GroupGrid gr;
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    const double lo = any ? (double)ordered_float(enc[3 * (size_t)c + a]) : 0.0;
    const double hi = any ? (double)ordered_float(enc[3 * (size_t)B + 3 * (size_t)c + a]) : 0.0;
    ext[a] = hi - lo;  // exact enough in double, never overflows
    const double q = ext[a] / h_min;  // h_min = inf gives 0
    g[a] = q >= (double)kAxisCells ? kAxisCells : (q >= 1.0 ? (uint32_t)q : 1u);
    gr.lo[a] = lo;
  }
  while ((uint64_t)g[0] * g[1] * g[2] > cap) {
    const int a = (g[0] >= g[1] && g[0] >= g[2]) ? 0 : (g[1] >= g[2] ? 1 : 2);
    g[a] = (g[a] + 1u) / 2u;
  }
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    // cell width max(ext / g, h_min): ext == 0 gives 1 / h_min
    const double by_ext = ext[a] > 0.0 ? (double)g[a] / ext[a] : INFINITY;
    gr.inv[a] = fmin(by_ext, 1.0 / h_min);
    gr.g[a] = g[a];
  }
  gr.base = cbase[c];
  grids[c] = gr;
}

// Cell of a point on one axis (v >= lo): floor of its scaled offset, clamped
// to the last cell.
__device__ __forceinline__ uint32_t point_cell(float v, double lo, double inv, uint32_t g) {
  const double u = ((double)v - lo) * inv;
  const uint32_t c = u < (double)g ? (uint32_t)u : g - 1u;
  return c < g ? c : g - 1u;
}

// Cell of a centre on one axis, which may lie outside the grid: clamped to
// [-2, g + 1] (the neighbourhood of a clamped value holds the same cells of
// the grid), NaN to -2.
__device__ __forceinline__ int centre_cell(float v, double lo, double inv, uint32_t g) {
  double u = ((double)v - lo) * inv;
  u = fmax(u, -2.0);  // NaN -> -2
  u = fmin(u, (double)g + 1.0);
  return (int)floor(u);
}

__global__ void __launch_bounds__(256)
group_bin(const float *__restrict__ xyz, uint32_t n, const uint32_t *__restrict__ poff,
          uint32_t B, const GroupGrid *__restrict__ grids, uint32_t sentinel,
          uint32_t *__restrict__ keys, uint32_t *__restrict__ vals,
          uint32_t *__restrict__ count) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = xyz[3 * (size_t)i], y = xyz[3 * (size_t)i + 1], z = xyz[3 * (size_t)i + 2];
  uint32_t key = sentinel;
  if (finite3(x, y, z)) {
    const GroupGrid &gr = grids[offset_owner(poff, B, i)];
    const uint32_t cx = point_cell(x, gr.lo[0], gr.inv[0], gr.g[0]);
    const uint32_t cy = point_cell(y, gr.lo[1], gr.inv[1], gr.g[1]);
    const uint32_t cz = point_cell(z, gr.lo[2], gr.inv[2], gr.g[2]);
    key = gr.base + (cz * gr.g[1] + cy) * gr.g[0] + cx;
  }
  keys[i] = key;
  vals[i] = i;
  atomicAdd(&count[key], 1u);
}

// Sorted points as float4 (x, y, z, global point index as bits).
__global__ void __launch_bounds__(256)
group_gather(const uint32_t *__restrict__ vals, const float *__restrict__ xyz, uint32_t n,
             float4 *__restrict__ pts) {
  const uint32_t p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n) return;
  const uint32_t i = vals[p];
  pts[p] = make_float4(xyz[3 * (size_t)i], xyz[3 * (size_t)i + 1], xyz[3 * (size_t)i + 2],
                       __uint_as_float(i));
}

__device__ __forceinline__ uint32_t lanes_below(uint32_t x) {
  return x >= 32u ? kFull : (1u << x) - 1u;
}

// Largest s in [0, 26] with shfl(key, s) <= v (key non-decreasing over lanes
// 0..26; key[0] <= v).  All lanes take part.
__device__ __forceinline__ uint32_t last_le(uint32_t key, uint32_t v) {
  uint32_t s = 0;
#pragma unroll
  for (uint32_t step = 16; step; step >>= 1) {
    const uint32_t cand = s + step;
    const uint32_t kc = __shfl_sync(kFull, key, cand < 27u ? cand : 26u);
    if (cand < 27u && kc <= v) s = cand;
  }
  return s;
}

// One warp per centre.  Shared memory: 27 * S point ids per warp, the kept
// hits of neighbour cell s (ascending, as the cell's points are in index
// order) at [s * S, s * S + kept_s).
//
// The 27 neighbour cells are scanned as one concatenated range of L points,
// 32 per step: lane l takes position v0 + l, finds its cell by a binary search
// over the cells' starts in that range, and a hit's rank in its cell is the
// cell's earlier hits plus the hits of the lanes before it in the same cell
// (a cell's positions are contiguous lanes of the step).
__global__ void __launch_bounds__(256)
ball_query(const float4 *__restrict__ pts, const uint32_t *__restrict__ cstart,
           const GroupGrid *__restrict__ grids, const uint32_t *__restrict__ poff,
           const float *__restrict__ centers, const uint32_t *__restrict__ coff, uint32_t B,
           uint32_t m, float r2, uint32_t S, int64_t *__restrict__ out_idx,
           uint32_t *__restrict__ out_hits) {
  extern __shared__ uint32_t s_hits[];
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const uint32_t wpb = blockDim.x >> 5;
  uint32_t *hits = s_hits + (size_t)warp * 27u * S;
  const uint32_t lt = (1u << lane) - 1u;
  for (uint32_t j = blockIdx.x * wpb + warp; j < m; j += gridDim.x * wpb) {
    const uint32_t c = offset_owner(coff, B, j);
    const GroupGrid &gr = grids[c];
    const float qx = centers[3 * (size_t)j], qy = centers[3 * (size_t)j + 1],
                qz = centers[3 * (size_t)j + 2];
    const int cx = centre_cell(qx, gr.lo[0], gr.inv[0], gr.g[0]);
    const int cy = centre_cell(qy, gr.lo[1], gr.inv[1], gr.g[1]);
    const int cz = centre_cell(qz, gr.lo[2], gr.inv[2], gr.g[2]);
    // lane s < 27: neighbour cell (cx - 1 + s % 3, cy - 1 + s / 3 % 3, cz - 1 + s / 9)
    uint32_t cb = 0, clen = 0;  // its first sorted position and point count
    if (lane < 27u) {
      const int x = cx - 1 + (int)(lane % 3u), y = cy - 1 + (int)(lane / 3u % 3u),
                z = cz - 1 + (int)(lane / 9u);
      if (x >= 0 && x < (int)gr.g[0] && y >= 0 && y < (int)gr.g[1] && z >= 0 &&
          z < (int)gr.g[2]) {
        const uint32_t cell =
            gr.base + ((uint32_t)z * gr.g[1] + (uint32_t)y) * gr.g[0] + (uint32_t)x;
        cb = cstart[cell];
        clen = cstart[cell + 1] - cb;
      }
    }
    uint32_t incl = clen;
#pragma unroll
    for (uint32_t o = 1; o < 32u; o <<= 1) {
      const uint32_t t = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += t;
    }
    const uint32_t vs = incl - clen;  // start of cell `lane` in the concatenated range
    const uint32_t L = __shfl_sync(kFull, incl, 31);
    uint32_t cnt = 0;  // lane s: hits of cell s so far
    for (uint32_t v0 = 0; v0 < L; v0 += 32u) {
      const uint32_t v = v0 + lane;
      const uint32_t s = last_le(vs, v);
      const uint32_t sb = __shfl_sync(kFull, cb, s), svs = __shfl_sync(kFull, vs, s);
      bool hit = false;
      uint32_t gid = 0;
      if (v < L) {
        const float4 p = pts[sb + (v - svs)];
        const float dx = __fsub_rn(p.x, qx), dy = __fsub_rn(p.y, qy), dz = __fsub_rn(p.z, qz);
        const float d2 =
            __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz));
        hit = d2 < r2;
        gid = __float_as_uint(p.w);
      }
      const uint32_t hm = __ballot_sync(kFull, hit);
      if (hm) {
        const uint32_t first_lane = svs > v0 ? svs - v0 : 0u;  // <= lane
        const uint32_t before =
            __shfl_sync(kFull, cnt, s) + __popc(hm & lt & ~lanes_below(first_lane));
        if (hit && before < S) hits[s * S + before] = gid;
        // lane s: this step's lanes [a, b) belong to cell s
        const uint32_t a = min(max(vs, v0), v0 + 32u) - v0;
        const uint32_t b = min(max(vs + clen, v0), v0 + 32u) - v0;
        cnt += __popc(hm & lanes_below(b) & ~lanes_below(a));
      }
    }
    const uint32_t kept = min(cnt, S);  // lanes >= 27 hold 0
    uint32_t kincl = kept;
#pragma unroll
    for (uint32_t o = 1; o < 32u; o <<= 1) {
      const uint32_t t = __shfl_up_sync(kFull, kincl, o);
      if (lane >= o) kincl += t;
    }
    const uint32_t kex = kincl - kept;
    const uint32_t T = __shfl_sync(kFull, kincl, 31);  // ids kept over all cells
    __syncwarp();
    const uint32_t pb = poff[c];
    const size_t ob = (size_t)j * S;
    if (T <= 32u) {
      // lane i < T takes the i-th kept id; a bitonic sort orders them
      const uint32_t s = last_le(kex, lane);
      const uint32_t off = lane - __shfl_sync(kFull, kex, s);
      uint32_t val = lane < T ? hits[s * S + off] : kNone;
#pragma unroll
      for (uint32_t k = 2; k <= 32u; k <<= 1)
#pragma unroll
        for (uint32_t jj = k >> 1; jj; jj >>= 1) {
          const uint32_t other = __shfl_xor_sync(kFull, val, jj);
          const bool up = (lane & k) == 0u, low = (lane & jj) == 0u;
          val = (low == up) ? min(val, other) : max(val, other);
        }
      const uint32_t first = __shfl_sync(kFull, val, 0);
      const uint32_t fill = T ? first : pb;
      for (uint32_t q = lane; q < S; q += 32u)
        out_idx[ob + q] = (int64_t)((q < T ? val : fill) - pb);
    } else {
      // merge the sorted per-cell lists: the S smallest ids, ascending
      uint32_t ptr = 0;
      uint32_t head = kept > 0u ? hits[lane * S] : kNone;
      uint32_t first = kNone, mine = 0, t = 0;
      for (; t < S; ++t) {
        const uint32_t mn = __reduce_min_sync(kFull, head);
        if (mn == kNone) break;
        if (head == mn) {
          ++ptr;
          head = ptr < kept ? hits[lane * S + ptr] : kNone;
        }
        if (t == 0u) first = mn;
        if ((t & 31u) == lane) mine = mn;
        if ((t & 31u) == 31u) out_idx[ob + (t - 31u) + lane] = (int64_t)(mine - pb);
      }
      for (uint32_t q = (t & ~31u) + lane; q < S; q += 32u)
        out_idx[ob + q] = (int64_t)((q < t ? mine : first) - pb);
    }
    if (lane == 0 && out_hits) out_hits[j] = min(T, S);
    __syncwarp();  // the hit lists are rewritten for the next centre
  }
}

// out[j] = xyz[poff[c] + idx[j]] for the cloud c of entry j; an index outside
// its cloud writes NaNs and sets bit 0 of *err.
__global__ void __launch_bounds__(256)
gather_points_kernel(const float *__restrict__ xyz, const uint32_t *__restrict__ poff,
                     const int64_t *__restrict__ idx, const uint32_t *__restrict__ ioff,
                     uint32_t B, uint32_t m, float *__restrict__ out,
                     uint32_t *__restrict__ err) {
  const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= m) return;
  const uint32_t c = offset_owner(ioff, B, j);
  const int64_t v = idx[j];
  const int64_t nc = (int64_t)poff[c + 1] - (int64_t)poff[c];
  if (v < 0 || v >= nc) {
    const float nan = __int_as_float(0x7fc00000);
    out[3 * (size_t)j] = out[3 * (size_t)j + 1] = out[3 * (size_t)j + 2] = nan;
    atomicOr(err, 1u);
    return;
  }
  const size_t p = (size_t)poff[c] + (size_t)v;
  out[3 * (size_t)j] = xyz[3 * p];
  out[3 * (size_t)j + 1] = xyz[3 * p + 1];
  out[3 * (size_t)j + 2] = xyz[3 * p + 2];
}

// out[(j * S + s) * 3 + a] = xyz[point idx[j * S + s] of j's cloud][a] -
// centers[j][a]; an index outside its cloud writes NaNs and sets bit 0 of *err.
__global__ void __launch_bounds__(256)
group_points_kernel(const float *__restrict__ xyz, const uint32_t *__restrict__ poff,
                    const float *__restrict__ centers, const uint32_t *__restrict__ coff,
                    uint32_t B, uint64_t total, uint32_t S, const int64_t *__restrict__ idx,
                    float *__restrict__ out, uint32_t *__restrict__ err) {
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= total) return;
  const uint32_t j = (uint32_t)(t / S);
  const uint32_t c = offset_owner(coff, B, j);
  const int64_t v = idx[t];
  const int64_t nc = (int64_t)poff[c + 1] - (int64_t)poff[c];
  if (v < 0 || v >= nc) {
    const float nan = __int_as_float(0x7fc00000);
    out[3 * t] = out[3 * t + 1] = out[3 * t + 2] = nan;
    atomicOr(err, 1u);
    return;
  }
  const size_t p = (size_t)poff[c] + (size_t)v;
#pragma unroll
  for (int a = 0; a < 3; ++a) out[3 * t + a] = __fsub_rn(xyz[3 * p + a], centers[3 * (size_t)j + a]);
}

inline uint32_t cdiv32(uint64_t a, uint64_t b) { return (uint32_t)((a + b - 1) / b); }

}  // namespace

// Warps per block of the ball query for S samples per centre: 27 * S ids of
// shared memory per warp, at most 256 threads and 64 KB per block.
int ball_query_warps(uint32_t S) {
  int w = 8;
  while (w > 1 && (size_t)w * 27u * S * 4u > (64u << 10)) w >>= 1;
  return w;
}

size_t ball_query_smem(uint32_t S) { return (size_t)ball_query_warps(S) * 27u * S * 4u; }

cudaError_t run_ball_query(const GroupArgs &a, cudaStream_t st, uint32_t &launches,
                           cudaEvent_t ev_query_begin, cudaEvent_t ev_query_end) {
  cudaError_t err;
  if (a.m == 0) return cudaSuccess;
  // box: minima start at the largest ordered value, maxima at the smallest
  if ((err = cudaMemsetAsync(a.box, 0xff, sizeof(uint32_t) * 3 * (size_t)a.B, st))) return err;
  if ((err = cudaMemsetAsync(a.box + 3 * (size_t)a.B, 0, sizeof(uint32_t) * 3 * (size_t)a.B, st)))
    return err;
  const uint32_t slices = std::max(1u, std::min(cdiv32(a.max_cloud, 2048), 1024u));
  group_bbox<<<dim3(slices, std::min(a.B, 65535u)), 256, 0, st>>>(a.xyz, a.poff, a.B, a.box);
  group_grid<<<cdiv32(a.B, 128), 128, 0, st>>>(a.box, a.cbase, a.B, a.h_min, a.grids);
  launches += 2;
  if ((err = cudaMemsetAsync(a.cstart, 0, sizeof(uint32_t) * ((size_t)a.cells + 1), st)))
    return err;
  uint32_t *keys = a.keys0, *vals = a.vals0;
  if (a.n > 0) {
    group_bin<<<cdiv32(a.n, 256), 256, 0, st>>>(a.xyz, a.n, a.poff, a.B, a.grids, a.cells,
                                                 a.keys0, a.vals0, a.cstart);
    launches += 1;
    if ((err = run_sort_pairs(&keys, &vals, a.keys1, a.vals1, a.n, a.cells, a.hist, a.partial,
                              st, launches)))
      return err;
  }
  if ((err = run_exclusive_scan(a.cstart, a.cstart, a.cells + 1, a.partial, st, launches)))
    return err;
  if (a.n > 0) {
    group_gather<<<cdiv32(a.n, 256), 256, 0, st>>>(vals, a.xyz, a.n, a.pts);
    launches += 1;
  }
  const int warps = ball_query_warps(a.S);
  const size_t smem = ball_query_smem(a.S);
  if ((err = cudaFuncSetAttribute(ball_query, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem)))
    return err;
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ball_query, 32 * warps, smem);
  const uint32_t want = cdiv32(a.m, (uint32_t)warps);
  const uint32_t cap = (uint32_t)std::max(1, sms * std::max(per_sm, 1));
  if (ev_query_begin && (err = cudaEventRecord(ev_query_begin, st))) return err;
  ball_query<<<std::min(want, cap), 32 * warps, smem, st>>>(
      a.pts, a.cstart, a.grids, a.poff, a.centers, a.coff, a.B, a.m, a.r2, a.S, a.out_idx,
      a.out_hits);
  launches += 1;
  if ((err = cudaGetLastError())) return err;
  if (ev_query_end && (err = cudaEventRecord(ev_query_end, st))) return err;
  return cudaSuccess;
}

cudaError_t run_gather_points(const float *xyz, const uint32_t *poff, const int64_t *idx,
                              const uint32_t *ioff, uint32_t B, uint32_t m, float *out,
                              uint32_t *err_flag, cudaStream_t st, uint32_t &launches) {
  if (m == 0) return cudaSuccess;
  gather_points_kernel<<<cdiv32(m, 256), 256, 0, st>>>(xyz, poff, idx, ioff, B, m, out,
                                                       err_flag);
  launches += 1;
  return cudaGetLastError();
}

cudaError_t run_group_points(const float *xyz, const uint32_t *poff, const float *centers,
                             const uint32_t *coff, uint32_t B, uint32_t m, uint32_t S,
                             const int64_t *idx, float *out, uint32_t *err_flag, cudaStream_t st,
                             uint32_t &launches) {
  const uint64_t total = (uint64_t)m * S;
  if (total == 0) return cudaSuccess;
  group_points_kernel<<<cdiv32(total, 256), 256, 0, st>>>(xyz, poff, centers, coff, B, total, S,
                                                          idx, out, err_flag);
  launches += 1;
  return cudaGetLastError();
}

}  // namespace nsfps
