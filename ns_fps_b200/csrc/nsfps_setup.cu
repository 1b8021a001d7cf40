// nsfps_setup.cu -- per-call setup of the sampling engine, all on the GPU:
//
//   1. bin_points      : quantise every point to its cell and bucket exactly as
//                        Point3D::compute_block_indices / compute_morton_code do
//                        (src/yuezu_fps.cpp:170-199, :411-416); key = bucket
//                        offset of the cloud + bucket.
//   2. stable LSD radix sort of (key, point) -- 8-bit digits, one upsweep /
//      scan / downsweep per digit.  Stability reproduces the reference's flat
//      leaf order: buckets ascending, points of a bucket in input order
//      (src/yuezu_fps.cpp:277-283, :431-438).
//   3. gather_points   : sorted float4 (x, y, z, d0) with d0 the distance to the
//                        cloud's first point, already min'ed against FLT_MAX
//                        (build_multilevel_cache, :418-438), plus run starts.
//   4. leaves          : runs of <= kLeafSize points of one bucket; per leaf the
//                        bounding box, the first maximum of d0 and the cell(s)
//                        whose cube membership selects the leaf.
//   5. plan            : for candidate CTA counts per cloud (leaves dealt
//                        round-robin to the CTAs), the largest point and leaf
//                        counts any CTA would hold, so the host can size
//                        shared memory.
//
// Everything here is O(N) memory; no array is sized by the number of buckets.
#include <algorithm>
#include <cfloat>

#include "nsfps_internal.cuh"
#include "nsfps_kernels.h"

namespace nsfps {

namespace {

constexpr uint32_t kFull = 0xffffffffu;

// ------------------------------------------------------------------ scans
// Three-phase device-wide scans over uint32 (sum or max).  Tile = 4096.
constexpr int kScanThreads = 512;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

template <bool MAX>
__device__ __forceinline__ uint32_t sop(uint32_t a, uint32_t b) {
  return MAX ? (a > b ? a : b) : a + b;
}

// Block-wide exclusive scan of one value per thread; returns the exclusive
// prefix and writes the block total.  s_warp holds >= 32 entries.
template <bool MAX>
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v,
                                                    uint32_t *s_warp,
                                                    uint32_t &total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t t = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl = sop<MAX>(incl, t);
  }
  uint32_t excl = __shfl_up_sync(kFull, incl, 1);
  if (lane == 0) excl = 0;
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < nwarps ? s_warp[lane] : 0;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t t = __shfl_up_sync(kFull, wi, o);
      if (lane >= o) wi = sop<MAX>(wi, t);
    }
    uint32_t we = __shfl_up_sync(kFull, wi, 1);
    if (lane == 0) we = 0;
    if (lane < nwarps) s_warp[lane] = we;
    if (lane == nwarps - 1) s_warp[32] = wi;
  }
  __syncthreads();
  const uint32_t res = sop<MAX>(s_warp[warp], excl);
  total = s_warp[32];
  __syncthreads();
  return res;
}

template <bool MAX>
__global__ void __launch_bounds__(kScanThreads)
scan_reduce(const uint32_t *__restrict__ in, uint32_t n,
            uint32_t *__restrict__ partial) {
  __shared__ uint32_t s_warp[33];
  const uint64_t base = (uint64_t)blockIdx.x * kScanTile + threadIdx.x * kScanItems;
  uint32_t acc = 0;
#pragma unroll
  for (int j = 0; j < kScanItems; ++j)
    if (base + j < n) acc = sop<MAX>(acc, in[base + j]);
  uint32_t total;
  block_excl_scan<MAX>(acc, s_warp, total);
  if (threadIdx.x == 0) partial[blockIdx.x] = total;
}

// Exclusive scan of the tile partials in place; partial[n] = grand total.
template <bool MAX>
__global__ void __launch_bounds__(1024)
scan_partials(uint32_t *partial, uint32_t n) {
  __shared__ uint32_t s_warp[33];
  uint32_t carry = 0;
  for (uint32_t base = 0; base < n; base += 1024) {
    const uint32_t i = base + threadIdx.x;
    const uint32_t v = i < n ? partial[i] : 0;
    uint32_t total;
    const uint32_t ex = block_excl_scan<MAX>(v, s_warp, total);
    if (i < n) partial[i] = sop<MAX>(carry, ex);
    carry = sop<MAX>(carry, total);
  }
  if (threadIdx.x == 0) partial[n] = carry;
}

template <bool MAX, bool INCLUSIVE>
__global__ void __launch_bounds__(kScanThreads)
scan_final(const uint32_t *in, uint32_t *out, uint32_t n,
           const uint32_t *__restrict__ partial) {
  // in and out may be the same array: every thread reads its own items
  // before the block barrier inside block_excl_scan and writes them after.
  __shared__ uint32_t s_warp[33];
  const uint64_t base = (uint64_t)blockIdx.x * kScanTile + threadIdx.x * kScanItems;
  uint32_t v[kScanItems];
  uint32_t acc = 0;
#pragma unroll
  for (int j = 0; j < kScanItems; ++j) {
    v[j] = (base + j < n) ? in[base + j] : 0;
    acc = sop<MAX>(acc, v[j]);
  }
  uint32_t total;
  uint32_t run = block_excl_scan<MAX>(acc, s_warp, total);
  run = sop<MAX>(partial[blockIdx.x], run);
#pragma unroll
  for (int j = 0; j < kScanItems; ++j) {
    const uint32_t nxt = sop<MAX>(run, v[j]);
    if (base + j < n) out[base + j] = INCLUSIVE ? nxt : run;
    run = nxt;
  }
}

template <bool MAX, bool INCLUSIVE>
void device_scan(const uint32_t *in, uint32_t *out, uint32_t n,
                 uint32_t *partial, cudaStream_t st, uint32_t &launches) {
  const uint32_t tiles = (n + kScanTile - 1) / kScanTile;
  if (tiles == 0) return;
  scan_reduce<MAX><<<tiles, kScanThreads, 0, st>>>(in, n, partial);
  scan_partials<MAX><<<1, 1024, 0, st>>>(partial, tiles);
  scan_final<MAX, INCLUSIVE><<<tiles, kScanThreads, 0, st>>>(in, out, n, partial);
  launches += 3;
}

// ------------------------------------------------------------- radix sort
// Tiles of 8 warps x R rounds x 32 lanes keys: R = 16 (4096 keys) for large
// inputs, R = 4 (1024 keys) below kSmallSortKeys so that small sorts still
// spread over the SMs.
constexpr int kRsThreads = 256;
// Fused setup of small clouds: threads per CTA, bits of the local point index
// in a sort word.
constexpr int kSmallThreads = 1024;
constexpr int kSmallWarps = kSmallThreads / 32;
// Largest sort rounds (words per lane) whose cloud is staged in shared memory.
constexpr int kSmallStageRounds = 10;
constexpr int kSmallIdxBits = 15;
constexpr uint32_t kSmallSortKeys = 1u << 19;

template <int R>
__global__ void __launch_bounds__(kRsThreads)
radix_upsweep(const uint32_t *__restrict__ kin, uint32_t n, int shift,
              uint32_t *__restrict__ hist, uint32_t ntiles) {
  constexpr int kTile = 8 * R * 32;
  __shared__ uint32_t cnt[256];
  cnt[threadIdx.x] = 0;
  __syncthreads();
  const uint64_t base = (uint64_t)blockIdx.x * kTile;
#pragma unroll 4
  for (int r = 0; r < kTile / kRsThreads; ++r) {
    const uint64_t idx = base + r * kRsThreads + threadIdx.x;
    if (idx < n) atomicAdd(&cnt[(kin[idx] >> shift) & 255u], 1u);
  }
  __syncthreads();
  hist[(uint64_t)threadIdx.x * ntiles + blockIdx.x] = cnt[threadIdx.x];
}

// Stable scatter: warp w of a tile owns keys [w*R*32, (w+1)*R*32) of the tile
// in R ordered rounds of 32; ranks inside a round come from __match_any_sync.
template <int R>
__global__ void __launch_bounds__(kRsThreads)
radix_downsweep(const uint32_t *__restrict__ kin,
                const uint32_t *__restrict__ vin, uint32_t *__restrict__ kout,
                uint32_t *__restrict__ vout, uint32_t n, int shift,
                const uint32_t *__restrict__ hist, uint32_t ntiles) {
  constexpr int kTile = 8 * R * 32;
  __shared__ uint32_t wcount[8][256];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 8 * 256; i += kRsThreads) (&wcount[0][0])[i] = 0;
  __syncthreads();
  const uint64_t base = (uint64_t)blockIdx.x * kTile + warp * (R * 32);
  const uint32_t lt = (1u << lane) - 1u;
  uint32_t key[R], val[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const uint64_t idx = base + r * 32 + lane;
    const bool valid = idx < n;
    key[r] = valid ? kin[idx] : 0u;
    val[r] = valid ? vin[idx] : 0u;
    const uint32_t d = valid ? ((key[r] >> shift) & 255u) : (256u + lane);
    const uint32_t peers = __match_any_sync(kFull, d);
    if (valid && (peers & lt) == 0) wcount[warp][d] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  {
    const int d = tid;  // 256 threads == 256 digits
    uint32_t running = hist[(uint64_t)d * ntiles + blockIdx.x];
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t c = wcount[w][d];
      wcount[w][d] = running;
      running += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const uint64_t idx = base + r * 32 + lane;
    const bool valid = idx < n;
    const uint32_t d = valid ? ((key[r] >> shift) & 255u) : (256u + lane);
    const uint32_t peers = __match_any_sync(kFull, d);
    if (valid) {
      const uint32_t pos = wcount[warp][d] + __popc(peers & lt);
      kout[pos] = key[r];
      vout[pos] = val[r];
    }
    __syncwarp();
    if (valid && (peers & lt) == 0) wcount[warp][d] += __popc(peers);
    __syncwarp();
  }
}

// ------------------------------------------------------------- binning
__device__ __forceinline__ uint32_t cloud_of(const uint32_t *__restrict__ poff,
                                             uint32_t B, uint32_t p) {
  // largest c < B with poff[c] <= p
  uint32_t lo = 0, hi = B;
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) >> 1;
    if (poff[mid] <= p) lo = mid; else hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(256)
bin_points(const float *__restrict__ xyz, uint32_t n,
           const uint32_t *__restrict__ poff, uint32_t B,
           const uint32_t *__restrict__ rid, const RangeDev *__restrict__ ranges,
           const uint32_t *__restrict__ boff, uint32_t *__restrict__ keys,
           uint32_t *__restrict__ vals) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t c = cloud_of(poff, B, i);
  const RangeDev &r = ranges[rid[c]];
  uint32_t cx, cy, cz;
  cell_of(r, xyz[3ull * i], xyz[3ull * i + 1], xyz[3ull * i + 2], cx, cy, cz);
  keys[i] = boff[c] + bucket_of_cell(r, cx, cy, cz);
  vals[i] = i;
}

__global__ void __launch_bounds__(256)
gather_points(const uint32_t *__restrict__ keys,
              const uint32_t *__restrict__ vals, const float *__restrict__ xyz,
              uint32_t n, const uint32_t *__restrict__ poff, uint32_t B,
              float4 *__restrict__ pts, uint32_t *__restrict__ perm,
              uint32_t *__restrict__ runflag) {
  const uint32_t p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n) return;
  const uint32_t v = vals[p];
  const uint32_t c = cloud_of(poff, B, v);
  const uint64_t q0 = 3ull * poff[c];
  const float x = xyz[3ull * v], y = xyz[3ull * v + 1], z = xyz[3ull * v + 2];
  const float d = sqdist(x, y, z, xyz[q0], xyz[q0 + 1], xyz[q0 + 2]);
  pts[p] = make_float4(x, y, z, (d < FLT_MAX) ? d : FLT_MAX);
  perm[p] = v;
  runflag[p] = (p == 0 || keys[p] != keys[p - 1]) ? p : 0u;
}

__global__ void __launch_bounds__(256)
leaf_flags(const uint32_t *__restrict__ run_start, uint32_t n,
           uint32_t *__restrict__ flag) {
  const uint32_t p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p < n) flag[p] = ((p - run_start[p]) % kLeafSize) == 0 ? 1u : 0u;
}

__global__ void __launch_bounds__(256)
leaf_scatter(const uint32_t *__restrict__ run_start,
             const uint32_t *__restrict__ leafid, uint32_t n,
             uint32_t *__restrict__ leaf_start, uint32_t *__restrict__ nleaves) {
  const uint32_t p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n) return;
  const bool f = ((p - run_start[p]) % kLeafSize) == 0;
  if (f) leaf_start[leafid[p]] = p;
  if (p == n - 1) {
    const uint32_t L = leafid[p] + (f ? 1u : 0u);
    leaf_start[L] = n;
    *nleaves = L;
  }
}

// Leaf l = sorted points [s, e) of one bucket of range r: its bounding box,
// the first maximum of d0 and the cell(s) whose cube membership selects it.
// point(j) gives sorted point j as (x, y, z, d0).
template <typename PointAt>
__device__ __forceinline__ void build_leaf_of(uint32_t l, uint32_t s, uint32_t e, uint32_t bucket,
                                              const RangeDev &r, PointAt point,
                                              float4 *__restrict__ leaf_lo,
                                              float4 *__restrict__ leaf_hi,
                                              float *__restrict__ leaf_md,
                                              uint32_t *__restrict__ leaf_pre) {
  float lx = FLT_MAX, ly = FLT_MAX, lz = FLT_MAX;
  float hx = -FLT_MAX, hy = -FLT_MAX, hz = -FLT_MAX;
  float md = -1.0f;
  uint32_t slot = 0;
  for (uint32_t j = s; j < e; ++j) {
    const float4 p = point(j);
    lx = fminf(lx, p.x); ly = fminf(ly, p.y); lz = fminf(lz, p.z);
    hx = fmaxf(hx, p.x); hy = fmaxf(hy, p.y); hz = fmaxf(hz, p.z);
    if (p.w > md) { md = p.w; slot = j - s; }
  }
  // Coordinates that are +-inf must not narrow the box below the points.
  // (fminf/fmaxf already skip NaN; FLT_MAX sentinels only remain when every
  // coordinate of an axis is NaN, and such leaves never change.)
  uint32_t cell0 = 0, npre = 0;
  if (r.direct) {
    cell0 = pack_cell(gather_axis(r, 0, bucket), gather_axis(r, 1, bucket),
                      gather_axis(r, 2, bucket));
    npre = 1;
  } else {
    // every cell whose code is congruent to the bucket modulo total_blocks
    const uint64_t lim = 1ull << r.total_bits;
    for (int j = 0; j < kMaxPreimages; ++j) {
      const uint64_t code = (uint64_t)bucket + (uint64_t)j * r.total;
      if (code >= lim) break;
      const uint32_t cx = gather_axis(r, 0, (uint32_t)code);
      const uint32_t cy = gather_axis(r, 1, (uint32_t)code);
      const uint32_t cz = gather_axis(r, 2, (uint32_t)code);
      if (cx >= r.blocks[0] || cy >= r.blocks[1] || cz >= r.blocks[2]) continue;
      const uint32_t pc = pack_cell(cx, cy, cz);
      if (npre == 0) cell0 = pc;
      else leaf_pre[(uint64_t)l * kMaxPreimages + npre - 1] = pc;
      ++npre;
    }
  }
  const uint32_t cnt = e - s;
  leaf_lo[l] = make_float4(lx, ly, lz, __uint_as_float(cnt | (slot << 8) | (npre << 16)));
  leaf_hi[l] = make_float4(hx, hy, hz, __uint_as_float(cell0));
  leaf_md[l] = md;
}

__device__ __forceinline__ void build_leaf(uint32_t l, uint32_t s, uint32_t e, uint32_t bucket,
                                           const RangeDev &r, const float4 *__restrict__ pts,
                                           float4 *__restrict__ leaf_lo,
                                           float4 *__restrict__ leaf_hi,
                                           float *__restrict__ leaf_md,
                                           uint32_t *__restrict__ leaf_pre) {
  build_leaf_of(l, s, e, bucket, r, [&](uint32_t j) { return pts[j]; }, leaf_lo, leaf_hi, leaf_md,
                leaf_pre);
}

__global__ void __launch_bounds__(256)
leaf_meta(const uint32_t *__restrict__ keys, const float4 *__restrict__ pts,
          const uint32_t *__restrict__ leaf_start,
          const uint32_t *__restrict__ nleaves,
          const uint32_t *__restrict__ poff, uint32_t B,
          const uint32_t *__restrict__ rid, const RangeDev *__restrict__ ranges,
          const uint32_t *__restrict__ boff, float4 *__restrict__ leaf_lo,
          float4 *__restrict__ leaf_hi, float *__restrict__ leaf_md,
          uint32_t *__restrict__ leaf_pre) {
  const uint32_t l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l >= *nleaves) return;
  const uint32_t s = leaf_start[l], e = leaf_start[l + 1];
  const uint32_t c = cloud_of(poff, B, s);
  build_leaf(l, s, e, keys[s] - boff[c], ranges[rid[c]], pts, leaf_lo, leaf_hi, leaf_md,
             leaf_pre);
}

__global__ void cloud_leaf_offsets(const uint32_t *__restrict__ leafid,
                                   const uint32_t *__restrict__ poff, uint32_t B,
                                   const uint32_t *__restrict__ nleaves,
                                   uint32_t *__restrict__ loff) {
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c < B) loff[c] = leafid[poff[c]];
  if (c == 0) loff[B] = *nleaves;
}

// plan[3*i + {0,1,2}] = max points / leaves / extra preimages per CTA for the
// i-th candidate CTA count, with the leaves of a cloud dealt round-robin to
// its CTAs (leaf l of the cloud goes to CTA l % P).
__global__ void plan_partition(const float4 *__restrict__ leaf_lo,
                               const uint32_t *__restrict__ loff, uint32_t B,
                               const uint32_t *__restrict__ cand, int ncand,
                               uint32_t total_ctas, uint32_t *__restrict__ plan) {
  // one warp per (candidate CTA count, cloud, CTA); lanes stride its leaves
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;
  for (uint32_t t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < total_ctas; t += nwarps) {
    // decode t -> (candidate i, cloud c, cta j)
    uint32_t rem = t;
    int i = 0;
    for (; i < ncand; ++i) {
      const uint32_t span = cand[i] * B;
      if (rem < span) break;
      rem -= span;
    }
    if (i >= ncand) continue;  // uniform over the warp
    const uint32_t P = cand[i];
    const uint32_t c = rem / P, j = rem % P;
    const uint32_t l0 = loff[c], l1 = loff[c + 1];
    uint32_t pts = 0, leaves = 0, extra = 0;
    for (uint32_t l = l0 + j + lane * P; l < l1; l += 32u * P) {
      const uint32_t w = __float_as_uint(leaf_lo[l].w);
      const uint32_t npre = w >> 16;
      pts += w & 0xffu;
      extra += npre > 1 ? npre - 1 : 0;
      ++leaves;
    }
    pts = __reduce_add_sync(0xffffffffu, pts);
    leaves = __reduce_add_sync(0xffffffffu, leaves);
    extra = __reduce_add_sync(0xffffffffu, extra);
    if (lane == 0) {
      atomicMax(&plan[3 * i], pts);
      atomicMax(&plan[3 * i + 1], leaves);
      atomicMax(&plan[3 * i + 2], extra);
    }
  }
}

// ------------------------------------------------- small clouds, fused
// Clouds of at most kSmallCloudMax points (24 x 1024): steps 1-5 with one
// CTA of 1024 threads per cloud, in one launch for a single cloud and two
// for a batch, instead of ~25.  The results are the pipeline's, bit for bit:
// the sort is stable by bucket, so each cloud's sorted order, leaves and plan
// entries are the same.

// Lanes of `valid` whose digit equals this lane's (its low `bits` bits; the
// rest are 0): one ballot per bit, a fixed cost whatever the digits
// (__match_any_sync slows down with the number of distinct values).
__device__ __forceinline__ uint32_t digit_peers(uint32_t d, int bits, uint32_t valid) {
  uint32_t peers = valid;
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    if (b >= bits) break;
    const bool one = (d >> b) & 1u;
    const uint32_t bal = __ballot_sync(kFull, one);
    peers &= one ? bal : ~bal;
  }
  return peers;
}

// A range copied into shared memory by the CTA's first threads (word by word;
// visible after the next barrier).
__device__ __forceinline__ void load_range(RangeDev &dst, const RangeDev &src) {
  static_assert(sizeof(RangeDev) % 4 == 0, "RangeDev is copied as words");
  constexpr int kWords = (int)(sizeof(RangeDev) / 4);
  if ((int)threadIdx.x < kWords)
    reinterpret_cast<uint32_t *>(&dst)[threadIdx.x] =
        reinterpret_cast<const uint32_t *>(&src)[threadIdx.x];
}

// Per-warp digit counts, warp-major with a padded row so that the lanes of a
// warp touching different digits hit different banks.
constexpr int kHistRow = 257;

// Leaves and plan entries of cloud c, whose cnt leaves start at the sorted
// positions lstart[s ..] with buckets lbucket[s ..] (s = poff[c]) and whose
// leaf offset is L0: small_build_leaves runs build_leaf for each; small_plan,
// for every candidate CTA count P, the largest point, leaf and
// extra-preimage counts of the P CTAs the leaves are dealt to (leaf i of the
// cloud to CTA i % P), merged into the plan with atomicMax as plan_partition
// does.  All threads of the CTA call them; s_acc holds >= kSmallAcc words,
// s_red >= 3 * ncand.
constexpr int kSmallAcc = 2 * 512;
__device__ __forceinline__ void small_build_leaves(
    uint32_t c, uint32_t L0, uint32_t cnt, const RangeDev &r, const float4 *__restrict__ pts,
    const uint32_t *__restrict__ poff, const uint32_t *__restrict__ lstart,
    const uint32_t *__restrict__ lbucket, uint32_t *__restrict__ leaf_start,
    float4 *__restrict__ leaf_lo, float4 *__restrict__ leaf_hi, float *__restrict__ leaf_md,
    uint32_t *__restrict__ leaf_pre) {
  const uint32_t s = poff[c], e = poff[c + 1];
  for (uint32_t i = threadIdx.x; i < cnt; i += kSmallThreads) {
    const uint32_t st = lstart[s + i], en = i + 1 < cnt ? lstart[s + i + 1] : e;
    leaf_start[L0 + i] = st;
    build_leaf(L0 + i, st, en, lbucket[s + i], r, pts, leaf_lo, leaf_hi, leaf_md, leaf_pre);
  }
}

// small_build_leaves for a single cloud staged in shared memory: each point
// from its sort word (buf, local sorted order) and the staged coordinates,
// d0 recomputed exactly as the sorted points hold it, instead of a load from
// global memory.
__device__ __forceinline__ void small_build_leaves_staged(
    uint32_t s, uint32_t e, uint32_t cnt, const RangeDev &r, const uint32_t *buf,
    const float *s_xyz, float qx, float qy, float qz, const uint32_t *__restrict__ lstart,
    const uint32_t *__restrict__ lbucket, uint32_t *__restrict__ leaf_start,
    float4 *__restrict__ leaf_lo, float4 *__restrict__ leaf_hi, float *__restrict__ leaf_md,
    uint32_t *__restrict__ leaf_pre) {
  constexpr uint32_t kIdxMask = (1u << kSmallIdxBits) - 1u;
  auto point = [&](uint32_t j) {
    const uint32_t i = buf[j - s] & kIdxMask;
    const float x = s_xyz[3 * i], y = s_xyz[3 * i + 1], z = s_xyz[3 * i + 2];
    const float d = sqdist(x, y, z, qx, qy, qz);
    return make_float4(x, y, z, (d < FLT_MAX) ? d : FLT_MAX);
  };
  for (uint32_t i = threadIdx.x; i < cnt; i += kSmallThreads) {
    const uint32_t st = lstart[s + i], en = i + 1 < cnt ? lstart[s + i + 1] : e;
    leaf_start[i] = st;
    build_leaf_of(i, st, en, lbucket[s + i], r, point, leaf_lo, leaf_hi, leaf_md, leaf_pre);
  }
}

__device__ __forceinline__ void small_plan(uint32_t L0, uint32_t cnt,
                                           const float4 *__restrict__ leaf_lo,
                                           const uint32_t *__restrict__ cand, int ncand,
                                           uint32_t *__restrict__ plan, uint32_t *s_acc,
                                           uint32_t *s_red) {
  const int tid = threadIdx.x;
  if (ncand == 0) return;  // (uniform over the CTA)
  for (int i = tid; i < kSmallAcc; i += kSmallThreads) s_acc[i] = 0u;
  for (int i = tid; i < 3 * ncand; i += kSmallThreads) s_red[i] = 0u;
  __syncthreads();  // the leaf writes before the call are visible to the whole CTA
  // this thread's leaves i = tid + 1024 m: their points and extra preimages
  uint32_t my_pts = 0, my_extra = 0;
  for (uint32_t i = tid; i < cnt; i += kSmallThreads) {
    const uint32_t w = __float_as_uint(leaf_lo[L0 + i].w);
    const uint32_t npre = w >> 16;
    my_pts += w & 0xffu;
    my_extra += npre > 1 ? npre - 1 : 0u;
  }
  // per candidate, the sums of its CTAs at s_acc[2 (off + j) + {0, 1}]
  const int lane = tid & 31;
  uint32_t off = 0;
  for (int ci = 0; ci < ncand; ++ci) {
    const uint32_t P = cand[ci];
    if ((kSmallThreads % P) == 0) {
      // every leaf of this thread goes to CTA tid % P
      uint32_t vp = my_pts, ve = my_extra;
      if (P < 32) {  // fold the lanes of one residue within the warp first
#pragma unroll
        for (uint32_t o = 16; o >= 1; o >>= 1)
          if (o >= P) {
            vp += __shfl_xor_sync(kFull, vp, o);
            ve += __shfl_xor_sync(kFull, ve, o);
          }
      }
      if (P >= 32 || (uint32_t)lane < P) {
        const uint32_t j = (uint32_t)tid % P;
        if (vp) atomicAdd(&s_acc[2 * (off + j)], vp);
        if (ve) atomicAdd(&s_acc[2 * (off + j) + 1], ve);
      }
    } else {
      for (uint32_t i = tid; i < cnt; i += kSmallThreads) {
        const uint32_t w = __float_as_uint(leaf_lo[L0 + i].w);
        const uint32_t npre = w >> 16;
        atomicAdd(&s_acc[2 * (off + i % P)], w & 0xffu);
        if (npre > 1) atomicAdd(&s_acc[2 * (off + i % P) + 1], npre - 1);
      }
    }
    off += P;
  }
  __syncthreads();
  off = 0;
  for (int ci = 0; ci < ncand; ++ci) {
    const uint32_t P = cand[ci];
    for (uint32_t j = tid; j < P; j += kSmallThreads) {
      atomicMax(&s_red[3 * ci], s_acc[2 * (off + j)]);
      atomicMax(&s_red[3 * ci + 1], cnt > j ? (cnt - j + P - 1) / P : 0u);
      atomicMax(&s_red[3 * ci + 2], s_acc[2 * (off + j) + 1]);
    }
    off += P;
  }
  __syncthreads();
  for (int i = tid; i < 3 * ncand; i += kSmallThreads) atomicMax(&plan[i], s_red[i]);
}

// small_sort: the cloud's points as words bucket << 15 | local index in
// shared memory, sorted by an LSD radix sort over the bucket bits (8-bit
// digits; warp w holds words [w R 32, (w+1) R 32) in registers in R ordered
// rounds, so warp order, round order and lane order are the input order and
// the scatter keeps it); then the sorted float4 points and permutation, and
// the cloud's leaf starts, buckets and count (per-cloud scratch indexed from
// the cloud's first point).  STAGE (clouds of at most 10 x 1024 points)
// keeps the coordinates in shared memory for the gather.  A single cloud
// (gridDim.x == 1) goes on to its leaves and plan in the same launch.
template <int R>
__global__ void __launch_bounds__(kSmallThreads, 1)
small_sort(const float *__restrict__ xyz, const uint32_t *__restrict__ poff,
           const uint32_t *__restrict__ rid, const RangeDev *__restrict__ ranges,
           float4 *__restrict__ pts, uint32_t *__restrict__ perm,
           uint32_t *__restrict__ lstart, uint32_t *__restrict__ lbucket,
           uint32_t *__restrict__ lcount, uint32_t *__restrict__ leaf_start,
           float4 *__restrict__ leaf_lo, float4 *__restrict__ leaf_hi,
           float *__restrict__ leaf_md, uint32_t *__restrict__ leaf_pre,
           uint32_t *__restrict__ loff, uint32_t *__restrict__ nleaves,
           const uint32_t *__restrict__ cand, int ncand, uint32_t *__restrict__ plan) {
  constexpr bool STAGE = R <= kSmallStageRounds;
  extern __shared__ uint32_t small_sm[];
  uint32_t *buf = small_sm;                                  // R * 1024 words
  uint32_t *hist = small_sm + R * kSmallThreads;             // kSmallWarps x kHistRow
  float *s_xyz = reinterpret_cast<float *>(hist + kSmallWarps * kHistRow);  // STAGE: 3 R 1024
  __shared__ uint32_t s_warp[33];
  __shared__ RangeDev s_range;
  __shared__ uint32_t s_lut[3][1024];  // Morton spread of every axis index
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t c = blockIdx.x;
  const uint32_t s = poff[c], nc = poff[c + 1] - s;
  load_range(s_range, ranges[rid[c]]);
  __syncthreads();
  const RangeDev &r = s_range;
  for (uint32_t a = 0; a < 3; ++a)
    for (uint32_t v = tid; v < r.blocks[a]; v += kSmallThreads) s_lut[a][v] = spread_axis(r, (int)a, v);
  if (STAGE)
    for (uint32_t i = tid; i < 3 * nc; i += kSmallThreads) s_xyz[i] = xyz[3ull * s + i];
  __syncthreads();
  const uint32_t maxb = r.total - 1u;
  const int kb = maxb ? 32 - __clz(maxb) : 0;  // bits of the largest bucket

#pragma unroll 4
  for (uint32_t i = tid; i < nc; i += kSmallThreads) {
    uint32_t cx, cy, cz;
    if (STAGE) {
      cell_of(r, s_xyz[3 * i], s_xyz[3 * i + 1], s_xyz[3 * i + 2], cx, cy, cz);
    } else {
      const uint64_t q = 3ull * (s + i);
      cell_of(r, xyz[q], xyz[q + 1], xyz[q + 2], cx, cy, cz);
    }
    const uint32_t code = s_lut[0][cx] | s_lut[1][cy] | s_lut[2][cz];  // bucket_of_cell
    buf[i] = ((r.direct ? code : code % r.total) << kSmallIdxBits) | i;
  }
  __syncthreads();

  const uint32_t lt = (1u << lane) - 1u;
  const uint32_t wbase = (uint32_t)warp * (R * 32);
  uint32_t *const hrow = hist + warp * kHistRow;
  for (int shift = kSmallIdxBits; shift < kSmallIdxBits + kb; shift += 8) {
    const int dbits = min(8, kSmallIdxBits + kb - shift);  // digit bits in use
    uint32_t v[R];
#pragma unroll
    for (int q = 0; q < R; ++q) {
      const uint32_t idx = wbase + q * 32 + lane;
      v[q] = idx < nc ? buf[idx] : 0u;
    }
    for (int i = tid; i < kSmallWarps * kHistRow; i += kSmallThreads) hist[i] = 0u;
    __syncthreads();
#pragma unroll
    for (int q = 0; q < R; ++q) {
      const bool valid = wbase + q * 32 + lane < nc;
      const uint32_t d = (v[q] >> shift) & 255u;
      const uint32_t peers = digit_peers(d, dbits, __ballot_sync(kFull, valid));
      if (valid && (peers & lt) == 0) hrow[d] += __popc(peers);
      __syncwarp();
    }
    __syncthreads();
    {  // (digit, warp) -> first output position: digits ascending, warps ascending
      uint32_t tot = 0;
      if (tid < 256)
        for (int w = 0; w < kSmallWarps; ++w) tot += hist[w * kHistRow + tid];
      uint32_t all;
      uint32_t run = block_excl_scan<false>(tid < 256 ? tot : 0u, s_warp, all);
      if (tid < 256)
        for (int w = 0; w < kSmallWarps; ++w) {
          const uint32_t cnt = hist[w * kHistRow + tid];
          hist[w * kHistRow + tid] = run;
          run += cnt;
        }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < R; ++q) {
      const bool valid = wbase + q * 32 + lane < nc;
      const uint32_t d = (v[q] >> shift) & 255u;
      const uint32_t peers = digit_peers(d, dbits, __ballot_sync(kFull, valid));
      if (valid) buf[hrow[d] + __popc(peers & lt)] = v[q];
      __syncwarp();
      if (valid && (peers & lt) == 0) hrow[d] += __popc(peers);
      __syncwarp();
    }
    __syncthreads();
  }

  // sorted points with d0 (the distance to the cloud's first point)
  constexpr uint32_t kIdxMask = (1u << kSmallIdxBits) - 1u;
  const float qx = nc ? xyz[3ull * s] : 0.0f, qy = nc ? xyz[3ull * s + 1] : 0.0f,
              qz = nc ? xyz[3ull * s + 2] : 0.0f;
  {
#pragma unroll 4
    for (uint32_t p = tid; p < nc; p += kSmallThreads) {
      const uint32_t i = buf[p] & kIdxMask;
      float x, y, z;
      if (STAGE) {
        x = s_xyz[3 * i]; y = s_xyz[3 * i + 1]; z = s_xyz[3 * i + 2];
      } else {
        const uint64_t q = 3ull * (s + i);
        x = xyz[q]; y = xyz[q + 1]; z = xyz[q + 2];
      }
      const float d = sqdist(x, y, z, qx, qy, qz);
      pts[s + p] = make_float4(x, y, z, (d < FLT_MAX) ? d : FLT_MAX);
      perm[s + p] = s + i;
    }
  }

  // leaves: runs of one bucket cut every kLeafSize points; thread t walks the
  // sorted positions [t E, (t+1) E).  A stride divisible by 4 puts a warp's
  // reads of buf in at most 8 banks (E = 16: 2 banks, the c3 clouds' walk took
  // 38 k cycles), so such an E is made odd.
  uint32_t E = (nc + kSmallThreads - 1) / kSmallThreads;
  if ((E & 3u) == 0u) E += 1u;
  const uint32_t p0 = min(nc, (uint32_t)tid * E), p1 = min(nc, p0 + E);
  auto run_mark = [&](uint32_t p) {
    return (p == 0 || (buf[p] >> kSmallIdxBits) != (buf[p - 1] >> kSmallIdxBits)) ? p : 0u;
  };
  uint32_t m = 0;
  for (uint32_t p = p0; p < p1; ++p) m = max(m, run_mark(p));
  uint32_t unused;
  const uint32_t carry = block_excl_scan<true>(m, s_warp, unused);  // last run start before p0
  uint32_t cur = carry, nl = 0;
  for (uint32_t p = p0; p < p1; ++p) {
    cur = max(cur, run_mark(p));
    nl += ((p - cur) % kLeafSize) == 0 ? 1u : 0u;
  }
  uint32_t total;
  uint32_t li = block_excl_scan<false>(nl, s_warp, total);
  cur = carry;
  for (uint32_t p = p0; p < p1; ++p) {
    cur = max(cur, run_mark(p));
    if (((p - cur) % kLeafSize) == 0) {
      lstart[s + li] = s + p;
      lbucket[s + li] = buf[p] >> kSmallIdxBits;
      ++li;
    }
  }
  if (gridDim.x > 1) {
    if (tid == 0) lcount[c] = total;
    return;
  }
  // one cloud: leaf offset 0, its leaves and the plan here
  if (tid == 0) {
    loff[0] = 0u;
    loff[1] = total;
    *nleaves = total;
    leaf_start[total] = s + nc;
  }
  __syncthreads();  // lstart / lbucket / pts written above are visible to the CTA
  if (STAGE)
    small_build_leaves_staged(s, s + nc, total, r, buf, s_xyz, qx, qy, qz, lstart, lbucket,
                              leaf_start, leaf_lo, leaf_hi, leaf_md, leaf_pre);
  else
    small_build_leaves(c, 0u, total, r, pts, poff, lstart, lbucket, leaf_start, leaf_lo, leaf_hi,
                       leaf_md, leaf_pre);
  small_plan(0u, total, leaf_lo, cand, ncand, plan, hist, buf);
}

// small_leaves (batches): per cloud, its leaf offset (the leaves of the
// clouds before it), then its leaves and plan entries.
__global__ void __launch_bounds__(kSmallThreads, 1)
small_leaves(const float4 *__restrict__ pts, const uint32_t *__restrict__ poff, uint32_t B,
             const uint32_t *__restrict__ rid, const RangeDev *__restrict__ ranges,
             const uint32_t *__restrict__ lstart, const uint32_t *__restrict__ lbucket,
             const uint32_t *__restrict__ lcount, uint32_t *__restrict__ leaf_start,
             float4 *__restrict__ leaf_lo, float4 *__restrict__ leaf_hi,
             float *__restrict__ leaf_md, uint32_t *__restrict__ leaf_pre,
             uint32_t *__restrict__ loff, uint32_t *__restrict__ nleaves,
             const uint32_t *__restrict__ cand, int ncand, uint32_t *__restrict__ plan) {
  __shared__ uint32_t s_warp[33];
  __shared__ RangeDev s_range;
  __shared__ uint32_t s_acc[kSmallAcc], s_red[3 * kMaxCand];
  const int tid = threadIdx.x;
  const uint32_t c = blockIdx.x;
  load_range(s_range, ranges[rid[c]]);
  uint32_t before = 0, all = 0;
  for (uint32_t i = tid; i < B; i += kSmallThreads) {
    const uint32_t v = lcount[i];
    all += v;
    before += i < c ? v : 0u;
  }
  uint32_t L0, L;
  block_excl_scan<false>(before, s_warp, L0);  // (its barriers publish s_range)
  block_excl_scan<false>(all, s_warp, L);
  if (tid == 0) {
    loff[c] = L0;
    if (c + 1 == B) {
      loff[B] = L;
      *nleaves = L;
      leaf_start[L] = poff[B];
    }
  }
  const uint32_t cnt = lcount[c];
  small_build_leaves(c, L0, cnt, s_range, pts, poff, lstart, lbucket, leaf_start, leaf_lo,
                     leaf_hi, leaf_md, leaf_pre);
  small_plan(L0, cnt, leaf_lo, cand, ncand, plan, s_acc, s_red);
}

// compute_bbox (src/yuezu_fps.cpp:648-670) of each cloud, on the device: the
// per-axis minimum and maximum of the cloud's points.  The reference scans
// from point 0 with `v < min` / `max < v`, which never take a NaN, so a NaN
// survives only as point 0's own coordinate; elsewhere NaNs are skipped.
// (Signed zeros can differ in which zero wins, which the +-BOUNDARY_EPS
// applied afterwards makes irrelevant.)
//
// Three launches: bbox_init sets the per-cloud extremes to their identities,
// cloud_bbox reduces slices of every cloud (grid x = slices, y = clouds) and
// merges them with integer atomics on order-preserving encodings of the
// floats, and bbox_final decodes them in place and applies point 0's NaNs.
__device__ __forceinline__ uint32_t ordered_bits(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float ordered_float(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

__global__ void bbox_init(uint32_t *__restrict__ enc, uint32_t B) {
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= B) return;
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    enc[6 * (size_t)c + a] = 0xffffffffu;
    enc[6 * (size_t)c + 3 + a] = 0u;
  }
}

__global__ void __launch_bounds__(256)
cloud_bbox(const float *__restrict__ xyz, const uint32_t *__restrict__ poff, uint32_t B,
           uint32_t *__restrict__ enc) {
  for (uint32_t c = blockIdx.y; c < B; c += gridDim.y) {
    const uint32_t s = poff[c], e = poff[c + 1];
    const uint32_t per = (e - s + gridDim.x - 1) / gridDim.x;
    const uint32_t b0 = s + blockIdx.x * per, b1 = min(e, b0 + per);
    uint32_t mn[3] = {0xffffffffu, 0xffffffffu, 0xffffffffu}, mx[3] = {0u, 0u, 0u};
    for (uint32_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) {
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        const float v = xyz[3 * (size_t)i + a];
        if (v != v) continue;
        const uint32_t o = ordered_bits(v);
        mn[a] = min(mn[a], o);
        mx[a] = max(mx[a], o);
      }
    }
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      mn[a] = __reduce_min_sync(0xffffffffu, mn[a]);
      mx[a] = __reduce_max_sync(0xffffffffu, mx[a]);
    }
    if ((threadIdx.x & 31u) == 0)
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        if (mn[a] != 0xffffffffu) atomicMin(&enc[6 * (size_t)c + a], mn[a]);
        if (mx[a] != 0u) atomicMax(&enc[6 * (size_t)c + 3 + a], mx[a]);
      }
  }
}

__global__ void bbox_final(const float *__restrict__ xyz, const uint32_t *__restrict__ poff,
                           uint32_t B, uint32_t *__restrict__ enc) {
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= B) return;
  const uint32_t s = poff[c], e = poff[c + 1];
  const float inf = __int_as_float(0x7f800000);
  float *out = reinterpret_cast<float *>(enc);
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    const uint32_t omn = enc[6 * (size_t)c + a], omx = enc[6 * (size_t)c + 3 + a];
    float lo = omn == 0xffffffffu ? inf : ordered_float(omn);
    float hi = omx == 0u ? -inf : ordered_float(omx);
    if (e > s) {  // point 0 starts the scan: a NaN there is kept
      const float v0 = xyz[3 * (size_t)s + a];
      if (v0 != v0) lo = hi = v0;
    }
    out[6 * (size_t)c + a] = lo;
    out[6 * (size_t)c + 3 + a] = hi;
  }
}

inline uint32_t cdiv(uint64_t a, uint64_t b) { return (uint32_t)((a + b - 1) / b); }

}  // namespace

// ------------------------------------------------------------------ driver
cudaError_t run_cloud_bbox(const float *xyz, const uint32_t *poff, uint32_t B,
                           uint32_t max_cloud, float *out, cudaStream_t st, uint32_t &launches) {
  if (B == 0) return cudaSuccess;
  uint32_t *enc = reinterpret_cast<uint32_t *>(out);
  const uint32_t slices = std::max(1u, std::min(cdiv(max_cloud, 2048), 1024u));
  bbox_init<<<cdiv(B, 128), 128, 0, st>>>(enc, B);
  cloud_bbox<<<dim3(slices, std::min(B, 65535u)), 256, 0, st>>>(xyz, poff, B, enc);
  bbox_final<<<cdiv(B, 128), 128, 0, st>>>(xyz, poff, B, enc);
  launches += 3;
  return cudaGetLastError();
}

template <int R>
cudaError_t small_sort_opt_in() {
  return cudaFuncSetAttribute(small_sort<R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)small_setup_smem(R));
}

cudaError_t small_setup_prepare() {
  // the shared-memory opt-in of every instance, set outside stream capture
  cudaError_t err;
  if ((err = small_sort_opt_in<4>())) return err;
  if ((err = small_sort_opt_in<8>())) return err;
  if ((err = small_sort_opt_in<kSmallStageRounds>())) return err;
  if ((err = small_sort_opt_in<16>())) return err;
  return small_sort_opt_in<24>();
}

size_t small_setup_smem(int rounds) {
  // sort words, digit counts, and the staged coordinates of clouds of at
  // most kSmallStageRounds x 512 points
  const size_t words = (size_t)rounds * kSmallThreads + kSmallWarps * kHistRow +
                       (rounds <= kSmallStageRounds ? 3 * (size_t)rounds * kSmallThreads : 0);
  return sizeof(uint32_t) * words;
}

int small_setup_rounds(uint32_t max_cloud) {
  for (int r : {4, 8, kSmallStageRounds, 16, 24})
    if (max_cloud <= (uint32_t)r * kSmallThreads) return r;
  return 0;
}

uint32_t radix_tiles(uint32_t n) {
  return n < kSmallSortKeys ? cdiv(n, 8 * 4 * 32) : cdiv(n, 8 * 16 * 32);
}

cudaError_t run_sort_pairs(uint32_t **keys, uint32_t **vals, uint32_t *keys_alt,
                           uint32_t *vals_alt, uint32_t n, uint32_t max_key, uint32_t *hist,
                           uint32_t *partial, cudaStream_t st, uint32_t &launches) {
  if (n == 0) return cudaSuccess;
  int bits = 0;
  while (bits < 32 && ((max_key >> bits) != 0)) ++bits;
  const int passes = (bits + 7) / 8;
  uint32_t *kin = *keys, *vin = *vals, *kout = keys_alt, *vout = vals_alt;
  const bool small = n < kSmallSortKeys;
  const uint32_t ntiles = radix_tiles(n);
  for (int pass = 0; pass < passes; ++pass) {
    const int shift = pass * 8;
    if (small)
      radix_upsweep<4><<<ntiles, kRsThreads, 0, st>>>(kin, n, shift, hist, ntiles);
    else
      radix_upsweep<16><<<ntiles, kRsThreads, 0, st>>>(kin, n, shift, hist, ntiles);
    device_scan<false, false>(hist, hist, 256u * ntiles, partial, st, launches);
    if (small)
      radix_downsweep<4><<<ntiles, kRsThreads, 0, st>>>(kin, vin, kout, vout, n, shift, hist,
                                                        ntiles);
    else
      radix_downsweep<16><<<ntiles, kRsThreads, 0, st>>>(kin, vin, kout, vout, n, shift, hist,
                                                         ntiles);
    launches += 2;
    uint32_t *t;
    t = kin; kin = kout; kout = t;
    t = vin; vin = vout; vout = t;
  }
  *keys = kin;
  *vals = vin;
  return cudaGetLastError();
}

cudaError_t run_exclusive_scan(const uint32_t *in, uint32_t *out, uint32_t n,
                               uint32_t *partial, cudaStream_t st, uint32_t &launches) {
  device_scan<false, false>(in, out, n, partial, st, launches);
  return cudaGetLastError();
}

template <int R>
cudaError_t launch_small_sort(const SetupArgs &a, cudaStream_t st) {
  small_sort<R><<<a.B, kSmallThreads, small_setup_smem(R), st>>>(
      a.xyz, a.poff, a.rid, a.ranges, a.pts, a.perm, a.tmp0, a.tmp1, a.keys1, a.leaf_start,
      a.leaf_lo, a.leaf_hi, a.leaf_md, a.leaf_pre, a.loff, a.scalars + kScalarLeaves, a.cand,
      a.ncand, a.plan);
  return cudaGetLastError();
}

cudaError_t run_setup(const SetupArgs &a, cudaStream_t st, uint32_t &launches) {
  const uint32_t n = a.n;
  const uint32_t B = a.B;
  cudaError_t err;
  if ((err = cudaMemsetAsync(a.scalars, 0, sizeof(uint32_t) * 8, st))) return err;

  if (a.small_rounds) {  // every cloud fits one CTA: two launches
    if ((err = cudaMemsetAsync(a.plan, 0, sizeof(uint32_t) * 3 * a.ncand, st))) return err;
    switch (a.small_rounds) {
      case 4: err = launch_small_sort<4>(a, st); break;
      case 8: err = launch_small_sort<8>(a, st); break;
      case kSmallStageRounds: err = launch_small_sort<kSmallStageRounds>(a, st); break;
      case 16: err = launch_small_sort<16>(a, st); break;
      case 24: err = launch_small_sort<24>(a, st); break;
      default: return cudaErrorInvalidValue;
    }
    if (err) return err;
    launches += 1;
    if (B > 1) {  // the leaf offsets need every cloud's leaf count
      small_leaves<<<B, kSmallThreads, 0, st>>>(a.pts, a.poff, B, a.rid, a.ranges, a.tmp0,
                                                a.tmp1, a.keys1, a.leaf_start, a.leaf_lo,
                                                a.leaf_hi, a.leaf_md, a.leaf_pre, a.loff,
                                                a.scalars + kScalarLeaves, a.cand, a.ncand,
                                                a.plan);
      launches += 1;
    }
    return cudaGetLastError();
  }

  bin_points<<<cdiv(n, 256), 256, 0, st>>>(a.xyz, n, a.poff, B, a.rid, a.ranges,
                                           a.boff, a.keys0, a.vals0);
  launches += 1;

  // radix passes cover the largest possible key (total buckets - 1)
  uint32_t *kin = a.keys0, *vin = a.vals0;
  if ((err = run_sort_pairs(&kin, &vin, a.keys1, a.vals1, n, a.max_key, a.hist, a.partial,
                            st, launches)))
    return err;
  // kin / vin now hold the sorted keys and point ids
  gather_points<<<cdiv(n, 256), 256, 0, st>>>(kin, vin, a.xyz, n, a.poff, B, a.pts,
                                              a.perm, a.tmp0);
  launches += 1;
  device_scan<true, true>(a.tmp0, a.tmp0, n, a.partial, st, launches);  // run starts
  leaf_flags<<<cdiv(n, 256), 256, 0, st>>>(a.tmp0, n, a.tmp1);
  launches += 1;
  device_scan<false, false>(a.tmp1, a.tmp1, n, a.partial, st, launches);  // leaf ids
  leaf_scatter<<<cdiv(n, 256), 256, 0, st>>>(a.tmp0, a.tmp1, n, a.leaf_start,
                                             a.scalars + kScalarLeaves);
  leaf_meta<<<cdiv(n, 256), 256, 0, st>>>(kin, a.pts, a.leaf_start,
                                          a.scalars + kScalarLeaves, a.poff, B,
                                          a.rid, a.ranges, a.boff, a.leaf_lo,
                                          a.leaf_hi, a.leaf_md, a.leaf_pre);
  cloud_leaf_offsets<<<cdiv(B + 1, 128), 128, 0, st>>>(a.tmp1, a.poff, B,
                                                       a.scalars + kScalarLeaves,
                                                       a.loff);
  launches += 3;

  if ((err = cudaMemsetAsync(a.plan, 0, sizeof(uint32_t) * 3 * a.ncand, st))) return err;
  uint64_t total = 0;
  for (int i = 0; i < a.ncand; ++i) total += (uint64_t)a.cand_host[i] * B;
  if (total) {
    const uint32_t blocks = (uint32_t)((total + 7) / 8 < 4096 ? (total + 7) / 8 : 4096);  // 8 warps each
    plan_partition<<<blocks, 256, 0, st>>>(a.leaf_lo, a.loff, B, a.cand, a.ncand,
                                           (uint32_t)total, a.plan);
    launches += 1;
  }
  return cudaGetLastError();
}

}  // namespace nsfps
