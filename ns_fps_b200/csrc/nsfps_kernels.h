// nsfps_kernels.h -- device buffers and launch entry points shared by the
// setup kernels (nsfps_setup.cu), the sampling loop (nsfps_loop.cu) and the
// host orchestration (nsfps_capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "nsfps_internal.cuh"

namespace nsfps {

// indices into the small scalar block (uint32) of the workspace
enum : int {
  kScalarLeaves = 0,   // total number of leaves
  kScalarStatus = 1,   // loop status bits (kStatusTimeout ...)
  kScalarCount = 8
};
constexpr uint32_t kStatusTimeout = 1u;
constexpr uint32_t kStatusBadPlan = 2u;

constexpr int kMaxCand = 16;

// Points from which a single cloud takes the grid-wide round loop (build-time).
// Measured on B200 from 5,000 to 90,000 points, the grid-wide loop over 64 or
// 128 CTAs beats one 16-CTA cluster by 8 to 41 %; below a few thousand points
// the cluster's cheaper launch and barrier are kept.
#ifndef NSFPS_GRID_MIN_POINTS
#define NSFPS_GRID_MIN_POINTS 4096u
#endif

// Threads per CTA of the sampling loop; a thread owns up to 8 leaves
// (template instances 1, 2, 3, 4, 6, 8).  Must be a multiple of 32, at most
// 512 (a build-time choice: -DNSFPS_LOOP_THREADS=...).
#ifndef NSFPS_LOOP_THREADS
#define NSFPS_LOOP_THREADS 256
#endif
constexpr int kLoopThreads = NSFPS_LOOP_THREADS;

struct SetupArgs {
  uint32_t n;                 // points over all clouds
  uint32_t B;                 // clouds
  uint32_t max_key;           // largest possible key (total buckets - 1)
  const float *xyz;           // n x 3 (device)
  const uint32_t *poff;       // B + 1 point offsets
  const uint32_t *rid;        // B range index per cloud
  const RangeDev *ranges;
  const uint32_t *boff;       // B bucket offsets
  uint32_t *keys0, *vals0, *keys1, *vals1;  // n each
  uint32_t *hist;             // 256 * radix_tiles(n) + 1
  uint32_t *partial;          // ceil(max scan length / 4096) + 2
  float4 *pts;                // n sorted (x, y, z, dist)
  uint32_t *perm;             // n sorted -> input point id
  uint32_t *tmp0, *tmp1;      // n each (run starts, leaf ids)
  uint32_t *leaf_start;       // n + 1
  float4 *leaf_lo, *leaf_hi;  // n each
  float *leaf_md;             // n
  uint32_t *leaf_pre;         // n * kMaxPreimages or null (direct ranges)
  uint32_t *loff;             // B + 1 leaf offsets
  uint32_t *scalars;          // kScalarCount
  const uint32_t *cand;       // candidate CTA counts (device)
  const uint32_t *cand_host;  // same, host copy
  int ncand;
  uint32_t *plan;             // 3 * ncand (device)
  // fused setup of small clouds (one CTA each, nsfps_setup.cu): register
  // rounds of its sort (small_setup_rounds of the largest cloud), or 0 for the
  // multi-launch pipeline.  Needs every cloud non-empty, every range's total
  // buckets <= kSmallMaxBuckets and candidate CTA counts summing to <= 512.
  int small_rounds;
};

cudaError_t run_setup(const SetupArgs &a, cudaStream_t st, uint32_t &launches);

// Largest cloud and bucket count of the fused setup of small clouds; its
// sort's register rounds for a largest cloud of max_cloud points (0: too
// large) and its dynamic shared memory.
constexpr uint32_t kSmallCloudMax = 24576;
constexpr uint32_t kSmallMaxBuckets = 1u << 17;
int small_setup_rounds(uint32_t max_cloud);
size_t small_setup_smem(int rounds);
// Sets the fused setup's shared-memory opt-in on the current device; call
// before run_setup (outside stream capture) when small_rounds is set.
cudaError_t small_setup_prepare();

// Tiles the radix sort splits n keys into.
uint32_t radix_tiles(uint32_t n);
// Stable LSD radix sort of n (key, value) pairs, 8-bit digits over the bits of
// max_key.  *keys / *vals hold the input and, on return, point at whichever of
// the two buffer pairs holds the sorted result.  hist: 256 * radix_tiles(n)
// + 1 entries; partial: ceil(256 * radix_tiles(n) / 4096) + 2.
cudaError_t run_sort_pairs(uint32_t **keys, uint32_t **vals, uint32_t *keys_alt,
                           uint32_t *vals_alt, uint32_t n, uint32_t max_key, uint32_t *hist,
                           uint32_t *partial, cudaStream_t st, uint32_t &launches);
// Exclusive prefix sum of n uint32 (in may equal out); partial: ceil(n / 4096)
// + 2 entries.
cudaError_t run_exclusive_scan(const uint32_t *in, uint32_t *out, uint32_t n,
                               uint32_t *partial, cudaStream_t st, uint32_t &launches);

// compute_bbox of each of B device-resident clouds (poff: B + 1 point
// offsets, device; max_cloud: points of the largest): out[6c .. 6c+5] =
// min x, y, z, max x, y, z.
cudaError_t run_cloud_bbox(const float *xyz, const uint32_t *poff, uint32_t B,
                           uint32_t max_cloud, float *out, cudaStream_t st, uint32_t &launches);

struct LoopArgs {
  uint32_t B;                 // clouds in this launch
  uint32_t k;                 // samples per cloud
  uint32_t P;                 // CTAs per cloud
  uint32_t max_pts;           // shared-memory capacity per CTA (points)
  uint32_t max_leaves;        // shared-memory capacity per CTA (leaves)
  uint32_t max_extra;         // extra preimage slots per CTA (hashed ranges)
  uint32_t max_tab;           // cube threshold floats per CTA
  const float4 *pts;
  const uint32_t *leaf_start;
  const float4 *leaf_lo, *leaf_hi;
  const float *leaf_md;
  const uint32_t *leaf_pre;
  const uint32_t *loff, *poff, *rid;
  const RangeDev *ranges;
  const float *tabs;          // cube half-width thresholds (RangeDev::tab_off)
  uint32_t *out_rank;         // B * k sorted positions of the samples
  uint32_t *out_count;        // B
  uint32_t *scalars;
  unsigned long long *stats;  // [0] reference-updated points, [1] evaluated
  uint32_t groups;            // grid-wide rounds: groups of P CTAs in the grid
  uint4 *glist;               // grid-wide rounds: 2 * P published lists per group (global)
  uint32_t *gbar;             // grid-wide rounds: one arrival counter per group (start at 0)
  long long timeout_ns;       // limit of every bounded wait
  // test hook: CTA `hold_cta` of cloud 0 does not publish at round / step
  // `hold_step` (-1: never), so that the waits for it run out
  int32_t hold_cta;
  uint32_t hold_step;
};

// Which shared-memory-resident sampling kernel to run.
struct LoopPlan {
  int mode;          // 0 = thread-block cluster (P <= 16), 1 = grid-wide (rounds only)
  int rounds;        // 1 = exchange rounds of candidates (nsfps_rounds.cu)
  uint32_t P;
  int leaves_per_thread;  // template instance (1, 2, 3, 4, 6, 8)
  bool direct;            // every cloud's buckets are its cells
  size_t smem_bytes;
};

// Smallest template instance of leaves per thread covering `leaves` leaves
// per CTA, or 0 when none does.
int loop_leaves_per_thread(uint32_t leaves);

// The round-based loop (direct ranges only): candidates per CTA of a part of
// a cloud over P <= 16 CTAs holding up to `pts` points per CTA, shared
// memory, launch.
int rounds_candidates_per_cta(uint32_t P, uint32_t pts);
int rounds_leaves_per_thread(uint32_t leaves);
size_t rounds_smem_bytes(uint32_t pts, uint32_t leaves, uint32_t tab);
int rounds_max_smem(uint32_t P);
cudaError_t run_rounds(const LoopArgs &a, const LoopPlan &plan, cudaStream_t st,
                       uint32_t &launches);
// Grid-wide rounds (groups of P co-resident CTAs, each sampling its share of
// the clouds, lists through global memory): candidates per CTA (0 when no
// grid-wide instance exists for P), the bytes of the global list buffers of
// `groups` groups, and how many clusters of P CTAs the device holds at once
// (for the choice between the two layouts; 0 when unknown).
int rounds_grid_candidates_per_cta(uint32_t P);
size_t rounds_grid_list_bytes(uint32_t P, uint32_t groups);
// Bytes of the global list buffers of batch groups over `ctas` CTAs in all,
// whatever their size.
size_t rounds_group_list_bytes(uint32_t ctas);
int rounds_cluster_capacity(uint32_t P, int m, size_t smem);

cudaError_t run_loop(const LoopArgs &a, const LoopPlan &plan, cudaStream_t st,
                     uint32_t &launches);

// out[c * k + i] = original index (within cloud c) of sample i.
cudaError_t run_epilogue(const uint32_t *out_rank, const uint32_t *out_count,
                         const uint32_t *perm, const uint32_t *poff, uint32_t B,
                         uint32_t k, uint64_t *out, cudaStream_t st,
                         uint32_t &launches);

size_t loop_smem_bytes(uint32_t pts, uint32_t leaves, uint32_t extra, uint32_t tab);
int loop_max_smem();  // bytes of dynamic shared memory a CTA may use

// ---- grouping after sampling (nsfps_group.cu)

// Uniform grid of one cloud for the ball query: cell of a point on axis a =
// floor((v - lo[a]) * inv[a]) (double), clamped to g[a] - 1; global cell id =
// base + (cz * g[1] + cy) * g[0] + cx.
struct GroupGrid {
  double lo[3];
  double inv[3];
  uint32_t g[3];
  uint32_t base;
};

struct GroupArgs {
  uint32_t n, B, m, S;        // points, clouds, centres, samples per centre
  uint32_t max_cloud;         // points of the largest cloud
  uint32_t cells;             // cells over all clouds; key `cells` = no cell
  float r2;                   // radius * radius (fp32)
  double h_min;               // smallest cell width: 1.01 * |radius|
  const float *xyz;           // n x 3 (device)
  const float *centers;       // m x 3 (device)
  const uint32_t *poff, *coff, *cbase;  // B + 1 point / centre / cell offsets
  uint32_t *box;              // 6 * B: per-cloud box as ordered integers
  GroupGrid *grids;           // B
  uint32_t *keys0, *vals0, *keys1, *vals1;  // n each
  uint32_t *hist, *partial;   // radix-sort histogram, scan partials
  uint32_t *cstart;           // cells + 1: per-cell counts, then cell starts
  float4 *pts;                // n sorted (x, y, z, point id bits)
  int64_t *out_idx;           // m * S
  uint32_t *out_hits;         // m, or null
};

int ball_query_warps(uint32_t S);
size_t ball_query_smem(uint32_t S);
// Grid build and query; the two events (may be null) bracket the query kernel.
cudaError_t run_ball_query(const GroupArgs &a, cudaStream_t st, uint32_t &launches,
                           cudaEvent_t ev_query_begin, cudaEvent_t ev_query_end);
cudaError_t run_gather_points(const float *xyz, const uint32_t *poff, const int64_t *idx,
                              const uint32_t *ioff, uint32_t B, uint32_t m, float *out,
                              uint32_t *err_flag, cudaStream_t st, uint32_t &launches);
cudaError_t run_group_points(const float *xyz, const uint32_t *poff, const float *centers,
                             const uint32_t *coff, uint32_t B, uint32_t m, uint32_t S,
                             const int64_t *idx, float *out, uint32_t *err_flag, cudaStream_t st,
                             uint32_t &launches);

// Address and size of the fixed scratch array (nsfps_static.cu) on the
// current device.
cudaError_t static_scratch_address(void **ptr, size_t *bytes);

}  // namespace nsfps
