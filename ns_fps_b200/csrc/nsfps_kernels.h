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

constexpr int kMaxCand = 8;

// Points from which a single cloud takes the grid-wide round loop (build-time).
#ifndef NSFPS_GRID_MIN_POINTS
#define NSFPS_GRID_MIN_POINTS 98304u
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
  uint32_t *hist;             // 256 * ceil(n / 4096)
  uint32_t *partial;          // ceil(max scan length / 4096) + 2
  float4 *pts;                // n sorted (x, y, z, dist)
  uint32_t *perm;             // n sorted -> input point id
  uint32_t *tmp0, *tmp1;      // n each (run starts, leaf ids)
  uint32_t *leaf_start;       // n + 1
  float4 *leaf_lo, *leaf_hi;  // n each
  float *leaf_md;             // n
  uint32_t *leaf_pre;         // n * (kMaxPreimages - 1) or null (direct ranges)
  uint32_t *loff;             // B + 1 leaf offsets
  uint32_t *scalars;          // kScalarCount
  const uint32_t *cand;       // candidate CTA counts (device)
  const uint32_t *cand_host;  // same, host copy
  int ncand;
  uint32_t *plan;             // 3 * ncand (device)
};

cudaError_t run_setup(const SetupArgs &a, cudaStream_t st, uint32_t &launches);

// compute_bbox of each of B device-resident clouds (poff: B + 1 point
// offsets, device): out[6c .. 6c+5] = min x, y, z, max x, y, z.
cudaError_t run_cloud_bbox(const float *xyz, const uint32_t *poff, uint32_t B, float *out,
                           cudaStream_t st, uint32_t &launches);

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
  uint4 *glist;               // grid-wide rounds: 2 * P published lists (global)
  uint32_t *gbar;             // grid-wide rounds: arrival counter (starts at 0)
  long long timeout_ns;
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

// The round-based loop (direct ranges only): candidates per CTA, shared
// memory, launch.
int rounds_candidates_per_cta(uint32_t P);
int rounds_leaves_per_thread(uint32_t leaves);
size_t rounds_smem_bytes(uint32_t pts, uint32_t leaves, uint32_t tab);
int rounds_max_smem(uint32_t P);
cudaError_t run_rounds(const LoopArgs &a, const LoopPlan &plan, cudaStream_t st,
                       uint32_t &launches);
// Grid-wide rounds (one cloud over P co-resident CTAs, lists through global
// memory): candidates per CTA and the bytes of the global list buffers.
int rounds_grid_candidates_per_cta(uint32_t P);
size_t rounds_grid_list_bytes(uint32_t P);

cudaError_t run_loop(const LoopArgs &a, const LoopPlan &plan, cudaStream_t st,
                     uint32_t &launches);

// out[c * k + i] = original index (within cloud c) of sample i.
cudaError_t run_epilogue(const uint32_t *out_rank, const uint32_t *out_count,
                         const uint32_t *perm, const uint32_t *poff, uint32_t B,
                         uint32_t k, uint64_t *out, cudaStream_t st,
                         uint32_t &launches);

size_t loop_smem_bytes(uint32_t pts, uint32_t leaves, uint32_t extra, uint32_t tab);
int loop_max_smem();  // bytes of dynamic shared memory a CTA may use

// Address and size of the fixed scratch array (nsfps_static.cu) on the
// current device.
cudaError_t static_scratch_address(void **ptr, size_t *bytes);

}  // namespace nsfps
