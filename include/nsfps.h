/*
 * nsfps.h -- C ABI of the B200-native farthest-point-sampling engine
 * (ns_fps_b200).  Drop-in for the sampling path of satreeby/ns_fps
 * (`yuezu_fps()` and its pybind11 surface `yuezu_fps.yuezu_fps_module`).
 *
 * Plain pointers and sizes only.  Every entry point returns NSFPS_OK (0) or an
 * NSFPS_ERR_* code; nsfps_last_error() then describes the failure (the text is
 * thread-local).  The caller owns every buffer.  Calls are thread-safe; calls
 * on the same device are serialised internally.
 *
 * Results are bit-exact with the reference `yuezu_fps()` built without
 * multiply-add contraction: the same sample indices, in the same order, with
 * the same early stop.
 */
#ifndef NSFPS_H_
#define NSFPS_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NSFPS_API __attribute__((visibility("default")))
#else
#define NSFPS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Compile-time constants of the reference (src/yuezu_fps.h:20-50), exposed
 * with the same names by the pybind11 module.  MORTON_BLOCK_SIZE and
 * CACHE_BLOCK_SIZE only shape the reference's internal tree; neither changes
 * which points are sampled. */
#define NSFPS_MORTON_BLOCK_SIZE 16
#define NSFPS_CACHE_BLOCK_SIZE 16
#define NSFPS_DEFAULT_X_BLOCKS 16
#define NSFPS_DEFAULT_Y_BLOCKS 16
#define NSFPS_DEFAULT_Z_BLOCKS 16
#define NSFPS_BOUNDARY_EPS 1e-6f

/* Limits of this engine (the reference allocates its bucket table up front
 * and is bounded by host memory instead). */
#define NSFPS_MAX_BLOCKS_PER_AXIS 1024u

enum nsfps_status {
  NSFPS_OK = 0,
  NSFPS_ERR_ARG = 1,         /* invalid argument (shape, range, pointer) */
  NSFPS_ERR_CUDA = 2,        /* a CUDA runtime call failed */
  NSFPS_ERR_OOM = 3,         /* device or host allocation failed */
  NSFPS_ERR_TIMEOUT = 4,     /* a bounded in-kernel wait gave up */
  NSFPS_ERR_UNSUPPORTED = 5  /* input beyond this engine's limits */
};

/* The user-facing part of the reference's SpaceRange (src/yuezu_fps.h:56-83):
 * bounds and per-axis block counts.  The derived fields (inv_bs, bit counts,
 * Morton LUTs) are recomputed from these exactly as make_range() does
 * (src/yuezu_fps.cpp:136-161) every time the range is used. */
typedef struct nsfps_range {
  float min_x, max_x;
  float min_y, max_y;
  float min_z, max_z;
  uint32_t x_blocks, y_blocks, z_blocks;
} nsfps_range;

/* Derived fields of a range, as the reference computes them. */
typedef struct nsfps_range_info {
  float inv_bs[3];       /* 1.0f / ((max - min) / (float)blocks)   src/yuezu_fps.cpp:140-142 */
  float block_size[3];   /* (max - min) / blocks                    src/yuezu_fps.cpp:7-11 */
  uint32_t bits[3];      /* max(1, ceil(log2(blocks)))              src/yuezu_fps.cpp:13-32 */
  uint32_t total_bits;   /* bits[0] + bits[1] + bits[2]             src/yuezu_fps.cpp:34-36 */
  uint64_t total_blocks; /* x_blocks * y_blocks * z_blocks          src/yuezu_fps.cpp:38-40 */
} nsfps_range_info;

/* Text of the last error on this thread ("" when none). */
NSFPS_API const char *nsfps_last_error(void);

/* Library version (major * 10000 + minor * 100 + patch). */
NSFPS_API int nsfps_version(void);

/* Number of CUDA devices visible to the library. */
NSFPS_API int nsfps_device_count(int *count);

/* make_range(): fills *out (replaces src/yuezu_fps.cpp:136-161 and the
 * pybind11 binding yuezu_fps/yuezu_fps_pybind.cpp:128-130). */
NSFPS_API int nsfps_make_range(float min_x, float max_x, float min_y, float max_y,
                     float min_z, float max_z, uint32_t x_blocks,
                     uint32_t y_blocks, uint32_t z_blocks, nsfps_range *out);

/* make_uniform_range(): blocks_per_dim on every axis (replaces
 * src/yuezu_fps.cpp:98-134, binding yuezu_fps_pybind.cpp:132-134). */
NSFPS_API int nsfps_make_uniform_range(float min_x, float max_x, float min_y,
                             float max_y, float min_z, float max_z,
                             uint32_t blocks_per_dim, nsfps_range *out);

/* SpaceRange::block_size_* / *_bits / total_bits / total_blocks and the
 * inv_bs fields (replaces src/yuezu_fps.cpp:7-40, yuezu_fps_pybind.cpp:118-125).
 * Fails with NSFPS_ERR_ARG for zero block counts. */
NSFPS_API int nsfps_range_get_info(const nsfps_range *r, nsfps_range_info *info);

/* Per-axis Morton LUT (x_lut_/y_lut_/z_lut_, src/yuezu_fps.cpp:52-97).
 * axis 0..2; lut receives 2^bits entries when cap allows; *len gets 2^bits. */
NSFPS_API int nsfps_range_get_lut(const nsfps_range *r, int axis, uint32_t *lut,
                        uint64_t cap, uint64_t *len);

/* compute_bbox(points, xb, yb, zb): bounds of the cloud widened by
 * BOUNDARY_EPS; an empty cloud gives [0,1]^3 with 1x1x1 blocks (replaces
 * src/yuezu_fps.cpp:643-670).  Runs on the host. */
NSFPS_API int nsfps_compute_bbox(const float *xyz, uint64_t n, uint32_t x_blocks,
                       uint32_t y_blocks, uint32_t z_blocks, nsfps_range *out);

/* Farthest point sampling of one cloud (replaces yuezu_fps(),
 * src/yuezu_fps.h:211-212 / src/yuezu_fps.cpp:676-730, as bound by
 * fps_numpy, yuezu_fps/yuezu_fps_pybind.cpp:67-86).
 *   xyz     n x 3 floats, dense, HOST memory
 *   range   NULL selects compute_bbox(points, 16, 16, 16) like fps(range=None)
 *   out     HOST buffer of capacity min(k, n) receiving original indices
 *   out_len receives the number of samples (< k when every remaining point is
 *           at distance 0 from the samples, as in the reference)
 *   device  CUDA device ordinal */
NSFPS_API int nsfps_fps(const float *xyz, uint64_t n, uint64_t k,
              const nsfps_range *range, uint64_t *out, uint64_t *out_len,
              int device);

/* fps_with_bbox(points, k, xb, yb, zb) (replaces
 * yuezu_fps/yuezu_fps_pybind.cpp:88-101). */
NSFPS_API int nsfps_fps_with_bbox(const float *xyz, uint64_t n, uint64_t k,
                        uint32_t x_blocks, uint32_t y_blocks,
                        uint32_t z_blocks, uint64_t *out, uint64_t *out_len,
                        int device);

/* Batched sampling: `count` independent clouds, the same k for each, whole
 * clouds sharded across `ndev` devices (one host thread per device, no
 * inter-GPU traffic).  Each cloud i is n[i] x 3 host floats; ranges holds one
 * range shared by all clouds (per_cloud_ranges == 0) or `count` ranges;
 * a NULL ranges selects compute_bbox(cloud, 16, 16, 16) per cloud.  out[i]
 * has capacity min(k, n[i]); out_len[i] receives each length.  devices == NULL
 * uses devices 0..ndev-1.  The reference has no batched entry point; this
 * replaces a loop of fps() calls (yuezu_fps_pybind.cpp:67-86). */
NSFPS_API int nsfps_fps_batched(const float *const *clouds, const uint64_t *n,
                      uint64_t count, uint64_t k, const nsfps_range *ranges,
                      int per_cloud_ranges, uint64_t *const *out,
                      uint64_t *out_len, const int *devices, int ndev);

/* Device-resident sampling for callers that keep clouds in HBM: `count`
 * clouds packed back to back in d_xyz (offsets[i]..offsets[i+1] points,
 * offsets in HOST memory, count + 1 entries), ranges as in
 * nsfps_fps_batched (host memory; NULL selects compute_bbox(cloud, 16, 16,
 * 16) per cloud, like fps(range=None), with the min/max reduction done on the
 * device, src/yuezu_fps.cpp:643-670), d_out a DEVICE buffer of
 * count * k uint64 (cloud i at d_out + i * k), out_len a HOST array of
 * `count` lengths.  Work is issued on `stream` (a cudaStream_t; NULL = the
 * legacy default stream) of the current device; the call returns after the
 * lengths are known (it synchronises `stream`).  No reference counterpart
 * (the reference is host-only); it exists so callers avoid a host round trip
 * per call. */
NSFPS_API int nsfps_fps_device(const float *d_xyz, const uint64_t *offsets,
                     uint64_t count, uint64_t k, const nsfps_range *ranges,
                     int per_cloud_ranges, uint64_t *d_out, uint64_t *out_len,
                     void *stream);

/* fps_with_bbox() for device-resident clouds: nsfps_fps_device with every
 * cloud's bounding box (reduced on the device, widened by BOUNDARY_EPS as in
 * compute_bbox) and x_blocks x y_blocks x z_blocks blocks (replaces the
 * binding yuezu_fps/yuezu_fps_pybind.cpp:88-101 and src/yuezu_fps.cpp:
 * 643-670 for clouds in HBM; it is also the range the reference's KITTI
 * benchmark builds, eval/src_cpu/compare_cpu_test_kitti.cpp:230-245). */
NSFPS_API int nsfps_fps_device_with_bbox(const float *d_xyz, const uint64_t *offsets,
                               uint64_t count, uint64_t k, uint32_t x_blocks,
                               uint32_t y_blocks, uint32_t z_blocks, uint64_t *d_out,
                               uint64_t *out_len, void *stream);

/* Limits of nsfps_fps_device_static(): points per call, and the size of the
 * fixed device scratch array that holds every intermediate buffer. */
#define NSFPS_STATIC_MAX_POINTS 65536u
#define NSFPS_STATIC_SCRATCH_BYTES (8u << 20)

/* No counterpart in the reference (which is host-only).  One device-resident
 * cloud, sampled without allocating any device memory: for callers that
 * cannot allocate mid-run, such as a host that has given all device memory to
 * its own pool, or a latency-bound loop where cudaMalloc / cudaFree would
 * synchronise the device.  Every intermediate buffer lives in one fixed
 * scratch array of NSFPS_STATIC_SCRATCH_BYTES per device, reserved with the
 * library's device code.
 *   d_xyz   n x 3 floats in DEVICE memory of the current device
 *   n       1 <= k < n <= NSFPS_STATIC_MAX_POINTS; larger n fails with
 *           NSFPS_ERR_ARG before any device work (k >= n or k == 0 fail with
 *           NSFPS_ERR_UNSUPPORTED, as in nsfps_fps_device)
 *   range   HOST memory, non-NULL
 *   d_out   DEVICE buffer of k uint64 (original indices)
 *   out_len HOST; receives the number of samples
 *   stream  cudaStream_t of the current device (NULL = legacy default stream)
 * Samples are identical to nsfps_fps_device() on the same input.  The first
 * call on a device resolves the array's address (cudaGetSymbolAddress, with
 * that device current) and creates the device's timing events; make that
 * first call before any stream capture.  The array is shared by all calls on
 * a device, so overlapping calls would race on it: calls take a per-device
 * lock and return only after their work on `stream` has finished, which runs
 * them one at a time.  Each call clears the counters that must start at zero
 * itself (cudaMemsetAsync on `stream`). */
NSFPS_API int nsfps_fps_device_static(const float *d_xyz, uint64_t n, uint64_t k,
                            const nsfps_range *range, uint64_t *d_out,
                            uint64_t *out_len, void *stream);

/* ---- Grouping after sampling.  No counterpart in the reference, which stops
 * at the sample indices (src/yuezu_fps.cpp:676-730, yuezu_fps_pybind.cpp:
 * 137-143); these are the operators a PointNet++-style pipeline applies to
 * them next.
 *
 * Ball query (PointNet++ query_ball_point semantics): for centre j, the first
 * `nsample` points k of its cloud in index order with d2 < radius * radius,
 * d2 = (dx*dx + dy*dy) + dz*dz, dx = x_k - cx, every operation fp32 rounded
 * to nearest with no multiply-add contraction (the sampler's distance,
 * src/yuezu_fps.cpp:205-209).  idx[j * nsample + s] holds point indices
 * within the cloud, ascending; slots past the hits repeat the first hit; a
 * centre with no hit gets 0 in every slot.  hits[j] = min(number of hits,
 * nsample).  Points with a non-finite coordinate are never hits; a negative
 * radius acts as its magnitude, a NaN or zero radius finds nothing. */
#define NSFPS_MAX_NSAMPLE 1024u

/* Device-resident, batched: `count` clouds packed in d_xyz
 * (point_offsets[i]..point_offsets[i+1]) and their centres packed in
 * d_centers (center_offsets[i]..center_offsets[i+1]); offsets in HOST memory
 * (count + 1 entries each).  d_idx (m x nsample int64) and d_hits (m uint32,
 * may be NULL) are DEVICE buffers indexed from the first centre of the call.
 * Work is issued on `stream` of the current device; the call returns after
 * the stream has drained (the per-device workspace is reused by the next
 * call).  Inputs are not modified. */
NSFPS_API int nsfps_ball_query_device(const float *d_xyz, const uint64_t *point_offsets,
                            const float *d_centers, const uint64_t *center_offsets,
                            uint64_t count, float radius, uint32_t nsample, int64_t *d_idx,
                            uint32_t *d_hits, void *stream);

/* The same for one cloud in HOST memory (n x 3 points, m x 3 centres);
 * idx (m x nsample) and hits (m, may be NULL) are HOST buffers. */
NSFPS_API int nsfps_ball_query(const float *xyz, uint64_t n, const float *centers, uint64_t m,
                     float radius, uint32_t nsample, int64_t *idx, uint32_t *hits,
                     int device);

/* Gather of sampled points (PointNet++ gather_operation on coordinates):
 * d_out[3j + a] = coordinate a of point d_idx[j] of entry j's cloud; entries
 * packed per cloud by idx_offsets (HOST, count + 1), points by point_offsets.
 * Device buffers, current device, returns after `stream` drained.  An index
 * outside its cloud gives NaNs at its entry and NSFPS_ERR_ARG. */
NSFPS_API int nsfps_gather_points_device(const float *d_xyz, const uint64_t *point_offsets,
                               const int64_t *d_idx, const uint64_t *idx_offsets,
                               uint64_t count, float *d_out, void *stream);

/* Grouped coordinates relative to each centre (PointNet++ grouping of
 * xyz followed by the subtraction of the centre): d_out[((j * nsample) + s)
 * * 3 + a] = xyz[d_idx[j * nsample + s]][a] - centers[j][a] (fp32, round to
 * nearest), d_idx as written by nsfps_ball_query_device.  Errors as in
 * nsfps_gather_points_device. */
NSFPS_API int nsfps_group_points_device(const float *d_xyz, const uint64_t *point_offsets,
                              const float *d_centers, const uint64_t *center_offsets,
                              uint64_t count, uint32_t nsample, const int64_t *d_idx,
                              float *d_out, void *stream);

/* Timing and work counters of the last call on this thread: stage times in
 * milliseconds measured with CUDA events on the launching stream (setup =
 * binning, sort and leaf build; loop = the persistent sampling kernel;
 * total = first to last event), the number of kernel launches, and the work
 * counters of the sampling loop: points in the buckets the reference updates
 * (summed over iterations), points actually re-evaluated after the exact
 * bounding-box skip, and the loop configuration (CTAs per cloud and mode:
 * 0 = per-step cluster loop, 2 = round-based cluster loop, 3 = round-based
 * loop over co-resident CTAs: 64 or 128 for a single cloud of at least 4,096
 * points, groups of up to 16 for a batch when the device cannot hold a
 * cluster per cloud).  After a ball query (mode 4): setup = the grid build,
 * loop = the query kernel, launches = its kernel launches; the work counters
 * are 0.
 * Enabled by nsfps_set_profiling. */
typedef struct nsfps_profile {
  float setup_ms, loop_ms, total_ms;
  uint32_t launches;
  uint32_t ctas_per_cloud;
  uint32_t mode;
  uint32_t leaves;
  uint64_t ref_points_updated;
  uint64_t points_evaluated;
  uint64_t iterations;
} nsfps_profile;

NSFPS_API int nsfps_set_profiling(int enable);
NSFPS_API int nsfps_last_profile(nsfps_profile *out);

/* ---- Test hooks.  No counterpart in the reference, whose GPU prototype
 * ignores CUDA errors (eval/src_gpu/yuezu_fps_gpu_optimized.cu:904-910) and
 * whose CPU path has no failure mode to test.  They drive this engine's error
 * paths without faulting the GPU:
 *   wait_limit_ns      limit of every bounded in-kernel wait (0 = the default,
 *                      2 s; the queue polling of worker warps gets twice it)
 *   withhold_cta       rank, among the CTAs of cloud 0, of one CTA that does
 *                      not publish its round-`withhold_step` candidate list
 *                      (round loops) or its step-`withhold_step` proposals
 *                      (per-step loop); every wait for it then runs out and
 *                      the call returns NSFPS_ERR_TIMEOUT with the device
 *                      still usable.  -1 = none.
 *   withhold_step      the round (round loops, from 0) or step (per-step loop,
 *                      from 1) at which it withholds
 *   fail_alloc_device  the next workspace request of an allocating entry point
 *                      on this device fails as if cudaMalloc had run out of
 *                      memory (NSFPS_ERR_OOM); it fires once.  -1 = none.
 * The hooks are process-wide and stay set until replaced; NULL restores the
 * defaults.  Not for production use. */
typedef struct nsfps_test_hooks {
  uint64_t wait_limit_ns;
  int32_t withhold_cta;
  uint32_t withhold_step;
  int32_t fail_alloc_device;
  int32_t reserved;
} nsfps_test_hooks;

NSFPS_API int nsfps_set_test_hooks(const nsfps_test_hooks *hooks);

#ifdef __cplusplus
}
#endif

#endif /* NSFPS_H_ */
