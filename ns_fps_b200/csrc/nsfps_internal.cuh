// nsfps_internal.cuh -- definitions shared by the engine's CUDA sources.
//
// Numerics contract (bit-exact with the reference built without FMA
// contraction):
//   * every float operation that the reference performs is issued here as the
//     matching round-to-nearest intrinsic (__fsub_rn / __fmul_rn / __fadd_rn /
//     __fdiv_rn / __fsqrt_rn), which the compiler never fuses; the sources are
//     also compiled with -fmad=false;
//   * float -> integer conversions reproduce what GCC emits for the reference
//     on x86-64 (cvttss2si): out-of-range and NaN give "integer indefinite".
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "nsfps.h"

namespace nsfps {

// Points per leaf.  Leaves are runs of at most kLeafSize consecutive points of
// one bucket in the sorted order.  The value is a tuning choice of this engine
// only: the sample sequence does not depend on it.
constexpr int kLeafSize = 16;
constexpr int kMaxAxisBits = 10;   // NSFPS_MAX_BLOCKS_PER_AXIS == 1 << 10
constexpr int kMaxPreimages = 8;   // code < 2^total_bits <= 8 * total_blocks

// Device copy of a SpaceRange with every derived field precomputed on the host
// exactly as make_range() does (src/yuezu_fps.cpp:136-161).
struct RangeDev {
  float mn[3];      // min_x, min_y, min_z
  float hi[3];      // max - BOUNDARY_EPS  (src/yuezu_fps.cpp:172-174)
  float inv_bs[3];  // 1.0f / ((max - min) / (float)blocks)
  float bsz[3];     // block_size_*() = (max - min) / blocks  (src/yuezu_fps.cpp:7-11)
  uint32_t blocks[3];
  uint32_t bits[3];
  uint32_t total;       // total_blocks()
  uint32_t total_bits;
  uint32_t direct;      // 1: every cell's Morton code is < total, so bucket == code
  uint8_t pos[3][kMaxAxisBits];  // Morton bit position of each axis bit
  uint8_t pad_[2];
  // Cube half-width tables (see cube_thresholds in nsfps_capi.cu): when
  // `fast_cube` is set, n_a = (int)ceil(sqrt(D) / block_size_a) is the count
  // of entries of table a (blocks[a] - 1 floats at tab_off[a]) that are < D,
  // and D > ovf[a] means the reference's int conversion overflows.
  uint32_t fast_cube;
  uint32_t tab_off[3];
  float ovf[3];
};

// Packed cell coordinates: x | y << 10 | z << 20.
__host__ __device__ __forceinline__ uint32_t pack_cell(uint32_t x, uint32_t y,
                                                       uint32_t z) {
  return x | (y << 10) | (z << 20);
}

#ifdef __CUDACC__

// (uint32_t)v as GCC compiles it for x86-64: cvttss2si to a 64-bit register,
// low 32 bits kept; NaN and |v| >= 2^63 give 0.
__device__ __forceinline__ uint32_t cvt_u32_x86(float v) {
  if (v >= 0.0f && v < 4294967296.0f) return __float2uint_rz(v);  // common case
  if (v >= -9223372036854775808.0f && v < 9223372036854775808.0f)
    return (uint32_t)__float2ll_rz(v);
  return 0u;
}

// (int)v on x86-64: cvttss2si 32-bit, INT_MIN when NaN or out of range.
__device__ __forceinline__ int32_t cvt_i32_x86(float v) {
  if (v >= -2147483648.0f && v < 2147483648.0f)
    return __float2int_rz(v);
  return (int32_t)0x80000000;
}

// One axis of Point3D::compute_block_indices (src/yuezu_fps.cpp:170-193):
// std::max(min, std::min(p, max - eps)), (p - min) * inv_bs, truncate, clamp.
__device__ __forceinline__ uint32_t cell_axis(float p, float mn, float hi,
                                              float inv, uint32_t blocks) {
  const float t = (hi < p) ? hi : p;   // std::min(p, hi)
  const float c = (mn < t) ? t : mn;   // std::max(mn, t)
  const uint32_t i = cvt_u32_x86(__fmul_rn(__fsub_rn(c, mn), inv));
  const uint32_t lim = blocks - 1u;
  return i < lim ? i : lim;
}

__device__ __forceinline__ void cell_of(const RangeDev &r, float x, float y,
                                        float z, uint32_t &cx, uint32_t &cy,
                                        uint32_t &cz) {
  cx = cell_axis(x, r.mn[0], r.hi[0], r.inv_bs[0], r.blocks[0]);
  cy = cell_axis(y, r.mn[1], r.hi[1], r.inv_bs[1], r.blocks[1]);
  cz = cell_axis(z, r.mn[2], r.hi[2], r.inv_bs[2], r.blocks[2]);
}

// Morton spread of one axis index (the reference's x_lut_[v], :52-66).
__device__ __forceinline__ uint32_t spread_axis(const RangeDev &r, int a,
                                                uint32_t v) {
  uint32_t code = 0;
#pragma unroll
  for (int k = 0; k < kMaxAxisBits; ++k)
    if (k < (int)r.bits[a] && ((v >> k) & 1u))
      code |= 1u << r.pos[a][k];
  return code;
}

// Inverse of the spread: the axis index encoded in `code`.
__device__ __forceinline__ uint32_t gather_axis(const RangeDev &r, int a,
                                                uint32_t code) {
  uint32_t v = 0;
#pragma unroll
  for (int k = 0; k < kMaxAxisBits; ++k)
    if (k < (int)r.bits[a])
      v |= ((code >> r.pos[a][k]) & 1u) << k;
  return v;
}

// Bucket of a cell: (lutx | luty | lutz) % total_blocks (:195-199, :411-416).
__device__ __forceinline__ uint32_t bucket_of_cell(const RangeDev &r,
                                                   uint32_t cx, uint32_t cy,
                                                   uint32_t cz) {
  const uint32_t code =
      spread_axis(r, 0, cx) | spread_axis(r, 1, cy) | spread_axis(r, 2, cz);
  return r.direct ? code : code % r.total;
}

// squared_distance(p, q) (src/yuezu_fps.cpp:205-209): (dx*dx + dy*dy) + dz*dz,
// dx = p.x - q.x, each operation rounded to nearest on its own.
__device__ __forceinline__ float sqdist(float px, float py, float pz, float qx,
                                        float qy, float qz) {
  const float dx = __fsub_rn(px, qx);
  const float dy = __fsub_rn(py, qy);
  const float dz = __fsub_rn(pz, qz);
  return __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)),
                   __fmul_rn(dz, dz));
}

#endif  // __CUDACC__

// ---------------------------------------------------------------- host side

// Fills a RangeDev from the user range; returns NSFPS_OK or NSFPS_ERR_ARG /
// NSFPS_ERR_UNSUPPORTED (message in *why).
int range_to_dev(const nsfps_range &r, RangeDev *out, const char **why);

// Appends the cube half-width thresholds of `r` to `pool` and records their
// offsets in `r` (sets fast_cube when the block sizes allow it).
void cube_thresholds(RangeDev &r, std::vector<float> &pool);

// Derived fields for the C ABI (nsfps_range_get_info / _get_lut).
int range_info(const nsfps_range &r, nsfps_range_info *info);

// Error reporting (thread-local text).
int set_error(int code, const char *fmt, ...);
void clear_error();

}  // namespace nsfps
