// ref_shim.cpp -- extern "C" entry points around the reference's own C++ API
// (satreeby/ns_fps src/yuezu_fps.h), compiled together with the reference
// source file where it lies (see oracle/Makefile).  TEST INFRASTRUCTURE: it is
// loaded only by tests/, __graft_entry__.smoke() and bench.py's reference /
// cpu_baseline legs, never by the product.
//
// Each function converts plain pointers into the reference's types the same
// way its pybind11 layer does (yuezu_fps/yuezu_fps_pybind.cpp:17-33
// numpy_to_points: Point3D(x, y, z, i)) and calls the reference unchanged.

#include "yuezu_fps.h"

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <exception>
#include <thread>
#include <vector>

namespace {

std::vector<Point3D> to_points(const float *xyz, uint64_t n) {
  std::vector<Point3D> pts;
  pts.reserve(n);
  for (uint64_t i = 0; i < n; ++i)
    pts.emplace_back(xyz[3 * i], xyz[3 * i + 1], xyz[3 * i + 2], (size_t)i);
  return pts;
}

SpaceRange range_of(const float *rng6, const uint32_t *blocks3) {
  return make_range(rng6[0], rng6[1], rng6[2], rng6[3], rng6[4], rng6[5],
                    blocks3[0], blocks3[1], blocks3[2]);
}

}  // namespace

extern "C" {

// yuezu_fps(points, k, make_range(...)) or, with use_bbox != 0,
// yuezu_fps(points, k, compute_bbox(points, xb, yb, zb))
// (yuezu_fps_pybind.cpp:67-101).  out has capacity k (or n when k >= n).
int ref_fps(const float *xyz, uint64_t n, uint64_t k, const float *rng6,
            const uint32_t *blocks3, int use_bbox, uint64_t *out,
            uint64_t *out_len) {
  try {
    auto pts = to_points(xyz, n);
    SpaceRange r = use_bbox ? compute_bbox(pts, blocks3[0], blocks3[1],
                                           blocks3[2])
                            : range_of(rng6, blocks3);
    auto res = yuezu_fps(pts, (size_t)k, r);
    for (size_t i = 0; i < res.size(); ++i)
      out[i] = res[i];
    *out_len = res.size();
    return 0;
  } catch (...) {
    return 1;
  }
}

// compute_bbox(points, xb, yb, zb) -> {min_x, max_x, min_y, max_y, min_z, max_z}
int ref_bbox(const float *xyz, uint64_t n, const uint32_t *blocks3,
             float *rng6_out) {
  auto pts = to_points(xyz, n);
  SpaceRange r = compute_bbox(pts, blocks3[0], blocks3[1], blocks3[2]);
  const float v[6] = {r.min_x, r.max_x, r.min_y, r.max_y, r.min_z, r.max_z};
  std::memcpy(rng6_out, v, sizeof(v));
  return 0;
}

// make_range(...) derived fields: f_out = {inv_bs_x/y/z, block_size_x/y/z},
// u_out = {x_bits, y_bits, z_bits, total_bits, total_blocks (low 32 bits)},
// luts may be null; each receives 2^bits entries.
int ref_range_info(const float *rng6, const uint32_t *blocks3, float *f_out,
                   uint32_t *u_out, uint32_t *lutx, uint32_t *luty,
                   uint32_t *lutz) {
  SpaceRange r = range_of(rng6, blocks3);
  f_out[0] = r.inv_bs_x;
  f_out[1] = r.inv_bs_y;
  f_out[2] = r.inv_bs_z;
  f_out[3] = r.block_size_x();
  f_out[4] = r.block_size_y();
  f_out[5] = r.block_size_z();
  u_out[0] = r.x_bits();
  u_out[1] = r.y_bits();
  u_out[2] = r.z_bits();
  u_out[3] = r.total_bits();
  u_out[4] = (uint32_t)r.total_blocks();
  if (lutx)
    std::memcpy(lutx, r.x_lut_.data(), r.x_lut_.size() * sizeof(uint32_t));
  if (luty)
    std::memcpy(luty, r.y_lut_.data(), r.y_lut_.size() * sizeof(uint32_t));
  if (lutz)
    std::memcpy(lutz, r.z_lut_.data(), r.z_lut_.size() * sizeof(uint32_t));
  return 0;
}

// Runs yuezu_fps on `count` clouds with `threads` host threads (whole clouds
// per thread; the reference itself is single-threaded and keeps no global
// state).  clouds[i] is n[i] x 3 floats; out[i] has capacity k or n[i].
// Returns 0 on success.  *seconds receives the wall time of the parallel part.
int ref_fps_many(const float *const *clouds, const uint64_t *n, uint64_t count,
                 uint64_t k, const float *rng6, const uint32_t *blocks3,
                 uint64_t *const *out, uint64_t *out_len, int threads,
                 double *seconds) {
  if (threads < 1)
    threads = 1;
  std::vector<std::vector<Point3D>> pts(count);
  for (uint64_t i = 0; i < count; ++i)
    pts[i] = to_points(clouds[i], n[i]);
  SpaceRange r = range_of(rng6, blocks3);
  std::atomic<uint64_t> next{0};
  std::atomic<int> failed{0};
  auto t0 = std::chrono::steady_clock::now();
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t)
    pool.emplace_back([&]() {
      for (;;) {
        uint64_t i = next.fetch_add(1);
        if (i >= count)
          return;
        try {
          auto res = yuezu_fps(pts[i], (size_t)k, r);
          for (size_t j = 0; j < res.size(); ++j)
            out[i][j] = res[j];
          out_len[i] = res.size();
        } catch (...) {
          failed = 1;
        }
      }
    });
  for (auto &th : pool)
    th.join();
  auto t1 = std::chrono::steady_clock::now();
  if (seconds)
    *seconds = std::chrono::duration<double>(t1 - t0).count();
  return failed.load();
}

}  // extern "C"
