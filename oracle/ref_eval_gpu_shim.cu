// ref_eval_gpu_shim.cu -- extern "C" entry point around the reference's own
// evaluation GPU sampler (satreeby/ns_fps eval/src_gpu/yuezu_fps_gpu.h:90-126,
// eval/src_gpu/yuezu_fps_gpu_optimized.cu:896-1062), compiled together with
// that source file where it lies (see oracle/Makefile).  TEST INFRASTRUCTURE:
// a reported, non-bit-exact GPU baseline (its distances start from 1e30, sum
// with contraction allowed and take the first index among equal maxima of
// 32 strided block scans), loaded only by tests/, never by the product.
//
// The points are converted the way the reference's own GPU test does
// (eval/src_gpu/test_gpu.cpp: Point3D(x, y, z, i)); the sampler is the
// reference's FpsGPU class, unchanged: initialize() copies the cloud, sorts
// it by Morton code and builds its tables, sample() runs three launches per
// step (block argmax, postprocess, grid-range update).

#include "yuezu_fps_gpu.h"

#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <vector>

extern "C" {

// Samples k points of the dense N x 3 cloud with make_range(rng6, blocks3).
// out has capacity k.  *init_ms / *sample_ms: host wall time of
// FpsGPU::initialize (allocation, host->device copy, sort) and of
// FpsGPU::sample (the steps and the device->host copy of the indices), each
// bracketed by cudaDeviceSynchronize.  Returns 0, 1 when initialize fails,
// 2 on a CUDA error.
int ref_eval_gpu_fps(const float *xyz, uint64_t n, uint64_t k, const float *rng6,
                     const uint32_t *blocks3, uint64_t *out, uint64_t *out_len,
                     double *init_ms, double *sample_ms) {
  using clk = std::chrono::steady_clock;
  std::vector<Point3D> pts;
  pts.reserve(n);
  for (uint64_t i = 0; i < n; ++i)
    pts.emplace_back(xyz[3 * i], xyz[3 * i + 1], xyz[3 * i + 2], (size_t)i);
  const SpaceRange r = make_range(rng6[0], rng6[1], rng6[2], rng6[3], rng6[4], rng6[5],
                                  blocks3[0], blocks3[1], blocks3[2]);
  *out_len = 0;
  int rc = 0;
  {
    FpsGPU fps;
    cudaDeviceSynchronize();
    const auto t0 = clk::now();
    if (!fps.initialize(pts, r)) return 1;
    cudaDeviceSynchronize();
    const auto t1 = clk::now();
    const std::vector<size_t> res = fps.sample((size_t)k);
    cudaDeviceSynchronize();
    const auto t2 = clk::now();
    *init_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    *sample_ms = std::chrono::duration<double, std::milli>(t2 - t1).count();
    for (size_t i = 0; i < res.size(); ++i) out[i] = res[i];
    *out_len = res.size();
    if (cudaGetLastError() != cudaSuccess) rc = 2;
  }
  return rc;
}

}  // extern "C"
