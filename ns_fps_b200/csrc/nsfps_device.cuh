// nsfps_device.cuh -- device helpers shared by the sampling-loop kernels
// (nsfps_loop.cu, nsfps_rounds.cu): cluster / mbarrier / st.async wrappers,
// the distance key, cell-cube packing and the exact cube half-widths.
#pragma once

#include <cfloat>

#include "nsfps_internal.cuh"
#include "nsfps_kernels.h"

namespace nsfps {
namespace {

constexpr uint32_t kFull = 0xffffffffu;
constexpr int kMaxClusterP = 16;
constexpr int kBufs = 4;  // exchange buffers rotating with the step / round


__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint32_t addr, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(addr), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Arms the current phase of a local mbarrier: one arrival plus `bytes` of
// expected transactions.
__device__ __forceinline__ void mbar_arm(uint32_t addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(addr),
               "r"(bytes)
               : "memory");
}

// Waits for the phase with the given parity; the thread is suspended (not
// spinning, so it takes no issue slots from working warps) for up to
// `suspend_ns` before the call returns false.
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity,
                                              uint32_t suspend_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity), "r"(suspend_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// 16 bytes into a (possibly remote) CTA's shared memory; the write counts
// 16 transaction bytes on that CTA's mbarrier.
__device__ __forceinline__ void st_async_v4(uint32_t addr, uint4 v, uint32_t mbar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
      "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(mbar)
      : "memory");
}

// 8 bytes, as above.
__device__ __forceinline__ void st_async_v2(uint32_t addr, uint32_t x, uint32_t y,
                                            uint32_t mbar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b32 [%0], {%1, %2}, [%3];" ::"r"(addr),
      "r"(x), "r"(y), "r"(mbar)
      : "memory");
}

// `bytes` from this CTA's shared memory to a (possibly remote) CTA's, through
// the bulk-copy engine; the copy counts its bytes on that CTA's mbarrier.
// Both addresses and the size are multiples of 16.  The source must have been
// made visible to the async proxy (fence_proxy_async_smem) first.
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst, uint32_t src, uint32_t bytes,
                                                     uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "r"(src), "r"(bytes), "r"(mbar)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until this thread's committed bulk copies have read their sources.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Release store / acquire load of a shared-memory word, block scope.
__device__ __forceinline__ void st_release_cta(uint32_t *p, uint32_t v) {
  asm volatile("st.release.cta.shared.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

// The same, by the threads whose `pred` holds (no divergent branch).
__device__ __forceinline__ void st_release_cta_if(bool pred, uint32_t *p, uint32_t v) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %2, 0;\n\t@q st.release.cta.shared.u32 [%0], %1;\n\t}" ::"r"(
          smem_u32(p)),
      "r"(v), "r"((uint32_t)pred)
      : "memory");
}

// Release add at GPU scope: the writes this thread has observed (its own,
// and those of threads it synchronised with, e.g. through __syncwarp) are
// visible to any thread that reads the new value with acquire semantics.
__device__ __forceinline__ void red_release_gpu_add(uint32_t *p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Acquire load of a global word, GPU scope.
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_acquire_cta(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}

// Two fp32 lanes in one 64-bit register (element 0 in the low word).
__device__ __forceinline__ unsigned long long f2pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void f2unpack(unsigned long long v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

// Squared distances of two points (packed x, y, z pairs) to one point q (each
// coordinate duplicated into both lanes) with the sm_100 packed fp32
// instructions: per lane exactly sqdist()'s ((dx*dx + dy*dy) + dz*dz), every
// operation IEEE round-to-nearest, no contraction.
__device__ __forceinline__ unsigned long long sqdist_x2(unsigned long long px, unsigned long long py,
                                                        unsigned long long pz, unsigned long long qx,
                                                        unsigned long long qy, unsigned long long qz) {
  unsigned long long r;
  asm("{\n\t.reg .b64 dx, dy, dz;\n\t"
      "sub.rn.f32x2 dx, %1, %4;\n\t"
      "sub.rn.f32x2 dy, %2, %5;\n\t"
      "sub.rn.f32x2 dz, %3, %6;\n\t"
      "mul.rn.f32x2 dx, dx, dx;\n\t"
      "mul.rn.f32x2 dy, dy, dy;\n\t"
      "mul.rn.f32x2 dz, dz, dz;\n\t"
      "add.rn.f32x2 dx, dx, dy;\n\t"
      "add.rn.f32x2 %0, dx, dz;\n\t}"
      : "=l"(r)
      : "l"(px), "l"(py), "l"(pz), "l"(qx), "l"(qy), "l"(qz));
  return r;
}

__device__ __forceinline__ float sqrt_approx(float x) {
  float r;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Order key of a distance: larger distance -> larger key; "no candidate"
// (negative distance) -> 0.  Distances are never NaN (they start at FLT_MAX
// and only take values d < old).
__device__ __forceinline__ uint32_t dkey(float d) {
  return d < 0.0f ? 0u : __float_as_uint(d) + 1u;
}

// A cube axis packed as lo | (width << 16); a cell index x is inside iff
// (x - lo) <= width in unsigned arithmetic.  kNoCell packs lo = 0xffff,
// width = 0, which no index can satisfy.
constexpr uint32_t kNoCell = 0x0000ffffu;

__device__ __forceinline__ bool in_box(uint32_t cell, uint32_t c0, uint32_t c1,
                                       uint32_t c2) {
  const uint32_t x = cell & 1023u, y = (cell >> 10) & 1023u, z = cell >> 20;
  return (x - (c0 & 0xffffu)) <= (c0 >> 16) && (y - (c1 & 0xffffu)) <= (c1 >> 16) &&
         (z - (c2 & 0xffffu)) <= (c2 >> 16);
}

// The per-axis range fields the publishing path needs, kept in registers.
struct AxisK {
  float mn, hi, inv, ovf, bsz;
  int blocks;
  const float *tab;  // shared-memory thresholds of this axis
};

// get_morton_codes_in_range (src/yuezu_fps.cpp:560-597) as a box of cells
// around q: half-width n_a = (int)ceil(sqrt(D) / block_size_a), clipped to the
// grid, packed per axis as lo | (width << 16); every axis is kNoCell when the
// reference's loops visit no cell (n < 0, or an int conversion that x86 turns
// into INT_MIN).  qc = the cell of q.
//
// fast (positive finite block sizes): n_a is read from the host's exact
// thresholds.  The guess ceil(sqrt_approx(D) * inv_bs) is within one of the
// IEEE result: the two ratios agree to a few parts in 10^7, and only
// n < blocks - 1 matters (larger half-widths all cover the whole axis), so an
// integer can lie between them only when the exact ratio is within ~4e-4 of
// it.  The three axes' guesses are checked against tab[n-1] < D <= tab[n]
// with independent loads and moved by one step without branching; a second
// miss, which the bound excludes, would fall back to walking the tables.
__device__ __forceinline__ void cube_of(const AxisK (&ax)[3], bool fast, const uint32_t (&qc)[3],
                                        float D, uint32_t (&out)[3]) {
  int n[3];
  bool empty = false;
  if (fast) {
    const float rad = sqrt_approx(D);
    float below[3], above[3];
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      const int top = ax[a].blocks - 1;
      empty = empty || (D > ax[a].ovf);
      const float guess = fminf(ceilf(rad * ax[a].inv), (float)top);
      n[a] = guess > 0.0f ? (int)guess : 0;  // NaN -> 0
      // table a has `top` entries; load only inside it
      below[a] = n[a] > 0 ? ax[a].tab[n[a] - 1] : -1.0f;
      above[a] = n[a] < top ? ax[a].tab[n[a]] : FLT_MAX;
    }
    bool again = false;
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      const int top = ax[a].blocks - 1;
      const int d = (D <= below[a]) ? -1 : ((D > above[a]) ? 1 : 0);
      n[a] += d;
      // one step is exact unless the neighbour threshold is crossed too
      again = again || (d < 0 && n[a] > 0 && D <= ax[a].tab[n[a] - 1]) ||
              (d > 0 && n[a] < top && D > ax[a].tab[n[a]]);
    }
    if (again) {  // excluded by the error bound; kept for safety
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        const int top = ax[a].blocks - 1;
        while (n[a] > 0 && D <= ax[a].tab[n[a] - 1]) --n[a];
        while (n[a] < top && D > ax[a].tab[n[a]]) ++n[a];
      }
    }
  } else {
    const float rad = __fsqrt_rn(D < 0.0f ? 0.0f : D);
#pragma unroll
    for (int a = 0; a < 3; ++a) {
      n[a] = cvt_i32_x86(ceilf(__fdiv_rn(rad, ax[a].bsz)));
      empty = empty || n[a] < 0;
      if (n[a] > ax[a].blocks) n[a] = ax[a].blocks;
    }
  }
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    const int top = ax[a].blocks - 1;
    const int l = (int)qc[a] - n[a] > 0 ? (int)qc[a] - n[a] : 0;
    const int h = (int)qc[a] + n[a] < top ? (int)qc[a] + n[a] : top;
    out[a] = empty ? kNoCell : ((uint32_t)l | ((uint32_t)(h - l) << 16));
  }
}

// Exclusive block scan of one value per thread.
template <int THREADS>
__device__ __forceinline__ uint32_t block_excl_sum(uint32_t v, uint32_t *s,
                                                   uint32_t &total) {
  constexpr int W = THREADS / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const uint32_t x = lane < W ? s[lane] : 0u;
    uint32_t xi = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(kFull, xi, o);
      if (lane >= o) xi += t;
    }
    s[lane] = xi - x;
    if (lane == 31) s[32] = xi;
  }
  __syncthreads();
  const uint32_t r = s[warp] + incl - v;
  total = s[32];
  __syncthreads();
  return r;
}

}  // namespace
}  // namespace nsfps
