/*
 * nsfps_oracle.c -- CPU restatement of the reference farthest-point sampler
 * (satreeby/ns_fps `yuezu_fps()`), used ONLY as a checker.
 *
 * TEST INFRASTRUCTURE.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py may load this library.  The
 * product (libnsfps.so and the yuezu_fps_module drop-in) never links or calls
 * it; there is no CPU fallback in the product path.
 *
 * Parity pin: this restatement is checked index-for-index against the
 * reference sources compiled in place (oracle/_ref, see oracle/Makefile) and
 * against the committed golden vectors under tests/golden/ (generated from
 * that compiled reference by tests/golden/make_golden.py).
 *
 * What the reference computes, restated over flat arrays instead of the
 * reference's MortonBlock / CacheBlock pointer tree:
 *
 *  - SpaceRange (src/yuezu_fps.cpp:98-161): inv_bs = 1.0f/((max-min)/(float)b),
 *    bits = max(1, ceil(log2 b)) (:45-50), bit-position interleave x->y->z over
 *    the common bits then the remaining bits in x,y,z order (:69-97), per-axis
 *    LUT of spread bits (:52-66).
 *  - Cell of a point (src/yuezu_fps.cpp:170-193): clamp to [min, max-1e-6f]
 *    with std::min/std::max semantics, multiply by inv_bs, truncate to
 *    uint32, clamp to blocks-1.  Bucket = (lutx|luty|lutz) % total_blocks
 *    (:195-199, :411-416).
 *  - Leaf order: every bucket keeps its points in input order (:277-283), and
 *    the cache tree walks buckets in ascending order (:431-438), so the flat
 *    order of all points is a STABLE sort by bucket.
 *  - Distances (:205-209, :234-265): d = (dx*dx + dy*dy) + dz*dz with
 *    dx = p.x - q.x, every operation rounded separately (no FMA); the cached
 *    distance starts at FLT_MAX (:215-218) and becomes min(old, d) keeping old
 *    unless d < old.
 *  - Global farthest point (:322-372, :549-558): strict '>' at the leaf and at
 *    every tree level means the winner is the largest distance, ties going to
 *    the smallest position in the flat order.
 *  - Driver (:676-730): N==0 or K==0 -> []; K>=N -> 0..N-1; sample 0 is input
 *    point 0 and its distances are applied to every point; each iteration
 *    stops if the global max is <= 0, otherwise emits the winner and updates
 *    ALL points of every bucket hit by the cell cube of half-width
 *    n_a = (int)ceil(sqrt(D)/block_size_a) around the winner's cell
 *    (:560-606).  A conversion that overflows int (x86 cvttss2si gives
 *    INT_MIN) makes the reference's cube loop visit no cell; negative n does
 *    the same.  Both are mirrored here.
 *
 * float->integer conversions follow what GCC emits for the reference on
 * x86-64 without AVX-512 (cvttss2si): out-of-range and NaN inputs give the
 * "integer indefinite" value.  This only matters for degenerate ranges.
 *
 * Build: -O2 -ffp-contract=off (see oracle/Makefile); no -ffast-math.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_BOUNDARY_EPS 1e-6f /* src/yuezu_fps.h:43-45 */

#define OR_OK 0
#define OR_ERR_ARG 1
#define OR_ERR_OOM 3

typedef struct {
  float min[3], max[3];
  uint32_t blocks[3];
  float inv_bs[3];   /* 1.0f / ((max - min) / (float)blocks)  :140-142 */
  float bsz[3];      /* (max - min) / blocks  (block_size_*)  :7-11    */
  float hi[3];       /* max - BOUNDARY_EPS                     :172-174 */
  uint32_t bits[3];
  uint32_t *lut[3];
  uint64_t total;
} or_range;

/* (uint32_t)float as emitted by GCC on x86-64: cvttss2si into a 64-bit
 * register, keep the low 32 bits. */
static inline uint32_t cvt_u32_x86(float v) {
  if (v >= -9223372036854775808.0f && v < 9223372036854775808.0f)
    return (uint32_t)(int64_t)v;
  return 0u;
}

/* (int)float on x86-64: cvttss2si 32-bit, INT_MIN when out of range. */
static inline int32_t cvt_i32_x86(float v) {
  if (v >= -2147483648.0f && v < 2147483648.0f)
    return (int32_t)v;
  return INT32_MIN;
}

/* std::min(a, b) == (b < a) ? b : a ; std::max(a, b) == (a < b) ? b : a */
static inline float std_min(float a, float b) { return (b < a) ? b : a; }
static inline float std_max(float a, float b) { return (a < b) ? b : a; }

/* src/yuezu_fps.cpp:45-50 */
static uint32_t or_calc_bits(uint32_t blocks) {
  uint32_t bits = 0;
  while (bits < 32 && (1u << bits) < blocks)
    ++bits;
  return bits ? bits : 1;
}

static void or_range_free(or_range *r) {
  for (int a = 0; a < 3; ++a) {
    free(r->lut[a]);
    r->lut[a] = NULL;
  }
}

/* make_range (src/yuezu_fps.cpp:136-161) with the bit interleave of :69-97
 * and the LUT of :52-66. */
static int or_range_init(or_range *r, const float rng[6],
                         const uint32_t blocks[3]) {
  memset(r, 0, sizeof(*r));
  for (int a = 0; a < 3; ++a) {
    if (blocks[a] == 0 || blocks[a] > (1u << 20))
      return OR_ERR_ARG;
    r->min[a] = rng[2 * a];
    r->max[a] = rng[2 * a + 1];
    r->blocks[a] = blocks[a];
    float span = r->max[a] - r->min[a];
    float bs = span / (float)blocks[a];
    r->inv_bs[a] = 1.0f / bs;
    r->bsz[a] = span / (float)blocks[a];
    r->hi[a] = r->max[a] - OR_BOUNDARY_EPS;
    r->bits[a] = or_calc_bits(blocks[a]);
  }
  if (r->bits[0] + r->bits[1] + r->bits[2] > 32)
    return OR_ERR_ARG;
  r->total = (uint64_t)blocks[0] * blocks[1] * blocks[2];

  uint32_t pos[3][32];
  uint32_t npos[3] = {0, 0, 0};
  uint32_t bit = 0;
  uint32_t xb = r->bits[0], yb = r->bits[1], zb = r->bits[2];
  uint32_t common = xb < yb ? xb : yb;
  common = common < zb ? common : zb;
  uint32_t maxb = xb > yb ? xb : yb;
  maxb = maxb > zb ? maxb : zb;
  for (uint32_t i = 0; i < common; ++i)
    for (int a = 0; a < 3; ++a)
      pos[a][npos[a]++] = bit++;
  for (uint32_t i = common; i < maxb; ++i)
    for (int a = 0; a < 3; ++a)
      if (i < r->bits[a])
        pos[a][npos[a]++] = bit++;

  for (int a = 0; a < 3; ++a) {
    uint32_t count = 1u << r->bits[a];
    r->lut[a] = (uint32_t *)malloc(sizeof(uint32_t) * count);
    if (!r->lut[a]) {
      or_range_free(r);
      return OR_ERR_OOM;
    }
    for (uint32_t v = 0; v < count; ++v) {
      uint32_t code = 0;
      for (uint32_t k = 0; k < r->bits[a]; ++k)
        if (v & (1u << k))
          code |= 1u << pos[a][k];
      r->lut[a][v] = code;
    }
  }
  return OR_OK;
}

/* Point3D::compute_block_indices, src/yuezu_fps.cpp:170-193 */
static inline void or_cell(const or_range *r, float x, float y, float z,
                           uint32_t c[3]) {
  const float p[3] = {x, y, z};
  for (int a = 0; a < 3; ++a) {
    float cl = std_max(r->min[a], std_min(p[a], r->hi[a]));
    uint32_t i = cvt_u32_x86((cl - r->min[a]) * r->inv_bs[a]);
    uint32_t lim = r->blocks[a] - 1;
    c[a] = i < lim ? i : lim;
  }
}

/* compute_morton_code + hash, src/yuezu_fps.cpp:195-199, :411-416 */
static inline uint64_t or_bucket_of_cell(const or_range *r, const uint32_t c[3]) {
  uint32_t code = r->lut[0][c[0]] | r->lut[1][c[1]] | r->lut[2][c[2]];
  return (uint64_t)code % r->total;
}

/* squared_distance, src/yuezu_fps.cpp:205-209 (each op rounded) */
static inline float or_sqd(float px, float py, float pz, float qx, float qy,
                           float qz) {
  /* compiled with -ffp-contract=off: no multiply-add fusion */
  float dx = px - qx, dy = py - qy, dz = pz - qz;
  return dx * dx + dy * dy + dz * dz;
}

typedef struct {
  float d;
  uint32_t rank;
} or_key;

/* larger distance wins; equal distance -> smaller flat rank */
static inline int or_better(or_key a, or_key b) {
  return a.d > b.d || (a.d == b.d && a.rank < b.rank);
}

typedef struct {
  uint64_t n, k, total;
  float *sx, *sy, *sz, *dist;
  uint64_t *orig;
  uint64_t *bstart; /* total + 1 */
  uint32_t *stamp;
  or_key *tree; /* 2 * size, leaves at [size, 2 size) */
  uint64_t size;
} or_state;

static void or_state_free(or_state *s) {
  free(s->sx);
  free(s->sy);
  free(s->sz);
  free(s->dist);
  free(s->orig);
  free(s->bstart);
  free(s->stamp);
  free(s->tree);
}

/* max over one bucket, first strict '>' wins (MortonBlock::update_distance
 * :245-261 then CacheBlock :339-343) */
static or_key or_bucket_max(const or_state *s, uint64_t b) {
  or_key best = {-1.0f, UINT32_MAX};
  for (uint64_t i = s->bstart[b]; i < s->bstart[b + 1]; ++i)
    if (s->dist[i] > best.d) {
      best.d = s->dist[i];
      best.rank = (uint32_t)i;
    }
  return best;
}

static void or_tree_set(or_state *s, uint64_t b, or_key v) {
  uint64_t i = b + s->size;
  s->tree[i] = v;
  for (i >>= 1; i >= 1; i >>= 1) {
    or_key l = s->tree[2 * i], r = s->tree[2 * i + 1];
    s->tree[i] = or_better(r, l) ? r : l;
  }
}

static void or_update_bucket(or_state *s, uint64_t b, float qx, float qy,
                             float qz) {
  for (uint64_t i = s->bstart[b]; i < s->bstart[b + 1]; ++i) {
    float d = or_sqd(s->sx[i], s->sy[i], s->sz[i], qx, qy, qz);
    if (d < s->dist[i])
      s->dist[i] = d;
  }
  or_tree_set(s, b, or_bucket_max(s, b));
}

/*
 * nsfps_oracle_fps: yuezu_fps(points, k, make_range(rng, blocks)).
 *   xyz      : n x 3 floats, dense
 *   out      : capacity k (receives original indices)
 *   sum_u    : optional, receives the number of points in all buckets the
 *              reference updates, summed over iterations 1..len-1 (the
 *              reference's per-iteration work, src/yuezu_fps.cpp:714-720)
 *   u_iter   : optional, capacity k, per-iteration point counts
 * Returns 0, OR_ERR_ARG or OR_ERR_OOM.
 */
int nsfps_oracle_fps(const float *xyz, uint64_t n, uint64_t k,
                     const float rng[6], const uint32_t blocks[3],
                     uint64_t *out, uint64_t *out_len, uint64_t *sum_u,
                     uint64_t *u_iter) {
  *out_len = 0;
  if (sum_u)
    *sum_u = 0;
  if (n == 0 || k == 0)
    return OR_OK;
  if (k >= n) {
    for (uint64_t i = 0; i < n; ++i)
      out[i] = i;
    *out_len = n;
    return OR_OK;
  }
  or_range r;
  int rc = or_range_init(&r, rng, blocks);
  if (rc)
    return rc;
  if (r.total > (1ull << 28) || n > 0xFFFFFFFFull) {
    or_range_free(&r);
    return OR_ERR_ARG;
  }

  or_state s;
  memset(&s, 0, sizeof(s));
  s.n = n;
  s.k = k;
  s.total = r.total;
  uint64_t *bucket = (uint64_t *)malloc(sizeof(uint64_t) * n);
  s.sx = (float *)malloc(sizeof(float) * n);
  s.sy = (float *)malloc(sizeof(float) * n);
  s.sz = (float *)malloc(sizeof(float) * n);
  s.dist = (float *)malloc(sizeof(float) * n);
  s.orig = (uint64_t *)malloc(sizeof(uint64_t) * n);
  s.bstart = (uint64_t *)calloc(r.total + 1, sizeof(uint64_t));
  s.stamp = (uint32_t *)calloc(r.total, sizeof(uint32_t));
  s.size = 1;
  while (s.size < r.total)
    s.size <<= 1;
  s.tree = (or_key *)malloc(sizeof(or_key) * 2 * s.size);
  if (!bucket || !s.sx || !s.sy || !s.sz || !s.dist || !s.orig || !s.bstart ||
      !s.stamp || !s.tree) {
    free(bucket);
    or_state_free(&s);
    or_range_free(&r);
    return OR_ERR_OOM;
  }

  /* binning + stable counting sort by bucket */
  for (uint64_t i = 0; i < n; ++i) {
    uint32_t c[3];
    or_cell(&r, xyz[3 * i], xyz[3 * i + 1], xyz[3 * i + 2], c);
    bucket[i] = or_bucket_of_cell(&r, c);
    s.bstart[bucket[i] + 1]++;
  }
  for (uint64_t b = 0; b < r.total; ++b)
    s.bstart[b + 1] += s.bstart[b];
  {
    uint64_t *fill = (uint64_t *)malloc(sizeof(uint64_t) * r.total);
    if (!fill) {
      free(bucket);
      or_state_free(&s);
      or_range_free(&r);
      return OR_ERR_OOM;
    }
    memcpy(fill, s.bstart, sizeof(uint64_t) * r.total);
    for (uint64_t i = 0; i < n; ++i) {
      uint64_t p = fill[bucket[i]]++;
      s.sx[p] = xyz[3 * i];
      s.sy[p] = xyz[3 * i + 1];
      s.sz[p] = xyz[3 * i + 2];
      s.orig[p] = i;
    }
    free(fill);
  }
  free(bucket);

  /* first sample: input point 0, applied to every point
   * (build_multilevel_cache, :418-438) */
  const float p0x = xyz[0], p0y = xyz[1], p0z = xyz[2];
  for (uint64_t i = 0; i < n; ++i) {
    float d = or_sqd(s.sx[i], s.sy[i], s.sz[i], p0x, p0y, p0z);
    s.dist[i] = (d < FLT_MAX) ? d : FLT_MAX;
  }
  for (uint64_t i = 0; i < 2 * s.size; ++i) {
    s.tree[i].d = -1.0f;
    s.tree[i].rank = UINT32_MAX;
  }
  for (uint64_t b = 0; b < r.total; ++b)
    s.tree[s.size + b] = or_bucket_max(&s, b);
  for (uint64_t i = s.size - 1; i >= 1; --i) {
    or_key a = s.tree[2 * i], c = s.tree[2 * i + 1];
    s.tree[i] = or_better(c, a) ? c : a;
  }

  out[0] = 0;
  uint64_t len = 1;
  if (u_iter)
    u_iter[0] = n;
  for (uint64_t it = 1; it < k; ++it) {
    or_key top = s.tree[1];
    float D = top.d;
    if (D <= 0.0f) /* :705-706 */
      break;
    uint32_t w = top.rank;
    out[len++] = s.orig[w];
    const float qx = s.sx[w], qy = s.sy[w], qz = s.sz[w];

    /* get_morton_codes_in_range, :560-597 */
    float dsq = D < 0.0f ? 0.0f : D;
    float rad = sqrtf(dsq);
    int32_t nn[3];
    int empty = 0;
    for (int a = 0; a < 3; ++a) {
      nn[a] = cvt_i32_x86(ceilf(rad / r.bsz[a]));
      if (nn[a] < 0)
        empty = 1;
    }
    uint64_t u = 0;
    if (!empty) {
      uint32_t c[3];
      or_cell(&r, qx, qy, qz, c);
      int64_t lo[3], hi[3];
      for (int a = 0; a < 3; ++a) {
        lo[a] = (int64_t)c[a] - nn[a];
        hi[a] = (int64_t)c[a] + nn[a];
        if (lo[a] < 0)
          lo[a] = 0;
        if (hi[a] > (int64_t)r.blocks[a] - 1)
          hi[a] = (int64_t)r.blocks[a] - 1;
      }
      const uint32_t tag = (uint32_t)it;
      for (int64_t bz = lo[2]; bz <= hi[2]; ++bz)
        for (int64_t by = lo[1]; by <= hi[1]; ++by)
          for (int64_t bx = lo[0]; bx <= hi[0]; ++bx) {
            uint32_t cc[3] = {(uint32_t)bx, (uint32_t)by, (uint32_t)bz};
            uint64_t b = or_bucket_of_cell(&r, cc);
            if (s.stamp[b] == tag)
              continue; /* a bucket hit twice gets the same result */
            s.stamp[b] = tag;
            u += s.bstart[b + 1] - s.bstart[b];
            or_update_bucket(&s, b, qx, qy, qz);
          }
    }
    if (sum_u)
      *sum_u += u;
    if (u_iter)
      u_iter[len - 1] = u;
  }
  *out_len = len;
  or_state_free(&s);
  or_range_free(&r);
  return OR_OK;
}

/* compute_bbox, src/yuezu_fps.cpp:648-670: out = {min_x-eps, max_x+eps, ...} */
void nsfps_oracle_bbox(const float *xyz, uint64_t n, float out[6]) {
  if (n == 0) {
    const float e[6] = {0, 1, 0, 1, 0, 1};
    memcpy(out, e, sizeof(e));
    return;
  }
  float mn[3] = {xyz[0], xyz[1], xyz[2]};
  float mx[3] = {xyz[0], xyz[1], xyz[2]};
  for (uint64_t i = 0; i < n; ++i)
    for (int a = 0; a < 3; ++a) {
      mn[a] = std_min(mn[a], xyz[3 * i + a]);
      mx[a] = std_max(mx[a], xyz[3 * i + a]);
    }
  for (int a = 0; a < 3; ++a) {
    out[2 * a] = mn[a] - OR_BOUNDARY_EPS;
    out[2 * a + 1] = mx[a] + OR_BOUNDARY_EPS;
  }
}

/* SpaceRange derived fields for host-logic tests:
 * f_out = {inv_bs x3, block_size x3}, u_out = {bits x3, total_bits},
 * luts (optional) receive 2^bits entries per axis. */
int nsfps_oracle_range_info(const float rng[6], const uint32_t blocks[3],
                            float f_out[6], uint32_t u_out[4], uint32_t *lutx,
                            uint32_t *luty, uint32_t *lutz) {
  or_range r;
  int rc = or_range_init(&r, rng, blocks);
  if (rc)
    return rc;
  for (int a = 0; a < 3; ++a) {
    f_out[a] = r.inv_bs[a];
    f_out[3 + a] = r.bsz[a];
    u_out[a] = r.bits[a];
  }
  u_out[3] = r.bits[0] + r.bits[1] + r.bits[2];
  uint32_t *dst[3] = {lutx, luty, lutz};
  for (int a = 0; a < 3; ++a)
    if (dst[a])
      memcpy(dst[a], r.lut[a], sizeof(uint32_t) * (1u << r.bits[a]));
  or_range_free(&r);
  return OR_OK;
}

/* Cell and bucket of each point (for host-logic tests of the binning). */
int nsfps_oracle_bin(const float *xyz, uint64_t n, const float rng[6],
                     const uint32_t blocks[3], uint32_t *cells /* n x 3 */,
                     uint64_t *buckets /* n */) {
  or_range r;
  int rc = or_range_init(&r, rng, blocks);
  if (rc)
    return rc;
  for (uint64_t i = 0; i < n; ++i) {
    uint32_t c[3];
    or_cell(&r, xyz[3 * i], xyz[3 * i + 1], xyz[3 * i + 2], c);
    if (cells) {
      cells[3 * i] = c[0];
      cells[3 * i + 1] = c[1];
      cells[3 * i + 2] = c[2];
    }
    if (buckets)
      buckets[i] = or_bucket_of_cell(&r, c);
  }
  or_range_free(&r);
  return OR_OK;
}

/* ---- Grouping after sampling.  The reference stops at the sample indices
 * (src/yuezu_fps.cpp:676-730) and has no ball query, so this part is not
 * pinned against it: it restates the PointNet++ query_ball_point definition
 * by brute force, with the sampler's distance (or_sqd, no FMA).  For each
 * centre, walk the points in index order, keep those with
 * d2 < radius * radius, stop after nsample; the remaining slots repeat the
 * first hit, or hold 0 when there is none.  hits[j] = number kept. */
int nsfps_oracle_ball_query(const float *xyz, uint64_t n, const float *centers,
                            uint64_t m, float radius, uint32_t nsample,
                            int64_t *idx, uint32_t *hits) {
  const float r2 = radius * radius;
  for (uint64_t j = 0; j < m; ++j) {
    const float cx = centers[3 * j], cy = centers[3 * j + 1],
                cz = centers[3 * j + 2];
    int64_t *row = idx + j * (uint64_t)nsample;
    uint32_t cnt = 0;
    for (uint64_t k = 0; k < n && cnt < nsample; ++k) {
      const float d2 =
          or_sqd(xyz[3 * k], xyz[3 * k + 1], xyz[3 * k + 2], cx, cy, cz);
      if (d2 < r2) {
        if (cnt == 0)
          for (uint32_t l = 0; l < nsample; ++l)
            row[l] = (int64_t)k;
        row[cnt++] = (int64_t)k;
      }
    }
    if (cnt == 0)
      for (uint32_t l = 0; l < nsample; ++l)
        row[l] = 0;
    if (hits)
      hits[j] = cnt;
  }
  return OR_OK;
}
