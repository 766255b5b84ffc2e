/*
 * oracle.c -- CPU restatement of Quiver's query hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA engine, loaded by
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg.  The
 * product never links or calls it.  Citations are path:line inside the
 * reference project (ruc-system/quiver-ae).
 *
 * Compile with -ffp-contract=off: every fused multiply-add below is an
 * explicit fmaf(), and every other operation is a separately rounded fp32
 * operation, so the results do not depend on the host compiler.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_PAGE 4096
#define ORC_PIVOTS 256
#define ORC_VISITED 0x80000000u
#define ORC_IDMASK 0x7fffffffu

/* ---------------------------------------------------------------- LUT -- */

/* pq_device.cuh:9-36.  q' = fl(q - c); for i ascending and every pivot j,
 * LUT[chunk(i)][j] = fma(q'_i - p_ij, q'_i - p_ij, LUT[chunk(i)][j]);
 * finally the query is overwritten with q'' = fl(q' + c), which is what the
 * exact-L2 stage later reads (kernel_q1.cuh:180 then kernel_helpers.cuh:477). */
void orc_build_lut(const orc_index* ix, const float* query, float* lut, float* q2) {
  const int64_t dim = ix->dim;
  const int32_t M = ix->num_chunks;
  memset(lut, 0, sizeof(float) * (size_t)M * ORC_PIVOTS);
  for (int64_t i = 0; i < dim; ++i) q2[i] = query[i] - ix->centroid[i];
  for (int32_t c = 0; c < M; ++c) {
    /* chunk c owns dims [off[c], off[c+1]) (pq_search.cu:157-163) */
    for (int64_t i = ix->chunk_offsets[c]; i < ix->chunk_offsets[c + 1]; ++i) {
      const float qi = q2[i];
      const float* p = ix->pivots_t + i * ORC_PIVOTS;
      float* row = lut + (size_t)c * ORC_PIVOTS;
      for (int j = 0; j < ORC_PIVOTS; ++j) {
        const float d = qi - p[j];
        row[j] = fmaf(d, d, row[j]);
      }
    }
  }
  for (int64_t i = 0; i < dim; ++i) q2[i] = q2[i] + ix->centroid[i];
}

/* kernel_helpers.cuh:280-285: dist = 0; dist += LUT[j*256 + code[j]]. */
float orc_adc(const float* lut, const uint8_t* code, int32_t M) {
  float d = 0.0f;
  for (int32_t j = 0; j < M; ++j) d = d + lut[j * ORC_PIVOTS + code[j]];
  return d;
}

/* ----------------------------------------------------------- exact L2 -- */

static inline float elem_as_float(const void* vec, int64_t i, int32_t dtype) {
  if (dtype == ORC_UINT8) return (float)((const uint8_t*)vec)[i];
  if (dtype == ORC_INT8) return (float)((const int8_t*)vec)[i];
  float f;
  memcpy(&f, (const uint8_t*)vec + 4 * i, 4);
  return f;
}

/* gpu_primitives.cuh:26-44.  Lane l accumulates dims l, l+32, ... with a
 * fused multiply-add; then val += shfl_down(val, off) for off = 16..1, and
 * lane 0 holds the result.  A lane whose source is out of range adds its own
 * value (shfl_down returns the caller's value); only lane 0 is returned. */
float orc_exact_l2(const float* q2, const void* vec, int64_t dim, int32_t dtype) {
  float v[32], t[32];
  for (int l = 0; l < 32; ++l) {
    float acc = 0.0f;
    for (int64_t i = l; i < dim; i += 32) {
      const float diff = q2[i] - elem_as_float(vec, i, dtype);
      acc = fmaf(diff, diff, acc);
    }
    v[l] = acc;
  }
  for (int off = 16; off > 0; off >>= 1) {
    for (int l = 0; l < 32; ++l) t[l] = v[l] + ((l + off < 32) ? v[l + off] : v[l]);
    memcpy(v, t, sizeof(v));
  }
  return v[0];
}

/* --------------------------------------------------------- list state -- */

typedef struct {
  uint32_t* lid; float* ldist; int size;      /* neighbor_id / neighbor_dist, ctx->size */
  uint32_t* tid; float* tdist;                /* tmp_id / tmp_dist */
  uint32_t* mid; float* mdist; int* mpos;     /* mv_id / mv_dist / mv_pos */
  int32_t* rid; float* rdist; int fc;         /* top-k: nns / distances / found_cnt */
  float* lut; float* q2;
  int64_t nbrs;                               /* neighbours scored */
  /* visited-filter mode: ids scheduled for expansion this query (open
   * addressing, id + 1, 0 = empty) */
  uint32_t* vset; int64_t vcap, vcount; int vfilter;
  int route_exact;                            /* diagnostic: exact L2 instead of ADC */
} orc_ctx;

static uint64_t vhash(uint32_t id) { return (uint64_t)id * 0x9E3779B97F4A7C15ull; }

static int vset_has(const orc_ctx* c, uint32_t id) {
  for (uint64_t h = vhash(id) & (c->vcap - 1);; h = (h + 1) & (c->vcap - 1)) {
    if (c->vset[h] == 0) return 0;
    if (c->vset[h] == id + 1) return 1;
  }
}

static void vset_add(orc_ctx* c, uint32_t id) {
  if (2 * (c->vcount + 1) > c->vcap) {  /* grow */
    const int64_t old = c->vcap;
    uint32_t* prev = c->vset;
    c->vcap = old * 2;
    c->vset = (uint32_t*)calloc((size_t)c->vcap, sizeof(uint32_t));
    c->vcount = 0;
    for (int64_t i = 0; i < old; ++i)
      if (prev[i]) vset_add(c, prev[i] - 1);
    free(prev);
  }
  uint64_t h = vhash(id) & (c->vcap - 1);
  for (; c->vset[h] != 0; h = (h + 1) & (c->vcap - 1))
    if (c->vset[h] == id + 1) return;
  c->vset[h] = id + 1;
  c->vcount++;
}

/* gpu_primitives.cuh:140-153: first index in [l, r) whose (dist, id&mask)
 * key is not below (d, x&mask). */
static int orc_lower_bound(const float* dist, const uint32_t* id, int l, int r,
                           float d, uint32_t x) {
  x &= ORC_IDMASK;
  while (l < r) {
    const int mid = (l + r) / 2;
    if (dist[mid] < d || (dist[mid] == d && (id[mid] & ORC_IDMASK) < x))
      l = mid + 1;
    else
      r = mid;
  }
  return l;
}

static inline int key_less(float ad, uint32_t aid, float bd, uint32_t bid) {
  aid &= ORC_IDMASK;
  bid &= ORC_IDMASK;
  return ad < bd || (ad == bd && aid < bid);
}

static inline const uint8_t* node_record(const orc_index* ix, int64_t v) {
  /* page = node / nodes_per_page (search.cu:240); the record sits at
   * (node % nodes_per_page) * node_size inside it (kernel_helpers.cuh:257). */
  return ix->pages + (v / ix->nodes_per_page) * ORC_PAGE +
         (v % ix->nodes_per_page) * ix->node_size;
}

/* kernel_helpers.cuh:232-357 (generic path).  Returns 0, or -1 for a
 * neighbour id >= N, -2 for a degree above R. */
static int orc_merge(const orc_index* ix, orc_ctx* c, int64_t node, int ef) {
  const uint8_t* rec = node_record(ix, node);
  const int sz = c->size < ef ? c->size : ef;            /* 253-255 */
  for (int i = 0; i < sz; ++i) {                          /* 265-268 */
    c->tid[i] = c->lid[i];
    c->tdist[i] = c->ldist[i];
  }
  uint32_t deg;
  memcpy(&deg, rec + ix->data_size, 4);                   /* 263, 271 */
  if (deg > (uint32_t)ix->max_degree) return -2;
  const int32_t M = ix->num_chunks;
  for (uint32_t t = 0; t < deg; ++t) {                    /* 278-285 */
    uint32_t nb;
    memcpy(&nb, rec + ix->data_size + 4 + 4 * (int64_t)t, 4);
    if ((int64_t)nb >= ix->num_points) return -1;
    c->tid[sz + t] = nb;
    c->tdist[sz + t] = c->route_exact
        ? orc_exact_l2(c->q2, node_record(ix, nb), ix->dim, ix->data_type)
        : orc_adc(c->lut, ix->codes + (int64_t)nb * M, M);
  }
  c->nbrs += deg;
  if (c->vfilter) {  /* visited-filter mode: drop ids already scheduled for expansion */
    uint32_t kept = 0;
    for (uint32_t t = 0; t < deg; ++t) {
      if (vset_has(c, c->tid[sz + t])) continue;
      c->tid[sz + kept] = c->tid[sz + t];
      c->tdist[sz + kept] = c->tdist[sz + t];
      ++kept;
    }
    deg = kept;
  }
  /* 300-329: sort the deg new pairs ascending by (dist, id&mask).  Keys are
   * distinct for an index whose adjacency lists hold distinct ids, so any
   * correct sort gives the reference's order.  Binary insertion sort. */
  uint32_t* nid = c->tid + sz;
  float* nd = c->tdist + sz;
  for (uint32_t t = 1; t < deg; ++t) {
    const uint32_t kid = nid[t];
    const float kd = nd[t];
    int lo = 0, hi = (int)t;
    while (lo < hi) {
      const int mid = (lo + hi) / 2;
      if (key_less(kd, kid, nd[mid], nid[mid])) hi = mid; else lo = mid + 1;
    }
    for (int s = (int)t; s > lo; --s) { nid[s] = nid[s - 1]; nd[s] = nd[s - 1]; }
    nid[lo] = kid;
    nd[lo] = kd;
  }
  /* 331-341: merge positions.  A new pair equal (by id) to a list entry is
   * placed right after it; a list entry is placed after every new pair with
   * a strictly smaller key. */
  for (uint32_t t = 0; t < deg; ++t) {
    int id = orc_lower_bound(c->tdist, c->tid, 0, sz, nd[t], nid[t]);
    if (id != sz && ((c->tid[id] ^ nid[t]) & ORC_IDMASK) == 0) id++;
    c->mpos[sz + t] = id + (int)t;
  }
  for (int i = 0; i < sz; ++i)
    c->mpos[i] = orc_lower_bound(nd, nid, 0, (int)deg, c->tdist[i], c->tid[i]) + i;
  for (int i = 0; i < sz + (int)deg; ++i) {               /* 344-347 */
    c->mid[c->mpos[i]] = c->tid[i];
    c->mdist[c->mpos[i]] = c->tdist[i];
  }
  const int target = (sz + (int)deg) < 2 * ef ? sz + (int)deg : 2 * ef; /* 350-355 */
  for (int i = 0; i < target; ++i) {
    c->lid[i] = c->mid[i];
    c->ldist[i] = c->mdist[i];
  }
  c->size = target;
  return 0;
}

/* kernel_helpers.cuh:65-104 (k <= 32) and gpu_primitives.cuh:99-138 (k > 32):
 * both insert at the count of entries <= d and cap the size at k. */
static void orc_topk_insert(orc_ctx* c, int k, float d, int32_t id) {
  int pos = 0;
  while (pos < c->fc && c->rdist[pos] <= d) ++pos;
  const int nsz = c->fc < k ? c->fc + 1 : k;
  for (int i = nsz - 1; i > pos; --i) {
    c->rdist[i] = c->rdist[i - 1];
    c->rid[i] = c->rid[i - 1];
  }
  c->rdist[pos] = d;
  c->rid[pos] = id;
  c->fc = nsz;
}

/* kernel_helpers.cuh:422-489 persistent_visit_select_dualwarp: warp 1 scores
 * the expanded node exactly and inserts it into the top-k (475-486); warp 0
 * drops entries whose id repeats the previous entry's (440-455), then takes
 * the first unvisited entry below min(size, ef), marks it, and truncates the
 * list to ef (456-473). */
static int32_t orc_visit_select(const orc_index* ix, orc_ctx* c, int64_t node,
                                int ef, int k) {
  const uint8_t* rec = node_record(ix, node);
  const float d = orc_exact_l2(c->q2, rec, ix->dim, ix->data_type);
  if (c->fc < k || d < c->rdist[k - 1]) orc_topk_insert(c, k, d, (int32_t)node);

  int sz = c->size;
  if (sz == 0) return -1;
  int w = 0;
  uint32_t prev = 0;
  for (int i = 0; i < sz; ++i) {
    const uint32_t cur = c->lid[i];
    const int dup = (i != 0) && (((cur ^ prev) & ORC_IDMASK) == 0);
    prev = cur;
    if (dup) continue;
    c->lid[w] = cur;
    c->ldist[w] = c->ldist[i];
    ++w;
  }
  sz = w;
  const int lim = sz < ef ? sz : ef;
  int32_t next = -1;
  for (int i = 0; i < lim; ++i) {
    if ((c->lid[i] & ORC_VISITED) == 0) {
      next = (int32_t)(c->lid[i] & ORC_IDMASK);
      c->lid[i] |= ORC_VISITED;
      break;
    }
  }
  c->size = lim;
  return next;
}

/* kernel_helpers.cuh:491-518 persistent_select_next_no_compact. */
static int32_t orc_select_no_compact(orc_ctx* c, int ef) {
  const int sz = c->size < ef ? c->size : ef;
  if (sz == 0) return -1;
  int32_t next = -1;
  for (int i = 0; i < sz; ++i) {
    if ((c->lid[i] & ORC_VISITED) == 0) {
      next = (int32_t)(c->lid[i] & ORC_IDMASK);
      c->lid[i] |= ORC_VISITED;
      break;
    }
  }
  c->size = sz;
  return next;
}

/* ----------------------------------------------------------- gpruning -- */

typedef struct {
  int step, cnt, last_fc;
  float last_top1, last_topk;
} orc_gp;

/* kernel_q1.cuh:294-315 and 524-545. Returns 1 when the query must stop. */
static int orc_gpruning(orc_gp* g, const orc_ctx* c, const orc_params* p) {
  const int k = p->topk;
  const int improved = c->fc > g->last_fc || c->rdist[0] < g->last_top1 ||
                       c->rdist[k - 1] < g->last_topk;
  if (g->step < p->gpruning_warmup_steps)
    g->cnt = 0;
  else
    g->cnt = improved ? 0 : g->cnt + 1;
  g->last_fc = c->fc;
  g->last_top1 = c->rdist[0];
  g->last_topk = c->rdist[k - 1];
  return p->early_exit_policy == ORC_EXIT_GPRUNING &&
         g->step >= p->gpruning_warmup_steps && p->gpruning_patience > 0 &&
         g->cnt >= p->gpruning_patience;
}


/* ------------------------------------------------------------ nav entry -- */

#define ORC_NAV_L 4   /* inkernel_nav.cuh:51 */
#define ORC_NAV_R 28  /* inkernel_nav.cuh:52 */

/* Neighbour i of nav node u as the reference reads it: graph[max_m * u + i]
 * for i < 28 (inkernel_nav.cuh:113-119), so a row shorter than 28 runs on
 * into the next row; past the array's end the row counts as ended. */
static int32_t nav_edge(const orc_nav* nav, int32_t u, int i) {
  const int64_t at = (int64_t)nav->max_m * u + i;
  if (at >= (int64_t)nav->num_node * nav->max_m) return -1;
  return nav->graph[at];
}

static float nav_dist(const orc_index* ix, const orc_nav* nav, const float* q, int32_t v) {
  const int64_t elem = ix->data_type == ORC_FLOAT ? 4 : 1;
  return orc_exact_l2(q, nav->data + (int64_t)v * ix->dim * elem, ix->dim, ix->data_type);
}

int64_t orc_nav_entry(const orc_index* ix, const orc_nav* nav, const float* q) {
  const int L = ORC_NAV_L, R = ORC_NAV_R;
  uint32_t pid[32];
  float pd[32];
  if (nav->start < 0 || nav->start >= nav->num_node) return -20;
  /* 82-94: the start node in slot 0, empty slots */
  pid[0] = (uint32_t)nav->start;
  pd[0] = nav_dist(ix, nav, q, nav->start);
  for (int l = 1; l < L + R; ++l) { pid[l] = 0xffffffffu; pd[l] = INFINITY; }
  int idx = 0;
  /* the four best only improve, so the walk ends; the cap is a safety net */
  const int64_t cap = 4 * (int64_t)nav->num_node + 64;
  for (int64_t hop = 0; idx != -1; ++hop) {
    if (hop > cap) return -21;
    const int32_t u = (int32_t)(pid[idx] & ORC_IDMASK);
    if (u >= nav->num_node) return -22;
    pid[idx] |= ORC_VISITED;                                  /* 101-104 */
    /* 113-135: four warps take 7 neighbour slots each; a warp stops at its
     * first -1, leaving its remaining slots as they were */
    for (int w = 0; w < 4; ++w) {
      for (int i = 7 * w; i < 7 * w + 7 && i < R; ++i) {
        const int32_t v = nav_edge(nav, u, i);
        if (v == -1) break;
        if (v < 0 || v >= nav->num_node) return -22;
        pid[i + L] = (uint32_t)v;
        pd[i + L] = nav_dist(ix, nav, q, v);
      }
    }
    /* 142-182: four rounds; round i moves the smallest remaining slot to i */
    for (int i = 0; i < L; ++i) {
      float dist[32];
      int pos[32];
      int dupl[32];
      for (int l = 0; l < 32; ++l) {
        dist[l] = pd[l];
        pos[l] = l;
        dupl[l] = 0;
        if (l < i) dist[l] = INFINITY;
        else if (i != 0 && ((pid[l] ^ pid[i - 1]) & ORC_IDMASK) == 0) dupl[l] = 1;
      }
      /* a copy of the previous round's pick gives it its visited bit and
       * leaves the race (the reference ORs from several lanes at once; here
       * every copy's bit is kept) */
      for (int l = 0; l < 32; ++l) {
        if (!dupl[l]) continue;
        pid[i - 1] |= pid[l];
        pd[l] = INFINITY;
        dist[l] = INFINITY;
      }
      /* 159-167: shfl_down argmin tree; a value replaces only a strictly
       * larger one, and a lane past 31 reads its own value */
      for (int off = 16; off > 0; off >>= 1) {
        float nd[32];
        int np[32];
        for (int l = 0; l < 32; ++l) {
          const int src = l + off < 32 ? l + off : l;
          nd[l] = dist[l];
          np[l] = pos[l];
          if (dist[src] < dist[l]) { nd[l] = dist[src]; np[l] = pos[src]; }
        }
        memcpy(dist, nd, sizeof(dist));
        memcpy(pos, np, sizeof(pos));
      }
      const int p0 = pos[0];
      if (i != p0) {                                            /* 170-180 */
        const float t = pd[i], y = pd[p0];
        if (t != y) {
          pd[i] = y; pd[p0] = t;
          const uint32_t m = pid[i]; pid[i] = pid[p0]; pid[p0] = m;
        }
      }
    }
    /* 186-191: the first unvisited slot, if it is one of the first four */
    idx = -1;
    for (int l = 0; l < 32; ++l) {
      if (!(pid[l] & ORC_VISITED)) { idx = l < L ? l : -1; break; }
    }
  }
  const uint32_t raw = pid[0] & ORC_IDMASK;                   /* 199-200 */
  if (raw >= (uint32_t)nav->num_node) return -23;
  const int32_t entry = nav->mapping[raw];
  if (entry < 0 || entry >= ix->num_points) return -24;
  return entry;
}

/* ------------------------------------------------------------- search -- */

/* One query, kernel_q1.cuh:180-704 with every issued lane completing before
 * the next poll: each pipe iteration expands the active lanes in lane order
 * (489-600), then refills the lanes that were idle (619-630). */
static int orc_search_one(const orc_index* ix, const orc_nav* nav, orc_ctx* c, const float* q,
                          const orc_params* p, int32_t* lane_req, int* out_steps) {
  const int ef = p->ef_search, k = p->topk, W = p->pipe_width;
  const int early = p->early_exit_policy != ORC_EXIT_NONE;
  orc_build_lut(ix, q, c->lut, c->q2);
  c->size = 0;
  c->fc = 0;
  c->nbrs = 0;
  for (int i = 0; i < k; ++i) { c->rdist[i] = INFINITY; c->rid[i] = -1; }
  for (int w = 0; w < W; ++w) lane_req[w] = -1;

  orc_gp g = {0, 0, 0, INFINITY, INFINITY};
  /* 149-202: the nav result when a nav graph is loaded, else the medoid;
   * nav reads the query before the centroid round trip */
  int64_t entry = ix->medoid;
  if (nav) {
    entry = orc_nav_entry(ix, nav, q);
    if (entry < 0) return (int)entry;
  }
  c->vfilter = p->visited_filter;
  c->route_exact = p->route_exact;
  if (c->vfilter) {
    memset(c->vset, 0, sizeof(uint32_t) * c->vcap);
    c->vcount = 0;
    vset_add(c, (uint32_t)entry);
  }
  int rc = orc_merge(ix, c, entry, ef);
  if (rc) return rc;
  lane_req[0] = orc_visit_select(ix, c, entry, ef, k);
  g.step = 1;
  int stop = 0;
  if (early && orc_gpruning(&g, c, p)) { stop = 1; lane_req[0] = -1; }
  for (int w = 1; w < W; ++w) lane_req[w] = orc_select_no_compact(c, ef); /* 367-371 */

  int active[64];
  const int64_t max_iters = ix->num_points + 64;
  int64_t iters = 0;
  while (!stop) {
    int any = 0;
    for (int w = 0; w < W; ++w) { active[w] = lane_req[w] != -1; any |= active[w]; }
    if (!any) break;                              /* converged, 421-425 */
    if (++iters > max_iters) return -3;
    if (c->vfilter)
      for (int w = 0; w < W; ++w)
        if (active[w]) vset_add(c, (uint32_t)lane_req[w]);
    for (int w = 0; w < W; ++w) {
      if (!active[w]) continue;
      const int64_t node = lane_req[w];
      rc = orc_merge(ix, c, node, ef);
      if (rc) return rc;
      lane_req[w] = orc_visit_select(ix, c, node, ef, k);
      g.step++;
      if (early && orc_gpruning(&g, c, p)) { stop = 1; lane_req[w] = -1; }
    }
    if (stop) break;
    for (int w = 0; w < W; ++w)
      if (!active[w]) lane_req[w] = orc_select_no_compact(c, ef);
  }
  *out_steps = g.step;
  return 0;
}

int orc_search(const orc_index* ix, const float* queries, int64_t nq,
               const orc_params* p, int32_t* ids, float* dists,
               int32_t* found, int32_t* steps, int64_t* nbrs) {
  return orc_search_nav(ix, NULL, queries, nq, p, ids, dists, found, steps, nbrs);
}

int orc_search_nav(const orc_index* ix, const orc_nav* nav, const float* queries, int64_t nq,
                   const orc_params* p, int32_t* ids, float* dists,
                   int32_t* found, int32_t* steps, int64_t* nbrs) {
  if (p->topk <= 0 || p->ef_search <= 0 || p->pipe_width <= 0 || p->pipe_width > 64)
    return -10;
  int err = 0;
  const int64_t cap = p->ef_search + ix->max_degree;
  const int64_t cap2 = 2 * cap + 64;
#ifdef _OPENMP
  int nthreads = p->num_threads > 0 ? p->num_threads : omp_get_max_threads();
#pragma omp parallel num_threads(nthreads)
#endif
  {
    orc_ctx c;
    memset(&c, 0, sizeof(c));
    c.lid = (uint32_t*)malloc(sizeof(uint32_t) * cap2);
    c.ldist = (float*)malloc(sizeof(float) * cap2);
    c.tid = (uint32_t*)malloc(sizeof(uint32_t) * cap2);
    c.tdist = (float*)malloc(sizeof(float) * cap2);
    c.mid = (uint32_t*)malloc(sizeof(uint32_t) * cap2);
    c.mdist = (float*)malloc(sizeof(float) * cap2);
    c.mpos = (int*)malloc(sizeof(int) * cap2);
    c.rid = (int32_t*)malloc(sizeof(int32_t) * p->topk);
    c.rdist = (float*)malloc(sizeof(float) * p->topk);
    c.lut = (float*)malloc(sizeof(float) * (size_t)ix->num_chunks * ORC_PIVOTS);
    c.q2 = (float*)malloc(sizeof(float) * ix->dim);
    c.vcap = 1024;
    c.vset = (uint32_t*)calloc((size_t)c.vcap, sizeof(uint32_t));
    int32_t lane_req[64];
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 8)
#endif
    for (int64_t qi = 0; qi < nq; ++qi) {
      int st = 0;
      const int rc = orc_search_one(ix, nav, &c, queries + qi * ix->dim, p, lane_req, &st);
      if (rc) {
#ifdef _OPENMP
#pragma omp critical
#endif
        { if (!err) err = rc; }
      }
      for (int i = 0; i < p->topk; ++i) {
        ids[qi * p->topk + i] = c.rid[i];
        dists[qi * p->topk + i] = c.rdist[i];
      }
      if (found) found[qi] = c.fc;
      if (steps) steps[qi] = st;
      if (nbrs) nbrs[qi] = c.nbrs;
    }
    free(c.lid); free(c.ldist); free(c.tid); free(c.tdist); free(c.mid);
    free(c.mdist); free(c.mpos); free(c.rid); free(c.rdist); free(c.lut); free(c.q2); free(c.vset);
  }
  return err;
}

/* bin/common/recall.hpp:44-62: hits of each result row against the first
 * topk ground-truth ids of the same row; a repeated result id that is in the
 * set counts each time it appears. */
double orc_calc_recall(const int32_t* results, const int32_t* gt, int64_t nq,
                       int64_t gt_width, int32_t topk) {
  int64_t hits = 0;
  for (int64_t i = 0; i < nq; ++i) {
    const int32_t* g = gt + i * gt_width;
    for (int32_t j = 0; j < topk; ++j) {
      const int32_t r = results[i * topk + j];
      for (int32_t t = 0; t < topk; ++t) {
        if (g[t] == r) { ++hits; break; }
      }
    }
  }
  return (double)hits / (double)(nq * (int64_t)topk);
}
