/*
 * oracle.h -- CPU restatement of Quiver's query hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA
 * engine is compared against.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it; the product never links it.
 *
 * Every function restates one piece of the reference (ruc-system/quiver-ae),
 * cited as path:line inside that project:
 *   LUT build + q'' round trip  src/shared/index/pq_device.cuh:9-36
 *   ADC                         src/quiver/kernel_core/kernel_helpers.cuh:271-286
 *   neighbour sort + merge      src/quiver/kernel_core/kernel_helpers.cuh:293-356
 *   lower_bound key             src/shared/common/gpu_primitives.cuh:140-153
 *   exact L2 (warp tree order)  src/shared/common/gpu_primitives.cuh:26-44
 *   top-k insert                src/quiver/kernel_core/kernel_helpers.cuh:65-104
 *   compaction + select         src/quiver/kernel_core/kernel_helpers.cuh:437-474
 *   select without compaction   src/quiver/kernel_core/kernel_helpers.cuh:491-518
 *   hop loop, W lanes, gpruning src/quiver/kernel_core/kernel_q1.cuh:199-425,489-654
 *   page addressing             src/quiver/search.cu:240, kernel_helpers.cuh:257
 *   nav entry search            src/quiver/kernel_core/inkernel_nav.cuh:60-201,
 *                               used by kernel_q1.cuh:149-202; files nav_graph.cu:12-73
 *
 * Floating point: fp32 round-to-nearest, fused multiply-add exactly where the
 * reference writes `acc += d * d` (nvcc's default --fmad=true contracts it),
 * sums in the order the reference's loops and shuffle trees perform them.
 */
#ifndef QV_ORACLE_H
#define QV_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_UINT8 = 0, ORC_FLOAT = 1, ORC_INT8 = 2 };
enum { ORC_EXIT_NONE = 0, ORC_EXIT_GPRUNING = 2 };

typedef struct {
  int64_t num_points;     /* N */
  int64_t dim;
  int64_t max_degree;     /* R = max_m0 */
  int64_t node_size;      /* bytes per node record */
  int64_t data_size;      /* dim * elem */
  int64_t nodes_per_page;
  int64_t num_pages;
  int64_t medoid;
  int32_t data_type;      /* ORC_UINT8 / ORC_FLOAT / ORC_INT8 */
  int32_t num_chunks;     /* M */
  const uint8_t* pages;   /* num_pages * 4096 bytes: the index file without its header page */
  const uint8_t* codes;   /* N * M */
  const float* pivots_t;  /* dim * 256, pivots_t[i*256+j] = pivot j, coordinate i */
  const float* centroid;  /* dim */
  const int32_t* chunk_offsets; /* M + 1 */
} orc_index;

typedef struct {
  int32_t topk;
  int32_t ef_search;
  int32_t pipe_width;           /* W */
  int32_t early_exit_policy;    /* ORC_EXIT_NONE or ORC_EXIT_GPRUNING */
  int32_t gpruning_warmup_steps;
  int32_t gpruning_patience;
  int32_t num_threads;          /* OpenMP threads for orc_search; <=0 means all */
  int32_t visited_filter;       /* 1: a node scheduled for expansion never re-enters the list
                                   (a mode of this build, not reference behaviour); 0: reference */
  int32_t route_exact;          /* diagnostic, not reference behaviour: 1 scores each neighbour by
                                   its exact L2 (orc_exact_l2 of its record's vector) instead of
                                   ADC, so a walk of the same graph without PQ error can be compared
                                   with the reference walk; 0: reference (ADC) */
} orc_params;

/* A navigation graph (src/shared/index/nav_graph.cu:12-73).  Vectors have
 * the base set's data type and dim. */
typedef struct {
  const uint8_t* data;     /* num_node * dim elements */
  const int32_t* graph;    /* num_node * max_m, -1 padded */
  const int32_t* mapping;  /* num_node: nav id -> base id */
  int32_t num_node;
  int32_t max_m;           /* <= 32 */
  int32_t start;
} orc_nav;

/* The in-kernel entry search for one query on its ORIGINAL vector (before
 * the centroid round trip), inkernel_nav.cuh:60-201: returns the base id
 * of the best nav node, or a negative code on a malformed nav graph. */
int64_t orc_nav_entry(const orc_index* ix, const orc_nav* nav, const float* query);

/* LUT [M x 256] and q'' [dim] for one query (pq_device.cuh:9-36). */
void orc_build_lut(const orc_index* ix, const float* query, float* lut, float* q2);

/* Sequential fp32 sum of M LUT entries (kernel_helpers.cuh:280-285). */
float orc_adc(const float* lut, const uint8_t* code, int32_t M);

/* square_sum_32 on one vector of `dtype` (gpu_primitives.cuh:26-44). */
float orc_exact_l2(const float* q2, const void* vec, int64_t dim, int32_t dtype);

/* Full search.  ids/dists are [nq x topk], found/steps/nbrs are [nq]
 * (steps = expansions, nbrs = neighbours scored by ADC).  Any of
 * found/steps/nbrs may be NULL.  Returns 0 on success, negative on a
 * malformed index (neighbour id out of range, degree above R). */
int orc_search(const orc_index* ix, const float* queries, int64_t nq,
               const orc_params* p, int32_t* ids, float* dists,
               int32_t* found, int32_t* steps, int64_t* nbrs);

/* orc_search with each query's entry from the nav graph (nav may be NULL:
 * entry = medoid, as orc_search). */
int orc_search_nav(const orc_index* ix, const orc_nav* nav, const float* queries, int64_t nq,
                   const orc_params* p, int32_t* ids, float* dists,
                   int32_t* found, int32_t* steps, int64_t* nbrs);

/* Recall@k as bin/common/recall.hpp:44-62 defines it. */
double orc_calc_recall(const int32_t* results, const int32_t* gt,
                       int64_t nq, int64_t gt_width, int32_t topk);

#ifdef __cplusplus
}
#endif
#endif
