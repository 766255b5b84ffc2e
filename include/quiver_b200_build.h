/*
 * quiver_b200_build.h -- index construction and synthetic inputs.
 *
 * The reference builds its indexes with DiskANN's build_disk_index
 * (CMakeLists.txt:36-39, deps/DiskANN, an empty submodule here), so this
 * library has no entry point in the reference to mirror.  It produces the
 * same on-disk layout the reference reads: a Vamana graph (R, L, alpha) with
 * a medoid entry point, PQ pivots / centroid / chunk offsets / codes, plus
 * the seeded Gaussian-mixture inputs and exact ground truth that stand in
 * for the SIFT/DEEP datasets.
 *
 * Synthetic values come from a counter-based generator: every value is a
 * pure function of (seed, stream, index) computed with IEEE double add,
 * multiply, divide and sqrt only, so a CPU and a GPU produce the same bits.
 */
#ifndef QUIVER_B200_BUILD_H
#define QUIVER_B200_BUILD_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Streams of the generator. */
#define QVB_STREAM_BASE 0
#define QVB_STREAM_QUERY 1

/* Gaussian mixture: n_centers centres, point = centre + sigma * N(0,1) per
 * coordinate (12-uniform Irwin-Hall approximation).  dtype QV_UINT8 (0):
 * centres uniform in [0,255], values rounded half-to-even and clipped to
 * [0,255].  dtype QV_FLOAT (1): centres are normalised N(0,1) directions,
 * points normalised after the noise.  Rows [row0, row0 + n) of stream
 * `stream` are written to `out` (n x dim). */
int qvb_synth_mixture(uint64_t seed, int32_t stream, int64_t row0, int64_t n, int64_t dim,
                      int64_t n_centers, double sigma, int32_t dtype, void* out, int32_t nthreads);

/* Exact top-k by squared L2 (ties by lower id).  ids/dists are [nq x k]. */
int qvb_ground_truth(const void* base, int64_t n, const void* queries, int64_t nq, int64_t dim,
                     int32_t dtype, int32_t k, int32_t* ids, float* dists, int32_t nthreads);

/* Batched Vamana graph (the DiskANN algorithm: greedy search from the
 * medoid, robust prune with alpha, reverse edges with re-prune).  passes = 2
 * runs alpha = 1 then `alpha`.  graph is [n x R] (-1 padded), degree [n]. */
int qvb_vamana(const void* base, int64_t n, int64_t dim, int32_t dtype, int32_t R, int32_t L,
               float alpha, int32_t passes, uint64_t seed, int32_t nthreads, int32_t* graph,
               int32_t* degree, int64_t* medoid);

/* PQ with M chunks x 256 centroids, trained by Lloyd iterations on a
 * sample of the centred data.  pivots [256 x dim], centroid [dim],
 * chunk_offsets [M + 1]. */
int qvb_pq_train(const void* base, int64_t n, int64_t dim, int32_t dtype, int32_t M,
                 int64_t sample, int32_t iters, uint64_t seed, int32_t nthreads, float* pivots,
                 float* centroid, int32_t* chunk_offsets);

/* Nearest pivot per chunk (ties by lower pivot index).  codes [n x M]. */
int qvb_pq_encode(const void* base, int64_t n, int64_t dim, int32_t dtype, int32_t M,
                  const float* pivots, const float* centroid, const int32_t* chunk_offsets,
                  int32_t nthreads, uint8_t* codes);

const char* qvb_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
