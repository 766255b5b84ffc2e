/*
 * quiver_b200.h -- C ABI of the B200 engine for Quiver's query hot path.
 *
 * The engine replaces the reference's GPU search engine behind its own
 * callers.  Every entry point names the reference interface it stands in
 * for (path:line inside ruc-system/quiver-ae).  No C++ or torch types cross
 * this boundary: plain pointers, sizes and an int status.
 *
 * Status: every function returns QV_OK (0) or a positive QV_ERR_* code and
 * sets a thread-local message readable through qv_last_error().  Nothing
 * throws across the ABI (the reference throws std::runtime_error from
 * CHECK_CUDA, src/shared/common/cuda_utils.cuh:17-24, and calls
 * std::exit(1) on bad configuration, src/quiver/search.cu:402-407; here both
 * become return codes so the caller decides).
 *
 * Threading: an engine is thread-compatible -- one search at a time per
 * engine, like run_persistent_search, which is called from one host thread.
 * Different engines may be used from different threads.
 */
#ifndef QUIVER_B200_H
#define QUIVER_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QV_OK 0
#define QV_ERR_INVALID_ARG 1  /* a parameter is out of its documented range */
#define QV_ERR_IO 2           /* an index/query file cannot be read */
#define QV_ERR_BAD_INDEX 3    /* index files are inconsistent or malformed */
#define QV_ERR_CUDA 4         /* a CUDA runtime call failed */
#define QV_ERR_DEVICE 5       /* the search kernel reported a fault in the data */
#define QV_ERR_UNSUPPORTED 6  /* a configuration this build does not implement */
#define QV_ERR_OOM 7          /* device or pinned host memory exhausted */

/* Element type of base vectors (src/shared/common/data_type.hpp:5-9). */
#define QV_UINT8 0
#define QV_FLOAT 1
#define QV_INT8 2

/* Where the graph pages (vector + adjacency records) live. */
#define QV_PAGES_HBM 0   /* device memory of the engine's GPU */
#define QV_PAGES_HOST 1  /* pinned, mapped host DRAM read over PCIe */
#define QV_PAGES_STRIPED 2  /* page p on stripe p mod S of S devices' HBM (S = 1, 2, 4 or 8, see
                               qv_engine_opts.stripe_devices); the search GPU reads the other
                               stripes with peer loads over NVLink / NVSwitch */
#define QV_PAGES_SHARED 3   /* the same striping across S processes, one per GPU: this engine
                               holds stripe stripe_rank in its own GPU's HBM and reads the
                               others from the processes that hold them (CUDA IPC); see
                               qv_engine_stripe_handle / qv_engine_attach_stripes */

/* Early-exit policy (src/quiver/io_control.cuh:41-46; the CLI accepts only
 * "none" and "gpruning", bin/quiver_search.cu:48-54). */
#define QV_EXIT_NONE 0
#define QV_EXIT_GPRUNING 2

/* PQ lookup-table precision inside the search kernel. */
#define QV_LUT_FP32 0  /* fp32 table, bit-identical ADC sums to the reference */

typedef struct qv_engine qv_engine;

/* Index layout, the fields of shared::Layout (src/shared/common/layout.hpp:7-19)
 * as parse_diskann_metadata fills them (bin/common/metadata.hpp:15-72). */
typedef struct {
  int64_t num_points;
  int64_t dim;
  int64_t max_degree;      /* max_m0 = R */
  int64_t node_size;       /* max_node_len */
  int64_t data_size;       /* dim * element size */
  int64_t nodes_per_page;
  int64_t num_pages;
  int64_t medoid;          /* enter_point */
  int32_t data_type;       /* QV_UINT8 / QV_FLOAT / QV_INT8 */
  int32_t num_chunks;      /* PQ subspaces M */
} qv_index_info;

/* Engine creation from an index directory.  Replaces
 * bin_common::prepare_search_setup (bin/common/search_setup.hpp:73-119) +
 * shared::create_mem_loader_sync (src/shared/io/loader.hpp:43-45) +
 * shared::PQSearch::read_data / init_device (src/shared/index/pq_search.cu:62-177). */
typedef struct {
  const char* index_dir;          /* holds *_disk.index and *_pq_pivots.bin / *_pq_compressed.bin */
  int32_t data_type;              /* QV_UINT8 / QV_FLOAT / QV_INT8 */
  const char* memory_backend;     /* "heap" or "mmap": how the page file is read (memory_backend.hpp:7-20) */
  const char* memory_index_file;  /* NULL or "" -> the discovered *_disk.index */
  int32_t device;                 /* CUDA ordinal */
  int32_t page_store;             /* QV_PAGES_HBM / _HOST / _STRIPED / _SHARED (see above) */
  int32_t validate;               /* 1: check every adjacency list at load (degree <= R, ids < N) */
  int32_t num_stripes;            /* QV_PAGES_STRIPED: S, a power of two <= 8 */
  const int32_t* stripe_devices;  /* QV_PAGES_STRIPED: [S] CUDA ordinals (repeats allowed); every one
                                     must be `device` or peer-accessible from it */
  int32_t stripe_rank;            /* QV_PAGES_SHARED: the stripe this engine holds, in [0, S) */
} qv_engine_opts;

/* Index arrays already in host memory, in the on-disk layouts:
 * pages = the *_disk.index file without its 4 KB header page
 * (src/shared/io/mem_loader.cpp:28-44), pivots = [256 x dim] fp32 as stored
 * in *_pq_pivots.bin, chunk_offsets = [M+1], codes = [N x M]. */
typedef struct {
  qv_index_info info;
  const uint8_t* pages;
  const uint8_t* codes;
  const float* pivots;
  const float* centroid;
  const int32_t* chunk_offsets;
} qv_index_arrays;

/* Search knobs.  Mirrors the arguments of quiver::run_persistent_search
 * (src/quiver/search.cuh:45-66) and the CLI defaults
 * (bin/common/cli_shared.hpp:14-25, bin/quiver_search.cu:67-79, 202-205). */
typedef struct {
  int32_t topk;                   /* default 10 */
  int32_t ef_search;              /* default 30 */
  int32_t pipe_width;             /* W lanes per query, 1..16 (cli_validation.hpp:9) */
  int32_t queries_per_block;      /* query slots (warps) per CTA, 1..8; 0 = auto */
  int32_t num_blocks;             /* persistent CTAs; 0 = one wave on every SM */
  int32_t early_exit_policy;      /* QV_EXIT_NONE / QV_EXIT_GPRUNING */
  int32_t gpruning_warmup_steps;  /* default 10 */
  int32_t gpruning_patience;      /* default 8 */
  int32_t lut_mode;               /* QV_LUT_FP32 */
  int32_t skip_nav;               /* 1: start every query at the medoid even when the engine holds
                                     a nav graph (the CLI's --skip-nav, bin/quiver_search.cu:118-122,
                                     241-245); default 0 */
  int32_t visited_filter;         /* 1: a node a query has scheduled for expansion never re-enters its
                                     candidate list, so no node is expanded twice and the top-k holds
                                     no repeats.  A mode of this engine, not reference behaviour (the
                                     reference tracks visited nodes only inside the list); results then
                                     differ from the reference's.  Needs one query per CTA; default 0 */
} qv_search_opts;

typedef struct {
  double h2d_ms;                  /* queries host -> device */
  double kernel_ms;               /* search kernel (CUDA events) */
  double d2h_ms;                  /* results device -> host */
  double total_ms;                /* whole call */
  int64_t expansions;             /* node records fetched (sum of per-query steps) */
  int64_t neighbors_scored;       /* PQ codes gathered (sum of degrees) */
  int32_t grid;                   /* CTAs launched */
  int32_t slots_per_block;        /* query slots (warps) per CTA */
  int32_t smem_per_block;         /* dynamic shared memory bytes per CTA */
  int32_t blocks_per_sm;          /* resident CTAs per SM */
} qv_search_stats;

const char* qv_version(void);
const char* qv_last_error(void);
void qv_search_opts_default(qv_search_opts* opts);

/* Parse and check an index directory on the host only (no GPU): discovery,
 * disk-index header, PQ files, geometry.  The file-reading half of
 * prepare_search_setup (bin/common/search_setup.hpp:73-119). */
int qv_index_probe(const char* index_dir, int32_t data_type, qv_index_info* info);

int qv_engine_create(const qv_engine_opts* opts, qv_engine** out);
int qv_engine_create_from_arrays(const qv_index_arrays* arrays, int32_t device,
                                 int32_t page_store, qv_engine** out);
int qv_engine_info(const qv_engine* engine, qv_index_info* info);

/* Navigation graph for the per-query entry search.  qv_engine_create loads
 * one when the index directory (or its nav/ child) holds nav_index,
 * nav_index.data and map.txt, as prepare_search_setup does
 * (bin/common/search_setup.hpp:96-105 with NavGraph::init,
 * src/shared/index/nav_graph.cu:12-73); every search then starts from the
 * node the in-kernel entry search picks (src/quiver/kernel_core/
 * inkernel_nav.cuh:60-201, called at kernel_q1.cuh:149-202) instead of the
 * medoid, unless its options set skip_nav.
 *
 * qv_engine_set_nav replaces the engine's nav graph from host arrays:
 * data = num_node vectors of the index's type and dim, graph = [num_node x
 * max_m] nav ids padded with -1 (0 < max_m <= 32), mapping = nav id -> base
 * id, start = the nav id the search begins at.  num_node == 0 removes it.
 * qv_engine_nav_info reports num_node (0: none), max_m and start. */
int qv_engine_set_nav(qv_engine* engine, const void* data, const int32_t* graph, const int32_t* mapping,
                      int32_t num_node, int32_t max_m, int32_t start);
int qv_engine_nav_info(const qv_engine* engine, int32_t* num_node, int32_t* max_m, int32_t* start);
void qv_engine_destroy(qv_engine* engine);

/* Search with HOST buffers: queries [nq x dim] fp32 (the reference's float
 * query array, bin/common/data_io.hpp:73-108), ids/dists [nq x topk] and
 * found [nq].  Unfilled result slots hold id -1 and distance +inf, as the
 * reference initialises them (kernel_q1.cuh:192-195).  Replaces
 * quiver::run_persistent_search (src/quiver/search.cuh:45-66).  `found` and
 * `stats` may be NULL. */
int qv_search(qv_engine* engine, const float* queries, int64_t nq, int64_t dim,
              const qv_search_opts* opts, int32_t* ids, float* dists,
              int32_t* found, qv_search_stats* stats);

/* qv_search plus the per-query service latency: query_ms[i] is the time
 * (ms, GPU global timer) from the moment a query slot took query i to the
 * moment its results were written.  The reference's QueryLatency(ms) runs
 * from host admission to host completion (src/quiver/search.cu:1007-1044);
 * with every query admitted at the call, the host view of query i is its
 * queueing delay plus this service time. */
int qv_search_timed(qv_engine* engine, const float* queries, int64_t nq, int64_t dim,
                    const qv_search_opts* opts, int32_t* ids, float* dists,
                    int32_t* found, float* query_ms, qv_search_stats* stats);

/* Streaming admission: the reference's run_persistent_search host loop
 * (src/quiver/search.cu:820-1198).  One persistent launch serves all nq
 * queries while the host admits them in order: the first
 * min(workers + prefeed, nq) before the launch, then, whenever completions
 * allow (in flight <= workers + prefeed), the next range -- at least
 * admit_min_batch queries unless it is the last range or nothing is pending
 * -- copied host-to-device on a second stream and made visible to the kernel
 * in stream order after the copy.  A worker that binds a query not yet fed
 * waits for it (at most feed_timeout_ms; then the call fails with
 * QV_ERR_DEVICE).  Latency follows the reference's QueryLatency(ms): the i-th
 * completion the host observes is charged to the i-th admitted query, from
 * the host time its admission started (the call's start for the first range)
 * to the time the host saw the completion count pass i.  Results equal
 * qv_search's bit for bit.  The caller's query array is page-locked for the
 * call (cudaHostRegister), as the reference does. */
typedef struct qv_stream_opts {
  int32_t prefeed;          /* admitted queries beyond the workers; < 0: as many as workers */
  int32_t admit_min_batch;  /* smallest admission while one is pending (reference: 32) */
  int32_t feed_timeout_ms;  /* bound on a worker's wait for its query */
  int32_t admit_limit;      /* admit at most this many queries (< 0: all); a test hook for the timeout */
} qv_stream_opts;
void qv_stream_opts_default(qv_stream_opts* opts);

typedef struct qv_stream_stats {
  double search_ms;         /* call start (before the first copy) to the last completion seen */
  double qps;               /* nq / search_ms */
  double lat_avg_ms, lat_p50_ms, lat_p90_ms, lat_p99_ms, lat_p999_ms, lat_max_ms;
  int64_t admissions;       /* host-to-device ranges submitted, the first included */
  int32_t workers;          /* CTAs (block kernel) or warps (warp kernel) of the launch */
  int32_t max_inflight;     /* workers + prefeed */
  int64_t expansions;       /* nodes expanded, all queries */
} qv_stream_stats;

int qv_search_stream(qv_engine* engine, const float* queries, int64_t nq, int64_t dim,
                     const qv_search_opts* opts, const qv_stream_opts* sopts,
                     int32_t* ids, float* dists, int32_t* found,
                     float* query_latency_ms, qv_stream_stats* stats);

/* Same search with DEVICE buffers on the engine's GPU, enqueued on `stream`
 * (a cudaStream_t; NULL = the engine's own stream, cudaStreamLegacy for the
 * legacy default stream) without a host
 * synchronisation.  steps [nq] (expansions) and nbrs [nq] (PQ codes
 * gathered) may be NULL.  Errors the kernel detects in the data are
 * reported by qv_check_device_status after the stream has drained. */
int qv_search_device(qv_engine* engine, const float* d_queries, int64_t nq,
                     const qv_search_opts* opts, int32_t* d_ids, float* d_dists,
                     int32_t* d_found, int32_t* d_steps, int64_t* d_nbrs,
                     void* stream);
int qv_check_device_status(qv_engine* engine);

/* Search with HOST buffers that allocates no device memory -- for callers
 * that may not call cudaMalloc once their index is loaded (a plugin whose
 * host application owns the device allocator, a serving loop that cannot
 * take an allocation's implicit synchronisation or its failure under memory
 * pressure).  This entry point has no counterpart in the reference.  The
 * search kernel's scratch -- work counter, error words and device copies of
 * the queries and results -- is a file-scope device array of
 * QV_NOALLOC_SCRATCH_BYTES, so a call may carry at most
 *   256 + align256(nq*dim*4) + 2*align256(nq*topk*4) + align256(nq*4)
 * bytes (about 7,000 queries of 128 dims at top-10); larger batches are
 * rejected with QV_ERR_INVALID_ARG before anything is copied or launched.
 * qv_engine_create / qv_engine_create_from_arrays, with the engine's device
 * current, look up the array's device address and load the search kernels,
 * so the array is placed on the device when the index is loaded (under
 * CUDA's lazy module loading too) and stays until the process exits; the
 * address does not survive a reset of the device's context.  Calls share
 * the array and it keeps the last call's contents: calls that overlap on
 * the GPU race and must be serialised by the caller.  Results equal
 * qv_search's. */
#define QV_NOALLOC_SCRATCH_BYTES (4u << 20)
int qv_search_noalloc(qv_engine* engine, const float* queries, int64_t nq, int64_t dim,
                      const qv_search_opts* opts, int32_t* ids, float* dists,
                      int32_t* found);

/* Page store shared by S processes (QV_PAGES_SHARED).  After
 * qv_engine_create, every process exports its stripe with
 * qv_engine_stripe_handle (QV_STRIPE_HANDLE_BYTES of CUDA IPC handle), the
 * processes exchange the handles (any host channel: the caller's process
 * group), and each passes all S handles, in stripe order, to
 * qv_engine_attach_stripes; searches are refused until then.  A process must
 * keep its engine alive while others may still search (destroy the engines
 * after a barrier). */
#define QV_STRIPE_HANDLE_BYTES 64
int qv_engine_stripe_handle(qv_engine* engine, void* handle);
int qv_engine_attach_stripes(qv_engine* engine, const void* handles);

/* Launch geometry qv_search_device would use (grid, slots, smem). */
int qv_plan(qv_engine* engine, const qv_search_opts* opts, int64_t nq,
            qv_search_stats* plan);

/* Component kernels on device buffers, for testing the stages in isolation.
 *   qv_build_lut_device: LUT [nq x M x 256] and q'' [nq x dim]
 *       (PQSearchData::init_query, src/shared/index/pq_device.cuh:9-36)
 *   qv_adc_device: dist[i] = sum_j LUT[q(i)][j][code(id[i])[j]] for pairs
 *       (query_of[i], ids[i]) (kernel_helpers.cuh:271-286)
 *   qv_exact_l2_device: square_sum_32 of q''[query_of[i]] against node ids[i]
 *       read from the page store (gpu_primitives.cuh:26-44) */
int qv_build_lut_device(qv_engine* engine, const float* d_queries, int64_t nq,
                        float* d_lut, float* d_q2, void* stream);
int qv_adc_device(qv_engine* engine, const float* d_lut, const int32_t* d_query_of,
                  const int32_t* d_ids, int64_t n, float* d_out, void* stream);
int qv_exact_l2_device(qv_engine* engine, const float* d_q2, const int32_t* d_query_of,
                       const int32_t* d_ids, int64_t n, float* d_out, void* stream);

/* Batched ADC over raw device buffers, no engine needed: query q scores
 * n_per_query codes with its LUT d_luts[q] ([M x 256] fp32, the layout
 * PQSearchData::init_query writes, pq_device.cuh:9-36), summing the M lookups
 * in chunk order like the search's scoring loop (kernel_helpers.cuh:271-286):
 *   d_out[q * n + i] = sum_j d_luts[q][j][code(id)[j]]
 * where id = d_ids[q * n + i] (a gather), or, with d_ids NULL,
 * id = d_first[q] + i (a contiguous range).  An id outside [0, num_points)
 * gives NaN and is not read.  d_codes is [num_points x M] uint8; M must be a
 * multiple of 4 and d_luts 16-byte aligned.  kernel picks the implementation:
 * QV_ADC_PIPE (M == 32, 16-byte aligned codes; for thousands of codes per
 * query), QV_ADC_THREAD (any M), or QV_ADC_AUTO.  Asynchronous on stream. */
/* Vamana graph built on the GPU: the construction of qvb_vamana
 * (include/quiver_b200_build.h) step for step -- same medoid, insertion
 * order, batches, distances and prune -- so the graph, degrees and medoid
 * equal the host builder's.  base is a HOST array [n x dim] of dtype
 * (QV_UINT8, QV_INT8, QV_FLOAT); R <= 128, L <= 256, dim <= 1024; graph
 * [n x R] (-1 padded), degree [n] and medoid are host outputs. */
int qv_vamana_gpu(const void* base, int64_t n, int64_t dim, int32_t dtype, int32_t R,
                  int32_t L, float alpha, int32_t passes, uint64_t seed, int32_t device,
                  int32_t* graph, int32_t* degree, int64_t* medoid);

/* The seeded Gaussian-mixture generator of qvb_synth_mixture and the PQ
 * encoder of qvb_pq_encode (include/quiver_b200_build.h) on the GPU, bit for
 * bit.  Host buffers in and out; `device` is the CUDA device used. */
int qv_synth_mixture_gpu(uint64_t seed, int32_t stream, int64_t row0, int64_t n, int64_t dim,
                         int64_t n_centers, double sigma, int32_t dtype, void* out, int32_t device);
int qv_pq_encode_gpu(const void* base, int64_t n, int64_t dim, int32_t dtype, int32_t M,
                     const float* pivots, const float* centroid, const int32_t* chunk_offsets,
                     int32_t device, uint8_t* codes);

#define QV_ADC_AUTO 0
#define QV_ADC_THREAD 1
#define QV_ADC_PIPE 2
int qv_adc_batch(const uint8_t* d_codes, int64_t num_points, int32_t M,
                 const float* d_luts, int64_t nq, const int32_t* d_ids,
                 const int64_t* d_first, int64_t n_per_query, float* d_out,
                 int32_t kernel, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* QUIVER_B200_H */
