// engine.cu -- host runtime and C ABI of the B200 search engine.
//
// Owns the device copies of one index (page store, PQ codes, transposed
// pivots, centroid, chunk offsets), plans the launch geometry of the
// persistent search kernel from its shared-memory footprint, and runs
// searches with host or device buffers.  Replaces the reference's
// quiver::run_persistent_search (src/quiver/search.cu:357-1361): there is
// no CPU poll thread and no host-mapped IO protocol, because node records
// are read by the kernel directly from HBM (or from mapped host DRAM).
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <memory>
#include <numeric>
#include <string>
#include <vector>

#include "index_io.h"
#include "quiver_b200.h"
#include "plan.h"

namespace {

thread_local std::string g_last_error;

struct CudaError : qv::IoError {
  explicit CudaError(const std::string& m) : qv::IoError(QV_ERR_CUDA, m) {}
};

void check_cuda(cudaError_t e, const char* what, int line) {
  if (e == cudaSuccess) return;
  const int code = (e == cudaErrorMemoryAllocation) ? QV_ERR_OOM : QV_ERR_CUDA;
  throw qv::IoError(code, std::string(what) + " failed: " + cudaGetErrorString(e) +
                              " (engine.cu:" + std::to_string(line) + ")");
}
#define CK(call) check_cuda((call), #call, __LINE__)

template <class F>
int guarded(F&& f) {
  try {
    f();
    return QV_OK;
  } catch (const qv::IoError& e) {
    g_last_error = e.what();
    return e.code;
  } catch (const std::bad_alloc&) {
    g_last_error = "host allocation failed";
    return QV_ERR_OOM;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return QV_ERR_INVALID_ARG;
  }
}

[[noreturn]] void fail(int code, const std::string& m) { throw qv::IoError(code, m); }

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

}  // namespace

struct qv_engine {
  int device = 0;
  qv::Layout L;
  int32_t M = 0;
  bool pages_host = false;
  uint8_t* d_pages = nullptr;   // what the kernel dereferences
  // striped page store: stripe s on stripe_dev[s]; stripe_table lives on `device`
  std::vector<int> stripe_dev;
  std::vector<uint8_t*> stripe_ptr;
  uint8_t** d_stripe_table = nullptr;
  int stripe_shift = 0;
  // QV_PAGES_SHARED: this process holds stripe stripe_rank; the others are
  // other processes' allocations opened by IPC (closed, not freed, here)
  bool shared = false, attached = false;
  int stripe_rank = -1;
  std::vector<void*> imported;
  uint8_t* h_pages = nullptr;   // pinned mapped host allocation (host store)
  uint8_t* d_codes = nullptr;
  float* d_pivots_t = nullptr;
  float* d_centroid = nullptr;
  int32_t* d_chunk_off = nullptr;
  int32_t* d_scratch = nullptr;  // [0] work counter, [1..4] error info
  // device address of g_qv_noalloc_scratch on `device`, resolved at creation
  unsigned char* d_noalloc = nullptr;
  int num_sms = 0;
  int max_smem_optin = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
  // staging for host-buffer searches
  float* d_q = nullptr;
  int32_t* d_ids = nullptr;
  float* d_dists = nullptr;
  int32_t* d_found = nullptr;
  int32_t* d_steps = nullptr;
  int64_t* d_nbrs = nullptr;
  int64_t* d_time = nullptr;
  int64_t cap_q = 0, cap_r = 0, cap_n = 0;
  // nav graph (entry search); nav_num_node == 0: none
  uint8_t* d_nav_data = nullptr;
  int32_t* d_nav_graph = nullptr;
  int32_t* d_nav_map = nullptr;
  int32_t nav_num_node = 0, nav_max_m = 0, nav_start = 0;
  // visited-filter mode: per-CTA tables, tags never reused until the counter wraps
  unsigned long long* d_visited = nullptr;
  size_t visited_bytes = 0;
  uint32_t visited_next = 1;
  // streaming admission: copy stream, per-worker completion counts (pinned,
  // mapped), feed values the copy stream writes to the device (pinned ring),
  // one event per ring slot
  cudaStream_t h2d_stream = nullptr;
  uint32_t* h_done = nullptr;
  int32_t* h_feed = nullptr;
  std::vector<cudaEvent_t> feed_ev;
  int64_t cap_done = 0;

  ~qv_engine() {
    if (device >= 0) cudaSetDevice(device);
    for (auto* p : {(void*)d_codes, (void*)d_pivots_t, (void*)d_centroid, (void*)d_chunk_off,
                    (void*)d_scratch, (void*)d_q, (void*)d_ids, (void*)d_dists, (void*)d_found,
                    (void*)d_steps, (void*)d_nbrs, (void*)d_time, (void*)d_nav_data, (void*)d_nav_graph,
                    (void*)d_nav_map, (void*)d_visited})
      if (p) cudaFree(p);
    if (pages_host) {
      if (h_pages) cudaFreeHost(h_pages);
    } else if (d_pages && stripe_ptr.empty()) {  // with stripes, d_pages is stripe 0
      cudaFree(d_pages);
    }
    for (void* p : imported) cudaIpcCloseMemHandle(p);
    for (size_t s = 0; s < stripe_ptr.size(); ++s) {
      if (!stripe_ptr[s] || (shared && static_cast<int>(s) != stripe_rank)) continue;
      cudaSetDevice(stripe_dev[s]);
      cudaFree(stripe_ptr[s]);
    }
    if (device >= 0) cudaSetDevice(device);
    if (d_stripe_table) cudaFree(d_stripe_table);
    for (auto& e : ev)
      if (e) cudaEventDestroy(e);
    for (auto& e : feed_ev)
      if (e) cudaEventDestroy(e);
    if (h_done) cudaFreeHost(h_done);
    if (h_feed) cudaFreeHost(h_feed);
    if (h2d_stream) cudaStreamDestroy(h2d_stream);
    if (stream) cudaStreamDestroy(stream);
  }
};

namespace {

// ------------------------------------------------------------ planning --

using qv::Plan;

void validate_opts(const qv_engine* e, const qv_search_opts& o) {
  if (e->shared && !e->attached)
    fail(QV_ERR_INVALID_ARG, "a shared page store needs every process's stripe (qv_engine_attach_stripes) first");
  if (o.topk < 1 || o.topk > 1024) fail(QV_ERR_INVALID_ARG, "topk must be in [1, 1024]");
  if (o.ef_search < 1 || o.ef_search > 4096) fail(QV_ERR_INVALID_ARG, "ef_search must be in [1, 4096]");
  if (o.pipe_width < 1 || o.pipe_width > qvk::kMaxPipeWidth)
    fail(QV_ERR_INVALID_ARG, "--pipe-width must be in [1, 16]");
  if (o.queries_per_block < 0 || o.queries_per_block > 8)
    fail(QV_ERR_INVALID_ARG, "--queries-per-block must be in [1, 8]");
  if (o.num_blocks < 0) fail(QV_ERR_INVALID_ARG, "--num-blocks must be positive");
  if (o.early_exit_policy != QV_EXIT_NONE && o.early_exit_policy != QV_EXIT_GPRUNING)
    fail(QV_ERR_INVALID_ARG, "early-exit policy must be none or gpruning");
  if (o.lut_mode != QV_LUT_FP32) fail(QV_ERR_UNSUPPORTED, "only the fp32 LUT mode is built");
  if (o.skip_nav != 0 && o.skip_nav != 1) fail(QV_ERR_INVALID_ARG, "skip_nav must be 0 or 1");
  if (o.visited_filter != 0 && o.visited_filter != 1) fail(QV_ERR_INVALID_ARG, "visited_filter must be 0 or 1");
  (void)e;
}

// Kernel specialisation for this index: neighbours per lane and PQ width.
void set_kernel_shape(const qv_engine* e, Plan& pl) {
  pl.smax = e->L.max_degree <= 64 ? 2 : 4;
  pl.mc = e->M == 32 ? 32 : 0;
}

// Binds pl.fn / pl.fn_stream for the index's element type, pl.block, pl.mc and pl.smax.
void bind_kernels(const qv_engine* e, Plan& pl) {
  switch (e->L.data_type) {
    case QV_UINT8: qv::bind_search_u8(pl); break;
    case QV_INT8: qv::bind_search_i8(pl); break;
    default: qv::bind_search_f32(pl); break;
  }
}

Plan make_plan(qv_engine* e, const qv_search_opts& o, int64_t nq) {
  validate_opts(e, o);
  Plan pl;
  const auto& L = e->L;
  set_kernel_shape(e, pl);
  pl.long_lists = o.ef_search > qvk::kBlock * qvk::kFastEntries;
  // --queries-per-block 0/1: one query per 128-thread CTA (the block kernel);
  // Q >= 2: Q one-warp query slots per CTA (the warp kernel).  Both give
  // identical results.
  pl.block = o.queries_per_block <= 1;
  if (o.visited_filter && !pl.block)
    fail(QV_ERR_UNSUPPORTED, "the visited-filter mode runs with one query per CTA (queries_per_block 0 or 1)");
  const int rp = 32 * pl.smax;
  const int G = pl.block ? qvk::kBlock / rp : (pl.smax <= 2 ? 4 : 2);
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    off = round_up(off, 16);
    const int64_t r = off;
    off += bytes;
    return static_cast<int32_t>(r);
  };
  auto& y = pl.lay;
  y.off_lut = take(int64_t(e->M) * qvk::kPivots * 4);
  y.off_q2 = take(L.dim * 4);
  y.off_lid = take(int64_t(o.ef_search) * 4);
  y.off_ldist = take(int64_t(o.ef_search) * 4);
  if (pl.block) {
    y.off_spos = take(qvk::kBlock * 4);   // new pairs by thread slot (distances)
    y.off_sflag = take(qvk::kBlock * 4);  //   (ids)
    y.off_r0 = take(qvk::kBlock * 4);     //   (insertion points)
    y.off_S = take(qvk::kBlock * 4);
    y.off_fsrc = take(qvk::kBlock * 4);
    y.off_misc = take(qvk::kMiscSlots * 4);
    y.off_sort = take(2 * 3 * qvk::kBlock * 4);
  } else {
    y.off_nid = take(rp * 4);
    y.off_ndist = take(rp * 4);
    y.off_mid = take((int64_t(o.ef_search) + rp) * 4);
    y.off_mdist = take((int64_t(o.ef_search) + rp) * 4);
  }
  y.off_rid = take(int64_t(o.topk) * 4);
  y.off_rdist = take(int64_t(o.topk) * 4);
  y.rec_stride = static_cast<int32_t>(round_up(L.data_size, 16));
  if (!pl.block) y.off_rec = take(int64_t(G) * y.rec_stride);  // the block kernel reads vectors in place
  y.off_lane = take(qvk::kMaxPipeWidth * 4);
  y.bytes = static_cast<int32_t>(round_up(off, 16));
  if (y.bytes > e->max_smem_optin)
    fail(QV_ERR_UNSUPPORTED, "one query slot needs " + std::to_string(y.bytes) +
                                 " B of shared memory, above the per-CTA limit");

  bind_kernels(e, pl);
  CK(cudaFuncSetAttribute(pl.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, e->max_smem_optin));
  CK(cudaFuncSetAttribute(pl.fn_stream, cudaFuncAttributeMaxDynamicSharedMemorySize, e->max_smem_optin));

  const int threads_per_slot = pl.block ? qvk::kBlock : 32;
  auto occupancy = [&](int slots) {
    int occ = 0;
    const int smem = slots * y.bytes;
    if (smem > e->max_smem_optin) return 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, pl.fn, slots * threads_per_slot, smem));
    return occ;
  };
  if (pl.block) {
    pl.slots = 1;
    pl.blocks_per_sm = occupancy(1);
    if (pl.blocks_per_sm == 0) fail(QV_ERR_UNSUPPORTED, "a query slot does not fit in shared memory");
  } else {
    pl.slots = o.queries_per_block;
    pl.blocks_per_sm = occupancy(pl.slots);
    if (pl.blocks_per_sm == 0)
      fail(QV_ERR_UNSUPPORTED, std::to_string(pl.slots) + " query slots of " + std::to_string(y.bytes) +
                                   " B do not fit in one CTA");
  }
  pl.smem = pl.slots * y.bytes;
  const int64_t wave = int64_t(pl.blocks_per_sm) * e->num_sms;
  int64_t grid = o.num_blocks > 0 ? std::min<int64_t>(o.num_blocks, wave) : wave;
  const int64_t needed = (nq + pl.slots - 1) / pl.slots;
  grid = std::max<int64_t>(1, std::min(grid, needed));
  pl.grid = static_cast<int>(grid);
  pl.threads = pl.slots * threads_per_slot;
  return pl;
}

qvk::SearchParams make_params(const qv_engine* e, const Plan& pl, const qv_search_opts& o,
                              const float* d_q, int64_t nq, int32_t* ids, float* dists,
                              int32_t* found, int32_t* steps, int64_t* nbrs, int64_t* times = nullptr) {
  qvk::SearchParams p{};
  p.pages = e->d_pages;
  p.stripe_table = reinterpret_cast<const unsigned long long*>(e->d_stripe_table);
  p.stripe_shift = e->stripe_shift;
  p.codes = e->d_codes;
  p.pivots_t = e->d_pivots_t;
  p.centroid = e->d_centroid;
  p.chunk_off = e->d_chunk_off;
  p.queries = d_q;
  p.out_ids = ids;
  p.out_dists = dists;
  p.out_found = found;
  p.out_steps = steps;
  p.out_nbrs = nbrs;
  p.out_time = times;
  p.work_counter = e->d_scratch;
  p.error_info = e->d_scratch + 1;
  p.num_points = e->L.num_points;
  p.nq = nq;
  // Each pipe iteration expands at least one unvisited node and a node is
  // expanded at most twice (the entry, once from the boot and once from the
  // list), so N + W + 8 iterations bound every legal walk.
  p.max_iters = e->L.num_points + o.pipe_width + 8;
  p.dim = static_cast<int32_t>(e->L.dim);
  p.M = e->M;
  p.R = static_cast<int32_t>(e->L.max_degree);
  p.node_size = static_cast<int32_t>(e->L.node_size);
  p.data_words = static_cast<int32_t>(e->L.data_size / 4);
  p.npp = static_cast<int32_t>(e->L.nodes_per_page);
  p.ef = o.ef_search;
  p.k = o.topk;
  p.W = o.pipe_width;
  p.early_policy = o.early_exit_policy;
  p.gp_warmup = o.gpruning_warmup_steps;
  p.gp_patience = o.gpruning_patience;
  p.medoid = static_cast<int32_t>(e->L.medoid);
  if (e->nav_num_node > 0 && !o.skip_nav) {
    p.nav_data = e->d_nav_data;
    p.nav_graph = e->d_nav_graph;
    p.nav_mapping = e->d_nav_map;
    p.nav_num_node = e->nav_num_node;
    p.nav_max_m = e->nav_max_m;
    p.nav_start = e->nav_start;
  }
  p.lay = pl.lay;
  return p;
}

// Visited-filter mode: one table of `cap` entries per persistent CTA; query
// qid of this search gets tag visited_next + qid (tags start at 1, 0 means
// empty), so tables are zeroed only when allocated or when the counter wraps.
void prepare_visited(qv_engine* e, const Plan& pl, const qv_search_opts& o, int64_t nq, qvk::SearchParams& p,
                     cudaStream_t st) {
  if (!o.visited_filter) return;
  int cap = 1024;
  while (cap < 8 * o.ef_search) cap <<= 1;
  const size_t need = static_cast<size_t>(pl.grid) * cap * sizeof(unsigned long long);
  if (need > e->visited_bytes) {
    if (e->d_visited) CK(cudaFree(e->d_visited));
    e->d_visited = nullptr;
    e->visited_bytes = 0;
    CK(cudaMalloc(&e->d_visited, need));
    e->visited_bytes = need;
    CK(cudaMemsetAsync(e->d_visited, 0, need, st));
    e->visited_next = 1;
  }
  if (static_cast<uint64_t>(e->visited_next) + static_cast<uint64_t>(nq) + 1 >= (1ull << 32)) {
    CK(cudaMemsetAsync(e->d_visited, 0, e->visited_bytes, st));
    e->visited_next = 1;
  }
  p.visited = e->d_visited;
  p.visited_cap = cap;
  p.visited_tag0 = e->visited_next;
  e->visited_next += static_cast<uint32_t>(nq);
}

void enqueue_search(qv_engine* e, const Plan& pl, const qvk::SearchParams& p, cudaStream_t st) {
  CK(cudaMemsetAsync(e->d_scratch, 0, 8 * sizeof(int32_t), st));
  pl.launch(p, pl.grid, pl.threads, pl.smem, st);
  CK(cudaGetLastError());
}

// Throws QV_ERR_DEVICE describing the search kernel's error words
// {code, query, node or step, spare} unless code is kErrNone.
void raise_device_error(const int32_t info[4]) {
  if (info[0] == qvk::kErrNone) return;
  const char* what = info[0] == qvk::kErrNeighborRange ? "a neighbour id >= num_points"
                   : info[0] == qvk::kErrDegree        ? "a stored degree above R"
                   : info[0] == qvk::kErrHopCap        ? "a walk beyond its iteration bound"
                   : info[0] == qvk::kErrNav           ? "a nav graph id out of range or a nav walk beyond its bound"
                   : info[0] == qvk::kErrVisited       ? "a full visited-filter table"
                   : info[0] == qvk::kErrFeed          ? "a query not admitted within the feed timeout"
                                                       : "an unknown device error";
  fail(QV_ERR_DEVICE, std::string("search kernel found ") + what + " (query " +
                          std::to_string(info[1]) + ", node/step " + std::to_string(info[2]) + ")");
}

void read_device_status(qv_engine* e) {
  int32_t info[4];
  CK(cudaMemcpy(info, e->d_scratch + 1, sizeof(info), cudaMemcpyDeviceToHost));
  raise_device_error(info);
}

}  // namespace

// ------------------------------------------------- no-alloc scratch array --
//
// qv_search_noalloc serves callers that may not allocate device memory on
// their search path: plugins whose host application owns the device
// allocator and forbids them from calling cudaMalloc, and serving loops
// where a cudaMalloc (with its implicit device synchronisation) or a failed
// allocation under memory pressure is not acceptable once the index is
// loaded.  The search kernel's scratch -- its work counter, its error words
// and the device copies of the queries and results -- lives in the
// file-scope array below instead of engine-owned allocations.  The array
// is 4 MiB.  Engine creation (qv_engine_create / _from_arrays), with the
// engine's device current, looks up the array's device address and loads
// the search kernels a no-alloc call can launch, so that under CUDA's lazy
// module loading the array and the kernels' code are placed on the device
// while the index is loaded, not by the first no-alloc call; from then on
// the device holds the array until the process exits.  The address is kept
// in the engine: an engine does not survive a reset of its device's
// context (cudaDeviceReset), and neither does the address.  All calls share
// the array and it keeps the last call's contents; the work counter and
// error words are cleared at the start of every call.  Calls that overlap
// on the GPU (two host threads, or two engines on one device) race on the
// array and must be serialised by the caller.
static __device__ __align__(256) unsigned char g_qv_noalloc_scratch[QV_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr size_t kNoallocHeader = 256;  // work counter + 4 error words, padded

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// With e->device current: resolve g_qv_noalloc_scratch's device address and
// load every search kernel qv_search_noalloc may launch for this index.
void prepare_noalloc(qv_engine* e) {
  void* ptr = nullptr;
  const cudaError_t rc = cudaGetSymbolAddress(&ptr, g_qv_noalloc_scratch);
  if (rc != cudaSuccess)
    fail(QV_ERR_CUDA, std::string("cudaGetSymbolAddress(g_qv_noalloc_scratch) failed: ") + cudaGetErrorString(rc));
  e->d_noalloc = static_cast<unsigned char*>(ptr);
  Plan pl;
  set_kernel_shape(e, pl);
  for (const int variant : {0, 1, 2}) {  // block kernel for short and long lists, warp kernel
    pl.block = variant < 2;
    pl.long_lists = variant == 1;
    bind_kernels(e, pl);
    cudaFuncAttributes attr;
    CK(cudaFuncGetAttributes(&attr, pl.fn));
  }
}

// ------------------------------------------------------ engine set-up --

void init_device_side(qv_engine* e, int device) {
  e->device = device;
  int count = 0;
  CK(cudaGetDeviceCount(&count));
  if (device < 0 || device >= count) fail(QV_ERR_INVALID_ARG, "CUDA device ordinal out of range");
  CK(cudaSetDevice(device));
  CK(cudaDeviceGetAttribute(&e->num_sms, cudaDevAttrMultiProcessorCount, device));
  CK(cudaDeviceGetAttribute(&e->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  CK(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
  for (auto& ev : e->ev) CK(cudaEventCreate(&ev));
  CK(cudaMalloc(&e->d_scratch, 8 * sizeof(int32_t)));
  CK(cudaMemset(e->d_scratch, 0, 8 * sizeof(int32_t)));
  prepare_noalloc(e);
}

void upload_pq(qv_engine* e, const float* pivots, const float* centroid, const int32_t* chunk_off,
               const uint8_t* codes) {
  const int64_t dim = e->L.dim;
  std::vector<float> pt(static_cast<size_t>(dim) * qvk::kPivots);
  for (int j = 0; j < qvk::kPivots; ++j)
    for (int64_t i = 0; i < dim; ++i) pt[i * qvk::kPivots + j] = pivots[j * dim + i];
  CK(cudaMalloc(&e->d_pivots_t, pt.size() * 4));
  CK(cudaMemcpy(e->d_pivots_t, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMalloc(&e->d_centroid, dim * 4));
  CK(cudaMemcpy(e->d_centroid, centroid, dim * 4, cudaMemcpyHostToDevice));
  CK(cudaMalloc(&e->d_chunk_off, (e->M + 1) * 4));
  CK(cudaMemcpy(e->d_chunk_off, chunk_off, (e->M + 1) * 4, cudaMemcpyHostToDevice));
  const size_t cb = static_cast<size_t>(e->L.num_points) * e->M;
  // +16 so 16-byte code loads of the last point stay inside the allocation
  CK(cudaMalloc(&e->d_codes, cb + 16));
  CK(cudaMemcpy(e->d_codes, codes, cb, cudaMemcpyHostToDevice));
}

// NavGraph::init's device copies (nav_graph.cu:70-72); replaces any earlier graph.
void upload_nav(qv_engine* e, const qv::NavHost& nav) {
  qv::check_nav(nav, e->L.dim, e->L.num_points);
  for (void* p : {(void*)e->d_nav_data, (void*)e->d_nav_graph, (void*)e->d_nav_map})
    if (p) CK(cudaFree(p));
  e->d_nav_data = nullptr;
  e->d_nav_graph = nullptr;
  e->d_nav_map = nullptr;
  e->nav_num_node = 0;
  CK(cudaMalloc(&e->d_nav_data, nav.data.size()));
  CK(cudaMemcpy(e->d_nav_data, nav.data.data(), nav.data.size(), cudaMemcpyHostToDevice));
  CK(cudaMalloc(&e->d_nav_graph, nav.graph.size() * 4));
  CK(cudaMemcpy(e->d_nav_graph, nav.graph.data(), nav.graph.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMalloc(&e->d_nav_map, nav.mapping.size() * 4));
  CK(cudaMemcpy(e->d_nav_map, nav.mapping.data(), nav.mapping.size() * 4, cudaMemcpyHostToDevice));
  e->nav_num_node = nav.num_node;
  e->nav_max_m = nav.max_m;
  e->nav_start = nav.start;
}

// The page store into HBM without holding it in host memory: 64 MB pieces are
// read into two pinned staging buffers in turn and copied while the next is
// read, so a 41 GB store needs 128 MB of host memory, not 41 GB.
void upload_pages_staged(qv_engine* e, const std::string& file, const std::string& backend) {
  constexpr int64_t kChunkPages = 16384;
  uint8_t* stage[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  auto release = [&] {
    for (int b = 0; b < 2; ++b) {
      if (done[b]) cudaEventDestroy(done[b]);
      if (stage[b]) cudaFreeHost(stage[b]);
    }
  };
  try {
    for (int b = 0; b < 2; ++b) {
      CK(cudaHostAlloc(reinterpret_cast<void**>(&stage[b]), kChunkPages * qv::kPage, cudaHostAllocDefault));
      CK(cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming));
    }
    const int64_t pages = e->L.num_pages;
    int b = 0;
    for (int64_t first = 0; first < pages; first += kChunkPages, b ^= 1) {
      const int64_t n = std::min<int64_t>(kChunkPages, pages - first);
      CK(cudaEventSynchronize(done[b]));  // the copy that last used this buffer has finished
      qv::read_page_range(file, pages, backend, first, n, stage[b]);
      CK(cudaMemcpyAsync(e->d_pages + first * qv::kPage, stage[b], static_cast<size_t>(n) * qv::kPage,
                         cudaMemcpyHostToDevice, e->stream));
      CK(cudaEventRecord(done[b], e->stream));
    }
    CK(cudaStreamSynchronize(e->stream));
  } catch (...) {
    cudaStreamSynchronize(e->stream);
    release();
    throw;
  }
  release();
}

void alloc_pages(qv_engine* e, int32_t page_store) {
  const size_t bytes = static_cast<size_t>(e->L.num_pages) * qv::kPage;
  if (page_store == QV_PAGES_HOST) {
    e->pages_host = true;
    CK(cudaHostAlloc(&e->h_pages, bytes, cudaHostAllocMapped | cudaHostAllocPortable));
    CK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&e->d_pages), e->h_pages, 0));
  } else if (page_store == QV_PAGES_HBM) {
    CK(cudaMalloc(&e->d_pages, bytes));
  } else if (page_store != QV_PAGES_STRIPED && page_store != QV_PAGES_SHARED) {
    fail(QV_ERR_INVALID_ARG, "page_store must be QV_PAGES_HBM, QV_PAGES_HOST, QV_PAGES_STRIPED or QV_PAGES_SHARED");
  }
}

// Striped page store: page p goes to stripe p & (S - 1) at local page
// p >> log2(S); stripes on other devices are read by peer loads, so peer
// access from the search device is enabled for each of them.
void stripe_pages(qv_engine* e, const uint8_t* host_pages, int32_t num_stripes, const int32_t* devices) {
  if (num_stripes < 1 || num_stripes > 8 || (num_stripes & (num_stripes - 1)) != 0 || !devices)
    fail(QV_ERR_INVALID_ARG, "num_stripes must be 1, 2, 4 or 8, with stripe_devices");
  int count = 0;
  CK(cudaGetDeviceCount(&count));
  for (int s = 0; s < num_stripes; ++s)
    if (devices[s] < 0 || devices[s] >= count) fail(QV_ERR_INVALID_ARG, "stripe device ordinal out of range");
  for (int s = 0; s < num_stripes; ++s) {
    const int d = devices[s];
    if (d == e->device) continue;
    int can = 0;
    CK(cudaDeviceCanAccessPeer(&can, e->device, d));
    if (!can)
      fail(QV_ERR_UNSUPPORTED, "device " + std::to_string(d) + " is not peer-accessible from device " +
                                   std::to_string(e->device));
    const cudaError_t pe = cudaDeviceEnablePeerAccess(d, 0);  // current device: e->device
    if (pe == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
    else if (pe != cudaSuccess) CK(pe);
  }
  int shift = 0;
  while ((1 << shift) < num_stripes) ++shift;
  const int64_t P = e->L.num_pages;
  e->stripe_dev.assign(devices, devices + num_stripes);
  e->stripe_ptr.assign(num_stripes, nullptr);
  std::vector<uint8_t> gather;
  for (int s = 0; s < num_stripes; ++s) {
    const int64_t n = P > s ? (P - s + num_stripes - 1) / num_stripes : 0;
    gather.resize(static_cast<size_t>(std::max<int64_t>(n, 1)) * qv::kPage);
    for (int64_t j = 0; j < n; ++j)
      std::memcpy(gather.data() + static_cast<size_t>(j) * qv::kPage,
                  host_pages + static_cast<size_t>(j * num_stripes + s) * qv::kPage, qv::kPage);
    CK(cudaSetDevice(e->stripe_dev[s]));
    CK(cudaMalloc(&e->stripe_ptr[s], gather.size()));
    CK(cudaMemcpy(e->stripe_ptr[s], gather.data(), static_cast<size_t>(n) * qv::kPage, cudaMemcpyHostToDevice));
  }
  CK(cudaSetDevice(e->device));
  CK(cudaMalloc(&e->d_stripe_table, sizeof(uint8_t*) * num_stripes));
  CK(cudaMemcpy(e->d_stripe_table, e->stripe_ptr.data(), sizeof(uint8_t*) * num_stripes, cudaMemcpyHostToDevice));
  e->stripe_shift = shift;
  e->d_pages = e->stripe_ptr[0];  // stripe 0 (the whole store when S == 1)
}

// QV_PAGES_SHARED: this process's stripe only (pages p = rank, rank + S, ...),
// read straight from the page file; the table is built at attach time.
void load_own_stripe(qv_engine* e, const std::string& page_file, int32_t num_stripes, int32_t rank) {
  if (num_stripes < 1 || num_stripes > 8 || (num_stripes & (num_stripes - 1)) != 0)
    fail(QV_ERR_INVALID_ARG, "num_stripes must be 1, 2, 4 or 8");
  if (rank < 0 || rank >= num_stripes) fail(QV_ERR_INVALID_ARG, "stripe_rank must be in [0, num_stripes)");
  const int64_t P = e->L.num_pages;
  const int64_t n = P > rank ? (P - rank + num_stripes - 1) / num_stripes : 0;
  std::vector<uint8_t> host(static_cast<size_t>(std::max<int64_t>(n, 1)) * qv::kPage);
  qv::read_stripe_pages(page_file, P, num_stripes, rank, host.data());
  int shift = 0;
  while ((1 << shift) < num_stripes) ++shift;
  e->shared = true;
  e->stripe_rank = rank;
  e->stripe_shift = shift;
  e->stripe_dev.assign(num_stripes, e->device);
  e->stripe_ptr.assign(num_stripes, nullptr);
  CK(cudaMalloc(&e->stripe_ptr[rank], host.size()));
  CK(cudaMemcpy(e->stripe_ptr[rank], host.data(), static_cast<size_t>(n) * qv::kPage, cudaMemcpyHostToDevice));
}

void ensure_staging(qv_engine* e, int64_t nq, int64_t k) {
  const int64_t q = nq * e->L.dim, r = nq * k;
  if (q > e->cap_q) {
    if (e->d_q) CK(cudaFree(e->d_q));
    CK(cudaMalloc(&e->d_q, q * 4));
    e->cap_q = q;
  }
  if (r > e->cap_r) {
    if (e->d_ids) CK(cudaFree(e->d_ids));
    if (e->d_dists) CK(cudaFree(e->d_dists));
    CK(cudaMalloc(&e->d_ids, r * 4));
    CK(cudaMalloc(&e->d_dists, r * 4));
    e->cap_r = r;
  }
  if (nq > e->cap_n) {
    for (void* p : {(void*)e->d_found, (void*)e->d_steps, (void*)e->d_nbrs, (void*)e->d_time})
      if (p) CK(cudaFree(p));
    CK(cudaMalloc(&e->d_time, nq * 16));
    CK(cudaMalloc(&e->d_found, nq * 4));
    CK(cudaMalloc(&e->d_steps, nq * 4));
    CK(cudaMalloc(&e->d_nbrs, nq * 8));
    e->cap_n = nq;
  }
}

float elapsed(cudaEvent_t a, cudaEvent_t b) {
  float ms = 0.f;
  CK(cudaEventElapsedTime(&ms, a, b));
  return ms;
}

// --------------------------------------------------- component kernels --

__global__ void lut_component_kernel(const qvk::SearchParams p, float* lut, float* q2) {
  const int lane = threadIdx.x & 31;
  const int64_t q = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (q >= p.nq) return;
  qvk::build_lut_warp(p, p.queries + q * p.dim, lut + q * int64_t(p.M) * qvk::kPivots,
                      q2 + q * p.dim, lane);
}

__global__ void adc_component_kernel(const uint8_t* __restrict__ codes, int M,
                                     const float* __restrict__ lut, const int32_t* __restrict__ qof,
                                     const int32_t* __restrict__ ids, int64_t n, float* out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float* t = lut + static_cast<int64_t>(qof[i]) * M * qvk::kPivots;
  const uint8_t* c = codes + static_cast<int64_t>(ids[i]) * M;
  float acc = 0.f;
  for (int j = 0; j < M; ++j) acc = __fadd_rn(acc, t[j * qvk::kPivots + c[j]]);
  out[i] = acc;
}

template <typename T>
__global__ void l2_component_kernel(const qvk::SearchParams p, const float* q2, const int32_t* qof,
                                    const int32_t* ids, int64_t n, float* out) {
  const int lane = threadIdx.x & 31;
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (i >= n) return;
  const int64_t v = ids[i];
  const T* vec = reinterpret_cast<const T*>(qvk::node_record(p, static_cast<uint32_t>(v)));
  const float d = qvk::exact_l2_warp<T>(q2 + static_cast<int64_t>(qof[i]) * p.dim, vec, p.dim, lane);
  if (lane == 0) out[i] = d;
}

}  // namespace

// ================================================================ C ABI ==

extern "C" {

const char* qv_version(void) { return "quiver-b200 0.1.0 (sm_100a)"; }

const char* qv_last_error(void) { return g_last_error.c_str(); }

}  // extern "C"

namespace qv {
void set_last_error(const std::string& m) { g_last_error = m; }
}  // namespace qv

extern "C" {

void qv_search_opts_default(qv_search_opts* o) {
  if (!o) return;
  o->topk = 10;
  o->ef_search = 30;
  o->pipe_width = 2;
  o->queries_per_block = 0;
  o->num_blocks = 0;
  o->early_exit_policy = QV_EXIT_GPRUNING;
  o->gpruning_warmup_steps = 10;
  o->gpruning_patience = 8;
  o->skip_nav = 0;
  o->visited_filter = 0;
  o->lut_mode = QV_LUT_FP32;
}

int qv_index_probe(const char* index_dir, int32_t data_type, qv_index_info* info) {
  return guarded([&] {
    if (!index_dir || !info) fail(QV_ERR_INVALID_ARG, "null argument");
    if (data_type != QV_UINT8 && data_type != QV_FLOAT && data_type != QV_INT8)
      fail(QV_ERR_INVALID_ARG, "data_type must be QV_UINT8, QV_FLOAT or QV_INT8");
    const std::string index_file = qv::find_index_file(index_dir);
    const std::string prefix = qv::find_pq_prefix(index_dir);
    const qv::Layout L = qv::parse_disk_index_header(index_file, data_type);
    const qv::PQTables pq = qv::read_pq(prefix + "_pivots.bin", prefix + "_compressed.bin");
    qv::check_layout(L, &pq);
    info->num_points = L.num_points;
    info->dim = L.dim;
    info->max_degree = L.max_degree;
    info->node_size = L.node_size;
    info->data_size = L.data_size;
    info->nodes_per_page = L.nodes_per_page;
    info->num_pages = L.num_pages;
    info->medoid = L.medoid;
    info->data_type = data_type;
    info->num_chunks = pq.num_chunks;
  });
}

int qv_engine_create(const qv_engine_opts* opts, qv_engine** out) {
  return guarded([&] {
    if (!opts || !out || !opts->index_dir) fail(QV_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    if (opts->data_type != QV_UINT8 && opts->data_type != QV_FLOAT && opts->data_type != QV_INT8)
      fail(QV_ERR_INVALID_ARG, "data_type must be QV_UINT8, QV_FLOAT or QV_INT8");
    const std::string dir = opts->index_dir;
    const std::string backend = opts->memory_backend && *opts->memory_backend ? opts->memory_backend : "heap";
    if (backend != "heap" && backend != "mmap")
      fail(QV_ERR_INVALID_ARG, "Unsupported --memory-backend '" + backend + "'. Expected one of: heap, mmap");
    const std::string index_file = qv::find_index_file(dir);
    const std::string page_file =
        opts->memory_index_file && *opts->memory_index_file ? opts->memory_index_file : index_file;
    const std::string prefix = qv::find_pq_prefix(dir);
    auto e = std::make_unique<qv_engine>();
    e->L = qv::parse_disk_index_header(index_file, opts->data_type);
    qv::PQTables pq = qv::read_pq(prefix + "_pivots.bin", prefix + "_compressed.bin");
    qv::check_layout(e->L, &pq);
    e->M = pq.num_chunks;
    init_device_side(e.get(), opts->device);
    alloc_pages(e.get(), opts->page_store);
    const size_t bytes = static_cast<size_t>(e->L.num_pages) * qv::kPage;
    if (e->pages_host) {
      qv::read_pages(page_file, e->L.num_pages, backend, e->h_pages);
      if (opts->validate) {
        const int64_t b = qv::validate_adjacency(e->L, e->h_pages);
        if (b >= 0) fail(QV_ERR_BAD_INDEX, "adjacency list of node " + std::to_string(b) + " is malformed");
      }
    } else if (opts->page_store == QV_PAGES_SHARED) {
      if (opts->validate) fail(QV_ERR_INVALID_ARG, "validate needs the whole page store, not one stripe");
      load_own_stripe(e.get(), page_file, opts->num_stripes, opts->stripe_rank);
    } else if (opts->page_store == QV_PAGES_HBM && !opts->validate) {
      upload_pages_staged(e.get(), page_file, backend);
    } else {
      std::vector<uint8_t> host(bytes);
      qv::read_pages(page_file, e->L.num_pages, backend, host.data());
      if (opts->validate) {
        const int64_t b = qv::validate_adjacency(e->L, host.data());
        if (b >= 0) fail(QV_ERR_BAD_INDEX, "adjacency list of node " + std::to_string(b) + " is malformed");
      }
      if (opts->page_store == QV_PAGES_STRIPED)
        stripe_pages(e.get(), host.data(), opts->num_stripes, opts->stripe_devices);
      else
        CK(cudaMemcpy(e->d_pages, host.data(), bytes, cudaMemcpyHostToDevice));
    }
    upload_pq(e.get(), pq.pivots.data(), pq.centroid.data(), pq.chunk_offsets.data(), pq.codes.data());
    // search_setup.hpp:96-105: a nav graph next to the index is used when present
    const std::string nav_dir = qv::find_nav_dir(dir);
    if (!nav_dir.empty()) upload_nav(e.get(), qv::read_nav(nav_dir, qv::element_size(e->L.data_type)));
    *out = e.release();
  });
}

int qv_engine_create_from_arrays(const qv_index_arrays* a, int32_t device, int32_t page_store,
                                 qv_engine** out) {
  return guarded([&] {
    if (!a || !out || !a->pages || !a->codes || !a->pivots || !a->centroid || !a->chunk_offsets)
      fail(QV_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    auto e = std::make_unique<qv_engine>();
    const auto& in = a->info;
    if (in.data_type != QV_UINT8 && in.data_type != QV_FLOAT && in.data_type != QV_INT8)
      fail(QV_ERR_INVALID_ARG, "data_type must be QV_UINT8, QV_FLOAT or QV_INT8");
    e->L.num_points = in.num_points;
    e->L.dim = in.dim;
    e->L.data_type = in.data_type;
    e->L.node_size = in.node_size;
    e->L.data_size = in.dim * qv::element_size(in.data_type);
    e->L.max_degree = (in.node_size - e->L.data_size) / 4 - 1;
    e->L.nodes_per_page = in.nodes_per_page;
    if (in.nodes_per_page <= 0) fail(QV_ERR_BAD_INDEX, "nodes_per_page must be positive");
    e->L.num_pages = (in.num_points + in.nodes_per_page - 1) / in.nodes_per_page;
    e->L.medoid = in.medoid;
    e->M = in.num_chunks;
    qv::PQTables shape;
    shape.dim = static_cast<int32_t>(in.dim);
    shape.num_chunks = in.num_chunks;
    shape.num_points = in.num_points;
    shape.chunk_offsets.assign(a->chunk_offsets, a->chunk_offsets + in.num_chunks + 1);
    qv::check_layout(e->L, &shape);
    init_device_side(e.get(), device);
    if (page_store == QV_PAGES_STRIPED)
      fail(QV_ERR_UNSUPPORTED, "a striped page store is created from an index directory (qv_engine_create)");
    alloc_pages(e.get(), page_store);
    const size_t bytes = static_cast<size_t>(e->L.num_pages) * qv::kPage;
    if (e->pages_host)
      std::memcpy(e->h_pages, a->pages, bytes);
    else
      CK(cudaMemcpy(e->d_pages, a->pages, bytes, cudaMemcpyHostToDevice));
    upload_pq(e.get(), a->pivots, a->centroid, a->chunk_offsets, a->codes);
    *out = e.release();
  });
}

int qv_engine_set_nav(qv_engine* e, const void* data, const int32_t* graph, const int32_t* mapping,
                      int32_t num_node, int32_t max_m, int32_t start) {
  return guarded([&] {
    if (!e) fail(QV_ERR_INVALID_ARG, "null argument");
    CK(cudaSetDevice(e->device));
    if (num_node == 0) {
      for (void* p : {(void*)e->d_nav_data, (void*)e->d_nav_graph, (void*)e->d_nav_map})
        if (p) CK(cudaFree(p));
      e->d_nav_data = nullptr;
      e->d_nav_graph = nullptr;
      e->d_nav_map = nullptr;
      e->nav_num_node = 0;
      return;
    }
    if (!data || !graph || !mapping) fail(QV_ERR_INVALID_ARG, "null argument");
    if (num_node < 0 || max_m <= 0 || max_m > 32) fail(QV_ERR_INVALID_ARG, "num_node >= 0 and 0 < max_m <= 32");
    qv::NavHost nav;
    nav.num_node = num_node;
    nav.data_len = static_cast<int32_t>(e->L.dim);
    nav.max_m = max_m;
    nav.start = start;
    const size_t vb = static_cast<size_t>(num_node) * e->L.dim * qv::element_size(e->L.data_type);
    nav.data.assign(static_cast<const uint8_t*>(data), static_cast<const uint8_t*>(data) + vb);
    nav.graph.assign(graph, graph + static_cast<size_t>(num_node) * max_m);
    nav.mapping.assign(mapping, mapping + num_node);
    upload_nav(e, nav);
  });
}

int qv_engine_nav_info(const qv_engine* e, int32_t* num_node, int32_t* max_m, int32_t* start) {
  return guarded([&] {
    if (!e || !num_node || !max_m || !start) fail(QV_ERR_INVALID_ARG, "null argument");
    *num_node = e->nav_num_node;
    *max_m = e->nav_max_m;
    *start = e->nav_start;
  });
}

int qv_engine_info(const qv_engine* e, qv_index_info* info) {
  return guarded([&] {
    if (!e || !info) fail(QV_ERR_INVALID_ARG, "null argument");
    info->num_points = e->L.num_points;
    info->dim = e->L.dim;
    info->max_degree = e->L.max_degree;
    info->node_size = e->L.node_size;
    info->data_size = e->L.data_size;
    info->nodes_per_page = e->L.nodes_per_page;
    info->num_pages = e->L.num_pages;
    info->medoid = e->L.medoid;
    info->data_type = e->L.data_type;
    info->num_chunks = e->M;
  });
}

void qv_engine_destroy(qv_engine* e) { delete e; }

int qv_engine_stripe_handle(qv_engine* e, void* handle) {
  return guarded([&] {
    if (!e || !handle) fail(QV_ERR_INVALID_ARG, "null argument");
    if (!e->shared) fail(QV_ERR_INVALID_ARG, "the engine's page store is not QV_PAGES_SHARED");
    static_assert(sizeof(cudaIpcMemHandle_t) == QV_STRIPE_HANDLE_BYTES, "IPC handle size");
    CK(cudaSetDevice(e->device));
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, e->stripe_ptr[e->stripe_rank]));
    std::memcpy(handle, &h, sizeof(h));
  });
}

int qv_engine_attach_stripes(qv_engine* e, const void* handles) {
  return guarded([&] {
    if (!e || !handles) fail(QV_ERR_INVALID_ARG, "null argument");
    if (!e->shared) fail(QV_ERR_INVALID_ARG, "the engine's page store is not QV_PAGES_SHARED");
    if (e->attached) fail(QV_ERR_INVALID_ARG, "stripes are already attached");
    CK(cudaSetDevice(e->device));
    const int S = static_cast<int>(e->stripe_ptr.size());
    // All or nothing: a failure closes the mappings this call opened, so the
    // engine is left as it was and the call can be retried.
    std::vector<void*> opened;
    auto undo = [&] {
      for (void* p : opened) cudaIpcCloseMemHandle(p);
      for (int s = 0; s < S; ++s)
        if (s != e->stripe_rank) e->stripe_ptr[s] = nullptr;
    };
    for (int s = 0; s < S; ++s) {
      if (s == e->stripe_rank) continue;
      cudaIpcMemHandle_t h;
      std::memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(s) * QV_STRIPE_HANDLE_BYTES,
                  sizeof(h));
      void* p = nullptr;
      const cudaError_t r = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
      if (r != cudaSuccess) {
        undo();
        fail(QV_ERR_CUDA, "opening stripe " + std::to_string(s) + ": " + cudaGetErrorString(r));
      }
      opened.push_back(p);
      e->stripe_ptr[s] = static_cast<uint8_t*>(p);
    }
    uint8_t** table = nullptr;
    cudaError_t r = cudaMalloc(&table, sizeof(uint8_t*) * S);
    if (r == cudaSuccess)
      r = cudaMemcpy(table, e->stripe_ptr.data(), sizeof(uint8_t*) * S, cudaMemcpyHostToDevice);
    if (r != cudaSuccess) {
      if (table) cudaFree(table);
      undo();
      fail(QV_ERR_CUDA, std::string("stripe table: ") + cudaGetErrorString(r));
    }
    e->imported.insert(e->imported.end(), opened.begin(), opened.end());
    e->d_stripe_table = table;
    e->d_pages = e->stripe_ptr[0];
    e->attached = true;
  });
}

int qv_plan(qv_engine* e, const qv_search_opts* opts, int64_t nq, qv_search_stats* plan) {
  return guarded([&] {
    if (!e || !opts || !plan) fail(QV_ERR_INVALID_ARG, "null argument");
    CK(cudaSetDevice(e->device));
    const Plan pl = make_plan(e, *opts, std::max<int64_t>(nq, 1));
    std::memset(plan, 0, sizeof(*plan));
    plan->grid = pl.grid;
    plan->slots_per_block = pl.slots;
    plan->smem_per_block = pl.smem;
    plan->blocks_per_sm = pl.blocks_per_sm;
  });
}

static int search_host(qv_engine* e, const float* queries, int64_t nq, int64_t dim, const qv_search_opts* opts,
                       int32_t* ids, float* dists, int32_t* found, float* query_ms, qv_search_stats* stats) {
  return guarded([&] {
    if (!e || !opts || (nq > 0 && (!queries || !ids || !dists))) fail(QV_ERR_INVALID_ARG, "null argument");
    if (nq < 0) fail(QV_ERR_INVALID_ARG, "nq must be non-negative");
    if (dim != e->L.dim)
      fail(QV_ERR_INVALID_ARG, "Query dimension mismatch: queries have " + std::to_string(dim) +
                                   " dims, but the index expects " + std::to_string(e->L.dim));
    const auto t0 = std::chrono::steady_clock::now();
    CK(cudaSetDevice(e->device));
    const Plan pl = make_plan(e, *opts, std::max<int64_t>(nq, 1));
    if (stats) std::memset(stats, 0, sizeof(*stats));
    if (nq == 0) return;
    ensure_staging(e, nq, opts->topk);
    const bool want_counts = stats != nullptr;
    cudaStream_t st = e->stream;
    CK(cudaEventRecord(e->ev[0], st));
    CK(cudaMemcpyAsync(e->d_q, queries, nq * dim * 4, cudaMemcpyHostToDevice, st));
    CK(cudaEventRecord(e->ev[1], st));
    auto p = make_params(e, pl, *opts, e->d_q, nq, e->d_ids, e->d_dists, e->d_found,
                         want_counts ? e->d_steps : nullptr, want_counts ? e->d_nbrs : nullptr,
                         query_ms ? e->d_time : nullptr);
    prepare_visited(e, pl, *opts, nq, p, st);
    enqueue_search(e, pl, p, st);
    CK(cudaEventRecord(e->ev[2], st));
    CK(cudaMemcpyAsync(ids, e->d_ids, nq * opts->topk * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(dists, e->d_dists, nq * opts->topk * 4, cudaMemcpyDeviceToHost, st));
    if (found) CK(cudaMemcpyAsync(found, e->d_found, nq * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaEventRecord(e->ev[3], st));
    CK(cudaStreamSynchronize(st));
    read_device_status(e);
    if (query_ms) {
      std::vector<int64_t> t(2 * nq);
      CK(cudaMemcpy(t.data(), e->d_time, nq * 16, cudaMemcpyDeviceToHost));
      for (int64_t i = 0; i < nq; ++i) query_ms[i] = static_cast<float>((t[2 * i + 1] - t[2 * i]) * 1e-6);
    }
    if (stats) {
      stats->h2d_ms = elapsed(e->ev[0], e->ev[1]);
      stats->kernel_ms = elapsed(e->ev[1], e->ev[2]);
      stats->d2h_ms = elapsed(e->ev[2], e->ev[3]);
      std::vector<int32_t> steps(nq);
      std::vector<int64_t> nbrs(nq);
      CK(cudaMemcpy(steps.data(), e->d_steps, nq * 4, cudaMemcpyDeviceToHost));
      CK(cudaMemcpy(nbrs.data(), e->d_nbrs, nq * 8, cudaMemcpyDeviceToHost));
      for (int64_t i = 0; i < nq; ++i) {
        stats->expansions += steps[i];
        stats->neighbors_scored += nbrs[i];
      }
      stats->grid = pl.grid;
      stats->slots_per_block = pl.slots;
      stats->smem_per_block = pl.smem;
      stats->blocks_per_sm = pl.blocks_per_sm;
      stats->total_ms =
          std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    }
  });
}

int qv_search(qv_engine* e, const float* queries, int64_t nq, int64_t dim, const qv_search_opts* opts,
              int32_t* ids, float* dists, int32_t* found, qv_search_stats* stats) {
  return search_host(e, queries, nq, dim, opts, ids, dists, found, nullptr, stats);
}

int qv_search_timed(qv_engine* e, const float* queries, int64_t nq, int64_t dim, const qv_search_opts* opts,
                    int32_t* ids, float* dists, int32_t* found, float* query_ms, qv_search_stats* stats) {
  return search_host(e, queries, nq, dim, opts, ids, dists, found, query_ms, stats);
}

void qv_stream_opts_default(qv_stream_opts* o) {
  if (!o) return;
  o->prefeed = -1;
  o->admit_min_batch = 32;
  o->feed_timeout_ms = 10000;
  o->admit_limit = -1;
}

}  // extern "C"

namespace {

// Page-locks a caller's host array for the duration of a call; an array that
// is already registered (or a platform that refuses) is used as it is.
struct HostRegistration {
  void* ptr = nullptr;
  HostRegistration(const void* p, size_t bytes) {
    if (!p || bytes == 0) return;
    if (cudaHostRegister(const_cast<void*>(p), bytes, cudaHostRegisterDefault) == cudaSuccess)
      ptr = const_cast<void*>(p);
    else
      cudaGetLastError();
  }
  ~HostRegistration() {
    if (ptr) cudaHostUnregister(ptr);
  }
  HostRegistration(const HostRegistration&) = delete;
  HostRegistration& operator=(const HostRegistration&) = delete;
};

void ensure_stream_buffers(qv_engine* e, int64_t workers, int64_t ring) {
  if (!e->h2d_stream) CK(cudaStreamCreateWithFlags(&e->h2d_stream, cudaStreamNonBlocking));
  if (workers > e->cap_done) {
    if (e->h_done) CK(cudaFreeHost(e->h_done));
    e->h_done = nullptr;
    CK(cudaHostAlloc(&e->h_done, workers * sizeof(uint32_t), cudaHostAllocMapped));
    e->cap_done = workers;
  }
  if (ring > static_cast<int64_t>(e->feed_ev.size())) {
    if (e->h_feed) CK(cudaFreeHost(e->h_feed));
    e->h_feed = nullptr;
    CK(cudaHostAlloc(&e->h_feed, ring * sizeof(int32_t), cudaHostAllocDefault));
    const size_t old = e->feed_ev.size();
    e->feed_ev.resize(ring, nullptr);
    for (size_t i = old; i < e->feed_ev.size(); ++i)
      CK(cudaEventCreateWithFlags(&e->feed_ev[i], cudaEventDisableTiming));
  }
}

}  // namespace

extern "C" {

int qv_search_stream(qv_engine* e, const float* queries, int64_t nq, int64_t dim, const qv_search_opts* opts,
                     const qv_stream_opts* sopts, int32_t* ids, float* dists, int32_t* found,
                     float* query_latency_ms, qv_stream_stats* stats) {
  return guarded([&] {
    if (!e || !opts || (nq > 0 && (!queries || !ids || !dists))) fail(QV_ERR_INVALID_ARG, "null argument");
    if (nq < 0) fail(QV_ERR_INVALID_ARG, "nq must be non-negative");
    if (nq > INT32_MAX / 2) fail(QV_ERR_INVALID_ARG, "nq above 2^30");
    if (dim != e->L.dim)
      fail(QV_ERR_INVALID_ARG, "Query dimension mismatch: queries have " + std::to_string(dim) +
                                   " dims, but the index expects " + std::to_string(e->L.dim));
    qv_stream_opts so;
    qv_stream_opts_default(&so);
    if (sopts) so = *sopts;
    if (so.admit_min_batch < 1) fail(QV_ERR_INVALID_ARG, "admit_min_batch must be >= 1");
    if (so.feed_timeout_ms < 1) fail(QV_ERR_INVALID_ARG, "feed_timeout_ms must be >= 1");
    CK(cudaSetDevice(e->device));
    const Plan pl = make_plan(e, *opts, std::max<int64_t>(nq, 1));
    if (stats) std::memset(stats, 0, sizeof(*stats));
    if (nq == 0) return;
    const int64_t workers = pl.block ? pl.grid : static_cast<int64_t>(pl.grid) * pl.slots;
    const int64_t prefeed = so.prefeed < 0 ? workers : so.prefeed;
    const int64_t max_inflight = std::max<int64_t>(1, workers + prefeed);
    const int64_t ring = std::max<int64_t>(64, 2 * max_inflight);
    ensure_staging(e, nq, opts->topk);
    ensure_stream_buffers(e, workers, ring);
    HostRegistration reg(queries, static_cast<size_t>(nq) * dim * sizeof(float));
    std::memset(e->h_done, 0, workers * sizeof(uint32_t));
    uint32_t* d_done = nullptr;
    CK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d_done), e->h_done, 0));
    auto p = make_params(e, pl, *opts, e->d_q, nq, e->d_ids, e->d_dists, e->d_found,
                         stats ? e->d_steps : nullptr, nullptr);
    p.feed = e->d_scratch + 6;
    p.done_slots = d_done;
    p.feed_timeout_ns = static_cast<int64_t>(so.feed_timeout_ms) * 1000000;
    cudaStream_t ks = e->stream, hs = e->h2d_stream;
    prepare_visited(e, pl, *opts, nq, p, ks);
    CK(cudaStreamSynchronize(ks));

    using clock = std::chrono::steady_clock;
    const auto t0 = clock::now();
    auto now_ms = [&] { return std::chrono::duration<double, std::milli>(clock::now() - t0).count(); };
    const int64_t limit = so.admit_limit < 0 ? nq : std::min<int64_t>(nq, so.admit_limit);
    std::vector<double> start(nq, 0.0), lat(nq, 0.0);
    // First range before the launch (search.cu:853-890): copied and made visible synchronously.
    const int64_t initial = std::min(max_inflight, limit);
    e->h_feed[0] = static_cast<int32_t>(initial);
    CK(cudaMemsetAsync(e->d_scratch, 0, 8 * sizeof(int32_t), hs));
    if (initial > 0) CK(cudaMemcpyAsync(e->d_q, queries, initial * dim * 4, cudaMemcpyHostToDevice, hs));
    CK(cudaMemcpyAsync(e->d_scratch + 6, e->h_feed, sizeof(int32_t), cudaMemcpyHostToDevice, hs));
    CK(cudaStreamSynchronize(hs));
    int64_t admissions = 1;
    pl.launch_stream(p, pl.grid, pl.threads, pl.smem, ks);
    CK(cudaGetLastError());

    // Admission loop (search.cu:983-1051): retire finished copies, charge new
    // completions, admit the next range when flow control allows.
    const volatile uint32_t* done_slots = e->h_done;
    int64_t last_done = 0, next = initial, head = 0, pending = 0;
    uint64_t polls = 0;
    while (last_done < nq) {
      while (pending > 0) {
        const cudaError_t q = cudaEventQuery(e->feed_ev[head]);
        if (q == cudaErrorNotReady) break;
        CK(q);
        head = (head + 1) % ring;
        --pending;
      }
      int64_t done = 0;
      for (int64_t w = 0; w < workers; ++w) done += done_slots[w];
      if (done > last_done) {
        const double t = now_ms();
        for (int64_t i = last_done; i < std::min(done, nq); ++i) lat[i] = t - start[i];
        last_done = std::min(done, nq);
        if (last_done >= nq) break;
      }
      const int64_t target = std::min(limit, last_done + max_inflight);
      const int64_t gap = target - next;
      if (gap > 0 && pending < ring && (gap >= so.admit_min_batch || target == limit || pending == 0)) {
        const double t = now_ms();
        const int64_t slot = (head + pending) % ring;
        e->h_feed[slot] = static_cast<int32_t>(target);
        CK(cudaMemcpyAsync(e->d_q + next * dim, queries + next * dim, gap * dim * 4, cudaMemcpyHostToDevice, hs));
        CK(cudaMemcpyAsync(e->d_scratch + 6, e->h_feed + slot, sizeof(int32_t), cudaMemcpyHostToDevice, hs));
        CK(cudaEventRecord(e->feed_ev[slot], hs));
        for (int64_t i = next; i < target; ++i) start[i] = t;
        next = target;
        ++pending;
        ++admissions;
      }
      if ((++polls & 255) == 0) {
        // The kernel ended (or failed) with queries still outstanding: a worker gave up on its feed.
        const cudaError_t q = cudaStreamQuery(ks);
        if (q == cudaSuccess) {
          int64_t d2 = 0;
          for (int64_t w = 0; w < workers; ++w) d2 += done_slots[w];
          if (d2 < nq) {
            CK(cudaStreamSynchronize(hs));
            read_device_status(e);
            fail(QV_ERR_DEVICE, "streaming search ended with " + std::to_string(d2) + " of " +
                                    std::to_string(nq) + " queries completed");
          }
        } else if (q != cudaErrorNotReady) {
          CK(q);
        }
      }
    }
    const double search_ms = now_ms();
    CK(cudaStreamSynchronize(ks));
    CK(cudaStreamSynchronize(hs));
    read_device_status(e);
    CK(cudaMemcpyAsync(ids, e->d_ids, nq * opts->topk * 4, cudaMemcpyDeviceToHost, ks));
    CK(cudaMemcpyAsync(dists, e->d_dists, nq * opts->topk * 4, cudaMemcpyDeviceToHost, ks));
    if (found) CK(cudaMemcpyAsync(found, e->d_found, nq * 4, cudaMemcpyDeviceToHost, ks));
    CK(cudaStreamSynchronize(ks));
    if (query_latency_ms)
      for (int64_t i = 0; i < nq; ++i) query_latency_ms[i] = static_cast<float>(lat[i]);
    if (stats) {
      // Percentiles as the reference reports them (search.cu:1140-1152).
      std::vector<double> sorted(lat);
      std::sort(sorted.begin(), sorted.end());
      const size_t n = sorted.size();
      stats->search_ms = search_ms;
      stats->qps = nq / (search_ms / 1000.0);
      stats->lat_avg_ms = std::accumulate(sorted.begin(), sorted.end(), 0.0) / n;
      stats->lat_p50_ms = sorted[n * 50 / 100];
      stats->lat_p90_ms = sorted[n * 90 / 100];
      stats->lat_p99_ms = sorted[n * 99 / 100];
      stats->lat_p999_ms = sorted[static_cast<size_t>(n * 0.999)];
      stats->lat_max_ms = sorted[n - 1];
      stats->admissions = admissions;
      stats->workers = static_cast<int32_t>(workers);
      stats->max_inflight = static_cast<int32_t>(max_inflight);
      std::vector<int32_t> steps(nq);
      CK(cudaMemcpy(steps.data(), e->d_steps, nq * 4, cudaMemcpyDeviceToHost));
      for (int64_t i = 0; i < nq; ++i) stats->expansions += steps[i];
    }
  });
}

int qv_search_device(qv_engine* e, const float* d_queries, int64_t nq, const qv_search_opts* opts,
                     int32_t* d_ids, float* d_dists, int32_t* d_found, int32_t* d_steps,
                     int64_t* d_nbrs, void* stream) {
  return guarded([&] {
    if (!e || !opts || (nq > 0 && (!d_queries || !d_ids || !d_dists))) fail(QV_ERR_INVALID_ARG, "null argument");
    if (nq < 0) fail(QV_ERR_INVALID_ARG, "nq must be non-negative");
    CK(cudaSetDevice(e->device));
    const Plan pl = make_plan(e, *opts, std::max<int64_t>(nq, 1));
    if (nq == 0) return;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e->stream;
    auto p = make_params(e, pl, *opts, d_queries, nq, d_ids, d_dists, d_found, d_steps, d_nbrs);
    prepare_visited(e, pl, *opts, nq, p, st);
    enqueue_search(e, pl, p, st);
  });
}

int qv_check_device_status(qv_engine* e) {
  return guarded([&] {
    if (!e) fail(QV_ERR_INVALID_ARG, "null argument");
    CK(cudaSetDevice(e->device));
    CK(cudaDeviceSynchronize());
    read_device_status(e);
  });
}


// ---------------------------------------------------- scratch-free search --
// (the scratch array and its set-up are defined before engine set-up)

int qv_search_noalloc(qv_engine* e, const float* queries, int64_t nq, int64_t dim, const qv_search_opts* opts,
                      int32_t* ids, float* dists, int32_t* found) {
  return guarded([&] {
    if (!e || !opts || (nq > 0 && (!queries || !ids || !dists))) fail(QV_ERR_INVALID_ARG, "null argument");
    if (nq < 0) fail(QV_ERR_INVALID_ARG, "nq must be non-negative");
    if (dim != e->L.dim)
      fail(QV_ERR_INVALID_ARG, "Query dimension mismatch: queries have " + std::to_string(dim) +
                                   " dims, but the index expects " + std::to_string(e->L.dim));
    if (opts->visited_filter)
      fail(QV_ERR_UNSUPPORTED, "the visited-filter mode needs per-CTA device tables; use qv_search");
    if (!e->d_noalloc) fail(QV_ERR_INVALID_ARG, "engine has no scratch address");
    CK(cudaSetDevice(e->device));
    const Plan pl = make_plan(e, *opts, std::max<int64_t>(nq, 1));
    if (nq == 0) return;
    const size_t k = static_cast<size_t>(opts->topk);
    // Bound nq before any product of it: every query needs dim*4 + 2*k*4 + 4
    // bytes of the array (before alignment), so a larger nq can never fit.
    const size_t per_query = static_cast<size_t>(dim) * 4 + 2 * k * 4 + 4;
    if (static_cast<uint64_t>(nq) > (QV_NOALLOC_SCRATCH_BYTES - kNoallocHeader) / per_query)
      fail(QV_ERR_INVALID_ARG, "qv_search_noalloc: " + std::to_string(nq) + " queries of " +
                                   std::to_string(per_query) + " bytes of scratch each are above its " +
                                   std::to_string(QV_NOALLOC_SCRATCH_BYTES) +
                                   "-byte maximum; split the batch or use qv_search");
    const size_t q_bytes = align256(static_cast<size_t>(nq) * dim * 4);
    const size_t r_bytes = align256(static_cast<size_t>(nq) * k * 4);
    const size_t f_bytes = align256(static_cast<size_t>(nq) * 4);
    const size_t need = kNoallocHeader + q_bytes + 2 * r_bytes + f_bytes;
    if (need > QV_NOALLOC_SCRATCH_BYTES)
      fail(QV_ERR_INVALID_ARG, "qv_search_noalloc: " + std::to_string(nq) + " queries need " + std::to_string(need) +
                                   " bytes of scratch, above its " + std::to_string(QV_NOALLOC_SCRATCH_BYTES) +
                                   "-byte maximum; split the batch or use qv_search");
    unsigned char* base = e->d_noalloc;
    int32_t* counters = reinterpret_cast<int32_t*>(base);
    float* d_q = reinterpret_cast<float*>(base + kNoallocHeader);
    int32_t* d_ids = reinterpret_cast<int32_t*>(base + kNoallocHeader + q_bytes);
    float* d_dists = reinterpret_cast<float*>(base + kNoallocHeader + q_bytes + r_bytes);
    int32_t* d_found = reinterpret_cast<int32_t*>(base + kNoallocHeader + q_bytes + 2 * r_bytes);
    cudaStream_t st = e->stream;
    CK(cudaMemsetAsync(counters, 0, 8 * sizeof(int32_t), st));
    CK(cudaMemcpyAsync(d_q, queries, static_cast<size_t>(nq) * dim * 4, cudaMemcpyHostToDevice, st));
    qvk::SearchParams p = make_params(e, pl, *opts, d_q, nq, d_ids, d_dists, d_found, nullptr, nullptr);
    p.work_counter = counters;
    p.error_info = counters + 1;
    pl.launch(p, pl.grid, pl.threads, pl.smem, st);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(ids, d_ids, static_cast<size_t>(nq) * k * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(dists, d_dists, static_cast<size_t>(nq) * k * 4, cudaMemcpyDeviceToHost, st));
    if (found) CK(cudaMemcpyAsync(found, d_found, static_cast<size_t>(nq) * 4, cudaMemcpyDeviceToHost, st));
    int32_t info[4];
    CK(cudaMemcpyAsync(info, counters + 1, sizeof(info), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    raise_device_error(info);
  });
}
int qv_build_lut_device(qv_engine* e, const float* d_queries, int64_t nq, float* d_lut, float* d_q2,
                        void* stream) {
  return guarded([&] {
    if (!e || (nq > 0 && (!d_queries || !d_lut || !d_q2))) fail(QV_ERR_INVALID_ARG, "null argument");
    CK(cudaSetDevice(e->device));
    if (nq <= 0) return;
    qv_search_opts o;
    qv_search_opts_default(&o);
    qvk::SearchParams p{};
    p.pivots_t = e->d_pivots_t;
    p.centroid = e->d_centroid;
    p.chunk_off = e->d_chunk_off;
    p.queries = d_queries;
    p.nq = nq;
    p.dim = static_cast<int32_t>(e->L.dim);
    p.M = e->M;
    const int warps_per_block = 4;
    const int64_t blocks = (nq + warps_per_block - 1) / warps_per_block;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e->stream;
    lut_component_kernel<<<static_cast<unsigned>(blocks), warps_per_block * 32, 0, st>>>(p, d_lut, d_q2);
    CK(cudaGetLastError());
    if (!stream) CK(cudaStreamSynchronize(st));
  });
}

int qv_adc_device(qv_engine* e, const float* d_lut, const int32_t* d_qof, const int32_t* d_ids, int64_t n,
                  float* d_out, void* stream) {
  return guarded([&] {
    if (!e || (n > 0 && (!d_lut || !d_qof || !d_ids || !d_out))) fail(QV_ERR_INVALID_ARG, "null argument");
    CK(cudaSetDevice(e->device));
    if (n <= 0) return;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e->stream;
    adc_component_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(e->d_codes, e->M, d_lut,
                                                                                 d_qof, d_ids, n, d_out);
    CK(cudaGetLastError());
    if (!stream) CK(cudaStreamSynchronize(st));
  });
}

int qv_exact_l2_device(qv_engine* e, const float* d_q2, const int32_t* d_qof, const int32_t* d_ids, int64_t n,
                       float* d_out, void* stream) {
  return guarded([&] {
    if (!e || (n > 0 && (!d_q2 || !d_qof || !d_ids || !d_out))) fail(QV_ERR_INVALID_ARG, "null argument");
    if (e->shared && !e->attached)
      fail(QV_ERR_INVALID_ARG, "a shared page store needs every process's stripe (qv_engine_attach_stripes) first");
    CK(cudaSetDevice(e->device));
    if (n <= 0) return;
    qvk::SearchParams p{};
    p.pages = e->d_pages;
    p.stripe_table = reinterpret_cast<const unsigned long long*>(e->d_stripe_table);
    p.stripe_shift = e->stripe_shift;
    p.dim = static_cast<int32_t>(e->L.dim);
    p.npp = static_cast<int32_t>(e->L.nodes_per_page);
    p.node_size = static_cast<int32_t>(e->L.node_size);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e->stream;
    const unsigned blocks = static_cast<unsigned>((n * 32 + 255) / 256);
    switch (e->L.data_type) {
      case QV_UINT8: l2_component_kernel<uint8_t><<<blocks, 256, 0, st>>>(p, d_q2, d_qof, d_ids, n, d_out); break;
      case QV_INT8: l2_component_kernel<int8_t><<<blocks, 256, 0, st>>>(p, d_q2, d_qof, d_ids, n, d_out); break;
      default: l2_component_kernel<float><<<blocks, 256, 0, st>>>(p, d_q2, d_qof, d_ids, n, d_out); break;
    }
    CK(cudaGetLastError());
    if (!stream) CK(cudaStreamSynchronize(st));
  });
}

}  // extern "C"
