// ref_harness.cu -- drives the REFERENCE's own persistent search kernel.
//
// TEST INFRASTRUCTURE ONLY: it produces golden outputs that pin the CPU
// oracle; the product never links it.  Built by oracle/ref_harness.py into
// oracle/_ref/ from the reference sources where they lie (-I <reference>/src);
// nothing of the reference is copied here.
//
// The reference kernel (src/quiver/kernel_core/kernel_q1.cuh, Q = 1) asks
// host poll threads for 4 KB pages through host-mapped IOControl words
// (src/quiver/io_control.cuh:11-39) and is fed queries through
// PersistentKernelComm::feed_count.  This harness plays the host side with
// one thread: every query is admitted before the launch, and the poll loop
// copies page node/npp of the in-memory page store into the lane's buffer
// and marks it ready -- what MemLoaderSync::submit_direct does
// (src/shared/io/mem_loader.cpp:104-117) behind cpu_poll_loop
// (src/quiver/search.cu:180-304).  Only pipe width 1 is driven: with W > 1
// the reference's traversal depends on completion order.
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "quiver/kernel_core/kernel_q1.cuh"

namespace {

// Set when the kernel did not finish: freeing would wait on it forever, so
// the buffers are left to process exit.
bool g_kernel_stuck = false;

struct DevBuf {
  void* p = nullptr;
  ~DevBuf() { if (p && !g_kernel_stuck) cudaFree(p); }
};

template <class T>
int launch(const quiver::PersistentKernelArgs& args, int grid, int smem, cudaStream_t st) {
  quiver::persistent_search_kernel<quiver::StreamingDispatch, T><<<grid, 128, smem, st>>>(args);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

#define HCK(x) do { if ((x) != cudaSuccess) { rc = -2; goto done; } } while (0)

}  // namespace

extern "C" int ref_run_search(
    const uint8_t* pages, int64_t num_pages, int64_t node_size, int64_t data_size, int64_t npp, int64_t dim,
    int64_t max_m, int64_t num_points, int64_t medoid, int32_t dtype, const uint8_t* codes, int32_t M,
    const float* pivots_t, const float* centroid, const int32_t* chunk_offsets, const float* queries, int32_t nq,
    int32_t topk, int32_t ef, int32_t early_policy, int32_t warmup, int32_t patience, int32_t num_blocks,
    int32_t* out_ids, float* out_dists, int32_t* out_found, int32_t* out_steps, double timeout_s,
    const void* nav_data, const int32_t* nav_graph, const int32_t* nav_mapping, int32_t nav_num_node,
    int32_t nav_max_m, int32_t nav_start) {
  using namespace quiver;
  int rc = 0;
  g_kernel_stuck = false;
  const int W = 1;
  const int aligned_ef = static_cast<int>((max_m + ef + 31) / 32 * 32);
  std::vector<int32_t> chunk_id(dim, -1);
  for (int c = 0; c < M; ++c)
    for (int i = chunk_offsets[c]; i < chunk_offsets[c + 1]; ++i) chunk_id[i] = c;

  DevBuf d_centroid, d_pivots_t, d_chunk_id, d_codes, d_pq_dists, d_pqdata, d_qdata, d_nid, d_ndist, d_ctx,
      d_nns, d_dist, d_fc, d_next, d_done, d_finish, d_stop, d_nav_data, d_nav_graph, d_nav_map;
  IOControl* h_ctl = nullptr;
  uint8_t* h_buf = nullptr;
  PersistentKernelComm* h_comm = nullptr;
  int32_t* h_out_nns = nullptr;
  float* h_out_dist = nullptr;
  int32_t* h_out_fc = nullptr;
  cudaStream_t st = nullptr;
  std::atomic<bool> stop_poll{false};
  std::thread poller;
  PersistentKernelArgs args{};
  shared::PQSearchData pqd{};
  int smem = 0;

  HCK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  HCK(cudaMalloc(&d_centroid.p, dim * 4));
  HCK(cudaMemcpy(d_centroid.p, centroid, dim * 4, cudaMemcpyHostToDevice));
  HCK(cudaMalloc(&d_pivots_t.p, dim * 256 * 4));
  HCK(cudaMemcpy(d_pivots_t.p, pivots_t, dim * 256 * 4, cudaMemcpyHostToDevice));
  HCK(cudaMalloc(&d_chunk_id.p, dim * 4));
  HCK(cudaMemcpy(d_chunk_id.p, chunk_id.data(), dim * 4, cudaMemcpyHostToDevice));
  HCK(cudaMalloc(&d_codes.p, num_points * M));
  HCK(cudaMemcpy(d_codes.p, codes, num_points * M, cudaMemcpyHostToDevice));
  HCK(cudaMalloc(&d_pq_dists.p, static_cast<size_t>(num_blocks) * 256 * M * 4));
  pqd.dim = static_cast<int>(dim);
  pqd.num_chunks = M;
  pqd.num_pts = static_cast<int>(num_points);
  pqd.centroid = static_cast<float*>(d_centroid.p);
  pqd.pivots_t = static_cast<float*>(d_pivots_t.p);
  pqd.chunk_id = static_cast<int*>(d_chunk_id.p);
  pqd.compressed_data = static_cast<uint8_t*>(d_codes.p);
  pqd.pq_dists = static_cast<float*>(d_pq_dists.p);
  HCK(cudaMalloc(&d_pqdata.p, sizeof(pqd)));
  HCK(cudaMemcpy(d_pqdata.p, &pqd, sizeof(pqd), cudaMemcpyHostToDevice));

  // nav graph (NavGraph::init, nav_graph.cu:12-73: vectors, -1 padded rows, map)
  if (nav_num_node > 0) {
    const size_t vb = static_cast<size_t>(nav_num_node) * dim * (dtype == 1 ? 4 : 1);
    HCK(cudaMalloc(&d_nav_data.p, vb));
    HCK(cudaMemcpy(d_nav_data.p, nav_data, vb, cudaMemcpyHostToDevice));
    HCK(cudaMalloc(&d_nav_graph.p, static_cast<size_t>(nav_num_node) * nav_max_m * 4));
    HCK(cudaMemcpy(d_nav_graph.p, nav_graph, static_cast<size_t>(nav_num_node) * nav_max_m * 4,
                   cudaMemcpyHostToDevice));
    HCK(cudaMalloc(&d_nav_map.p, static_cast<size_t>(nav_num_node) * 4));
    HCK(cudaMemcpy(d_nav_map.p, nav_mapping, static_cast<size_t>(nav_num_node) * 4, cudaMemcpyHostToDevice));
  }
  HCK(cudaMalloc(&d_qdata.p, static_cast<size_t>(nq) * dim * 4));
  HCK(cudaMemcpy(d_qdata.p, queries, static_cast<size_t>(nq) * dim * 4, cudaMemcpyHostToDevice));
  HCK(cudaMalloc(&d_nid.p, static_cast<size_t>(num_blocks) * aligned_ef * 4));
  HCK(cudaMalloc(&d_ndist.p, static_cast<size_t>(num_blocks) * aligned_ef * 4));
  HCK(cudaMalloc(&d_ctx.p, sizeof(shared::Data) * num_blocks));
  HCK(cudaMalloc(&d_nns.p, static_cast<size_t>(num_blocks) * topk * 4));
  HCK(cudaMalloc(&d_dist.p, static_cast<size_t>(num_blocks) * topk * 4));
  HCK(cudaMalloc(&d_fc.p, num_blocks * 4));
  HCK(cudaMalloc(&d_next.p, 4));
  HCK(cudaMemset(d_next.p, 0, 4));
  HCK(cudaMalloc(&d_done.p, 4));
  HCK(cudaMemset(d_done.p, 0, 4));
  HCK(cudaMalloc(&d_finish.p, nq * 4));
  HCK(cudaMemset(d_finish.p, 0xff, nq * 4));
  HCK(cudaMalloc(&d_stop.p, nq * 4));
  HCK(cudaMemset(d_stop.p, 0xff, nq * 4));

  HCK(cudaHostAlloc(&h_ctl, sizeof(IOControl) * num_blocks * W, cudaHostAllocMapped));
  for (int i = 0; i < num_blocks * W; ++i) { h_ctl[i].status = IO_IDLE; h_ctl[i].node_id = 0; }
  HCK(cudaHostAlloc(&h_buf, static_cast<size_t>(num_blocks) * W * shared::PAGE_SIZE, cudaHostAllocMapped));
  HCK(cudaHostAlloc(&h_comm, sizeof(PersistentKernelComm), cudaHostAllocMapped));
  HCK(cudaHostAlloc(&h_out_nns, static_cast<size_t>(nq) * topk * 4, cudaHostAllocMapped));
  HCK(cudaHostAlloc(&h_out_dist, static_cast<size_t>(nq) * topk * 4, cudaHostAllocMapped));
  HCK(cudaHostAlloc(&h_out_fc, nq * 4, cudaHostAllocMapped));
  std::memset(h_comm, 0, sizeof(*h_comm));
  {
    IOControl* d_ctl_ptr = nullptr;
    uint8_t* d_buf_ptr = nullptr;
    PersistentKernelComm* d_comm = nullptr;
    HCK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d_ctl_ptr), h_ctl, 0));
    HCK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d_buf_ptr), h_buf, 0));
    HCK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d_comm), h_comm, 0));
    h_comm->controls = d_ctl_ptr;
    h_comm->buffers = d_buf_ptr;
    h_comm->pipe_w = W;
    h_comm->num_blocks = num_blocks;
    h_comm->total_queries = nq;
    h_comm->feed_count = nq;  // every query admitted up front
    h_comm->terminate = 0;
    h_comm->queries_completed = 0;
    args.comm = d_comm;
    int32_t *d_onns = nullptr, *d_ofc = nullptr;
    float* d_odist = nullptr;
    HCK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d_onns), h_out_nns, 0));
    HCK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d_odist), h_out_dist, 0));
    HCK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d_ofc), h_out_fc, 0));
    args.d_out_nns = d_onns;
    args.d_out_distances = d_odist;
    args.d_out_found_cnt = d_ofc;
  }
  args.d_next_query = static_cast<int*>(d_next.p);
  args.d_queries_done = static_cast<int*>(d_done.p);
  args.d_all_qdata = static_cast<float*>(d_qdata.p);
  args.d_entry_nodes = nullptr;
  args.enter_point = static_cast<int32_t>(medoid);
  args.nav_data_dev = nullptr;
  if (nav_num_node > 0) {  // what run_persistent_search sets (search.cu:597-605)
    args.nav_data_dev = static_cast<uint8_t*>(d_nav_data.p);
    args.nav_graph_dev = static_cast<int*>(d_nav_graph.p);
    args.nav_mapping_dev = static_cast<int*>(d_nav_map.p);
    args.nav_num_node = nav_num_node;
    args.nav_data_len = static_cast<int>(dim);
    args.nav_max_m = nav_max_m;
    args.nav_start = nav_start;
    args.nav_init_ef = ef < 5 ? ef : 5;
  }
  args.pq_data = static_cast<shared::PQSearchData*>(d_pqdata.p);
  args.num_chunks = M;
  args.pq_dists = static_cast<float*>(d_pq_dists.p);
  args.compressed_data = static_cast<uint8_t*>(d_codes.p);
  args.nodes_per_page = static_cast<int>(npp);
  args.node_size = static_cast<int>(node_size);
  args.data_size = static_cast<int>(data_size);
  args.num_dims = static_cast<int>(dim);
  args.max_m = static_cast<int>(max_m);
  args.ef_search = ef;
  args.aligned_ef = aligned_ef;
  args.topk = topk;
  args.pipe_w = W;
  args.queries_per_block = 1;
  args.num_blocks = num_blocks;
  args.pq_block_offset = 0;
  args.total_queries = nq;
  args.batch_offset = 0;
  args.d_neighbors_id = static_cast<uint32_t*>(d_nid.p);
  args.d_neighbors_dist = static_cast<float*>(d_ndist.p);
  args.d_ctx = static_cast<shared::Data*>(d_ctx.p);
  args.d_nns = static_cast<int*>(d_nns.p);
  args.d_distances = static_cast<float*>(d_dist.p);
  args.d_found_cnt = static_cast<int*>(d_fc.p);
  args.early_exit_policy = early_policy;
  args.early_exit_gpruning_warmup_steps = warmup;
  args.early_exit_gpruning_patience = patience;
  args.darth_comm_slots = nullptr;
  args.d_early_exit_stop_step = static_cast<int*>(d_stop.p);
  args.d_finish_step = static_cast<int*>(d_finish.p);

  // page server: IO_REQUESTED -> copy page node / npp -> IO_READY
  poller = std::thread([&] {
    const int slots = num_blocks * W;
    while (!stop_poll.load(std::memory_order_relaxed)) {
      for (int i = 0; i < slots; ++i) {
        int32_t expected = IO_REQUESTED;
        if (__atomic_load_n(&h_ctl[i].status, __ATOMIC_ACQUIRE) != IO_REQUESTED) continue;
        if (!__atomic_compare_exchange_n(&h_ctl[i].status, &expected, (int32_t)IO_SUBMITTED, false,
                                         __ATOMIC_ACQ_REL, __ATOMIC_RELAXED))
          continue;
        const int64_t node = h_ctl[i].node_id;
        const int64_t page = node / npp;
        if (node >= 0 && page < num_pages)
          std::memcpy(h_buf + static_cast<size_t>(i) * shared::PAGE_SIZE, pages + page * shared::PAGE_SIZE,
                      shared::PAGE_SIZE);
        __atomic_store_n(&h_ctl[i].status, (int32_t)IO_READY, __ATOMIC_RELEASE);
      }
    }
  });

  smem = static_cast<int>((((sizeof(int) * 3 + sizeof(float) * 2) * (ef + max_m)) + 7) & ~size_t(7)) +
         static_cast<int>(node_size);
  if (dtype == 0)
    rc = launch<uint8_t>(args, num_blocks, smem, st);
  else if (dtype == 2)
    rc = launch<int8_t>(args, num_blocks, smem, st);
  else
    rc = launch<float>(args, num_blocks, smem, st);
  if (rc == 0) {
    const auto t0 = std::chrono::steady_clock::now();
    while (__atomic_load_n(&h_comm->queries_completed, __ATOMIC_ACQUIRE) < nq) {
      if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) {
        rc = -3;
        break;
      }
      std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
    __atomic_store_n(&h_comm->terminate, 1, __ATOMIC_RELEASE);
    // the kernel's remaining blocks leave their admission spin on terminate
    const auto t1 = std::chrono::steady_clock::now();
    while (cudaStreamQuery(st) == cudaErrorNotReady) {
      if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t1).count() > timeout_s) {
        rc = -4;
        g_kernel_stuck = true;
        break;
      }
      std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
  }
  stop_poll.store(true);
  poller.join();
  if (rc == 0 && cudaStreamSynchronize(st) != cudaSuccess) rc = -5;
  if (rc == 0) {
    std::memcpy(out_ids, h_out_nns, static_cast<size_t>(nq) * topk * 4);
    std::memcpy(out_dists, h_out_dist, static_cast<size_t>(nq) * topk * 4);
    std::memcpy(out_found, h_out_fc, nq * 4);
    if (cudaMemcpy(out_steps, d_finish.p, nq * 4, cudaMemcpyDeviceToHost) != cudaSuccess) rc = -6;
  }
done:
  if (poller.joinable()) {
    stop_poll.store(true);
    poller.join();
  }
  if (rc != -4) {  // a kernel still running keeps its mapped buffers until process exit
    if (h_ctl) cudaFreeHost(h_ctl);
    if (h_buf) cudaFreeHost(h_buf);
    if (h_comm) cudaFreeHost(h_comm);
    if (h_out_nns) cudaFreeHost(h_out_nns);
    if (h_out_dist) cudaFreeHost(h_out_dist);
    if (h_out_fc) cudaFreeHost(h_out_fc);
    if (st) cudaStreamDestroy(st);
  }
  return rc;
}
