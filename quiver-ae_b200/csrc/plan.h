// plan.h -- launch plan shared by the engine and the per-type kernel units.
#pragma once

#include <cuda_runtime.h>

#include "search_block.cuh"
#include "search_kernel.cuh"

namespace qv {

struct Plan {
  qvk::SlotLayout lay;
  bool block = true;    // one 128-thread CTA per query; false: `slots` one-warp queries per CTA
  int smax = 2;         // neighbours per lane (R <= 32 * smax)
  int mc = 0;           // PQ code width the kernel is specialised for (0 = any)
  int slots = 1;        // query slots (warps) per CTA
  bool long_lists = false;  // block kernel: ef above 512 (the group merge's in-place path for long lists)
  int blocks_per_sm = 0;
  int grid = 0;
  int smem = 0;
  int threads = 0;      // CTA size
  const void* fn = nullptr;
  void (*launch)(const qvk::SearchParams&, int grid, int block, int smem, cudaStream_t) = nullptr;
  // the streaming-admission instantiation of the same kernel (waits for each query's feed)
  const void* fn_stream = nullptr;
  void (*launch_stream)(const qvk::SearchParams&, int grid, int block, int smem, cudaStream_t) = nullptr;
};

// Defined in search_u8.cu / search_i8.cu / search_f32.cu: pick the kernel
// instantiation for pl.mc and pl.smax.
void bind_search_u8(Plan& pl);
void bind_search_i8(Plan& pl);
void bind_search_f32(Plan& pl);

template <typename T, int MC, int SMAX, bool STREAM>
void launch_search(const qvk::SearchParams& p, int grid, int block, int smem, cudaStream_t st) {
  qvk::search_kernel<T, MC, SMAX, STREAM><<<grid, block, smem, st>>>(p);
}

template <typename T, int MC, int RP, bool STREAM, bool LONG>
void launch_block(const qvk::SearchParams& p, int grid, int block, int smem, cudaStream_t st) {
  qvk::search_block_kernel<T, MC, RP, STREAM, LONG><<<grid, block, smem, st>>>(p);
}

template <typename T, int MC, int RP, bool LONG>
void bind_block(Plan& pl) {
  pl.fn = reinterpret_cast<const void*>(&qvk::search_block_kernel<T, MC, RP, false, LONG>);
  pl.launch = &launch_block<T, MC, RP, false, LONG>;
  pl.fn_stream = reinterpret_cast<const void*>(&qvk::search_block_kernel<T, MC, RP, true, LONG>);
  pl.launch_stream = &launch_block<T, MC, RP, true, LONG>;
}

template <typename T, int MC, int SMAX>
void bind_one(Plan& pl) {
  if (pl.block) {
    if (pl.long_lists) bind_block<T, MC, 32 * SMAX, true>(pl);
    else bind_block<T, MC, 32 * SMAX, false>(pl);
  } else {
    pl.fn = reinterpret_cast<const void*>(&qvk::search_kernel<T, MC, SMAX, false>);
    pl.launch = &launch_search<T, MC, SMAX, false>;
    pl.fn_stream = reinterpret_cast<const void*>(&qvk::search_kernel<T, MC, SMAX, true>);
    pl.launch_stream = &launch_search<T, MC, SMAX, true>;
  }
}

// PQ widths with a register-blocked code path; any other M uses MC = 0.
template <typename T>
void bind_type(Plan& pl) {
  if (pl.mc == 32) {
    if (pl.smax == 2) bind_one<T, 32, 2>(pl); else bind_one<T, 32, 4>(pl);
  } else {
    pl.mc = 0;
    if (pl.smax == 2) bind_one<T, 0, 2>(pl); else bind_one<T, 0, 4>(pl);
  }
}

}  // namespace qv
