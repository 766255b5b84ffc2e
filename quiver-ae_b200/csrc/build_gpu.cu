// build_gpu.cu -- the workload generator and the PQ encoder of index_build.cpp
// on the GPU, bit for bit: the same hash streams, the same IEEE double
// operations in the same order (each product and sum separately rounded, as
// the host code compiled with -ffp-contract=off computes them) for the
// mixture, and the same sequential fp32 sums and first-minimum choice for
// the PQ codes.  Host buffers in and out; the work is sliced so the device
// footprint stays bounded at any n.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <string>
#include <vector>

#include "quiver_b200.h"
#include "synth_common.h"

namespace qv {
void set_last_error(const std::string& m);
}

namespace {

using qv_synth::gauss;
using qv_synth::hash3;

constexpr int64_t kSliceRows = 1 << 22;  // rows per device slice
constexpr int kMaxChunkWidth = 64;

__device__ __forceinline__ double noisy(const double* cen, double sigma, uint64_t seed, uint64_t stream, uint64_t idx) {
  return __dadd_rn(*cen, __dmul_rn(sigma, gauss(seed, stream, idx)));
}

__global__ void synth_kernel(uint64_t seed, int32_t stream, int64_t row0, int64_t n, int32_t dim, int64_t k,
                             double sigma, int32_t dtype, const double* __restrict__ centers, void* out) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= n) return;
  const uint64_t row = static_cast<uint64_t>(row0 + r);
  const int64_t c = static_cast<int64_t>(hash3(seed, qv_synth::kAssignStream + stream, row) % static_cast<uint64_t>(k));
  const double* cen = centers + c * dim;
  const uint64_t ns = qv_synth::kNoiseStream + stream;
  if (dtype == QV_UINT8) {
    uint8_t* o = static_cast<uint8_t*>(out) + r * dim;
    for (int d = 0; d < dim; ++d) {
      double v = rint(noisy(cen + d, sigma, seed, ns, row * static_cast<uint64_t>(dim) + d));
      v = v < 0.0 ? 0.0 : (v > 255.0 ? 255.0 : v);
      o[d] = static_cast<uint8_t>(v);
    }
  } else {
    double nrm = 0.0;
    for (int d = 0; d < dim; ++d) {
      const double x = noisy(cen + d, sigma, seed, ns, row * static_cast<uint64_t>(dim) + d);
      nrm = __dadd_rn(nrm, __dmul_rn(x, x));
    }
    nrm = __dsqrt_rn(nrm);
    float* o = static_cast<float*>(out) + r * dim;
    for (int d = 0; d < dim; ++d)
      o[d] = __double2float_rn(__ddiv_rn(noisy(cen + d, sigma, seed, ns, row * static_cast<uint64_t>(dim) + d), nrm));
  }
}

__device__ __forceinline__ float elem_f(const void* base, int32_t dtype, int64_t i) {
  if (dtype == QV_UINT8) return static_cast<float>(static_cast<const uint8_t*>(base)[i]);
  if (dtype == QV_INT8) return static_cast<float>(static_cast<const int8_t*>(base)[i]);
  return static_cast<const float*>(base)[i];
}

// grid (row blocks, M): each block holds chunk c's 256 centroids in shared memory.
__global__ void pq_encode_kernel(const void* __restrict__ base, int64_t n, int32_t dim, int32_t dtype,
                                 const float* __restrict__ pivots, const float* __restrict__ centroid,
                                 const int32_t* __restrict__ offs, int32_t M, uint8_t* __restrict__ codes) {
  extern __shared__ float piv[];
  const int c = blockIdx.y;
  const int lo = offs[c], w = offs[c + 1] - lo;
  for (int i = threadIdx.x; i < 256 * w; i += blockDim.x) piv[i] = pivots[(i / w) * dim + lo + (i % w)];
  __syncthreads();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float r[kMaxChunkWidth];
#pragma unroll 4
  for (int t = 0; t < w; ++t) r[t] = __fsub_rn(elem_f(base, dtype, i * dim + lo + t), centroid[lo + t]);
  float best = 3.4e38f;
  int bj = 0;
  for (int j = 0; j < 256; ++j) {
    float dd = 0.f;
    for (int t = 0; t < w; ++t) {
      const float u = __fsub_rn(r[t], piv[j * w + t]);
      dd = __fadd_rn(dd, __fmul_rn(u, u));
    }
    if (dd < best) {
      best = dd;
      bj = j;
    }
  }
  codes[i * M + c] = static_cast<uint8_t>(bj);
}

struct DeviceBuffers {
  std::vector<void*> ptrs;
  ~DeviceBuffers() {
    for (void* p : ptrs) cudaFree(p);
  }
  void* alloc(size_t bytes, std::string& err) {
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, std::max<size_t>(bytes, 16));
    if (e != cudaSuccess) {
      if (err.empty()) err = std::string("cudaMalloc: ") + cudaGetErrorString(e);
      return nullptr;
    }
    ptrs.push_back(p);
    return p;
  }
};

int fail(int code, const std::string& m) {
  qv::set_last_error(m);
  return code;
}

}  // namespace

extern "C" int qv_synth_mixture_gpu(uint64_t seed, int32_t stream, int64_t row0, int64_t n, int64_t dim,
                                    int64_t n_centers, double sigma, int32_t dtype, void* out, int32_t device) {
  if (!out || n < 0 || dim <= 0 || n_centers <= 0 || (dtype != QV_UINT8 && dtype != QV_FLOAT))
    return fail(QV_ERR_INVALID_ARG, "qv_synth_mixture_gpu: invalid argument");
  if (n == 0) return QV_OK;
  if (cudaSetDevice(device) != cudaSuccess) return fail(QV_ERR_CUDA, "qv_synth_mixture_gpu: cannot select device");
  cudaGetLastError();  // launches below are checked with it: drop an error left by an earlier call
  const std::vector<double> centers = qv_synth::mixture_centers(seed, n_centers, dim, dtype);
  const size_t esize = dtype == QV_UINT8 ? 1 : 4;
  std::string err;
  DeviceBuffers b;
  double* d_c = static_cast<double*>(b.alloc(centers.size() * 8, err));
  const int64_t slice = std::min(n, kSliceRows);
  void* d_out = b.alloc(static_cast<size_t>(slice) * dim * esize, err);
  if (!err.empty()) return fail(QV_ERR_OOM, "qv_synth_mixture_gpu: " + err);
  if (cudaMemcpy(d_c, centers.data(), centers.size() * 8, cudaMemcpyHostToDevice) != cudaSuccess)
    return fail(QV_ERR_CUDA, "qv_synth_mixture_gpu: copy of the centres failed");
  for (int64_t s0 = 0; s0 < n; s0 += slice) {
    const int64_t cnt = std::min(slice, n - s0);
    synth_kernel<<<static_cast<unsigned>((cnt + 127) / 128), 128>>>(seed, stream, row0 + s0, cnt,
                                                                     static_cast<int32_t>(dim), n_centers, sigma,
                                                                     dtype, d_c, d_out);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess)
      e = cudaMemcpy(static_cast<uint8_t*>(out) + static_cast<size_t>(s0) * dim * esize, d_out,
                     static_cast<size_t>(cnt) * dim * esize, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail(QV_ERR_CUDA, std::string("qv_synth_mixture_gpu: ") + cudaGetErrorString(e));
  }
  return QV_OK;
}

extern "C" int qv_pq_encode_gpu(const void* base, int64_t n, int64_t dim, int32_t dtype, int32_t M,
                                const float* pivots, const float* centroid, const int32_t* chunk_offsets,
                                int32_t device, uint8_t* codes) {
  if (!base || !pivots || !centroid || !chunk_offsets || !codes || n < 0 || dim <= 0 || M <= 0 || M > dim ||
      (dtype != QV_UINT8 && dtype != QV_INT8 && dtype != QV_FLOAT))
    return fail(QV_ERR_INVALID_ARG, "qv_pq_encode_gpu: invalid argument");
  int maxw = 0;
  for (int c = 0; c < M; ++c) {
    const int w = chunk_offsets[c + 1] - chunk_offsets[c];
    if (w <= 0 || chunk_offsets[c] < 0 || chunk_offsets[c + 1] > dim)
      return fail(QV_ERR_INVALID_ARG, "qv_pq_encode_gpu: bad chunk offsets");
    maxw = std::max(maxw, w);
  }
  if (maxw > kMaxChunkWidth) return fail(QV_ERR_UNSUPPORTED, "qv_pq_encode_gpu: chunk wider than 64 dims");
  if (n == 0) return QV_OK;
  if (cudaSetDevice(device) != cudaSuccess) return fail(QV_ERR_CUDA, "qv_pq_encode_gpu: cannot select device");
  cudaGetLastError();  // launches below are checked with it: drop an error left by an earlier call
  const size_t esize = dtype == QV_FLOAT ? 4 : 1;
  std::string err;
  DeviceBuffers b;
  float* d_piv = static_cast<float*>(b.alloc(static_cast<size_t>(256) * dim * 4, err));
  float* d_cen = static_cast<float*>(b.alloc(static_cast<size_t>(dim) * 4, err));
  int32_t* d_off = static_cast<int32_t*>(b.alloc(static_cast<size_t>(M + 1) * 4, err));
  const int64_t slice = std::min(n, kSliceRows);
  void* d_base = b.alloc(static_cast<size_t>(slice) * dim * esize, err);
  uint8_t* d_codes = static_cast<uint8_t*>(b.alloc(static_cast<size_t>(slice) * M, err));
  if (!err.empty()) return fail(QV_ERR_OOM, "qv_pq_encode_gpu: " + err);
  // A chunk's 256 centroids sit in shared memory: up to 64 KB, above the 48 KB a launch gets by default.
  const size_t smem = static_cast<size_t>(256) * maxw * 4;
  cudaError_t e = cudaFuncSetAttribute(pq_encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e == cudaSuccess) e = cudaMemcpy(d_piv, pivots, static_cast<size_t>(256) * dim * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(d_cen, centroid, static_cast<size_t>(dim) * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(d_off, chunk_offsets, static_cast<size_t>(M + 1) * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail(QV_ERR_CUDA, std::string("qv_pq_encode_gpu: ") + cudaGetErrorString(e));
  for (int64_t s0 = 0; s0 < n; s0 += slice) {
    const int64_t cnt = std::min(slice, n - s0);
    e = cudaMemcpy(d_base, static_cast<const uint8_t*>(base) + static_cast<size_t>(s0) * dim * esize,
                   static_cast<size_t>(cnt) * dim * esize, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return fail(QV_ERR_CUDA, std::string("qv_pq_encode_gpu: ") + cudaGetErrorString(e));
    const dim3 grid(static_cast<unsigned>((cnt + 255) / 256), static_cast<unsigned>(M));
    pq_encode_kernel<<<grid, 256, smem>>>(d_base, cnt, static_cast<int32_t>(dim), dtype, d_piv, d_cen, d_off, M,
                                          d_codes);
    e = cudaGetLastError();
    if (e == cudaSuccess)
      e = cudaMemcpy(codes + static_cast<size_t>(s0) * M, d_codes, static_cast<size_t>(cnt) * M,
                     cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail(QV_ERR_CUDA, std::string("qv_pq_encode_gpu: ") + cudaGetErrorString(e));
  }
  return QV_OK;
}
