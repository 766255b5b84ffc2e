// synth_common.h -- the seeded generator of the synthetic workloads, shared by
// the host builder (index_build.cpp) and the GPU one (build_gpu.cu).  Every
// value is a pure function of (seed, stream, index) built from 64-bit integer
// hashing and IEEE double add / multiply / divide / sqrt, so the host and the
// GPU produce the same bits.
#pragma once

#include <cmath>
#include <cstdint>
#include <vector>

#include "quiver_b200.h"

#if defined(__CUDACC__)
#define QV_HD __host__ __device__
#else
#define QV_HD
#endif

namespace qv_synth {

QV_HD inline uint64_t mix64(uint64_t z) {  // splitmix64 finaliser
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}
QV_HD inline uint64_t hash3(uint64_t seed, uint64_t stream, uint64_t idx) {
  return mix64(mix64(seed * 0x9e3779b97f4a7c15ULL + stream) ^ (idx * 0xd1b54a32d192ed03ULL + 0x632be59bd9b4e019ULL));
}
// (h >> 11) * 2^-53: the product is exact, so no rounding choice is involved.
QV_HD inline double u01(uint64_t h) { return static_cast<double>(h >> 11) * (1.0 / 9007199254740992.0); }
// Irwin-Hall(12) - 6: mean 0, variance 1.
QV_HD inline double gauss(uint64_t seed, uint64_t stream, uint64_t idx) {
  double s = 0.0;
  for (int t = 0; t < 12; ++t) s = s + u01(hash3(seed, stream, idx * 12 + t));
  return s - 6.0;
}

constexpr uint64_t kCenterStream = 1000, kAssignStream = 2000, kNoiseStream = 3000;

inline std::vector<double> mixture_centers(uint64_t seed, int64_t k, int64_t dim, int32_t dtype) {
  std::vector<double> c(static_cast<size_t>(k * dim));
  for (int64_t i = 0; i < k; ++i) {
    double* row = c.data() + i * dim;
    if (dtype == QV_FLOAT) {
      double nrm = 0.0;
      for (int64_t d = 0; d < dim; ++d) {
        row[d] = gauss(seed, kCenterStream, static_cast<uint64_t>(i * dim + d));
        nrm = nrm + row[d] * row[d];
      }
      nrm = std::sqrt(nrm);
      for (int64_t d = 0; d < dim; ++d) row[d] = row[d] / nrm;
    } else {
      for (int64_t d = 0; d < dim; ++d) row[d] = u01(hash3(seed, kCenterStream, i * dim + d)) * 255.0;
    }
  }
  return c;
}

}  // namespace qv_synth
