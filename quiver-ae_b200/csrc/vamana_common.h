// vamana_common.h -- host-side pieces of the Vamana construction that the
// OpenMP builder (index_build.cpp) and the GPU builder (vamana_gpu.cu) share,
// so both insert the same points in the same batches from the same medoid.
//
// Construction (Subramanya et al., "DiskANN", NeurIPS 2019): greedy search
// from the medoid with list size L, RobustPrune(p, V, alpha, R) over at most
// kMaxOcclusion candidates, reverse edges re-pruned when a list overflows.  Points are inserted in batches in
// a seeded order; the searches of a batch run on the graph as it stood when
// the batch began.  Pass 0 (of two) uses alpha = 1 and batches that double
// from 1; later passes use the final alpha and full batches.
#pragma once

#include <algorithm>
#include <cstdint>
#include <numeric>
#include <vector>

#include "synth_common.h"

namespace qv_vamana {

using qv_synth::hash3;

// The point nearest the mean (sums in double, in index order; first minimum).
template <typename T>
int64_t medoid(const T* data, int64_t n, int64_t dim) {
  std::vector<double> mean(static_cast<size_t>(dim), 0.0);
  for (int64_t i = 0; i < n; ++i)
    for (int64_t d = 0; d < dim; ++d) mean[d] += static_cast<double>(data[i * dim + d]);
  for (auto& m : mean) m /= static_cast<double>(n);
  double best = 1e300;
  int64_t med = 0;
  for (int64_t i = 0; i < n; ++i) {
    double s = 0.0;
    for (int64_t d = 0; d < dim; ++d) {
      const double t = static_cast<double>(data[i * dim + d]) - mean[d];
      s += t * t;
    }
    if (s < best) {
      best = s;
      med = i;
    }
  }
  return med;
}

// Insertion order: seeded Fisher-Yates.
inline std::vector<int64_t> insertion_order(uint64_t seed, int64_t n) {
  std::vector<int64_t> perm(static_cast<size_t>(n));
  std::iota(perm.begin(), perm.end(), 0);
  for (int64_t i = n - 1; i > 0; --i) {
    const int64_t j = static_cast<int64_t>(hash3(seed, 77, static_cast<uint64_t>(i)) % static_cast<uint64_t>(i + 1));
    std::swap(perm[i], perm[j]);
  }
  return perm;
}

// Batches grow to 2 % of n, at most 2^21 points (for n <= 1M that is at
// most 20,000 points).
inline int64_t max_batch(int64_t n) { return std::max<int64_t>(1, std::min<int64_t>(n / 50, int64_t(1) << 21)); }

// RobustPrune keeps at most this many of its candidates, nearest first (after removing the point itself and
// repeated ids), before the occlusion loop: DiskANN's candidate cap for pruning (its max_occlusion_size,
// default 750).  Only a reverse-edge pool of a node that many new points link to in one batch reaches it.
constexpr int32_t kMaxOcclusion = 750;

inline float pass_alpha(int32_t pass, int32_t passes, float alpha_final) {
  return (passes > 1 && pass == 0) ? 1.0f : alpha_final;
}

inline int64_t first_batch(int32_t pass, int64_t n) { return pass == 0 ? 1 : max_batch(n); }

}  // namespace qv_vamana
