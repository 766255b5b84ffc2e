// index_build.cpp -- Vamana graph, PQ tables, synthetic mixtures and exact
// ground truth on the host (OpenMP).  See include/quiver_b200_build.h.
//
// The graph follows the published Vamana construction (Subramanya et al.,
// "DiskANN", NeurIPS 2019): greedy search from the medoid with list size L,
// RobustPrune(p, V, alpha, R), reverse edges re-pruned when a list
// overflows.  Points are inserted in batches whose searches run in parallel
// on the graph as it stood when the batch began, so the result does not
// depend on the thread count.
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

#include "quiver_b200.h"
#include "quiver_b200_build.h"
#include "synth_common.h"
#include "vamana_common.h"

namespace {

thread_local std::string g_err;

// ------------------------------------------------------------ generator --

using qv_vamana::hash3;
using qv_synth::gauss;
using qv_synth::mixture_centers;
using qv_synth::kAssignStream;
using qv_synth::kNoiseStream;

// ------------------------------------------------------------ distances --

template <typename T>
struct Dist;

template <>
struct Dist<uint8_t> {
  static float l2(const uint8_t* a, const uint8_t* b, int64_t dim) {
    int32_t s = 0;
    for (int64_t i = 0; i < dim; ++i) {
      const int32_t d = int32_t(a[i]) - int32_t(b[i]);
      s += d * d;
    }
    return static_cast<float>(s);
  }
};
template <>
struct Dist<int8_t> {
  static float l2(const int8_t* a, const int8_t* b, int64_t dim) {
    int32_t s = 0;
    for (int64_t i = 0; i < dim; ++i) {
      const int32_t d = int32_t(a[i]) - int32_t(b[i]);
      s += d * d;
    }
    return static_cast<float>(s);
  }
};
template <>
struct Dist<float> {
  static float l2(const float* a, const float* b, int64_t dim) {
    float s = 0.f;
    for (int64_t i = 0; i < dim; ++i) {
      const float d = a[i] - b[i];
      s += d * d;
    }
    return s;
  }
};

// ------------------------------------------------------------- Vamana --

struct Cand {
  float d;
  int32_t id;
  bool operator<(const Cand& o) const { return d < o.d || (d == o.d && id < o.id); }
};

template <typename T>
struct Vamana {
  const T* data;
  int64_t n, dim;
  int32_t R, L;
  std::vector<int32_t>& graph;   // n x R
  std::vector<int32_t>& degree;  // n
  int64_t medoid = 0;

  const T* vec(int64_t i) const { return data + i * dim; }
  float dist(int64_t a, int64_t b) const { return Dist<T>::l2(vec(a), vec(b), dim); }

  struct Scratch {
    std::vector<uint32_t> seen;
    uint32_t epoch = 0;
    std::vector<Cand> list;
    std::vector<uint8_t> expanded_flag;
    std::vector<Cand> expanded;
    std::vector<Cand> pool;
    std::vector<uint8_t> pruned;
  };

  void greedy(int64_t q, Scratch& s) const {
    if (++s.epoch == 0) {
      std::fill(s.seen.begin(), s.seen.end(), 0u);
      s.epoch = 1;
    }
    s.list.clear();
    s.expanded_flag.clear();
    s.expanded.clear();
    s.list.push_back({dist(q, medoid), static_cast<int32_t>(medoid)});
    s.expanded_flag.push_back(0);
    s.seen[medoid] = s.epoch;
    while (true) {
      size_t k = 0;
      while (k < s.list.size() && s.expanded_flag[k]) ++k;
      if (k == s.list.size()) break;
      s.expanded_flag[k] = 1;
      const Cand cur = s.list[k];
      s.expanded.push_back(cur);
      const int32_t* nb = graph.data() + cur.id * int64_t(R);
      for (int32_t t = 0; t < degree[cur.id]; ++t) {
        const int32_t v = nb[t];
        if (s.seen[v] == s.epoch) continue;
        s.seen[v] = s.epoch;
        const Cand c{dist(q, v), v};
        if (static_cast<int32_t>(s.list.size()) == L && !(c < s.list.back())) continue;
        const auto it = std::upper_bound(s.list.begin(), s.list.end(), c);
        const size_t pos = static_cast<size_t>(it - s.list.begin());
        s.list.insert(it, c);
        s.expanded_flag.insert(s.expanded_flag.begin() + pos, 0);
        if (static_cast<int32_t>(s.list.size()) > L) {
          s.list.pop_back();
          s.expanded_flag.pop_back();
        }
      }
    }
  }

  // RobustPrune: pool holds (d(p, c), c); result written to out (<= R).
  void robust_prune(int64_t p, std::vector<Cand>& pool, float alpha, Scratch& s,
                    std::vector<int32_t>& out) const {
    std::sort(pool.begin(), pool.end());
    size_t w = 0;
    for (size_t i = 0; i < pool.size(); ++i) {
      if (pool[i].id == p) continue;
      if (w > 0 && pool[w - 1].id == pool[i].id) continue;
      pool[w++] = pool[i];
    }
    pool.resize(std::min<size_t>(w, static_cast<size_t>(qv_vamana::kMaxOcclusion)));
    s.pruned.assign(pool.size(), 0);
    out.clear();
    for (size_t i = 0; i < pool.size() && static_cast<int32_t>(out.size()) < R; ++i) {
      if (s.pruned[i]) continue;
      out.push_back(pool[i].id);
      for (size_t j = i + 1; j < pool.size(); ++j) {
        if (s.pruned[j]) continue;
        if (alpha * dist(pool[i].id, pool[j].id) < pool[j].d) s.pruned[j] = 1;
      }
    }
  }

  void run(float alpha_final, int32_t passes, uint64_t seed, int nthreads) {
    medoid = qv_vamana::medoid(data, n, dim);
    std::fill(degree.begin(), degree.end(), 0);
    std::fill(graph.begin(), graph.end(), -1);
    const std::vector<int64_t> perm = qv_vamana::insertion_order(seed, n);
    const int64_t max_batch = qv_vamana::max_batch(n);
    std::vector<Scratch> scratch(static_cast<size_t>(nthreads));
    for (auto& s : scratch) s.seen.assign(static_cast<size_t>(n), 0u);
    std::vector<std::vector<int32_t>> newlist;
    for (int32_t pass = 0; pass < passes; ++pass) {
      const float alpha = qv_vamana::pass_alpha(pass, passes, alpha_final);
      int64_t start = 0;
      int64_t bsize = qv_vamana::first_batch(pass, n);
      while (start < n) {
        const int64_t end = std::min(n, start + bsize);
        const int64_t cnt = end - start;
        newlist.assign(static_cast<size_t>(cnt), {});
#pragma omp parallel for schedule(dynamic, 4) num_threads(nthreads)
        for (int64_t b = 0; b < cnt; ++b) {
          Scratch& s = scratch[omp_get_thread_num()];
          const int64_t p = perm[start + b];
          greedy(p, s);
          s.pool = s.expanded;
          const int32_t* nb = graph.data() + p * int64_t(R);
          for (int32_t t = 0; t < degree[p]; ++t) s.pool.push_back({dist(p, nb[t]), nb[t]});
          robust_prune(p, s.pool, alpha, s, newlist[b]);
        }
        // install the new out-lists
        std::vector<std::pair<int32_t, int32_t>> rev;
        for (int64_t b = 0; b < cnt; ++b) {
          const int64_t p = perm[start + b];
          const auto& nl = newlist[b];
          degree[p] = static_cast<int32_t>(nl.size());
          std::copy(nl.begin(), nl.end(), graph.begin() + p * int64_t(R));
          std::fill(graph.begin() + p * int64_t(R) + nl.size(), graph.begin() + (p + 1) * int64_t(R), -1);
          for (int32_t j : nl) rev.push_back({j, static_cast<int32_t>(p)});
        }
        std::sort(rev.begin(), rev.end());
        std::vector<size_t> heads;
        for (size_t i = 0; i < rev.size(); ++i)
          if (i == 0 || rev[i].first != rev[i - 1].first) heads.push_back(i);
        heads.push_back(rev.size());
        const int64_t groups = static_cast<int64_t>(heads.size()) - 1;
#pragma omp parallel for schedule(dynamic, 16) num_threads(nthreads)
        for (int64_t g = 0; g < groups; ++g) {
          Scratch& s = scratch[omp_get_thread_num()];
          const int32_t j = rev[heads[g]].first;
          int32_t* nb = graph.data() + j * int64_t(R);
          int32_t deg = degree[j];
          std::vector<int32_t> add;
          for (size_t i = heads[g]; i < heads[g + 1]; ++i) {
            const int32_t p = rev[i].second;
            if (p == j) continue;
            bool present = false;
            for (int32_t t = 0; t < deg && !present; ++t) present = nb[t] == p;
            if (!present) add.push_back(p);
          }
          if (deg + static_cast<int32_t>(add.size()) <= R) {
            for (int32_t p : add) nb[deg++] = p;
            degree[j] = deg;
          } else {
            s.pool.clear();
            for (int32_t t = 0; t < deg; ++t) s.pool.push_back({dist(j, nb[t]), nb[t]});
            for (int32_t p : add) s.pool.push_back({dist(j, p), p});
            std::vector<int32_t> out;
            robust_prune(j, s.pool, alpha, s, out);
            std::copy(out.begin(), out.end(), nb);
            for (size_t t = out.size(); t < static_cast<size_t>(R); ++t) nb[t] = -1;
            degree[j] = static_cast<int32_t>(out.size());
          }
        }
        start = end;
        bsize = std::min(max_batch, bsize * 2);
      }
    }
  }
};

template <typename T>
void vamana_t(const void* base, int64_t n, int64_t dim, int32_t R, int32_t L, float alpha, int32_t passes,
              uint64_t seed, int nthreads, int32_t* graph, int32_t* degree, int64_t* medoid) {
  std::vector<int32_t> g(static_cast<size_t>(n * R)), deg(static_cast<size_t>(n));
  Vamana<T> v{static_cast<const T*>(base), n, dim, R, L, g, deg};
  v.run(alpha, passes, seed, nthreads);
  std::copy(g.begin(), g.end(), graph);
  std::copy(deg.begin(), deg.end(), degree);
  *medoid = v.medoid;
}

// ---------------------------------------------------------------- PQ ----

inline float elem(const void* base, int32_t dtype, int64_t i) {
  if (dtype == QV_UINT8) return static_cast<float>(static_cast<const uint8_t*>(base)[i]);
  if (dtype == QV_INT8) return static_cast<float>(static_cast<const int8_t*>(base)[i]);
  return static_cast<const float*>(base)[i];
}

void chunk_layout(int64_t dim, int32_t M, int32_t* off) {
  off[0] = 0;
  for (int32_t c = 0; c < M; ++c)
    off[c + 1] = off[c] + static_cast<int32_t>(dim / M + (c < dim % M ? 1 : 0));
}

int resolve_threads(int32_t t) { return t > 0 ? t : omp_get_max_threads(); }

}  // namespace

extern "C" {

const char* qvb_last_error(void) { return g_err.c_str(); }

int qvb_synth_mixture(uint64_t seed, int32_t stream, int64_t row0, int64_t n, int64_t dim, int64_t n_centers,
                      double sigma, int32_t dtype, void* out, int32_t nthreads) {
  if (!out || n < 0 || dim <= 0 || n_centers <= 0 || (dtype != QV_UINT8 && dtype != QV_FLOAT)) {
    g_err = "qvb_synth_mixture: invalid argument";
    return QV_ERR_INVALID_ARG;
  }
  const std::vector<double> centers = mixture_centers(seed, n_centers, dim, dtype);
  const int nt = resolve_threads(nthreads);
#pragma omp parallel num_threads(nt)
  {
    std::vector<double> x(static_cast<size_t>(dim));
#pragma omp for schedule(static)
    for (int64_t r = 0; r < n; ++r) {
      const uint64_t row = static_cast<uint64_t>(row0 + r);
      const int64_t c = static_cast<int64_t>(hash3(seed, kAssignStream + stream, row) % static_cast<uint64_t>(n_centers));
      const double* cen = centers.data() + c * dim;
      for (int64_t d = 0; d < dim; ++d)
        x[d] = cen[d] + sigma * gauss(seed, kNoiseStream + stream, row * static_cast<uint64_t>(dim) + d);
      if (dtype == QV_UINT8) {
        uint8_t* o = static_cast<uint8_t*>(out) + r * dim;
        for (int64_t d = 0; d < dim; ++d) {
          double v = std::rint(x[d]);
          v = v < 0.0 ? 0.0 : (v > 255.0 ? 255.0 : v);
          o[d] = static_cast<uint8_t>(v);
        }
      } else {
        double nrm = 0.0;
        for (int64_t d = 0; d < dim; ++d) nrm = nrm + x[d] * x[d];
        nrm = std::sqrt(nrm);
        float* o = static_cast<float*>(out) + r * dim;
        for (int64_t d = 0; d < dim; ++d) o[d] = static_cast<float>(x[d] / nrm);
      }
    }
  }
  return QV_OK;
}

int qvb_ground_truth(const void* base, int64_t n, const void* queries, int64_t nq, int64_t dim, int32_t dtype,
                     int32_t k, int32_t* ids, float* dists, int32_t nthreads) {
  if (!base || !queries || !ids || !dists || k <= 0 || k > n) {
    g_err = "qvb_ground_truth: invalid argument";
    return QV_ERR_INVALID_ARG;
  }
  const int nt = resolve_threads(nthreads);
#pragma omp parallel num_threads(nt)
  {
    std::vector<std::pair<double, int32_t>> all(static_cast<size_t>(n));
#pragma omp for schedule(dynamic, 4)
    for (int64_t q = 0; q < nq; ++q) {
      for (int64_t i = 0; i < n; ++i) {
        double s = 0.0;
        for (int64_t d = 0; d < dim; ++d) {
          const double t = static_cast<double>(elem(queries, dtype, q * dim + d)) -
                           static_cast<double>(elem(base, dtype, i * dim + d));
          s += t * t;
        }
        all[i] = {s, static_cast<int32_t>(i)};
      }
      std::partial_sort(all.begin(), all.begin() + k, all.end());
      for (int32_t j = 0; j < k; ++j) {
        ids[q * k + j] = all[j].second;
        dists[q * k + j] = static_cast<float>(all[j].first);
      }
    }
  }
  return QV_OK;
}

int qvb_vamana(const void* base, int64_t n, int64_t dim, int32_t dtype, int32_t R, int32_t L, float alpha,
               int32_t passes, uint64_t seed, int32_t nthreads, int32_t* graph, int32_t* degree,
               int64_t* medoid) {
  if (!base || !graph || !degree || !medoid || n <= 0 || R <= 0 || L <= 0 || passes <= 0) {
    g_err = "qvb_vamana: invalid argument";
    return QV_ERR_INVALID_ARG;
  }
  const int nt = resolve_threads(nthreads);
  if (dtype == QV_UINT8)
    vamana_t<uint8_t>(base, n, dim, R, L, alpha, passes, seed, nt, graph, degree, medoid);
  else if (dtype == QV_INT8)
    vamana_t<int8_t>(base, n, dim, R, L, alpha, passes, seed, nt, graph, degree, medoid);
  else
    vamana_t<float>(base, n, dim, R, L, alpha, passes, seed, nt, graph, degree, medoid);
  return QV_OK;
}

int qvb_pq_train(const void* base, int64_t n, int64_t dim, int32_t dtype, int32_t M, int64_t sample,
                 int32_t iters, uint64_t seed, int32_t nthreads, float* pivots, float* centroid,
                 int32_t* chunk_offsets) {
  if (!base || !pivots || !centroid || !chunk_offsets || n <= 0 || M <= 0 || M > dim) {
    g_err = "qvb_pq_train: invalid argument";
    return QV_ERR_INVALID_ARG;
  }
  const int nt = resolve_threads(nthreads);
  chunk_layout(dim, M, chunk_offsets);
  // seeded sample without replacement (partial Fisher-Yates)
  const int64_t ns = std::min(n, std::max<int64_t>(sample, 256));
  std::vector<int64_t> idx(static_cast<size_t>(n));
  std::iota(idx.begin(), idx.end(), 0);
  for (int64_t i = 0; i < ns; ++i) {
    const int64_t j = i + static_cast<int64_t>(hash3(seed, 91, static_cast<uint64_t>(i)) % static_cast<uint64_t>(n - i));
    std::swap(idx[i], idx[j]);
  }
  std::vector<double> mean(static_cast<size_t>(dim), 0.0);
  for (int64_t s = 0; s < ns; ++s)
    for (int64_t d = 0; d < dim; ++d) mean[d] += elem(base, dtype, idx[s] * dim + d);
  for (int64_t d = 0; d < dim; ++d) centroid[d] = static_cast<float>(mean[d] / static_cast<double>(ns));
  std::vector<float> X(static_cast<size_t>(ns * dim));
  for (int64_t s = 0; s < ns; ++s)
    for (int64_t d = 0; d < dim; ++d) X[s * dim + d] = elem(base, dtype, idx[s] * dim + d) - centroid[d];
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
  for (int32_t c = 0; c < M; ++c) {
    const int32_t lo = chunk_offsets[c], w = chunk_offsets[c + 1] - lo;
    std::vector<float> C(static_cast<size_t>(256 * w));
    for (int j = 0; j < 256; ++j)
      for (int32_t t = 0; t < w; ++t) C[j * w + t] = X[(j % ns) * dim + lo + t];
    std::vector<int32_t> assign(static_cast<size_t>(ns));
    std::vector<double> acc(static_cast<size_t>(256 * w));
    std::vector<int64_t> count(256);
    for (int32_t it = 0; it < iters; ++it) {
      for (int64_t s = 0; s < ns; ++s) {
        const float* x = X.data() + s * dim + lo;
        float best = 3.4e38f;
        int32_t bj = 0;
        for (int j = 0; j < 256; ++j) {
          float dd = 0.f;
          for (int32_t t = 0; t < w; ++t) {
            const float u = x[t] - C[j * w + t];
            dd += u * u;
          }
          if (dd < best) { best = dd; bj = j; }
        }
        assign[s] = bj;
      }
      std::fill(acc.begin(), acc.end(), 0.0);
      std::fill(count.begin(), count.end(), 0);
      for (int64_t s = 0; s < ns; ++s) {
        ++count[assign[s]];
        for (int32_t t = 0; t < w; ++t) acc[assign[s] * w + t] += X[s * dim + lo + t];
      }
      for (int j = 0; j < 256; ++j)
        if (count[j] > 0)
          for (int32_t t = 0; t < w; ++t) C[j * w + t] = static_cast<float>(acc[j * w + t] / count[j]);
    }
    for (int j = 0; j < 256; ++j)
      for (int32_t t = 0; t < w; ++t) pivots[j * dim + lo + t] = C[j * w + t];
  }
  return QV_OK;
}

int qvb_pq_encode(const void* base, int64_t n, int64_t dim, int32_t dtype, int32_t M, const float* pivots,
                  const float* centroid, const int32_t* chunk_offsets, int32_t nthreads, uint8_t* codes) {
  if (!base || !pivots || !centroid || !chunk_offsets || !codes) {
    g_err = "qvb_pq_encode: invalid argument";
    return QV_ERR_INVALID_ARG;
  }
  const int nt = resolve_threads(nthreads);
#pragma omp parallel num_threads(nt)
  {
    std::vector<float> r(static_cast<size_t>(dim));
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      for (int64_t d = 0; d < dim; ++d) r[d] = elem(base, dtype, i * dim + d) - centroid[d];
      for (int32_t c = 0; c < M; ++c) {
        const int32_t lo = chunk_offsets[c], hi = chunk_offsets[c + 1];
        float best = 3.4e38f;
        int32_t bj = 0;
        for (int j = 0; j < 256; ++j) {
          float dd = 0.f;
          for (int32_t t = lo; t < hi; ++t) {
            const float u = r[t] - pivots[j * dim + t];
            dd += u * u;
          }
          if (dd < best) { best = dd; bj = j; }
        }
        codes[i * M + c] = static_cast<uint8_t>(bj);
      }
    }
  }
  return QV_OK;
}

}  // extern "C"
