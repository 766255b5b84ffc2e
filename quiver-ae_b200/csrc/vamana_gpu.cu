// vamana_gpu.cu -- the batched Vamana construction of index_build.cpp, run on
// the GPU step for step, so both builders produce the same graph.
//
// Per batch of points (the schedule, insertion order and medoid come from
// vamana_common.h):
//  1. search_prune_kernel, one warp per point: greedy search from the medoid
//     with list size L on the graph as the batch found it (candidates
//     ordered by (distance, id); a per-search hash set marks seen nodes),
//     then RobustPrune(p, expanded + current out-list, alpha, R);
//  2. install_kernel: the new out-lists replace the old ones and every new
//     edge p -> j is emitted as the key (j << 32 | p);
//  3. the keys are radix-sorted (CUB), grouping them by j with p ascending;
//  4. reverse_kernel, one warp per group: the p's not already in j's list
//     are appended in order when they fit, else j's list is re-pruned from
//     old list + new p's.
// Distances are the host builder's: integer sums of squared differences for
// 8-bit data (exact, any order), and for fp32 a sequential sum of separately
// rounded products (the host builds with -ffp-contract=off), so every
// comparison -- list order, prune test -- gives the same answer.
#include <cuda_runtime.h>

#include <cub/cub.cuh>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "quiver_b200.h"
#include "vamana_common.h"

namespace qv {
void set_last_error(const std::string& m);
}

namespace {

constexpr int kWarps = 4;  // warps per CTA
constexpr int kMaxR = 128;
constexpr int kMaxL = 256;
constexpr int kExpCap = 2048;                // expansions recorded per search
constexpr int kPoolCap = kExpCap + kMaxR;    // expanded + current out-list
constexpr int kSeenCap = 32768;              // hash-set entries per search (power of 2)
constexpr int kChunk = 32768;                // searches per launch (bounds the scratch)
constexpr unsigned long long kNoKey = ~0ull;

enum BuildError : int32_t { kBuildOk = 0, kErrExpansions = 1, kErrSeen = 2 };

struct VArgs {
  const void* data;
  int64_t n;
  int32_t dim, R, L, Lpad;
  int32_t* graph;   // [n x R], -1 padded
  int32_t* degree;  // [n]
  const int64_t* perm;
  int64_t medoid;
  int32_t* newlist;  // [batch x R]: the batch's new out-lists, installed after all its searches
  int32_t* newdeg;   // [batch]
  unsigned long long* seen;  // [kChunk x kSeenCap]
  float* pool_d;             // [kChunk x 2 kPoolCap]
  int32_t* pool_i;
  int32_t* err;  // [2]: code, detail
};

// ------------------------------------------------------------- distances --

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T>
struct VDist;

template <>
struct VDist<uint8_t> {
  __device__ static float l2(const uint8_t* a, const uint8_t* b, int dim) {
    uint32_t s = 0;
    int i = 0;
    if (aligned16(a) && aligned16(b))
      for (; i + 16 <= dim; i += 16) {
        const uint4 x = *reinterpret_cast<const uint4*>(a + i), y = *reinterpret_cast<const uint4*>(b + i);
        uint32_t d;
        d = __vabsdiffu4(x.x, y.x); s = __dp4a(d, d, s);
        d = __vabsdiffu4(x.y, y.y); s = __dp4a(d, d, s);
        d = __vabsdiffu4(x.z, y.z); s = __dp4a(d, d, s);
        d = __vabsdiffu4(x.w, y.w); s = __dp4a(d, d, s);
      }
    for (; i < dim; ++i) {
      const int32_t d = int32_t(a[i]) - int32_t(b[i]);
      s += static_cast<uint32_t>(d * d);
    }
    return __int2float_rn(static_cast<int32_t>(s));
  }
};

template <>
struct VDist<int8_t> {
  __device__ static float l2(const int8_t* a, const int8_t* b, int dim) {
    uint32_t s = 0;
    int i = 0;
    if (aligned16(a) && aligned16(b))
      for (; i + 16 <= dim; i += 16) {
        const uint4 x = *reinterpret_cast<const uint4*>(a + i), y = *reinterpret_cast<const uint4*>(b + i);
        uint32_t d;
        d = __vabsdiffs4(x.x, y.x); s = __dp4a(d, d, s);
        d = __vabsdiffs4(x.y, y.y); s = __dp4a(d, d, s);
        d = __vabsdiffs4(x.z, y.z); s = __dp4a(d, d, s);
        d = __vabsdiffs4(x.w, y.w); s = __dp4a(d, d, s);
      }
    for (; i < dim; ++i) {
      const int32_t d = int32_t(a[i]) - int32_t(b[i]);
      s += static_cast<uint32_t>(d * d);
    }
    return __int2float_rn(static_cast<int32_t>(s));
  }
};

template <>
struct VDist<float> {
  __device__ static float l2(const float* a, const float* b, int dim) {
    float s = 0.f;
    int i = 0;
    if (aligned16(a) && aligned16(b))
      for (; i + 4 <= dim; i += 4) {
        const float4 x = *reinterpret_cast<const float4*>(a + i), y = *reinterpret_cast<const float4*>(b + i);
        float d;
        d = __fsub_rn(x.x, y.x); s = __fadd_rn(s, __fmul_rn(d, d));
        d = __fsub_rn(x.y, y.y); s = __fadd_rn(s, __fmul_rn(d, d));
        d = __fsub_rn(x.z, y.z); s = __fadd_rn(s, __fmul_rn(d, d));
        d = __fsub_rn(x.w, y.w); s = __fadd_rn(s, __fmul_rn(d, d));
      }
    for (; i < dim; ++i) {
      const float d = __fsub_rn(a[i], b[i]);
      s = __fadd_rn(s, __fmul_rn(d, d));
    }
    return s;
  }
};

// (d, id) order of the host's Cand
__device__ __forceinline__ bool cand_less(float da, int32_t ia, float db, int32_t ib) {
  return da < db || (da == db && ia < ib);
}

__device__ __forceinline__ void set_error(int32_t* err, int32_t code, int32_t detail) {
  if (atomicCAS(err, 0, code) == 0) err[1] = detail;
}

// Inserts id into this search's set; true when it was not there yet.
__device__ bool seen_insert(unsigned long long* tab, uint32_t tag, int32_t id, int32_t* err) {
  const unsigned long long mine = (static_cast<unsigned long long>(tag) << 32) | static_cast<uint32_t>(id);
  uint32_t h = (static_cast<uint32_t>(id) * 2654435761u) & (kSeenCap - 1);
  for (int probe = 0; probe < kSeenCap; ++probe) {
    const unsigned long long e = __ldcg(tab + h);
    if (e == mine) return false;
    if (static_cast<uint32_t>(e >> 32) != tag) {  // empty or left by an earlier search
      const unsigned long long prev = atomicCAS(tab + h, e, mine);
      if (prev == e) return true;
      if (prev == mine) return false;
    }
    h = (h + 1) & (kSeenCap - 1);
  }
  set_error(err, kErrSeen, id);
  return false;
}

// RobustPrune(p, pool, alpha, R) of index_build.cpp: sort the pool by (d, id),
// drop p and repeats, keep the nearest kMaxOcclusion, then take the nearest
// remaining candidate and discard every later one it covers
// (alpha * d(c, c') < d(p, c')).  pool_d/pool_i hold
// P entries; sd/si are scratch of the same size; returns the out-degree.
template <typename T>
__device__ int robust_prune(const VArgs& a, int64_t p, float* pd, int32_t* pi, int P, float* sd, int32_t* si,
                            float alpha, int32_t* out, uint32_t* pruned, int lane) {
  const T* data = static_cast<const T*>(a.data);
  for (int i = lane; i < P; i += 32) {
    const float d = pd[i];
    const int32_t id = pi[i];
    int r = 0;
    for (int j = 0; j < P; ++j) {
      const float dj = pd[j];
      const int32_t ij = pi[j];
      r += cand_less(dj, ij, d, id) || (dj == d && ij == id && j < i);
    }
    sd[r] = d;
    si[r] = id;
  }
  __syncwarp();
  int w = 0;
  for (int base = 0; base < P; base += 32) {
    const int i = base + lane;
    const bool keep = i < P && si[i] != p && (i == 0 || si[i - 1] != si[i]);
    const uint32_t m = __ballot_sync(0xffffffffu, keep);
    if (keep) {
      const int at = w + __popc(m & ((1u << lane) - 1u));
      pd[at] = sd[i];
      pi[at] = si[i];
    }
    w += __popc(m);
  }
  w = min(w, qv_vamana::kMaxOcclusion);  // the candidate cap, nearest first
  for (int k = lane; k < (w + 31) / 32; k += 32) pruned[k] = 0u;
  __syncwarp();
  int o = 0;
  for (int i = 0; i < w; ++i) {
    if ((pruned[i >> 5] >> (i & 31)) & 1u) continue;
    if (lane == 0) out[o] = pi[i];
    ++o;
    if (o == a.R) break;
    const T* vi = data + static_cast<int64_t>(pi[i]) * a.dim;
    for (int j = i + 1 + lane; j < w; j += 32) {
      if ((pruned[j >> 5] >> (j & 31)) & 1u) continue;
      if (__fmul_rn(alpha, VDist<T>::l2(vi, data + static_cast<int64_t>(pi[j]) * a.dim, a.dim)) < pd[j])
        atomicOr(&pruned[j >> 5], 1u << (j & 31));
    }
    __syncwarp();
  }
  __syncwarp();
  return o;
}

// Shared memory of one warp.
struct WarpSmem {
  float* ld[2];
  int32_t* li[2];
  uint8_t* lf[2];
  float* cd;
  int32_t* ci;
  float* cd2;
  int32_t* ci2;
  uint32_t* pruned;
  uint8_t* qv;
};

__host__ __device__ inline size_t warp_smem_bytes(int Lpad, int dim, int esize) {
  const size_t list = 2 * static_cast<size_t>(Lpad) * (4 + 4 + 1);
  const size_t cands = 4 * static_cast<size_t>(kMaxR) * 4;
  const size_t pr = (kPoolCap + 31) / 32 * 4;
  const size_t q = static_cast<size_t>(dim) * esize;
  return (list + 15) / 16 * 16 + cands + (pr + 15) / 16 * 16 + (q + 15) / 16 * 16;
}

__device__ WarpSmem carve(uint8_t* base, int Lpad) {
  WarpSmem s;
  s.ld[0] = reinterpret_cast<float*>(base);
  s.ld[1] = s.ld[0] + Lpad;
  s.li[0] = reinterpret_cast<int32_t*>(s.ld[1] + Lpad);
  s.li[1] = s.li[0] + Lpad;
  s.lf[0] = reinterpret_cast<uint8_t*>(s.li[1] + Lpad);
  s.lf[1] = s.lf[0] + Lpad;
  uint8_t* q = base + (2 * static_cast<size_t>(Lpad) * 9 + 15) / 16 * 16;
  s.cd = reinterpret_cast<float*>(q);
  s.ci = reinterpret_cast<int32_t*>(s.cd + kMaxR);
  s.cd2 = reinterpret_cast<float*>(s.ci + kMaxR);
  s.ci2 = reinterpret_cast<int32_t*>(s.cd2 + kMaxR);
  s.pruned = reinterpret_cast<uint32_t*>(s.ci2 + kMaxR);
  s.qv = reinterpret_cast<uint8_t*>(s.pruned) + ((kPoolCap + 31) / 32 * 4 + 15) / 16 * 16;
  return s;
}

// ------------------------------------------------- 1. search and prune --

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) search_prune_kernel(const VArgs a, int64_t first, int cnt,
                                                                   int64_t row0, uint32_t tag0, float alpha) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int w = blockIdx.x * kWarps + wib;
  if (w >= cnt) return;
  const size_t wbytes = warp_smem_bytes(a.Lpad, a.dim, sizeof(T));
  WarpSmem s = carve(smem + wib * wbytes, a.Lpad);
  const T* data = static_cast<const T*>(a.data);
  const int64_t p = a.perm[first + w];
  const uint32_t tag = tag0 + static_cast<uint32_t>(w);
  unsigned long long* seen = a.seen + static_cast<size_t>(w) * kSeenCap;
  float* exp_d = a.pool_d + static_cast<size_t>(w) * 2 * kPoolCap;
  int32_t* exp_i = a.pool_i + static_cast<size_t>(w) * 2 * kPoolCap;
  T* qv = reinterpret_cast<T*>(s.qv);
  for (int d = lane; d < a.dim; d += 32) qv[d] = data[p * a.dim + d];
  __syncwarp();
  if (lane == 0) {
    seen_insert(seen, tag, static_cast<int32_t>(a.medoid), a.err);
    s.ld[0][0] = VDist<T>::l2(qv, data + a.medoid * a.dim, a.dim);
    s.li[0][0] = static_cast<int32_t>(a.medoid);
    s.lf[0][0] = 0;
  }
  __syncwarp();
  int cur = 0, size = 1, nexp = 0;
  while (true) {
    int k = -1;
    for (int base = 0; base < size && k < 0; base += 32) {
      const int idx = base + lane;
      const uint32_t m = __ballot_sync(0xffffffffu, idx < size && s.lf[cur][idx] == 0);
      if (m) k = base + __ffs(m) - 1;
    }
    if (k < 0) break;
    if (nexp == kExpCap) {
      if (lane == 0) {
        set_error(a.err, kErrExpansions, static_cast<int32_t>(p));
        a.newdeg[row0 + w] = 0;
      }
      return;
    }
    const int32_t u = s.li[cur][k];
    if (lane == 0) {
      s.lf[cur][k] = 1;
      exp_d[nexp] = s.ld[cur][k];
      exp_i[nexp] = u;
    }
    ++nexp;
    // new candidates: the neighbours of u not seen before, in list order
    const int deg = a.degree[u];
    const int32_t* nb = a.graph + static_cast<int64_t>(u) * a.R;
    int cnt_c = 0;
    for (int t0 = 0; t0 < deg; t0 += 32) {
      const int t = t0 + lane;
      bool fresh = false;
      int32_t v = 0;
      float d = 0.f;
      if (t < deg) {
        v = nb[t];
        fresh = seen_insert(seen, tag, v, a.err);
        if (fresh) d = VDist<T>::l2(qv, data + static_cast<int64_t>(v) * a.dim, a.dim);
      }
      const uint32_t m = __ballot_sync(0xffffffffu, fresh);
      if (fresh) {
        const int at = cnt_c + __popc(m & ((1u << lane) - 1u));
        s.cd[at] = d;
        s.ci[at] = v;
      }
      cnt_c += __popc(m);
    }
    __syncwarp();
    // sort the candidates (distinct ids: the rank is unique)
    for (int j = lane; j < cnt_c; j += 32) {
      const float d = s.cd[j];
      const int32_t id = s.ci[j];
      int r = 0;
      for (int t = 0; t < cnt_c; ++t) r += cand_less(s.cd[t], s.ci[t], d, id);
      s.cd2[r] = d;
      s.ci2[r] = id;
    }
    __syncwarp();
    // new list = the L smallest of list and candidates (the host inserts one at a time and keeps L)
    const int nxt = cur ^ 1;
    for (int i = lane; i < size; i += 32) {
      const float d = s.ld[cur][i];
      const int32_t id = s.li[cur][i];
      int lo = 0, hi = cnt_c;  // candidates before list[i]
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (cand_less(s.cd2[mid], s.ci2[mid], d, id)) lo = mid + 1; else hi = mid;
      }
      const int pos = i + lo;
      if (pos < a.L) {
        s.ld[nxt][pos] = d;
        s.li[nxt][pos] = id;
        s.lf[nxt][pos] = s.lf[cur][i];
      }
    }
    for (int j = lane; j < cnt_c; j += 32) {
      const float d = s.cd2[j];
      const int32_t id = s.ci2[j];
      int lo = 0, hi = size;  // list entries before candidate j
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (cand_less(s.ld[cur][mid], s.li[cur][mid], d, id)) lo = mid + 1; else hi = mid;
      }
      const int pos = j + lo;
      if (pos < a.L) {
        s.ld[nxt][pos] = d;
        s.li[nxt][pos] = id;
        s.lf[nxt][pos] = 0;
      }
    }
    __syncwarp();
    size = min(a.L, size + cnt_c);
    cur = nxt;
  }
  // pool = expanded nodes + p's current out-list
  const int degp = a.degree[p];
  const int32_t* nbp = a.graph + p * a.R;
  for (int t = lane; t < degp; t += 32) {
    const int32_t v = nbp[t];
    exp_d[nexp + t] = VDist<T>::l2(qv, data + static_cast<int64_t>(v) * a.dim, a.dim);
    exp_i[nexp + t] = v;
  }
  __syncwarp();
  int32_t* out = a.newlist + static_cast<size_t>(row0 + w) * a.R;
  const int o = robust_prune<T>(a, p, exp_d, exp_i, nexp + degp, exp_d + kPoolCap, exp_i + kPoolCap, alpha, out,
                                s.pruned, lane);
  if (lane == 0) a.newdeg[row0 + w] = o;
}

// ------------------------------------------------------ 2. install --

__global__ void install_kernel(const VArgs a, int64_t first, int64_t cnt, unsigned long long* keys) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= cnt * a.R) return;
  const int b = static_cast<int>(i / a.R), t = static_cast<int>(i % a.R);
  const int64_t p = a.perm[first + b];
  const int deg = a.newdeg[b];
  const int32_t j = t < deg ? a.newlist[static_cast<int64_t>(b) * a.R + t] : -1;
  a.graph[p * a.R + t] = j;
  if (t == 0) a.degree[p] = deg;
  keys[i] = j >= 0 ? (static_cast<unsigned long long>(static_cast<uint32_t>(j)) << 32) |
                                   static_cast<uint32_t>(p)
                             : kNoKey;
}

// Pools above this size are cut to their kMaxOcclusion nearest by a radix
// select before the (quadratic) rank sort of robust_prune.
constexpr int kSelectAbove = 1024;

// One warp: moves the `keep` smallest of the P keys (float bits of pd[i], pi[i])
// -- which are distinct, as the ids of a reverse-edge pool are -- to the front of
// pd / pi in their old order, by an 8-bit-digit radix select over the 64-bit
// keys.  Distances are >= 0, so their float bits order like the floats.
// hist: 256 words of this warp's shared memory.  Returns keep.
__device__ int select_nearest(float* pd, int32_t* pi, int P, int keep, unsigned* hist, int lane) {
  auto key = [&](int i) {
    return (static_cast<unsigned long long>(__float_as_uint(pd[i])) << 32) | static_cast<uint32_t>(pi[i]);
  };
  unsigned long long prefix = 0;  // the digits of the keep-th smallest key found so far
  int need = keep;                // its rank among the keys that share those digits
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int b = lane; b < 256; b += 32) hist[b] = 0u;
    __syncwarp();
    const unsigned long long hi = shift == 56 ? 0ull : (~0ull << (shift + 8));
    for (int i = lane; i < P; i += 32) {
      const unsigned long long k = key(i);
      if ((k & hi) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
    }
    __syncwarp();
    unsigned c[8], sum = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      c[t] = hist[8 * lane + t];
      sum += c[t];
    }
    unsigned incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const unsigned excl = incl - sum;
    const bool mine = excl < static_cast<unsigned>(need) && static_cast<unsigned>(need) <= incl;
    const int src = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
    int digit = 0;
    unsigned before = excl;
    if (mine) {
      for (int t = 0; t < 8; ++t) {
        if (before + c[t] >= static_cast<unsigned>(need)) {
          digit = 8 * lane + t;
          break;
        }
        before += c[t];
      }
    }
    digit = __shfl_sync(0xffffffffu, digit, src);
    before = __shfl_sync(0xffffffffu, before, src);
    prefix |= static_cast<unsigned long long>(digit) << shift;
    need -= static_cast<int>(before);
    __syncwarp();
  }
  // prefix is now the keep-th smallest key itself: keep every key <= it, in order
  int w = 0;
  for (int base = 0; base < P; base += 32) {
    const int i = base + lane;
    float dv = 0.f;
    int32_t iv = 0;
    bool take = false;
    if (i < P) {
      dv = pd[i];
      iv = pi[i];
      take = ((static_cast<unsigned long long>(__float_as_uint(dv)) << 32) | static_cast<uint32_t>(iv)) <= prefix;
    }
    const unsigned m = __ballot_sync(0xffffffffu, take);
    __syncwarp();  // every lane has read its entry before any moves down
    if (take) {
      const int at = w + __popc(m & ((1u << lane) - 1u));
      pd[at] = dv;
      pi[at] = iv;
    }
    w += __popc(m);
    __syncwarp();
  }
  return w;
}

// ------------------------------------------------------ 4. reverse edges --

struct RevArgs {
  const unsigned long long* keys;
  int64_t total;
  const int32_t* heads;  // group start indices, ascending
  int32_t* nheads;       // [0] groups, [1] valid keys, [2] longest group
  float* pd;             // per-warp pools of 2 (R + longest group) entries
  int32_t* pi;
  uint32_t* bits;        // per-warp prune flags, bits_per_warp words
  int64_t pool_per_warp;
  int64_t bits_per_warp;
};

// Group starts (unordered) and the number of valid keys.
__global__ void heads_kernel(const unsigned long long* keys, int64_t total, int32_t* heads, int32_t* nheads) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const unsigned long long k = keys[i];
  if (k == kNoKey) return;
  if (i == 0 || (keys[i - 1] >> 32) != (k >> 32)) heads[atomicAdd(nheads, 1)] = static_cast<int32_t>(i);
  if (i + 1 == total || keys[i + 1] == kNoKey) nheads[1] = static_cast<int32_t>(i + 1);
}

// Longest group, from the sorted starts.
__global__ void longest_kernel(const int32_t* heads, int32_t* nheads) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  const int nh = nheads[0];
  if (g >= nh) return;
  const int end = g + 1 < nh ? heads[g + 1] : nheads[1];
  atomicMax(nheads + 2, end - heads[g]);
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) reverse_kernel(const VArgs a, RevArgs r, float alpha) {
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int nh = r.nheads[0];
  const T* data = static_cast<const T*>(a.data);
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * kWarps + wib;
  float* wpd = r.pd + wid * r.pool_per_warp;
  int32_t* wpi = r.pi + wid * r.pool_per_warp;
  uint32_t* pruned = r.bits + wid * r.bits_per_warp;
  __shared__ unsigned s_hist[kWarps][256];
  for (int g = static_cast<int>(wid); g < nh; g += gridDim.x * kWarps) {
    const int64_t h = r.heads[g];
    const int32_t j = static_cast<int32_t>(r.keys[h] >> 32);
    const int64_t e = g + 1 < nh ? r.heads[g + 1] : r.nheads[1];
    int32_t* nb = a.graph + static_cast<int64_t>(j) * a.R;
    const int deg = a.degree[j];
    // the p's of the group that are new to j, in ascending order
    int nadd = 0;
    for (int64_t base = h; base < e; base += 32) {
      const int64_t k = base + lane;
      bool add = false;
      if (k < e) {
        const int32_t p = static_cast<int32_t>(r.keys[k] & 0xffffffffu);
        add = p != j;
        for (int t = 0; t < deg && add; ++t) add = nb[t] != p;
      }
      nadd += __popc(__ballot_sync(0xffffffffu, add));
    }
    if (deg + nadd <= a.R) {
      int at = deg;
      for (int64_t base = h; base < e; base += 32) {
        const int64_t k = base + lane;
        bool add = false;
        int32_t p = 0;
        if (k < e) {
          p = static_cast<int32_t>(r.keys[k] & 0xffffffffu);
          add = p != j;
          for (int t = 0; t < deg && add; ++t) add = nb[t] != p;
        }
        const uint32_t m = __ballot_sync(0xffffffffu, add);
        if (add) nb[at + __popc(m & ((1u << lane) - 1u))] = p;
        at += __popc(m);
      }
      __syncwarp();
      if (lane == 0) a.degree[j] = deg + nadd;
      continue;
    }
    // overflow: re-prune old list + new p's (P <= R + longest group: the pool fits)
    int P = deg + nadd;
    float* pd = wpd;
    int32_t* pi = wpi;
    const T* vj = data + static_cast<int64_t>(j) * a.dim;
    for (int t = lane; t < deg; t += 32) {
      pd[t] = VDist<T>::l2(vj, data + static_cast<int64_t>(nb[t]) * a.dim, a.dim);
      pi[t] = nb[t];
    }
    int at = deg;
    for (int64_t base = h; base < e; base += 32) {
      const int64_t k = base + lane;
      bool add = false;
      int32_t p = 0;
      if (k < e) {
        p = static_cast<int32_t>(r.keys[k] & 0xffffffffu);
        add = p != j;
        for (int t = 0; t < deg && add; ++t) add = nb[t] != p;
      }
      const uint32_t m = __ballot_sync(0xffffffffu, add);
      if (add) {
        const int q = at + __popc(m & ((1u << lane) - 1u));
        pd[q] = VDist<T>::l2(vj, data + static_cast<int64_t>(p) * a.dim, a.dim);
        pi[q] = p;
      }
      at += __popc(m);
    }
    __syncwarp();
    // a large pool (a node many of the batch's points link to) goes to its kMaxOcclusion nearest first:
    // the same candidates robust_prune keeps, since the pool holds neither j nor a repeated id
    if (P > kSelectAbove) P = select_nearest(pd, pi, P, qv_vamana::kMaxOcclusion, s_hist[wib], lane);
    // prune into the list itself: robust_prune reads only the pool, so nb can take the result
    const int o = robust_prune<T>(a, j, pd, pi, P, pd + P, pi + P, alpha, nb, pruned, lane);
    for (int t = o + lane; t < a.R; t += 32) nb[t] = -1;
    __syncwarp();
    if (lane == 0) a.degree[j] = o;
  }
}

template <typename T>
int run_vamana(const T* h_data, int64_t n, int32_t dim, int32_t R, int32_t L, float alpha_final, int32_t passes,
               uint64_t seed, int32_t* h_graph, int32_t* h_degree, int64_t* h_medoid, std::string& err) {
  auto ck = [&](cudaError_t e, const char* what) {
    if (e != cudaSuccess && err.empty()) err = std::string(what) + ": " + cudaGetErrorString(e);
    return e == cudaSuccess;
  };
  const int64_t medoid = qv_vamana::medoid(h_data, n, dim);
  int dev = 0, num_sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
  const std::vector<int64_t> perm = qv_vamana::insertion_order(seed, n);
  const int64_t max_batch = qv_vamana::max_batch(n);
  VArgs a{};
  a.n = n;
  a.dim = dim;
  a.R = R;
  a.L = L;
  a.Lpad = (L + 31) / 32 * 32;
  a.medoid = medoid;
  const size_t wbytes = warp_smem_bytes(a.Lpad, dim, sizeof(T));
  const size_t smem = kWarps * wbytes;
  std::vector<void*> allocs;
  auto alloc = [&](size_t bytes) -> void* {
    void* p = nullptr;
    if (!ck(cudaMalloc(&p, std::max<size_t>(bytes, 16)), "cudaMalloc")) return nullptr;
    allocs.push_back(p);
    return p;
  };
  const int64_t max_keys = max_batch * R;
  void* d_data = alloc(static_cast<size_t>(n) * dim * sizeof(T));
  a.graph = static_cast<int32_t*>(alloc(static_cast<size_t>(n) * R * 4));
  a.degree = static_cast<int32_t*>(alloc(static_cast<size_t>(n) * 4));
  int64_t* d_perm = static_cast<int64_t*>(alloc(static_cast<size_t>(n) * 8));
  a.newlist = static_cast<int32_t*>(alloc(static_cast<size_t>(max_batch) * R * 4));
  a.newdeg = static_cast<int32_t*>(alloc(static_cast<size_t>(max_batch) * 4));
  const int64_t chunk = std::min<int64_t>(kChunk, max_batch);  // searches per launch
  a.seen = static_cast<unsigned long long*>(alloc(static_cast<size_t>(chunk) * kSeenCap * 8));
  a.pool_d = static_cast<float*>(alloc(static_cast<size_t>(chunk) * 2 * kPoolCap * 4));
  a.pool_i = static_cast<int32_t*>(alloc(static_cast<size_t>(chunk) * 2 * kPoolCap * 4));
  a.err = static_cast<int32_t*>(alloc(16));
  unsigned long long* keys = static_cast<unsigned long long*>(alloc(static_cast<size_t>(max_keys) * 8));
  unsigned long long* keys2 = static_cast<unsigned long long*>(alloc(static_cast<size_t>(max_keys) * 8));
  int32_t* heads = static_cast<int32_t*>(alloc(static_cast<size_t>(max_keys) * 4));
  int32_t* heads2 = static_cast<int32_t*>(alloc(static_cast<size_t>(max_keys) * 4));
  int32_t* nheads = static_cast<int32_t*>(alloc(16));
  size_t sort_bytes = 0, hsort_bytes = 0;
  cub::DeviceRadixSort::SortKeys(nullptr, sort_bytes, keys, keys2, static_cast<int>(max_keys));
  cub::DeviceRadixSort::SortKeys(nullptr, hsort_bytes, heads, heads2, static_cast<int>(max_keys));
  void* sort_tmp = alloc(std::max(sort_bytes, hsort_bytes));
  // reverse-phase pools, grown on demand: (warps) x 2 (R + longest group) entries
  float* rpd = nullptr;
  int32_t* rpi = nullptr;
  uint32_t* rbits = nullptr;
  int64_t rpool_entries = 0, rbits_words = 0;
  auto cleanup = [&] {
    for (void* p : allocs) cudaFree(p);
    if (rpd) cudaFree(rpd);
    if (rpi) cudaFree(rpi);
    if (rbits) cudaFree(rbits);
  };
  if (!err.empty()) {
    cleanup();
    return QV_ERR_OOM;
  }
  a.data = d_data;
  a.perm = d_perm;
  ck(cudaMemcpy(d_data, h_data, static_cast<size_t>(n) * dim * sizeof(T), cudaMemcpyHostToDevice), "copy data");
  ck(cudaMemcpy(d_perm, perm.data(), static_cast<size_t>(n) * 8, cudaMemcpyHostToDevice), "copy order");
  ck(cudaMemset(a.graph, 0xff, static_cast<size_t>(n) * R * 4), "memset");
  ck(cudaMemset(a.degree, 0, static_cast<size_t>(n) * 4), "memset");
  ck(cudaMemset(a.seen, 0, static_cast<size_t>(chunk) * kSeenCap * 8), "memset");
  ck(cudaMemset(a.err, 0, 16), "memset");
  ck(cudaMemset(a.newdeg, 0, static_cast<size_t>(max_batch) * 4), "memset");
  ck(cudaFuncSetAttribute(search_prune_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          static_cast<int>(smem)),
     "smem attribute");
  uint32_t tag = 1;
  // QV_BUILD_LOG=1: one stderr line per batch with the time of its searches and of its reverse-edge phase
  // (synchronising after each, so only for diagnosis) and the size of its largest reverse-edge group
  const char* log_env = std::getenv("QV_BUILD_LOG");
  const bool log = log_env && *log_env && *log_env != '0';
  auto now_ms = [&] {
    if (log) cudaDeviceSynchronize();
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
  };
  for (int32_t pass = 0; pass < passes && err.empty(); ++pass) {
    const float alpha = qv_vamana::pass_alpha(pass, passes, alpha_final);
    int64_t start = 0;
    int64_t bsize = qv_vamana::first_batch(pass, n);
    while (start < n && err.empty()) {
      const int64_t end = std::min(n, start + bsize);
      const int64_t cnt = end - start;
      const double t0 = log ? now_ms() : 0.0;
      for (int64_t c0 = 0; c0 < cnt; c0 += chunk) {
        const int ch = static_cast<int>(std::min<int64_t>(chunk, cnt - c0));
        if (tag + static_cast<uint32_t>(ch) < tag) {  // tags wrapped: clear the sets
          ck(cudaMemset(a.seen, 0, static_cast<size_t>(chunk) * kSeenCap * 8), "memset");
          tag = 1;
        }
        search_prune_kernel<T><<<(ch + kWarps - 1) / kWarps, kWarps * 32, smem>>>(a, start + c0, ch, c0, tag,
                                                                                   alpha);
        tag += static_cast<uint32_t>(ch);
      }
      const double t1 = log ? now_ms() : 0.0;
      const int64_t total = cnt * R;
      install_kernel<<<static_cast<unsigned>((total + 255) / 256), 256>>>(a, start, cnt, keys);
      ck(cub::DeviceRadixSort::SortKeys(sort_tmp, sort_bytes, keys, keys2, static_cast<int>(total)), "sort");
      ck(cudaMemsetAsync(nheads, 0, 16), "memset");
      heads_kernel<<<static_cast<unsigned>((total + 255) / 256), 256>>>(keys2, total, heads, nheads);
      int32_t nh[3] = {0, 0, 0};
      ck(cudaMemcpy(nh, nheads, 12, cudaMemcpyDeviceToHost), "group count");
      if (nh[0] > 0) {
        ck(cub::DeviceRadixSort::SortKeys(sort_tmp, hsort_bytes, heads, heads2, nh[0]), "sort");
        longest_kernel<<<static_cast<unsigned>((nh[0] + 255) / 256), 256>>>(heads2, nheads);
        ck(cudaMemcpy(nh, nheads, 12, cudaMemcpyDeviceToHost), "longest group");
        const int64_t per_warp = 2 * (static_cast<int64_t>(R) + nh[2]);
        // as many warps as groups, at most 16 per SM, within ~4 GB of pools
        int64_t warps = std::min<int64_t>(nh[0], static_cast<int64_t>(num_sms) * 16);
        warps = std::max<int64_t>(kWarps, std::min<int64_t>(warps, (int64_t(4) << 30) / (8 * per_warp)));
        warps = (warps + kWarps - 1) / kWarps * kWarps;
        const int64_t bits_per_warp = (R + static_cast<int64_t>(nh[2]) + 31) / 32;
        if (warps * per_warp > rpool_entries || warps * bits_per_warp > rbits_words) {
          if (rpd) cudaFree(rpd);
          if (rpi) cudaFree(rpi);
          if (rbits) cudaFree(rbits);
          rpd = nullptr;
          rpi = nullptr;
          rbits = nullptr;
          rpool_entries = warps * per_warp;
          rbits_words = warps * bits_per_warp;
          if (!ck(cudaMalloc(&rpd, static_cast<size_t>(rpool_entries) * 4), "cudaMalloc") ||
              !ck(cudaMalloc(&rpi, static_cast<size_t>(rpool_entries) * 4), "cudaMalloc") ||
              !ck(cudaMalloc(&rbits, static_cast<size_t>(rbits_words) * 4), "cudaMalloc"))
            break;
        }
        RevArgs r{keys2, total, heads2, nheads, rpd, rpi, rbits, per_warp, bits_per_warp};
        reverse_kernel<T><<<static_cast<unsigned>(warps / kWarps), kWarps * 32>>>(a, r, alpha);
      }
      if (log)
        std::fprintf(stderr, "[vamana_gpu] pass %d batch at %lld: %lld points, search %.1f ms, reverse %.1f ms, "
                     "%d groups, largest %d\n", pass, static_cast<long long>(start), static_cast<long long>(cnt),
                     t1 - t0, now_ms() - t1, nh[0], nh[2]);
      int32_t e[2] = {0, 0};
      ck(cudaGetLastError(), "build kernel launch");  // a refused launch leaves the error words clear
      ck(cudaMemcpy(e, a.err, 8, cudaMemcpyDeviceToHost), "build kernels");
      if (e[0] != kBuildOk && err.empty())
        err = e[0] == kErrExpansions ? "a greedy search expanded more than " + std::to_string(kExpCap) +
                                           " nodes (point " + std::to_string(e[1]) + ")"
                                     : "a greedy search saw more than " + std::to_string(kSeenCap) + " nodes";
      start = end;
      bsize = std::min(max_batch, bsize * 2);
    }
  }
  if (err.empty()) {
    ck(cudaMemcpy(h_graph, a.graph, static_cast<size_t>(n) * R * 4, cudaMemcpyDeviceToHost), "copy graph");
    ck(cudaMemcpy(h_degree, a.degree, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost), "copy degree");
    *h_medoid = medoid;
  }
  cleanup();
  return err.empty() ? QV_OK : QV_ERR_CUDA;
}

}  // namespace

extern "C" int qv_vamana_gpu(const void* base, int64_t n, int64_t dim, int32_t dtype, int32_t R, int32_t L,
                             float alpha, int32_t passes, uint64_t seed, int32_t device, int32_t* graph,
                             int32_t* degree, int64_t* medoid) {
  if (!base || !graph || !degree || !medoid || n <= 1 || dim <= 0 || dim > 1024 || R < 1 || R > kMaxR ||
      L < 1 || L > kMaxL || passes < 1 || n >= (int64_t(1) << 31)) {
    qv::set_last_error("qv_vamana_gpu: invalid argument (n in [2, 2^31), dim <= 1024, R <= " +
                       std::to_string(kMaxR) + ", L <= " + std::to_string(kMaxL) + ")");
    return QV_ERR_INVALID_ARG;
  }
  if (dtype != QV_UINT8 && dtype != QV_INT8 && dtype != QV_FLOAT) {
    qv::set_last_error("qv_vamana_gpu: unknown data type");
    return QV_ERR_INVALID_ARG;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    qv::set_last_error("qv_vamana_gpu: cannot select device " + std::to_string(device));
    return QV_ERR_CUDA;
  }
  cudaGetLastError();  // launches are checked with it: drop an error left by an earlier call
  std::string err;
  int rc;
  if (dtype == QV_UINT8)
    rc = run_vamana(static_cast<const uint8_t*>(base), n, static_cast<int32_t>(dim), R, L, alpha, passes, seed,
                    graph, degree, medoid, err);
  else if (dtype == QV_INT8)
    rc = run_vamana(static_cast<const int8_t*>(base), n, static_cast<int32_t>(dim), R, L, alpha, passes, seed,
                    graph, degree, medoid, err);
  else
    rc = run_vamana(static_cast<const float*>(base), n, static_cast<int32_t>(dim), R, L, alpha, passes, seed,
                    graph, degree, medoid, err);
  if (rc != QV_OK) qv::set_last_error("qv_vamana_gpu: " + err);
  return rc;
}
