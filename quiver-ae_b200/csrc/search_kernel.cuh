// search_kernel.cuh -- persistent beam-search kernel for sm_100a.
//
// One warp owns one query slot end to end: it builds the query's PQ lookup
// table in its own shared-memory slice, then runs the graph walk with no
// block-level barrier.  A CTA holds several independent slots; the grid is
// one persistent wave and warps pull query ids from a device counter.
//
// Semantics are those of the reference's persistent kernel (paths inside
// ruc-system/quiver-ae):
//   LUT + q''            src/shared/index/pq_device.cuh:9-36
//   ADC                  src/quiver/kernel_core/kernel_helpers.cuh:271-286
//   merge into the list  src/quiver/kernel_core/kernel_helpers.cuh:293-356
//   exact L2 + top-k     src/shared/common/gpu_primitives.cuh:26-44,
//                        src/quiver/kernel_core/kernel_helpers.cuh:65-104
//   compaction + select  src/quiver/kernel_core/kernel_helpers.cuh:437-518
//   lanes + gpruning     src/quiver/kernel_core/kernel_q1.cuh:180-704
// with every issued lane ready at the next poll (pages are resident, so a
// fetch completes before the warp looks again).  All fp32 arithmetic that
// feeds a comparison is spelled out with _rn intrinsics so contraction
// cannot change a bit.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace qvk {

constexpr int kPageSize = 4096;
constexpr int kPivots = 256;
constexpr uint32_t kVisited = 0x80000000u;
constexpr uint32_t kIdMask = 0x7fffffffu;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kMaxPipeWidth = 16;

// error_info[0] codes written by the kernel (first error wins).
enum DeviceError : int32_t {
  kErrNone = 0,
  kErrNeighborRange = 1,  // adjacency entry >= num_points
  kErrDegree = 2,         // stored degree > R
  kErrHopCap = 3,         // walk exceeded its iteration bound
  kErrNav = 4,            // nav graph: id out of range or entry search over its bound
  kErrVisited = 5,        // visited-filter table full
  kErrFeed = 6,           // streaming admission: a query was not fed within the feed timeout
};

// Byte offsets of one query slot's arrays inside the CTA's shared memory.
struct SlotLayout {
  int32_t bytes;                 // slot size, multiple of 16
  int32_t off_lut;               // float [M * 256]
  int32_t off_q2;                // float [dim]
  int32_t off_lid, off_ldist;    // candidate list, capacity ef
  int32_t off_nid, off_ndist;    // sorted new neighbours, capacity 32 * SMAX
  int32_t off_mid, off_mdist;    // merged list, capacity ef + 32 * SMAX
  int32_t off_rid, off_rdist;    // top-k, capacity k
  int32_t off_rec;               // kGroup record vectors
  int32_t rec_stride;            // bytes per staged vector, multiple of 16
  int32_t off_lane;              // int [W] pending node per pipe lane
  // block kernel only
  int32_t off_spos;              // float [128] new pairs by thread slot
  int32_t off_sflag;             // uint [128]   (their ids)
  int32_t off_r0;                // int [128]    (their insertion points in the list)
  int32_t off_S;                 // int [128] insertion points of the surviving pairs, ascending
  int32_t off_fsrc;              // int [128] thread slot of the j-th survivor
  int32_t off_misc;              // int [80] block scalars
  int32_t off_sort;              // uint [2][3][128] exchange buffers of the many-pair sort
};

struct SearchParams {
  const uint8_t* pages;          // page store: page p at pages + p * 4096 (stripe_shift == 0)
  // striped page store (stripe_shift > 0): page p is page p >> stripe_shift of
  // stripe p & (2^stripe_shift - 1), whose base (possibly another GPU's
  // memory, read over NVLink) is stripe_table[stripe]
  const unsigned long long* stripe_table;  // stripe base addresses
  int32_t stripe_shift;
  const uint8_t* codes;          // [N x M] PQ codes
  const float* pivots_t;         // [dim x 256]
  const float* centroid;         // [dim]
  const int32_t* chunk_off;      // [M + 1]
  const float* queries;          // [nq x dim]
  int32_t* out_ids;              // [nq x k]
  float* out_dists;              // [nq x k]
  int32_t* out_found;            // [nq] or null
  int32_t* out_steps;            // [nq] or null
  int64_t* out_nbrs;             // [nq] or null
  int64_t* out_time;             // [2 * nq] globaltimer at bind / finish, or null
  int32_t* work_counter;         // zero before launch
  int32_t* error_info;           // [4], zero before launch
  int64_t num_points;
  int64_t nq;
  int64_t max_iters;             // bound on pipe iterations per query
  int32_t dim, M, R, node_size, data_words, npp;
  int32_t ef, k, W;
  int32_t early_policy, gp_warmup, gp_patience;
  int32_t medoid;
  // nav graph (entry search per query); nav_graph == nullptr: entry = medoid
  const uint8_t* nav_data;       // [nav_num_node x dim], base data type
  const int32_t* nav_graph;      // [nav_num_node x nav_max_m], -1 padded
  const int32_t* nav_mapping;    // [nav_num_node] nav id -> base id
  int32_t nav_num_node, nav_max_m, nav_start;
  // visited-filter mode (not reference behaviour): per persistent CTA a
  // table of visited_cap entries (tag << 32 | id); visited == nullptr: off
  unsigned long long* visited;
  int32_t visited_cap;           // power of two
  uint32_t visited_tag0;         // tag of query qid = visited_tag0 + qid
  // streaming admission (feed == nullptr: every query is in `queries` at launch).
  // Queries [0, *feed) have been copied in; the host advances *feed in stream
  // order after each copy.  A worker (CTA of the block kernel, warp of the
  // warp kernel) that binds query qid waits until *feed > qid, at most
  // feed_timeout_ns, and after each query stores its running completion count
  // to done_slots[worker] (host-mapped memory the host polls).
  const int32_t* feed;
  uint32_t* done_slots;
  int64_t feed_timeout_ns;
  SlotLayout lay;
};

struct Slot {
  float* lut;
  float* q2;
  uint32_t* lid;
  float* ldist;
  uint32_t* nid;
  float* ndist;
  uint32_t* mid;
  float* mdist;
  int32_t* rid;
  float* rdist;
  uint8_t* rec;
  int32_t* lane;
};

__device__ __forceinline__ Slot make_slot(uint8_t* base, const SlotLayout& L) {
  Slot s;
  s.lut = reinterpret_cast<float*>(base + L.off_lut);
  s.q2 = reinterpret_cast<float*>(base + L.off_q2);
  s.lid = reinterpret_cast<uint32_t*>(base + L.off_lid);
  s.ldist = reinterpret_cast<float*>(base + L.off_ldist);
  s.nid = reinterpret_cast<uint32_t*>(base + L.off_nid);
  s.ndist = reinterpret_cast<float*>(base + L.off_ndist);
  s.mid = reinterpret_cast<uint32_t*>(base + L.off_mid);
  s.mdist = reinterpret_cast<float*>(base + L.off_mdist);
  s.rid = reinterpret_cast<int32_t*>(base + L.off_rid);
  s.rdist = reinterpret_cast<float*>(base + L.off_rdist);
  s.rec = base + L.off_rec;
  s.lane = reinterpret_cast<int32_t*>(base + L.off_lane);
  return s;
}

// (dist, id & mask) ordering of the reference's pair_less / lower_bound.
__device__ __forceinline__ bool key_less(float ad, uint32_t ai, float bd, uint32_t bi) {
  ai &= kIdMask;
  bi &= kIdMask;
  return ad < bd || (ad == bd && ai < bi);
}

// First index in [0, n) whose key is not below (x, xi).
__device__ __forceinline__ int lower_bound_s(const float* d, const uint32_t* id, int n,
                                             float x, uint32_t xi) {
  xi &= kIdMask;
  int l = 0, r = n;
  while (l < r) {
    const int m = (l + r) >> 1;
    const float dm = d[m];
    if (dm < x || (dm == x && (id[m] & kIdMask) < xi))
      l = m + 1;
    else
      r = m;
  }
  return l;
}

__device__ __forceinline__ void fma4(float4& a, float q, const float4 p) {
  float d;
  d = __fsub_rn(q, p.x); a.x = __fmaf_rn(d, d, a.x);
  d = __fsub_rn(q, p.y); a.y = __fmaf_rn(d, d, a.y);
  d = __fsub_rn(q, p.z); a.z = __fmaf_rn(d, d, a.z);
  d = __fsub_rn(q, p.w); a.w = __fmaf_rn(d, d, a.w);
}

// LUT[c][j] = sum over dims i of chunk c, ascending, of fma((q'_i - p_ij)^2);
// q2 first receives q' = q - c and ends as q'' = q' + c.  Lane l owns
// pivots 4l..4l+3 and 128+4l..128+4l+3 of every chunk row.
__device__ __forceinline__ void build_lut_warp(const SearchParams& p, const float* __restrict__ q,
                                               float* lut, float* q2, int lane) {
  for (int i = lane; i < p.dim; i += 32) q2[i] = __fsub_rn(__ldg(q + i), __ldg(p.centroid + i));
  __syncwarp();
  int c_lo = __ldg(p.chunk_off);
  for (int c = 0; c < p.M; ++c) {
    const int c_hi = __ldg(p.chunk_off + c + 1);
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int i = c_lo; i < c_hi; ++i) {
      const float qi = q2[i];
      const float4* row = reinterpret_cast<const float4*>(p.pivots_t + (size_t)i * kPivots);
      fma4(a, qi, __ldg(row + lane));
      fma4(b, qi, __ldg(row + 32 + lane));
    }
    float4* lrow = reinterpret_cast<float4*>(lut + (size_t)c * kPivots);
    lrow[lane] = a;
    lrow[32 + lane] = b;
    c_lo = c_hi;
  }
  __syncwarp();
  for (int i = lane; i < p.dim; i += 32) q2[i] = __fadd_rn(q2[i], __ldg(p.centroid + i));
  __syncwarp();
}

// square_sum_32: lane-strided fused accumulation, then the shfl_down tree.
template <typename T>
__device__ __forceinline__ float exact_l2_warp(const float* q2, const T* vec, int dim, int lane) {
  float acc = 0.f;
  for (int i = lane; i < dim; i += 32) {
    const float diff = __fsub_rn(q2[i], static_cast<float>(vec[i]));
    acc = __fmaf_rn(diff, diff, acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(kFull, acc, off));
  return __shfl_sync(kFull, acc, 0);
}

// Register bitonic sort of 32*S (dist, id) pairs, element e = s*32 + lane,
// ascending by key.
template <int S>
__device__ __forceinline__ void bitonic_sort(float (&d)[S], uint32_t (&id)[S], int lane) {
  constexpr int N = 32 * S;
#pragma unroll
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 32) {
        const int js = j >> 5;
#pragma unroll
        for (int s = 0; s < S; ++s) {
          const int t = s ^ js;
          if (t > s) {
            const bool asc = ((s * 32 + lane) & k) == 0;
            const bool sw = asc ? key_less(d[t], id[t], d[s], id[s])
                                : key_less(d[s], id[s], d[t], id[t]);
            if (sw) {
              const float td = d[s]; d[s] = d[t]; d[t] = td;
              const uint32_t ti = id[s]; id[s] = id[t]; id[t] = ti;
            }
          }
        }
      } else {
#pragma unroll
        for (int s = 0; s < S; ++s) {
          const float od = __shfl_xor_sync(kFull, d[s], j);
          const uint32_t oi = __shfl_xor_sync(kFull, id[s], j);
          const bool asc = ((s * 32 + lane) & k) == 0;
          const bool lower = (lane & j) == 0;
          const bool other_less = key_less(od, oi, d[s], id[s]);
          const bool take = (lower == asc) ? other_less : !other_less;
          if (take) { d[s] = od; id[s] = oi; }
        }
      }
    }
  }
}

// Merge the sorted list L[0,sz) with the sorted new pairs N[0,deg) exactly as
// the reference positions them (kernel_helpers.cuh:331-347): a new pair whose
// id equals the list entry it lands on goes right after it; then drop every
// entry whose id repeats its predecessor's (kernel_helpers.cuh:440-455) and
// keep the first ef.  The reference truncates to 2*ef before dropping; since
// the list never holds more than ef entries, at most ef pairs are dropped and
// the first ef survivors are the same.  Returns the new list size.
__device__ __forceinline__ int merge_warp(const Slot& s, int sz, int deg, int ef, int lane) {
  for (int e = lane; e < deg; e += 32) {
    const float d = s.ndist[e];
    const uint32_t id = s.nid[e];
    int r = lower_bound_s(s.ldist, s.lid, sz, d, id);
    if (r < sz && ((s.lid[r] ^ id) & kIdMask) == 0) ++r;
    s.mid[r + e] = id;
    s.mdist[r + e] = d;
  }
  for (int i = lane; i < sz; i += 32) {
    const float d = s.ldist[i];
    const uint32_t id = s.lid[i];
    const int pos = i + lower_bound_s(s.ndist, s.nid, deg, d, id);
    s.mid[pos] = id;
    s.mdist[pos] = d;
  }
  __syncwarp();
  const int total = sz + deg;
  int out = 0;
  for (int b = 0; b < total && out < ef; b += 32) {
    const int pidx = b + lane;
    uint32_t id = 0;
    float d = 0.f;
    bool keep = false;
    if (pidx < total) {
      id = s.mid[pidx];
      d = s.mdist[pidx];
      keep = !(pidx > 0 && ((id ^ s.mid[pidx - 1]) & kIdMask) == 0);
    }
    const unsigned m = __ballot_sync(kFull, keep);
    const int o = out + __popc(m & ((1u << lane) - 1u));
    if (keep && o < ef) {
      s.lid[o] = id;
      s.ldist[o] = d;
    }
    out += __popc(m);
  }
  __syncwarp();
  return out < ef ? out : ef;
}

// First unvisited entry in [0, size): mark it and return its id, or -1.
__device__ __forceinline__ int32_t select_warp(const Slot& s, int size, int lane) {
  for (int b = 0; b < size; b += 32) {
    const int i = b + lane;
    const bool unv = i < size && (s.lid[i] & kVisited) == 0;
    const unsigned m = __ballot_sync(kFull, unv);
    if (m) {
      const int f = b + __ffs(m) - 1;
      const uint32_t id = s.lid[f];
      __syncwarp();
      if (lane == 0) s.lid[f] = id | kVisited;
      __syncwarp();
      return static_cast<int32_t>(id & kIdMask);
    }
  }
  return -1;
}

// Insert (d, id) at the count of entries <= d, capping the size at k
// (kernel_helpers.cuh:65-104; gpu_primitives.cuh:99-138 for k > 32).
__device__ __forceinline__ int topk_insert_warp(int32_t* rid, float* rdist, int fc, int k, float d,
                                                int32_t id, int lane) {
  const int nsz = fc < k ? fc + 1 : k;
  if (k <= 32) {
    const bool valid = lane < fc;
    const float od = valid ? rdist[lane] : 0.f;
    const int32_t oi = valid ? rid[lane] : 0;
    const int pos = __popc(__ballot_sync(kFull, valid && od <= d));
    const float pd = __shfl_up_sync(kFull, od, 1);
    const int32_t pi = __shfl_up_sync(kFull, oi, 1);
    __syncwarp();
    if (lane < nsz) {
      if (lane == pos) {
        rdist[lane] = d;
        rid[lane] = id;
      } else if (lane > pos) {
        rdist[lane] = pd;
        rid[lane] = pi;
      }
    }
  } else {
    int pos = 0;
    for (int b = 0; b < fc; b += 32) {
      const int i = b + lane;
      pos += __popc(__ballot_sync(kFull, i < fc && rdist[i] <= d));
    }
    for (int b = ((nsz - 1) >> 5) << 5; b >= 0; b -= 32) {
      const int i = b + lane;
      const bool mv = i > pos && i < nsz;
      float v = 0.f;
      int32_t vi = 0;
      if (mv) { v = rdist[i - 1]; vi = rid[i - 1]; }
      __syncwarp();
      if (mv) { rdist[i] = v; rid[i] = vi; }
      __syncwarp();
    }
    if (lane == 0) { rdist[pos] = d; rid[pos] = id; }
  }
  __syncwarp();
  return nsz;
}

struct QueryState {
  int size;        // candidate list length (<= ef)
  int fc;          // top-k fill
  int step;        // expansions so far (reference's step_recall_step)
  int cnt;         // gpruning no-improvement counter
  int last_fc;
  float last_top1, last_topk;
  int64_t nbrs;    // PQ codes gathered
};

// kernel_q1.cuh:524-545.  Every lane computes the same answer.
__device__ __forceinline__ bool gpruning_stop(const SearchParams& p, const Slot& s, QueryState& q) {
  const float top1 = s.rdist[0];
  const float topk = s.rdist[p.k - 1];
  const bool improved = q.fc > q.last_fc || top1 < q.last_top1 || topk < q.last_topk;
  if (q.step < p.gp_warmup)
    q.cnt = 0;
  else
    q.cnt = improved ? 0 : q.cnt + 1;
  q.last_fc = q.fc;
  q.last_top1 = top1;
  q.last_topk = topk;
  return p.early_policy == 2 && q.step >= p.gp_warmup && p.gp_patience > 0 &&
         q.cnt >= p.gp_patience;
}

__device__ __forceinline__ void report_error(const SearchParams& p, int code, int64_t qid,
                                             int64_t detail, int lane) {
  if (lane == 0) {
    if (atomicCAS(p.error_info, 0, code) == 0) {
      p.error_info[1] = static_cast<int32_t>(qid);
      p.error_info[2] = static_cast<int32_t>(detail);
    }
  }
}



// ----------------------------------------------------------- visited mode
// A mode of this build, off by default (the reference tracks visited nodes
// only by bit 31 inside the candidate list, so a node that fell out of the
// list can come back and be expanded again): each query keeps the nodes it
// has scheduled for expansion in an open-addressing table of its CTA, in
// global memory (L2-resident), and a new pair whose id is there never
// re-enters the list.  Entries carry the query's tag, so the table is never
// cleared between queries.

__device__ __forceinline__ uint32_t visited_hash(uint32_t id) {
  id ^= id >> 16;
  id *= 0x85ebca6bu;
  id ^= id >> 13;
  id *= 0xc2b2ae35u;
  return id ^ (id >> 16);
}

__device__ __forceinline__ unsigned long long* visited_table(const SearchParams& p, int slot) {
  return p.visited + static_cast<size_t>(slot) * p.visited_cap;
}

// Returns false when the table is full (bounded probe).
static __device__ __noinline__ bool visited_insert(unsigned long long* tab, int cap, uint32_t tag, uint32_t id) {
  const unsigned long long want = (static_cast<unsigned long long>(tag) << 32) | id;
  uint32_t h = visited_hash(id) & static_cast<uint32_t>(cap - 1);
  for (int n = 0; n < cap; ++n) {
    unsigned long long cur = __ldcg(tab + h);
    for (int tries = 0; tries < 4; ++tries) {
      if (static_cast<uint32_t>(cur >> 32) != tag) {  // empty or another query's entry: claim it
        const unsigned long long old = atomicCAS(tab + h, cur, want);
        if (old == cur) return true;
        cur = old;
        continue;
      }
      if (static_cast<uint32_t>(cur) == id) return true;
      break;
    }
    h = (h + 1) & static_cast<uint32_t>(cap - 1);
  }
  return false;
}

static __device__ __noinline__ bool visited_has(const unsigned long long* tab, int cap, uint32_t tag, uint32_t id) {
  uint32_t h = visited_hash(id) & static_cast<uint32_t>(cap - 1);
  for (int n = 0; n < cap; ++n) {
    const unsigned long long cur = __ldcg(tab + h);
    if (static_cast<uint32_t>(cur >> 32) != tag) return false;
    if (static_cast<uint32_t>(cur) == id) return true;
    h = (h + 1) & static_cast<uint32_t>(cap - 1);
  }
  return false;
}

// ---------------------------------------------------------------- nav entry
// The entry search of src/quiver/kernel_core/inkernel_nav.cuh:60-201: a
// 32-slot queue (4 best + 28 neighbours of the node expanded last), exact L2
// (square_sum_32 order) on the query as given, before the centroid round
// trip.  Results depend on its exact steps, restated here in this
// repository's code:
//   * neighbour i < 28 of node u is graph[max_m * u + i] (a row shorter than
//     28 runs on into the next one; past the array's end it ends);
//   * four chunks of 7 neighbour slots each stop at their first -1 and leave
//     the rest of their slots as they were;
//   * round i of four: a copy of the previous round's pick hands it its
//     visited bit and drops out (the reference ORs from several lanes in one
//     store; here every copy's bit is kept), then a shfl_down argmin tree
//     (a value replaces only a strictly smaller one) names the slot moved to
//     i, and the swap is skipped when the two distances are equal;
//   * the walk goes on while one of the first four slots is unvisited.
constexpr int kNavL = 4;
constexpr int kNavR = 28;

__device__ __forceinline__ int32_t nav_edge(const SearchParams& p, int32_t u, int i) {
  const int64_t at = static_cast<int64_t>(p.nav_max_m) * u + i;
  return at < static_cast<int64_t>(p.nav_num_node) * p.nav_max_m ? __ldg(p.nav_graph + at) : -1;
}

template <typename T>
__device__ __forceinline__ const T* nav_vec(const SearchParams& p, int32_t v) {
  return reinterpret_cast<const T*>(p.nav_data) + static_cast<int64_t>(v) * p.dim;
}

// One warp: neighbour slots [i0, i1) of nav node u (stops at the first -1).
// Returns false on an id outside the nav graph.
template <typename T>
__device__ __forceinline__ bool nav_fill_warp(const SearchParams& p, const float* q, int32_t u, int i0, int i1,
                                              uint32_t* pid, float* pd, int lane) {
  for (int i = i0; i < i1; ++i) {
    const int32_t v = nav_edge(p, u, i);
    if (v == -1) break;
    if (v < 0 || v >= p.nav_num_node) return false;
    const float d = exact_l2_warp<T>(q, nav_vec<T>(p, v), p.dim, lane);
    if (lane == 0) {
      pid[i + kNavL] = static_cast<uint32_t>(v);
      pd[i + kNavL] = d;
    }
  }
  return true;
}

// One warp: the four selection rounds, then the first unvisited slot when it
// is one of the first four (else -1), the same on every lane.
__device__ __forceinline__ int nav_select_warp(uint32_t* pid, float* pd, int lane) {
#pragma unroll 1
  for (int i = 0; i < kNavL; ++i) {
    float dist = pd[lane];
    int pos = lane;
    bool dup = false;
    if (lane < i) dist = __int_as_float(0x7f800000);
    else if (i != 0 && ((pid[lane] ^ pid[i - 1]) & kIdMask) == 0) dup = true;
    __syncwarp();
    if (dup) {
      atomicOr(&pid[i - 1], pid[lane]);
      pd[lane] = __int_as_float(0x7f800000);
      dist = __int_as_float(0x7f800000);
    }
    __syncwarp();
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const int op = __shfl_down_sync(kFull, pos, off);
      const float od = __shfl_down_sync(kFull, dist, off);
      if (od < dist) {
        dist = od;
        pos = op;
      }
    }
    if (lane == 0 && i != pos) {
      const float t = pd[i], y = pd[pos];
      if (t != y) {
        pd[i] = y;
        pd[pos] = t;
        const uint32_t m = pid[i];
        pid[i] = pid[pos];
        pid[pos] = m;
      }
    }
    __syncwarp();
  }
  const unsigned unv = __ballot_sync(kFull, !(pid[lane] & kVisited));
  const int x = unv ? __ffs(unv) - 1 : 32;
  return x < kNavL ? x : -1;
}

// One warp, the whole entry search (the warp kernel).  Returns the base id,
// or -1 after reporting kErrNav.
template <typename T>
__device__ int32_t nav_entry_warp(const SearchParams& p, const float* q, uint32_t* pid, float* pd, int64_t qid,
                                  int lane) {
  const float d0 = exact_l2_warp<T>(q, nav_vec<T>(p, p.nav_start), p.dim, lane);
  pid[lane] = lane == 0 ? static_cast<uint32_t>(p.nav_start) : 0xffffffffu;
  pd[lane] = lane == 0 ? d0 : __int_as_float(0x7f800000);
  __syncwarp();
  const int64_t cap = 4 * static_cast<int64_t>(p.nav_num_node) + 64;
  int idx = 0;
  for (int64_t hop = 0; idx != -1; ++hop) {
    const int32_t u = static_cast<int32_t>(pid[idx] & kIdMask);
    bool ok = hop <= cap && u < p.nav_num_node;
    __syncwarp();
    if (lane == 0) pid[idx] |= kVisited;
    __syncwarp();
    for (int w = 0; w < 4 && ok; ++w) ok = nav_fill_warp<T>(p, q, u, 7 * w, 7 * w + 7, pid, pd, lane);
    if (!ok) {
      report_error(p, kErrNav, qid, u, lane);
      return -1;
    }
    __syncwarp();
    idx = nav_select_warp(pid, pd, lane);
  }
  const uint32_t raw = pid[0] & kIdMask;
  const int32_t entry = raw < static_cast<uint32_t>(p.nav_num_node) ? __ldg(p.nav_mapping + raw) : -1;
  if (entry < 0 || entry >= p.num_points) {
    report_error(p, kErrNav, qid, raw, lane);
    return -1;
  }
  return entry;
}

// Node v's record in the page store: page v / npp at offset (v % npp) *
// node_size (search.cu:240, kernel_helpers.cuh:257); ids are below 2^31, so
// 32-bit division.
__device__ __forceinline__ const uint8_t* node_record(const SearchParams& p, uint32_t v) {
  const uint32_t npp = static_cast<uint32_t>(p.npp);
  const uint32_t page = v / npp;
  const size_t off = static_cast<size_t>(v % npp) * p.node_size;
  if (p.stripe_shift == 0) return p.pages + static_cast<size_t>(page) * kPageSize + off;
  const uint8_t* base =
      reinterpret_cast<const uint8_t*>(__ldg(p.stripe_table + (page & ((1u << p.stripe_shift) - 1u))));
  return base + static_cast<size_t>(page >> p.stripe_shift) * kPageSize + off;
}

__device__ __forceinline__ uint32_t code_byte(const uint4& v, int b) {
  const uint32_t w = (b < 4) ? v.x : (b < 8) ? v.y : (b < 12) ? v.z : v.w;
  return (w >> ((b & 3) * 8)) & 0xffu;
}

// Records processed together: their fetches and code gathers overlap.
template <int SMAX>
struct GroupSize { static constexpr int value = SMAX <= 2 ? 4 : 2; };

// Expand the pipe lanes in `mask` in ascending lane order.  For every lane:
// merge its node's neighbours into the list, score the node exactly into
// the top-k, select the lane's next node, count the step and test gpruning.
// Returns 0 or a DeviceError.
template <typename T, int MC, int SMAX>
__device__ int expand_lanes(const SearchParams& p, const Slot& s, QueryState& q,
                            uint32_t mask, bool& stop, int64_t qid, int lane) {
  constexpr int G = GroupSize<SMAX>::value;
  constexpr int NV = MC > 0 ? MC / 16 : 1;
  while (mask) {
    int ws[G];
    int32_t node[G];
    int gact = 0;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      ws[g] = 0;
      node[g] = 0;
      if (mask) {
        ws[g] = __ffs(mask) - 1;
        mask &= mask - 1;
        node[g] = s.lane[ws[g]];
        ++gact;
      }
    }
    // 1. fetch: degree and neighbour ids into registers, the vector part of
    //    the record into this slot's staging buffer.
    uint32_t deg[G];
    uint32_t nb[G][SMAX];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      deg[g] = 0;
#pragma unroll
      for (int t = 0; t < SMAX; ++t) nb[g][t] = 0;
      if (g < gact) {
        const int64_t v = node[g];
        const uint32_t* rec = reinterpret_cast<const uint32_t*>(node_record(p, static_cast<uint32_t>(v)));
        deg[g] = rec[p.data_words];
#pragma unroll
        for (int t = 0; t < SMAX; ++t) {
          const int e = t * 32 + lane;
          if (e < p.R) nb[g][t] = rec[p.data_words + 1 + e];
        }
        uint32_t* dst = reinterpret_cast<uint32_t*>(s.rec + g * p.lay.rec_stride);
        for (int i = lane; i < p.data_words; i += 32) dst[i] = rec[i];
      }
    }
    // 2. validate the adjacency before any gather.
    int bad = 0;
    int64_t bad_detail = 0;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (g < gact) {
        if (deg[g] > static_cast<uint32_t>(p.R)) { bad = kErrDegree; bad_detail = node[g]; }
#pragma unroll
        for (int t = 0; t < SMAX; ++t) {
          const uint32_t e = t * 32 + lane;
          if (e < deg[g] && static_cast<int64_t>(nb[g][t]) >= p.num_points) {
            bad = kErrNeighborRange;
            bad_detail = node[g];
          }
        }
      }
    }
    bad = __reduce_max_sync(kFull, bad);
    if (bad) {
      report_error(p, bad, qid, bad_detail, lane);
      return bad;
    }
    // 3. gather PQ codes of every neighbour of the group, then ADC.
    float nd[G][SMAX];
    if constexpr (MC > 0) {
      uint4 cw[G][SMAX][NV];
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int t = 0; t < SMAX; ++t) {
          const uint32_t e = t * 32 + lane;
          if (g < gact && e < deg[g]) {
            const uint4* src = reinterpret_cast<const uint4*>(p.codes + static_cast<int64_t>(nb[g][t]) * MC);
#pragma unroll
            for (int v = 0; v < NV; ++v) cw[g][t][v] = __ldg(src + v);
          } else {
#pragma unroll
            for (int v = 0; v < NV; ++v) cw[g][t][v] = make_uint4(0, 0, 0, 0);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int t = 0; t < SMAX; ++t) {
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < MC; ++j)
            acc = __fadd_rn(acc, s.lut[j * kPivots + code_byte(cw[g][t][j >> 4], j & 15)]);
          nd[g][t] = acc;
        }
      }
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int t = 0; t < SMAX; ++t) {
          const uint32_t e = t * 32 + lane;
          float acc = 0.f;
          if (g < gact && e < deg[g]) {
            const uint8_t* src = p.codes + static_cast<int64_t>(nb[g][t]) * p.M;
            for (int j = 0; j < p.M; ++j) acc = __fadd_rn(acc, s.lut[j * kPivots + __ldg(src + j)]);
          }
          nd[g][t] = acc;
        }
      }
    }
    __syncwarp();
    // 4. in lane order: sort, merge, visit, select, gpruning.
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (g < gact) {
        float kd[SMAX];
        uint32_t ki[SMAX];
#pragma unroll
        for (int t = 0; t < SMAX; ++t) {
          const uint32_t e = t * 32 + lane;
          const bool live = e < deg[g];
          kd[t] = live ? nd[g][t] : __int_as_float(0x7f800000);
          ki[t] = live ? nb[g][t] : 0xffffffffu;
        }
        bitonic_sort<SMAX>(kd, ki, lane);
#pragma unroll
        for (int t = 0; t < SMAX; ++t) {
          s.ndist[t * 32 + lane] = kd[t];
          s.nid[t * 32 + lane] = ki[t];
        }
        __syncwarp();
        q.size = merge_warp(s, q.size, static_cast<int>(deg[g]), p.ef, lane);
        q.nbrs += deg[g];
        const float dx = exact_l2_warp<T>(s.q2, reinterpret_cast<const T*>(s.rec + g * p.lay.rec_stride),
                                          p.dim, lane);
        if (q.fc < p.k || dx < s.rdist[p.k - 1]) q.fc = topk_insert_warp(s.rid, s.rdist, q.fc, p.k, dx, node[g], lane);
        int32_t next = select_warp(s, q.size, lane);
        q.step += 1;
        if (p.early_policy != 0 && gpruning_stop(p, s, q)) {
          stop = true;
          next = -1;
        }
        if (lane == 0) s.lane[ws[g]] = next;
        __syncwarp();
      }
    }
  }
  return 0;
}

__device__ __forceinline__ int64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return static_cast<int64_t>(t);
}

__device__ __forceinline__ int32_t load_feed(const int32_t* f) {
  int32_t v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}

// Streaming admission: true once query qid has been fed.  The wait is bounded
// by p.feed_timeout_ns of the global timer (and by an iteration count, each
// iteration sleeping at least 64 ns); when it runs out the worker reports
// kErrFeed and the caller stops.
static __device__ bool wait_fed(const SearchParams& p, int64_t qid) {
  if (!p.feed || load_feed(p.feed) > qid) return true;
  const int64_t t0 = globaltimer_ns();
  const int64_t max_iters = p.feed_timeout_ns / 64 + 1024;
  unsigned sleep_ns = 64;
  for (int64_t it = 0; it < max_iters; ++it) {
    __nanosleep(sleep_ns);
    if (load_feed(p.feed) > qid) return true;
    if (globaltimer_ns() - t0 > p.feed_timeout_ns) break;
    sleep_ns = sleep_ns < 2048 ? 2 * sleep_ns : 2048;
  }
  report_error(p, kErrFeed, qid, load_feed(p.feed), 0);
  return false;
}

// Streaming admission: publish a worker's running completion count.
__device__ __forceinline__ void mark_done(const SearchParams& p, int worker, uint32_t count) {
  if (p.done_slots) {
    volatile uint32_t* slot = p.done_slots + worker;
    *slot = count;
  }
}

template <typename T, int MC, int SMAX>
__device__ void run_query(const SearchParams& p, const Slot& s, int64_t qid, int lane) {
  if (p.out_time && lane == 0) p.out_time[2 * qid] = globaltimer_ns();
  build_lut_warp(p, p.queries + qid * p.dim, s.lut, s.q2, lane);
  for (int i = lane; i < p.k; i += 32) {
    s.rid[i] = -1;
    s.rdist[i] = __int_as_float(0x7f800000);
  }
  for (int w = lane; w < p.W; w += 32) s.lane[w] = -1;
  __syncwarp();
  int32_t entry = p.medoid;
  if (p.nav_graph) {  // the neighbour arrays are free until the first merge
    entry = nav_entry_warp<T>(p, p.queries + qid * p.dim, s.nid, s.ndist, qid, lane);
    __syncwarp();
  }
  if (lane == 0) s.lane[0] = entry;
  __syncwarp();

  QueryState q;
  q.size = 0;
  q.fc = 0;
  q.step = 0;
  q.cnt = 0;
  q.last_fc = 0;
  q.last_top1 = __int_as_float(0x7f800000);
  q.last_topk = __int_as_float(0x7f800000);
  q.nbrs = 0;
  bool stop = false;

  // boot: expand the entry on lane 0, then seed lanes 1..W-1.
  int err = entry < 0 ? static_cast<int>(kErrNav) : expand_lanes<T, MC, SMAX>(p, s, q, 1u, stop, qid, lane);
  if (!err) {
    for (int w = 1; w < p.W; ++w) {
      const int32_t nx = select_warp(s, q.size, lane);
      if (lane == 0) s.lane[w] = nx;
      __syncwarp();
    }
    int64_t iters = 0;
    while (!stop) {
      uint32_t active = 0;
      for (int w = 0; w < p.W; ++w)
        if (s.lane[w] != -1) active |= 1u << w;
      if (!active) break;
      if (++iters > p.max_iters) {
        report_error(p, kErrHopCap, qid, q.step, lane);
        err = kErrHopCap;
        break;
      }
      err = expand_lanes<T, MC, SMAX>(p, s, q, active, stop, qid, lane);
      if (err || stop) break;
      for (int w = 0; w < p.W; ++w) {
        if (!(active & (1u << w))) {
          const int32_t nx = select_warp(s, q.size, lane);
          if (lane == 0) s.lane[w] = nx;
          __syncwarp();
        }
      }
    }
  }
  for (int i = lane; i < p.k; i += 32) {
    p.out_ids[qid * p.k + i] = s.rid[i];
    p.out_dists[qid * p.k + i] = s.rdist[i];
  }
  if (lane == 0) {
    if (p.out_found) p.out_found[qid] = err ? -1 : q.fc;
    if (p.out_steps) p.out_steps[qid] = q.step;
    if (p.out_nbrs) p.out_nbrs[qid] = q.nbrs;
    if (p.out_time) p.out_time[2 * qid + 1] = globaltimer_ns();
  }
  __syncwarp();
}

template <typename T, int MC, int SMAX, bool STREAM>
__global__ void __launch_bounds__(256) search_kernel(const SearchParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const Slot s = make_slot(smem + static_cast<size_t>(warp) * p.lay.bytes, p.lay);
  const int worker = blockIdx.x * (blockDim.x >> 5) + warp;
  uint32_t done = 0;
  while (true) {
    int qid = 0;
    if (lane == 0) {
      qid = atomicAdd(p.work_counter, 1);
      if constexpr (STREAM)
        if (qid < p.nq && !wait_fed(p, qid)) qid = INT32_MAX;
    }
    qid = __shfl_sync(kFull, qid, 0);
    if (qid >= p.nq) break;
    run_query<T, MC, SMAX>(p, s, qid, lane);
    if constexpr (STREAM)
      if (lane == 0) mark_done(p, worker, ++done);
  }
}

}  // namespace qvk
