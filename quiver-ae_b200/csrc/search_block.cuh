// search_block.cuh -- persistent beam-search kernel, one 128-thread CTA per
// query slot (sm_100a).
//
// Same semantics as search_kernel.cuh's warp kernel (the reference's
// kernel_q1.cuh walk with every issued lane ready at the next poll); the
// work of a hop is spread over four warps:
//   fetch + ADC   one neighbour per thread; a group of 128 / RP pipe lanes
//                 (RP = R rounded up to 64 or 128) is fetched and scored at
//                 once, so their node-record and code gathers overlap; the
//                 last warp of each record scores its node exactly under the
//                 code gathers;
//   group merge   the group's records are merged into the list in one pass
//                 (merge_group): every new pair filters itself against a full
//                 list's last entry and binary-searches its insertion point,
//                 dropping out when its id is listed; warp 0 ranks the
//                 survivors and computes each lane's next pick from the
//                 insertion points alone, while warp 1 visits the records'
//                 nodes (top-k, gpruning); then old entries move up by the
//                 survivors inserted before them, survivors land, entries
//                 pushed past ef are dropped and the picks are marked visited.
//                 Lists of up to 512 entries are moved from registers, longer
//                 ones in place chunk by chunk.  Three barriers per group (plus
//                 one per moved chunk of a long list).
#pragma once

#include "search_kernel.cuh"

namespace qvk {

constexpr int kBlock = 128;
constexpr int kFastEntries = 4;   // list entries per thread held in registers (lists of up to 512)

// block scalars (misc[])
enum : int {
  kMiscQid = 0,
  kMiscErr = 1,
  kMiscSize = 2,
  kMiscHint = 3,
  kMiscFc = 4,
  kMiscStop = 5,
  kMiscWtot = 8,    // [4] survivors per warp
  kMiscDeg = 12,    // [4] degree of each record of the group
  kMiscNode = 16,   // [4] node of each record of the group
  kMiscWs = 20,     // [4] lane of each record of the group
  kMiscStep = 40,
  kMiscCnt = 41,
  kMiscLastFc = 42,
  kMiscLastTop1 = 43,  // float bits
  kMiscLastTopk = 44,  // float bits
  kMiscNbrsLo = 45,
  kMiscNbrsHi = 46,
  kMiscWords = 48,  // words zeroed at the start of a query
  // group merge (merge_group)
  kMiscGMask = 48,  // [4] per-warp ballots of the pairs that may enter the list
  kMiscGFu1 = 52,   // [4] per-warp first unvisited entry at or after the hint
  kMiscGFu2 = 56,   // [4] per-warp second one
  kMiscGNs = 60,    // surviving pairs after removing repeated ids
  kMiscGPos0 = 61,  // final position of the first record's pick (-1: none or cut)
  kMiscGPos1 = 62,  // final position of the second record's pick (-1: none or cut)
  kMiscGStop0 = 63, // stop flag right after the first record's visit
  kMiscGId0 = 64,   // first record's pick (-1: none)
  kMiscGId1 = 65,   // second record's pick (-1: none)
  kMiscGHint = 66,  // hint after the merge
  kMiscDx = 67,     // [2] exact distance of each record's node (float bits)
  kMiscGRep = 72,   // [4] many-pair merge: sorted positions of pairs repeating an id
  kMiscNavIdx = 76, // nav entry search: next slot to expand (-1: done)
  kMiscNavErr = 77, // nav entry search: an id outside the nav graph
  kMiscSlots = 80,
};

struct BSlot {
  float* lut;
  float* q2;
  uint32_t* lid;
  float* ldist;
  float* sd;        // [128] new pairs by thread slot
  uint32_t* si;
  int* r0;          // [128] their insertion points in the list
  int* S;           // [128] insertion points of the survivors, ascending
  int* fsrc;        // [128] thread slot of the j-th survivor
  int32_t* rid;
  float* rdist;
  int32_t* lane;
  int* misc;
  uint32_t* sortbuf;  // [2][3][128] many-pair sort exchange buffers
};

__device__ __forceinline__ BSlot make_bslot(uint8_t* base, const SlotLayout& L) {
  BSlot s;
  s.lut = reinterpret_cast<float*>(base + L.off_lut);
  s.q2 = reinterpret_cast<float*>(base + L.off_q2);
  s.lid = reinterpret_cast<uint32_t*>(base + L.off_lid);
  s.ldist = reinterpret_cast<float*>(base + L.off_ldist);
  s.sd = reinterpret_cast<float*>(base + L.off_spos);
  s.si = reinterpret_cast<uint32_t*>(base + L.off_sflag);
  s.r0 = reinterpret_cast<int*>(base + L.off_r0);
  s.S = reinterpret_cast<int*>(base + L.off_S);
  s.fsrc = reinterpret_cast<int*>(base + L.off_fsrc);
  s.rid = reinterpret_cast<int32_t*>(base + L.off_rid);
  s.rdist = reinterpret_cast<float*>(base + L.off_rdist);
  s.lane = reinterpret_cast<int32_t*>(base + L.off_lane);
  s.misc = reinterpret_cast<int*>(base + L.off_misc);
  s.sortbuf = reinterpret_cast<uint32_t*>(base + L.off_sort);
  return s;
}

// #{ j < n : S[j] <= x } for ascending S.
__device__ __forceinline__ int count_le(const int* S, int n, int x) {
  int l = 0, r = n;
  while (l < r) {
    const int m = (l + r) >> 1;
    if (S[m] <= x) l = m + 1; else r = m;
  }
  return l;
}

// LUT + q'' with 128 threads: thread t owns pivots 2t, 2t+1 of every chunk
// row.  Per LUT entry the dims of its chunk are accumulated in ascending
// order with a fused multiply-add, as pq_device.cuh:179-186 does.
__device__ __forceinline__ void build_lut_block(const SearchParams& p, const float* __restrict__ q,
                                                float* lut, float* q2) {
  const int tid = threadIdx.x;
  for (int i = tid; i < p.dim; i += kBlock) q2[i] = __fsub_rn(__ldg(q + i), __ldg(p.centroid + i));
  __syncthreads();
  int c = 0;
  int c_hi = __ldg(p.chunk_off + 1);
  float2 acc = make_float2(0.f, 0.f);
  constexpr int PF = 8;
  for (int i0 = 0; i0 < p.dim; i0 += PF) {
    float2 pv[PF];
#pragma unroll
    for (int u = 0; u < PF; ++u)
      if (i0 + u < p.dim)
        pv[u] = __ldg(reinterpret_cast<const float2*>(p.pivots_t + (size_t)(i0 + u) * kPivots) + tid);
#pragma unroll
    for (int u = 0; u < PF; ++u) {
      const int i = i0 + u;
      if (i >= p.dim) break;
      while (i >= c_hi) {  // close chunk c (chunks may be empty)
        reinterpret_cast<float2*>(lut + (size_t)c * kPivots)[tid] = acc;
        acc = make_float2(0.f, 0.f);
        ++c;
        c_hi = __ldg(p.chunk_off + c + 1);
      }
      const float qi = q2[i];
      float d = __fsub_rn(qi, pv[u].x);
      acc.x = __fmaf_rn(d, d, acc.x);
      d = __fsub_rn(qi, pv[u].y);
      acc.y = __fmaf_rn(d, d, acc.y);
    }
  }
  for (; c < p.M; ++c) {  // the last chunk and any trailing empty ones
    reinterpret_cast<float2*>(lut + (size_t)c * kPivots)[tid] = acc;
    acc = make_float2(0.f, 0.f);
  }
  __syncthreads();
  for (int i = tid; i < p.dim; i += kBlock) q2[i] = __fadd_rn(q2[i], __ldg(p.centroid + i));
  __syncthreads();
}

__device__ __forceinline__ const uint8_t* record_ptr(const SearchParams& p, uint32_t v) { return node_record(p, v); }

// The last warp of each active group scores the group's node exactly
// (square_sum_32 order: lane l accumulates dims l, l + 32, ... with fused
// multiply-adds, then the shfl_down tree), lane 0 keeps the distance.  For
// byte vectors of up to 128 dims the warp loaded the vector with the record
// (vw = word `lane`), and the bytes of dim l + 32 j come from word
// l / 4 + 8 j by shuffle; otherwise the vector is read from the page store.
template <typename T, int RP>
__device__ __forceinline__ bool dx_warp(bool mine) {
  return mine && ((threadIdx.x >> 5) + 1) % (RP / 32) == 0;
}

template <typename T>
__device__ __forceinline__ bool dx_from_word(const SearchParams& p) {
  return sizeof(T) == 1 && p.dim <= 128;
}

template <typename T, int RP>
__device__ __forceinline__ void exact_l2_group(const SearchParams& p, const BSlot& s, bool mine, int g,
                                               const uint32_t* rec, uint32_t vw) {
  const int lane = threadIdx.x & 31;
  if (!dx_warp<T, RP>(mine)) return;
  float dx;
  if (dx_from_word<T>(p)) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t w = __shfl_sync(kFull, vw, (lane >> 2) + 8 * j);
      const int i = lane + 32 * j;
      if (i < p.dim) {
        const uint32_t b = (w >> (8 * (lane & 3))) & 0xffu;
        const float x = static_cast<float>(static_cast<T>(b));
        const float diff = __fsub_rn(s.q2[i], x);
        acc = __fmaf_rn(diff, diff, acc);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(kFull, acc, off));
    dx = __shfl_sync(kFull, acc, 0);
  } else {
    dx = exact_l2_warp<T>(s.q2, reinterpret_cast<const T*>(rec), p.dim, lane);
  }
  if (lane == 0) s.misc[kMiscDx + g] = __float_as_int(dx);
}

// Warp 0: first unvisited entry at or after the hint; marks it, advances the
// hint and stores the result in lane[w] (-1 instead when the query stopped).
__device__ __forceinline__ void select_block_warp(const BSlot& s, int w, int lane) {
  const int size = s.misc[kMiscSize];
  const int h = s.misc[kMiscHint];
  int32_t next = -1;
  for (int b = h; b < size; b += 32) {
    const int i = b + lane;
    const bool unv = i < size && (s.lid[i] & kVisited) == 0;
    const unsigned m = __ballot_sync(kFull, unv);
    if (m) {
      const int f = b + __ffs(m) - 1;
      const uint32_t id = s.lid[f];
      __syncwarp();
      if (lane == 0) {
        s.lid[f] = id | kVisited;
        s.misc[kMiscHint] = f + 1;
      }
      next = static_cast<int32_t>(id & kIdMask);
      break;
    }
  }
  if (lane == 0) {
    if (next == -1) s.misc[kMiscHint] = size;
    s.lane[w] = s.misc[kMiscStop] ? -1 : next;
  }
  __syncwarp();
}

// One warp: the expanded node's exact distance dx (computed while its record
// was fetched) into the top-k, then the step count and gpruning
// (kernel_q1.cuh:524-545) on its lane 0.  The per-query counters live in
// misc[] because the visiting warp changes with the record.
__device__ __forceinline__ void visit_warp(const SearchParams& p, const BSlot& s, float dx, int node, int deg,
                                           int lane) {
  int fc = s.misc[kMiscFc];
  if (fc < p.k || dx < s.rdist[p.k - 1]) {
    fc = topk_insert_warp(s.rid, s.rdist, fc, p.k, dx, node, lane);
    if (lane == 0) s.misc[kMiscFc] = fc;
  }
  if (lane == 0) {
    const int step = s.misc[kMiscStep] + 1;
    s.misc[kMiscStep] = step;
    const uint64_t nb = (static_cast<uint64_t>(static_cast<uint32_t>(s.misc[kMiscNbrsHi])) << 32 |
                         static_cast<uint32_t>(s.misc[kMiscNbrsLo])) + static_cast<uint64_t>(deg);
    s.misc[kMiscNbrsLo] = static_cast<int>(static_cast<uint32_t>(nb));
    s.misc[kMiscNbrsHi] = static_cast<int>(static_cast<uint32_t>(nb >> 32));
    if (p.early_policy != 0) {
      const float top1 = s.rdist[0];
      const float topk = s.rdist[p.k - 1];
      const bool improved = fc > s.misc[kMiscLastFc] || top1 < __int_as_float(s.misc[kMiscLastTop1]) ||
                            topk < __int_as_float(s.misc[kMiscLastTopk]);
      int cnt = s.misc[kMiscCnt];
      if (step < p.gp_warmup)
        cnt = 0;
      else
        cnt = improved ? 0 : cnt + 1;
      s.misc[kMiscCnt] = cnt;
      s.misc[kMiscLastFc] = fc;
      s.misc[kMiscLastTop1] = __float_as_int(top1);
      s.misc[kMiscLastTopk] = __float_as_int(topk);
      if (p.early_policy == 2 && step >= p.gp_warmup && p.gp_patience > 0 && cnt >= p.gp_patience)
        s.misc[kMiscStop] = 1;
    }
  }
}

// Position (0-based) of the n-th set bit of m; n < popc(m).
__device__ __forceinline__ int nth_set_bit(unsigned m, int n) {
  int pos = 0;
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const int c = __popc(m & ((1u << w) - 1u));
    if (n >= c) {
      n -= c;
      m >>= w;
      pos += w;
    }
  }
  return pos;
}

// Many-pair ranking for merge_group (more than 32 surviving pairs): a
// bitonic sort of the group's 128 slots by (dist, id, record, slot), pairs
// that cannot enter the list last.  Strides below 32 exchange by shuffle,
// the three of 32 and 64 through shared memory (two buffers, so one barrier
// each).  The records' order puts the first record's copy of an id first,
// and a sorted pair whose predecessor has its id drops out; the others
// compact themselves by the count of dropped pairs before them (a bitmask
// over sorted positions) and store their insertion point and slot at their
// rank in S / fsrc, as the small path does.  Ends with a barrier; the
// survivor count goes to kMiscGNs.
template <int RP>
__device__ __forceinline__ void merge_group_many_rank(const BSlot& s, int npre, bool pre, float d, uint32_t id) {
  const int tid = threadIdx.x;
  uint32_t khi = pre ? __float_as_uint(d) : 0xffffffffu;
  uint32_t klo = pre ? (((id & kIdMask) << 1) | (tid >= RP ? 1u : 0u)) : 0xffffffffu;
  uint32_t slot = static_cast<uint32_t>(tid);
  int buf = 0;
#pragma unroll
  for (int k = 2; k <= kBlock; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const int partner = tid ^ j;
      uint32_t ohi, olo, osl;
      if (j >= 32) {
        uint32_t* b = s.sortbuf + buf * 3 * kBlock;
        b[tid] = khi;
        b[kBlock + tid] = klo;
        b[2 * kBlock + tid] = slot;
        __syncthreads();
        ohi = b[partner];
        olo = b[kBlock + partner];
        osl = b[2 * kBlock + partner];
        buf ^= 1;
      } else {
        ohi = __shfl_xor_sync(kFull, khi, j);
        olo = __shfl_xor_sync(kFull, klo, j);
        osl = __shfl_xor_sync(kFull, slot, j);
      }
      const bool mine_less = khi < ohi || (khi == ohi && (klo < olo || (klo == olo && slot < osl)));
      const bool want_min = ((tid & k) == 0) == (tid < partner);
      if (mine_less != want_min) {
        khi = ohi;
        klo = olo;
        slot = osl;
      }
    }
  }
  // sorted: position tid holds (khi, klo, slot); the first npre are pairs
  uint32_t* b = s.sortbuf + buf * 3 * kBlock;
  b[tid] = khi;
  b[kBlock + tid] = klo;
  __syncthreads();
  const bool rep = tid > 0 && tid < npre && b[tid - 1] == khi && (b[kBlock + tid - 1] >> 1) == (klo >> 1);
  if (rep) atomicOr(reinterpret_cast<unsigned*>(&s.misc[kMiscGRep + (tid >> 5)]), 1u << (tid & 31));
  __syncthreads();
  int nrep = 0, before = 0;
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const unsigned rx = static_cast<unsigned>(s.misc[kMiscGRep + x]);
    const int w = tid >> 5;
    nrep += __popc(rx);
    before += x < w ? __popc(rx) : (x == w ? __popc(rx & ((1u << (tid & 31)) - 1u)) : 0);
  }
  if (tid < npre && !rep) {
    const int rank = tid - before;
    s.S[rank] = s.r0[slot];
    s.fsrc[rank] = static_cast<int>(slot);
  }
  if (tid == 0) s.misc[kMiscGNs] = npre - nrep;
  __syncthreads();
}

// Warp 0, many-pair path: both lanes' picks from the sorted survivors
// (S = insertion points, fsrc = slots, ascending by key), with the same rules
// as the small path; writes the same block scalars.
template <int RP>
__device__ __forceinline__ void merge_group_picks_sorted(const SearchParams& p, const BSlot& s, int gact, int sz) {
  const int lane = threadIdx.x & 31;
  const int ef = p.ef;
  constexpr int kNone = 0x7fffffff;
  const int ns = s.misc[kMiscGNs];
  const int a = lane < 4 ? s.misc[kMiscGFu1 + lane] : kNone;
  const int b = lane < 4 ? s.misc[kMiscGFu2 + lane] : kNone;
  const int fu1 = __reduce_min_sync(kFull, a);
  const int fu2 = __reduce_min_sync(kFull, a == fu1 ? b : a);
  // the first survivor from the group's first record
  int lA = -1;
  for (int b0 = 0; b0 < ns && lA < 0; b0 += 32) {
    const int j = b0 + lane;
    const unsigned fa = __ballot_sync(kFull, j < ns && s.fsrc[j] < RP);
    if (fa) lA = b0 + __ffs(fa) - 1;
  }
  int sel0 = -1, id0 = -1, pos0 = -1;
  if (lA >= 0 && (fu1 == kNone || s.S[lA] <= fu1)) {
    sel0 = 0;
    id0 = static_cast<int>(s.si[s.fsrc[lA]] & kIdMask);
    pos0 = s.S[lA] + lA;
  } else if (fu1 != kNone) {
    sel0 = 1;
    id0 = static_cast<int>(s.lid[fu1] & kIdMask);
    pos0 = fu1 + count_le(s.S, ns, fu1);
  }
  int id1 = -1, pos1 = -1;
  if (gact == 2) {
    const int ls = (sel0 == 0 && lA == 0) ? 1 : 0;
    const int lo = sel0 == 1 ? fu2 : fu1;
    if (ls < ns && (lo == kNone || s.S[ls] <= lo)) {
      pos1 = s.S[ls] + ls;
      id1 = static_cast<int>(s.si[s.fsrc[ls]] & kIdMask);
    } else if (lo != kNone) {
      pos1 = lo + count_le(s.S, ns, lo);
      id1 = static_cast<int>(s.lid[lo] & kIdMask);
    }
    if (pos1 >= ef) { pos1 = -1; id1 = -1; }
  }
  if (pos0 >= ef) pos0 = -1;
  if (lane == 0) {
    const int nsize = min(sz + ns, ef);
    s.misc[kMiscGPos0] = pos0;
    s.misc[kMiscGPos1] = pos1;
    s.misc[kMiscGId0] = id0;
    s.misc[kMiscGId1] = id1;
    s.misc[kMiscGHint] = gact == 2 ? (id1 >= 0 ? pos1 + 1 : nsize) : (id0 >= 0 ? pos0 + 1 : nsize);
  }
}

// Last phase of merge_group: old entries at or after the first insertion
// point move up by the number of insertion points at or below them
// (lc: this thread's entries tid, tid + 128, ... read before anything
// moved), survivors land at insertion point + rank, entries pushed past ef
// are dropped, the writers of the two picks set their visited bits, and
// thread 0 stores the size, the hint and the lanes' next nodes.
struct ListCopy {
  uint32_t id[kFastEntries];
  float d[kFastEntries];
};

__device__ __forceinline__ void merge_group_write(const SearchParams& p, const BSlot& s, int gact, int sz,
                                                  const ListCopy lc) {
  const int tid = threadIdx.x;
  const int ef = p.ef;
  const int ns = s.misc[kMiscGNs];
  const int pos0 = s.misc[kMiscGPos0];
  const int pos1 = s.misc[kMiscGPos1];
  const int first = ns > 0 ? s.S[0] : 0x7fffffff;
#pragma unroll
  for (int x = 0; x < kFastEntries; ++x) {
    const int i = tid + kBlock * x;
    if (i < sz) {
      const int dst = i >= first ? i + count_le(s.S, ns, i) : i;
      const bool mark = dst == pos0 || dst == pos1;
      if (dst < ef && (dst != i || mark)) {
        s.lid[dst] = lc.id[x] | (mark ? kVisited : 0u);
        s.ldist[dst] = lc.d[x];
      }
    }
  }
  if (tid < ns) {
    const int fp = s.S[tid] + tid;
    const int src = s.fsrc[tid];
    if (fp >= 0 && fp < ef && src >= 0 && src < kBlock) {
      const bool mark = fp == pos0 || fp == pos1;
      s.lid[fp] = s.si[src] | (mark ? kVisited : 0u);
      s.ldist[fp] = s.sd[src];
    }
  }
  if (tid == 0) {
    s.misc[kMiscSize] = min(sz + ns, ef);
    s.misc[kMiscHint] = s.misc[kMiscGHint];
    const int id0 = s.misc[kMiscGId0];
    s.lane[s.misc[kMiscWs]] = (id0 >= 0 && !s.misc[kMiscGStop0]) ? id0 : -1;
    if (gact == 2) {
      const int id1 = s.misc[kMiscGId1];
      s.lane[s.misc[kMiscWs + 1]] = (id1 >= 0 && !s.misc[kMiscStop]) ? id1 : -1;
    }
  }
  __syncthreads();
}

// The write phase for lists longer than the registers hold (more than 512
// entries): the same moves as merge_group_write, done in place in 128-entry
// chunks from the highest down to the one holding the first insertion point.
// An entry only moves up, so a chunk's writes never touch the lower chunks
// still to be read, and every write into a chunk's positions comes after the
// barrier that follows that chunk's reads: one barrier per chunk.  Picks are
// marked by whoever writes their final position; a pick that is an old entry
// before the first insertion point does not move and is marked in place.
__device__ __forceinline__ void merge_group_write_long(const SearchParams& p, const BSlot& s, int gact, int sz) {
  const int tid = threadIdx.x;
  const int ef = p.ef;
  const int ns = s.misc[kMiscGNs];
  const int pos0 = s.misc[kMiscGPos0];
  const int pos1 = s.misc[kMiscGPos1];
  const int first = ns > 0 ? s.S[0] : 0x7fffffff;
  if (first < sz) {
    for (int cb = ((sz - 1) / kBlock) * kBlock; cb >= (first / kBlock) * kBlock; cb -= kBlock) {
      const int i = cb + tid;
      const bool mv = i >= first && i < sz;
      uint32_t xid = 0;
      float xd = 0.f;
      int dst = 0;
      if (mv) {
        xid = s.lid[i];
        xd = s.ldist[i];
        dst = i + count_le(s.S, ns, i);
      }
      __syncthreads();
      if (mv && dst < ef) {
        const bool mark = dst == pos0 || dst == pos1;
        s.lid[dst] = xid | (mark ? kVisited : 0u);
        s.ldist[dst] = xd;
      }
    }
  }
  if (tid < ns) {
    const int fp = s.S[tid] + tid;
    const int src = s.fsrc[tid];
    if (fp >= 0 && fp < ef && src >= 0 && src < kBlock) {
      const bool mark = fp == pos0 || fp == pos1;
      s.lid[fp] = s.si[src] | (mark ? kVisited : 0u);
      s.ldist[fp] = s.sd[src];
    }
  }
  if (tid == 0) {
    // survivors land at or after `first` and moved entries above it, so
    // positions below it still hold their old, unmoved entries
    if (pos0 >= 0 && pos0 < first && pos0 < sz) s.lid[pos0] |= kVisited;
    if (pos1 >= 0 && pos1 < first && pos1 < sz) s.lid[pos1] |= kVisited;
    s.misc[kMiscSize] = min(sz + ns, ef);
    s.misc[kMiscHint] = s.misc[kMiscGHint];
    const int id0 = s.misc[kMiscGId0];
    s.lane[s.misc[kMiscWs]] = (id0 >= 0 && !s.misc[kMiscGStop0]) ? id0 : -1;
    if (gact == 2) {
      const int id1 = s.misc[kMiscGId1];
      s.lane[s.misc[kMiscWs + 1]] = (id1 >= 0 && !s.misc[kMiscStop]) ? id1 : -1;
    }
  }
  __syncthreads();
}

// Warp 1: visit the group's nodes in lane order, keeping the stop flag right
// after the first visit for the first lane.
__device__ __forceinline__ void merge_group_visits(const SearchParams& p, const BSlot& s, int gact, int lane) {
  visit_warp(p, s, __int_as_float(s.misc[kMiscDx]), s.misc[kMiscNode], s.misc[kMiscDeg], lane);
  __syncwarp();
  if (lane == 0) s.misc[kMiscGStop0] = s.misc[kMiscStop];
  if (gact == 2) {
    __syncwarp();
    visit_warp(p, s, __int_as_float(s.misc[kMiscDx + 1]), s.misc[kMiscNode + 1], s.misc[kMiscDeg + 1], lane);
  }
}

// Many-pair path of merge_group: rank, read this thread's old entries (the
// list does not move until the write phase), picks on warp 0 and visits on
// warp 1, then the write phase.
template <int RP>
__device__ __forceinline__ void merge_group_many(const SearchParams& p, const BSlot& s, int gact, int sz, int npre,
                                                 bool pre, float d, uint32_t id, bool long_list) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  merge_group_many_rank<RP>(s, npre, pre, d, id);
  ListCopy lc;
  if (!long_list) {
#pragma unroll
    for (int x = 0; x < kFastEntries; ++x) {
      const int i = tid + kBlock * x;
      lc.id[x] = i < sz ? s.lid[i] : 0u;
      lc.d[x] = i < sz ? s.ldist[i] : 0.f;
    }
  }
  if (warp == 0) merge_group_picks_sorted<RP>(p, s, gact, sz);
  if (warp == 1) merge_group_visits(p, s, gact, lane);
  __syncthreads();
  if (long_list)
    merge_group_write_long(p, s, gact, sz);
  else
    merge_group_write(p, s, gact, sz, lc);
}

// Merge the records of one group (one or two pipe lanes, in lane order) into
// the list in a single pass, visit their nodes and pick each lane's next node.
//
// Applying the records one after the other keeps the first ef entries of
// "list + first record's pairs" and then the first ef of "that + second
// record's pairs", dropping pairs whose id is already present.  An id always
// has the same key within a query, so this equals the first ef entries of the
// union of the list and both records' pairs with repeated keys removed; a
// pair that repeats a list entry or an earlier pair drops out, and an entry
// that the first merge would cut is cut by the union's ef as well.  What
// the order still decides is the visited marks: the first lane's pick is the
// first unvisited entry of the list after the first record alone, and it is
// marked before the second lane picks the first unvisited entry of the
// union.  Both picks are computed from the insertion points below, before
// anything moves.
//
// When more than 32 pairs survive the filter (the opening hops of a query),
// all threads rank them instead (merge_group_many_rank) and warp 0 takes the
// picks from the sorted survivors.
//
// The caller does not wait for the group's fetch and scoring to finish in
// every warp: phase A needs only this thread's own pair and the list (last
// written before the previous group's final barrier), so the first barrier
// here also publishes what the fetch wrote (degrees, nodes, exact distances,
// the error word).  Returns false, right after that barrier, when the fetch
// reported a device error.
template <typename T, int RP, bool LONG>
__device__ __forceinline__ bool merge_group(const SearchParams& p, const BSlot& s, int gact, bool live, float d,
                                            uint32_t id) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int sz = s.misc[kMiscSize];
  const int h = s.misc[kMiscHint];
  const int ef = p.ef;

  // Phase A: filter against a full list's last entry, insertion point, drop
  // pairs whose id is listed; old entries into registers; the first two
  // unvisited entries at or after the hint.
  bool pre = false;
  int r = 0;
  if (live) {
    bool cand = true;
    if (sz == ef) cand = key_less(d, id, s.ldist[sz - 1], s.lid[sz - 1]);
    if (cand) {
      r = lower_bound_s(s.ldist, s.lid, sz, d, id);
      pre = !(r < sz && ((s.lid[r] ^ id) & kIdMask) == 0);
      if (pre && p.visited)
        pre = !visited_has(visited_table(p, blockIdx.x), p.visited_cap, p.visited_tag0 + s.misc[kMiscQid], id);
      if (pre) {
        s.sd[tid] = d;
        s.si[tid] = id;
        s.r0[tid] = r;
      }
    }
  }
  const unsigned bal = __ballot_sync(kFull, pre);
  // uniform: sz was read after a barrier; kernels for ef <= 512 compile without the long path
  const bool long_list = LONG && sz > kBlock * kFastEntries;
  uint32_t vid[kFastEntries];
  float vd[kFastEntries];
  int f1 = 0x7fffffff, f2 = 0x7fffffff;
  if (!long_list) {
#pragma unroll
    for (int x = 0; x < kFastEntries; ++x) {
      const int i = tid + kBlock * x;
      vid[x] = 0;
      vd[x] = 0.f;
      if (i < sz) {
        vid[x] = s.lid[i];
        vd[x] = s.ldist[i];
        if (i >= h && (vid[x] & kVisited) == 0) {
          if (f1 == 0x7fffffff) f1 = i; else if (f2 == 0x7fffffff) f2 = i;
        }
      }
    }
  } else if (warp == 0) {
    // the list stays in shared memory (merge_group_write_long moves it); warp 0
    // finds the first two unvisited entries at or after the hint in 32-entry
    // windows (entries before the hint are all visited, so this is short)
    for (int b = h; b < sz && f2 == 0x7fffffff; b += 32) {
      const int i = b + lane;
      unsigned m = __ballot_sync(kFull, i < sz && (s.lid[i] & kVisited) == 0);
      if (m && f1 == 0x7fffffff) {
        f1 = b + __ffs(m) - 1;
        m &= m - 1;
      }
      if (m) f2 = b + __ffs(m) - 1;
    }
    f2 = lane == 0 ? f2 : 0x7fffffff;  // lane 0 alone carries the pair into the reduction below
    f1 = lane == 0 ? f1 : 0x7fffffff;
  }
  {
    const int w1 = __reduce_min_sync(kFull, f1);
    const int w2 = __reduce_min_sync(kFull, f1 == w1 ? f2 : f1);
    if (lane == 0) {
      s.misc[kMiscGMask + warp] = static_cast<int>(bal);
      s.misc[kMiscGFu1 + warp] = w1;
      s.misc[kMiscGFu2 + warp] = w2;
      s.misc[kMiscGRep + warp] = 0;
    }
  }
  __syncthreads();
  if (s.misc[kMiscErr]) return false;  // uniform: read after the barrier

  unsigned m[4];
  int npre = 0;
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    m[x] = static_cast<unsigned>(s.misc[kMiscGMask + x]);
    npre += __popc(m[x]);
  }
  // Phase B: warp 0 ranks the surviving pairs and computes both picks; warp
  // 1 visits the records' nodes in lane order.
  if (npre > 32) {  // uniform: every thread read the same ballots
    merge_group_many<RP>(p, s, gact, sz, npre, pre, d, id, long_list);
    return true;
  }
  if (warp == 0) {
    int slot = -1;
    float dd = 0.f;
    uint32_t ii = 0;
    int rr = 0;
    if (lane < npre) {
      int n = lane, base = 0;
      unsigned mm = m[0];
      if (n >= __popc(m[0])) {
        n -= __popc(m[0]); mm = m[1]; base = 32;
        if (n >= __popc(m[1])) {
          n -= __popc(m[1]); mm = m[2]; base = 64;
          if (n >= __popc(m[2])) { n -= __popc(m[2]); mm = m[3]; base = 96; }
        }
      }
      slot = base + nth_set_bit(mm, n);
      dd = s.sd[slot];
      ii = s.si[slot];
      rr = s.r0[slot];
    }
    unsigned lessm = 0, eqm = 0;
    for (int j = 0; j < npre; ++j) {
      const float dj = __shfl_sync(kFull, dd, j);
      const uint32_t ij = __shfl_sync(kFull, ii, j);
      if (key_less(dj, ij, dd, ii)) lessm |= 1u << j;
      else if (j < lane && ((ij ^ ii) & kIdMask) == 0) eqm |= 1u << j;
    }
    const bool valid = lane < npre && eqm == 0;  // first copy of its id
    const unsigned vm = __ballot_sync(kFull, valid);
    const bool inA = slot < RP;                   // from the group's first record
    const unsigned am = __ballot_sync(kFull, valid && inA);
    const int rank = __popc(lessm & vm);
    const int rankA = __popc(lessm & am);
    if (valid) {
      s.S[rank] = rr;
      s.fsrc[rank] = slot;
    }
    // first two unvisited old entries at or after the hint
    const int a = lane < 4 ? s.misc[kMiscGFu1 + lane] : 0x7fffffff;
    const int b = lane < 4 ? s.misc[kMiscGFu2 + lane] : 0x7fffffff;
    const int fu1 = __reduce_min_sync(kFull, a);
    const int fu2 = __reduce_min_sync(kFull, a == fu1 ? b : a);
    constexpr int kNone = 0x7fffffff;
    // surviving pairs that land before old entry i
    auto count_all = [&](int i) { return __popc(__ballot_sync(kFull, valid && rr <= i)); };
    const unsigned bA = __ballot_sync(kFull, valid && inA && rankA == 0);
    const unsigned b0 = __ballot_sync(kFull, valid && rank == 0);
    const unsigned b1 = __ballot_sync(kFull, valid && rank == 1);
    const int lA = bA ? __ffs(bA) - 1 : -1;
    const int l0 = b0 ? __ffs(b0) - 1 : -1;
    const int l1 = b1 ? __ffs(b1) - 1 : -1;
    const int rA = __shfl_sync(kFull, rr, lA < 0 ? 0 : lA);
    const uint32_t iA = __shfl_sync(kFull, ii, lA < 0 ? 0 : lA);
    const int rank_lA = __shfl_sync(kFull, rank, lA < 0 ? 0 : lA);
    const int cf1 = fu1 != kNone ? count_all(fu1) : 0;
    const int cf2 = fu2 != kNone ? count_all(fu2) : 0;
    // The first lane's pick: the first unvisited entry of "list + first
    // record", i.e. the first record's smallest survivor or the first
    // unvisited old entry, whichever has the smaller key (a survivor with
    // insertion point r precedes old entry i exactly when r <= i).  Its
    // position there is below ef: nothing of the first record precedes it.
    int sel0 = -1;  // 0: survivor lA, 1: old entry fu1
    int id0 = -1, pos0 = -1;
    if (lA >= 0 && (fu1 == kNone || rA <= fu1)) {
      sel0 = 0;
      id0 = static_cast<int>(iA & kIdMask);
      pos0 = rA + rank_lA;          // final position, counting the second record too
    } else if (fu1 != kNone) {
      sel0 = 1;
      id0 = static_cast<int>(s.lid[fu1] & kIdMask);
      pos0 = fu1 + cf1;
    }
    int id1 = -1, pos1 = -1;
    if (gact == 2) {
      // The second lane's pick: the first unvisited entry of the merged list
      // once the first pick is marked.
      const int ls = (sel0 == 0 && l0 == lA) ? l1 : l0;
      const int lo = sel0 == 1 ? fu2 : fu1;
      const int rs = __shfl_sync(kFull, rr, ls < 0 ? 0 : ls);
      const int ks = __shfl_sync(kFull, rank, ls < 0 ? 0 : ls);
      const uint32_t is = __shfl_sync(kFull, ii, ls < 0 ? 0 : ls);
      if (ls >= 0 && (lo == kNone || rs <= lo)) {
        pos1 = rs + ks;
        id1 = static_cast<int>(is & kIdMask);
      } else if (lo != kNone) {
        pos1 = lo + (lo == fu1 ? cf1 : cf2);
        id1 = static_cast<int>(s.lid[lo] & kIdMask);
      }
      if (pos1 >= ef) { pos1 = -1; id1 = -1; }
    }
    if (pos0 >= ef) pos0 = -1;  // picked, then cut by the second record
    if (lane == 0) {
      const int ns = __popc(vm);
      const int nsize = min(sz + ns, ef);
      s.misc[kMiscGNs] = ns;
      s.misc[kMiscGPos0] = pos0;
      s.misc[kMiscGPos1] = pos1;
      s.misc[kMiscGId0] = id0;
      s.misc[kMiscGId1] = id1;
      s.misc[kMiscGHint] = gact == 2 ? (id1 >= 0 ? pos1 + 1 : nsize) : (id0 >= 0 ? pos0 + 1 : nsize);
    }
  } else if (warp == 1) {
    merge_group_visits(p, s, gact, lane);
  }
  __syncthreads();

  if (long_list) {
    merge_group_write_long(p, s, gact, sz);
    return true;
  }
  ListCopy lc;
#pragma unroll
  for (int x = 0; x < kFastEntries; ++x) {
    lc.id[x] = vid[x];
    lc.d[x] = vd[x];
  }
  merge_group_write(p, s, gact, sz, lc);
  return true;
}

// Expand the lanes in `mask`, in lane order, G = 128 / RP records at a time.
template <typename T, int MC, int RP, bool LONG>
__device__ int expand_block(const SearchParams& p, const BSlot& s, uint32_t mask, int64_t qid) {
  constexpr int G = kBlock / RP;
  constexpr int NV = MC > 0 ? MC / 16 : 1;
  const int tid = threadIdx.x;
  const int g = tid / RP, e = tid % RP;
  if (p.visited) {  // visited mode: every node this pipe iteration expands is scheduled now
    if (tid < kMaxPipeWidth && ((mask >> tid) & 1u) &&
        !visited_insert(visited_table(p, blockIdx.x), p.visited_cap, p.visited_tag0 + s.misc[kMiscQid],
                        static_cast<uint32_t>(s.lane[tid])) &&
        atomicCAS(&s.misc[kMiscErr], 0, kErrVisited) == 0)
      report_error(p, kErrVisited, qid, s.lane[tid], 0);
    __syncthreads();
    if (s.misc[kMiscErr]) return s.misc[kMiscErr];
  }
  while (mask) {
    int ws[G], gact = 0;
#pragma unroll
    for (int x = 0; x < G; ++x) {
      ws[x] = 0;
      if (mask) {
        ws[x] = __ffs(mask) - 1;
        mask &= mask - 1;
        ++gact;
      }
    }
    const bool mine = g < gact;
    int64_t node = 0;
    uint32_t deg = 0, nb = 0;
    const uint32_t* rec = nullptr;
    uint32_t vw = 0;
    if (mine) {
      node = s.lane[ws[g]];
      rec = reinterpret_cast<const uint32_t*>(record_ptr(p, static_cast<uint32_t>(node)));
      deg = rec[p.data_words];
      if (e < p.R) nb = rec[p.data_words + 1 + e];
      if (dx_warp<T, RP>(mine) && dx_from_word<T>(p) && (tid & 31) < p.data_words) vw = rec[tid & 31];
      if (e == 0) {
        s.misc[kMiscDeg + g] = static_cast<int>(deg);
        s.misc[kMiscNode + g] = static_cast<int>(node);
        s.misc[kMiscWs + g] = ws[g];
      }
    }
    const bool bad_deg = mine && deg > static_cast<uint32_t>(p.R);
    const bool live = mine && !bad_deg && e < deg;
    const bool bad_nb = live && static_cast<int64_t>(nb) >= p.num_points;
    if (bad_deg || bad_nb) {
      if (atomicCAS(&s.misc[kMiscErr], 0, bad_deg ? kErrDegree : kErrNeighborRange) == 0)
        report_error(p, bad_deg ? kErrDegree : kErrNeighborRange, qid, node, 0);
    }
    float d = __int_as_float(0x7f800000);
    if constexpr (MC > 0) {
      uint4 cw[NV];
      if (live && !bad_nb) {
        const uint4* src = reinterpret_cast<const uint4*>(p.codes + static_cast<int64_t>(nb) * MC);
#pragma unroll
        for (int v = 0; v < NV; ++v) cw[v] = __ldg(src + v);
      }
      exact_l2_group<T, RP>(p, s, mine, g, rec, vw);  // while the code loads are in flight
      if (live && !bad_nb) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < MC; ++j) acc = __fadd_rn(acc, s.lut[j * kPivots + code_byte(cw[j >> 4], j & 15)]);
        d = acc;
      }
    } else {
      exact_l2_group<T, RP>(p, s, mine, g, rec, vw);
      if (live && !bad_nb) {
        const uint8_t* src = p.codes + static_cast<int64_t>(nb) * p.M;
        float acc = 0.f;
        for (int j = 0; j < p.M; ++j) acc = __fadd_rn(acc, s.lut[j * kPivots + __ldg(src + j)]);
        d = acc;
      }
    }
    if (!merge_group<T, RP, LONG>(p, s, gact, live, d, nb)) return s.misc[kMiscErr];
  }
  return 0;
}

// The nav entry search (see nav_select_warp) with the block's four warps
// taking 7 neighbour slots each, as inkernel_nav.cuh:109-136 splits them;
// warp 0 selects.  The queue lives in the many-pair sort buffer, free at
// query start.  Returns the base id, or -1 after reporting kErrNav.
template <typename T>
__device__ int32_t nav_entry_block(const SearchParams& p, const BSlot& s, const float* q, int64_t qid) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* pid = s.sortbuf;
  float* pd = reinterpret_cast<float*>(s.sortbuf + 32);
  if (warp == 0) {
    const float d0 = exact_l2_warp<T>(q, nav_vec<T>(p, p.nav_start), p.dim, lane);
    pid[lane] = lane == 0 ? static_cast<uint32_t>(p.nav_start) : 0xffffffffu;
    pd[lane] = lane == 0 ? d0 : __int_as_float(0x7f800000);
  }
  if (tid == 0) s.misc[kMiscNavErr] = 0;
  __syncthreads();
  const int64_t cap = 4 * static_cast<int64_t>(p.nav_num_node) + 64;
  int idx = 0;
  for (int64_t hop = 0; idx != -1; ++hop) {
    const int32_t u = static_cast<int32_t>(pid[idx] & kIdMask);
    if (hop > cap || u >= p.nav_num_node) {  // uniform: every thread read the same slot
      report_error(p, kErrNav, qid, u, tid);
      return -1;
    }
    __syncthreads();
    if (tid == 0) pid[idx] |= kVisited;
    if (!nav_fill_warp<T>(p, q, u, 7 * warp, 7 * warp + 7, pid, pd, lane) && lane == 0)
      s.misc[kMiscNavErr] = 1;
    __syncthreads();
    if (s.misc[kMiscNavErr]) {
      report_error(p, kErrNav, qid, u, tid);
      return -1;
    }
    if (warp == 0) {
      const int x = nav_select_warp(pid, pd, lane);
      if (lane == 0) s.misc[kMiscNavIdx] = x;
    }
    __syncthreads();
    idx = s.misc[kMiscNavIdx];
  }
  const uint32_t raw = pid[0] & kIdMask;
  const int32_t entry = raw < static_cast<uint32_t>(p.nav_num_node) ? __ldg(p.nav_mapping + raw) : -1;
  __syncthreads();  // everyone has read the queue before the sort buffer is reused
  if (entry < 0 || entry >= p.num_points) {
    report_error(p, kErrNav, qid, raw, tid);
    return -1;
  }
  return entry;
}

template <typename T, int MC, int RP, bool LONG>
__device__ void run_query_block(const SearchParams& p, const BSlot& s, int64_t qid) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (p.out_time && tid == 0) p.out_time[2 * qid] = globaltimer_ns();
  build_lut_block(p, p.queries + qid * p.dim, s.lut, s.q2);
  for (int i = tid; i < p.k; i += kBlock) {
    s.rid[i] = -1;
    s.rdist[i] = __int_as_float(0x7f800000);
  }
  int32_t entry = p.medoid;
  if (p.nav_graph) entry = nav_entry_block<T>(p, s, p.queries + qid * p.dim, qid);
  if (tid < kMaxPipeWidth) s.lane[tid] = (tid == 0) ? entry : -1;
  if (tid < kMiscWords && tid != kMiscQid) s.misc[tid] = 0;
  if (tid == kMiscLastTop1 || tid == kMiscLastTopk) s.misc[tid] = 0x7f800000;  // +inf
  __syncthreads();

  int err = entry < 0 ? static_cast<int>(kErrNav) : expand_block<T, MC, RP, LONG>(p, s, 1u, qid);  // boot: lane 0
  if (!err) {
    // lanes 1..W-1 are seeded whether or not the boot hop stopped the query
    // (kernel_q1.cuh:367-371); their picks matter only when it did not
    if (warp == 0)
      for (int w = 1; w < p.W; ++w) select_block_warp(s, w, lane);
    __syncthreads();
    int64_t iters = 0;
    const uint32_t all_lanes = (p.W >= 32) ? 0xffffffffu : ((1u << p.W) - 1u);
    while (!s.misc[kMiscStop]) {
      uint32_t active = 0;
      for (int w = 0; w < p.W; ++w)
        if (s.lane[w] != -1) active |= 1u << w;
      if (!active) break;
      if (++iters > p.max_iters) {
        if (tid == 0) report_error(p, kErrHopCap, qid, iters, 0);
        err = kErrHopCap;
        break;
      }
      // lane[] is next written by the merges, after at least one barrier
      // inside expand_block, so every thread has read it by then.
      err = expand_block<T, MC, RP, LONG>(p, s, active, qid);
      if (err || s.misc[kMiscStop]) break;
      // Idle lanes pick their next node; when every lane was active nothing
      // is written here and the merge's final barrier already ordered the
      // next iteration's reads.  `active` is uniform.
      if (active != all_lanes) {
        if (warp == 0)
          for (int w = 0; w < p.W; ++w)
            if (!(active & (1u << w))) select_block_warp(s, w, lane);
        __syncthreads();
      }
    }
  }
  for (int i = tid; i < p.k; i += kBlock) {
    p.out_ids[qid * p.k + i] = s.rid[i];
    p.out_dists[qid * p.k + i] = s.rdist[i];
  }
  if (tid == 0) {
    if (p.out_found) p.out_found[qid] = err ? -1 : s.misc[kMiscFc];
    if (p.out_steps) p.out_steps[qid] = s.misc[kMiscStep];
    if (p.out_nbrs)
      p.out_nbrs[qid] = static_cast<int64_t>(static_cast<uint64_t>(static_cast<uint32_t>(s.misc[kMiscNbrsHi])) << 32 |
                                             static_cast<uint32_t>(s.misc[kMiscNbrsLo]));
    if (p.out_time) p.out_time[2 * qid + 1] = globaltimer_ns();
  }
  __syncthreads();
}

// STREAM: queries arrive while the kernel runs (streaming admission: wait for
// each query's feed, publish completions); otherwise every query is present at
// launch and the loop carries no streaming code.  LONG: ef may exceed 512, so
// the group merge also carries the in-place path for long lists.
template <typename T, int MC, int RP, bool STREAM, bool LONG>
__global__ void __launch_bounds__(kBlock, 5) search_block_kernel(const SearchParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const BSlot s = make_bslot(smem, p.lay);
  uint32_t done = 0;
  while (true) {
    if (threadIdx.x == 0) {
      int q = atomicAdd(p.work_counter, 1);
      if constexpr (STREAM)
        if (q < p.nq && !wait_fed(p, q)) q = INT32_MAX;
      s.misc[kMiscQid] = q;
    }
    __syncthreads();
    const int qid = s.misc[kMiscQid];
    __syncthreads();
    if (qid >= p.nq) break;
    run_query_block<T, MC, RP, LONG>(p, s, qid);
    if constexpr (STREAM)
      if (threadIdx.x == 0) mark_done(p, blockIdx.x, ++done);
  }
}

}  // namespace qvk
