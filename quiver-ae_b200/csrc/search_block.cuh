// search_block.cuh -- persistent beam-search kernel, one 128-thread CTA per
// query slot (sm_100a).
//
// Same semantics as search_kernel.cuh's warp kernel (the reference's
// kernel_q1.cuh walk with every issued lane ready at the next poll); the
// work of a hop is spread over four warps:
//   fetch + ADC   one neighbour per thread; a group of 128 / RP pipe lanes
//                 (RP = R rounded up to 64 or 128) is fetched and scored at
//                 once, so their node-record and code gathers overlap;
//   merge         every new pair finds its rank among the new pairs and its
//                 insertion point in the list (binary search); pairs already
//                 in the list are dropped (kernel_helpers.cuh:331-335 places
//                 them right after their twin and :440-455 removes them);
//                 the survivors' final positions come from a block prefix
//                 count; the list then shifts in place from the first
//                 insertion point, highest chunk first, and the survivors
//                 drop into the gaps; entries pushed past ef are discarded;
//   visit         warp 3 scores the expanded node exactly and updates the
//                 top-k while the other warps merge;
//   select        warp 0 scans for the first unvisited entry starting from
//                 a lower bound that the merge keeps up to date, instead of
//                 from index 0.
#pragma once

#include "search_kernel.cuh"

namespace qvk {

constexpr int kBlock = 128;

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
};

struct BSlot {
  float* lut;
  float* q2;
  uint32_t* lid;
  float* ldist;
  float* nd;        // [G * RP] new pair distances, slot order
  uint32_t* ni;     // [G * RP] new pair ids
  int* spos;
  int* sflag;
  int* sorder;
  int* S;
  int* fpos;
  int* fsrc;
  int32_t* rid;
  float* rdist;
  uint8_t* rec;
  int32_t* lane;
  int* misc;
};

__device__ __forceinline__ BSlot make_bslot(uint8_t* base, const SlotLayout& L) {
  BSlot s;
  s.lut = reinterpret_cast<float*>(base + L.off_lut);
  s.q2 = reinterpret_cast<float*>(base + L.off_q2);
  s.lid = reinterpret_cast<uint32_t*>(base + L.off_lid);
  s.ldist = reinterpret_cast<float*>(base + L.off_ldist);
  s.nd = reinterpret_cast<float*>(base + L.off_ndist);
  s.ni = reinterpret_cast<uint32_t*>(base + L.off_nid);
  s.spos = reinterpret_cast<int*>(base + L.off_spos);
  s.sflag = reinterpret_cast<int*>(base + L.off_sflag);
  s.sorder = reinterpret_cast<int*>(base + L.off_sorder);
  s.S = reinterpret_cast<int*>(base + L.off_S);
  s.fpos = reinterpret_cast<int*>(base + L.off_fpos);
  s.fsrc = reinterpret_cast<int*>(base + L.off_fsrc);
  s.rid = reinterpret_cast<int32_t*>(base + L.off_rid);
  s.rdist = reinterpret_cast<float*>(base + L.off_rdist);
  s.rec = base + L.off_rec;
  s.lane = reinterpret_cast<int32_t*>(base + L.off_lane);
  s.misc = reinterpret_cast<int*>(base + L.off_misc);
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

// Per-query state that only thread 0 needs (gpruning, counters).
struct BlockQuery {
  int step, cnt, last_fc;
  float last_top1, last_topk;
  int64_t nbrs;
};

// Warp 0: first unvisited entry at or after the hint; marks it, advances the
// hint and stores the result in lane[w].  Returns the node (warp-uniform).
__device__ __forceinline__ int32_t select_block_warp(const BSlot& s, int w, int lane) {
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
  if (next == -1 && lane == 0) s.misc[kMiscHint] = size;
  if (lane == 0) s.lane[w] = next;
  __syncwarp();
  return next;
}

// Merge record gg of the current group into the list, visit its node on
// warp 3, then select the lane's next node and test gpruning on warp 0.
template <typename T, int RP>
__device__ __forceinline__ void merge_visit_select(const SearchParams& p, const BSlot& s, int gg,
                                                   BlockQuery& bq) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int sz = s.misc[kMiscSize];
  const int deg = s.misc[kMiscDeg + gg];
  const int node = s.misc[kMiscNode + gg];
  const float* nd = s.nd + gg * RP;
  const uint32_t* ni = s.ni + gg * RP;
  // M1: the new pairs arrive as RP / 32 sorted runs of 32 (sorted per warp
  // after the ADC).  A pair's rank among them is its index in its run plus,
  // for every other run, the pairs below it (pairs of lower runs win ties,
  // so the ranks are a permutation).  A pair whose id repeats an earlier
  // pair's (an adjacency list that repeats an id) is dropped like one whose
  // id is already in the list: the reference's compaction keeps one of
  // adjacent equal ids.
  if (tid < RP) {
    const float kd = nd[tid];
    const uint32_t ki = ni[tid];
    if (ki != 0xffffffffu) {
      const int run = tid >> 5, i = tid & 31;
      const float* rd = nd + (run << 5);
      const uint32_t* ri = ni + (run << 5);
      int rnew = i;
      bool twin = i > 0 && ((ri[i - 1] ^ ki) & kIdMask) == 0 && rd[i - 1] == kd;
#pragma unroll
      for (int o = 0; o < RP / 32; ++o) {
        if (o == run) continue;
        const float* od = nd + (o << 5);
        const uint32_t* oi = ni + (o << 5);
        const int lb = lower_bound_s(od, oi, 32, kd, ki);
        if (o < run) {
          const bool eq = lb < 32 && od[lb] == kd && ((oi[lb] ^ ki) & kIdMask) == 0;
          rnew += lb + (eq ? 1 : 0);
          twin = twin || eq;
        } else {
          rnew += lb;
        }
      }
      const int r = lower_bound_s(s.ldist, s.lid, sz, kd, ki);
      const bool dup = twin || (r < sz && ((s.lid[r] ^ ki) & kIdMask) == 0);
      s.spos[rnew] = r;
      s.sflag[rnew] = dup ? 0 : 1;
      s.sorder[rnew] = tid;
    }
  }
  if (warp == 3) {  // visit: exact distance of the expanded node into the top-k
    const float dx = exact_l2_warp<T>(s.q2, reinterpret_cast<const T*>(s.rec + gg * p.lay.rec_stride), p.dim,
                                      lane);
    const int fc = s.misc[kMiscFc];
    if (fc < p.k || dx < s.rdist[p.k - 1]) {
      const int nfc = topk_insert_warp(s.rid, s.rdist, fc, p.k, dx, node, lane);
      if (lane == 0) s.misc[kMiscFc] = nfc;
    }
  }
  __syncthreads();
  // M2: survivors in key order get ranks by a block prefix count
  const int surv = (tid < deg) ? s.sflag[tid] : 0;
  const unsigned bal = __ballot_sync(kFull, surv);
  if (lane == 0) s.misc[kMiscWtot + warp] = __popc(bal);
  __syncthreads();
  int before = 0, nsurv = 0;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int t = s.misc[kMiscWtot + w];
    before += (w < warp) ? t : 0;
    nsurv += t;
  }
  if (surv) {
    const int j = before + __popc(bal & ((1u << lane) - 1u));
    s.S[j] = s.spos[tid];
    s.fpos[j] = s.spos[tid] + j;
    s.fsrc[j] = s.sorder[tid];
  }
  __syncthreads();
  // M3: shift the list in place from the first insertion point, high chunks first
  if (nsurv > 0) {
    const int first = s.S[0];
    if (first < sz) {
      for (int cb = ((sz - 1) / kBlock) * kBlock; cb >= (first / kBlock) * kBlock; cb -= kBlock) {
        const int i = cb + tid;
        const bool mv = i >= first && i < sz;
        uint32_t vid = 0;
        float vd = 0.f;
        int dst = 0;
        if (mv) {
          vid = s.lid[i];
          vd = s.ldist[i];
          dst = i + count_le(s.S, nsurv, i);
        }
        __syncthreads();
        if (mv && dst < p.ef) {
          s.lid[dst] = vid;
          s.ldist[dst] = vd;
        }
        __syncthreads();
      }
    }
    // M4: survivors into the gaps
    if (tid < nsurv) {
      const int fp = s.fpos[tid];
      if (fp < p.ef) {
        const int src = s.fsrc[tid];
        s.lid[fp] = ni[src];
        s.ldist[fp] = nd[src];
      }
    }
    if (tid == 0) {
      const int nsize = min(sz + nsurv, p.ef);
      const int h = s.misc[kMiscHint];
      const int nh = min(h + count_le(s.S, nsurv, h), s.S[0]);
      s.misc[kMiscSize] = nsize;
      s.misc[kMiscHint] = min(nh, nsize);
    }
    __syncthreads();
  }
  // select + gpruning
  if (warp == 0) {
    const int w = s.misc[kMiscWs + gg];
    int32_t next = select_block_warp(s, w, lane);
    if (lane == 0) {
      bq.step += 1;
      bq.nbrs += deg;
      if (p.early_policy != 0) {
        const int fc = s.misc[kMiscFc];
        const float top1 = s.rdist[0];
        const float topk = s.rdist[p.k - 1];
        const bool improved = fc > bq.last_fc || top1 < bq.last_top1 || topk < bq.last_topk;
        if (bq.step < p.gp_warmup)
          bq.cnt = 0;
        else
          bq.cnt = improved ? 0 : bq.cnt + 1;
        bq.last_fc = fc;
        bq.last_top1 = top1;
        bq.last_topk = topk;
        if (p.early_policy == 2 && bq.step >= p.gp_warmup && p.gp_patience > 0 && bq.cnt >= p.gp_patience) {
          s.misc[kMiscStop] = 1;
          s.lane[w] = -1;
        }
      }
    }
    (void)next;
  }
  __syncthreads();
}

// Expand the lanes in `mask`, in lane order, G = 128 / RP records at a time.
template <typename T, int MC, int RP>
__device__ int expand_block(const SearchParams& p, const BSlot& s, uint32_t mask, int64_t qid, BlockQuery& bq) {
  constexpr int G = kBlock / RP;
  constexpr int NV = MC > 0 ? MC / 16 : 1;
  const int tid = threadIdx.x;
  const int g = tid / RP, e = tid % RP;
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
    if (mine) {
      node = s.lane[ws[g]];
      const uint32_t* rec = reinterpret_cast<const uint32_t*>(p.pages + (node / p.npp) * kPageSize +
                                                              (node % p.npp) * p.node_size);
      deg = rec[p.data_words];
      if (e < p.R) nb = rec[p.data_words + 1 + e];
      uint32_t* dst = reinterpret_cast<uint32_t*>(s.rec + g * p.lay.rec_stride);
      for (int i = e; i < p.data_words; i += RP) dst[i] = rec[i];
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
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < MC; ++j) acc = __fadd_rn(acc, s.lut[j * kPivots + code_byte(cw[j >> 4], j & 15)]);
        d = acc;
      }
    } else {
      if (live && !bad_nb) {
        const uint8_t* src = p.codes + static_cast<int64_t>(nb) * p.M;
        float acc = 0.f;
        for (int j = 0; j < p.M; ++j) acc = __fadd_rn(acc, s.lut[j * kPivots + __ldg(src + j)]);
        d = acc;
      }
    }
    {  // each warp sorts its 32 pairs; padding (inf, 0xffffffff) sorts last
      float kd[1] = {d};
      uint32_t ki[1] = {live ? nb : 0xffffffffu};
      bitonic_sort<1>(kd, ki, tid & 31);
      s.nd[g * RP + e] = kd[0];
      s.ni[g * RP + e] = ki[0];
    }
    __syncthreads();
    if (s.misc[kMiscErr]) return s.misc[kMiscErr];
    for (int gg = 0; gg < gact; ++gg) merge_visit_select<T, RP>(p, s, gg, bq);
  }
  return 0;
}

template <typename T, int MC, int RP>
__device__ void run_query_block(const SearchParams& p, const BSlot& s, int64_t qid) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (p.out_time && tid == 0) p.out_time[2 * qid] = globaltimer_ns();
  build_lut_block(p, p.queries + qid * p.dim, s.lut, s.q2);
  for (int i = tid; i < p.k; i += kBlock) {
    s.rid[i] = -1;
    s.rdist[i] = __int_as_float(0x7f800000);
  }
  if (tid < kMaxPipeWidth) s.lane[tid] = (tid == 0) ? p.medoid : -1;
  if (tid == 0) {
    s.misc[kMiscErr] = 0;
    s.misc[kMiscSize] = 0;
    s.misc[kMiscHint] = 0;
    s.misc[kMiscFc] = 0;
    s.misc[kMiscStop] = 0;
  }
  BlockQuery bq;
  bq.step = 0;
  bq.cnt = 0;
  bq.last_fc = 0;
  bq.last_top1 = __int_as_float(0x7f800000);
  bq.last_topk = __int_as_float(0x7f800000);
  bq.nbrs = 0;
  __syncthreads();

  int err = expand_block<T, MC, RP>(p, s, 1u, qid, bq);  // boot: the entry on lane 0
  if (!err) {
    if (warp == 0)
      for (int w = 1; w < p.W; ++w) select_block_warp(s, w, lane);
    __syncthreads();
    int64_t iters = 0;
    while (!s.misc[kMiscStop]) {
      uint32_t active = 0;
      for (int w = 0; w < p.W; ++w)
        if (s.lane[w] != -1) active |= 1u << w;
      if (!active) break;
      if (++iters > p.max_iters) {
        if (tid == 0) report_error(p, kErrHopCap, qid, bq.step, 0);
        err = kErrHopCap;
        break;
      }
      __syncthreads();  // everyone has read lane[] before it changes
      err = expand_block<T, MC, RP>(p, s, active, qid, bq);
      if (err || s.misc[kMiscStop]) break;
      if (warp == 0)
        for (int w = 0; w < p.W; ++w)
          if (!(active & (1u << w))) select_block_warp(s, w, lane);
      __syncthreads();
    }
  }
  for (int i = tid; i < p.k; i += kBlock) {
    p.out_ids[qid * p.k + i] = s.rid[i];
    p.out_dists[qid * p.k + i] = s.rdist[i];
  }
  if (tid == 0) {
    if (p.out_found) p.out_found[qid] = err ? -1 : s.misc[kMiscFc];
    if (p.out_steps) p.out_steps[qid] = bq.step;
    if (p.out_nbrs) p.out_nbrs[qid] = bq.nbrs;
    if (p.out_time) p.out_time[2 * qid + 1] = globaltimer_ns();
  }
  __syncthreads();
}

template <typename T, int MC, int RP>
__global__ void __launch_bounds__(kBlock) search_block_kernel(const SearchParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const BSlot s = make_bslot(smem, p.lay);
  while (true) {
    if (threadIdx.x == 0) s.misc[kMiscQid] = atomicAdd(p.work_counter, 1);
    __syncthreads();
    const int qid = s.misc[kMiscQid];
    __syncthreads();
    if (qid >= p.nq) break;
    run_query_block<T, MC, RP>(p, s, qid);
  }
}

}  // namespace qvk
