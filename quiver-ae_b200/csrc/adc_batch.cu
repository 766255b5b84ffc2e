// adc_batch.cu -- batched PQ asymmetric distances over many (query, code) pairs.
//
// The ADC step of the search (kernel_helpers.cuh:271-286: d = sum over the M
// chunks of LUT[j][code[j]], summed in chunk order in fp32), run over a batch:
// query q scores n_per_query codes, given either as ids (a gather, the access
// pattern of the search's neighbour scoring) or as a contiguous range starting
// at first[q] (a stream, as a scan over a list of codes).  Inside the search
// the same arithmetic is latency bound (one hop's 64 codes at a time); here it
// is bound by memory, and by shared-memory lookups.
//
// Two kernels:
//  * pipe (M == 32): eight lanes per code, four chunks per lane.  A lane looks
//    up its four chunks, adds them to the partial sum it received from the lane
//    before it (shfl_up), so the fp32 sum runs in chunk order 0..31 exactly as
//    the sequential loop does.  Codes flow through the eight lanes diagonally
//    (lane j works on code m - j at step m), so every lane is busy every step.
//    The LUT is staged once per group of lanes, each copy with its columns
//    rotated by the group number, so the 32 lookups of one warp instruction
//    fall in 32 different banks.  Codes stream into a per-warp ring of 32-code
//    batches with cp.async, several batches ahead; gathered ids stream into
//    their own ring further ahead, so no warp waits on an id load.
//  * thread (any M): one thread per code, LUT rows in shared memory; 16-byte
//    code loads when M == 32.  Random codes put several lanes of a warp on the
//    same bank, which bounds it at about 3.5 shared-memory wavefronts per lookup
//    instruction.
// An id outside [0, num_points) yields NaN for that pair and reads nothing.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <string>

#include "quiver_b200.h"

namespace qv {
void set_last_error(const std::string& m);
}

namespace {

constexpr int kPivots = 256;
constexpr float kNaN = __builtin_nanf("");

// ------------------------------------------------------------ arguments --

struct AdcArgs {
  const uint8_t* codes;
  int64_t num_points;
  int32_t M;
  const float* luts;  // [nq][M][256]
  int64_t nq;
  const int32_t* ids;   // [nq][per_q], or null
  const int64_t* first; // [nq] when ids is null
  int64_t per_q;
  float* out;  // [nq][per_q]
  int64_t nchunk;  // work items per query
  int64_t chunk;   // codes per work item (the last one of a query may be shorter)
};

// Code id of pair (q, i); -1 when it is outside [0, num_points).
__device__ __forceinline__ int64_t pair_code(const AdcArgs& a, int64_t q, int64_t i) {
  const int64_t id = a.ids ? static_cast<int64_t>(__ldg(a.ids + q * a.per_q + i)) : __ldg(a.first + q) + i;
  return (id >= 0 && id < a.num_points) ? id : -1;
}

// --------------------------------------------------------- pipe (M == 32) --

// Warps per CTA and ring depth; one CTA per SM, so shared memory bounds their product.
#ifndef QV_ADC_PIPE_WARPS
#define QV_ADC_PIPE_WARPS 16
#endif
#ifndef QV_ADC_PIPE_RING
#define QV_ADC_PIPE_RING 4
#endif
#ifndef QV_ADC_PIPE_COPIES
#define QV_ADC_PIPE_COPIES 4
#endif
constexpr int kPipeWarps = QV_ADC_PIPE_WARPS;
constexpr int kPipeThreads = kPipeWarps * 32;
constexpr int kLutCopies = QV_ADC_PIPE_COPIES;  // 2: two groups share a copy and stagger; 4: one each
constexpr int kLutWords = 32 * kPivots;      // one copy: 256 rows x 32 columns
constexpr int kRingBatches = QV_ADC_PIPE_RING;  // per warp: 32-code batches in shared memory (power of 2)
constexpr int kCodeAhead = kRingBatches - 1; // code batches in flight ahead of the one consumed
constexpr int kIdSlots = kRingBatches;       // per warp: 32-id batches in shared memory
constexpr int kBatchWords = 32 * 8;          // one batch of 32 codes
// Ring slot s sits at words (s + 1) * 256; words 0..255 mirror the last slot, so the batch before slot 0 is
// always the 256 words below it.
constexpr int kRingWords = (kRingBatches + 1) * kBatchWords;
constexpr size_t kLutBytes = (size_t)kLutCopies * kLutWords * 4;
constexpr size_t kRingBytes = (size_t)kPipeWarps * kRingWords * 4;
constexpr size_t kIdBytes = (size_t)kPipeWarps * kIdSlots * 32 * 4;
constexpr size_t kPipeSmem = kLutBytes + kRingBytes + kIdBytes + (size_t)kPipeWarps * kRingBatches * 8;

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool pred) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  const int n = pred ? 4 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// Per-lane constants of the pipe kernel.
struct PipeLane {
  int j, g, rot;
  uint32_t sel[4];   // byte_perm selectors: the chunk byte this lane looks up at lookup e
  uint32_t off4[4];  // byte offset of that chunk's column in the lane's LUT copy
};

// Eight diagonal steps of one 32-code batch.  At step r lane (g, j) adds chunks 4j..4j+3 of its group's code
// m = 8b + r - j to the partial sum lane j - 1 handed over, so a code's sum leaves lane 7 complete and in chunk
// order.  CHECKED: codes of the step may lie outside the warp's range or have bad ids (edge batches).
template <bool CHECKED>
__device__ __forceinline__ void pipe_steps(const PipeLane& L, const unsigned char* lutb, const uint32_t* P,
                                           float* qout, int b, int n, uint2 bprev, uint2 bcur, float& acc) {
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const uint32_t w = P[32 * r];
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      v[e] = *reinterpret_cast<const float*>(lutb + L.off4[e] + (__byte_perm(w, 0, L.sel[e]) << 7));
    const float up = __shfl_up_sync(0xffffffffu, acc, 1, 8);
    float s = (L.j == 0) ? 0.f : up;
    if constexpr (kLutCopies == 4) {
      s = __fadd_rn(s, v[0]);
      s = __fadd_rn(s, v[1]);
      s = __fadd_rn(s, v[2]);
      s = __fadd_rn(s, v[3]);
    } else {
      s = __fadd_rn(s, L.rot ? v[2] : v[0]);
      s = __fadd_rn(s, L.rot ? v[3] : v[1]);
      s = __fadd_rn(s, L.rot ? v[0] : v[2]);
      s = __fadd_rn(s, L.rot ? v[1] : v[3]);
    }
    acc = s;
    if constexpr (CHECKED) {
      const int m = 8 * b + r - L.j;
      if (L.j == 7 && m >= 0 && 4 * m + L.g < n) {
        const uint2 mask = (r == 7) ? bcur : bprev;
        const int p = 4 * (m & 7) + L.g;  // the code's position in its batch
        qout[4 * m + L.g] = (((p < 16 ? mask.x : mask.y) >> (2 * (p & 15))) & 1u) ? kNaN : s;
      }
    } else {
      if (L.j == 7) qout[32 * b - 28 + L.g + 4 * r] = s;
    }
  }
}

__global__ void __launch_bounds__(kPipeThreads, 1) adc_pipe32_kernel(const AdcArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // Lane (g, j) -- group g = lanes 8g..8g+7, j = lane & 7 -- adds chunks 4j..4j+3 of its group's code.
  // Copy c of the LUT holds chunk k of centroid x at word c*8192 + x*32 + ((k + c) & 31).  With four copies
  // group g reads copy g; with two, groups read copy g & 1 and groups 2 and 3 look up their four chunks in the
  // order 2, 3, 0, 1.  Either way the 32 lanes of a lookup instruction hit 32 different banks.
  float* lutc = reinterpret_cast<float*>(smem);
  uint32_t* ring = reinterpret_cast<uint32_t*>(smem + kLutBytes) + warp * kRingWords;
  int32_t* idring = reinterpret_cast<int32_t*>(smem + kLutBytes + kRingBytes) + warp * (kIdSlots * 32);
  uint32_t* badm = reinterpret_cast<uint32_t*>(smem + kLutBytes + kRingBytes + kIdBytes) + warp * 2 * kRingBatches;
  PipeLane L;
  L.j = lane & 7;
  L.g = lane >> 3;
  L.rot = kLutCopies == 4 ? 0 : (L.g >> 1) * 2;
  const int cpy = L.g & (kLutCopies - 1);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int o = (e + L.rot) & 3;
    L.sel[e] = 0x4440u | static_cast<uint32_t>(o);
    L.off4[e] = 4u * static_cast<uint32_t>(cpy * kLutWords + ((4 * L.j + o + cpy) & 31));
  }
  const int64_t items = a.nq * a.nchunk;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int64_t q = it / a.nchunk;
    const int64_t c0 = (it % a.nchunk) * a.chunk;
    const int64_t c1 = min(a.per_q, c0 + a.chunk);
    // This warp's codes: [lo, lo + n) of the query, whole 32-code batches.
    const int64_t nb = (c1 - c0 + 31) / 32;
    const int64_t nbw = (nb + kPipeWarps - 1) / kPipeWarps;
    const int64_t lo = min(c1, c0 + warp * nbw * 32);
    const int n = static_cast<int>(min(c1, lo + nbw * 32) - lo);
    const int nbatch = (n + 31) / 32;
    const int32_t* qids = a.ids ? a.ids + q * a.per_q + lo : nullptr;
    const int64_t qfirst = a.ids ? 0 : __ldg(a.first + q) + lo;
    float* qout = a.out + q * a.per_q + lo;
    // Batch B's ids go to id slot B % kIdSlots, fetched kIdSlots batches before its codes; its codes go to
    // ring slot B % kRingBatches (and to the mirror for the last slot), fetched kCodeAhead batches ahead.
    auto fetch_ids = [&](int B) {
      const int k = B * 32 + lane;
      const bool in = B < nbatch && k < n;
      cp_async4(idring + (B & (kIdSlots - 1)) * 32 + lane, in ? qids + k : a.ids, in);
    };
    // Lane L fetches half L & 1 of codes L / 2 and 16 + L / 2 of the batch, so each cp.async instruction writes
    // 512 contiguous bytes of the ring.  badm[2 * slot + i] gets the ballot of out-of-range ids of codes
    // 16i .. 16i + 15 (code c at bit 2(c - 16i)); those codes read as zeros and their outputs become NaN.
    // A range that lies inside [0, num_points) needs no per-code checks: its codes are read straight from
    // cbase, and no output of it can be NaN.
    const bool plain = qids == nullptr && qfirst >= 0 && qfirst + n <= a.num_points;
    const uint8_t* cbase = plain ? a.codes + qfirst * 32 : a.codes;
    auto fetch_codes = [&](int B) {
      const int slot = B & (kRingBatches - 1);
      if (plain) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int c = 16 * i + (lane >> 1);
          const int k = B * 32 + c;
          const bool in = k < n;
          const uint8_t* src = (in ? cbase + static_cast<int64_t>(k) * 32 : a.codes) + 16 * (lane & 1);
          const int word = c * 8 + 4 * (lane & 1);
          cp_async16(ring + (slot + 1) * kBatchWords + word, src, in);
          if (slot == kRingBatches - 1) cp_async16(ring + word, src, in);
        }
        return;
      }
      uint32_t bad[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int c = 16 * i + (lane >> 1);
        const int k = B * 32 + c;
        const bool in = B < nbatch && k < n;
        int64_t id = -1;
        if (in) id = qids ? static_cast<int64_t>(idring[(B & (kIdSlots - 1)) * 32 + c]) : qfirst + k;
        const bool ok = in && id >= 0 && id < a.num_points;
        const uint8_t* src = (ok ? a.codes + id * 32 : a.codes) + 16 * (lane & 1);
        const int word = c * 8 + 4 * (lane & 1);
        cp_async16(ring + (slot + 1) * kBatchWords + word, src, ok);
        if (slot == kRingBatches - 1) cp_async16(ring + word, src, ok);
        bad[i] = __ballot_sync(0xffffffffu, in && !ok);
      }
      if (lane == 0) {
        badm[2 * slot] = bad[0];
        badm[2 * slot + 1] = bad[1];
      }
    };
    __syncthreads();  // every warp is done with the previous item's LUT
    if (qids) {
      for (int B = 0; B < kIdSlots; ++B) fetch_ids(B);
      cp_async_commit();
    }
    const float* Lq = a.luts + q * kLutWords;
    for (int i = tid; i < kLutWords; i += kPipeThreads) {
      const int k = i & 31, x = i >> 5;
      const float v = __ldg(Lq + k * kPivots + x);
#pragma unroll
      for (int c = 0; c < kLutCopies; ++c) lutc[c * kLutWords + x * 32 + ((k + c) & 31)] = v;
    }
    cp_async_wait<0>();
    __syncthreads();
    // Group k of cp.async copies holds the codes of batch k and the ids of batch k + kIdSlots.
#pragma unroll 1
    for (int B = 0; B < kCodeAhead; ++B) {
      fetch_codes(B);
      if (qids) fetch_ids(B + kIdSlots);
      cp_async_commit();
    }
    const unsigned char* lutb = reinterpret_cast<const unsigned char*>(lutc);
    float acc = 0.f;
#pragma unroll 1
    for (int b = 0; b <= nbatch; ++b) {  // b == nbatch drains the diagonal
      cp_async_wait<kCodeAhead - 1>();
      __syncwarp();
      // Word j of code m of group g sits at ring word 32(m - 8b) + lane past slot b's start (m - 8b in -7..7).
      const uint32_t* P = ring + ((b & (kRingBatches - 1)) + 1) * kBatchWords - 32 * L.j + lane;
      const int sp = (b - 1) & (kRingBatches - 1), sc = b & (kRingBatches - 1);
      const uint2 bprev = (b > 0 && !plain) ? make_uint2(badm[2 * sp], badm[2 * sp + 1]) : make_uint2(0u, 0u);
      const uint2 bcur = plain ? make_uint2(0u, 0u) : make_uint2(badm[2 * sc], badm[2 * sc + 1]);
      if (b >= 1 && b + 2 <= nbatch && (bprev.x | bprev.y | bcur.x | bcur.y) == 0)
        pipe_steps<false>(L, lutb, P, qout, b, n, bprev, bcur, acc);
      else
        pipe_steps<true>(L, lutb, P, qout, b, n, bprev, bcur, acc);
      __syncwarp();
      // Ring slot and id slot of batch b - 1 are free again.
      fetch_codes(b + kCodeAhead);
      if (qids) fetch_ids(b + kCodeAhead + kIdSlots);
      cp_async_commit();
    }
    cp_async_wait<0>();
  }
}

// ---------------------------------------------------- thread (any M) --

constexpr int kThreadThreads = 512;
constexpr int kThreadUnroll = 4;

template <int MC>  // MC == 32: codes read as two 16-byte words; MC == 0: byte loads, any M
__global__ void __launch_bounds__(kThreadThreads) adc_thread_kernel(const AdcArgs a) {
  extern __shared__ __align__(16) float lut[];
  const int tid = threadIdx.x;
  const int M = MC > 0 ? MC : a.M;
  const int lut_words = M * kPivots;
  const int64_t items = a.nq * a.nchunk;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int64_t q = it / a.nchunk;
    const int64_t c0 = (it % a.nchunk) * a.chunk;
    const int64_t c1 = min(a.per_q, c0 + a.chunk);
    __syncthreads();
    const float4* src = reinterpret_cast<const float4*>(a.luts + q * lut_words);
    for (int i = tid; i < lut_words / 4; i += kThreadThreads) reinterpret_cast<float4*>(lut)[i] = __ldg(src + i);
    __syncthreads();
    float* qout = a.out + q * a.per_q;
    for (int64_t b = c0; b < c1; b += static_cast<int64_t>(kThreadThreads) * kThreadUnroll) {
      int64_t id[kThreadUnroll];
#pragma unroll
      for (int u = 0; u < kThreadUnroll; ++u) {
        const int64_t i = b + u * kThreadThreads + tid;
        id[u] = i < c1 ? pair_code(a, q, i) : -2;
      }
      if constexpr (MC == 32) {
        uint4 cw[kThreadUnroll][2];
#pragma unroll
        for (int u = 0; u < kThreadUnroll; ++u)
#pragma unroll
          for (int v = 0; v < 2; ++v)
            cw[u][v] = id[u] >= 0 ? __ldg(reinterpret_cast<const uint4*>(a.codes + id[u] * 32) + v)
                                  : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < kThreadUnroll; ++u) {
          if (id[u] == -2) continue;
          float acc = 0.f;
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const uint4& v = cw[u][k >> 4];
            const uint32_t word = (k & 15) < 4 ? v.x : (k & 15) < 8 ? v.y : (k & 15) < 12 ? v.z : v.w;
            acc = __fadd_rn(acc, lut[k * kPivots + ((word >> ((k & 3) * 8)) & 0xffu)]);
          }
          qout[b + u * kThreadThreads + tid] = id[u] >= 0 ? acc : kNaN;
        }
      } else {
#pragma unroll
        for (int u = 0; u < kThreadUnroll; ++u) {
          if (id[u] == -2) continue;
          float acc = kNaN;
          if (id[u] >= 0) {
            const uint8_t* c = a.codes + id[u] * M;
            acc = 0.f;
            for (int k = 0; k < M; ++k) acc = __fadd_rn(acc, lut[k * kPivots + __ldg(c + k)]);
          }
          qout[b + u * kThreadThreads + tid] = acc;
        }
      }
    }
  }
}

int fail(int code, const std::string& m) {
  qv::set_last_error(m);
  return code;
}

}  // namespace

extern "C" int qv_adc_batch(const uint8_t* d_codes, int64_t num_points, int32_t M, const float* d_luts, int64_t nq,
                            const int32_t* d_ids, const int64_t* d_first, int64_t n_per_query, float* d_out,
                            int32_t kernel, void* stream) {
  if (nq < 0 || n_per_query < 0 || num_points < 0) return fail(QV_ERR_INVALID_ARG, "qv_adc_batch: negative size");
  if (M < 1 || M > 128) return fail(QV_ERR_INVALID_ARG, "qv_adc_batch: M must be in [1, 128]");
  if (kernel < QV_ADC_AUTO || kernel > QV_ADC_PIPE) return fail(QV_ERR_INVALID_ARG, "qv_adc_batch: unknown kernel");
  if (nq == 0 || n_per_query == 0) return QV_OK;
  if (!d_codes || !d_luts || !d_out || (!d_ids && !d_first))
    return fail(QV_ERR_INVALID_ARG, "qv_adc_batch: codes, luts, out and one of ids / first are required");
  if (n_per_query > INT32_MAX / 2) return fail(QV_ERR_INVALID_ARG, "qv_adc_batch: n_per_query too large");
  if ((reinterpret_cast<uintptr_t>(d_luts) & 15) != 0 || (M % 4) != 0)
    return fail(QV_ERR_INVALID_ARG, "qv_adc_batch: luts must be 16-byte aligned and M a multiple of 4");
  const bool codes16 = (reinterpret_cast<uintptr_t>(d_codes) & 15) == 0;
  const bool pipe_ok = M == 32 && codes16;
  if (kernel == QV_ADC_PIPE && !pipe_ok)
    return fail(QV_ERR_UNSUPPORTED, "qv_adc_batch: the pipe kernel needs M == 32 and 16-byte aligned codes");
  // The pipe kernel streams contiguous ranges faster than the thread kernel once an item holds thousands of
  // codes; for gathered ids the thread kernel's 16-byte loads keep more random reads in flight.
  const bool pipe = kernel == QV_ADC_PIPE || (kernel == QV_ADC_AUTO && pipe_ok && !d_ids && n_per_query >= 4096);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return fail(QV_ERR_CUDA, "qv_adc_batch: no CUDA device");
  const void* fn;
  size_t smem;
  int threads;
  if (pipe) {
    fn = reinterpret_cast<const void*>(&adc_pipe32_kernel);
    smem = kPipeSmem;
    threads = kPipeThreads;
  } else {
    fn = M == 32 && codes16 ? reinterpret_cast<const void*>(&adc_thread_kernel<32>)
                            : reinterpret_cast<const void*>(&adc_thread_kernel<0>);
    smem = static_cast<size_t>(M) * kPivots * 4;
    threads = kThreadThreads;
  }
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return fail(QV_ERR_CUDA, "qv_adc_batch: cudaFuncSetAttribute failed");
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem) != cudaSuccess || per_sm < 1)
    return fail(QV_ERR_CUDA, "qv_adc_batch: kernel does not fit on an SM");
  const int64_t slots = static_cast<int64_t>(per_sm) * sms;
  // Split queries into work items: about eight waves of items over the resident CTAs keeps the last wave's
  // idle share small, and items long enough that staging the LUT is a small share of an item.
  const int64_t min_chunk = pipe ? 8192 : 2048;
  int64_t nchunk = std::max<int64_t>(1, (8 * slots + nq - 1) / nq);
  nchunk = std::min<int64_t>(nchunk, std::max<int64_t>(1, n_per_query / min_chunk));
  const int64_t chunk = (n_per_query + nchunk - 1) / nchunk;
  nchunk = (n_per_query + chunk - 1) / chunk;
  const AdcArgs args{d_codes, num_points, M, d_luts, nq, d_ids, d_first, n_per_query, d_out, nchunk, chunk};
  const int64_t grid = std::min<int64_t>(slots, nq * nchunk);
  if (pipe)
    adc_pipe32_kernel<<<static_cast<unsigned>(grid), threads, smem, st>>>(args);
  else if (M == 32 && codes16)
    adc_thread_kernel<32><<<static_cast<unsigned>(grid), threads, smem, st>>>(args);
  else
    adc_thread_kernel<0><<<static_cast<unsigned>(grid), threads, smem, st>>>(args);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(QV_ERR_CUDA, std::string("qv_adc_batch launch: ") + cudaGetErrorString(e));
  return QV_OK;
}
