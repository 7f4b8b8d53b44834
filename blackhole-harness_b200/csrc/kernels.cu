// kernels.cu — the small kernels around the grouped GEMM: the align plan, the
// bit-exact dequantization, the top-k combine, the fp32 -> 16-bit cast and
// the router.
#include <algorithm>
#include <atomic>
#include <mutex>

#include <cub/block/block_scan.cuh>

#include "decode.cuh"
#include "internal.cuh"

namespace hexmoe {

// Device error word: bit flags of DeviceError, set by any kernel of this library.
__device__ int32_t g_dev_err;

int32_t* device_error_word() {
  // per-device cache of the symbol's address; first calls from several host
  // threads serialise on the mutex, later ones read the atomic slot only
  static std::atomic<int32_t*> addr[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  int32_t* a = addr[dev].load(std::memory_order_acquire);
  if (a) return a;
  std::lock_guard<std::mutex> lock(mu);
  a = addr[dev].load(std::memory_order_relaxed);
  if (!a) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dev_err) != cudaSuccess) return nullptr;
    a = static_cast<int32_t*>(p);
    addr[dev].store(a, std::memory_order_release);
  }
  return a;
}

cudaError_t read_device_error(int32_t* value, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(value, g_dev_err, sizeof(int32_t));
  if (e != cudaSuccess || !clear) return e;
  const int32_t z = 0;
  return cudaMemcpyToSymbol(g_dev_err, &z, sizeof(z));
}

// global expert -> (tier << 16) | local; -1 where no tier holds the expert.
__global__ void expert_map_kernel(hexmoe_layer_desc d, int32_t* map) {
  for (int e = threadIdx.x; e < d.num_experts; e += blockDim.x) map[e] = -1;
  __syncthreads();
  for (int t = 0; t < d.num_tiers; ++t)
    for (int i = threadIdx.x; i < d.tiers[t].n; i += blockDim.x) {
      const int g = d.tiers[t].experts[i];
      if (g >= 0 && g < d.num_experts) map[g] = (t << 16) | i;
      else atomicOr(&g_dev_err, kDevErrExpertId);
    }
}

cudaError_t launch_build_expert_map(const hexmoe_layer_desc& d, int32_t* map, cudaStream_t st) {
  expert_map_kernel<<<1, 1024, 0, st>>>(d, map);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// align (runtime/blackhole_runtime/hex_moe.py:201-222), stable.
//
// The slots are cut into contiguous segments, one per warp (one CTA of
// kAlignWarps warps for up to kAlignOneCta slots; beyond that kAlignSeg slots
// per CTA, kAlignSeg / kAlignWarps per warp).  Count: each warp counts its
// segment per expert, 32 slots at a time: the lanes holding the same expert
// are found with one ballot per bit of the id (7 for 96 experts; the cost of
// __match_any_sync grows with the number of distinct values in the warp,
// here nearly 32), and their leader adds the group size to the warp's row of
// hist[warp][E].  Plan: per expert, exclusive prefixes of the counts over
// warps (and CTAs), the expert's total and block count, and an exclusive scan
// of the block counts over experts.  Scatter: each warp walks its segment
// again in order; a slot goes to its expert's run at the warp's running
// position plus its rank among equal lanes of the chunk.  Segments in order,
// chunks in order, lanes in order: the order of a stable sort.  Every warp
// loads kAlignBatch chunks of ids before working through them.
// With several CTAs the three steps are three kernels (count, plan, scatter)
// that hand the per-(CTA, expert) counts and then run offsets over a scratch
// array of CTAs x E int32.
constexpr int kAlignWarps = 16;
constexpr int kAlignBatch = 8;
constexpr int kAlignThreads = kAlignWarps * 32;
constexpr int kAlignMaxExperts = 2048;
constexpr int64_t kAlignOneCta = 8192;   // slots one CTA aligns alone
constexpr int kAlignSeg = 2048;          // slots per CTA beyond that
constexpr int kAlignSmemMax = (kAlignWarps + 2) * kAlignMaxExperts * 4;
using AlignScan = cub::BlockScan<int32_t, kAlignThreads>;

// Lanes whose v equals this lane's (v < 2^nbits): the AND over the id bits of
// the ballot of lanes that agree with this lane on that bit.
__device__ __forceinline__ unsigned equal_lanes(uint32_t v, int nbits) {
  unsigned m = 0xffffffffu;
  for (int b = 0; b < nbits; ++b) {
    const bool bit = (v >> b) & 1u;
    const unsigned bal = __ballot_sync(0xffffffffu, bit);
    m &= bit ? bal : ~bal;
  }
  return m;
}

// Ragged slot space (the expert-parallel receive side): slots form segments of
// seg_len, of which only the first counts[seg] are present; the rest are not
// slots at all (skipped, not errors).  counts == nullptr: every slot present.
struct AlignRagged {
  const int32_t* counts;
  int64_t seg_len;
  int32_t* inv;   // optional [S]: the plan row each slot is scattered to
  __device__ __forceinline__ bool present(int64_t s) const {
    return !counts || (s % seg_len) < __ldg(counts + s / seg_len);
  }
  // [s_begin, s_end) clipped to the present prefix of its segment when it lies
  // in one segment (the several-CTA align's warp ranges always do)
  __device__ __forceinline__ int64_t clip_end(int64_t s_begin, int64_t s_end) const {
    if (!counts || s_begin >= s_end) return s_end;
    const int64_t seg = s_begin / seg_len;
    if ((s_end - 1) / seg_len != seg) return s_end;
    const int64_t e = seg * seg_len + __ldg(counts + seg);
    return e < s_end ? e : s_end;
  }
};

// Expert ids of chunks c0, c0 + 32, ... (kAlignBatch of them) for this lane,
// every load issued before the first is used; -1 past s_end or for an id
// outside 0..E-1 (which also sets the error word).
template <bool I64>
__device__ __forceinline__ void load_ids(const void* ids, int64_t c0, int64_t s_end, int lane, int32_t E,
                                         const AlignRagged& rg, int32_t* dev_err, int32_t (&ev)[kAlignBatch]) {
  int64_t raw[kAlignBatch];
  bool live[kAlignBatch];
#pragma unroll
  for (int u = 0; u < kAlignBatch; ++u) {
    const int64_t s = c0 + u * 32 + lane;
    live[u] = s < s_end && rg.present(s);
    raw[u] = live[u] ? (I64 ? __ldg(static_cast<const int64_t*>(ids) + s)
                            : static_cast<int64_t>(__ldg(static_cast<const int32_t*>(ids) + s)))
                     : -1;
  }
#pragma unroll
  for (int u = 0; u < kAlignBatch; ++u) {
    const bool in_seg = live[u];
    const bool bad = in_seg && (raw[u] < 0 || raw[u] >= E);
    if (bad) atomicOr(dev_err, kDevErrExpertId);
    ev[u] = (in_seg && !bad) ? static_cast<int32_t>(raw[u]) : -1;
  }
}

// Count: my_hist[e] += slots of expert e in [s_begin, s_end).
template <bool I64>
__device__ void warp_count(const void* ids, int64_t s_begin, int64_t s_end, int lane, int32_t E, int id_bits,
                           const AlignRagged& rg, int32_t* my_hist, int32_t* dev_err) {
  s_end = rg.clip_end(s_begin, s_end);
  for (int64_t c0 = s_begin; c0 < s_end; c0 += 32 * kAlignBatch) {
    int32_t ev[kAlignBatch];
    load_ids<I64>(ids, c0, s_end, lane, E, rg, dev_err, ev);
#pragma unroll
    for (int u = 0; u < kAlignBatch; ++u) {
      const int32_t e = ev[u];
      const unsigned peers = equal_lanes(static_cast<uint32_t>(e + 1), id_bits);
      if (e >= 0 && (peers & ((1u << lane) - 1u)) == 0) my_hist[e] += __popc(peers);
      __syncwarp();
    }
  }
}

// Scatter: slot s of expert e goes to sid[my_pos[e] + its rank in the chunk];
// my_pos[e] advances past the chunk's slots of e.
template <bool I64>
__device__ void warp_scatter(const void* ids, int64_t s_begin, int64_t s_end, int lane, int32_t E, int id_bits,
                             const AlignRagged& rg, int32_t* my_pos, int32_t* sid, int32_t* dev_err) {
  s_end = rg.clip_end(s_begin, s_end);
  for (int64_t c0 = s_begin; c0 < s_end; c0 += 32 * kAlignBatch) {
    int32_t ev[kAlignBatch];
    load_ids<I64>(ids, c0, s_end, lane, E, rg, dev_err, ev);
#pragma unroll
    for (int u = 0; u < kAlignBatch; ++u) {
      const int32_t e = ev[u];
      const unsigned peers = equal_lanes(static_cast<uint32_t>(e + 1), id_bits);
      int32_t base = 0;
      if (e >= 0) base = my_pos[e];
      __syncwarp();
      if (e >= 0) {
        const int rank = __popc(peers & ((1u << lane) - 1u));
        sid[base + rank] = static_cast<int32_t>(c0 + u * 32 + lane);
        if (rg.inv) rg.inv[c0 + u * 32 + lane] = base + rank;
        if (rank == 0) my_pos[e] = base + __popc(peers);
      }
      __syncwarp();
    }
  }
}

// Plan from the experts' totals counts[e] (shared memory, thread t holding
// experts t*kPer .. t*kPer+kPer-1): block counts, their exclusive scan into
// blk_start[e] (shared), npp, the expert of every block (-1 past the last)
// and sorted_ids = S on every padding slot.  All threads; blk_start is
// visible to the whole CTA on return.
__device__ void plan_runs(const int32_t* counts, int32_t* blk_start, int64_t S, int32_t E, int32_t bm, int32_t* sid,
                          int32_t* eid, int32_t* npp, typename AlignScan::TempStorage& scan_tmp,
                          int32_t& total_blocks) {
  constexpr int kPer = kAlignMaxExperts / kAlignThreads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int32_t nblk[kPer];
  int32_t local_sum = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = threadIdx.x * kPer + j;
    nblk[j] = e < E ? (counts[e] + bm - 1) / bm : 0;
    local_sum += nblk[j];
  }
  int32_t excl, agg;
  AlignScan(scan_tmp).ExclusiveSum(local_sum, excl, agg);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = threadIdx.x * kPer + j;
    if (e < E) {
      blk_start[e] = excl;
      excl += nblk[j];
    }
  }
  if (threadIdx.x == 0) {
    total_blocks = agg;
    npp[0] = agg * bm;
  }
  __syncthreads();
  const int64_t max_blocks = (S + bm - 1) / bm + (E < S ? E : S);
  for (int e = warp; e < E; e += kAlignWarps) {
    const int32_t b0 = blk_start[e];
    const int32_t nb = (counts[e] + bm - 1) / bm;
    for (int j = lane; j < nb; j += 32) eid[b0 + j] = e;
    for (int64_t i = static_cast<int64_t>(b0) * bm + counts[e] + lane; i < static_cast<int64_t>(b0 + nb) * bm;
         i += 32)
      sid[i] = static_cast<int32_t>(S);
  }
  for (int64_t b = total_blocks + threadIdx.x; b < max_blocks; b += kAlignThreads) eid[b] = -1;
  for (int64_t i = static_cast<int64_t>(total_blocks) * bm + threadIdx.x; i < max_blocks * bm; i += kAlignThreads)
    sid[i] = static_cast<int32_t>(S);
}

// Small batches (decode: up to kAlignSmall slots, up to kAlignSmall experts, no
// ragged slot space): one CTA of kAlignSmall threads, one slot each, with a
// short loop body (a cold kernel of this size is bound by instruction fetch,
// not by its work).  Keys e * 2048 + s are sorted ascending with a bitonic
// network in shared memory, which orders the slots by expert and, within an
// expert, by slot: the same stable order as the kernels below.  A slot's place
// is its expert's first padded row plus its rank among the expert's slots.
constexpr int kAlignSmall = 1024;

// Exclusive prefix sums of a and b over the CTA's threads (in thread order),
// and their totals.  All kAlignSmall threads.
__device__ __forceinline__ void small_scan2(int32_t a, int32_t b, int32_t& ea, int32_t& eb, int32_t& ta, int32_t& tb,
                                            int32_t* wsum) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t ia = a, ib = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t ua = __shfl_up_sync(0xffffffffu, ia, o), ub = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) { ia += ua; ib += ub; }
  }
  if (lane == 31) { wsum[warp] = ia; wsum[32 + warp] = ib; }
  __syncthreads();
  if (warp == 0) {
    int32_t va = wsum[lane], vb = wsum[32 + lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t ua = __shfl_up_sync(0xffffffffu, va, o), ub = __shfl_up_sync(0xffffffffu, vb, o);
      if (lane >= o) { va += ua; vb += ub; }
    }
    wsum[64 + lane] = va;        // inclusive prefix over warps
    wsum[96 + lane] = vb;
  }
  __syncthreads();
  const int32_t wa = warp ? wsum[64 + warp - 1] : 0, wb = warp ? wsum[96 + warp - 1] : 0;
  ea = wa + ia - a;
  eb = wb + ib - b;
  ta = wsum[64 + 31];
  tb = wsum[96 + 31];
}

template <bool I64>
__global__ void __launch_bounds__(kAlignSmall, 1)
    align_small_kernel(const void* __restrict__ ids, int32_t S, int32_t E, int32_t bm, int32_t* __restrict__ sid,
                       int32_t* __restrict__ eid, int32_t* __restrict__ npp, int32_t* dev_err) {
  __shared__ uint32_t key[kAlignSmall];
  __shared__ int32_t cnt[kAlignSmall];      // per expert: slots, then its first place in the sorted keys
  __shared__ int32_t bstart[kAlignSmall];   // per expert: first block
  __shared__ int32_t wsum[128];
  const int t = threadIdx.x;
  pdl_wait();
  cnt[t] = 0;
  __syncthreads();
  uint32_t k = 0xFFFFFFFFu;                 // past every valid key: bad ids sort last and are dropped
  if (t < S) {
    const int64_t v = I64 ? __ldg(static_cast<const int64_t*>(ids) + t)
                          : static_cast<int64_t>(__ldg(static_cast<const int32_t*>(ids) + t));
    if (v < 0 || v >= E) {
      atomicOr(dev_err, kDevErrExpertId);
    } else {
      k = (static_cast<uint32_t>(v) << 11) | static_cast<uint32_t>(t);
      atomicAdd(&cnt[v], 1);
    }
  }
  key[t] = k;
  int n = 1;
  while (n < S) n <<= 1;
  __syncthreads();
#pragma unroll 1
  for (int size = 2; size <= n; size <<= 1) {
#pragma unroll 1
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const int u = t ^ stride;
      if (t < n && u > t) {
        const uint32_t a = key[t], b = key[u];
        if ((a > b) == ((t & size) == 0)) { key[t] = b; key[u] = a; }
      }
      __syncthreads();
    }
  }
  const int32_t c = t < E ? cnt[t] : 0;
  const int32_t nb = (c + bm - 1) / bm;
  int32_t c0, b0, valid, total_blocks;
  small_scan2(c, nb, c0, b0, valid, total_blocks, wsum);
  if (t < E) {
    cnt[t] = c0;
    bstart[t] = b0;
    for (int j = c; j < nb * bm; ++j) sid[b0 * bm + j] = static_cast<int32_t>(S);   // the run's padding
    for (int j = 0; j < nb; ++j) eid[b0 + j] = t;
  }
  __syncthreads();
  if (t < valid) {
    const uint32_t kk = key[t];
    const int e = static_cast<int>(kk >> 11), s = static_cast<int>(kk & 2047u);
    sid[bstart[e] * bm + (t - cnt[e])] = s;
  }
  const int64_t max_blocks = (S + bm - 1) / bm + (E < S ? E : S);
  for (int64_t b = total_blocks + t; b < max_blocks; b += kAlignSmall) eid[b] = -1;
  for (int64_t i = static_cast<int64_t>(total_blocks) * bm + t; i < max_blocks * bm; i += kAlignSmall)
    sid[i] = static_cast<int32_t>(S);
  if (t == 0) npp[0] = total_blocks * bm;
  pdl_launch_dependents();
}

// One CTA: count, plan, scatter.
template <bool I64>
__global__ void __launch_bounds__(kAlignThreads, 1)
    align_kernel(const void* __restrict__ ids, int64_t S, int32_t E, int32_t bm, int32_t* __restrict__ sid,
                 int32_t* __restrict__ eid, int32_t* __restrict__ npp, AlignRagged rg, int32_t* dev_err) {
  extern __shared__ int32_t sh[];
  int32_t* hist = sh;                                  // [kAlignWarps][E]
  int32_t* blk_start = sh + kAlignWarps * E;           // [E]
  int32_t* counts = blk_start + E;                     // [E]
  __shared__ typename AlignScan::TempStorage scan_tmp;
  __shared__ int32_t total_blocks;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int id_bits = 32 - __clz(E);   // bits of e + 1 (0 = no expert), e < E
  pdl_wait();
  for (int i = threadIdx.x; i < kAlignWarps * E; i += kAlignThreads) hist[i] = 0;
  __syncthreads();
  const int64_t seg = (S + kAlignWarps - 1) / kAlignWarps;
  const int64_t s_begin = warp * seg;
  const int64_t s_end = s_begin + seg < S ? s_begin + seg : S;
  warp_count<I64>(ids, s_begin, s_end, lane, E, id_bits, rg, hist + warp * E, dev_err);
  __syncthreads();
  // per expert: exclusive prefix of the warps' counts, and the total
  constexpr int kPer = kAlignMaxExperts / kAlignThreads;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = threadIdx.x * kPer + j;
    if (e < E) {
      int32_t acc = 0;
      for (int w = 0; w < kAlignWarps; ++w) {
        const int32_t v = hist[w * E + e];
        hist[w * E + e] = acc;
        acc += v;
      }
      counts[e] = acc;
    }
  }
  plan_runs(counts, blk_start, S, E, bm, sid, eid, npp, scan_tmp, total_blocks);
  for (int i = threadIdx.x; i < kAlignWarps * E; i += kAlignThreads) hist[i] += blk_start[i % E] * bm;
  __syncthreads();
  warp_scatter<I64>(ids, s_begin, s_end, lane, E, id_bits, rg, hist + warp * E, sid, dev_err);
  pdl_launch_dependents();
}

// Several CTAs, step 1: cnt[g][e] = slots of expert e in CTA g's segment.
template <bool I64>
__global__ void __launch_bounds__(kAlignThreads, 1)
    align_count_kernel(const void* __restrict__ ids, int64_t S, int32_t E, int32_t* __restrict__ cnt,
                       AlignRagged rg, int32_t* dev_err) {
  extern __shared__ int32_t hist[];                    // [kAlignWarps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int id_bits = 32 - __clz(E);
  pdl_wait();
  for (int i = threadIdx.x; i < kAlignWarps * E; i += kAlignThreads) hist[i] = 0;
  __syncthreads();
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kAlignSeg, r1 = r0 + kAlignSeg < S ? r0 + kAlignSeg : S;
  const int64_t s_begin = r0 + warp * (kAlignSeg / kAlignWarps);
  const int64_t s_end = s_begin + kAlignSeg / kAlignWarps < r1 ? s_begin + kAlignSeg / kAlignWarps : r1;
  warp_count<I64>(ids, s_begin, s_end, lane, E, id_bits, rg, hist + warp * E, dev_err);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kAlignThreads) {
    int32_t acc = 0;
    for (int w = 0; w < kAlignWarps; ++w) acc += hist[w * E + e];
    cnt[static_cast<int64_t>(blockIdx.x) * E + e] = acc;
  }
  pdl_launch_dependents();
}

// Step 2 (one CTA): the plan, and cnt[g][e] := sorted_ids position of CTA
// g's first slot of expert e.
__global__ void __launch_bounds__(kAlignThreads, 1)
    align_plan_kernel(int32_t* __restrict__ cnt, int32_t G, int64_t S, int32_t E, int32_t bm,
                      int32_t* __restrict__ sid, int32_t* __restrict__ eid, int32_t* __restrict__ npp) {
  extern __shared__ int32_t sh[];
  int32_t* blk_start = sh;                             // [E]
  int32_t* counts = sh + E;                            // [E]
  __shared__ typename AlignScan::TempStorage scan_tmp;
  __shared__ int32_t total_blocks;
  pdl_wait();
  constexpr int kPer = kAlignMaxExperts / kAlignThreads;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = threadIdx.x * kPer + j;
    if (e < E) {
      int32_t acc = 0;
      for (int g0 = 0; g0 < G; g0 += 16) {
        // sixteen CTAs' counts loaded before any is rewritten: loads in flight, not one at a time
        int32_t v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) v[u] = g0 + u < G ? cnt[static_cast<int64_t>(g0 + u) * E + e] : 0;
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          if (g0 + u < G) cnt[static_cast<int64_t>(g0 + u) * E + e] = acc;
          acc += v[u];
        }
      }
      counts[e] = acc;
    }
  }
  plan_runs(counts, blk_start, S, E, bm, sid, eid, npp, scan_tmp, total_blocks);
  for (int64_t i = threadIdx.x; i < static_cast<int64_t>(G) * E; i += kAlignThreads)
    cnt[i] += blk_start[i % E] * bm;
  pdl_launch_dependents();
}

// Step 3: each CTA scatters its segment from its run offsets.
template <bool I64>
__global__ void __launch_bounds__(kAlignThreads, 1)
    align_scatter_kernel(const void* __restrict__ ids, int64_t S, int32_t E, const int32_t* __restrict__ off,
                         int32_t* __restrict__ sid, AlignRagged rg, int32_t* dev_err) {
  extern __shared__ int32_t hist[];                    // [kAlignWarps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int id_bits = 32 - __clz(E);
  pdl_wait();
  for (int i = threadIdx.x; i < kAlignWarps * E; i += kAlignThreads) hist[i] = 0;
  __syncthreads();
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kAlignSeg, r1 = r0 + kAlignSeg < S ? r0 + kAlignSeg : S;
  const int64_t s_begin = r0 + warp * (kAlignSeg / kAlignWarps);
  const int64_t s_end = s_begin + kAlignSeg / kAlignWarps < r1 ? s_begin + kAlignSeg / kAlignWarps : r1;
  warp_count<I64>(ids, s_begin, s_end, lane, E, id_bits, rg, hist + warp * E, dev_err);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kAlignThreads) {
    int32_t pos = off[static_cast<int64_t>(blockIdx.x) * E + e];
    for (int w = 0; w < kAlignWarps; ++w) {
      const int32_t v = hist[w * E + e];
      hist[w * E + e] = pos;
      pos += v;
    }
  }
  __syncthreads();
  warp_scatter<I64>(ids, s_begin, s_end, lane, E, id_bits, rg, hist + warp * E, sid, dev_err);
  pdl_launch_dependents();
}

size_t align_scratch_bytes(int64_t S, int32_t E) {
  if (S <= kAlignOneCta) return 0;
  const int64_t G = (S + kAlignSeg - 1) / kAlignSeg;
  return static_cast<size_t>((G * E * 4 + 255) / 256 * 256);
}

cudaError_t launch_align(const void* ids, bool ids64, int64_t S, int32_t E, int32_t bm, int32_t* sid, int32_t* eid,
                         int32_t* npp, int32_t* scratch, size_t scratch_bytes, int32_t* dev_err, cudaStream_t st,
                         bool pdl, const int32_t* seg_counts, int64_t seg_len, int32_t* inv) {
  const AlignRagged rg{seg_counts, seg_counts ? seg_len : 1, inv};
  if (E > kAlignMaxExperts) return cudaErrorInvalidValue;
  static std::atomic<bool> configured[64] = {};   // per device
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev].load(std::memory_order_relaxed)) {
      const void* kerns[] = {reinterpret_cast<const void*>(align_kernel<true>),
                             reinterpret_cast<const void*>(align_kernel<false>),
                             reinterpret_cast<const void*>(align_count_kernel<true>),
                             reinterpret_cast<const void*>(align_count_kernel<false>),
                             reinterpret_cast<const void*>(align_scatter_kernel<true>),
                             reinterpret_cast<const void*>(align_scatter_kernel<false>)};
      for (const void* k : kerns) {
        e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kAlignSmemMax);
        if (e != cudaSuccess) return e;
      }
      configured[dev].store(true, std::memory_order_release);
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kAlignThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const size_t hist_bytes = static_cast<size_t>(kAlignWarps) * E * sizeof(int32_t);
  const size_t need = align_scratch_bytes(S, E);
  if (!seg_counts && !inv && S <= kAlignSmall && E <= kAlignSmall) {
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kAlignSmall);
    const int32_t S32 = static_cast<int32_t>(S);
    return ids64 ? cudaLaunchKernelEx(&cfg, align_small_kernel<true>, ids, S32, E, bm, sid, eid, npp, dev_err)
                 : cudaLaunchKernelEx(&cfg, align_small_kernel<false>, ids, S32, E, bm, sid, eid, npp, dev_err);
  }
  if (need == 0 || !scratch || scratch_bytes < need) {
    cfg.gridDim = dim3(1);
    cfg.dynamicSmemBytes = hist_bytes + 2 * E * sizeof(int32_t);
    return ids64 ? cudaLaunchKernelEx(&cfg, align_kernel<true>, ids, S, E, bm, sid, eid, npp, rg, dev_err)
                 : cudaLaunchKernelEx(&cfg, align_kernel<false>, ids, S, E, bm, sid, eid, npp, rg, dev_err);
  }
  const int32_t G = static_cast<int32_t>((S + kAlignSeg - 1) / kAlignSeg);
  cfg.gridDim = dim3(G);
  cfg.dynamicSmemBytes = hist_bytes;
  e = ids64 ? cudaLaunchKernelEx(&cfg, align_count_kernel<true>, ids, S, E, scratch, rg, dev_err)
            : cudaLaunchKernelEx(&cfg, align_count_kernel<false>, ids, S, E, scratch, rg, dev_err);
  if (e != cudaSuccess) return e;
  cfg.numAttrs = 1;   // the next two follow kernels of this library
  cfg.gridDim = dim3(1);
  cfg.dynamicSmemBytes = 2 * E * sizeof(int32_t);
  e = cudaLaunchKernelEx(&cfg, align_plan_kernel, scratch, G, S, E, bm, sid, eid, npp);
  if (e != cudaSuccess) return e;
  cfg.gridDim = dim3(G);
  cfg.dynamicSmemBytes = hist_bytes;
  return ids64 ? cudaLaunchKernelEx(&cfg, align_scatter_kernel<true>, ids, S, E, static_cast<const int32_t*>(scratch),
                                    sid, rg, dev_err)
               : cudaLaunchKernelEx(&cfg, align_scatter_kernel<false>, ids, S, E,
                                    static_cast<const int32_t*>(scratch), sid, rg, dev_err);
}

// ---------------------------------------------------------------------------
// Dequantization (blackhole/anatomy/hex.py:180-204; the reference kernel is
// _hex_dequant_kernel, runtime/blackhole_runtime/hex_moe.py:154-168).  One
// thread per (expert, row, 32-input block): w = levels[code] * (fp8 * es),
// both products rounded to nearest in fp32, then to the output type.
template <int OUT>  // HEXMOE_F32 / HEXMOE_BF16 / HEXMOE_F16
__global__ void dequant_kernel(hexmoe_parts parts, int bits, int block, int n, int rows, int cols, int rows_pad,
                               int cols_pad, const int32_t* __restrict__ experts, void* __restrict__ out,
                               int64_t stride_e, int64_t stride_row, int64_t row_off) {
  const int nblk = cols / 32;
  const int64_t total = static_cast<int64_t>(n) * rows * nblk;
  const int wpr = cols_pad / 32 * bits;
  const int spr = cols_pad / block;
  const int L = 1 << bits;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int blk = static_cast<int>(i % nblk);
    const int64_t er = i / nblk;
    const int o = static_cast<int>(er % rows);
    const int e = static_cast<int>(er / rows);
    const int64_t rrow = static_cast<int64_t>(e) * rows_pad + o;
    const uint32_t* wp = parts.idx + rrow * wpr + blk * bits;
    uint32_t w[4];
    for (int j = 0; j < bits; ++j) w[j] = __ldg(wp + j);
    const uint32_t code = __ldg(parts.block_scale + rrow * spr + (blk * 32) / block);
    const float s = __fmul_rn(fp8_hex_value(code), __ldg(parts.expert_scale + e));
    const float* lev = parts.levels + static_cast<int64_t>(e) * L;
    const int ge = experts ? __ldg(experts + e) : e;
    char* dst = static_cast<char*>(out);
    const int64_t base = ge * stride_e + (row_off + o) * stride_row + static_cast<int64_t>(blk) * 32;
#pragma unroll 4
    for (int j = 0; j < 32; ++j) {
      const int off = j * bits;
      const int wi = off >> 5, sh = off & 31;
      uint32_t v = w[wi] >> sh;
      if (sh + bits > 32) v |= w[wi + 1] << (32 - sh);
      const float val = __fmul_rn(__ldg(lev + (v & (L - 1))), s);
      if (OUT == HEXMOE_F32) reinterpret_cast<float*>(dst)[base + j] = val;
      else if (OUT == HEXMOE_BF16) reinterpret_cast<__nv_bfloat16*>(dst)[base + j] = __float2bfloat16_rn(val);
      else reinterpret_cast<__half*>(dst)[base + j] = __float2half_rn(val);
    }
  }
}

cudaError_t launch_dequant(const hexmoe_parts& parts, int bits, int block, int n, int rows, int cols, int rows_pad,
                           int cols_pad, const int32_t* experts, void* out, int out_dtype, int64_t stride_e,
                           int64_t stride_row, int64_t row_off, cudaStream_t st) {
  const int64_t total = static_cast<int64_t>(n) * rows * (cols / 32);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t want = (total + threads - 1) / threads;
  const int grid = static_cast<int>(want < 148 * 16 ? want : 148 * 16);
  if (out_dtype == HEXMOE_F32)
    dequant_kernel<HEXMOE_F32><<<grid, threads, 0, st>>>(parts, bits, block, n, rows, cols, rows_pad, cols_pad,
                                                         experts, out, stride_e, stride_row, row_off);
  else if (out_dtype == HEXMOE_BF16)
    dequant_kernel<HEXMOE_BF16><<<grid, threads, 0, st>>>(parts, bits, block, n, rows, cols, rows_pad, cols_pad,
                                                          experts, out, stride_e, stride_row, row_off);
  else
    dequant_kernel<HEXMOE_F16><<<grid, threads, 0, st>>>(parts, bits, block, n, rows, cols, rows_pad, cols_pad,
                                                         experts, out, stride_e, stride_row, row_off);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Tiled index copy (hexmoe_tile_index): one thread per output word, in output
// order (coalesced stores).  Output word o = (((((e * m_tiles + m) * ksteps +
// s) * 4 + h) * 4 + b) * 32 + p) * 4 + j holds, one per nibble, the 8 codes of
// inputs s*128 + b*32 + j*8 .. +7 of row m*128 + h*32 + (p ^ 2b) of expert e.
// A 128-row step is 8 KB of contiguous memory and so is each 32-row slice h of
// it (2 KB), so a kernel can stream tiles of 32, 64 or 128 rows with one copy
// per step; within block b of a slice the rows are permuted by flipping bits
// 1-2 of the row index with b, so that a kernel reading rows g (+ 8i) of blocks
// 0..3 at once (lane = (g, b)) hits 8 distinct shared-memory bank groups per
// quarter warp, while the 32 rows of one block stay 32 consecutive 16-byte
// chunks.
// A stored 32-input
// block is `bits` little-endian words with code i at bits [i*bits, i*bits+bits)
// (hex_ref.pack, hex_ref.py:49-61): 4-bit words are already nibble-packed;
// 3-bit word j is the 24 bits from bit 24*j, which never reach past the
// block's third word.
__global__ void tile_index_kernel(const uint32_t* __restrict__ idx, int bits, int rows_pad, int cols_pad,
                                  int64_t total, uint32_t* __restrict__ out) {
  const int m_tiles = rows_pad / 128, ksteps = cols_pad / 128;
  const int64_t wpr = static_cast<int64_t>(cols_pad) / 32 * bits;
  for (int64_t o = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; o < total;
       o += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(o & 3), b = static_cast<int>((o >> 7) & 3);
    const int r = static_cast<int>(((o >> 9) & 3) * 32 + (((o >> 2) & 31) ^ (2 * b)));   // the row stored here
    const int64_t rest = o >> 11;
    const int s = static_cast<int>(rest % ksteps);
    const int64_t em = rest / ksteps;
    const int m = static_cast<int>(em % m_tiles);
    const int64_t e = em / m_tiles;
    const uint32_t* src = idx + (e * rows_pad + m * 128 + r) * wpr + static_cast<int64_t>(s * 4 + b) * bits;
    uint32_t w;
    if (bits == 4) {
      w = __ldg(src + j);
    } else {
      const int start = 24 * j, wi = start >> 5, sh = start & 31;
      uint32_t v = __ldg(src + wi) >> sh;
      if (sh + 24 > 32) v |= __ldg(src + wi + 1) << (32 - sh);
      w = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) w |= ((v >> (3 * i)) & 7u) << (4 * i);
    }
    out[o] = w;
  }
}

cudaError_t launch_tile_index(const uint32_t* idx, int bits, int n, int rows_pad, int cols_pad, uint32_t* out,
                              cudaStream_t st) {
  const int64_t total = static_cast<int64_t>(n) * rows_pad * cols_pad / 8;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int grid = static_cast<int>(std::min<int64_t>((total + threads - 1) / threads, 148 * 32));
  tile_index_kernel<<<grid, threads, 0, st>>>(idx, bits, rows_pad, cols_pad, total, out);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Combine (runtime/blackhole_runtime/hex_moe.py:325, y.view(T, k, H).sum(1)):
// out[t, h] = sum_j y[r(t, j), h], fp32 accumulation in slot order, with
// r(t, j) = t*k + j, or rows[t*k + j] when a row map is given (the expert-
// parallel combine, whose rows come back in dispatch order); a mapped row
// outside 0..y_rows-1 adds nothing and sets the error word.
template <typename YT, int OUT>
__global__ void combine_kernel(const YT* __restrict__ y, int64_t T, int32_t k, int32_t H, int64_t ld_y,
                               const int32_t* __restrict__ rows, int64_t y_rows, void* __restrict__ out) {
  pdl_wait();
  const int hv = H / 8;
  const int64_t total = T * hv;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / hv;
    const int h8 = static_cast<int>(i % hv) * 8;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j0 = 0; j0 < k; j0 += 8) {
      // up to 8 rows loaded before the first is added (loads in flight together), added in slot order
      uint4 v[8];
      bool ok[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + u;
        int64_t r = t * k + j;
        ok[u] = j < k;
        if (ok[u] && rows) {
          r = __ldg(rows + r);
          if (r < 0 || r >= y_rows) {
            if (h8 == 0) atomicOr(&g_dev_err, kDevErrExpertId);
            ok[u] = false;
          }
        }
        v[u] = ok[u] ? *reinterpret_cast<const uint4*>(y + r * ld_y + h8) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (!ok[u]) continue;
        const YT* e = reinterpret_cast<const YT*>(&v[u]);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += static_cast<float>(e[q]);
      }
    }
    const int64_t o = t * H + h8;
    if (OUT == HEXMOE_F32) {
      float4* d = reinterpret_cast<float4*>(static_cast<float*>(out) + o);
      d[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      d[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
      uint4 r;
      uint32_t* rr = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
      for (int q = 0; q < 4; ++q) rr[q] = pack2<OUT == HEXMOE_BF16>(acc[2 * q], acc[2 * q + 1]);
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + o) = r;
    }
  }
}

template <typename YT>
static cudaError_t combine_dispatch(const YT* y, int64_t T, int32_t k, int32_t H, int64_t ld_y,
                                    const int32_t* rows, int64_t y_rows, void* out, int out_dtype, cudaStream_t st,
                                    bool pdl) {
  const int64_t total = T * (H / 8);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t want = (total + threads - 1) / threads;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(want < 148 * 8 ? want : 148 * 8));
  cfg.blockDim = dim3(threads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (out_dtype == HEXMOE_F32)
    return cudaLaunchKernelEx(&cfg, combine_kernel<YT, HEXMOE_F32>, y, T, k, H, ld_y, rows, y_rows, out);
  if (out_dtype == HEXMOE_BF16)
    return cudaLaunchKernelEx(&cfg, combine_kernel<YT, HEXMOE_BF16>, y, T, k, H, ld_y, rows, y_rows, out);
  return cudaLaunchKernelEx(&cfg, combine_kernel<YT, HEXMOE_F16>, y, T, k, H, ld_y, rows, y_rows, out);
}

cudaError_t launch_combine(const void* y, int y_dtype, int64_t T, int32_t topk, int32_t H, int64_t ld_y,
                           const int32_t* rows, int64_t y_rows, void* out, int out_dtype, cudaStream_t st, bool pdl) {
  if (y_dtype == HEXMOE_BF16)
    return combine_dispatch(static_cast<const __nv_bfloat16*>(y), T, topk, H, ld_y, rows, y_rows, out, out_dtype, st,
                            pdl);
  return combine_dispatch(static_cast<const __half*>(y), T, topk, H, ld_y, rows, y_rows, out, out_dtype, st, pdl);
}

// ---------------------------------------------------------------------------
// Plan-ordered activations: xs[r] = x[sorted_ids[r] / topk] (one warp per row,
// 16-byte vectors), so the grouped GEMM loads each block's tokens as one TMA
// box instead of one gather per token.  f32 input is rounded to bf16 here.
template <typename XT>
__global__ void gather_rows_kernel(const XT* __restrict__ x, int32_t H, const int32_t* __restrict__ sid,
                                   const int32_t* __restrict__ npp, int64_t max_rows, int32_t topk, int64_t S,
                                   const int32_t* __restrict__ slot_row, uint16_t* __restrict__ xs) {
  pdl_wait();
  const int64_t rows = min(static_cast<int64_t>(__ldg(npp)), max_rows);
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; r < rows; r += nwarps) {
    const int s = __ldg(sid + r);
    if (s >= S) continue;
    const int64_t xr = slot_row ? static_cast<int64_t>(__ldg(slot_row + s)) : static_cast<int64_t>(s / topk);
    const XT* src = x + xr * H;
    uint4* dst = reinterpret_cast<uint4*>(xs + r * H);
    for (int c = lane; c < H / 8; c += 32) {
      if constexpr (sizeof(XT) == 2) {
        dst[c] = __ldg(reinterpret_cast<const uint4*>(src) + c);
      } else {
        const float4 a = __ldg(reinterpret_cast<const float4*>(src) + 2 * c);
        const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 2 * c + 1);
        dst[c] = make_uint4(pack2<true>(a.x, a.y), pack2<true>(a.z, a.w), pack2<true>(b.x, b.y),
                            pack2<true>(b.z, b.w));
      }
    }
  }
  pdl_launch_dependents();
}

cudaError_t launch_gather_rows(const void* x, int x_dtype, int64_t T, int32_t H, const int32_t* sid,
                               const int32_t* npp, int64_t max_rows, int32_t topk, int64_t S, void* xs,
                               cudaStream_t st, bool pdl, const int32_t* slot_row) {
  (void)T;
  if (max_rows == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t warps = max_rows < 148 * 64 ? max_rows : 148 * 64;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((warps * 32 + threads - 1) / threads));
  cfg.blockDim = dim3(threads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  uint16_t* out = static_cast<uint16_t*>(xs);
  if (x_dtype == HEXMOE_F32)
    return cudaLaunchKernelEx(&cfg, gather_rows_kernel<float>, static_cast<const float*>(x), H, sid, npp, max_rows,
                              topk, S, slot_row, out);
  return cudaLaunchKernelEx(&cfg, gather_rows_kernel<uint16_t>, static_cast<const uint16_t*>(x), H, sid, npp,
                            max_rows, topk, S, slot_row, out);
}

// ---------------------------------------------------------------------------
__global__ void cast_kernel(const float* __restrict__ x, uint16_t* __restrict__ out, bool bf16, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (bf16) {
      const __nv_bfloat16 v = __float2bfloat16_rn(x[i]);
      out[i] = *reinterpret_cast<const uint16_t*>(&v);
    } else {
      const __half v = __float2half_rn(x[i]);
      out[i] = *reinterpret_cast<const uint16_t*>(&v);
    }
  }
}

cudaError_t launch_cast_to16(const float* x, void* out, bool bf16, int64_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  const int64_t want = (n + 255) / 256;
  cast_kernel<<<static_cast<unsigned>(want < 148 * 8 ? want : 148 * 8), 256, 0, st>>>(
      x, static_cast<uint16_t*>(out), bf16, n);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Router: one warp per token.  softmax in fp32, then k rounds of a warp-wide
// arg-max (ties -> lower expert id), optional renormalisation.
template <int DT>
__global__ void route_topk_kernel(const void* __restrict__ logits, int64_t T, int32_t E, int32_t k, int renorm,
                                  float* __restrict__ w, int32_t* __restrict__ ids) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  if (t >= T) return;
  auto logit = [&](int e) -> float {
    const int64_t i = t * E + e;
    if (DT == HEXMOE_F32) return static_cast<const float*>(logits)[i];
    if (DT == HEXMOE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(logits)[i]);
    return __half2float(static_cast<const __half*>(logits)[i]);
  };
  float m = -INFINITY;
  for (int e = lane; e < E; e += 32) m = fmaxf(m, logit(e));
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float sum = 0.f;
  for (int e = lane; e < E; e += 32) sum += expf(logit(e) - m);
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.0f / sum;
  // k rounds; experts already chosen are skipped by id (k <= 32)
  float picked_w[32];
  int picked_id[32];
  float wsum = 0.f;
  for (int r = 0; r < k; ++r) {
    float best = -INFINITY;
    int bid = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      bool used = false;
      for (int q = 0; q < r; ++q) used |= picked_id[q] == e;
      if (used) continue;
      const float v = logit(e);
      if (v > best || (v == best && e < bid)) { best = v; bid = e; }
    }
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bid, o);
      if (ob > best || (ob == best && oi < bid)) { best = ob; bid = oi; }
    }
    picked_id[r] = bid;
    picked_w[r] = expf(best - m) * inv;
    wsum += picked_w[r];
  }
  if (lane == 0) {
    for (int r = 0; r < k; ++r) {
      w[t * k + r] = renorm ? picked_w[r] / wsum : picked_w[r];
      ids[t * k + r] = picked_id[r];
    }
  }
}

cudaError_t launch_route_topk(const void* logits, int dtype, int64_t T, int32_t E, int32_t k, int renorm, float* w,
                              int32_t* ids, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  const int threads = 256;
  const unsigned grid = static_cast<unsigned>((T * 32 + threads - 1) / threads);
  if (dtype == HEXMOE_F32) route_topk_kernel<HEXMOE_F32><<<grid, threads, 0, st>>>(logits, T, E, k, renorm, w, ids);
  else if (dtype == HEXMOE_BF16)
    route_topk_kernel<HEXMOE_BF16><<<grid, threads, 0, st>>>(logits, T, E, k, renorm, w, ids);
  else route_topk_kernel<HEXMOE_F16><<<grid, threads, 0, st>>>(logits, T, E, k, renorm, w, ids);
  return cudaGetLastError();
}

}  // namespace hexmoe

namespace hexmoe {

// ---------------------------------------------------------------------------
// Code tables of one projection of a tier (layer create): for expert e and fp8
// scale code c, the expert's level table times fp8(c) * expert_scale[e],
// rounded to the operand type, as byte planes (decode.cuh Table8 / Table16):
// out[e * 256 + c] (3-bit) or out[e * 512 + c] and out[e * 512 + 256 + c]
// (4-bit: entries 0-7 / 8-15 low planes, then high planes).  The same values
// the grouped GEMM builds per tile: T[l] = rne16(levels[l] * (fp8(c) * es)).
template <bool BF16>
__global__ void code_table_kernel(const float* __restrict__ levels, const float* __restrict__ es, int bits, int n,
                                  uint4* __restrict__ out) {
  const int L = 1 << bits;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * 256; i += gridDim.x * blockDim.x) {
    const int e = i >> 8, c = i & 255;
    const float s = __fmul_rn(fp8_hex_value(static_cast<uint32_t>(c)), __ldg(es + e));
    const float* lev = levels + static_cast<int64_t>(e) * L;
    float lv[16];
    for (int l = 0; l < L; ++l) lv[l] = __ldg(lev + l);
    if (bits == 3) {
      const Table8 t = make_table8<BF16>(lv, s);
      out[static_cast<int64_t>(e) * 256 + c] = make_uint4(t.l0, t.l1, t.h0, t.h1);
    } else {
      const Table16 t = make_table16<BF16>(lv, s);
      out[static_cast<int64_t>(e) * 512 + c] = make_uint4(t.la0, t.la1, t.lb0, t.lb1);
      out[static_cast<int64_t>(e) * 512 + 256 + c] = make_uint4(t.ha0, t.ha1, t.hb0, t.hb1);
    }
  }
}

cudaError_t launch_code_tables(const float* levels, const float* es, int bits, int n, bool bf16, uint4* out,
                               cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int threads = 256;
  const int grid = std::min(n, 148 * 4);
  if (bf16) code_table_kernel<true><<<grid, threads, 0, st>>>(levels, es, bits, n, out);
  else code_table_kernel<false><<<grid, threads, 0, st>>>(levels, es, bits, n, out);
  return cudaGetLastError();
}

}  // namespace hexmoe
