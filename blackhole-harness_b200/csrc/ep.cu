// ep.cu — expert parallelism for the HEX MoE layer over peer memory
// (hexmoe_ep_*).  The reference runs one GPU and refuses expert parallelism
// (runtime/blackhole_runtime/vllm_hex.py:101-102); this is new work.
//
// Experts are sharded contiguously: rank r owns global experts [r*P, (r+1)*P),
// P = ceil(E / world).  Every rank owns one region of device memory that it
// exports by CUDA IPC and every other rank maps, so kernels on any rank load
// from and store into any rank's region over NVLink (plain loads and stores
// from SMs):
//
//   flags      disp[world], ret[world] (uint64): the epoch a source's dispatch /
//              a destination's return has completed, written with release
//              stores at system scope, polled with acquire loads
//   counts     rows[world], slots[world]: what each source sent this epoch
//   xcopy      [cap][H] 16-bit: this rank's own token rows (the owners of
//              their experts pull them from here)
//   rowslot    [world][cap+1] int32: per row received from a source (one per
//              token of it with a slot here, in token order), its first slot
//              in the source's segment; entry rows[src] = slots[src]
//   rowtok     [world][cap] int32: per received row, the source's token index
//   rec_exp    [world][seg_len] int32: per received slot, its global expert
//   rec_w      [world][seg_len] f32:   per received slot, its top-k weight
//   rec_dst    [world][seg_len] int32: per received slot, where its output row
//              goes: src * cap * topk + t * topk + j (token t's j-th slot at
//              source src)
//   ret        [cap * topk][H] 16-bit: the per-slot output rows of this rank's
//              tokens, row t * topk + j, stored by whichever rank owns the
//              slot's expert
//
// One forward, all on the caller's stream, no host synchronisation:
//   plan      (a CTA per 256 tokens) per token and destination rank, the row
//             position and the first slot offset (stable scans over tokens);
//             the last CTA adds up the CTAs' totals and advances the epoch
//   send      (all SMs) each token row copied into this rank's own xcopy, and
//             its slot and row records stored into every rank that owns one
//             of its experts; the last CTA writes the counts and raises
//             disp[me] = epoch on every rank
//   wait      (1 CTA) disp[src] >= epoch for every source (bounded)
//   experts   the layer over the received slots: align over the ragged slot
//             space (which also records each slot's plan row), then the pull
//             gather (a warp per received row: the row loaded once from its
//             source's xcopy over NVLink and stored to the plan rows of all its
//             slots here), gate/up, down; the down GEMM's
//             epilogue stores each slot's row (top-k weight applied, rounded
//             once) straight into its source's ret over NVLink, so the return
//             runs under the GEMM, and every thread ends with a system fence
//   signal    (1 CTA) ret flag[me] = epoch on every rank
//   wait      ret flag[d] >= epoch for every destination (bounded)
//   combine   out[t] = sum over j of ret[t * topk + j] in fp32, rounded once:
//             the single-GPU layer's combine over the same per-slot rows, so
//             the output equals the single-GPU layer's bit for bit
//
// Buffers are single: a source rewrites its xcopy and rank d's records for
// epoch e only after its own combine of epoch e-1 saw d's return flag of e-1,
// which d raised after its down GEMM of e-1 (after d's gather had read xcopy,
// and the last reader of the records) had finished; and d writes a source's ret
// for epoch e only after it saw that source's dispatch of e, issued after the
// source's combine of e-1 had read ret.  So every rank must
// run every forward (the same sequence of calls on every rank).  Every wait is
// bounded (2 s): a missing peer sets the device error word (timeout) instead of
// hanging the GPU.
#include <algorithm>
#include <cstring>
#include <type_traits>

#include "decode.cuh"
#include "internal.cuh"

namespace hexmoe {

constexpr int kEpMaxWorld = HEXMOE_EP_MAX_WORLD;
constexpr uint64_t kEpWaitNs = 2000000000ull;

struct EpArgs {
  uint8_t* peer[kEpMaxWorld];   // every rank's region base (own included)
  uint8_t* self;
  int32_t rank, world, E, P, H, topk;
  int64_t cap, seg_len;
  // region offsets
  uint64_t o_disp, o_ret_flag, o_rows, o_slots, o_xcopy, o_rowslot, o_rowtok, o_exp, o_w, o_dst, o_ret;
  // this rank's private state
  int64_t* epoch;
  uint32_t* done;               // [3]: CTAs finished in send / return / plan
  int32_t* tot;                 // [world][2]: rows and slots sent to every rank
  int32_t* pos;                 // [cap][world]: token t's row position at rank d within its plan CTA, -1 = none
  int32_t* soff;                // [cap][world]: first slot offset of token t at rank d within its plan CTA
  int64_t* plan_tot;            // [plan CTAs][kEpMaxWorld]: each plan CTA's totals (rows << 32 | slots)
  int64_t* plan_off;            // [plan CTAs][kEpMaxWorld]: their exclusive offsets over CTAs
  int32_t* cmap;                // [cap * topk]: the combine's row of slot (t, j): t * topk + j, -1 = bad expert id
  int32_t* inv;                 // [world * seg_len]: the plan row of every received slot (written by the align)
  int32_t* dev_err;
};

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

template <typename T>
__device__ __forceinline__ T* at(uint8_t* base, uint64_t off) {
  return reinterpret_cast<T*>(base + off);
}

// ---------------------------------------------------------------- plan
// One thread per token, kPlanThreads tokens per CTA, many CTAs.  Per token and
// destination rank d: c = (1 << 32 | slots) when the token has slots at d, else
// 0.  Each CTA scans c over its tokens (exclusive, per d) into the token's
// local row position and first slot offset, and stores its totals; the last
// CTA to finish turns the totals into per-CTA offsets (exclusive over CTAs, so
// token order is kept), the per-rank totals, and advances the epoch.  The send
// kernel adds the CTA offset to the local position.
constexpr int kPlanThreads = 256;

template <bool I64>
__device__ __forceinline__ void token_counts(const EpArgs& a, const void* ids, int64_t t, int64_t (&c)[kEpMaxWorld]) {
  int32_t n[kEpMaxWorld];
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d) n[d] = 0;
  for (int j = 0; j < a.topk; ++j) {
    const int64_t e = I64 ? __ldg(static_cast<const int64_t*>(ids) + t * a.topk + j)
                          : static_cast<int64_t>(__ldg(static_cast<const int32_t*>(ids) + t * a.topk + j));
    const bool bad = e < 0 || e >= a.E;
    a.cmap[t * a.topk + j] = bad ? -1 : static_cast<int32_t>(t * a.topk + j);
    if (bad) {
      atomicOr(a.dev_err, kDevErrExpertId);
      continue;
    }
    const int d = static_cast<int>(e / a.P);
#pragma unroll
    for (int q = 0; q < kEpMaxWorld; ++q) n[q] += q == d ? 1 : 0;
  }
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d) c[d] = n[d] ? (1ll << 32) + n[d] : 0;
}

template <bool I64>
__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(EpArgs a, const void* __restrict__ ids, int64_t T) {
  __shared__ int64_t wtot[kPlanThreads / 32][kEpMaxWorld];
  __shared__ bool last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kPlanThreads + tid;
  int64_t c[kEpMaxWorld];
  if (t < T) token_counts<I64>(a, ids, t, c);
  else {
#pragma unroll
    for (int d = 0; d < kEpMaxWorld; ++d) c[d] = 0;
  }
  int64_t incl[kEpMaxWorld];
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d) {
    int64_t v = c[d];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    incl[d] = v;
    if (lane == 31) wtot[warp][d] = v;
  }
  __syncthreads();
  int64_t* cta_tot = a.plan_tot + static_cast<int64_t>(blockIdx.x) * kEpMaxWorld;
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d) {
    int64_t before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < kPlanThreads / 32; ++w) {
      const int64_t v = wtot[w][d];
      before += w < warp ? v : 0;
      all += v;
    }
    const int64_t ex = before + incl[d] - c[d];
    if (t < T && d < a.world) {
      a.pos[t * a.world + d] = c[d] ? static_cast<int32_t>(ex >> 32) : -1;
      a.soff[t * a.world + d] = static_cast<int32_t>(ex & 0xffffffffll);
    }
    if (tid == 0) cta_tot[d] = all;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(a.done + 2, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (tid < kEpMaxWorld) {
    // exclusive offsets over the CTAs for destination d = tid
    int64_t run = 0;
    for (unsigned g = 0; g < gridDim.x; ++g) {
      const int64_t v = *reinterpret_cast<volatile int64_t*>(a.plan_tot + static_cast<int64_t>(g) * kEpMaxWorld + tid);
      a.plan_off[static_cast<int64_t>(g) * kEpMaxWorld + tid] = run;
      run += v;
    }
    if (tid < a.world) {
      a.tot[2 * tid] = static_cast<int32_t>(run >> 32);
      a.tot[2 * tid + 1] = static_cast<int32_t>(run & 0xffffffffll);
    }
  }
  if (tid == 0) {
    *a.epoch = *a.epoch + 1;
    a.done[2] = 0;
  }
}

// ---------------------------------------------------------------- send
// A warp per token: its row is copied into this rank's xcopy (rounded to bf16
// from f32 input); lanes j < topk write the slot records into the rank that
// owns expert j, the lane of a rank's first slot also the row record.
constexpr int kSendThreads = 256;

template <typename XT, bool I64>
__global__ void __launch_bounds__(kSendThreads) ep_send_kernel(EpArgs a, const XT* __restrict__ x,
                                                                const void* __restrict__ ids,
                                                                const float* __restrict__ w, int64_t T) {
  const int lane = threadIdx.x & 31;
  const int64_t epoch = *a.epoch;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kSendThreads) >> 5;
  const int hv = a.H / 8;                         // 16-byte vectors of 8 16-bit values per row
  for (int64_t t = (blockIdx.x * static_cast<int64_t>(kSendThreads) + threadIdx.x) >> 5; t < T; t += nwarps) {
    int32_t pos[kEpMaxWorld], so[kEpMaxWorld];
    const int64_t* off = a.plan_off + (t / kPlanThreads) * kEpMaxWorld;
#pragma unroll
    for (int d = 0; d < kEpMaxWorld; ++d) {
      const int64_t o = d < a.world ? __ldg(off + d) : 0;
      pos[d] = d < a.world ? __ldg(a.pos + t * a.world + d) : -1;
      so[d] = d < a.world ? __ldg(a.soff + t * a.world + d) + static_cast<int32_t>(o & 0xffffffffll) : 0;
      if (pos[d] >= 0) pos[d] += static_cast<int32_t>(o >> 32);
    }
    uint4* own = at<uint4>(a.self, a.o_xcopy) + t * hv;
    for (int c0 = 0; c0 < hv; c0 += 8 * 32) {
      uint4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = c0 + i * 32 + lane;
        if (c < hv) {
          if constexpr (sizeof(XT) == 2) {
            v[i] = __ldg(reinterpret_cast<const uint4*>(x + t * a.H) + c);
          } else {
            const float4 p0 = __ldg(reinterpret_cast<const float4*>(x + t * a.H) + 2 * c);
            const float4 p1 = __ldg(reinterpret_cast<const float4*>(x + t * a.H) + 2 * c + 1);
            v[i] = make_uint4(pack2<true>(p0.x, p0.y), pack2<true>(p0.z, p0.w), pack2<true>(p1.x, p1.y),
                              pack2<true>(p1.z, p1.w));
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = c0 + i * 32 + lane;
        if (c < hv) own[c] = v[i];
      }
    }
    // slot records (topk <= 32): the j-th slot of token t at its owner rank d
    int64_t e = -1;
    if (lane < a.topk)
      e = I64 ? __ldg(static_cast<const int64_t*>(ids) + t * a.topk + lane)
              : static_cast<int64_t>(__ldg(static_cast<const int32_t*>(ids) + t * a.topk + lane));
    const bool ok = lane < a.topk && e >= 0 && e < a.E;
    const int d = ok ? static_cast<int>(e / a.P) : -1 - lane;
    const unsigned same = __match_any_sync(0xffffffffu, d);
    if (ok) {
      const int rk = __popc(same & ((1u << lane) - 1u));
      int32_t my_pos = 0, my_so = 0;
#pragma unroll
      for (int q = 0; q < kEpMaxWorld; ++q)
        if (q == d) { my_pos = pos[q]; my_so = so[q]; }
      uint8_t* R = a.peer[d];
      const int64_t seg = static_cast<int64_t>(a.rank) * a.seg_len;
      if (rk == 0) {
        at<int32_t>(R, a.o_rowslot)[static_cast<int64_t>(a.rank) * (a.cap + 1) + my_pos] = my_so;
        at<int32_t>(R, a.o_rowtok)[static_cast<int64_t>(a.rank) * a.cap + my_pos] = static_cast<int32_t>(t);
      }
      at<int32_t>(R, a.o_exp)[seg + my_so + rk] = static_cast<int32_t>(e);
      at<float>(R, a.o_w)[seg + my_so + rk] = __ldg(w + t * a.topk + lane);
      at<int32_t>(R, a.o_dst)[seg + my_so + rk] = static_cast<int32_t>((a.rank * a.cap + t) * a.topk + lane);
    }
  }
  // the last CTA to finish publishes the counts and raises the dispatch flags
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = atomicAdd(a.done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x < a.world) {
    __threadfence_system();
    const int d = threadIdx.x;
    uint8_t* R = a.peer[d];
    const int32_t rows = a.tot[2 * d], slots = a.tot[2 * d + 1];
    at<int32_t>(R, a.o_rows)[a.rank] = rows;
    at<int32_t>(R, a.o_slots)[a.rank] = slots;
    at<int32_t>(R, a.o_rowslot)[static_cast<int64_t>(a.rank) * (a.cap + 1) + rows] = slots;
    __threadfence_system();
    st_release_sys(at<uint64_t>(R, a.o_disp) + a.rank, static_cast<uint64_t>(epoch));
  }
  if (last && threadIdx.x == 0) *a.done = 0;
}

// ---------------------------------------------------------------- wait
// Thread d polls flag[d] of this rank's region until it reaches the epoch;
// gives up after kEpWaitNs with the timeout bit in the device error word.
__global__ void ep_wait_kernel(EpArgs a, uint64_t o_flags) {
  const int d = threadIdx.x;
  if (d < a.world) {
    const uint64_t want = static_cast<uint64_t>(*a.epoch);
    const uint64_t* f = at<uint64_t>(a.self, o_flags) + d;
    if (ld_acquire_sys(f) < want) {
      const uint64_t t0 = globaltimer();
      while (ld_acquire_sys(f) < want) {
        if (globaltimer() - t0 > kEpWaitNs) {
          atomicOr(a.dev_err, kDevErrTimeout);
          break;
        }
        __nanosleep(100);
      }
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------- gather
// A warp per received row (source src, its row rho): the token row is loaded
// once from the source's xcopy (over NVLink for another rank) and stored to the
// plan rows of its slots here, slots s0 .. s1-1 of the source's segment.
template <bool PDL>
__global__ void __launch_bounds__(kSendThreads) ep_gather_kernel(EpArgs a, uint16_t* __restrict__ xs) {
  if (PDL) pdl_wait();   // inv comes from the align
  const int lane = threadIdx.x & 31;
  int64_t start[kEpMaxWorld + 1];
  start[0] = 0;
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d)
    start[d + 1] = start[d] + (d < a.world ? __ldg(at<int32_t>(a.self, a.o_rows) + d) : 0);
  const int64_t total = start[kEpMaxWorld];
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kSendThreads) >> 5;
  const int hv = a.H / 8;
  for (int64_t g = (blockIdx.x * static_cast<int64_t>(kSendThreads) + threadIdx.x) >> 5; g < total; g += nwarps) {
    int src = 0;
#pragma unroll
    for (int d = 1; d < kEpMaxWorld; ++d)
      if (g >= start[d]) src = d;
    const int64_t rho = g - start[src];
    const int32_t* rs = at<int32_t>(a.self, a.o_rowslot) + static_cast<int64_t>(src) * (a.cap + 1);
    const int32_t s0 = __ldg(rs + rho), s1 = __ldg(rs + rho + 1);
    const int32_t tok = __ldg(at<int32_t>(a.self, a.o_rowtok) + static_cast<int64_t>(src) * a.cap + rho);
    uint8_t* P = a.self;
#pragma unroll
    for (int q = 0; q < kEpMaxWorld; ++q) P = q == src ? a.peer[q] : P;
    const uint4* row = at<const uint4>(P, a.o_xcopy) + static_cast<int64_t>(tok) * hv;
    const int32_t* inv = a.inv + static_cast<int64_t>(src) * a.seg_len;
    for (int c0 = 0; c0 < hv; c0 += 8 * 32) {
      uint4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = c0 + i * 32 + lane;
        if (c < hv) v[i] = __ldcv(row + c);   // another rank's memory, rewritten every epoch: not cached
      }
      for (int s = s0; s < s1; ++s) {
        uint4* dst = reinterpret_cast<uint4*>(xs + static_cast<int64_t>(__ldg(inv + s)) * a.H);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = c0 + i * 32 + lane;
          if (c < hv) dst[c] = v[i];
        }
      }
    }
  }
  if (PDL) pdl_launch_dependents();
}

// ---------------------------------------------------------------- signal
// After the down GEMM, whose threads all ended with a system-scope fence after
// their peer stores: ret flag[this rank] = epoch on every rank.
__global__ void ep_signal_kernel(EpArgs a) {
  const int d = threadIdx.x;
  if (d < a.world) {
    const uint64_t epoch = static_cast<uint64_t>(*a.epoch);
    uint8_t* R = a.self;
#pragma unroll
    for (int q = 0; q < kEpMaxWorld; ++q) R = q == d ? a.peer[q] : R;
    __threadfence_system();
    st_release_sys(at<uint64_t>(R, a.o_ret_flag) + a.rank, epoch);
  }
}

}  // namespace hexmoe

using namespace hexmoe;

struct hexmoe_ep {
  int device, rank, world, E, P, H, topk, row_dtype;
  int64_t cap, seg_len;
  uint64_t o_disp, o_ret_flag, o_rows, o_slots, o_xcopy, o_rowslot, o_rowtok, o_exp, o_w, o_dst, o_ret;
  size_t region_bytes;
  uint8_t* region;
  uint8_t* peer[kEpMaxWorld];
  bool opened[kEpMaxWorld];
  bool connected;
  uint8_t* local;
  int64_t* epoch;
  uint32_t* done;
  int32_t *tot, *pos, *soff, *cmap, *inv;
  int64_t *plan_tot, *plan_off;
  int64_t last_tokens;
};

namespace {

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

EpArgs ep_args(const hexmoe_ep* ep, int32_t* dev_err) {
  EpArgs a{};
  for (int d = 0; d < kEpMaxWorld; ++d) a.peer[d] = d < ep->world ? ep->peer[d] : nullptr;
  a.self = ep->region;
  a.rank = ep->rank; a.world = ep->world; a.E = ep->E; a.P = ep->P; a.H = ep->H; a.topk = ep->topk;
  a.cap = ep->cap; a.seg_len = ep->seg_len;
  a.o_disp = ep->o_disp; a.o_ret_flag = ep->o_ret_flag; a.o_rows = ep->o_rows; a.o_slots = ep->o_slots;
  a.o_xcopy = ep->o_xcopy; a.o_rowslot = ep->o_rowslot; a.o_rowtok = ep->o_rowtok;
  a.o_exp = ep->o_exp; a.o_w = ep->o_w; a.o_dst = ep->o_dst;
  a.o_ret = ep->o_ret;
  a.epoch = ep->epoch; a.done = ep->done; a.tot = ep->tot; a.pos = ep->pos; a.soff = ep->soff;
  a.plan_tot = ep->plan_tot; a.plan_off = ep->plan_off; a.cmap = ep->cmap; a.inv = ep->inv;
  a.dev_err = dev_err;
  return a;
}

int ep_check(const hexmoe_ep* ep, const char* what) {
  if (!ep) return report_error(HEXMOE_E_ARG, what);
  if (!ep->connected) return report_error(HEXMOE_E_ARG, "expert parallel context is not connected (hexmoe_ep_connect)");
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != ep->device) return report_error(HEXMOE_E_ARG, "expert parallel context belongs to another device");
  return HEXMOE_OK;
}

// Grid of the send / gather kernels: a few CTAs per SM, warps looping over
// their tokens / rows (each send CTA ends with one system-scope fence, so
// fewer, longer-lived CTAs fence less).
int grid_for(int64_t work_warps, int per_cta_warps, int ctas_per_sm = 2) {
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (work_warps + per_cta_warps - 1) / per_cta_warps;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(sms) * ctas_per_sm)));
}

// The GatherHook of the slot-space forward: ep_gather_kernel after the align
// (programmatic dependent launch, as the kernels around it).
cudaError_t ep_gather_launch(const void* ctx, void* xs, const int32_t* inv, cudaStream_t st) {
  EpArgs a = *static_cast<const EpArgs*>(ctx);
  a.inv = const_cast<int32_t*>(inv);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid_for(static_cast<int64_t>(a.world) * a.cap, kSendThreads / 32, 4)));
  cfg.blockDim = dim3(kSendThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, ep_gather_kernel<true>, a, static_cast<uint16_t*>(xs));
}

}  // namespace

extern "C" {

int hexmoe_ep_init(int32_t rank, int32_t world, int32_t num_experts, int32_t hidden, int32_t topk,
                   int64_t max_tokens, int32_t row_dtype, hexmoe_ep** out) {
  if (!out) return report_error(HEXMOE_E_ARG, "hexmoe_ep_init: null out");
  *out = nullptr;
  if (world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world)
    return report_error(HEXMOE_E_ARG, "hexmoe_ep_init: rank / world outside 0 <= rank < world <= 8");
  if (num_experts <= 0 || hidden <= 0 || hidden % 8 || topk <= 0 || topk > 32 || topk > num_experts || max_tokens <= 0)
    return report_error(HEXMOE_E_ARG, "hexmoe_ep_init: bad experts / hidden / topk / max_tokens");
  if (row_dtype != HEXMOE_BF16 && row_dtype != HEXMOE_F16)
    return report_error(HEXMOE_E_DTYPE, "hexmoe_ep_init: rows are BF16 or F16");
  if (max_tokens * topk >= (1ll << 31) / world) return report_error(HEXMOE_E_ARG, "hexmoe_ep_init: max_tokens too large");
  auto* ep = new hexmoe_ep();
  cudaGetDevice(&ep->device);
  ep->rank = rank; ep->world = world; ep->E = num_experts; ep->P = (num_experts + world - 1) / world;
  ep->H = hidden; ep->topk = topk; ep->row_dtype = row_dtype; ep->cap = max_tokens;
  ep->seg_len = (max_tokens * topk + 2047) / 2048 * 2048;
  const size_t W = static_cast<size_t>(world);
  size_t off = 0;
  ep->o_disp = off; off += 8 * kEpMaxWorld;
  ep->o_ret_flag = off; off += 8 * kEpMaxWorld;
  ep->o_rows = off; off += 4 * kEpMaxWorld;
  ep->o_slots = off; off += 4 * kEpMaxWorld;
  off = up256(off);
  const size_t header = off;
  ep->o_xcopy = off; off = up256(off + static_cast<size_t>(ep->cap) * hidden * 2);
  ep->o_rowslot = off; off = up256(off + W * (ep->cap + 1) * 4);
  ep->o_rowtok = off; off = up256(off + W * ep->cap * 4);
  ep->o_exp = off; off = up256(off + W * ep->seg_len * 4);
  ep->o_w = off; off = up256(off + W * ep->seg_len * 4);
  ep->o_dst = off; off = up256(off + W * ep->seg_len * 4);
  ep->o_ret = off; off = up256(off + static_cast<size_t>(ep->cap) * topk * hidden * 2);
  ep->region_bytes = off;
  cudaError_t e = cudaMalloc(&ep->region, ep->region_bytes);
  if (e != cudaSuccess) { delete ep; return report_cuda_error(e, "hexmoe_ep_init: region allocation"); }
  const size_t plan_ctas = static_cast<size_t>((ep->cap + kPlanThreads - 1) / kPlanThreads);
  const size_t local_bytes = up256(8 + 16) + up256(W * 2 * 4) + 2 * up256(ep->cap * W * 4) +
                             2 * up256(plan_ctas * kEpMaxWorld * 8) + up256(static_cast<size_t>(ep->cap) * topk * 4) +
                             up256(W * ep->seg_len * 4);
  e = cudaMalloc(&ep->local, local_bytes);
  if (e == cudaSuccess) e = cudaMemset(ep->region, 0, header);
  if (e == cudaSuccess) e = cudaMemset(ep->local, 0, local_bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(ep->region);
    if (ep->local) cudaFree(ep->local);
    delete ep;
    return report_cuda_error(e, "hexmoe_ep_init: local state");
  }
  size_t lo = 0;
  ep->epoch = reinterpret_cast<int64_t*>(ep->local);
  ep->done = reinterpret_cast<uint32_t*>(ep->local + 8);
  lo = up256(8 + 16);
  ep->tot = reinterpret_cast<int32_t*>(ep->local + lo); lo += up256(W * 2 * 4);
  ep->pos = reinterpret_cast<int32_t*>(ep->local + lo); lo += up256(ep->cap * W * 4);
  ep->soff = reinterpret_cast<int32_t*>(ep->local + lo); lo += up256(ep->cap * W * 4);
  ep->plan_tot = reinterpret_cast<int64_t*>(ep->local + lo); lo += up256(plan_ctas * kEpMaxWorld * 8);
  ep->plan_off = reinterpret_cast<int64_t*>(ep->local + lo); lo += up256(plan_ctas * kEpMaxWorld * 8);
  ep->cmap = reinterpret_cast<int32_t*>(ep->local + lo); lo += up256(static_cast<size_t>(ep->cap) * topk * 4);
  ep->inv = reinterpret_cast<int32_t*>(ep->local + lo);
  for (int d = 0; d < kEpMaxWorld; ++d) { ep->peer[d] = nullptr; ep->opened[d] = false; }
  ep->peer[rank] = ep->region;
  ep->connected = world == 1;
  *out = ep;
  return HEXMOE_OK;
}

int hexmoe_ep_handle(const hexmoe_ep* ep, void* handle_out) {
  if (!ep || !handle_out) return report_error(HEXMOE_E_ARG, "hexmoe_ep_handle: null argument");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ep->region);
  if (e != cudaSuccess) return report_cuda_error(e, "hexmoe_ep_handle: cudaIpcGetMemHandle");
  static_assert(sizeof(h) == HEXMOE_EP_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  return HEXMOE_OK;
}

int hexmoe_ep_connect(hexmoe_ep* ep, const void* handles) {
  if (!ep || (!handles && ep->world > 1)) return report_error(HEXMOE_E_ARG, "hexmoe_ep_connect: null argument");
  if (ep->connected) return HEXMOE_OK;
  const uint8_t* hb = static_cast<const uint8_t*>(handles);
  for (int r = 0; r < ep->world; ++r) {
    if (r == ep->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hb + static_cast<size_t>(r) * HEXMOE_EP_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return report_cuda_error(e, "hexmoe_ep_connect: cudaIpcOpenMemHandle");
    ep->peer[r] = static_cast<uint8_t*>(p);
    ep->opened[r] = true;
  }
  ep->connected = true;
  return HEXMOE_OK;
}

size_t hexmoe_ep_workspace_bytes(const hexmoe_ep* ep, const hexmoe_layer* local, int32_t block_m) {
  if (!ep || !local) return 0;
  return slots_workspace_bytes(local, static_cast<int64_t>(ep->world) * ep->seg_len, block_m);
}

int hexmoe_ep_dispatch(hexmoe_ep* ep, const void* x, int32_t x_dtype, int64_t tokens, const float* topk_weights,
                       const void* topk_ids, int32_t ids_dtype, void* stream) {
  if (int rc = ep_check(ep, "hexmoe_ep_dispatch: null context")) return rc;
  if (tokens < 0 || tokens > ep->cap)
    return report_error(HEXMOE_E_ARG, "hexmoe_ep_dispatch: tokens outside 0..max_tokens of the context");
  if (x_dtype != ep->row_dtype && !(x_dtype == HEXMOE_F32 && ep->row_dtype == HEXMOE_BF16))
    return report_error(HEXMOE_E_DTYPE, "hexmoe_ep_dispatch: x dtype must be the row dtype (or F32 for BF16 rows)");
  if (ids_dtype != HEXMOE_I32 && ids_dtype != HEXMOE_I64) return report_error(HEXMOE_E_DTYPE, "ids dtype");
  if (tokens > 0 && (!x || !topk_weights || !topk_ids || reinterpret_cast<uintptr_t>(x) % 16))
    return report_error(HEXMOE_E_ARG, "hexmoe_ep_dispatch: null or unaligned pointer");
  int32_t* dev_err = device_error_word();
  if (!dev_err) return report_error(HEXMOE_E_CUDA, "device error word unavailable");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const EpArgs a = ep_args(ep, dev_err);
  const bool i64 = ids_dtype == HEXMOE_I64;
  const unsigned plan_grid = static_cast<unsigned>(std::max<int64_t>(1, (tokens + kPlanThreads - 1) / kPlanThreads));
  if (i64) ep_plan_kernel<true><<<plan_grid, kPlanThreads, 0, st>>>(a, topk_ids, tokens);
  else ep_plan_kernel<false><<<plan_grid, kPlanThreads, 0, st>>>(a, topk_ids, tokens);
  const int grid = grid_for(tokens, kSendThreads / 32);
  if (x_dtype == HEXMOE_F32) {
    if (i64) ep_send_kernel<float, true><<<grid, kSendThreads, 0, st>>>(a, static_cast<const float*>(x), topk_ids, topk_weights, tokens);
    else ep_send_kernel<float, false><<<grid, kSendThreads, 0, st>>>(a, static_cast<const float*>(x), topk_ids, topk_weights, tokens);
  } else {
    if (i64) ep_send_kernel<uint16_t, true><<<grid, kSendThreads, 0, st>>>(a, static_cast<const uint16_t*>(x), topk_ids, topk_weights, tokens);
    else ep_send_kernel<uint16_t, false><<<grid, kSendThreads, 0, st>>>(a, static_cast<const uint16_t*>(x), topk_ids, topk_weights, tokens);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return report_cuda_error(e, "hexmoe_ep_dispatch launch");
  ep->last_tokens = tokens;
  return HEXMOE_OK;
}

int hexmoe_ep_experts(hexmoe_ep* ep, const hexmoe_layer* local, int32_t block_m, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (int rc = ep_check(ep, "hexmoe_ep_experts: null context")) return rc;
  int32_t* dev_err = device_error_word();
  if (!dev_err) return report_error(HEXMOE_E_CUDA, "device error word unavailable");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const EpArgs a = ep_args(ep, dev_err);
  ep_wait_kernel<<<1, 32, 0, st>>>(a, ep->o_disp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return report_cuda_error(e, "hexmoe_ep_experts: wait launch");
  const int64_t S = static_cast<int64_t>(ep->world) * ep->seg_len;
  if (local) {
    const hexmoe_layer_desc* d = layer_desc(local);
    if (d->hidden != ep->H || d->num_experts != ep->E)
      return report_error(HEXMOE_E_ARG, "hexmoe_ep_experts: the local layer's hidden / num_experts differ from the context");
    const size_t need = slots_workspace_bytes(local, S, block_m);
    if (!workspace || workspace_bytes < need)
      return report_error(HEXMOE_E_ARG, "hexmoe_ep_experts: workspace smaller than hexmoe_ep_workspace_bytes");
    uint8_t* R = ep->region;
    // the down GEMM stores slot (src, t, j)'s row at ret row t * topk + j of rank src
    SlotOut so{};
    so.row = reinterpret_cast<const int32_t*>(R + ep->o_dst);
    for (int r = 0; r < kEpMaxWorld; ++r)
      so.base[r] = r < ep->world ? reinterpret_cast<uint16_t*>(ep->peer[r] + ep->o_ret) : nullptr;
    so.seg_rows = static_cast<int32_t>(ep->cap * ep->topk);
    so.fence = 1;
    // the activation rows come from the pull gather (the align records each slot's plan row)
    const GatherHook gh{ep_gather_launch, &a, ep->inv};
    int rc = forward_slot_space(local, R + ep->o_xcopy, ep->row_dtype, S,
                                reinterpret_cast<const int32_t*>(R + ep->o_exp), reinterpret_cast<const float*>(R + ep->o_w),
                                nullptr, reinterpret_cast<const int32_t*>(R + ep->o_slots), ep->seg_len, nullptr,
                                block_m, workspace, workspace_bytes, st, nullptr, &so, &gh);
    if (rc) return rc;
  }
  // without local experts nothing can have been routed here: only the flags
  ep_signal_kernel<<<1, 32, 0, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return report_cuda_error(e, "hexmoe_ep_experts: signal launch");
  return HEXMOE_OK;
}

int hexmoe_ep_combine(hexmoe_ep* ep, int64_t tokens, void* out, int32_t out_dtype, void* stream) {
  if (int rc = ep_check(ep, "hexmoe_ep_combine: null context")) return rc;
  if (tokens != ep->last_tokens) return report_error(HEXMOE_E_ARG, "hexmoe_ep_combine: tokens differ from the dispatch");
  if (out_dtype != HEXMOE_F32 && out_dtype != ep->row_dtype)
    return report_error(HEXMOE_E_DTYPE, "hexmoe_ep_combine: out dtype must be the row dtype or F32");
  if (tokens > 0 && (!out || reinterpret_cast<uintptr_t>(out) % 16))
    return report_error(HEXMOE_E_ARG, "hexmoe_ep_combine: null or unaligned out");
  int32_t* dev_err = device_error_word();
  if (!dev_err) return report_error(HEXMOE_E_CUDA, "device error word unavailable");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const EpArgs a = ep_args(ep, dev_err);
  ep_wait_kernel<<<1, 32, 0, st>>>(a, ep->o_ret_flag);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && tokens > 0)
    e = launch_combine(ep->region + ep->o_ret, ep->row_dtype, tokens, ep->topk, ep->H, ep->H, ep->cmap,
                       tokens * ep->topk, out, out_dtype, st, false);
  if (e != cudaSuccess) return report_cuda_error(e, "hexmoe_ep_combine launch");
  return HEXMOE_OK;
}

int hexmoe_ep_forward(hexmoe_ep* ep, const hexmoe_layer* local, const void* x, int32_t x_dtype, int64_t tokens,
                      const float* topk_weights, const void* topk_ids, int32_t ids_dtype, void* out, int32_t out_dtype,
                      int32_t block_m, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = hexmoe_ep_dispatch(ep, x, x_dtype, tokens, topk_weights, topk_ids, ids_dtype, stream)) return rc;
  if (int rc = hexmoe_ep_experts(ep, local, block_m, workspace, workspace_bytes, stream)) return rc;
  return hexmoe_ep_combine(ep, tokens, out, out_dtype, stream);
}

int hexmoe_ep_destroy(hexmoe_ep* ep) {
  if (!ep) return HEXMOE_OK;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != ep->device) cudaSetDevice(ep->device);
  for (int r = 0; r < kEpMaxWorld; ++r)
    if (ep->opened[r]) cudaIpcCloseMemHandle(ep->peer[r]);
  cudaFree(ep->region);
  cudaFree(ep->local);
  if (prev >= 0 && prev != ep->device) cudaSetDevice(prev);
  delete ep;
  return HEXMOE_OK;
}

}  // extern "C"
