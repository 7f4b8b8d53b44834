// api.cu — the C ABI of libhexmoe.so (include/hexmoe.h).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "internal.cuh"

using namespace hexmoe;

struct hexmoe_layer {
  hexmoe_layer_desc desc;
  int device;
  int num_sms;
  // tiled copies of the idx stacks (hexmoe_tile_index layout) per tier (gate,
  // up, down), carved from one allocation owned by the layer
  void* tiled_mem;
  const uint8_t* idx_t[kMaxTiers][3];
  // code tables of every (tier, projection) for bf16 [0] and f16 [1] operands
  // (launch_code_tables layout), read by the small-batch kernels
  void* tab_mem;
  const uint4* tab[kMaxTiers][3][2];
};

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(HEXMOE_E_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D row-major tensor map: inner dimension `cols` elements, `rows` rows, row
// pitch `pitch_bytes`, box {box_cols, box_rows}.
int make_tmap(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t cols, uint64_t rows,
              uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz, const char* what) {
  auto fn = encode_fn();
  if (!fn) return fail(HEXMOE_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (reinterpret_cast<uintptr_t>(base) % 16) return fail(HEXMOE_E_ARG, "%s: base address not 16-byte aligned", what);
  if (pitch_bytes % 16) return fail(HEXMOE_E_ARG, "%s: row pitch %llu not a multiple of 16 bytes", what,
                                    static_cast<unsigned long long>(pitch_bytes));
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  (void)elem_bytes;
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HEXMOE_E_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
  return HEXMOE_OK;
}

// The small-batch kernels' view of a row-major 16-bit [rows, cols] matrix:
// 3-D (64 columns, rows, cols / 64 column chunks), box {64, box_rows, 2}, 128-B
// swizzle, so one load brings 128 consecutive inputs of box_rows rows as two
// 64-input halves of box_rows x 128 B each (the layout two 2-D boxes of 64
// columns would give).
int make_tmap_chunks(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t cols, uint64_t rows,
                     uint64_t pitch_bytes, uint32_t box_rows, const char* what) {
  auto fn = encode_fn();
  if (!fn) return fail(HEXMOE_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (reinterpret_cast<uintptr_t>(base) % 16) return fail(HEXMOE_E_ARG, "%s: base address not 16-byte aligned", what);
  if (pitch_bytes % 16 || cols % 64) return fail(HEXMOE_E_UNSUPPORTED, "%s: row pitch %llu / columns %llu (block_m 8 needs a multiple of 64)", what,
                                                   static_cast<unsigned long long>(pitch_bytes),
                                                   static_cast<unsigned long long>(cols));
  cuuint64_t dims[3] = {64, rows, cols / 64};
  cuuint64_t strides[2] = {pitch_bytes, 128};
  cuuint32_t box[3] = {64, box_rows, 2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HEXMOE_E_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
  return HEXMOE_OK;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// The tile height hexmoe_forward picks: the small-batch kernels (8) while an
// expert averages at most 8 slots (decode), then the tcgen05 GEMM's heights.
int auto_block_m(int64_t S, int32_t E, int32_t hidden) {
  const int64_t avg = (S + E - 1) / std::max(E, 1);
  if (avg <= 8 && hidden % 64 == 0) return kDecBlock;   // the small-batch kernels read 64-input column chunks
  if (avg <= 8) return 16;
  if (avg <= 16) return 16;
  if (avg <= 32) return 32;
  if (avg <= 64) return 64;
  return 128;
}

struct WsLayout {
  size_t sid, eid, npp, align, xs, act, y, total;
  int64_t max_blocks;
};

WsLayout ws_layout(const hexmoe_layer_desc& d, int64_t T, int32_t k, int32_t bm, int32_t x_dtype) {
  WsLayout w{};
  const int64_t S = T * k;
  w.max_blocks = (S + bm - 1) / bm + std::min<int64_t>(d.num_experts, S);
  size_t off = 0;
  w.sid = off; off = align_up(off + sizeof(int32_t) * w.max_blocks * bm, 256);
  w.eid = off; off = align_up(off + sizeof(int32_t) * w.max_blocks, 256);
  w.npp = off; off = align_up(off + 16, 256);
  w.align = off; off = align_up(off + align_scratch_bytes(S, d.num_experts), 256);
  (void)x_dtype;
  w.xs = off; off = align_up(off + 2 * static_cast<size_t>(w.max_blocks) * bm * d.hidden, 256);
  w.act = off; off = align_up(off + 2 * static_cast<size_t>(w.max_blocks) * bm * d.inter_pad, 256);
  w.y = off; off = align_up(off + 2 * static_cast<size_t>(S) * d.hidden, 256);
  w.total = off;
  return w;
}

bool valid_block_m(int bm) { return bm == kDecBlock || bm == 16 || bm == 32 || bm == 64 || bm == 128; }

int check_dtype16(int32_t dt, const char* what) {
  if (dt != HEXMOE_F32 && dt != HEXMOE_BF16 && dt != HEXMOE_F16) return fail(HEXMOE_E_DTYPE, "%s: bad dtype %d", what, dt);
  return HEXMOE_OK;
}

// Shared-memory and TMEM carve-up of one GEMM launch (see GemmParams).  The
// index ring takes the widest stage (k_idx of 512, 384, 256 or 128 inputs;
// k_idx/128 tiled steps of 8 KB per projection) that divides k_pad and still
// leaves an activation ring of useful depth.
int plan_gemm(GemmParams& p, bool glu, int bm, int k_pad, int block) {
  const int nproj = glu ? 2 : 1;
  const uint32_t spr = static_cast<uint32_t>(k_pad / block);
  p.sz_scale = static_cast<uint32_t>(align_up(128u * spr, 1024));
  p.off_tab = glu ? 8192 : 8192 + 2048;                // after control block, fp8 table, tile records (+ down's
                                                       // 2 KB epilogue staging)
  p.off_scale = static_cast<uint32_t>(align_up(p.off_tab + 2u * nproj * 512u * 16u, 1024));
  p.off_idx = static_cast<uint32_t>(align_up(p.off_scale + 2u * nproj * p.sz_scale, 1024));
  p.sz_b = static_cast<uint32_t>(align_up(2u * bm * 128u, 1024));
  const int64_t budget = 232448 - 1024 - p.off_idx;
  const int db_min = bm >= 64 ? 3 : 4;
  p.di = 0;
  // gate/up prefers 128-input stages (a deeper ring in the same space; measured
  // faster); down, the widest
  const int order[2][4] = {{512, 384, 256, 128}, {128, 512, 384, 256}};
  for (int k_idx : order[glu ? 1 : 0]) {
    if (k_pad % k_idx) continue;
    const uint32_t sz = static_cast<uint32_t>(nproj * (k_idx / 128)) * kStepBytes;
    for (int di = kMaxDI; di >= 2; --di) {
      const int64_t rem = budget - static_cast<int64_t>(di) * sz;
      if (rem <= 0) continue;
      const int db = static_cast<int>(std::min<int64_t>(kMaxDB, rem / p.sz_b));
      if (db >= db_min || (k_idx == 128 && db >= 2)) {
        p.k_idx = k_idx; p.sz_idx = sz; p.di = di; p.db = db;
        break;
      }
    }
    if (p.di) break;
  }
  if (!p.di) return fail(HEXMOE_E_UNSUPPORTED, "reduction length %d / block_m %d do not fit shared memory", k_pad, bm);
  p.off_b = static_cast<uint32_t>(align_up(p.off_idx + static_cast<size_t>(p.di) * p.sz_idx, 1024));
  p.smem_bytes = std::max<uint32_t>(p.off_b + p.db * p.sz_b + 1024, 120 * 1024);
  // MMA issuers: one thread per projection (its own accumulator); with N <= 64
  // columns a tcgen05.mma keeps its issuing thread busy longer than the tensor
  // pipe takes to run it, so where an issuer warp is free (down: one
  // projection) and tensor memory allows, two threads take alternate 128-input
  // steps into two accumulators that the epilogue adds (ksplit 2: at least two
  // steps, and three operand stages left).  Gate/up would need two more warps,
  // and the registers they take from the decoders cost more than the split
  // gains (measured).
  p.a_stride = static_cast<uint32_t>(64 * nproj);   // one 128-input step per operand stage
  for (int ksplit = 2; ksplit >= 1; --ksplit) {
    if (ksplit == 2 && (k_pad / kKStep < 2 || bm > 64 || nproj * 2 > kMmaWarps)) continue;
    p.ksplit = ksplit;
    p.n_iss = nproj * ksplit;
    p.acc_stride = static_cast<uint32_t>(p.n_iss * bm);
    p.nbuf = (2 * p.acc_stride + 2 * p.a_stride <= kTmemCols) ? 2 : 1;
    p.a_base = p.nbuf * p.acc_stride;
    p.da = static_cast<int>(std::min<uint32_t>(kMaxDA, (kTmemCols - p.a_base) / p.a_stride));
    if (ksplit == 1 || p.da >= 3) break;
  }
  if (p.da < 2) return fail(HEXMOE_E_UNSUPPORTED, "block_m %d leaves no tensor memory for operands", bm);
  return HEXMOE_OK;
}

// Tile height and CTAs per SM of a small-batch launch (rows_pad, k_pad, block
// and bits of p set): the tallest tiles (128, 64, 32 rows) that still give
// two CTAs per SM a tile each for the plan's most blocks, else 32-row tiles
// (never more step groups than steps); two CTAs per SM once there are more
// tiles than SMs and the carve-up fits, else one with the deeper ring.
bool plan_small(DecParams& p, int nproj, int64_t max_blocks, int num_sms, int& per_sm) {
  const int ksteps = p.k_pad / kKStep;
  int rq = 4;
  for (int c : {4, 2, 1}) {
    if (c < 4 && 8 / c > ksteps) break;             // more step groups than steps
    rq = c;
    if (max_blocks * (p.rows_pad / (32 * c)) >= 2 * num_sms) break;
  }
  p.m128 = p.rows_pad / kTileM;
  p.m_tiles = p.rows_pad / (32 * rq);
  per_sm = max_blocks * p.m_tiles > num_sms && plan_decode(p, nproj, 2, rq) ? 2 : 1;
  return per_sm == 2 || plan_decode(p, nproj, 1, rq);
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) cudaSetDevice(dev);
    else prev = -1;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};


int run_gate_up(const hexmoe_layer* layer, const void* xs, bool bf16, int64_t tokens, int32_t topk,
                const int32_t* sid, const int32_t* eid, const int32_t* npp, int32_t bm, void* act, int32_t* dev_err,
                cudaStream_t st, bool pdl) {
  const hexmoe_layer_desc& d = layer->desc;
  const int64_t S = tokens * topk;
  const int64_t max_blocks = (S + bm - 1) / bm + std::min<int64_t>(d.num_experts, S);
  const CUtensorMapDataType dt16 = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  GemmParams p{};
  for (int t = 0; t < d.num_tiers; ++t) {
    p.bs[t][0] = d.tiers[t].gate.block_scale; p.bs[t][1] = d.tiers[t].up.block_scale;
    p.es[t][0] = d.tiers[t].gate.expert_scale; p.es[t][1] = d.tiers[t].up.expert_scale;
    p.lev[t][0] = d.tiers[t].gate.levels; p.lev[t][1] = d.tiers[t].up.levels;
    p.bits[t] = d.tiers[t].bits;
  }
  p.num_tiers = d.num_tiers;
  p.expert_map = d.expert_map;
  p.num_experts = d.num_experts;
  p.sorted_ids = sid; p.expert_ids = eid; p.npp = npp;
  p.bm = bm; p.max_blocks = static_cast<int32_t>(max_blocks);
  p.num_slots = static_cast<int32_t>(S);
  p.rows_pad = d.inter_pad; p.rows_store = d.inter_pad;
  p.k_pad = d.hidden_pad; p.block = d.block;
  p.m_tiles = d.inter_pad / kTileM;
  p.out = act; p.ld_out = d.inter_pad;
  p.topk_w = nullptr;
  p.dev_err = dev_err;
  if (bm == kDecBlock) {
    DecParams q{};
    for (int t = 0; t < d.num_tiers; ++t)
      for (int j = 0; j < 2; ++j) {
        q.idx_t[t][j] = layer->idx_t[t][j];
        q.bs[t][j] = p.bs[t][j];
        q.tab[t][j] = layer->tab[t][j][bf16 ? 0 : 1];
      }
    for (int t = 0; t < d.num_tiers; ++t) q.bits[t] = p.bits[t];
    q.num_tiers = d.num_tiers; q.expert_map = d.expert_map; q.num_experts = d.num_experts;
    q.sorted_ids = sid; q.expert_ids = eid; q.npp = npp; q.num_slots = static_cast<int32_t>(S);
    q.rows_pad = d.inter_pad; q.rows_store = d.inter_pad; q.k_pad = d.hidden_pad;
    q.block = d.block; q.m_tiles = d.inter_pad / kTileM; q.ksteps = d.hidden_pad / kKStep;
    q.out = act; q.ld_out = d.inter_pad; q.topk_w = nullptr; q.dev_err = dev_err;
    int per_sm = 1;
    if (!plan_small(q, 2, max_blocks, layer->num_sms, per_sm))
      return fail(HEXMOE_E_UNSUPPORTED, "hidden %d does not fit the small-batch kernel", d.hidden_pad);
    if (int rc = make_tmap_chunks(&q.tm_b, xs, dt16, d.hidden, static_cast<uint64_t>(max_blocks) * bm, 2ull * d.hidden,
                                  kDecBlock, "x_sorted tensor map"))
      return rc;
    const int grid = static_cast<int>(std::min<int64_t>(per_sm * layer->num_sms, max_blocks * q.m_tiles));
    cudaError_t e = launch_decode_gemm(q, true, bf16, grid, st, pdl);
    if (e != cudaSuccess) return cuda_fail(e, "gate/up (small batch) launch");
    return HEXMOE_OK;
  }
  if (int rc = plan_gemm(p, true, bm, d.hidden_pad, d.block)) return rc;
  for (int t = 0; t < d.num_tiers; ++t) {
    p.idx_t[t][0] = layer->idx_t[t][0];
    p.idx_t[t][1] = layer->idx_t[t][1];
  }
  if (int rc = make_tmap(&p.tm_b, xs, dt16, 2, d.hidden, static_cast<uint64_t>(max_blocks) * bm, 2ull * d.hidden, 64,
                         static_cast<uint32_t>(bm), CU_TENSOR_MAP_SWIZZLE_128B, "x_sorted tensor map"))
    return rc;
  const int grid = static_cast<int>(std::min<int64_t>(layer->num_sms, max_blocks * p.m_tiles));
  cudaError_t e = launch_gemm(p, true, bf16, grid, st, pdl);
  if (e != cudaSuccess) return cuda_fail(e, "gate/up launch");
  return HEXMOE_OK;
}

int run_down(const hexmoe_layer* layer, const void* act, bool bf16, int64_t tokens, int32_t topk,
             const float* topk_weights, const int32_t* sid, const int32_t* eid, const int32_t* npp, int32_t bm,
             void* y, int32_t* dev_err, cudaStream_t st, bool pdl, const SlotOut* slot_out = nullptr) {
  const hexmoe_layer_desc& d = layer->desc;
  const int64_t S = tokens * topk;
  const int64_t max_blocks = (S + bm - 1) / bm + std::min<int64_t>(d.num_experts, S);
  const CUtensorMapDataType dt16 = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  GemmParams q{};
  for (int t = 0; t < d.num_tiers; ++t) {
    q.bs[t][0] = d.tiers[t].down.block_scale;
    q.es[t][0] = d.tiers[t].down.expert_scale;
    q.lev[t][0] = d.tiers[t].down.levels;
    q.bits[t] = d.tiers[t].bits;
  }
  q.num_tiers = d.num_tiers;
  q.expert_map = d.expert_map;
  q.num_experts = d.num_experts;
  q.sorted_ids = sid; q.expert_ids = eid; q.npp = npp;
  q.bm = bm; q.max_blocks = static_cast<int32_t>(max_blocks);
  q.num_slots = static_cast<int32_t>(S);
  q.rows_pad = d.hidden_pad; q.rows_store = d.hidden;
  q.k_pad = d.inter_pad; q.block = d.block;
  q.m_tiles = d.hidden_pad / kTileM;
  q.out = y; q.ld_out = d.hidden;
  q.topk_w = topk_weights;
  if (slot_out) q.slot_out = *slot_out;
  q.dev_err = dev_err;
  if (bm == kDecBlock) {
    DecParams r{};
    for (int t = 0; t < d.num_tiers; ++t) {
      r.idx_t[t][0] = layer->idx_t[t][2];
      r.bs[t][0] = q.bs[t][0];
      r.tab[t][0] = layer->tab[t][2][bf16 ? 0 : 1];
      r.bits[t] = q.bits[t];
    }
    r.num_tiers = d.num_tiers; r.expert_map = d.expert_map; r.num_experts = d.num_experts;
    r.sorted_ids = sid; r.expert_ids = eid; r.npp = npp; r.num_slots = static_cast<int32_t>(S);
    r.rows_pad = d.hidden_pad; r.rows_store = d.hidden; r.k_pad = d.inter_pad;
    r.block = d.block; r.m_tiles = d.hidden_pad / kTileM; r.ksteps = d.inter_pad / kKStep;
    r.out = y; r.ld_out = d.hidden; r.topk_w = topk_weights; r.slot_out = q.slot_out; r.dev_err = dev_err;
    int per_sm = 1;
    if (!plan_small(r, 1, max_blocks, layer->num_sms, per_sm))
      return fail(HEXMOE_E_UNSUPPORTED, "inter %d does not fit the small-batch kernel", d.inter_pad);
    if (int rc = make_tmap_chunks(&r.tm_b, act, dt16, d.inter_pad, static_cast<uint64_t>(max_blocks) * bm,
                                  2ull * d.inter_pad, kDecBlock, "act tensor map"))
      return rc;
    const int grid = static_cast<int>(std::min<int64_t>(per_sm * layer->num_sms, max_blocks * r.m_tiles));
    cudaError_t e = launch_decode_gemm(r, false, bf16, grid, st, pdl);
    if (e != cudaSuccess) return cuda_fail(e, "down (small batch) launch");
    return HEXMOE_OK;
  }
  if (int rc = plan_gemm(q, false, bm, d.inter_pad, d.block)) return rc;
  for (int t = 0; t < d.num_tiers; ++t) q.idx_t[t][0] = layer->idx_t[t][2];
  if (int rc = make_tmap(&q.tm_b, act, dt16, 2, d.inter_pad, static_cast<uint64_t>(max_blocks) * bm,
                         2ull * d.inter_pad, 64, static_cast<uint32_t>(bm), CU_TENSOR_MAP_SWIZZLE_128B, "act tensor map"))
    return rc;
  const int grid = static_cast<int>(std::min<int64_t>(layer->num_sms, max_blocks * q.m_tiles));
  cudaError_t e = launch_gemm(q, false, bf16, grid, st, pdl);
  if (e != cudaSuccess) return cuda_fail(e, "down launch");
  return HEXMOE_OK;
}

int check_phase(const hexmoe_layer* layer, int32_t dt, int64_t tokens, int32_t topk, int32_t bm) {
  if (!layer) return fail(HEXMOE_E_ARG, "null layer");
  if (dt != HEXMOE_BF16 && dt != HEXMOE_F16) return fail(HEXMOE_E_DTYPE, "phase dtype must be BF16 or F16");
  if (tokens < 0 || topk <= 0 || topk > layer->desc.num_experts) return fail(HEXMOE_E_ARG, "tokens / topk");
  if (!valid_block_m(bm)) return fail(HEXMOE_E_ARG, "block_m %d not in {8, 16, 32, 64, 128}", bm);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != layer->device) return fail(HEXMOE_E_ARG, "layer was created on device %d, current device is %d", layer->device, dev);
  return HEXMOE_OK;
}

}  // namespace

int hexmoe::report_error(int code, const char* msg) { return fail(code, "%s", msg); }
int hexmoe::report_cuda_error(cudaError_t e, const char* what) { return cuda_fail(e, what); }

extern "C" {

int hexmoe_abi_version(void) { return HEXMOE_ABI_VERSION; }

const char* hexmoe_last_error(void) { return g_last_error.c_str(); }

int hexmoe_device_status(int device, int clear, int32_t* status_out) {
  DeviceGuard g(device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "hexmoe_device_status: synchronize");
  int32_t v = 0;
  e = read_device_error(&v, clear != 0);
  if (e != cudaSuccess) return cuda_fail(e, "hexmoe_device_status: read");
  if (status_out) *status_out = v;
  return HEXMOE_OK;
}

int hexmoe_build_expert_map(const hexmoe_layer_desc* desc, int32_t* map_out, void* stream) {
  if (!desc || !map_out) return fail(HEXMOE_E_ARG, "hexmoe_build_expert_map: null argument");
  if (desc->num_experts <= 0 || desc->num_tiers < 1 || desc->num_tiers > kMaxTiers)
    return fail(HEXMOE_E_ARG, "hexmoe_build_expert_map: %d experts, %d tiers", desc->num_experts, desc->num_tiers);
  if (!device_error_word()) return fail(HEXMOE_E_CUDA, "device error word unavailable");
  cudaError_t e = launch_build_expert_map(*desc, map_out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "expert map launch");
  return HEXMOE_OK;
}

int hexmoe_layer_create(const hexmoe_layer_desc* desc, hexmoe_layer** out) {
  if (!desc || !out) return fail(HEXMOE_E_ARG, "hexmoe_layer_create: null argument");
  *out = nullptr;
  const hexmoe_layer_desc& d = *desc;
  if (d.num_experts <= 0 || d.num_experts > 2048) return fail(HEXMOE_E_ARG, "num_experts %d outside 1..2048", d.num_experts);
  if (d.hidden <= 0 || d.inter <= 0 || d.hidden % 32 || d.inter % 32)
    return fail(HEXMOE_E_ARG, "hidden %d / inter %d must be positive multiples of 32", d.hidden, d.inter);
  if (d.hidden_pad < d.hidden || d.inter_pad < d.inter || d.hidden_pad % 128 || d.inter_pad % 128)
    return fail(HEXMOE_E_ARG, "hidden_pad %d / inter_pad %d must be multiples of 128 covering hidden / inter",
                d.hidden_pad, d.inter_pad);
  if (d.block != 32 && d.block != 128) return fail(HEXMOE_E_ARG, "scale block %d is not 32 or 128", d.block);
  if (d.num_tiers < 1 || d.num_tiers > kMaxTiers) return fail(HEXMOE_E_ARG, "num_tiers %d outside 1..%d", d.num_tiers, kMaxTiers);
  if (!d.expert_map) return fail(HEXMOE_E_ARG, "expert_map is null");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int major = 0, minor = 0, sms = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (major != 10 || minor != 0)
    return fail(HEXMOE_E_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", dev, major, minor);
  size_t tiled_bytes = 0;
  size_t tiled_off[kMaxTiers][3];
  for (int t = 0; t < d.num_tiers; ++t) {
    const hexmoe_tier& tr = d.tiers[t];
    if (tr.bits != 3 && tr.bits != 4) return fail(HEXMOE_E_ARG, "tier %d: bits %d is not 3 or 4", t, tr.bits);
    if (tr.n <= 0 || tr.n > 65535) return fail(HEXMOE_E_ARG, "tier %d: %d experts", t, tr.n);
    const hexmoe_parts* parts[3] = {&tr.gate, &tr.up, &tr.down};
    for (int j = 0; j < 3; ++j) {
      const hexmoe_parts& pp = *parts[j];
      if (!pp.idx || !pp.block_scale || !pp.expert_scale || !pp.levels)
        return fail(HEXMOE_E_ARG, "tier %d projection %d: null part", t, j);
      if (reinterpret_cast<uintptr_t>(pp.block_scale) % 16)
        return fail(HEXMOE_E_ARG, "tier %d projection %d: block_scale not 16-byte aligned", t, j);
      const int rows = j < 2 ? d.inter_pad : d.hidden_pad;
      const int cols = j < 2 ? d.hidden_pad : d.inter_pad;
      tiled_off[t][j] = tiled_bytes;
      tiled_bytes += align_up(static_cast<size_t>(tr.n) * rows * cols / 2, 256);
    }
  }
  if (!device_error_word()) return fail(HEXMOE_E_CUDA, "device error word unavailable");
  // The tiled copies: every earlier write to the stacks (on any stream) must
  // have landed, so wait for the device, then tile on a private stream.
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "hexmoe_layer_create: device synchronize");
  void* mem = nullptr;
  e = cudaMalloc(&mem, tiled_bytes);
  if (e != cudaSuccess) return cuda_fail(e, "hexmoe_layer_create: tiled index allocation");
  cudaStream_t st = nullptr;
  e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
  if (e != cudaSuccess) { cudaFree(mem); return cuda_fail(e, "hexmoe_layer_create: stream"); }
  auto* L = new hexmoe_layer();
  L->desc = d;
  L->device = dev;
  L->num_sms = sms;
  L->tiled_mem = mem;
  for (int t = 0; t < d.num_tiers && e == cudaSuccess; ++t) {
    const hexmoe_tier& tr = d.tiers[t];
    const hexmoe_parts* parts[3] = {&tr.gate, &tr.up, &tr.down};
    for (int j = 0; j < 3 && e == cudaSuccess; ++j) {
      const int rows = j < 2 ? d.inter_pad : d.hidden_pad;
      const int cols = j < 2 ? d.hidden_pad : d.inter_pad;
      uint8_t* dst = static_cast<uint8_t*>(mem) + tiled_off[t][j];
      L->idx_t[t][j] = dst;
      e = launch_tile_index(parts[j]->idx, tr.bits, tr.n, rows, cols, reinterpret_cast<uint32_t*>(dst), st);
    }
  }
  // code tables: per tier and projection, n x (256 or 512) x 16 B, for bf16 and f16
  size_t tab_bytes = 0;
  size_t tab_off[kMaxTiers][3];
  for (int t = 0; t < d.num_tiers; ++t)
    for (int j = 0; j < 3; ++j) {
      tab_off[t][j] = tab_bytes;
      tab_bytes += 2 * align_up(static_cast<size_t>(d.tiers[t].n) * (d.tiers[t].bits == 3 ? 256 : 512) * 16, 256);
    }
  if (e == cudaSuccess) e = cudaMalloc(&L->tab_mem, tab_bytes);
  for (int t = 0; t < d.num_tiers && e == cudaSuccess; ++t) {
    const hexmoe_tier& tr = d.tiers[t];
    const hexmoe_parts* parts[3] = {&tr.gate, &tr.up, &tr.down};
    const size_t one = align_up(static_cast<size_t>(tr.n) * (tr.bits == 3 ? 256 : 512) * 16, 256);
    for (int j = 0; j < 3 && e == cudaSuccess; ++j)
      for (int k = 0; k < 2 && e == cudaSuccess; ++k) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(L->tab_mem) + tab_off[t][j] + k * one);
        L->tab[t][j][k] = dst;
        e = launch_code_tables(parts[j]->levels, parts[j]->expert_scale, tr.bits, tr.n, k == 0, dst, st);
      }
  }
  const cudaError_t es = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = es;
  cudaStreamDestroy(st);
  if (e != cudaSuccess) {
    hexmoe_layer_destroy(L);
    return cuda_fail(e, "hexmoe_layer_create: tiling the index streams / code tables");
  }
  *out = L;
  return HEXMOE_OK;
}

int hexmoe_layer_destroy(hexmoe_layer* layer) {
  if (!layer) return HEXMOE_OK;
  if (layer->tiled_mem || layer->tab_mem) {
    DeviceGuard g(layer->device);
    if (layer->tiled_mem) cudaFree(layer->tiled_mem);
    if (layer->tab_mem) cudaFree(layer->tab_mem);
  }
  delete layer;
  return HEXMOE_OK;
}

size_t hexmoe_forward_workspace_bytes(const hexmoe_layer* layer, int64_t tokens, int32_t topk, int32_t block_m,
                                      int32_t x_dtype) {
  if (!layer || tokens < 0 || topk <= 0) return 0;
  const int bm = block_m > 0 ? block_m : auto_block_m(tokens * topk, layer->desc.num_experts, layer->desc.hidden);
  return ws_layout(layer->desc, tokens, topk, bm, x_dtype).total;
}

}  // extern "C"

namespace {

// hexmoe_forward, or with slots_out its per-slot rows instead of the combine.
// slot_row (optional): the x row of every slot (else slot / topk); seg_counts /
// seg_len (optional): a ragged slot space, of which only the first
// seg_counts[g] slots of every seg_len-slot segment exist (expert parallelism).
int forward_impl(const hexmoe_layer* layer, const void* x, int32_t x_dtype, int64_t tokens, int32_t topk,
                 const float* topk_weights, const void* topk_ids, int32_t ids_dtype, void* out, int32_t out_dtype,
                 void* slots_out, int32_t block_m, void* workspace, size_t workspace_bytes, void* stream,
                 const int32_t* slot_row = nullptr, const int32_t* seg_counts = nullptr, int64_t seg_len = 0,
                 const SlotOut* slot_out = nullptr, const GatherHook* gather = nullptr) {
  if (!layer) return fail(HEXMOE_E_ARG, "hexmoe_forward: null layer");
  const hexmoe_layer_desc& d = layer->desc;
  if (tokens < 0 || topk <= 0 || topk > d.num_experts) return fail(HEXMOE_E_ARG, "tokens %lld / topk %d", static_cast<long long>(tokens), topk);
  if (int rc = check_dtype16(x_dtype, "x")) return rc;
  if (int rc = check_dtype16(out_dtype, "out")) return rc;
  if (!slots_out && out_dtype != x_dtype && out_dtype != HEXMOE_F32)
    return fail(HEXMOE_E_DTYPE, "out dtype must be x dtype or f32");
  if (ids_dtype != HEXMOE_I32 && ids_dtype != HEXMOE_I64) return fail(HEXMOE_E_DTYPE, "ids dtype %d", ids_dtype);
  if (tokens == 0) return HEXMOE_OK;
  if (!x || !topk_weights || !topk_ids || !out || !workspace) return fail(HEXMOE_E_ARG, "hexmoe_forward: null pointer");
  if (slots_out && reinterpret_cast<uintptr_t>(slots_out) % 16) return fail(HEXMOE_E_ARG, "y must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(out) % 16 ||
      reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(HEXMOE_E_ARG, "x / out must be 16-byte and workspace 256-byte aligned");
  const int64_t S = tokens * topk;
  if (S >= (1ll << 31) - 1) return fail(HEXMOE_E_ARG, "too many slots");
  const int bm = block_m > 0 ? block_m : auto_block_m(S, d.num_experts, d.hidden);
  if (!valid_block_m(bm)) return fail(HEXMOE_E_ARG, "block_m %d not in {8, 16, 32, 64, 128}", bm);
  const WsLayout w = ws_layout(d, tokens, topk, bm, x_dtype);
  if (workspace_bytes < w.total)
    return fail(HEXMOE_E_ARG, "workspace %zu bytes < %zu needed", workspace_bytes, w.total);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != layer->device) return fail(HEXMOE_E_ARG, "layer was created on device %d, current device is %d", layer->device, dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* dev_err = device_error_word();
  if (!dev_err) return fail(HEXMOE_E_CUDA, "device error word unavailable");
  char* ws = static_cast<char*>(workspace);
  int32_t* sid = reinterpret_cast<int32_t*>(ws + w.sid);
  int32_t* eid = reinterpret_cast<int32_t*>(ws + w.eid);
  int32_t* npp = reinterpret_cast<int32_t*>(ws + w.npp);
  void* act = ws + w.act;
  void* y = slots_out ? slots_out : ws + w.y;
  const bool bf16 = x_dtype != HEXMOE_F16;     // f32 activations are computed in bf16
  void* xs = ws + w.xs;
  cudaError_t e = launch_align(topk_ids, ids_dtype == HEXMOE_I64, S, d.num_experts, bm, sid, eid, npp,
                               reinterpret_cast<int32_t*>(ws + w.align), align_scratch_bytes(S, d.num_experts), dev_err,
                               st, true, seg_counts, seg_len, gather ? gather->inv : nullptr);
  if (e != cudaSuccess) return cuda_fail(e, "align launch");

  e = gather ? gather->launch(gather->ctx, xs, gather->inv, st)
             : launch_gather_rows(x, x_dtype, tokens, d.hidden, sid, npp, w.max_blocks * bm, topk, S, xs, st, true,
                                  slot_row);
  if (e != cudaSuccess) return cuda_fail(e, "gather launch");
  int rc = run_gate_up(layer, xs, bf16, tokens, topk, sid, eid, npp, bm, act, dev_err, st, true);
  if (rc) return rc;
  rc = run_down(layer, act, bf16, tokens, topk, topk_weights, sid, eid, npp, bm, y, dev_err, st, true, slot_out);
  if (rc) return rc;
  if (slots_out) return HEXMOE_OK;

  // ---- combine
  e = launch_combine(y, bf16 ? HEXMOE_BF16 : HEXMOE_F16, tokens, topk, d.hidden, d.hidden, nullptr, S, out, out_dtype,
                     st, true);
  if (e != cudaSuccess) return cuda_fail(e, "combine launch");
  return HEXMOE_OK;
}

}  // namespace

const hexmoe_layer_desc* hexmoe::layer_desc(const hexmoe_layer* layer) { return layer ? &layer->desc : nullptr; }

size_t hexmoe::slots_workspace_bytes(const hexmoe_layer* layer, int64_t num_slots, int32_t block_m) {
  if (!layer || num_slots < 0) return 0;
  const int bm = block_m > 0 ? block_m : auto_block_m(num_slots, layer->desc.num_experts, layer->desc.hidden);
  return ws_layout(layer->desc, num_slots, 1, bm, HEXMOE_BF16).total;
}

int hexmoe::forward_slot_space(const hexmoe_layer* layer, const void* x, int32_t x_dtype, int64_t num_slots,
                               const int32_t* slot_expert, const float* slot_weight, const int32_t* slot_row,
                               const int32_t* seg_counts, int64_t seg_len, void* y, int32_t block_m, void* workspace,
                               size_t workspace_bytes, cudaStream_t st, void** y_used, const SlotOut* slot_out,
                               const GatherHook* gather) {
  if (!layer) return fail(HEXMOE_E_ARG, "forward_slot_space: null layer");
  if (!y) {
    // the per-slot rows go to the workspace's own y region
    const int bm = block_m > 0 ? block_m : auto_block_m(num_slots, layer->desc.num_experts, layer->desc.hidden);
    const WsLayout w = ws_layout(layer->desc, num_slots, 1, bm, x_dtype);
    if (!workspace || workspace_bytes < w.total) return fail(HEXMOE_E_ARG, "forward_slot_space: workspace too small");
    y = static_cast<char*>(workspace) + w.y;
  }
  if (y_used) *y_used = y;
  return forward_impl(layer, x, x_dtype, num_slots, 1, slot_weight, slot_expert, HEXMOE_I32, y,
                      x_dtype == HEXMOE_F16 ? HEXMOE_F16 : HEXMOE_BF16, y, block_m, workspace, workspace_bytes, st,
                      slot_row, seg_counts, seg_len, slot_out, gather);
}

extern "C" {

int hexmoe_forward(const hexmoe_layer* layer, const void* x, int32_t x_dtype, int64_t tokens, int32_t topk,
                   const float* topk_weights, const void* topk_ids, int32_t ids_dtype, void* out, int32_t out_dtype,
                   int32_t block_m, void* workspace, size_t workspace_bytes, void* stream) {
  return forward_impl(layer, x, x_dtype, tokens, topk, topk_weights, topk_ids, ids_dtype, out, out_dtype, nullptr,
                      block_m, workspace, workspace_bytes, stream);
}

int hexmoe_forward_slots(const hexmoe_layer* layer, const void* x, int32_t x_dtype, int64_t tokens, int32_t topk,
                         const float* topk_weights, const void* topk_ids, int32_t ids_dtype, void* y,
                         int32_t block_m, void* workspace, size_t workspace_bytes, void* stream) {
  if (!y && tokens > 0) return fail(HEXMOE_E_ARG, "hexmoe_forward_slots: null y");
  return forward_impl(layer, x, x_dtype, tokens, topk, topk_weights, topk_ids, ids_dtype, y,
                      x_dtype == HEXMOE_F16 ? HEXMOE_F16 : HEXMOE_BF16, y, block_m, workspace, workspace_bytes, stream);
}

int hexmoe_gather(const void* x, int32_t x_dtype, int64_t tokens, int32_t hidden, int32_t topk, int32_t num_experts,
                  const int32_t* sorted_ids, const int32_t* npp, int32_t block_m, void* x_sorted, void* stream) {
  if (check_dtype16(x_dtype, "x")) return HEXMOE_E_DTYPE;
  if (tokens < 0 || hidden <= 0 || hidden % 32 || topk <= 0 || num_experts <= 0 || block_m <= 0)
    return fail(HEXMOE_E_ARG, "hexmoe_gather: bad sizes");
  if (tokens == 0) return HEXMOE_OK;
  if (!x || !sorted_ids || !npp || !x_sorted || reinterpret_cast<uintptr_t>(x) % 16 ||
      reinterpret_cast<uintptr_t>(x_sorted) % 16)
    return fail(HEXMOE_E_ARG, "hexmoe_gather: null or unaligned pointer");
  const int64_t S = tokens * topk;
  const int64_t max_blocks = (S + block_m - 1) / block_m + std::min<int64_t>(num_experts, S);
  cudaError_t e = launch_gather_rows(x, x_dtype, tokens, hidden, sorted_ids, npp, max_blocks * block_m, topk, S,
                                     x_sorted, static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess) return cuda_fail(e, "gather launch");
  return HEXMOE_OK;
}

int hexmoe_gate_up(const hexmoe_layer* layer, const void* x_sorted, int32_t x_dtype, int64_t tokens, int32_t topk,
                   const int32_t* sorted_ids, const int32_t* expert_ids, const int32_t* npp, int32_t block_m,
                   void* act, void* stream) {
  if (int rc = check_phase(layer, x_dtype, tokens, topk, block_m)) return rc;
  if (tokens == 0) return HEXMOE_OK;
  if (!x_sorted || !sorted_ids || !expert_ids || !npp || !act) return fail(HEXMOE_E_ARG, "hexmoe_gate_up: null pointer");
  int32_t* dev_err = device_error_word();
  if (!dev_err) return fail(HEXMOE_E_CUDA, "device error word unavailable");
  return run_gate_up(layer, x_sorted, x_dtype == HEXMOE_BF16, tokens, topk, sorted_ids, expert_ids, npp, block_m, act,
                     dev_err, static_cast<cudaStream_t>(stream), false);
}

int hexmoe_down(const hexmoe_layer* layer, const void* act, int32_t act_dtype, int64_t tokens, int32_t topk,
                const float* topk_weights, const int32_t* sorted_ids, const int32_t* expert_ids, const int32_t* npp,
                int32_t block_m, void* y, void* stream) {
  if (int rc = check_phase(layer, act_dtype, tokens, topk, block_m)) return rc;
  if (tokens == 0) return HEXMOE_OK;
  if (!act || !topk_weights || !sorted_ids || !expert_ids || !npp || !y)
    return fail(HEXMOE_E_ARG, "hexmoe_down: null pointer");
  if (reinterpret_cast<uintptr_t>(y) % 16) return fail(HEXMOE_E_ARG, "hexmoe_down: y must be 16-byte aligned");
  int32_t* dev_err = device_error_word();
  if (!dev_err) return fail(HEXMOE_E_CUDA, "device error word unavailable");
  return run_down(layer, act, act_dtype == HEXMOE_BF16, tokens, topk, topk_weights, sorted_ids, expert_ids, npp,
                  block_m, y, dev_err, static_cast<cudaStream_t>(stream), false);
}

int hexmoe_combine(const void* y, int32_t y_dtype, int64_t tokens, int32_t topk, int32_t hidden, void* out,
                   int32_t out_dtype, void* stream) {
  if (y_dtype != HEXMOE_BF16 && y_dtype != HEXMOE_F16) return fail(HEXMOE_E_DTYPE, "y dtype must be BF16 or F16");
  if (check_dtype16(out_dtype, "out")) return HEXMOE_E_DTYPE;
  if (tokens < 0 || topk <= 0 || hidden <= 0 || hidden % 8) return fail(HEXMOE_E_ARG, "combine: tokens / topk / hidden");
  if (tokens == 0) return HEXMOE_OK;
  if (!y || !out || reinterpret_cast<uintptr_t>(y) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return fail(HEXMOE_E_ARG, "combine: y / out must be non-null and 16-byte aligned");
  cudaError_t e = launch_combine(y, y_dtype, tokens, topk, hidden, hidden, nullptr, tokens * topk, out, out_dtype,
                                 static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess) return cuda_fail(e, "combine launch");
  return HEXMOE_OK;
}

int hexmoe_combine_rows(const void* y, int32_t y_dtype, int64_t y_rows, int64_t tokens, int32_t topk, int32_t hidden,
                        const int32_t* rows, void* out, int32_t out_dtype, void* stream) {
  if (y_dtype != HEXMOE_BF16 && y_dtype != HEXMOE_F16) return fail(HEXMOE_E_DTYPE, "y dtype must be BF16 or F16");
  if (check_dtype16(out_dtype, "out")) return HEXMOE_E_DTYPE;
  if (tokens < 0 || topk <= 0 || hidden <= 0 || hidden % 8 || y_rows < 0)
    return fail(HEXMOE_E_ARG, "combine_rows: tokens / topk / hidden / y_rows");
  if (tokens == 0) return HEXMOE_OK;
  if (!y || !out || !rows || reinterpret_cast<uintptr_t>(y) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return fail(HEXMOE_E_ARG, "combine_rows: y / rows / out must be non-null, y and out 16-byte aligned");
  cudaError_t e = launch_combine(y, y_dtype, tokens, topk, hidden, hidden, rows, y_rows, out, out_dtype,
                                 static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess) return cuda_fail(e, "combine_rows launch");
  return HEXMOE_OK;
}

size_t hexmoe_align_workspace_bytes(int64_t num_slots, int32_t num_experts) {
  return align_scratch_bytes(num_slots, num_experts);
}

int hexmoe_align(const void* ids, int32_t ids_dtype, int64_t num_slots, int32_t num_experts, int32_t block_m,
                 int32_t* sorted_ids, int32_t* expert_ids, int32_t* npp, void* workspace, size_t workspace_bytes,
                 void* stream) {
  if (ids_dtype != HEXMOE_I32 && ids_dtype != HEXMOE_I64) return fail(HEXMOE_E_DTYPE, "ids dtype %d", ids_dtype);
  if (num_slots < 0 || num_slots >= (1ll << 31) - 1) return fail(HEXMOE_E_ARG, "num_slots %lld", static_cast<long long>(num_slots));
  if (num_experts <= 0 || num_experts > 2048) return fail(HEXMOE_E_ARG, "num_experts %d outside 1..2048", num_experts);
  if (block_m <= 0) return fail(HEXMOE_E_ARG, "block_m %d", block_m);
  if (!npp || (num_slots > 0 && (!ids || !sorted_ids || !expert_ids))) return fail(HEXMOE_E_ARG, "hexmoe_align: null pointer");
  if (workspace && reinterpret_cast<uintptr_t>(workspace) % 16) return fail(HEXMOE_E_ARG, "hexmoe_align: workspace not 16-byte aligned");
  int32_t* dev_err = device_error_word();
  if (!dev_err) return fail(HEXMOE_E_CUDA, "device error word unavailable");
  cudaError_t e = launch_align(ids, ids_dtype == HEXMOE_I64, num_slots, num_experts, block_m, sorted_ids, expert_ids,
                               npp, static_cast<int32_t*>(workspace), workspace ? workspace_bytes : 0, dev_err,
                               static_cast<cudaStream_t>(stream), false);
  if (e != cudaSuccess) return cuda_fail(e, "align launch");
  return HEXMOE_OK;
}

int hexmoe_dequant(const hexmoe_parts* parts, int32_t bits, int32_t block, int32_t n, int32_t rows, int32_t cols,
                   int32_t rows_pad, int32_t cols_pad, const int32_t* experts, void* out, int32_t out_dtype,
                   int64_t stride_e, int64_t stride_row, int64_t row_off, void* stream) {
  if (!parts || !out) return fail(HEXMOE_E_ARG, "hexmoe_dequant: null pointer");
  if (bits != 3 && bits != 4) return fail(HEXMOE_E_ARG, "bits %d is not 3 or 4", bits);
  if (block != 32 && block != 128) return fail(HEXMOE_E_ARG, "scale block %d is not 32 or 128", block);
  if (n < 0 || rows < 0 || cols < 0 || cols % 32 || rows_pad < rows || cols_pad < cols || cols_pad % block)
    return fail(HEXMOE_E_ARG, "hexmoe_dequant: bad shape n=%d rows=%d cols=%d pad=%d,%d", n, rows, cols, rows_pad, cols_pad);
  if (check_dtype16(out_dtype, "out")) return HEXMOE_E_DTYPE;
  cudaError_t e = launch_dequant(*parts, bits, block, n, rows, cols, rows_pad, cols_pad, experts, out, out_dtype,
                                 stride_e, stride_row, row_off, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dequant launch");
  return HEXMOE_OK;
}

int hexmoe_tile_index(const uint32_t* idx, int32_t bits, int32_t n, int32_t rows_pad, int32_t cols_pad, uint32_t* out,
                      void* stream) {
  if (bits != 3 && bits != 4) return fail(HEXMOE_E_ARG, "bits %d is not 3 or 4", bits);
  if (n < 0 || rows_pad < 0 || cols_pad < 0 || rows_pad % 128 || cols_pad % 128)
    return fail(HEXMOE_E_ARG, "hexmoe_tile_index: n=%d rows_pad=%d cols_pad=%d (multiples of 128 expected)", n,
                rows_pad, cols_pad);
  if (static_cast<int64_t>(n) * rows_pad * cols_pad == 0) return HEXMOE_OK;
  if (!idx || !out) return fail(HEXMOE_E_ARG, "hexmoe_tile_index: null pointer");
  cudaError_t e = launch_tile_index(idx, bits, n, rows_pad, cols_pad, out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tile_index launch");
  return HEXMOE_OK;
}

int hexmoe_route_topk(const void* logits, int32_t logits_dtype, int64_t tokens, int32_t num_experts, int32_t topk,
                      int32_t renormalize, float* topk_weights, int32_t* topk_ids, void* stream) {
  if (check_dtype16(logits_dtype, "logits")) return HEXMOE_E_DTYPE;
  if (tokens < 0 || num_experts <= 0 || topk <= 0 || topk > 32 || topk > num_experts)
    return fail(HEXMOE_E_ARG, "route_topk: tokens %lld experts %d topk %d", static_cast<long long>(tokens), num_experts, topk);
  if (tokens > 0 && (!logits || !topk_weights || !topk_ids)) return fail(HEXMOE_E_ARG, "route_topk: null pointer");
  cudaError_t e = launch_route_topk(logits, logits_dtype, tokens, num_experts, topk, renormalize, topk_weights,
                                    topk_ids, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "route_topk launch");
  return HEXMOE_OK;
}

}  // extern "C"
