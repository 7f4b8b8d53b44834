// internal.cuh — structures shared by the C ABI (api.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "hexmoe.h"

namespace hexmoe {

constexpr int kMaxTiers = HEXMOE_MAX_TIERS;
constexpr int kTileM = 128;      // weight rows per tile (UMMA M)
constexpr int kKStep = 128;      // reduction elements per activation (B operand) stage
constexpr int kMaxDI = 8;        // deepest index-word ring
constexpr int kMaxDB = 8;        // deepest activation ring
constexpr int kMaxDA = 8;        // deepest TMEM operand ring
#ifndef HEXMOE_DEC_GROUPS
#define HEXMOE_DEC_GROUPS 1
#endif
constexpr int kDecGroups = HEXMOE_DEC_GROUPS;   // groups of 8 decoder warps, taking 128-input sub-blocks in turn
constexpr int kDecWarps = 8 * kDecGroups;
constexpr int kBWarp = 6 + kDecWarps;   // activation producer
constexpr int kMmaWarps = 2;            // MMA issuers: warp 1 and warp kBWarp+1
constexpr int kGemmThreads = (kBWarp + kMmaWarps) * 32;  // index TMA, MMA, 4 epilogue, decoders, activation TMA, MMA
constexpr uint32_t kTmemCols = 512;

constexpr uint32_t kStepBytes = 8192;   // one 128-row x 128-input step of a tiled index stream

// Where the down projection stores its per-slot rows.  row == nullptr: the
// plain layout, slot s at y + s * ld_out.  Otherwise (the expert-parallel
// return) slot s goes to global row g = row[s] of the concatenated per-slot
// buffers of all ranks: base[g / seg_rows] + (g % seg_rows) * ld_out, a peer's
// memory for another rank's tokens; fence: every thread of the kernel ends
// with a system-scope fence, so its peer stores are visible before a later
// kernel on the stream raises the return flags.
struct SlotOut {
  const int32_t* row;
  uint16_t* base[HEXMOE_EP_MAX_WORLD];
  int32_t seg_rows;
  int32_t fence;
};

// The down epilogue's destination of slot id g (see SlotOut).
__device__ __forceinline__ uint16_t* slot_out_row(const SlotOut& so, uint16_t* y, int64_t ld_out, int g) {
  if (!so.row) return y + static_cast<int64_t>(g) * ld_out;
  const int sg = g / so.seg_rows;
  uint16_t* b = so.base[0];
#pragma unroll
  for (int i = 1; i < HEXMOE_EP_MAX_WORLD; ++i) b = sg == i ? so.base[i] : b;
  return b + static_cast<int64_t>(g - sg * so.seg_rows) * ld_out;
}

// The expert-parallel receive side's own gather (ep.cu): launch(ctx, xs, inv,
// st) writes the plan-ordered activation rows xs itself, given inv [num_slots],
// the plan row of every slot, which the align writes.  Replaces the plain
// gather pass of the slot-space forward.
struct GatherHook {
  cudaError_t (*launch)(const void* ctx, void* xs, const int32_t* inv, cudaStream_t st);
  const void* ctx;
  int32_t* inv;
};

// Everything the grouped-GEMM kernel needs; passed by value as a
// __grid_constant__ parameter (tensor maps must live in parameter space).
struct GemmParams {
  CUtensorMap tm_b;                  // B rows in plan order: x_sorted [rows, H] (gate/up) or act [rows, I_pad] (down)
  const uint8_t* idx_t[kMaxTiers][2];  // tiled index streams (hexmoe_tile_index layout)
  const uint8_t* bs[kMaxTiers][2];
  const float* es[kMaxTiers][2];
  const float* lev[kMaxTiers][2];
  int32_t bits[kMaxTiers];
  int32_t num_tiers;
  const int32_t* expert_map;   // [E]: (tier << 16) | local, -1 = no tier
  int32_t num_experts;
  const int32_t* sorted_ids;   // [max_blocks * bm], align() layout
  const int32_t* expert_ids;   // [max_blocks]
  const int32_t* npp;          // [1]
  int32_t bm;                  // tokens per tile (align block_m), multiple of 16, <= 128
  int32_t max_blocks;
  int32_t num_slots;           // S = T * topk
  int32_t rows_pad;            // weight rows per expert in the stack
  int32_t rows_store;          // rows written to the output (<= rows_pad)
  int32_t k_pad;               // reduction length (multiple of 128)
  int32_t block;               // scale block: 32 or 128
  int32_t m_tiles;             // rows_pad / 128
  // shared-memory carve-up (byte offsets from the 1024-aligned base)
  uint32_t off_tab;            // per-tile code tables: [2][nproj][2 planes][256] x 16 B
  uint32_t off_scale, sz_scale;  // two tile-scale buffers
  int32_t k_idx;               // reduction elements per index stage (128..512, divides k_pad)
  int32_t di;                  // index ring depth
  uint32_t off_idx, sz_idx;    // index stage: [nproj][k_idx/128 steps][4 blocks][128 rows][4 words]
  int32_t db;                  // activation ring depth
  uint32_t off_b, sz_b;        // activation stage: [2 halves][bm rows][64 x 16-bit], 128-B swizzled
  uint32_t smem_bytes;         // dynamic shared memory to request
  // TMEM carve-up (columns)
  int32_t nbuf;                // accumulator buffers (1 or 2)
  int32_t n_iss;               // MMA issuing threads: nproj x ksplit
  int32_t ksplit;              // accumulators per projection: 2 = issuers take alternate 128-input steps
  int32_t da;                  // operand ring depth
  uint32_t acc_stride;         // columns per accumulator buffer
  uint32_t a_base, a_stride;   // operand ring: first column, columns per stage
  // output
  void* out;                   // gate/up: act [max_blocks*bm, ld_out]; down: y [S, ld_out]
  int64_t ld_out;
  const float* topk_w;         // down: [S]
  SlotOut slot_out;            // down: where each slot's row goes
  int32_t* dev_err;
};

// Launches the persistent grouped GEMM (gate/up with SwiGLU when glu, else down
// with the top-k weight); returns a cudaError_t.
cudaError_t launch_gemm(const GemmParams& p, bool glu, bool bf16, int grid, cudaStream_t stream, bool pdl);

// The small-batch grouped GEMM (decode_gemm.cu): align blocks of kDecBlock
// slots; persistent CTAs over the tiles (block, 32, 64 or 128 weight rows), a
// producer warp streaming 128-input steps through a shared-memory ring, 8
// consumer warps of 32 rows each.
constexpr int kDecBlock = 8;
constexpr int kDecStages = 16;   // deepest step ring
struct DecParams {
  CUtensorMap tm_b;                     // plan-ordered B rows (x_sorted or act): boxes of 64 inputs x 8 rows, 128-B swizzle
  const uint8_t* idx_t[kMaxTiers][2];   // tiled index streams (hexmoe_tile_index layout)
  const uint8_t* bs[kMaxTiers][2];      // block scales [n, rows_pad, k_pad/block]
  const uint4* tab[kMaxTiers][2];       // code tables [n][256 (3-bit) or 512 (4-bit)] of the operand type
  int32_t bits[kMaxTiers];
  int32_t num_tiers;
  const int32_t* expert_map;
  int32_t num_experts;
  const int32_t* sorted_ids;            // align plan with block_m = kDecBlock
  const int32_t* expert_ids;
  const int32_t* npp;
  int32_t num_slots;
  int32_t rows_pad, rows_store, k_pad, block, m_tiles, ksteps;
  int32_t block_log2;                   // log2(block), set by plan_decode
  int32_t rq;                           // tile height in 32-row slices (1, 2, 4): m_tiles = rows_pad / (32 rq)
  int32_t m128;                         // rows_pad / 128 (the tiled copy's row tiles)
  int32_t ds;                           // ring depth (stages)
  uint32_t stage_bytes, off_tab, tab_bytes, off_sc, sc_bytes, off_red, smem_bytes;   // shared-memory carve-up
  void* out;                            // gate/up: act [plan rows, ld_out]; down: y [S, ld_out]
  int64_t ld_out;
  const float* topk_w;
  SlotOut slot_out;                     // down: where each slot's row goes
  int32_t* dev_err;
};
// The shared-memory carve-up (block and tier bits set) for per_sm (1 or 2) CTAs
// on an SM and tiles of 32 rq rows; false when it does not fit.
bool plan_decode(DecParams& p, int nproj, int per_sm, int rq);
cudaError_t launch_decode_gemm(const DecParams& p, bool glu, bool bf16, int grid, cudaStream_t st, bool pdl);
// Code tables of one projection of a tier (kernels.cu): out [n][256 or 512] uint4.
cudaError_t launch_code_tables(const float* levels, const float* es, int bits, int n, bool bf16, uint4* out,
                               cudaStream_t st);

// Small kernels (kernels.cu).
// seg_counts (optional): the ragged slot space of the expert-parallel receive
// side, segments of seg_len slots of which only the first seg_counts[g] exist.
// inv (optional, [S]): receives the plan row of every present slot.
cudaError_t launch_align(const void* ids, bool ids64, int64_t S, int32_t E, int32_t bm, int32_t* sid, int32_t* eid,
                         int32_t* npp, int32_t* scratch, size_t scratch_bytes, int32_t* dev_err, cudaStream_t st,
                         bool pdl, const int32_t* seg_counts = nullptr, int64_t seg_len = 0, int32_t* inv = nullptr);
size_t align_scratch_bytes(int64_t S, int32_t E);
cudaError_t launch_dequant(const hexmoe_parts& parts, int bits, int block, int n, int rows, int cols, int rows_pad,
                           int cols_pad, const int32_t* experts, void* out, int out_dtype, int64_t stride_e,
                           int64_t stride_row, int64_t row_off, cudaStream_t st);
// rows: optional [T*topk] map of y rows (nullptr: row t*topk + j), y_rows: rows of y.
cudaError_t launch_combine(const void* y, int y_dtype, int64_t T, int32_t topk, int32_t H, int64_t ld_y,
                           const int32_t* rows, int64_t y_rows, void* out, int out_dtype, cudaStream_t st, bool pdl);
// Tiled copy of one idx stack (hexmoe_tile_index layout).
cudaError_t launch_tile_index(const uint32_t* idx, int bits, int n, int rows_pad, int cols_pad, uint32_t* out,
                              cudaStream_t st);
cudaError_t launch_cast_to16(const float* x, void* out, bool bf16, int64_t n, cudaStream_t st);
// x_sorted[r] = x[row(sorted_ids[r])] for every plan row r < npp holding a slot,
// row(s) = s / topk, or slot_row[s] when a map is given (x in x_dtype, x_sorted
// 16-bit: bf16 for f32 input); padding rows untouched.
cudaError_t launch_gather_rows(const void* x, int x_dtype, int64_t T, int32_t H, const int32_t* sid,
                               const int32_t* npp, int64_t max_rows, int32_t topk, int64_t S, void* xs,
                               cudaStream_t st, bool pdl, const int32_t* slot_row = nullptr);
cudaError_t launch_route_topk(const void* logits, int dtype, int64_t T, int32_t E, int32_t k, int renorm, float* w,
                              int32_t* ids, cudaStream_t st);
// The layer's description (api.cu).
const hexmoe_layer_desc* layer_desc(const hexmoe_layer* layer);
// The layer forward up to its per-slot rows y[num_slots, hidden] (16-bit) over
// a general slot space: slot s has expert slot_expert[s], weight slot_weight[s]
// and activation row x[slot_row[s]]; with seg_counts, only the first
// seg_counts[g] slots of each seg_len-slot segment exist (the others are never
// read or written).  Workspace: slots_workspace_bytes(layer, num_slots, block_m);
// y == nullptr puts the rows into the workspace's own y region.  *y_used
// (optional) receives where they went.  slot_out (optional) routes the rows
// elsewhere (SlotOut); y is then not written.  gather (optional) replaces the
// gather pass (GatherHook); slot_row is then unused.
int forward_slot_space(const hexmoe_layer* layer, const void* x, int32_t x_dtype, int64_t num_slots,
                       const int32_t* slot_expert, const float* slot_weight, const int32_t* slot_row,
                       const int32_t* seg_counts, int64_t seg_len, void* y, int32_t block_m, void* workspace,
                       size_t workspace_bytes, cudaStream_t st, void** y_used = nullptr,
                       const SlotOut* slot_out = nullptr, const GatherHook* gather = nullptr);
size_t slots_workspace_bytes(const hexmoe_layer* layer, int64_t num_slots, int32_t block_m);
int32_t* device_error_word();  // address of this device's error word (nullptr on failure)
cudaError_t read_device_error(int32_t* value, bool clear);   // synchronous, current device
cudaError_t launch_build_expert_map(const hexmoe_layer_desc& d, int32_t* map, cudaStream_t st);
// Record `msg` as the calling thread's hexmoe_last_error() and return `code`.
int report_error(int code, const char* msg);
int report_cuda_error(cudaError_t e, const char* what);

}  // namespace hexmoe
