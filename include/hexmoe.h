/*
 * hexmoe.h — C ABI of libhexmoe.so, the sm_100a HEX fused-MoE layer.
 *
 * HEX (Header-Encoded eXperts) stores one expert matrix W [rows, cols] as
 *   idx          uint32 [rows, cols/32*bits]  one little-endian bit stream of `bits`
 *                                            (3 or 4) per block of 32 inputs
 *   block_scale  uint8  [rows, cols/block]   fp8 e4m3 code per `block` inputs
 *   expert_scale float32                     one per matrix
 *   levels       float32 [2^bits]            the expert's own sorted table
 *   W[o, i] = levels[idx(o, i)] * (fp8(block_scale[o, i / block]) * expert_scale)
 * stacked over the n experts of a tier (experts sharing one index width).  The
 * reference layout (blackhole/anatomy/hex.py:21-31, runtime/blackhole_runtime/
 * hex_ref.py:1-12) fixes block = 32; block = 128 is accepted as well (same bit
 * stream, one scale per 128 inputs).
 *
 * Every entry point takes plain device pointers and sizes, runs on the caller's
 * stream (a cudaStream_t passed as void*, NULL = legacy default stream), makes
 * no host synchronisation and allocates no device memory: scratch is a caller
 * buffer sized by the matching *_workspace_bytes() call.  The exceptions are
 * hexmoe_layer_create / hexmoe_layer_destroy (load time: they synchronise and
 * own the layer's tiled index copy) and hexmoe_device_status.  Calls are re-entrant;
 * a layer handle is immutable after creation and may be shared across streams.
 * Every call returns HEXMOE_OK or an error code; hexmoe_last_error() gives the
 * message of the calling thread's last failure.
 */
#ifndef HEXMOE_H
#define HEXMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define HEXMOE_API __attribute__((visibility("default")))
#else
#define HEXMOE_API
#endif

#define HEXMOE_ABI_VERSION 1
#define HEXMOE_MAX_TIERS 4

/* Status codes.  The reference raises AssertionError / ValueError for the
 * argument cases (hex_moe.py:289-290, vllm_hex.py:101-139). */
enum hexmoe_status {
  HEXMOE_OK = 0,
  HEXMOE_E_ARG = 1,         /* bad shape, size, pointer alignment or value     */
  HEXMOE_E_DTYPE = 2,       /* unsupported dtype code                         */
  HEXMOE_E_CUDA = 3,        /* a CUDA runtime / driver call failed            */
  HEXMOE_E_UNSUPPORTED = 4, /* no sm_100 device, or a limit of this build      */
  HEXMOE_E_DEVICE = 5       /* a kernel flagged an error (see hexmoe_device_status) */
};

/* Element types of activations / outputs. */
enum hexmoe_dtype { HEXMOE_F32 = 0, HEXMOE_BF16 = 1, HEXMOE_F16 = 2 };
/* Element types of expert-id tensors. */
enum hexmoe_index_dtype { HEXMOE_I32 = 0, HEXMOE_I64 = 1 };

/* One projection of one tier: the four HEX parts, stacked over the tier's experts.
 * `rows`/`cols` of the stack are given by the owning layer (rows_pad, cols_pad). */
typedef struct hexmoe_parts {
  const uint32_t* idx;          /* [n, rows_pad, cols_pad/32*bits]       */
  const uint8_t* block_scale;   /* [n, rows_pad, cols_pad/block]         */
  const float* expert_scale;    /* [n]                                   */
  const float* levels;          /* [n, 2^bits]                           */
} hexmoe_parts;

/* One tier (runtime/blackhole_runtime/hex_moe.py:174-198, HexTier). */
typedef struct hexmoe_tier {
  int32_t bits;                 /* 3 (8 levels) or 4 (16 levels)         */
  int32_t n;                    /* experts in this tier                  */
  const int32_t* experts;       /* device int32 [n]: global expert ids   */
  hexmoe_parts gate, up, down;  /* gate/up: [I, H], down: [H, I]         */
} hexmoe_tier;

/* A routed-expert SwiGLU MoE layer split over HEX tiers.
 * hidden_pad / inter_pad are the row lengths the parts are stored with: a
 * multiple of 128 at least hidden / inter.  They equal hidden / inter for every
 * production shape (the parts are then read exactly as the reference stores
 * them); smaller shapes are zero-padded once at load time by the host layer. */
typedef struct hexmoe_layer_desc {
  int32_t num_experts;          /* E: global ids are 0..E-1              */
  int32_t hidden;               /* H                                     */
  int32_t inter;                /* I (moe_intermediate)                  */
  int32_t hidden_pad;
  int32_t inter_pad;
  int32_t block;                /* fp8 scale block: 32 or 128            */
  int32_t num_tiers;            /* 1..HEXMOE_MAX_TIERS                   */
  hexmoe_tier tiers[HEXMOE_MAX_TIERS];
  /* device int32 [num_experts]: (tier << 16) | local index of every global
   * expert, -1 where no tier holds it (hexmoe_build_expert_map fills it) */
  const int32_t* expert_map;
} hexmoe_layer_desc;

typedef struct hexmoe_layer hexmoe_layer;   /* opaque, immutable after create */

/* Library identity. */
HEXMOE_API int hexmoe_abi_version(void);
HEXMOE_API const char* hexmoe_last_error(void);

/* Reads (and, with clear != 0, resets) the device error word of `device` that
 * kernels set on a bounded-wait timeout or an out-of-range expert id.  Blocks
 * until the device is idle.  0 means no error was recorded. */
HEXMOE_API int hexmoe_device_status(int device, int clear, int32_t* status_out);

/* Fills map_out[num_experts] (device) from desc->tiers[].experts: the
 * global -> (tier, local) lookup of HexTier.prepare (hex_moe.py:193-196),
 * for all tiers at once.  desc->expert_map is not read. */
HEXMOE_API int hexmoe_build_expert_map(const hexmoe_layer_desc* desc, int32_t* map_out, void* stream);

/* Builds the kernel-side view of a layer on the current device: the
 * global->(tier, local) expert map and a tiled copy of every idx stack
 * (hexmoe_tile_index layout), which the grouped GEMM streams instead of the
 * stored stacks.  Replaces the per-call argument marshalling of _launch
 * (hex_moe.py:286-301) and the lookup built in HexTier.prepare
 * (hex_moe.py:193-196).
 * The copy takes n * rows_pad * cols_pad / 2 bytes of device memory per
 * projection (one cudaMalloc, freed by hexmoe_layer_destroy) and snapshots the
 * index streams: create waits for the device to go idle first, so it must not
 * run inside stream capture, and later writes to the stacks are not seen.
 * The stored stacks stay in use for hexmoe_dequant. */
HEXMOE_API int hexmoe_layer_create(const hexmoe_layer_desc* desc, hexmoe_layer** out);
HEXMOE_API int hexmoe_layer_destroy(hexmoe_layer* layer);

/* The tiled index layout the grouped GEMM reads.  idx: [n, rows_pad,
 * cols_pad/32*bits] u32, the stored HEX stream (hex_ref.pack,
 * hex_ref.py:49-61: per 32-input block `bits` little-endian words).  out:
 * [n, rows_pad/128, cols_pad/128, 4, 4, 32, 4] u32 (n*rows_pad*cols_pad/2
 * bytes): for weight-row tile m, 128-input step s, 32-row slice h, 32-input
 * block b of the step and position p, 4 words whose nibble i of word j holds
 * the code of input s*128 + b*32 + j*8 + i of tile row h*32 + (p ^ (2*b))
 * (3-bit codes with bit 3 clear; the row permutation spreads the shared-memory
 * banks of the kernels that read several blocks of one row at once).  One step
 * of one tile is 8 KB of contiguous memory, each 32-row slice of it 2 KB.
 * rows_pad and cols_pad: multiples of 128.  Asynchronous on `stream`. */
HEXMOE_API int hexmoe_tile_index(const uint32_t* idx, int32_t bits, int32_t n, int32_t rows_pad,
                                 int32_t cols_pad, uint32_t* out, void* stream);

/* Scratch bytes hexmoe_forward needs for `tokens` tokens at top-`topk` with
 * tile height `block_m` and activation dtype x_dtype.  block_m 16, 32, 64 or
 * 128: the tcgen05 grouped GEMM with tiles of that many slots of one expert;
 * 8: the small-batch (decode) kernels, mma.sync over weights decoded in
 * registers, one CTA per 8 slots of one expert and 16 weight rows; 0 =
 * automatic, as default_config hex_moe.py:264-283 picks it. */
HEXMOE_API size_t hexmoe_forward_workspace_bytes(const hexmoe_layer* layer, int64_t tokens, int32_t topk,
                                      int32_t block_m, int32_t x_dtype);

/* Routed-expert output out[T, H] = sum_j w[t, j] * down_e(silu(gate_e x_t) * up_e x_t),
 * e = topk_ids[t, j].  Replaces hex_moe (hex_moe.py:374-382) / hex_moe_fused
 * (hex_moe.py:304-325).  x [T, H] (row stride H) in x_dtype; topk_weights f32
 * [T, topk]; topk_ids [T, topk] in ids_dtype (global ids); out [T, H] in
 * out_dtype (x_dtype, or F32).  The activation handed from gate/up to down is
 * rounded to the compute dtype (bf16 for F32 inputs) as in the reference. */
HEXMOE_API int hexmoe_forward(const hexmoe_layer* layer, const void* x, int32_t x_dtype, int64_t tokens,
                   int32_t topk, const float* topk_weights, const void* topk_ids,
                   int32_t ids_dtype, void* out, int32_t out_dtype, int32_t block_m,
                   void* workspace, size_t workspace_bytes, void* stream);

/* hexmoe_forward up to, not including, the combine: y[t*topk + j, :] =
 * w[t, j] * down_e(silu(gate_e x_t) * up_e x_t) rounded to the 16-bit compute
 * type (x_dtype, BF16 for F32 x), one row per slot in slot order.  The
 * expert-parallel path (blackhole_b200.ep) runs its received rows through this
 * at topk = 1 and sums them on their source rank.  Same workspace as
 * hexmoe_forward. */
HEXMOE_API int hexmoe_forward_slots(const hexmoe_layer* layer, const void* x, int32_t x_dtype, int64_t tokens,
                                    int32_t topk, const float* topk_weights, const void* topk_ids,
                                    int32_t ids_dtype, void* y, int32_t block_m, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* hexmoe_forward for callers that cannot allocate device memory and so have no
 * workspace to pass (a serving process whose memory pool already holds nearly
 * all of the GPU, a plugin host that owns every device allocation, a loop that
 * must not synchronise on cudaMalloc).  No counterpart in the reference: its
 * Triton launches take their scratch from torch's allocator.  Same arguments
 * and result as hexmoe_forward, minus the workspace: the scratch is one fixed
 * array of HEXMOE_NOALLOC_SCRATCH_BYTES inside the library, held by every GPU
 * that loads it until the process exits.  Calls whose scratch need
 * (hexmoe_forward_workspace_bytes) exceeds it fail with HEXMOE_E_ARG.  The
 * first call on a device looks the array up on that device (make it before any
 * stream capture).  All calls on a device share the array: calls that overlap
 * on the GPU race and must be ordered by the caller.  Allocates nothing. */
#define HEXMOE_NOALLOC_SCRATCH_BYTES (32u << 20)
HEXMOE_API int hexmoe_forward_noalloc(const hexmoe_layer* layer, const void* x, int32_t x_dtype, int64_t tokens,
                                      int32_t topk, const float* topk_weights, const void* topk_ids,
                                      int32_t ids_dtype, void* out, int32_t out_dtype, int32_t block_m,
                                      void* stream);

/* The phases of hexmoe_forward, for callers that own the plan (or time the
 * phases apart).  They replace the two _launch calls per tier and the sum of
 * hex_moe_fused (hex_moe.py:286-301, 321-325); one call covers every tier.
 *   plan      sorted_ids / expert_ids / npp from hexmoe_align with block_m
 *   gather    x_sorted[r] = x[sorted_ids[r] / topk] for every plan row r that
 *             holds a slot; x_sorted [max_blocks*block_m, hidden], 16-bit
 *             (BF16 for an F32 x), padding rows untouched
 *   gate/up   act[r, o] = silu(x_sorted[r] . Wg[e, o]) * (x_sorted[r] . Wu[e, o])
 *             for every plan row r, rounded to x_sorted's dtype; act is
 *             [max_blocks*block_m, inter_pad] (padding rows untouched)
 *   down      y[slot, h] = (act[r] . Wd[e, h]) * topk_weights[slot], slot =
 *             sorted_ids[r]; y [tokens*topk, hidden] in act's dtype
 *   combine   out[t, h] = sum_j y[t*topk + j, h] (fp32 sum, rounded once)
 * x / act / y dtypes: BF16 or F16. */
HEXMOE_API int hexmoe_gather(const void* x, int32_t x_dtype, int64_t tokens, int32_t hidden, int32_t topk,
                             int32_t num_experts, const int32_t* sorted_ids, const int32_t* npp,
                             int32_t block_m, void* x_sorted, void* stream);
HEXMOE_API int hexmoe_gate_up(const hexmoe_layer* layer, const void* x_sorted, int32_t x_dtype, int64_t tokens,
                              int32_t topk, const int32_t* sorted_ids, const int32_t* expert_ids,
                              const int32_t* npp, int32_t block_m, void* act, void* stream);
HEXMOE_API int hexmoe_down(const hexmoe_layer* layer, const void* act, int32_t act_dtype, int64_t tokens,
                           int32_t topk, const float* topk_weights, const int32_t* sorted_ids,
                           const int32_t* expert_ids, const int32_t* npp, int32_t block_m, void* y,
                           void* stream);
HEXMOE_API int hexmoe_combine(const void* y, int32_t y_dtype, int64_t tokens, int32_t topk, int32_t hidden,
                              void* out, int32_t out_dtype, void* stream);

/* The combine with the slot rows given by a map: out[t, h] = sum_j
 * y[rows[t*topk + j], h] (fp32 sum in j order, rounded once), for per-slot
 * rows that come back from expert-parallel ranks in dispatch order rather than
 * slot order.  y [y_rows, hidden]; a row index outside 0..y_rows-1 adds nothing
 * and sets the device error word. */
HEXMOE_API int hexmoe_combine_rows(const void* y, int32_t y_dtype, int64_t y_rows, int64_t tokens, int32_t topk,
                                   int32_t hidden, const int32_t* rows, void* out, int32_t out_dtype,
                                   void* stream);

/* Group slots by expert, each expert's run padded to block_m (align,
 * hex_moe.py:201-222): sorted_ids int32 [max_blocks*block_m] (padding = S),
 * expert_ids int32 [max_blocks] (-1 = unused), npp int32 [1] = padded length,
 * with max_blocks = ceil(S/block_m) + min(E, S).  Stable: slots of one expert
 * keep their order, so the output equals the reference's bit for bit.
 * workspace: hexmoe_align_workspace_bytes(S, E) bytes (16-byte aligned; 0 for
 * small S, where NULL is fine).  With it, large S is aligned by many CTAs;
 * without it (NULL or too small) by one, with the same result. */
HEXMOE_API size_t hexmoe_align_workspace_bytes(int64_t num_slots, int32_t num_experts);
HEXMOE_API int hexmoe_align(const void* ids, int32_t ids_dtype, int64_t num_slots, int32_t num_experts,
                 int32_t block_m, int32_t* sorted_ids, int32_t* expert_ids, int32_t* npp,
                 void* workspace, size_t workspace_bytes, void* stream);

/* Dequantize one projection of one tier (the _hex_dequant_kernel launches of
 * dequant_all, hex_moe.py:154-168 and 328-346): for local expert e < n, row o <
 * rows, input i < cols,
 *   out[experts[e] * stride_e + (row_off + o) * stride_row + i]
 *     = levels[e, code] * (fp8(block_scale[e, o, i/block]) * expert_scale[e])
 * computed in fp32 with round-to-nearest products, then rounded to out_dtype
 * (RNE).  Bit-exact against blackhole/anatomy/hex.py:180-204.  experts may be
 * NULL (then e itself is the output index).  rows_pad/cols_pad: stored shape. */
HEXMOE_API int hexmoe_dequant(const hexmoe_parts* parts, int32_t bits, int32_t block, int32_t n,
                   int32_t rows, int32_t cols, int32_t rows_pad, int32_t cols_pad,
                   const int32_t* experts, void* out, int32_t out_dtype, int64_t stride_e,
                   int64_t stride_row, int64_t row_off, void* stream);

/* ---------------------------------------------------------------------------
 * Expert parallelism over NVLink peer memory.  No counterpart in the reference,
 * which runs each MoE layer on one GPU and refuses expert parallelism
 * (vllm_hex.py:101-102); these replace, for a multi-GPU node, what hex_moe
 * (hex_moe.py:374-382) does on one GPU.
 *
 * Experts are sharded contiguously: rank r of `world` owns global experts
 * [r*P, (r+1)*P), P = ceil(num_experts / world), and runs them as a
 * hexmoe_layer built from its own tiers only (global expert ids kept).  Each
 * rank's context owns one device region that every other rank maps through
 * CUDA IPC; kernels store slot records and per-slot output rows straight into
 * the owning rank's region and load token rows from the source's region, with
 * plain loads and stores, and signal with epoch flags
 * (release / acquire at system scope).  Nothing synchronises with the host, so
 * a forward can be captured in a CUDA graph.
 *
 * Per forward: every token row crosses once per rank that owns one of its
 * experts (not once per slot), pulled by the owner; the owner runs its experts on the received
 * slots, and its down GEMM stores each slot's weighted output row (rounded
 * once to the row dtype) straight into the home rank's buffer at the slot's
 * place; the home rank sums a token's k rows in top-k order in fp32 and rounds
 * once.  That is the single-GPU layer's arithmetic: the output equals
 * hexmoe_forward's bit for bit at every world size.
 *
 * Protocol rules: every rank calls init, exchanges handles (hexmoe_ep_handle,
 * gathered in rank order by the caller), connects, and then runs the same
 * sequence of forwards (dispatch -> experts -> combine) on one stream; a rank
 * with no tokens still takes part.  Destroy only after every rank has finished
 * its last forward (a host barrier).  A peer that stops taking part makes the
 * others' bounded waits (2 s) run out: they set the timeout bit of the device
 * error word and return instead of hanging.  Expert ids outside 0..E-1 are
 * dropped and set the expert-id bit. */
#define HEXMOE_EP_MAX_WORLD 8
#define HEXMOE_EP_HANDLE_BYTES 64
typedef struct hexmoe_ep hexmoe_ep;

/* Context of rank `rank` of `world` on the current device, for up to
 * max_tokens tokens per rank per forward, top-`topk` over num_experts global
 * experts of width `hidden`; rows travel as row_dtype (BF16 or F16).  Allocates
 * the shared region ((1 + topk) x max_tokens x hidden x 2 bytes of rows plus
 * ~12 x world x max_tokens x (topk + 1) bytes of records) and its private
 * state; synchronises the device. */
HEXMOE_API int hexmoe_ep_init(int32_t rank, int32_t world, int32_t num_experts, int32_t hidden, int32_t topk,
                              int64_t max_tokens, int32_t row_dtype, hexmoe_ep** out);
/* The CUDA IPC handle (HEXMOE_EP_HANDLE_BYTES) of this rank's region. */
HEXMOE_API int hexmoe_ep_handle(const hexmoe_ep* ep, void* handle_out);
/* Maps every other rank's region from the gathered handles [world][64] (rank order). */
HEXMOE_API int hexmoe_ep_connect(hexmoe_ep* ep, const void* handles);
/* Scratch bytes hexmoe_ep_experts / hexmoe_ep_forward need with this rank's layer. */
HEXMOE_API size_t hexmoe_ep_workspace_bytes(const hexmoe_ep* ep, const hexmoe_layer* local, int32_t block_m);
/* Phase 1: route this rank's tokens to the owners of their experts (x [T,
 * hidden] in row_dtype, or F32 with BF16 rows; weights f32 [T, topk]; ids
 * [T, topk] global). */
HEXMOE_API int hexmoe_ep_dispatch(hexmoe_ep* ep, const void* x, int32_t x_dtype, int64_t tokens,
                                  const float* topk_weights, const void* topk_ids, int32_t ids_dtype, void* stream);
/* Phase 2: wait for every rank's dispatch, run `local` (NULL on a rank that owns
 * no experts) on the received slots; the down GEMM returns every slot's row to
 * its home rank as it computes it. */
HEXMOE_API int hexmoe_ep_experts(hexmoe_ep* ep, const hexmoe_layer* local, int32_t block_m, void* workspace,
                                 size_t workspace_bytes, void* stream);
/* Phase 3: wait for every rank's return; out [T, hidden] (row_dtype or F32). */
HEXMOE_API int hexmoe_ep_combine(hexmoe_ep* ep, int64_t tokens, void* out, int32_t out_dtype, void* stream);
/* The three phases in one call. */
HEXMOE_API int hexmoe_ep_forward(hexmoe_ep* ep, const hexmoe_layer* local, const void* x, int32_t x_dtype,
                                 int64_t tokens, const float* topk_weights, const void* topk_ids, int32_t ids_dtype,
                                 void* out, int32_t out_dtype, int32_t block_m, void* workspace,
                                 size_t workspace_bytes, void* stream);
HEXMOE_API int hexmoe_ep_destroy(hexmoe_ep* ep);

/* Router: probabilities = softmax(logits[t, :E]) in fp32, the topk largest
 * (ties: lower expert id first), renormalised to sum 1 when renormalize != 0
 * (Qwen3 norm_topk_prob).  logits f32/bf16/f16 [T, E] row stride E.  The
 * reference leaves routing to vLLM (vllm_hex.py:145-146); this is its
 * counterpart for callers that route on the device themselves. */
HEXMOE_API int hexmoe_route_topk(const void* logits, int32_t logits_dtype, int64_t tokens,
                      int32_t num_experts, int32_t topk, int32_t renormalize,
                      float* topk_weights, int32_t* topk_ids, void* stream);

/* ---- The quantizer: the producer side of the HEX format.
 * Replaces blackhole/anatomy/hex.py:207-227 `quantize(W, L, block, energy, H)`
 * (block_scales 60-70, fit_table 73-90, nearest 93-95, GPTQ onto the table
 * gptq_table 256-282, pack_bits 136-150), batched over a stack of n matrices.
 * Without a Hessian it equals the reference bit for bit.  W [n, out, in] f32
 * (16-byte aligned), in a multiple of `block` (32 or 128); levels 8 or 16.
 * energy (optional) [n, in] f32: the per-input mean x^2 that weights the table
 * fit by energy * block_scale^2.  sample_idx (optional) [sample] int64 flat
 * positions in [out, in]: the values the table is fitted on (the reference
 * draws 2^17 of them with numpy default_rng(0) when a matrix has more); null
 * fits every value.  iters: Lloyd iterations (20 in the reference).
 * hinv_u / dead (optional, together): GPTQ rounding instead of nearest, with
 * hinv_u [n, in, in] f32 the upper Cholesky factor of each matrix's damped
 * inverse Hessian and dead [n, in] u8 its dead inputs (hex.py:234-253 prepares
 * both from H; blackhole_b200.quant does it on the device).  Outputs, in the
 * layout of one tier's projection: idx_out [n, out, in/32*bits] u32,
 * block_scale_out [n, out, in/block] u8 (fp8 e4m3 codes), expert_scale_out [n]
 * f32, levels_out [n, levels] f32.  Workspace: hexmoe_quantize_workspace_bytes
 * (256-byte aligned; gptq != 0 when hinv_u is given).  Asynchronous on
 * `stream`. */
HEXMOE_API size_t hexmoe_quantize_workspace_bytes(int32_t n, int32_t out, int32_t in, int32_t block,
                                                  int64_t sample, int32_t weighted, int32_t gptq);
HEXMOE_API int hexmoe_quantize(const float* W, int32_t n, int32_t out, int32_t in, int32_t levels, int32_t block,
                               const float* energy, const int64_t* sample_idx, int64_t sample, int32_t iters,
                               const float* hinv_u, const uint8_t* dead, uint32_t* idx_out,
                               uint8_t* block_scale_out, float* expert_scale_out, float* levels_out,
                               void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* HEXMOE_H */
