// decode_gemm.cu — small-batch HEX grouped GEMM for decode (align block_m 8).
//
// With a handful of tokens per expert every weight streams once and the tensor
// work is tiny; what bounds the layer is decoding HEX codes at the rate HBM
// delivers them.  These kernels decode into registers and feed the operands
// straight to mma.sync (m16n8k16, fp32 accumulate): no staging of operands in
// tensor memory and no hand-off of operand stages between warps.
//
//   gate/up (GLU):  act[row, o] = silu(x_row . Wg[e, o]) * (x_row . Wu[e, o])
//   down:           y[slot, o]  = (act_row . Wd[e, o]) * topk_weight[slot]
//
// Persistent CTAs over the tiles (align block b of <= 8 slots of one expert,
// 128 weight rows m), 8 x kSbGroups consumer warps + 1 producer warp:
//   producer   per tile the expert's code tables (built at layer creation: the
//              level table times each fp8 scale code and the expert scale,
//              rounded to the operand type) and the tile's fp8 scale codes into
//              one of two buffers (no global load on the consumers' path); per
//              128-input step the tile's codes (per projection 4 bulk copies of
//              2 KB: one 32-input block of all 128 rows each, from the layer's
//              tiled nibble copy) and the block's 8 activation rows (two TMA
//              boxes of 64 inputs, 128-B swizzle) into a ring of stages
//   consumers  warp w of a group owns rows 16w .. 16w+15 of the tile; the
//              groups take the 128-input steps in turn (more warps in flight to
//              hide shared-memory and decode latency); per step a warp decodes
//              its codes with prmt lookups into operand pairs and issues the
//              MMAs; at the end of a tile groups 1.. hand their sums to group 0,
//              which adds them in group order (a fixed order on every run) and
//              applies SwiGLU (gate/up) or the top-k weight (down)
//
// Fragments.  Lane (g = lane/4, q = lane%4) owns rows g and g+8 of its warp's
// 16 and the 32-input block q of each step.  The reduction index inside each
// 16-wide MMA is permuted the same way in A and B: MMA chunk c of a step takes,
// from lane (g, q), inputs q*32 + 4c + {0,1} (k = 2q, 2q+1) and q*32 + 4c +
// {2,3} (k = 2q+8, 2q+9), so a lane's A registers are its own decoded pairs and
// its B registers its own 32 consecutive inputs of token g.
//
// Shared-memory banks.  The 4 blocks of a step are copied 2048 + 32 bytes
// apart, so the 8 lanes of a quarter warp (rows g, g+1, blocks 0..3) read 8
// distinct 16-byte bank groups; table entries are shared by the 4 lanes of a
// row (one scale code per row and 128 inputs), at most 2 rows per quarter warp.
// Every wait is bounded: a lost arrival sets the device error word and the
// kernel returns after its in-flight copies land.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "decode.cuh"
#include "internal.cuh"

namespace hexmoe {

constexpr uint32_t kDecBlockStride = 2048 + 32;              // one 32-input block of 128 rows, padded
constexpr uint32_t kDecProjStride = 4 * kDecBlockStride;     // one projection of a step
constexpr uint32_t kDecXBytes = 2 * 8 * 128;                 // 8 rows x 128 inputs (two swizzled boxes)
constexpr uint32_t kDecCtrl = 1024;                          // barriers
#ifndef HEXMOE_SB_ACC
#define HEXMOE_SB_ACC 1
#endif
constexpr int kSbAcc = HEXMOE_SB_ACC;                         // accumulator sets per projection (1, 2, 4 or 8)
#ifndef HEXMOE_SB_GROUPS
#define HEXMOE_SB_GROUPS 2
#endif
constexpr int kSbGroups = HEXMOE_SB_GROUPS;   // groups of kSbWarps consumer warps taking the steps in turn
constexpr int kSbConsumers = kSbWarps * kSbGroups;

struct DecCtrl {
  uint64_t c_full[kDecStages], c_empty[kDecStages];   // step ring
  uint64_t t_full[2], t_empty[2];                     // table buffers
  uint64_t r_full[2], r_empty[2];                     // partial sums handed between step groups
  int32_t abort;
};
static_assert(sizeof(DecCtrl) <= kDecCtrl, "decode control block");

template <bool BF16>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

template <int BITS>
__device__ __forceinline__ uint4 dec8(uint32_t w, const uint4& lo, const uint4& hi) {
  if constexpr (BITS == 3) return dec8_n3(w, table8_from(lo));
  else return dec8_b4(w, table16_from(lo, hi));
}

struct DecTile {
  int b, m, tier, local, bits;
  bool ok;
};

__device__ __forceinline__ DecTile dec_tile(const DecParams& p, int t) {
  DecTile ti;
  ti.b = t / p.m_tiles;
  ti.m = t - ti.b * p.m_tiles;
  const int eg = __ldg(p.expert_ids + ti.b);
  const int map = (eg >= 0 && eg < p.num_experts) ? __ldg(p.expert_map + eg) : -1;
  ti.ok = map >= 0 && (map >> 16) < p.num_tiers;
  ti.tier = ti.ok ? (map >> 16) : 0;
  ti.local = map & 0xFFFF;
  ti.bits = p.bits[ti.tier];
  return ti;
}

__device__ __forceinline__ void dec_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > 200000000ull) return;
  }
}

// Producer (one lane): tables per tile, codes + activation boxes per step.
// Tile t takes its steps starting at step t % ksteps (then wrapping): the
// tiles in flight on all SMs start at different offsets of their 128 KB
// streams instead of all reading the same offset at once.
template <bool GLU>
__device__ void dec_producer(const DecParams& p, uint8_t* smem, DecCtrl* c, int num_tiles) {
  constexpr int NPROJ = GLU ? 2 : 1;
  volatile int* abort_flag = &c->abort;
  uint32_t cs = 0, cph = 0;
  int issued = 0, tissued = 0;
  bool aborted = false;
  for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x) {
    const DecTile ti = dec_tile(p, t);
    if (!ti.ok) continue;
    const uint32_t tabn = ti.bits == 3 ? 256u : 512u;
    const int tb = tissued & 1;
    if (!mbar_wait(&c->t_empty[tb], ((tissued >> 1) & 1) ^ 1, abort_flag, p.dev_err)) { aborted = true; break; }
    const uint32_t scb = 128u * static_cast<uint32_t>(p.k_pad / p.block);   // the tile's scale codes, one projection
    mbar_arrive_expect_tx(&c->t_full[tb], NPROJ * (tabn * 16u + scb));
    for (int j = 0; j < NPROJ; ++j) {
      bulk_load(smem + p.off_tab + (tb * NPROJ + j) * p.tab_bytes, p.tab[ti.tier][j] + static_cast<size_t>(ti.local) * tabn,
                tabn * 16u, &c->t_full[tb]);
      bulk_load(smem + p.off_sc + (tb * NPROJ + j) * p.sc_bytes,
                p.bs[ti.tier][j] + (static_cast<size_t>(ti.local) * p.rows_pad + static_cast<size_t>(ti.m) * 128) * (scb / 128u),
                scb, &c->t_full[tb]);
    }
    ++tissued;
    const size_t tile_base = (static_cast<size_t>(ti.local) * p.m_tiles + ti.m) * p.ksteps * kStepBytes;
    const int rot = t % p.ksteps;
    for (int k = 0; k < p.ksteps; ++k) {
      const int s = k + rot < p.ksteps ? k + rot : k + rot - p.ksteps;
      // a spinning wait: the ring refills the moment a stage frees (a sleeping
      // poll here lets the ring drain and the consumers starve)
      if (!mbar_wait(&c->c_empty[cs], cph ^ 1, abort_flag, p.dev_err)) { aborted = true; break; }
      uint8_t* st = smem + kDecCtrl + cs * p.stage_bytes;
      mbar_arrive_expect_tx(&c->c_full[cs], NPROJ * 4u * 2048u + kDecXBytes);
      tma_load_2d(st, &p.tm_b, &c->c_full[cs], s * 128, ti.b * kDecBlock);
      tma_load_2d(st + kDecXBytes / 2, &p.tm_b, &c->c_full[cs], s * 128 + 64, ti.b * kDecBlock);
      for (int j = 0; j < NPROJ; ++j)
        for (int q = 0; q < 4; ++q)
          bulk_load(st + kDecXBytes + j * kDecProjStride + q * kDecBlockStride,
                    p.idx_t[ti.tier][j] + tile_base + static_cast<size_t>(s) * kStepBytes + q * 2048u, 2048u,
                    &c->c_full[cs]);
      ++issued;
      if (++cs == static_cast<uint32_t>(p.ds)) { cs = 0; cph ^= 1; }
    }
  }
  if (aborted) {
    // let every copy already issued land before the CTA (and its smem) goes away
    for (int i = 1; i <= p.ds && i <= issued; ++i) {
      const int qq = issued - i;
      dec_drain(&c->c_full[qq % p.ds], (qq / p.ds) & 1);
    }
    for (int i = 1; i <= 2 && i <= tissued; ++i) {
      const int qq = tissued - i;
      dec_drain(&c->t_full[qq & 1], (qq >> 1) & 1);
    }
  }
}

// Consumer warp `cw`: rows 16*(cw % kSbWarps) .. +15 of each tile, the steps s
// with s % kSbGroups == cw / kSbWarps.  Groups 1.. hand their partial sums to
// group 0 through shared memory (two buffers); group 0 adds them in group order
// and runs the epilogue.
template <bool GLU, bool BF16>
__device__ void dec_consumer(const DecParams& p, uint8_t* smem, DecCtrl* c, int num_tiles, int cw, int lane) {
  constexpr int NPROJ = GLU ? 2 : 1;
  volatile int* abort_flag = &c->abort;
  const int g = lane >> 2, q = lane & 3;
  const int warp = cw % kSbWarps, grp = cw / kSbWarps;
  float* red = reinterpret_cast<float*>(smem + p.off_red);   // [2][kSbGroups-1][kSbWarps][NPROJ][4][32]
  const uint32_t spr = static_cast<uint32_t>(p.k_pad / p.block);
  uint32_t cs = 0, cph = 0;
  int tused = 0;
  uint16_t* out16 = reinterpret_cast<uint16_t*>(p.out);
  for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
    const DecTile ti = dec_tile(p, t);
    if (!ti.ok) {
      if (warp == 0 && lane == 0) atomicOr(p.dev_err, kDevErrNoTier);
      continue;
    }
    const int tb = tused & 1;
    if (!mbar_wait(&c->t_full[tb], (tused >> 1) & 1, abort_flag, p.dev_err)) return;
    const uint8_t* tabs = smem + p.off_tab + tb * NPROJ * p.tab_bytes;
    const int r_lo = ti.m * 128 + warp * 16 + g;            // rows r_lo and r_lo + 8 of the expert
    const uint8_t* sb[NPROJ];                                // this lane's row r_lo in the tile's scale codes (smem)
#pragma unroll
    for (int j = 0; j < NPROJ; ++j) sb[j] = smem + p.off_sc + (tb * NPROJ + j) * p.sc_bytes + (warp * 16 + g) * spr;
    // kSbAcc independent accumulator sets per projection (chunk c goes to set c %
    // kSbAcc), added in set order at the end: short dependency chains of MMAs
    float acc[NPROJ][kSbAcc][4];
#pragma unroll
    for (int j = 0; j < NPROJ; ++j)
#pragma unroll
      for (int a = 0; a < kSbAcc; ++a)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][a][i] = 0.f;
    bool aborted = false;
    auto run = [&](auto bits_c) {
      constexpr int BITS = decltype(bits_c)::value;
      // scale codes of the next step, loaded one step ahead
      uint32_t scn[NPROJ][2];
      auto load_sc = [&](int s) {
        const uint32_t sci = static_cast<uint32_t>((s * 128 + q * 32) / p.block);
#pragma unroll
        for (int j = 0; j < NPROJ; ++j) {
          scn[j][0] = sb[j][sci];
          scn[j][1] = sb[j][8 * spr + sci];
        }
      };
      const int rot = t % p.ksteps;
      auto step_at = [&](int k) { return k + rot < p.ksteps ? k + rot : k + rot - p.ksteps; };
      if (grp < p.ksteps) load_sc(step_at(grp));
#pragma unroll 1
      for (int k = 0; k < p.ksteps; ++k) {
        if (k % kSbGroups != grp) {           // another group's step: only the ring position moves
          if (++cs == static_cast<uint32_t>(p.ds)) { cs = 0; cph ^= 1; }
          continue;
        }
        uint32_t sc[NPROJ][2];
#pragma unroll
        for (int j = 0; j < NPROJ; ++j) { sc[j][0] = scn[j][0]; sc[j][1] = scn[j][1]; }
        if (k + kSbGroups < p.ksteps) load_sc(step_at(k + kSbGroups));
        if (!mbar_wait(&c->c_full[cs], cph, abort_flag, p.dev_err)) { aborted = true; return; }
        const uint8_t* st = smem + kDecCtrl + cs * p.stage_bytes;
        // token g's 32 inputs of block q: half q/2 of the step, 16-byte chunks (q%2)*4 .. +3, swizzled by row
        uint32_t xr[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t cc = static_cast<uint32_t>((q & 1) * 4 + i);
          const uint4 v = *reinterpret_cast<const uint4*>(st + (q >> 1) * 1024 + g * 128 + ((cc ^ g) << 4));
          xr[4 * i] = v.x; xr[4 * i + 1] = v.y; xr[4 * i + 2] = v.z; xr[4 * i + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < NPROJ; ++j) {
          const uint8_t* cb = st + kDecXBytes + j * kDecProjStride + q * kDecBlockStride + (warp * 16 + g) * 16;
          const uint4 w0 = *reinterpret_cast<const uint4*>(cb);
          const uint4 w1 = *reinterpret_cast<const uint4*>(cb + 128);
          const uint4* tab = reinterpret_cast<const uint4*>(tabs + j * p.tab_bytes);
          const uint4 t0 = tab[sc[j][0]], t1 = tab[sc[j][1]];
          uint4 h0 = t0, h1 = t1;
          if constexpr (BITS == 4) {
            h0 = tab[256 + sc[j][0]];
            h1 = tab[256 + sc[j][1]];
          }
          const uint32_t wa[4] = {w0.x, w0.y, w0.z, w0.w}, wb[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int jw = 0; jw < 4; ++jw) {
            const uint4 oa = dec8<BITS>(wa[jw], t0, h0);   // row g: inputs 8jw .. 8jw+7 of block q
            const uint4 ob = dec8<BITS>(wb[jw], t1, h1);   // row g + 8
            mma16816<BF16>(acc[j][(2 * jw) % kSbAcc], oa.x, ob.x, oa.y, ob.y, xr[4 * jw], xr[4 * jw + 1]);
            mma16816<BF16>(acc[j][(2 * jw + 1) % kSbAcc], oa.z, ob.z, oa.w, ob.w, xr[4 * jw + 2], xr[4 * jw + 3]);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&c->c_empty[cs]);
        if (++cs == static_cast<uint32_t>(p.ds)) { cs = 0; cph ^= 1; }
      }
    };
    if (ti.bits == 3) run(std::integral_constant<int, 3>{});
    else run(std::integral_constant<int, 4>{});
    if (aborted) return;
    __syncwarp();
    if (lane == 0) mbar_arrive(&c->t_empty[tb]);
    const int par = tused & 1, use = tused >> 1;
    ++tused;
#pragma unroll
    for (int j = 0; j < NPROJ; ++j)
#pragma unroll
      for (int a = 1; a < kSbAcc; ++a)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][0][i] += acc[j][a][i];
    if constexpr (kSbGroups > 1) {
      float* rb = red + static_cast<size_t>(par) * (kSbGroups - 1) * kSbWarps * NPROJ * 128;
      if (grp > 0) {
        // hand the partial sums to group 0 (the buffer of this parity is free once
        // group 0 has read what was written into it two tiles ago)
        if (!mbar_wait(&c->r_empty[par], (use & 1) ^ 1, abort_flag, p.dev_err)) return;
        float* dst = rb + ((grp - 1) * kSbWarps + warp) * NPROJ * 128;
#pragma unroll
        for (int j = 0; j < NPROJ; ++j)
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[(j * 4 + i) * 32 + lane] = acc[j][0][i];
        __syncwarp();
        if (lane == 0) mbar_arrive(&c->r_full[par]);
        continue;
      }
      if (!mbar_wait(&c->r_full[par], use & 1, abort_flag, p.dev_err)) return;
      for (int gg = 1; gg < kSbGroups; ++gg) {
        const float* src = rb + ((gg - 1) * kSbWarps + warp) * NPROJ * 128;
#pragma unroll
        for (int j = 0; j < NPROJ; ++j)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[j][0][i] += src[(j * 4 + i) * 32 + lane];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&c->r_empty[par]);
    }
    // epilogue: c0, c1 = (row g, tokens 2q, 2q+1), c2, c3 = (row g+8, same tokens)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int n = 2 * q + (i & 1);
      const int row = r_lo + (i >> 1) * 8;
      const int slot = __ldg(p.sorted_ids + static_cast<int64_t>(ti.b) * kDecBlock + n);
      if (slot >= p.num_slots || row >= p.rows_store) continue;
      float r;
      int64_t o;
      if constexpr (GLU) {
        const float gg = acc[0][0][i];
        r = __fdividef(gg, 1.0f + __expf(-gg)) * acc[1][0][i];   // silu(gate) * up, as the tcgen05 epilogue
        o = (static_cast<int64_t>(ti.b) * kDecBlock + n) * p.ld_out + row;
      } else {
        r = acc[0][0][i] * __ldg(p.topk_w + slot);
        o = static_cast<int64_t>(slot) * p.ld_out + row;
      }
      out16[o] = static_cast<uint16_t>(pack2<BF16>(r, 0.f) & 0xFFFFu);
    }
  }
}

template <bool GLU, bool BF16>
__global__ void __launch_bounds__((kSbConsumers + 1) * 32, 1) hex_decode_kernel(const __grid_constant__ DecParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  DecCtrl* c = reinterpret_cast<DecCtrl*>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kDecStages; ++i) { mbar_init(&c->c_full[i], 1); mbar_init(&c->c_empty[i], kSbWarps); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&c->t_full[i], 1); mbar_init(&c->t_empty[i], kSbConsumers);
      mbar_init(&c->r_full[i], kSbWarps * (kSbGroups - 1)); mbar_init(&c->r_empty[i], kSbWarps);
    }
    c->abort = 0;
    fence_mbar_init();
  }
  if (warp == kSbConsumers && lane == 0) prefetch_tmap(&p.tm_b);
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();   // the plan and the B rows come from the previous kernels
  const int num_tiles = (__ldg(p.npp) / kDecBlock) * p.m_tiles;
  if (warp == kSbConsumers) {
    if (lane == 0) dec_producer<GLU>(p, smem, c, num_tiles);
  } else {
    dec_consumer<GLU, BF16>(p, smem, c, num_tiles, warp, lane);
  }
}

template <bool GLU, bool BF16>
static cudaError_t launch_dec(const DecParams& p, int grid, cudaStream_t st, bool pdl) {
  auto kern = hex_decode_kernel<GLU, BF16>;
  static std::atomic<int> configured_bytes[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const int bytes = static_cast<int>(p.smem_bytes);
  if (bytes > configured_bytes[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(mu);
    if (bytes > configured_bytes[dev].load(std::memory_order_relaxed)) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      if (e != cudaSuccess) return e;
      configured_bytes[dev].store(bytes, std::memory_order_release);
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3((kSbConsumers + 1) * 32);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

// Shared-memory carve-up for one projection pair (2) or one projection (1).
bool plan_decode(DecParams& p, int nproj) {
  p.stage_bytes = (kDecXBytes + nproj * kDecProjStride + 1023u) / 1024u * 1024u;
  p.tab_bytes = 512u * 16u;
  p.sc_bytes = (128u * static_cast<uint32_t>(p.k_pad / p.block) + 127u) / 128u * 128u;
  const uint32_t fixed = 2u * nproj * (p.tab_bytes + p.sc_bytes) + 2u * (kSbGroups - 1) * kSbWarps * nproj * 128u * 4u;
  const uint32_t budget = 227u * 1024u - 1024u - kDecCtrl;   // dynamic smem per CTA, minus alignment slack
  if (fixed + 2u * p.stage_bytes > budget) return false;
  p.ds = static_cast<int32_t>(std::min<uint32_t>(kDecStages, (budget - fixed) / p.stage_bytes));
  p.off_tab = kDecCtrl + p.ds * p.stage_bytes;
  p.off_sc = p.off_tab + 2u * nproj * p.tab_bytes;
  p.off_red = p.off_sc + 2u * nproj * p.sc_bytes;
  p.smem_bytes = p.off_red + 2u * (kSbGroups - 1) * kSbWarps * nproj * 128u * 4u + 1024u;
  return true;
}

cudaError_t launch_decode_gemm(const DecParams& p, bool glu, bool bf16, int grid, cudaStream_t st, bool pdl) {
  if (glu) return bf16 ? launch_dec<true, true>(p, grid, st, pdl) : launch_dec<true, false>(p, grid, st, pdl);
  return bf16 ? launch_dec<false, true>(p, grid, st, pdl) : launch_dec<false, false>(p, grid, st, pdl);
}

}  // namespace hexmoe
