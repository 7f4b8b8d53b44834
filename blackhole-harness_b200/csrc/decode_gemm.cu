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
// 32 RQ weight rows m, RQ = 1, 2 or 4: the smallest tiles while there are few
// of them, so that small batches spread over the SMs), RQ x (8 / RQ) consumer
// warps + 1 producer warp; two
// CTAs per SM (each with half the shared memory) once there are more tiles
// than SMs, since the consumers are bound by instruction latency more than by
// issue, and one CTA with the deeper ring while there are few tiles:
//   producer   per tile the expert's code tables (built at layer creation: the
//              level table times each fp8 scale code and the expert scale,
//              rounded to the operand type) and the tile's fp8 scale codes into
//              one of two buffers; per 128-input step the tile's codes (one
//              RQ x 2 KB bulk copy per projection from the layer's tiled nibble
//              copy) and the block's 8 activation rows (one 3-D TMA box: two
//              halves of 64 inputs, 128-B swizzle) into a ring of stages; few
//              copies per stage, since issuing a copy costs the one producer
//              thread about as much as a 2 KB copy takes to stream
//   consumers  warp (rq, kg) owns rows 32 rq .. 32 rq + 31 of the tile (two
//              16-row MMA tiles) and the steps k with k % (8 / RQ) == kg; per step
//              a lane decodes 4 rows x 32 inputs per projection with prmt
//              lookups into operand pairs and issues the MMAs; at the end of a
//              tile the step groups 1.. hand their sums to group 0 through
//              shared memory, which adds them in group order (a fixed order on
//              every run) and applies SwiGLU (gate/up) or the top-k weight
//              (down)
// 32 rows per warp halve the per-step work that is not decoding (the ring
// wait, the activation fragment loads, the scale-code and table loads, the
// release) per decoded weight against 16 rows per warp.
//
// Fragments.  Lane (g = lane/4, q = lane%4) owns rows g, g+8 (MMA tile 0) and
// g+16, g+24 (MMA tile 1) of its warp's 32 and the 32-input block q of each
// step.  The reduction index inside each 16-wide MMA is permuted the same way
// in A and B: MMA chunk c of a step takes, from lane (g, q), inputs q*32 + 4c +
// {0,1} (k = 2q, 2q+1) and q*32 + 4c + {2,3} (k = 2q+8, 2q+9), so a lane's A
// registers are its own decoded pairs and its B registers its own 32
// consecutive inputs of token g.
//
// Shared-memory banks.  In the tiled copy, block q of a 32-row slice holds row
// r at position r ^ 2q, so the 8 lanes of a quarter warp (rows g, g+1, blocks
// 0..3) read 8 distinct 16-byte bank groups of the contiguous 2 KB slice; table
// entries are shared by the 4 lanes of a row (one scale code per row and 128
// inputs), at most 2 rows per quarter warp.
// Every wait is bounded: a lost arrival sets the device error word and the
// kernel returns after its in-flight copies land.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

#include "decode.cuh"
#include "internal.cuh"

namespace hexmoe {

constexpr uint32_t kDecSlice = 2048;                         // 32 rows x 128 inputs of codes (one slice of a step)
constexpr uint32_t kDecXBytes = 2 * 8 * 128;                 // 8 rows x 128 inputs (two swizzled boxes)
constexpr uint32_t kDecCtrl = 1024;                          // barriers
constexpr int kDecRows = 32;                                 // weight rows per consumer warp
constexpr int kDecConsumers = 8;                             // RQ row slices x 8 / RQ step groups
constexpr int kDecThreads = (kDecConsumers + 1) * 32;

// A tile as the producer hands it to the consumers with the tile's tables
// (one per table buffer): the consumers read no tile list, slot id or top-k
// weight from global memory themselves.
struct DecRec {
  int32_t b, m, bits, end;     // end: no more tiles for this CTA
  int32_t slot[kDecBlock];     // the block's slot ids (>= num_slots: padding)
  float w[kDecBlock];          // down: their top-k weights
};

struct DecCtrl {
  uint64_t c_full[kDecStages], c_empty[kDecStages];   // step ring (released by the RQ warps of a step group)
  uint64_t t_full[2], t_empty[2];                     // table buffers (and their tile records)
  uint64_t r_full, r_empty;                           // partial sums handed from step groups 1.. to group 0
  int32_t abort;
  DecRec rec[2];
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

// A ring position (stage, phase) moved by `n` stages, -ds < n (a step group
// moves back when the next tile's first step of the group precedes where its
// last step left it).
__device__ __forceinline__ void ring_move(int& pos, uint32_t& ph, int n, int ds) {
  pos += n;
  while (pos >= ds) { pos -= ds; ph ^= 1u; }
  while (pos < 0) { pos += ds; ph ^= 1u; }
}

// Bounded wait taken by lane 0 and its result given to the whole warp (the
// producer warp's lanes then take the same path).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* dev_err, int lane) {
  bool ok = true;
  if (lane == 0) ok = mbar_wait(bar, parity, abort, dev_err);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// Producer (one warp; lane 0 issues the copies): per tile its record, tables
// and scale codes, per step codes + activation box; an end record last.
template <bool GLU, int RQ>
__device__ void dec_producer(const DecParams& p, uint8_t* smem, DecCtrl* c, int num_tiles, int lane) {
  constexpr int NPROJ = GLU ? 2 : 1;
  constexpr uint32_t kProj = RQ * kDecSlice;           // one projection's codes of a step
  volatile int* abort_flag = &c->abort;
  int cs = 0;
  uint32_t cph = 0;
  int issued = 0, tissued = 0;
  bool aborted = false;
  for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x) {
    const DecTile ti = dec_tile(p, t);
    if (!ti.ok) {
      if (lane == 0) atomicOr(p.dev_err, kDevErrNoTier);
      continue;
    }
    const uint32_t tabn = ti.bits == 3 ? 256u : 512u;
    const int tb = tissued & 1;
    if (!warp_wait(&c->t_empty[tb], ((tissued >> 1) & 1) ^ 1, abort_flag, p.dev_err, lane)) { aborted = true; break; }
    DecRec* rec = &c->rec[tb];
    if (lane < kDecBlock) {
      const int sl = __ldg(p.sorted_ids + static_cast<int64_t>(ti.b) * kDecBlock + lane);
      rec->slot[lane] = sl;
      rec->w[lane] = (!GLU && sl < p.num_slots) ? __ldg(p.topk_w + sl) : 0.f;
    }
    if (lane == 0) {
      rec->b = ti.b; rec->m = ti.m; rec->bits = ti.bits; rec->end = 0;
    }
    __syncwarp();
    const uint32_t scb = static_cast<uint32_t>(RQ * kDecRows) * static_cast<uint32_t>(p.k_pad >> p.block_log2);  // tile's scale codes, one projection
    if (lane == 0) {
      mbar_arrive_expect_tx(&c->t_full[tb], NPROJ * (tabn * 16u + scb));
      for (int j = 0; j < NPROJ; ++j) {
        bulk_load(smem + p.off_tab + (tb * NPROJ + j) * p.tab_bytes,
                  p.tab[ti.tier][j] + static_cast<size_t>(ti.local) * tabn, tabn * 16u, &c->t_full[tb]);
        bulk_load(smem + p.off_sc + (tb * NPROJ + j) * p.sc_bytes,
                  p.bs[ti.tier][j] + (static_cast<size_t>(ti.local) * p.rows_pad + static_cast<size_t>(ti.m) * (RQ * kDecRows)) *
                                         static_cast<size_t>(p.k_pad >> p.block_log2),
                  scb, &c->t_full[tb]);
      }
    }
    ++tissued;
    // the tile's rows in the tiled copy: 128-row tile r0 / 128, slices from (r0 % 128) / 32
    const int r0 = ti.m * RQ * kDecRows;
    const size_t tile_base = (static_cast<size_t>(ti.local) * p.m128 + (r0 >> 7)) * p.ksteps * kStepBytes +
                             static_cast<size_t>((r0 & 127) >> 5) * kDecSlice;
    for (int s = 0; s < p.ksteps; ++s) {
      // a spinning wait: the ring refills the moment a stage frees (a sleeping
      // poll here lets the ring drain and the consumers starve)
      if (!warp_wait(&c->c_empty[cs], cph ^ 1, abort_flag, p.dev_err, lane)) { aborted = true; break; }
      if (lane == 0) {
        uint8_t* st = smem + kDecCtrl + cs * p.stage_bytes;
        mbar_arrive_expect_tx(&c->c_full[cs], NPROJ * kProj + kDecXBytes);
        tma_load_3d(st, &p.tm_b, &c->c_full[cs], 0, ti.b * kDecBlock, 2 * s);
        for (int j = 0; j < NPROJ; ++j)
          bulk_load(st + kDecXBytes + j * kProj, p.idx_t[ti.tier][j] + tile_base + static_cast<size_t>(s) * kStepBytes,
                    kProj, &c->c_full[cs]);
      }
      ++issued;
      if (++cs == p.ds) { cs = 0; cph ^= 1; }
    }
  }
  if (!aborted) {
    // the end record: the consumers stop at it
    const int tb = tissued & 1;
    if (warp_wait(&c->t_empty[tb], ((tissued >> 1) & 1) ^ 1, abort_flag, p.dev_err, lane)) {
      if (lane == 0) {
        c->rec[tb].end = 1;
        mbar_arrive(&c->t_full[tb]);
      }
      return;
    }
    aborted = true;
  }
  if (aborted && lane == 0) {
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

// Consumer warp `cw` = (rq, kg): rows 32*rq .. 32*rq+31 of each tile, the
// steps k with k % KG == kg.
template <bool GLU, bool BF16, int RQ>
__device__ void dec_consumer(const DecParams& p, uint8_t* smem, DecCtrl* c, int cw, int lane) {
  constexpr int NPROJ = GLU ? 2 : 1;
  constexpr int KG = kDecConsumers / RQ;
  constexpr uint32_t kProj = RQ * kDecSlice;
  constexpr int NACC = NPROJ * 2 * 4;                       // accumulators per lane
  volatile int* abort_flag = &c->abort;
  const int g = lane >> 2, q = lane & 3;
  const int rq = cw % RQ, kg = cw / RQ;
  float* red = reinterpret_cast<float*>(smem + p.off_red);   // [KG-1][RQ][NACC][32]
  const uint32_t spr = static_cast<uint32_t>(p.k_pad >> p.block_log2);
  // this lane's 16-byte chunks of token g's 32 inputs of block q (two 64-input
  // boxes, 128-B swizzle by row)
  uint32_t xo[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t cc = static_cast<uint32_t>((q & 1) * 4 + i);
    xo[i] = (q >> 1) * 1024u + g * 128u + ((cc ^ static_cast<uint32_t>(g)) << 4);
  }
  const uint32_t row_w = static_cast<uint32_t>(rq * kDecRows + g);   // the lane's first row in the tile
  // where rows row_w + 8i sit in block q of the warp's slice (the tiled copy's r ^ 2q)
  const uint32_t code_off = rq * kDecSlice + q * 512u + static_cast<uint32_t>(g ^ (2 * q)) * 16u;
  int cpos = 0;
  uint32_t cph = 0;
  ring_move(cpos, cph, kg, p.ds);                           // the group's first stage
  int tused = 0, rused = 0;
  uint16_t* out16 = reinterpret_cast<uint16_t*>(p.out);
  for (;;) {
    const int tb = tused & 1;
    if (!mbar_wait(&c->t_full[tb], (tused >> 1) & 1, abort_flag, p.dev_err)) return;
    const DecRec& rec = c->rec[tb];
    if (rec.end) return;
    const int tile_b = rec.b, tile_m = rec.m, tile_bits = rec.bits;
    // this lane's tokens 2q, 2q+1 of the block (read before the record is released)
    const int slot0 = rec.slot[2 * q], slot1 = rec.slot[2 * q + 1];
    const float w0 = rec.w[2 * q], w1 = rec.w[2 * q + 1];
    const uint8_t* tabs = smem + p.off_tab + tb * NPROJ * p.tab_bytes;
    const uint8_t* scb = smem + p.off_sc + tb * NPROJ * p.sc_bytes + row_w * spr;
    float acc[NPROJ][2][4];
#pragma unroll
    for (int j = 0; j < NPROJ; ++j)
#pragma unroll
      for (int s = 0; s < 2; ++s)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][s][i] = 0.f;
    bool aborted = false;
    int k = kg;
    auto run = [&](auto bits_c) {
      constexpr int BITS = decltype(bits_c)::value;
#pragma unroll 1
      for (; k < p.ksteps; k += KG) {
        const uint32_t sci = static_cast<uint32_t>(k * 128 + q * 32) >> p.block_log2;
        if (!mbar_wait(&c->c_full[cpos], cph, abort_flag, p.dev_err)) { aborted = true; return; }
        const uint8_t* st = smem + kDecCtrl + cpos * p.stage_bytes;
        uint32_t xr[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 v = *reinterpret_cast<const uint4*>(st + xo[i]);
          xr[4 * i] = v.x; xr[4 * i + 1] = v.y; xr[4 * i + 2] = v.z; xr[4 * i + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < NPROJ; ++j) {
          const uint8_t* cb = st + kDecXBytes + j * kProj + code_off;
          const uint8_t* sj = scb + j * p.sc_bytes + sci;
          const uint4* tab = reinterpret_cast<const uint4*>(tabs + j * p.tab_bytes);
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            // rows 16 s + g and 16 s + g + 8 of the warp's 32
            const uint4 w0 = *reinterpret_cast<const uint4*>(cb + (16 * s) * 16);
            const uint4 w1 = *reinterpret_cast<const uint4*>(cb + (16 * s + 8) * 16);
            const uint32_t c0 = sj[(16 * s) * spr], c1 = sj[(16 * s + 8) * spr];
            const uint4 t0 = tab[c0], t1 = tab[c1];
            uint4 h0 = t0, h1 = t1;
            if constexpr (BITS == 4) {
              h0 = tab[256 + c0];
              h1 = tab[256 + c1];
            }
            const uint32_t wa[4] = {w0.x, w0.y, w0.z, w0.w}, wb[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int jw = 0; jw < 4; ++jw) {
              const uint4 oa = dec8<BITS>(wa[jw], t0, h0);   // row 16s + g: inputs 8jw .. 8jw+7 of block q
              const uint4 ob = dec8<BITS>(wb[jw], t1, h1);   // row 16s + g + 8
              mma16816<BF16>(acc[j][s], oa.x, ob.x, oa.y, ob.y, xr[4 * jw], xr[4 * jw + 1]);
              mma16816<BF16>(acc[j][s], oa.z, ob.z, oa.w, ob.w, xr[4 * jw + 2], xr[4 * jw + 3]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&c->c_empty[cpos]);
        ring_move(cpos, cph, KG, p.ds);
      }
    };
    if (tile_bits == 3) run(std::integral_constant<int, 3>{});
    else run(std::integral_constant<int, 4>{});
    if (aborted) return;
    // the group's first step of the next tile: ksteps + kg stages past this tile's start
    ring_move(cpos, cph, p.ksteps + kg - k, p.ds);
    __syncwarp();
    if (lane == 0) mbar_arrive(&c->t_empty[tb]);
    ++tused;
    if constexpr (KG > 1) {
      const int ru = rused++;
      if (kg > 0) {
        // hand the partial sums to group 0 (the buffer is free once group 0 has
        // read what was written into it for the previous tile)
        if (!mbar_wait(&c->r_empty, (ru & 1) ^ 1, abort_flag, p.dev_err)) return;
        float* dst = red + static_cast<size_t>((kg - 1) * RQ + rq) * NACC * 32;
#pragma unroll
        for (int j = 0; j < NPROJ; ++j)
#pragma unroll
          for (int s = 0; s < 2; ++s)
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[((j * 2 + s) * 4 + i) * 32 + lane] = acc[j][s][i];
        __syncwarp();
        if (lane == 0) mbar_arrive(&c->r_full);
        continue;
      }
      if (!mbar_wait(&c->r_full, ru & 1, abort_flag, p.dev_err)) return;
#pragma unroll
      for (int gg = 1; gg < KG; ++gg) {
        const float* src = red + static_cast<size_t>((gg - 1) * RQ + rq) * NACC * 32;
#pragma unroll
        for (int j = 0; j < NPROJ; ++j)
#pragma unroll
          for (int s = 0; s < 2; ++s)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[j][s][i] += src[((j * 2 + s) * 4 + i) * 32 + lane];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&c->r_empty);
    }
    // epilogue: acc[.][s][0..1] = (row 16s + g, tokens 2q, 2q+1), [2..3] = (row 16s + g + 8, same tokens)
    uint16_t* drow[2] = {nullptr, nullptr};   // down: the output rows of tokens 2q, 2q+1
    if constexpr (!GLU) {
      const int sl[2] = {slot0, slot1};
#pragma unroll
      for (int u = 0; u < 2; ++u)
        if (sl[u] < p.num_slots)
          drow[u] = slot_out_row(p.slot_out, out16, p.ld_out, p.slot_out.row ? __ldg(p.slot_out.row + sl[u]) : sl[u]);
    }
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int n = 2 * q + (i & 1);
        const int row = tile_m * (RQ * kDecRows) + static_cast<int>(row_w) + 16 * s + (i >> 1) * 8;
        const int sl = (i & 1) ? slot1 : slot0;
        if (sl >= p.num_slots || row >= p.rows_store) continue;
        if constexpr (GLU) {
          const float gv = acc[0][s][i];
          const float r = __fdividef(gv, 1.0f + __expf(-gv)) * acc[1][s][i];   // silu(gate) * up, as the tcgen05 epilogue
          out16[(static_cast<int64_t>(tile_b) * kDecBlock + n) * p.ld_out + row] =
              static_cast<uint16_t>(pack2<BF16>(r, 0.f) & 0xFFFFu);
        } else {
          const float r = acc[0][s][i] * ((i & 1) ? w1 : w0);
          drow[i & 1][row] = static_cast<uint16_t>(pack2<BF16>(r, 0.f) & 0xFFFFu);
        }
      }
  }
}

template <bool GLU, bool BF16, int RQ>
__global__ void __launch_bounds__(kDecThreads, 2) hex_decode_kernel(const __grid_constant__ DecParams p) {
  constexpr int KG = kDecConsumers / RQ;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  DecCtrl* c = reinterpret_cast<DecCtrl*>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kDecStages; ++i) { mbar_init(&c->c_full[i], 1); mbar_init(&c->c_empty[i], RQ); }
    for (int i = 0; i < 2; ++i) { mbar_init(&c->t_full[i], 1); mbar_init(&c->t_empty[i], kDecConsumers); }
    mbar_init(&c->r_full, RQ * (KG - 1));
    mbar_init(&c->r_empty, RQ);
    c->abort = 0;
    fence_mbar_init();
  }
  if (warp == kDecConsumers && lane == 0) prefetch_tmap(&p.tm_b);
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();   // the plan and the B rows come from the previous kernels
  const int num_tiles = (__ldg(p.npp) / kDecBlock) * p.m_tiles;
  if (warp == kDecConsumers) {
    dec_producer<GLU, RQ>(p, smem, c, num_tiles, lane);
  } else {
    dec_consumer<GLU, BF16, RQ>(p, smem, c, warp, lane);
  }
  if (!GLU && p.slot_out.fence) __threadfence_system();   // peer stores visible before the return flags
}

template <bool GLU, bool BF16, int RQ>
static cudaError_t launch_dec(const DecParams& p, int grid, cudaStream_t st, bool pdl) {
  auto kern = hex_decode_kernel<GLU, BF16, RQ>;
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
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

// Shared-memory carve-up for one projection pair (2) or one projection (1),
// for `per_sm` CTAs on an SM (1 or 2) and tiles of 32 rq rows (1, 2 or 4).
// p.block and the tiers' bits must be set.
bool plan_decode(DecParams& p, int nproj, int per_sm, int rq) {
  int max_bits = 3;
  for (int t = 0; t < p.num_tiers; ++t) max_bits = std::max(max_bits, static_cast<int>(p.bits[t]));
  const int kg = kDecConsumers / rq;
  p.rq = rq;
  p.block_log2 = p.block == 128 ? 7 : 5;
  p.stage_bytes = (kDecXBytes + nproj * rq * kDecSlice + 1023u) / 1024u * 1024u;
  p.tab_bytes = (max_bits == 3 ? 256u : 512u) * 16u;
  p.sc_bytes = (static_cast<uint32_t>(rq * kDecRows) * static_cast<uint32_t>(p.k_pad / p.block) + 127u) / 128u * 128u;
  const uint32_t red = static_cast<uint32_t>(kg - 1) * rq * nproj * 8u * 32u * 4u;
  const uint32_t fixed = 2u * nproj * (p.tab_bytes + p.sc_bytes) + red;
  const uint32_t budget = (per_sm == 2 ? 113u : 227u) * 1024u - 1024u - kDecCtrl;   // per CTA, minus alignment slack
  if (fixed + static_cast<uint32_t>(std::min(kg, 4) + 1) * p.stage_bytes > budget) return false;
  p.ds = static_cast<int32_t>(std::min<uint32_t>(kDecStages, (budget - fixed) / p.stage_bytes));
  p.off_tab = kDecCtrl + p.ds * p.stage_bytes;
  p.off_sc = p.off_tab + 2u * nproj * p.tab_bytes;
  p.off_red = p.off_sc + 2u * nproj * p.sc_bytes;
  p.smem_bytes = p.off_red + red + 1024u;
  return true;
}

template <int RQ>
static cudaError_t launch_dec_rq(const DecParams& p, bool glu, bool bf16, int grid, cudaStream_t st, bool pdl) {
  if (glu) return bf16 ? launch_dec<true, true, RQ>(p, grid, st, pdl) : launch_dec<true, false, RQ>(p, grid, st, pdl);
  return bf16 ? launch_dec<false, true, RQ>(p, grid, st, pdl) : launch_dec<false, false, RQ>(p, grid, st, pdl);
}

cudaError_t launch_decode_gemm(const DecParams& p, bool glu, bool bf16, int grid, cudaStream_t st, bool pdl) {
  if (p.rq == 1) return launch_dec_rq<1>(p, glu, bf16, grid, st, pdl);
  if (p.rq == 2) return launch_dec_rq<2>(p, glu, bf16, grid, st, pdl);
  if (p.rq == 4) return launch_dec_rq<4>(p, glu, bf16, grid, st, pdl);
  return cudaErrorInvalidValue;
}

}  // namespace hexmoe
