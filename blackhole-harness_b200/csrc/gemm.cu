// gemm.cu — persistent, warp-specialised HEX grouped GEMM for sm_100a.
//
// One launch covers every tier of a layer for one projection pair:
//   gate/up (GLU):  act[row, o] = silu(x_t . Wg[e, o]) * (x_t . Wu[e, o])
//   down:           y[slot, o]  = (act_row . Wd[e, o]) * topk_weight[slot]
// over the tiles (align block b, 128-row weight tile m) of the align() plan.
// The weight tile is the UMMA M side (128 rows) and the block's tokens the N
// side (16..128 columns), so a decode step with a handful of tokens per expert
// still streams every weight once at full width.
//
// Warp roles (32 x (8 + 8 x decoder groups) threads):
//   warp 0      producer: per tile a record (block, weight tile, tier, valid
//               rows, level tables, expert scales, the block's slot ids and
//               top-k weights) into a small shared ring and the tile's fp8
//               scale codes (1-D bulk copy); the index words of the weight
//               tile from the layer's tiled copy of the index stream, where a
//               128-row x 128-input step is 8 KB of contiguous memory: one 1-D
//               bulk copy per projection and stage (k_idx/128 steps) into a
//               ring the decoders release
//   warp 6+dec  activation producer: the block's rows of the plan-ordered
//               activations, two 64-column boxes per 128 inputs, into a ring
//               the MMA releases (its own warp, so a full activation ring never
//               delays the next index stage)
//   warp 1,     TMEM allocation (warp 1); one thread of each issues tcgen05.mma
//   last warp   (A operand from TMEM, B from 128-B swizzled smem) and
//               tcgen05.commit: gate and up one each; down one, or both (each
//               over alternate 128-input steps into its own accumulator,
//               summed by the epilogue) where an M=128 x N<=64 MMA costs its
//               issuing thread more than the tensor pipe takes to run it
//   warps 2-5   epilogue: tcgen05.ld of the accumulators, SwiGLU (gate/up) or
//               the top-k weight (down), 16-bit stores; ahead of the decoders, the
//               code tables: the level table scaled by every one of the 256
//               fp8 scale codes and rounded to the operand type (shared
//               memory, two buffers)
//   warps 6..   decoders, groups of 8 taking 128-input sub-blocks in turn: per
//               32-input block one 16-byte load of its 32 codes (a nibble
//               each; a warp's loads cover 512 contiguous bytes, free of bank
//               conflicts: the tiled copy permutes rows only inside groups of
//               8), one code-table load and prmt lookups of the codes
//               into one of two 16-register buffers, written to
//               TMEM with tcgen05.st while the other buffer's store drains; a
//               half-stage goes to the MMA once both its stores are done
// Every wait is bounded (ptx.cuh): a lost arrival ends the kernel with the
// device error word set instead of hanging.
#include <atomic>
#include <mutex>
#include <type_traits>

#include "decode.cuh"
#include "internal.cuh"

namespace hexmoe {

constexpr int kRecs = 4;   // tile records in flight

struct Ctrl {
  uint64_t x_full[kMaxDI], x_empty[kMaxDI];   // index-word ring
  uint64_t b_full[kMaxDB], b_empty[kMaxDB];   // activation ring
  uint64_t a_full[kMaxDA], a_empty[kMaxDA];   // TMEM operand ring
  uint64_t s_full[2], s_empty[2];             // tile scale buffers
  uint64_t t_full[2], t_empty[2];             // accumulator buffers
  uint64_t i_full[kRecs], i_empty[kRecs];     // tile records
  uint64_t tab_ready[2], tab_empty[2];        // code tables built / released (per buffer)
  uint64_t drain[kMmaWarps];   // one per MMA issuer
  uint32_t tmem_base;
  int32_t abort;
};
static_assert(sizeof(Ctrl) <= 2048, "control block");
constexpr uint32_t kOffLut = 2048;    // fp8 decode table (256 floats)
constexpr uint32_t kOffRec = 3072;    // tile records (kRecs x 1280 B, up to 8192)

struct TileRec {
  int32_t b, m, tier, local, bits, cnt, ok, pad;
  float es[2];
  float lev[2][16];
  int32_t slot[128];    // down: the block's slot ids (valid rows)
  float w[128];         // down: their top-k weights
  uint8_t pad_to_1280[1280 - 40 - 128 - 1024];
};
static_assert(sizeof(TileRec) == 1280 && kOffRec + kRecs * 1280 <= 8192, "tile records");
constexpr uint32_t kOffStage = 8192;  // down epilogue: per warp 8 tokens x 32 rows of 16-bit outputs (4 x 512 B)

struct TileInfo {
  int32_t b, m, tier, local, bits;
  bool ok;
};

__device__ __forceinline__ TileInfo tile_info(const GemmParams& p, int t) {
  TileInfo ti;
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

// Valid (non-padding) rows of align block b: a prefix of the block.
__device__ __forceinline__ int block_rows(const GemmParams& p, int b, int lane) {
  int cnt = 0;
  for (int r0 = 0; r0 < p.bm; r0 += 32) {
    const int r = r0 + lane;
    const bool v = r < p.bm && __ldg(p.sorted_ids + static_cast<size_t>(b) * p.bm + r) < p.num_slots;
    cnt += __popc(__ballot_sync(0xffffffffu, v));
  }
  return cnt;
}

// Bounded wait that ignores the abort flag (used to drain in-flight copies).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > 200000000ull) return;
  }
}

// Decode the 32-input block BLK (0..3) of one 128-input step of a row into 16
// packed operand registers (K order).  w: the row's 16 tiled words of the step
// (4 per block); tab: this projection's code tables (plane 0, then plane 1 at
// +256); code: the block's fp8 scale code.
template <int BLK>
__device__ __forceinline__ void decode_block(const uint32_t (&w)[16], int bits, const uint4* tab, uint32_t code,
                                             uint32_t* r) {
  uint4 ch[4];
  if (bits == 3) {
    const Table8 tb = table8_from(tab[code]);
    dec32_n3(w[4 * BLK], w[4 * BLK + 1], w[4 * BLK + 2], w[4 * BLK + 3], tb, ch);
  } else {
    const Table16 tb = table16_from(tab[code], tab[256 + code]);
    dec32_b4(w[4 * BLK], w[4 * BLK + 1], w[4 * BLK + 2], w[4 * BLK + 3], tb, ch);
  }
#pragma unroll
  for (int cq = 0; cq < 4; ++cq) {
    r[cq * 4 + 0] = ch[cq].x;
    r[cq * 4 + 1] = ch[cq].y;
    r[cq * 4 + 2] = ch[cq].z;
    r[cq * 4 + 3] = ch[cq].w;
  }
}

// KS: the split issue of down (p.ksplit == 2), a separate instantiation so the
// other kernels carry none of its code.
template <bool GLU, bool BF16, bool KS>
__global__ void __launch_bounds__(kGemmThreads, 1) hex_gemm_kernel(const __grid_constant__ GemmParams p) {
  static_assert(!(GLU && KS), "gate/up keeps one issuer per projection");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Ctrl* c = reinterpret_cast<Ctrl*>(smem);
  float* lut = reinterpret_cast<float*>(smem + kOffLut);
  TileRec* recs = reinterpret_cast<TileRec*>(smem + kOffRec);   // stride 1280 B
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NPROJ = GLU ? 2 : 1;
  volatile int* abort_flag = &c->abort;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kMaxDI; ++i) { mbar_init(&c->x_full[i], 1); mbar_init(&c->x_empty[i], kDecWarps); }
    const int stage_users = p.n_iss / p.ksplit;   // issuers reading one operand / activation stage
    for (int i = 0; i < kMaxDB; ++i) { mbar_init(&c->b_full[i], 1); mbar_init(&c->b_empty[i], stage_users); }
    for (int i = 0; i < kMaxDA; ++i) { mbar_init(&c->a_full[i], 8); mbar_init(&c->a_empty[i], stage_users); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&c->s_full[i], 1); mbar_init(&c->s_empty[i], kDecWarps);
      mbar_init(&c->t_full[i], p.n_iss); mbar_init(&c->t_empty[i], 4);
      mbar_init(&c->tab_ready[i], 4); mbar_init(&c->tab_empty[i], kDecWarps);
    }
    for (int i = 0; i < kRecs; ++i) { mbar_init(&c->i_full[i], 1); mbar_init(&c->i_empty[i], 5 + kMmaWarps + kDecWarps); }
    for (int i = 0; i < kMmaWarps; ++i) mbar_init(&c->drain[i], 1);
    c->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) prefetch_tmap(&p.tm_b);
  if (warp == 1) {
    tmem_alloc(&c->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp >= 6 && warp < 14) lut[threadIdx.x - 192] = fp8_hex_value(static_cast<uint32_t>(threadIdx.x - 192));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = c->tmem_base;

  pdl_launch_dependents();
  pdl_wait();  // the plan (and, for down, act) come from the previous kernels

  const int nbv = __ldg(p.npp) / p.bm;
  const int num_tiles = nbv * p.m_tiles;
  const int ksteps = p.k_pad / kKStep;        // activation stages per tile
  const int spi = p.k_idx / kKStep;           // 128-input sub-blocks per index stage
  const uint32_t spr = static_cast<uint32_t>(p.k_pad / p.block);   // scale bytes per weight row
  const uint32_t scale_tile = 128u * spr;                           // per projection
  uint8_t* xring = smem + p.off_idx;
  uint8_t* bring = smem + p.off_b;
  uint8_t* scale_buf = smem + p.off_scale;
  uint4* tabs = reinterpret_cast<uint4*>(smem + p.off_tab);        // [2][NPROJ][2 planes][256]

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol_stream = l2_policy_evict_first();
    uint32_t xs = 0, xph = 0;
    int x_issued = 0, s_issued = 0;
    bool aborted = false;
    int cur = 0;
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x, ++cur) {
      const TileInfo ti = tile_info(p, t);
      const int cnt = block_rows(p, ti.b, lane);
      const int ri = cur % kRecs;
      if (!mbar_wait_idle(&c->i_empty[ri], ((cur / kRecs) & 1) ^ 1, abort_flag, p.dev_err)) { aborted = true; break; }
      {
        TileRec* rec = recs + ri;
        const int L = 1 << ti.bits;
        if (lane < 16) {
          for (int q = 0; q < NPROJ; ++q)
            rec->lev[q][lane] = (ti.ok && lane < L) ? __ldg(p.lev[ti.tier][q] + ti.local * L + lane) : 0.0f;
        }
        if (lane < NPROJ) rec->es[lane] = ti.ok ? __ldg(p.es[ti.tier][lane] + ti.local) : 0.0f;
        if (!GLU) {
          for (int r = lane; r < cnt; r += 32) {
            const int slot = __ldg(p.sorted_ids + static_cast<size_t>(ti.b) * p.bm + r);
            rec->slot[r] = p.slot_out.row ? __ldg(p.slot_out.row + slot) : slot;   // where its row goes
            rec->w[r] = __ldg(p.topk_w + slot);
          }
        }
        if (lane == 0) {
          rec->b = ti.b; rec->m = ti.m; rec->tier = ti.tier; rec->local = ti.local;
          rec->bits = ti.bits; rec->cnt = cnt; rec->ok = ti.ok;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&c->i_full[ri]);
      }
      if (!ti.ok) continue;
      const uint32_t proj_bytes = static_cast<uint32_t>(spi) * kStepBytes;   // one projection's part of a stage
      const size_t tile_base = (static_cast<size_t>(ti.local) * p.m_tiles + ti.m) * ksteps * kStepBytes;
      const int sb = s_issued & 1;
      if (!mbar_wait_idle(&c->s_empty[sb], ((s_issued >> 1) & 1) ^ 1, abort_flag, p.dev_err)) { aborted = true; break; }
      if (lane == 0) {
        mbar_arrive_expect_tx(&c->s_full[sb], scale_tile * NPROJ);
        for (int j = 0; j < NPROJ; ++j) {
          const uint8_t* src =
              p.bs[ti.tier][j] + (static_cast<size_t>(ti.local) * p.rows_pad + static_cast<size_t>(ti.m) * 128) * spr;
          bulk_load(scale_buf + (sb * NPROJ + j) * p.sz_scale, src, scale_tile, &c->s_full[sb]);
        }
      }
      ++s_issued;
      for (int kb = 0; kb < ksteps; kb += spi) {
        {
          if (!mbar_wait_idle(&c->x_empty[xs], xph ^ 1, abort_flag, p.dev_err)) { aborted = true; break; }
          if (lane == 0) {
            uint8_t* dst = xring + xs * p.sz_idx;
            mbar_arrive_expect_tx(&c->x_full[xs], NPROJ * proj_bytes);
            for (int j = 0; j < NPROJ; ++j)
              bulk_load_hint(dst + j * proj_bytes, p.idx_t[ti.tier][j] + tile_base + static_cast<size_t>(kb) * kStepBytes,
                             proj_bytes, &c->x_full[xs], pol_stream);
          }
          ++x_issued;
          if (++xs == static_cast<uint32_t>(p.di)) { xs = 0; xph ^= 1; }
        }
      }
    }
    if (aborted && lane == 0) {
      // let every copy already issued land before the CTA (and its smem) goes away
      for (int i = 1; i <= 2 && i <= s_issued; ++i) {
        const int q = s_issued - i;
        drain_wait(&c->s_full[q & 1], (q >> 1) & 1);
      }
      for (int i = 1; i <= p.di && i <= x_issued; ++i) {
        const int q = x_issued - i;
        drain_wait(&c->x_full[q % p.di], (q / p.di) & 1);
      }
    }
  } else if (warp == kBWarp) {
    // ------------------------------------------------------------ activation producer
    uint32_t bs = 0, bph = 0;
    int b_issued = 0;
    bool aborted = false;
    int cur = 0;
    const uint32_t b_bytes = static_cast<uint32_t>(p.bm) * 256u;
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x, ++cur) {
      const int ri = cur % kRecs;
      if (!mbar_wait_idle(&c->i_full[ri], (cur / kRecs) & 1, abort_flag, p.dev_err)) { aborted = true; break; }
      const int ok = recs[ri].ok, b = recs[ri].b;
      __syncwarp();
      if (lane == 0) mbar_arrive(&c->i_empty[ri]);
      if (!ok) continue;
      for (int kb = 0; kb < ksteps; ++kb) {
        if (!mbar_wait_idle(&c->b_empty[bs], bph ^ 1, abort_flag, p.dev_err)) { aborted = true; break; }
        if (lane == 0) {
          uint8_t* bdst = bring + bs * p.sz_b;
          mbar_arrive_expect_tx(&c->b_full[bs], b_bytes);
          tma_load_2d(bdst, &p.tm_b, &c->b_full[bs], kb * kKStep, b * p.bm);
          tma_load_2d(bdst + p.bm * 128, &p.tm_b, &c->b_full[bs], kb * kKStep + 64, b * p.bm);
        }
        ++b_issued;
        if (++bs == static_cast<uint32_t>(p.db)) { bs = 0; bph ^= 1; }
      }
    }
    if (aborted && lane == 0) {
      for (int i = 1; i <= p.db && i <= b_issued; ++i) {
        const int q = b_issued - i;
        drain_wait(&c->b_full[q % p.db], (q / p.db) & 1);
      }
    }
  } else if (warp == 1 || warp > kBWarp) {
    // ------------------------------------------------------------ MMA issuers
    // Issuer mi owns projection mi % nproj and, with ksplit 2, the 128-input
    // steps of parity mi / nproj, into accumulator mi; issuers beyond n_iss only
    // follow the tile records.
    const int mi = warp == 1 ? 0 : warp - kBWarp;
    const bool active = mi < p.n_iss;
    const int proj = mi % NPROJ, part = mi / NPROJ;
    uint32_t bs = 0, bph = 0, as = 0, aph = 0;
    bool aborted = false;
    int cur = 0, acc_it = 0;
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x, ++cur) {
      const int ri = cur % kRecs;
      if (!mbar_wait(&c->i_full[ri], (cur / kRecs) & 1, abort_flag, p.dev_err)) { aborted = true; break; }
      const int ok = recs[ri].ok, cnt = recs[ri].cnt;
      __syncwarp();
      if (lane == 0) mbar_arrive(&c->i_empty[ri]);
      if (!ok || !active) continue;
      const uint32_t n_mma = static_cast<uint32_t>(max(16, (cnt + 15) & ~15));
      const uint32_t idesc = umma_idesc(BF16, 128, n_mma);
      const int ab = acc_it % p.nbuf;
      if (!mbar_wait(&c->t_empty[ab], ((acc_it / p.nbuf) & 1) ^ 1, abort_flag, p.dev_err)) { aborted = true; break; }
      ++acc_it;
      tc_fence_after();
      const uint32_t d = tmem + ab * p.acc_stride + mi * p.bm;
      const uint32_t h_step = static_cast<uint32_t>(p.bm * 128) >> 4;   // descriptor units per 64-input half
      for (int ks = 0, kpar = 0; ks < ksteps && !aborted; ++ks, kpar ^= 1) {
        if (KS && kpar != part) {
          // the other issuer's step: only the ring positions move
          if (++as == static_cast<uint32_t>(p.da)) { as = 0; aph ^= 1; }
          if (++bs == static_cast<uint32_t>(p.db)) { bs = 0; bph ^= 1; }
          continue;
        }
        if (!mbar_wait(&c->b_full[bs], bph, abort_flag, p.dev_err)) { aborted = true; break; }
        const uint64_t bdesc = sw128_desc(smem_u32(bring + bs * p.sz_b));
        if (!mbar_wait(&c->a_full[as], aph, abort_flag, p.dev_err)) { aborted = true; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a0 = tmem + p.a_base + as * p.a_stride + proj * 64;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint64_t bh = bdesc + h * h_step;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_f16_ts(d, a0 + h * 32 + kk * 8, bh + kk * 2, idesc, (ks != (KS ? part : 0)) || (h | kk) != 0);
          }
          umma_commit(&c->a_empty[as]);
        }
        __syncwarp();
        if (++as == static_cast<uint32_t>(p.da)) { as = 0; aph ^= 1; }
        if (aborted) break;
        if (lane == 0) umma_commit(&c->b_empty[bs]);
        __syncwarp();
        if (++bs == static_cast<uint32_t>(p.db)) { bs = 0; bph ^= 1; }
      }
      if (aborted) break;
      if (lane == 0) umma_commit(&c->t_full[ab]);
      __syncwarp();
    }
    if (aborted && active && lane == 0) {
      umma_commit(&c->drain[mi]);   // every MMA this thread issued has finished once this arrives
      drain_wait(&c->drain[mi], 0);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const int et = threadIdx.x - 64;         // 0..127: first code-table entry this thread builds
    int cur = 0, acc_it = 0, built = 0;
    bool aborted = false;
    // Code tables of the tile whose record is `rc` (every thread of the 4 warps):
    // entry (code e % 256) of projection e / 256 = levels x fp8(code) x expert scale,
    // rounded to the operand type, as byte planes.  Built here, ahead of the
    // decoders, so the decoders only decode: two tiles ahead with two accumulator
    // buffers, one with a single buffer (there the index producer reaches record
    // n+2 only after tile n's epilogue has freed the accumulator, so waiting for
    // that record before tile n's epilogue would never end).
    auto build_tables = [&](int rc) -> bool {
      const int rr = rc % kRecs;
      if (!mbar_wait_idle(&c->i_full[rr], (rc / kRecs) & 1, abort_flag, p.dev_err)) return false;
      const TileRec& rec = recs[rr];
      if (!rec.ok) return true;
      const int tb = built & 1;
      if (!mbar_wait_idle(&c->tab_empty[tb], ((built >> 1) & 1) ^ 1, abort_flag, p.dev_err)) return false;
      for (int e = et; e < 256 * NPROJ; e += 128) {
        const int j = e >> 8, code = e & 255;
        const float s = __fmul_rn(lut[code], rec.es[j]);
        uint4* tj = tabs + (tb * NPROJ + j) * 512;
        if (rec.bits == 3) {
          const Table8 t8 = make_table8<BF16>(rec.lev[j], s);
          tj[code] = make_uint4(t8.l0, t8.l1, t8.h0, t8.h1);
        } else {
          const Table16 t16 = make_table16<BF16>(rec.lev[j], s);
          tj[code] = make_uint4(t16.la0, t16.la1, t16.lb0, t16.lb1);
          tj[256 + code] = make_uint4(t16.ha0, t16.ha1, t16.hb0, t16.hb1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&c->tab_ready[tb]);
      ++built;
      return true;
    };
    const int ahead = p.nbuf >= 2 ? 2 : 1;
    for (int k = 0; k < ahead && !aborted; ++k)
      if (static_cast<int>(blockIdx.x + k * gridDim.x) < num_tiles) aborted = !build_tables(k);
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x, ++cur) {
      if (t + ahead * static_cast<int>(gridDim.x) < num_tiles && !build_tables(cur + ahead)) break;
      const int ri = cur % kRecs;
      if (!mbar_wait_idle(&c->i_full[ri], (cur / kRecs) & 1, abort_flag, p.dev_err)) break;
      const int ok = recs[ri].ok, cnt = recs[ri].cnt, b = recs[ri].b, m = recs[ri].m;
      __syncwarp();
      if (!ok) {
        if (lane == 0) mbar_arrive(&c->i_empty[ri]);
        if (warp == 2 && lane == 0) atomicOr(p.dev_err, kDevErrNoTier);
        continue;
      }
      const int ab = acc_it % p.nbuf;
      if (!mbar_wait_idle(&c->t_full[ab], (acc_it / p.nbuf) & 1, abort_flag, p.dev_err)) break;
      ++acc_it;
      tc_fence_after();
      // gate/up: lanes pair up on adjacent outputs (o, o + 1): one shuffle per two
      // values, then each lane stores one packed pair, the even lane for token n
      // and the odd lane for token n + 1.  Down (whose per-slot rows are the
      // larger write, scattered over the slots): the warp's 32 rows of 8 tokens
      // go through a 512-byte staging tile in shared memory, and each lane stores
      // 8 consecutive outputs of one token as one 16-byte vector.  Down reads the
      // block's slot ids and top-k weights from the tile record (the same
      // address for the whole warp).
      const bool odd = lane & 1;
      const int o_pair = m * 128 + row - (odd ? 1 : 0);
      const bool store_pair = o_pair < p.rows_store;          // rows_store is even
      uint16_t* out16 = reinterpret_cast<uint16_t*>(p.out);
      const uint32_t d0 = tl + ab * p.acc_stride;
      for (int n0 = 0; n0 < cnt; n0 += 16) {
        uint32_t g[16], u[16];
        tmem_ld16(d0 + n0, g);
        if (GLU) tmem_ld16(d0 + p.bm + n0, u);
        tmem_ld_wait();
        if (KS) {
          // split issue: the odd-step accumulator (columns bm on) adds in
          uint32_t g2[16];
          tmem_ld16(d0 + p.bm + n0, g2);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) g[j] = __float_as_uint(__uint_as_float(g[j]) + __uint_as_float(g2[j]));
        }
        if (n0 + 16 >= cnt) {
          // every accumulator column of the tile is in registers: free the buffer now
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&c->t_empty[ab]);
        }
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (GLU) {
            // silu(g) = g / (1 + e^-g) with CUDA's fast exp and divide intrinsics
            // (relative error about 2^-20, far below the bf16 / f16 rounding of
            // act that follows; tests/test_gpu_probe.py bounds it at one unit in
            // the last place); a large negative g gives -0
            const float gg = __uint_as_float(g[j]);
            v[j] = __fdividef(gg, 1.0f + __expf(-gg)) * __uint_as_float(u[j]);
          } else {
            v[j] = __uint_as_float(g[j]) * recs[ri].w[n0 + j];
          }
        }
        if constexpr (GLU) {
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const float keep = odd ? v[j + 1] : v[j];
            const float other = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[j + 1], 1);
            const int n = n0 + j + (odd ? 1 : 0);
            if (n < cnt && store_pair) {
              const size_t orow = static_cast<size_t>(b) * p.bm + n;
              *reinterpret_cast<uint32_t*>(out16 + orow * p.ld_out + o_pair) =
                  odd ? pack2<BF16>(other, keep) : pack2<BF16>(keep, other);
            }
          }
        } else {
          uint16_t* stg = reinterpret_cast<uint16_t*>(smem + kOffStage) + (warp - 2) * 256;   // [8 tokens][32 rows]
          const int tok = lane >> 2, part = lane & 3;
          const int o8 = m * 128 + q * 32 + part * 8;                   // this lane's 8 outputs (rows_store % 8 == 0)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            __syncwarp();
#pragma unroll
            for (int jj = 0; jj < 8; ++jj)
              stg[jj * 32 + lane] = static_cast<uint16_t>(pack2<BF16>(v[8 * h + jj], 0.f) & 0xFFFFu);
            __syncwarp();
            const int n = n0 + 8 * h + tok;
            if (n < cnt && o8 < p.rows_store) {
              const uint4 val = *reinterpret_cast<const uint4*>(stg + tok * 32 + part * 8);
              *reinterpret_cast<uint4*>(slot_out_row(p.slot_out, out16, p.ld_out, recs[ri].slot[n]) + o8) = val;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&c->i_empty[ri]);
    }
  } else {
    // ------------------------------------------------------------ decoders
    const int d = warp - 6;
    const int group = d >> 3;                // takes the 128-input sub-blocks kb with kb % kDecGroups == group
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int role = (d & 7) >> 2;           // gate/up: projection; down: which half of a sub-block
    const int proj = GLU ? role : 0;
    const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16);
    uint32_t xs = 0, xph = 0, as = 0, aph = 0;
    bool aborted = false;
    int cur = 0, work = 0;
    int pending = -1;                        // operand stage stored to TMEM but not yet handed over
    uint32_t ba[16], bb[16];                 // decoded 32-input blocks, alternating store buffers
#pragma unroll
    for (int i = 0; i < 16; ++i) ba[i] = bb[i] = 0u;
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x, ++cur) {
      const int ri = cur % kRecs;
      if (!mbar_wait(&c->i_full[ri], (cur / kRecs) & 1, abort_flag, p.dev_err)) { aborted = true; break; }
      const int ok = recs[ri].ok, bits = recs[ri].bits;
      const int tb = work & 1;
      __syncwarp();
      if (lane == 0) mbar_arrive(&c->i_empty[ri]);
      if (!ok) continue;
      if (!mbar_wait(&c->tab_ready[tb], (work >> 1) & 1, abort_flag, p.dev_err)) { aborted = true; break; }
      const int sb = work & 1;
      if (!mbar_wait(&c->s_full[sb], (work >> 1) & 1, abort_flag, p.dev_err)) { aborted = true; break; }
      ++work;
      const uint4* tab = tabs + (tb * NPROJ + proj) * 512;
      const uint8_t* srow = scale_buf + (sb * NPROJ + proj) * p.sz_scale + row * spr;
      // the sub-block loop is specialised on the tile's index width: no per-block branch
      auto kb_loop = [&](auto bits_c) {
        constexpr int BITS = decltype(bits_c)::value;
        int sub = -1, grp = kDecGroups - 1;     // position in the index stage / in the group rotation
        // scale codes of the 4 blocks of a 128-input step, one byte each, loaded one step ahead
        auto load_sc = [&](int k) -> uint32_t {
          return p.block == 32 ? *reinterpret_cast<const uint32_t*>(srow + k * 4)
                               : static_cast<uint32_t>(srow[k]) * 0x01010101u;
        };
        uint32_t sc_next = load_sc(0);
        for (int kb = 0; kb < ksteps && !aborted; ++kb) {
          const uint32_t sc = sc_next;
          if (kb + 1 < ksteps) sc_next = load_sc(kb + 1);
          if (++sub == spi) sub = 0;
          if (++grp == kDecGroups) grp = 0;
          const bool mine_k = grp == group;
          if (sub == 0) {
            if (!mbar_wait(&c->x_full[xs], xph, abort_flag, p.dev_err)) { aborted = true; break; }
          }
          uint32_t w[16];
          if (mine_k) {
            // this row's 4 words of each 32-input block: [proj][sub][32-row slice][block][row ^ 2 block] x 16 B
            const uint4* w4 = reinterpret_cast<const uint4*>(xring + xs * p.sz_idx) + (proj * spi + sub) * 512 +
                              (row >> 5) * 128;
            const int rs = row & 31;
            const uint4 v0 = w4[rs], v1 = w4[32 + (rs ^ 2)], v2 = w4[64 + (rs ^ 4)], v3 = w4[96 + (rs ^ 6)];
            w[0] = v0.x; w[1] = v0.y; w[2] = v0.z; w[3] = v0.w;
            w[4] = v1.x; w[5] = v1.y; w[6] = v1.z; w[7] = v1.w;
            w[8] = v2.x; w[9] = v2.y; w[10] = v2.z; w[11] = v2.w;
            w[12] = v3.x; w[13] = v3.y; w[14] = v3.z; w[15] = v3.w;
          }
          if (sub == spi - 1) {
            // every sub-block of the stage this group reads is in registers: release it
            __syncwarp();
            if (lane == 0) mbar_arrive(&c->x_empty[xs]);
            if (++xs == static_cast<uint32_t>(p.di)) { xs = 0; xph ^= 1; }
          }
          if (!mine_k) {
            // another group's operand stage
            as += 1;
            if (as >= static_cast<uint32_t>(p.da)) { as -= p.da; aph ^= 1; }
            continue;
          }
          bool have_stage = false;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const bool mine = GLU || role == h;
            if (mine) {
              // the two 32-input blocks of this half go through alternating
              // 16-register buffers: a block is decoded while the other buffer's
              // store is in flight, and each wait names the buffer it frees
              const uint32_t acol = tl + p.a_base + as * p.a_stride + proj * 64 + h * 32;
              if (h == 0) decode_block<0>(w, BITS, tab, sc & 255u, ba);
              else decode_block<2>(w, BITS, tab, (sc >> 16) & 255u, ba);
              tmem_st_wait_keep(bb);
              if (!have_stage) {
                if (pending >= 0) {
                  // the previous step's stores are done: hand its stage to the MMA
                  // (before waiting for a free stage, which may be that one's successor in the ring)
                  tc_fence_before();
                  __syncwarp();
                  if (lane == 0) mbar_arrive(&c->a_full[pending]);
                  pending = -1;
                }
                if (!mbar_wait(&c->a_empty[as], aph ^ 1, abort_flag, p.dev_err)) { aborted = true; break; }
                tc_fence_after();
                have_stage = true;
              }
              tmem_st16(acol, ba);
              if (h == 0) decode_block<1>(w, BITS, tab, (sc >> 8) & 255u, bb);
              else decode_block<3>(w, BITS, tab, sc >> 24, bb);
              tmem_st_wait_keep(ba);
              tmem_st16(acol + 16, bb);
            }
          }
          pending = static_cast<int>(as);
          if (++as == static_cast<uint32_t>(p.da)) { as = 0; aph ^= 1; }
        }
      };
      if (bits == 3) kb_loop(std::integral_constant<int, 3>{});
      else kb_loop(std::integral_constant<int, 4>{});
      if (pending >= 0 && !aborted) {
        // end of the tile: hand over the last half-stage now
        tmem_st_wait_keep(bb);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&c->a_full[pending]);
        pending = -1;
      }
      __syncwarp();
      if (!aborted && lane == 0) {
        mbar_arrive(&c->tab_empty[tb]);
        mbar_arrive(&c->s_empty[sb]);
      }
    }
    if (pending >= 0) tmem_st_wait();
  }

  if (!GLU && p.slot_out.fence) __threadfence_system();   // peer stores visible before the return flags
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

template <bool GLU, bool BF16, bool KS>
static cudaError_t launch_one(const GemmParams& p, int grid, cudaStream_t stream, bool pdl) {
  auto kern = hex_gemm_kernel<GLU, BF16, KS>;
  // per device and instantiation, raised monotonically; the mutex keeps two
  // host threads from racing on the first launches
  static std::atomic<int> configured_bytes[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  const int bytes = static_cast<int>(p.smem_bytes);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (bytes > configured_bytes[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(mu);
    if (bytes > configured_bytes[dev].load(std::memory_order_relaxed)) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      if (e != cudaSuccess) return e;
      configured_bytes[dev].store(bytes, std::memory_order_release);
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

cudaError_t launch_gemm(const GemmParams& p, bool glu, bool bf16, int grid, cudaStream_t stream, bool pdl) {
  // gate/up never splits its issue (two projections already take both issuer warps)
  if (glu) {
    if (p.ksplit != 1) return cudaErrorInvalidValue;
    return bf16 ? launch_one<true, true, false>(p, grid, stream, pdl) : launch_one<true, false, false>(p, grid, stream, pdl);
  }
  if (p.ksplit == 2)
    return bf16 ? launch_one<false, true, true>(p, grid, stream, pdl) : launch_one<false, false, true>(p, grid, stream, pdl);
  return bf16 ? launch_one<false, true, false>(p, grid, stream, pdl) : launch_one<false, false, false>(p, grid, stream, pdl);
}

}  // namespace hexmoe
