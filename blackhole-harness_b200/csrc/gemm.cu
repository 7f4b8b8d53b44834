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
// Warp roles (448 threads):
//   warp 0      TMA: index words of the weight tile (2-D tensor map, 128 rows x
//               128 inputs per stage), the token rows of the block (gate/up: one
//               row gather per token, down: one box), and once per tile the
//               tile's fp8 scale codes (1-D bulk copy)
//   warp 1      TMEM allocation; one thread issues tcgen05.mma (A operand from
//               TMEM, B from 128-B swizzled smem) and tcgen05.commit
//   warps 2-5   epilogue: tcgen05.ld of the accumulators, SwiGLU (gate/up) or
//               top-k weight (down), 16-bit stores
//   warps 6-13  decode: per (row, 32-input block) the scaled level table, then
//               prmt lookups of the packed codes, written to TMEM with tcgen05.st
// Every wait is bounded (ptx.cuh): a lost arrival ends the kernel with the
// device error word set instead of hanging.
#include "decode.cuh"
#include "internal.cuh"

namespace hexmoe {

struct Ctrl {
  uint64_t r_full[kMaxDR], r_empty[kMaxDR];   // index / token-row ring
  uint64_t a_full[kMaxDA], a_empty[kMaxDA];   // TMEM operand ring
  uint64_t s_full[2], s_empty[2];             // tile scale buffers
  uint64_t t_full[2], t_empty[2];             // accumulator buffers
  uint64_t drain;
  uint32_t tmem_base;
  int32_t abort;
};
static_assert(sizeof(Ctrl) <= 2048, "control block");
constexpr uint32_t kOffLut = 2048;            // fp8 decode table (256 floats)

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

template <bool BF16>
__device__ __forceinline__ uint32_t to16x2(float lo, float hi) {
  return pack2<BF16>(lo, hi);
}


// Decode the 32-input block BLK (0..3) of one stage row into 16 packed operand
// registers (K order).  w: the row's stage words; sc: the stage's 4 scale codes.
template <bool BF16, int BLK>
__device__ __forceinline__ void decode_block(const uint32_t (&w)[16], int bits, uint32_t sc, const float* lut,
                                             const float (&lev)[16], float es, uint32_t* r) {
  const float s = __fmul_rn(lut[(sc >> (8 * BLK)) & 255u], es);
  uint4 ch[4];
  if (bits == 3) {
    const Table8 tb = make_table8<BF16>(lev, s);
    dec32_b3(w[3 * BLK], w[3 * BLK + 1], w[3 * BLK + 2], tb, ch);
  } else {
    const Table16 tb = make_table16<BF16>(lev, s);
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

template <bool GLU, bool BF16>
__global__ void __launch_bounds__(kGemmThreads, 1) hex_gemm_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Ctrl* c = reinterpret_cast<Ctrl*>(smem);
  float* lut = reinterpret_cast<float*>(smem + kOffLut);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NPROJ = GLU ? 2 : 1;
  volatile int* abort_flag = &c->abort;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kMaxDR; ++i) { mbar_init(&c->r_full[i], 1); mbar_init(&c->r_empty[i], 1); }
    for (int i = 0; i < kMaxDA; ++i) { mbar_init(&c->a_full[i], 8); mbar_init(&c->a_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&c->s_full[i], 1); mbar_init(&c->s_empty[i], 8);
      mbar_init(&c->t_full[i], 1); mbar_init(&c->t_empty[i], 4);
    }
    mbar_init(&c->drain, 1);
    c->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int t = 0; t < p.num_tiers; ++t)
      for (int j = 0; j < NPROJ; ++j) prefetch_tmap(&p.tm_idx[t][j]);
    prefetch_tmap(&p.tm_b);
  }
  if (warp == 1) {
    tmem_alloc(&c->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp >= 6) {
    for (int i = threadIdx.x - 192; i < 256; i += 256) lut[i] = fp8_hex_value(static_cast<uint32_t>(i));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = c->tmem_base;

  pdl_launch_dependents();
  pdl_wait();  // the plan (and, for down, act) come from the previous kernels

  const int nbv = __ldg(p.npp) / p.bm;
  const int num_tiles = nbv * p.m_tiles;
  const int ksteps = p.k_pad / kKStep;
  const uint32_t spr = static_cast<uint32_t>(p.k_pad / p.block);   // scale bytes per weight row
  const uint32_t scale_tile = 128u * spr;                           // per projection
  uint8_t* ring = smem + p.off_ring;
  uint8_t* scale_buf = smem + p.off_scale;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    const uint64_t pol_stream = l2_policy_evict_first();
    uint32_t rs = 0, rph = 0;
    int issued = 0, s_issued = 0;
    bool aborted = false;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x) {
      const TileInfo ti = tile_info(p, t);
      if (!ti.ok) continue;
      const int cur = it++;
      const int cnt = block_rows(p, ti.b, lane);
      const uint32_t wbox = 4u * ti.bits;                         // index words per row per stage
      const uint32_t idx_bytes = NPROJ * 128u * wbox * 4u;
      const uint32_t b_bytes = GLU ? static_cast<uint32_t>(cnt) * 256u : static_cast<uint32_t>(p.bm) * 256u;
      const int sb = cur & 1;
      if (!mbar_wait(&c->s_empty[sb], ((cur >> 1) & 1) ^ 1, abort_flag, p.dev_err)) { aborted = true; break; }
      if (lane == 0) {
        mbar_arrive_expect_tx(&c->s_full[sb], scale_tile * NPROJ);
        for (int j = 0; j < NPROJ; ++j) {
          const uint8_t* src =
              p.bs[ti.tier][j] + (static_cast<size_t>(ti.local) * p.rows_pad + static_cast<size_t>(ti.m) * 128) * spr;
          bulk_load(scale_buf + (sb * NPROJ + j) * p.sz_scale, src, scale_tile, &c->s_full[sb]);
        }
      }
      ++s_issued;
      // token rows this lane gathers (gate/up): r = lane + 32 j
      int src_row[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = lane + 32 * j;
        src_row[j] = -1;
        if (GLU && r < cnt) src_row[j] = __ldg(p.sorted_ids + static_cast<size_t>(ti.b) * p.bm + r) / p.topk;
      }
      const int32_t wrow = ti.local * p.rows_pad + ti.m * 128;
      for (int ks = 0; ks < ksteps; ++ks) {
        if (!mbar_wait(&c->r_empty[rs], rph ^ 1, abort_flag, p.dev_err)) { aborted = true; break; }
        uint8_t* stage = ring + rs * p.sz_stage;
        uint8_t* bdst = stage + p.sz_idx;
        if (lane == 0) {
          mbar_arrive_expect_tx(&c->r_full[rs], idx_bytes + b_bytes);
          for (int j = 0; j < NPROJ; ++j)
            tma_load_2d_hint(stage + j * 128 * wbox * 4, &p.tm_idx[ti.tier][j], &c->r_full[rs],
                             ks * static_cast<int>(wbox), wrow, pol_stream);
          if (!GLU) {
            tma_load_2d(bdst, &p.tm_b, &c->r_full[rs], ks * kKStep, ti.b * p.bm);
            tma_load_2d(bdst + p.bm * 128, &p.tm_b, &c->r_full[rs], ks * kKStep + 64, ti.b * p.bm);
          }
        }
        __syncwarp();
        if (GLU) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (src_row[j] >= 0) {
              const int r = lane + 32 * j;
              tma_load_2d(bdst + r * 128, &p.tm_b, &c->r_full[rs], ks * kKStep, src_row[j]);
              tma_load_2d(bdst + p.bm * 128 + r * 128, &p.tm_b, &c->r_full[rs], ks * kKStep + 64, src_row[j]);
            }
          }
        }
        ++issued;
        if (++rs == static_cast<uint32_t>(p.dr)) { rs = 0; rph ^= 1; }
      }
    }
    if (aborted && lane == 0) {
      // let every copy already issued land before the CTA (and its smem) goes away
      for (int i = 1; i <= 2 && i <= s_issued; ++i) {
        const int q = s_issued - i;
        drain_wait(&c->s_full[q & 1], (q >> 1) & 1);
      }
      const int n = issued < p.dr ? issued : p.dr;
      for (int i = 1; i <= n; ++i) {
        const int q = issued - i;
        drain_wait(&c->r_full[q % p.dr], (q / p.dr) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    uint32_t rs = 0, rph = 0, as = 0, aph = 0;
    bool aborted = false;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x) {
      const TileInfo ti = tile_info(p, t);
      if (!ti.ok) continue;
      const int cur = it++;
      const int cnt = block_rows(p, ti.b, lane);
      const uint32_t n_mma = static_cast<uint32_t>(max(16, (cnt + 15) & ~15));
      const uint32_t idesc = umma_idesc(BF16, 128, n_mma);
      const int ab = cur % p.nbuf;
      if (!mbar_wait(&c->t_empty[ab], ((cur / p.nbuf) & 1) ^ 1, abort_flag, p.dev_err)) { aborted = true; break; }
      tc_fence_after();
      const uint32_t d0 = tmem + ab * p.acc_stride;
      const uint32_t d1 = d0 + p.bm;
      for (int ks = 0; ks < ksteps && !aborted; ++ks) {
        if (!mbar_wait(&c->r_full[rs], rph, abort_flag, p.dev_err)) { aborted = true; break; }
        const uint32_t bbase = smem_u32(ring + rs * p.sz_stage + p.sz_idx);
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait(&c->a_full[as], aph, abort_flag, p.dev_err)) { aborted = true; break; }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a0 = tmem + p.a_base + as * p.a_stride;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t bd = sw128_desc(bbase + h * p.bm * 128 + kk * 32);
              const uint32_t acc = (ks | h | kk) != 0;
              umma_f16_ts(d0, a0 + kk * 8, bd, idesc, acc);
              if (GLU) umma_f16_ts(d1, a0 + 32 + kk * 8, bd, idesc, acc);
            }
            umma_commit(&c->a_empty[as]);
          }
          __syncwarp();
          if (++as == static_cast<uint32_t>(p.da)) { as = 0; aph ^= 1; }
        }
        if (aborted) break;
        if (lane == 0) umma_commit(&c->r_empty[rs]);
        __syncwarp();
        if (++rs == static_cast<uint32_t>(p.dr)) { rs = 0; rph ^= 1; }
      }
      if (aborted) break;
      if (lane == 0) umma_commit(&c->t_full[ab]);
      __syncwarp();
    }
    if (aborted && lane == 0) {
      umma_commit(&c->drain);   // every MMA issued so far has finished once this arrives
      drain_wait(&c->drain, 0);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16);
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      const TileInfo ti = tile_info(p, t);
      if (!ti.ok) {
        if (warp == 2 && lane == 0) atomicOr(p.dev_err, kDevErrNoTier);
        continue;
      }
      const int cur = it++;
      const int cnt = block_rows(p, ti.b, lane);
      const int ab = cur % p.nbuf;
      if (!mbar_wait(&c->t_full[ab], (cur / p.nbuf) & 1, abort_flag, p.dev_err)) break;
      tc_fence_after();
      const int o = ti.m * 128 + row;
      const bool store_row = o < p.rows_store;
      const uint32_t d0 = tl + ab * p.acc_stride;
      for (int n0 = 0; n0 < cnt; n0 += 16) {
        uint32_t g[16], u[16];
        tmem_ld16(d0 + n0, g);
        if (GLU) tmem_ld16(d0 + p.bm + n0, u);
        tmem_ld_wait();
        if (GLU) {
          __nv_bfloat16* out_b = reinterpret_cast<__nv_bfloat16*>(p.out);
          __half* out_h = reinterpret_cast<__half*>(p.out);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = n0 + j;
            if (n < cnt && store_row) {
              const float gv = __uint_as_float(g[j]);
              const float uv = __uint_as_float(u[j]);
              const float a = gv / (1.0f + expf(-gv)) * uv;
              const size_t off = (static_cast<size_t>(ti.b) * p.bm + n) * p.ld_out + o;
              if (BF16) out_b[off] = __float2bfloat16_rn(a);
              else out_h[off] = __float2half_rn(a);
            }
          }
        } else {
          __nv_bfloat16* out_b = reinterpret_cast<__nv_bfloat16*>(p.out);
          __half* out_h = reinterpret_cast<__half*>(p.out);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = n0 + j;
            if (n < cnt && store_row) {
              const int slot = __ldg(p.sorted_ids + static_cast<size_t>(ti.b) * p.bm + n);
              const float v = __uint_as_float(g[j]) * __ldg(p.topk_w + slot);
              const size_t off = static_cast<size_t>(slot) * p.ld_out + o;
              if (BF16) out_b[off] = __float2bfloat16_rn(v);
              else out_h[off] = __float2half_rn(v);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&c->t_empty[ab]);
    }
  } else {
    // ------------------------------------------------------------ decoders
    const int d = warp - 6;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int role = d >> 2;                 // gate/up: projection; down: block parity
    const int proj = GLU ? role : 0;
    const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16);
    uint32_t rs = 0, rph = 0, as = 0, aph = 0;
    bool aborted = false;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x) {
      const TileInfo ti = tile_info(p, t);
      if (!ti.ok) continue;
      const int cur = it++;
      const int L = 1 << ti.bits;
      float lev[16];
      const float* lsrc = p.lev[ti.tier][proj] + ti.local * L;
#pragma unroll
      for (int l = 0; l < 16; ++l) lev[l] = l < L ? __ldg(lsrc + l) : 0.0f;
      const float es = __ldg(p.es[ti.tier][proj] + ti.local);
      const int sb = cur & 1;
      if (!mbar_wait(&c->s_full[sb], (cur >> 1) & 1, abort_flag, p.dev_err)) { aborted = true; break; }
      const uint8_t* srow = scale_buf + (sb * NPROJ + proj) * p.sz_scale + row * spr;
      const uint32_t wbox = 4u * ti.bits;
      for (int ks = 0; ks < ksteps && !aborted; ++ks) {
        if (!mbar_wait(&c->r_full[rs], rph, abort_flag, p.dev_err)) { aborted = true; break; }
        const uint32_t* wsrc =
            reinterpret_cast<const uint32_t*>(ring + rs * p.sz_stage) + (proj * 128 + row) * wbox;
        uint32_t w[16];
        const uint4* w4 = reinterpret_cast<const uint4*>(wsrc);
        {
          const uint4 v0 = w4[0], v1 = w4[1], v2 = w4[2];
          w[0] = v0.x; w[1] = v0.y; w[2] = v0.z; w[3] = v0.w;
          w[4] = v1.x; w[5] = v1.y; w[6] = v1.z; w[7] = v1.w;
          w[8] = v2.x; w[9] = v2.y; w[10] = v2.z; w[11] = v2.w;
          if (ti.bits == 4) {
            const uint4 v3 = w4[3];
            w[12] = v3.x; w[13] = v3.y; w[14] = v3.z; w[15] = v3.w;
          } else {
            w[12] = w[13] = w[14] = w[15] = 0u;
          }
        }
        uint32_t sc;   // scale codes of the 4 blocks of this stage, one byte each
        if (p.block == 32) sc = *reinterpret_cast<const uint32_t*>(srow + ks * 4);
        else sc = static_cast<uint32_t>(srow[ks]) * 0x01010101u;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait(&c->a_empty[as], aph ^ 1, abort_flag, p.dev_err)) { aborted = true; break; }
          tc_fence_after();
          const uint32_t acol = tl + p.a_base + as * p.a_stride;
          if (GLU) {
            uint32_t r[32];
            if (h == 0) {
              decode_block<BF16, 0>(w, ti.bits, sc, lut, lev, es, r);
              decode_block<BF16, 1>(w, ti.bits, sc, lut, lev, es, r + 16);
            } else {
              decode_block<BF16, 2>(w, ti.bits, sc, lut, lev, es, r);
              decode_block<BF16, 3>(w, ti.bits, sc, lut, lev, es, r + 16);
            }
            tmem_st32(acol + proj * 32, r);
          } else {
            uint32_t r[16];
            if (h == 0) {
              if (role == 0) decode_block<BF16, 0>(w, ti.bits, sc, lut, lev, es, r);
              else decode_block<BF16, 1>(w, ti.bits, sc, lut, lev, es, r);
            } else {
              if (role == 0) decode_block<BF16, 2>(w, ti.bits, sc, lut, lev, es, r);
              else decode_block<BF16, 3>(w, ti.bits, sc, lut, lev, es, r);
            }
            tmem_st16(acol + role * 16, r);
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&c->a_full[as]);
          if (++as == static_cast<uint32_t>(p.da)) { as = 0; aph ^= 1; }
        }
        if (++rs == static_cast<uint32_t>(p.dr)) { rs = 0; rph ^= 1; }
      }
      __syncwarp();
      if (!aborted && lane == 0) mbar_arrive(&c->s_empty[sb]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

template <bool GLU, bool BF16>
static cudaError_t launch_one(const GemmParams& p, int grid, cudaStream_t stream, bool pdl) {
  auto kern = hex_gemm_kernel<GLU, BF16>;
  static int configured_bytes = 0;   // per instantiation; raised monotonically
  const int bytes = static_cast<int>(p.smem_bytes);
  if (bytes > configured_bytes) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    configured_bytes = bytes;
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
  if (glu) return bf16 ? launch_one<true, true>(p, grid, stream, pdl) : launch_one<true, false>(p, grid, stream, pdl);
  return bf16 ? launch_one<false, true>(p, grid, stream, pdl) : launch_one<false, false>(p, grid, stream, pdl);
}

}  // namespace hexmoe
