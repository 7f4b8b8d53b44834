/*
 * hex_oracle.c — CPU restatement of the reference HEX fused-MoE path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests, the
 * smoke check and bench.py's CPU-baseline leg compare the CUDA library with.
 * Nothing in the product (libhexmoe.so, the blackhole_b200 package) links,
 * imports or calls it.
 *
 * Each function names the reference lines it restates (paths are relative to
 * the OliverVillson/BlackHole-Harness tree).  Pinned against golden vectors
 * produced by running the Python reference (tests/golden/make_golden.py).
 *
 * Build: see oracle/Makefile (gcc -O2 -fopenmp -shared).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define HEX_BLOCK 32

/* fp8 e4m3 code -> float, the HEX decode (blackhole/anatomy/hex.py:199-203,
 * runtime/blackhole_runtime/hex_ref.py:41-45):
 *   ex = (c >> 3) & 15, mt = c & 7
 *   s  = ex == 0 ? mt / 8 * 0.015625 : (1 + mt / 8) * 2^(ex - 7),  negated if c & 128.
 * Codes 0x7F / 0xFF therefore decode to +-480, not NaN.  Every value is exact
 * in float. */
float hexo_fp8(uint8_t c) {
  int ex = (c >> 3) & 15, mt = c & 7;
  float s = ex == 0 ? (float)mt / 8.0f * 0.015625f : (1.0f + (float)mt / 8.0f) * ldexpf(1.0f, ex - 7);
  return (c & 128) ? -s : s;
}

/* Code of input i in one row's bit stream: block i/32 owns `bits` words, value j
 * of the block sits at stream bits j*bits .. j*bits+bits-1, little-endian
 * across words (hex.py:153-166, hex.py:187-196). */
static inline unsigned hexo_code(const uint32_t* row_words, int64_t i, int bits) {
  const uint32_t* w = row_words + (i / HEX_BLOCK) * bits;
  int off = (int)(i % HEX_BLOCK) * bits;
  int wi = off >> 5, sh = off & 31;
  uint64_t v = (uint64_t)w[wi] >> sh;
  if (sh + bits > 32) v |= (uint64_t)w[wi + 1] << (32 - sh);
  return (unsigned)(v & ((1u << bits) - 1));
}

/* hex_dequant (hex.py:180-204): W[e, o, i] = v * s with
 *   v = levels[e, code], s = fp8(block_scale[e, o, i/block]) * expert_scale[e],
 * both products rounded to float.  `block` 32 is the reference layout; 128 is
 * the same formula with one scale per 128 inputs (equal to repeating each code
 * four times in a block-32 scale tensor).  rows_pad/cols_pad give the stored
 * shape; W is [n, rows, cols] (logical). */
void hexo_dequant(const uint32_t* idx, const uint8_t* bs, const float* es, const float* lev,
                  int64_t n, int64_t rows, int64_t cols, int64_t rows_pad, int64_t cols_pad,
                  int bits, int block, float* W) {
  int64_t wpr = cols_pad / HEX_BLOCK * bits, spr = cols_pad / block;
  int L = 1 << bits;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t e = 0; e < n; e++)
    for (int64_t o = 0; o < rows; o++) {
      const uint32_t* rw = idx + (e * rows_pad + o) * wpr;
      const uint8_t* rs = bs + (e * rows_pad + o) * spr;
      float* out = W + (e * rows + o) * cols;
      for (int64_t i = 0; i < cols; i++) {
        float s = hexo_fp8(rs[i / block]) * es[e];
        out[i] = lev[e * L + hexo_code(rw, i, bits)] * s;
      }
    }
}

/* pack (runtime/blackhole_runtime/hex_ref.py:49-61; hex.py:136-150): codes
 * [rows, cols] (cols a multiple of 32) -> words [rows, cols/32*bits]. */
void hexo_pack(const uint8_t* codes, int64_t rows, int64_t cols, int bits, uint32_t* words) {
  int64_t wpr = cols / HEX_BLOCK * bits;
  memset(words, 0, (size_t)(rows * wpr) * sizeof(uint32_t));
  for (int64_t r = 0; r < rows; r++)
    for (int64_t i = 0; i < cols; i++) {
      uint32_t* w = words + r * wpr + (i / HEX_BLOCK) * bits;
      int off = (int)(i % HEX_BLOCK) * bits, wi = off >> 5, sh = off & 31;
      uint64_t c = codes[r * cols + i] & ((1u << bits) - 1);
      w[wi] |= (uint32_t)((c << sh) & 0xFFFFFFFFu);
      if (sh + bits > 32) w[wi + 1] |= (uint32_t)(c >> (32 - sh));
    }
}

/* unpack_bits (hex.py:153-166). */
void hexo_unpack(const uint32_t* words, int64_t rows, int64_t cols, int bits, uint8_t* codes) {
  int64_t wpr = cols / HEX_BLOCK * bits;
  for (int64_t r = 0; r < rows; r++)
    for (int64_t i = 0; i < cols; i++) codes[r * cols + i] = (uint8_t)hexo_code(words + r * wpr, i, bits);
}

/* align (runtime/blackhole_runtime/hex_moe.py:201-222): group slots by expert
 * (stable), pad each expert's run to block_m.  sorted_ids has
 * max_blocks*block_m entries, max_blocks = ceil(S/block_m) + min(n, S);
 * padding holds S; expert_ids[b] = expert of block b or -1; npp = padded
 * length.  Returns max_blocks, or -1 on an id outside [0, n). */
int64_t hexo_align(const int64_t* ids, int64_t S, int64_t n, int64_t block_m, int32_t* sorted_ids,
                   int32_t* expert_ids, int32_t* npp) {
  int64_t max_blocks = (S + block_m - 1) / block_m + (n < S ? n : S);
  int64_t* counts = calloc((size_t)n + 1, sizeof(int64_t));
  int64_t* start = calloc((size_t)n + 1, sizeof(int64_t));
  int64_t* cursor = calloc((size_t)n + 1, sizeof(int64_t));
  for (int64_t s = 0; s < S; s++) {
    if (ids[s] < 0 || ids[s] >= n) { free(counts); free(start); free(cursor); return -1; }
    counts[ids[s]]++;
  }
  int64_t blk = 0;
  for (int64_t e = 0; e < n; e++) {
    start[e] = blk * block_m;
    blk += (counts[e] + block_m - 1) / block_m;
  }
  for (int64_t i = 0; i < max_blocks * block_m; i++) sorted_ids[i] = (int32_t)S;
  for (int64_t s = 0; s < S; s++) sorted_ids[start[ids[s]] + cursor[ids[s]]++] = (int32_t)s;
  int64_t b = 0;
  for (int64_t e = 0; e < n; e++)
    for (int64_t k = 0; k < (counts[e] + block_m - 1) / block_m; k++) expert_ids[b++] = (int32_t)e;
  for (; b < max_blocks; b++) expert_ids[b] = -1;
  *npp = (int32_t)(blk * block_m);
  free(counts); free(start); free(cursor);
  return max_blocks;
}

/* Round float to bf16 (nearest even) and back, as torch's .to(bfloat16). */
static inline float hexo_round_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) { u = 0x7FC00000u; }
  else { u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u; }
  memcpy(&f, &u, 4);
  return f;
}

/* Round float to IEEE half (nearest even) and back. */
static inline float hexo_round_f16(float f) {
  _Float16 h = (_Float16)f;
  return (float)h;
}

typedef struct hexo_proj {
  const uint32_t* idx;
  const uint8_t* bs;
  const float* es;
  const float* lev;
} hexo_proj;

typedef struct hexo_tier {
  int32_t bits;
  int32_t n;
  const int64_t* experts;      /* [n] global ids */
  hexo_proj gate, up, down;    /* stored as [n, I_pad, H_pad/32*bits], [n, H_pad, I_pad/32*bits] */
} hexo_tier;

/* moe_reference (runtime/blackhole_runtime/hex_ref.py:77-94):
 *   per tier: dequantize gate/up/down of every expert in fp32 (hex_dequant);
 *   per expert e (tier order, then local order): (tok, slot) = pairs with
 *   topk_ids[tok, slot] == e in row-major order; a = x[tok];
 *   h = silu(a Wg^T) * (a Wu^T), rounded to the activation dtype;
 *   out[tok] += (h Wd^T) * topk_weights[tok, slot]   (fp32 accumulation).
 * x is given as float; act_dtype 0 = f32 (no rounding), 1 = bf16, 2 = f16.
 * Weights can be pre-dequantized once (wcache != NULL: per tier three float
 * buffers, filled when *filled == 0), which is the "matmul only" timing. */
void hexo_moe_reference(const float* x, int64_t T, int64_t H, int64_t I, int64_t H_pad,
                        int64_t I_pad, const float* topk_w, const int64_t* topk_ids, int64_t k,
                        const hexo_tier* tiers, int32_t num_tiers, int32_t block,
                        int32_t act_dtype, float* out, float** wcache, int32_t* filled) {
  memset(out, 0, (size_t)(T * H) * sizeof(float));
  int64_t* tok = malloc(sizeof(int64_t) * (size_t)(T * k + 1));
  int64_t* slot = malloc(sizeof(int64_t) * (size_t)(T * k + 1));
  float* h = NULL;
  size_t h_cap = 0;
  for (int32_t ti = 0; ti < num_tiers; ti++) {
    const hexo_tier* t = &tiers[ti];
    float *Wg, *Wu, *Wd;
    int own = 0;
    if (wcache) {
      Wg = wcache[3 * ti]; Wu = wcache[3 * ti + 1]; Wd = wcache[3 * ti + 2];
    } else {
      Wg = malloc(sizeof(float) * (size_t)(t->n * I * H));
      Wu = malloc(sizeof(float) * (size_t)(t->n * I * H));
      Wd = malloc(sizeof(float) * (size_t)(t->n * H * I));
      own = 1;
    }
    if (!wcache || !*filled) {
      hexo_dequant(t->gate.idx, t->gate.bs, t->gate.es, t->gate.lev, t->n, I, H, I_pad, H_pad, t->bits, block, Wg);
      hexo_dequant(t->up.idx, t->up.bs, t->up.es, t->up.lev, t->n, I, H, I_pad, H_pad, t->bits, block, Wu);
      hexo_dequant(t->down.idx, t->down.bs, t->down.es, t->down.lev, t->n, H, I, H_pad, I_pad, t->bits, block, Wd);
    }
    for (int64_t le = 0; le < t->n; le++) {
      int64_t e = t->experts[le], m = 0;
      for (int64_t r = 0; r < T; r++)
        for (int64_t j = 0; j < k; j++)
          if (topk_ids[r * k + j] == e) { tok[m] = r; slot[m] = j; m++; }
      if (!m) continue;
      if (h_cap < (size_t)(m * I)) { free(h); h_cap = (size_t)(m * I); h = malloc(sizeof(float) * h_cap); }
      const float* wg = Wg + le * I * H;
      const float* wu = Wu + le * I * H;
      const float* wd = Wd + le * H * I;
#pragma omp parallel for collapse(2) schedule(static)
      for (int64_t q = 0; q < m; q++)
        for (int64_t o = 0; o < I; o++) {
          const float* a = x + tok[q] * H;
          const float* g = wg + o * H;
          const float* u = wu + o * H;
          float sg = 0.f, su = 0.f;
#pragma omp simd reduction(+ : sg, su)
          for (int64_t i = 0; i < H; i++) { sg += a[i] * g[i]; su += a[i] * u[i]; }
          float v = sg / (1.0f + expf(-sg)) * su;
          if (act_dtype == 1) v = hexo_round_bf16(v);
          else if (act_dtype == 2) v = hexo_round_f16(v);
          h[q * I + o] = v;
        }
      /* out.index_add_: contributions in pair order; a token appears at most once per
       * expert unless topk_ids repeats an expert within a row, so keep the order. */
      for (int64_t q = 0; q < m; q++) {
        float wq = topk_w[tok[q] * k + slot[q]];
        float* orow = out + tok[q] * H;
        const float* hq = h + q * I;
#pragma omp parallel for schedule(static)
        for (int64_t o = 0; o < H; o++) {
          const float* d = wd + o * I;
          float acc = 0.f;
#pragma omp simd reduction(+ : acc)
          for (int64_t i = 0; i < I; i++) acc += hq[i] * d[i];
          orow[o] += acc * wq;
        }
      }
    }
    if (own) { free(Wg); free(Wu); free(Wd); }
  }
  if (wcache) *filled = 1;
  free(h); free(tok); free(slot);
}

/* Decode table of all 256 codes (for known-answer tests). */
void hexo_fp8_table(float* out256) {
  for (int c = 0; c < 256; c++) out256[c] = hexo_fp8((uint8_t)c);
}

/* Thread count of the OpenMP loops above (0 = leave as is); returns the count in use. */
#include <omp.h>
int hexo_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
}
