// quant.cu — the HEX quantizer on the GPU: the producer side of the format.
//
// A stack of n matrices W [n, out, in] (f32) becomes the saved HEX parts of
// blackhole/anatomy/hex.py:207-227 (quantize without a Hessian): per matrix
// an expert scale, fp8 e4m3 block-scale codes, a level table of L = 2^bits
// values fitted by weighted 1-D k-means, and the nearest-level index of every
// weight packed as the layout's bit stream.  The arithmetic follows the
// reference step by step in the precision it computes in (float32 array
// arithmetic, the expert scale as a Python float, float64 sums in the table
// fit), so the outputs equal the reference's bit for bit; oracle/hexquant.py
// restates it on the CPU and tests/golden/quant.npz holds the reference's own
// outputs.
//
//   quant_amax_kernel     one CTA per matrix: es = max(max|W| / 448, 1e-30)
//                         (block_scales, hex.py:60-70)
//   quant_scales_kernel   one thread per (matrix, row, scale block): the
//                         block's fp8 scale (st.encode: nearest finite code,
//                         ties to the smaller value, st.py:67-86) and the
//                         stored code of blk / es
//   quant_sample_kernel   the fit sample: the block-normalised value (and
//                         weight) of every sampled position
//   (cub segmented radix sort of the sample, for the initial quantiles)
//   quant_fit_kernel      one CTA per matrix: np.quantile initial levels and
//                         Lloyd iterations (fit_table, hex.py:73-90)
//   quant_pack_kernel     one thread per (matrix, row, 32 inputs): nearest
//                         level (hex.py:93-95) and pack_bits (hex.py:136-150)
#include <algorithm>
#include <cstring>

#include <cub/device/device_segmented_radix_sort.cuh>

#include "internal.cuh"

namespace hexmoe {

namespace {

constexpr int kQuantThreads = 1024;
constexpr int kFitThreads = 256;       // per-thread float64 sums of 16 levels need the registers
constexpr float kFp8Max = 448.0f;

// e4m3fn value of a code (NaN codes 0x7F / 0xFF never come out of encode).
__device__ __forceinline__ float e4m3_value(uint32_t c) {
  const uint32_t e = (c >> 3) & 15u, m = c & 7u;
  const float v = e == 0 ? static_cast<float>(m) * 0.001953125f : __uint_as_float(((e + 120u) << 23) | (m << 20));
  return (c & 128u) ? -v : v;
}

// The finite e4m3 codes in ascending value order, equal values in code order
// (a stable sort): -448 .. -2^-9 (0xFE .. 0x81), +0 (0x00), -0 (0x80), 2^-9 ..
// 448 (0x01 .. 0x7E).  254 positions.
__device__ __forceinline__ uint32_t sorted_code(int p) {
  if (p < 126) return 0xFEu - static_cast<uint32_t>(p);
  if (p == 126) return 0x00u;
  if (p == 127) return 0x80u;
  return static_cast<uint32_t>(p - 127);
}

// st.encode(x, "F8_E4M3"): clip to +-448, i = searchsorted (first position
// whose value >= x) clipped to 1..253, then the lower neighbour when it is
// at least as close.
__device__ uint32_t e4m3_encode(float x) {
  const float xc = fminf(fmaxf(x, -kFp8Max), kFp8Max);
  int lo = 0, hi = 254;   // first position with value >= xc, in [0, 254]
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (e4m3_value(sorted_code(mid)) >= xc) hi = mid;
    else lo = mid + 1;
  }
  const int i = min(max(lo, 1), 253);
  const float a = e4m3_value(sorted_code(i - 1)), b = e4m3_value(sorted_code(i));
  return fabsf(a - xc) <= fabsf(b - xc) ? sorted_code(i - 1) : sorted_code(i);
}

__device__ __forceinline__ float block_max(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0.f;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// es[e] = max(float(max |W_e|) / 448.0, 1e-30): the reference divides the
// float32 maximum as a Python (double) float; the float32 of it is what every
// later step multiplies and divides by (NumPy casts the Python float to the
// array's float32) and what is stored.
__global__ void __launch_bounds__(kQuantThreads) quant_amax_kernel(const float* __restrict__ W, int64_t per, float* es) {
  __shared__ float red[32];
  const float* w = W + static_cast<int64_t>(blockIdx.x) * per;
  float m = 0.f;
  for (int64_t i = threadIdx.x; i < per; i += blockDim.x) m = fmaxf(m, fabsf(__ldg(w + i)));
  m = block_max(m, red);
  if (threadIdx.x == 0) es[blockIdx.x] = static_cast<float>(fmax(static_cast<double>(m) / 448.0, 1e-30));
}

// Per (matrix, row, scale block): blk = fp8(min(amax / es, 448)) * es, 1.0
// where that is not positive; the stored code is encode(min(blk / es, 448))
// (quantize re-encodes the block scales it got, hex.py:225).
__global__ void quant_scales_kernel(const float* __restrict__ W, int n, int out, int in, int block,
                                    const float* __restrict__ es, float* __restrict__ blk_out,
                                    uint8_t* __restrict__ code_out) {
  const int nblk = in / block;
  const int64_t total = static_cast<int64_t>(n) * out * nblk;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t er = i / nblk;
    const int b = static_cast<int>(i - er * nblk);
    const int e = static_cast<int>(er / out);
    const float* w = W + er * in + static_cast<int64_t>(b) * block;
    float amax = 0.f;
    for (int j = 0; j < block; j += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(w + j));
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    const float s = __ldg(es + e);
    float blk = __fmul_rn(e4m3_value(e4m3_encode(fminf(__fdiv_rn(amax, s), kFp8Max))), s);
    if (!(blk > 0.f)) blk = 1.0f;
    blk_out[i] = blk;
    code_out[i] = static_cast<uint8_t>(e4m3_encode(fminf(__fdiv_rn(blk, s), kFp8Max)));
  }
}

// xn = clip(W / blk, -1, 1) (float32 division) and the fit weight
// energy[col] * blk^2 (float32), hex.py:66-67, 219-221.
__device__ __forceinline__ float norm_value(const float* W, const float* blk, int in, int block, int64_t er, int col) {
  const float v = __fdiv_rn(__ldg(W + er * in + col), __ldg(blk + er * (in / block) + col / block));
  return fminf(fmaxf(v, -1.0f), 1.0f);
}

__global__ void quant_sample_kernel(const float* __restrict__ W, int n, int out, int in, int block,
                                    const float* __restrict__ blk, const float* __restrict__ energy,
                                    const int64_t* __restrict__ sample_idx, int64_t ns, float* __restrict__ xs,
                                    float* __restrict__ ws) {
  const int64_t total = static_cast<int64_t>(n) * ns;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i / ns, s = i - e * ns;
    const int64_t pos = sample_idx ? __ldg(sample_idx + s) : s;   // flat index into [out, in]
    const int row = static_cast<int>(pos / in), col = static_cast<int>(pos - static_cast<int64_t>(row) * in);
    const int64_t er = e * out + row;
    xs[i] = norm_value(W, blk, in, block, er, col);
    if (ws) {
      const float b = __ldg(blk + er * (in / block) + col / block);
      ws[i] = __fmul_rn(__ldg(energy + e * in + col), __fmul_rn(b, b));
    }
  }
}

__global__ void quant_offsets_kernel(int n, int64_t ns, int* off) {
  for (int i = threadIdx.x; i <= n; i += blockDim.x) off[i] = static_cast<int>(i * ns);
}

// One CTA per matrix: initial levels np.quantile(x, linspace(0, 1, L+2)[1:-1])
// (method 'linear': virtual index (ns-1)*q, numpy's _lerp in float64 from the
// float32 neighbours), then `iters` Lloyd steps: every value to the level
// whose midpoint interval holds it (float32 midpoints, searchsorted left),
// float64 sums of x*w and w per level, new level = sum / weight where the
// level has weight, sorted, rounded to float32.
__global__ void __launch_bounds__(kFitThreads) quant_fit_kernel(const float* __restrict__ xs,
                                                                  const float* __restrict__ ws,
                                                                  const float* __restrict__ sorted, int64_t ns,
                                                                  int L, int iters, float* __restrict__ lev_out) {
  __shared__ float lev[16], mids[16];
  __shared__ double part[kFitThreads / 32][2][16];   // per warp, per (num, den), per level
  const int e = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* x = xs + static_cast<int64_t>(e) * ns;
  const float* w = ws ? ws + static_cast<int64_t>(e) * ns : nullptr;
  if (threadIdx.x == 0) {
    const float* srt = sorted + static_cast<int64_t>(e) * ns;
    // each product and sum rounded on its own (no fused multiply-add), as numpy computes them
    const double step = __ddiv_rn(1.0, static_cast<double>(L + 1));
    for (int i = 0; i < L; ++i) {
      const double q = __dmul_rn(static_cast<double>(i + 1), step);
      const double v = __dmul_rn(static_cast<double>(ns - 1), q);
      const double fl = floor(v);
      int64_t pi = static_cast<int64_t>(fl), ni = pi + 1;
      if (v >= static_cast<double>(ns - 1)) pi = ni = ns - 1;
      const double gamma = __dadd_rn(v, -fl);
      const float a = srt[pi], b = srt[ni];
      const float diff = __fadd_rn(b, -a);                        // float32 subtract
      const double r = gamma >= 0.5
                           ? __dadd_rn(static_cast<double>(b), -__dmul_rn(static_cast<double>(diff), __dadd_rn(1.0, -gamma)))
                           : __dadd_rn(static_cast<double>(a), __dmul_rn(static_cast<double>(diff), gamma));
      lev[i] = static_cast<float>(r);
    }
  }
  __syncthreads();
  for (int it = 0; it < iters; ++it) {
    if (threadIdx.x < L - 1) mids[threadIdx.x] = __fdiv_rn(__fadd_rn(lev[threadIdx.x + 1], lev[threadIdx.x]), 2.0f);
    __syncthreads();
    double num[16], den[16];
#pragma unroll
    for (int l = 0; l < 16; ++l) num[l] = den[l] = 0.0;
    for (int64_t i = threadIdx.x; i < ns; i += blockDim.x) {
      const float xv = __ldg(x + i);
      const float wv = w ? __ldg(w + i) : 1.0f;
      int a = 0;
      for (int l = 0; l < L - 1; ++l) a += mids[l] < xv ? 1 : 0;
      const double xw = static_cast<double>(__fmul_rn(xv, wv));
#pragma unroll
      for (int l = 0; l < 16; ++l)
        if (l == a) { num[l] += xw; den[l] += static_cast<double>(wv); }
    }
    // fixed-order reduction: lanes by a butterfly, warps in order
#pragma unroll
    for (int l = 0; l < 16; ++l) {
      for (int o = 16; o > 0; o >>= 1) {
        num[l] += __shfl_xor_sync(0xffffffffu, num[l], o);
        den[l] += __shfl_xor_sync(0xffffffffu, den[l], o);
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int l = 0; l < 16; ++l) { part[warp][0][l] = num[l]; part[warp][1][l] = den[l]; }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      double nl[16];
      for (int l = 0; l < L; ++l) {
        double sn = 0.0, sd = 0.0;
        for (int ww = 0; ww < static_cast<int>(blockDim.x >> 5); ++ww) { sn += part[ww][0][l]; sd += part[ww][1][l]; }
        nl[l] = sd > 0.0 ? __ddiv_rn(sn, fmax(sd, 1e-30)) : static_cast<double>(lev[l]);
      }
      for (int i = 1; i < L; ++i) {   // insertion sort (L <= 16)
        const double v = nl[i];
        int j = i - 1;
        while (j >= 0 && nl[j] > v) { nl[j + 1] = nl[j]; --j; }
        nl[j + 1] = v;
      }
      for (int l = 0; l < L; ++l) lev[l] = static_cast<float>(nl[l]);
    }
    __syncthreads();
  }
  if (threadIdx.x < L) lev_out[static_cast<int64_t>(e) * L + threadIdx.x] = lev[threadIdx.x];
}

// One thread per (matrix, row, 32 inputs): codes = number of midpoints below
// xn, packed `bits` words per 32 inputs (value i at bits i*bits ..).
__global__ void quant_pack_kernel(const float* __restrict__ W, int n, int out, int in, int block,
                                  const float* __restrict__ blk, const float* __restrict__ levels, int bits,
                                  uint32_t* __restrict__ idx_out) {
  const int L = 1 << bits;
  const int n32 = in / 32;
  const int64_t total = static_cast<int64_t>(n) * out * n32;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t er = i / n32;
    const int c0 = static_cast<int>(i - er * n32) * 32;
    const int e = static_cast<int>(er / out);
    float mids[15];
    const float* lv = levels + static_cast<int64_t>(e) * L;
    for (int l = 0; l < L - 1; ++l) mids[l] = __fdiv_rn(__fadd_rn(__ldg(lv + l + 1), __ldg(lv + l)), 2.0f);
    uint32_t words[4] = {0u, 0u, 0u, 0u};
    for (int j = 0; j < 32; ++j) {
      const float xv = norm_value(W, blk, in, block, er, c0 + j);
      uint32_t a = 0;
      for (int l = 0; l < L - 1; ++l) a += mids[l] < xv ? 1u : 0u;
      const int off = j * bits, wi = off >> 5, sh = off & 31;
      words[wi] |= a << sh;
      if (sh + bits > 32) words[wi + 1] |= a >> (32 - sh);
    }
    uint32_t* dst = idx_out + er * (n32 * bits) + static_cast<int64_t>(c0 / 32) * bits;
    for (int k = 0; k < bits; ++k) dst[k] = words[k];
  }
}

// GPTQ onto the table (gptq_table, hex.py:256-282): one CTA per (matrix, 128
// rows), one thread per row (rows never interact: the sweep couples columns
// only).  Per 128-column block: the rows' current values and the block of U
// (the upper Cholesky factor of the damped inverse Hessian) in shared memory;
// columns in order, each rounded onto levels x scale (nearest level of the
// clipped scaled value), its error e = (w - q) / U[j, j] spread over the
// block's later columns (w -= e U[j, :]) and kept in place of the column; then
// the later columns of the matrix take the block's errors at once
// (W[:, b1:] -= E U[b0:b1, b1:], an FP32 product over shared-memory panels of
// U).  The codes chosen are the GPTQ indices (nearest(Q / scale) of the
// reference gives back the same level).  W_work: the matrix with dead inputs
// zeroed, updated in place.
constexpr int kGptqRows = 128;
constexpr int kGptqCols = 128;
constexpr int kGptqPitch = kGptqCols + 1;   // row pitch of the rows' block (floats): conflict-free per-thread rows

__global__ void gptq_init_kernel(const float* __restrict__ W, const uint8_t* __restrict__ dead, int n, int out, int in,
                                 float* __restrict__ Ww) {
  const int64_t total = static_cast<int64_t>(n) * out * in;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i / (static_cast<int64_t>(out) * in);
    const int col = static_cast<int>(i % in);
    Ww[i] = __ldg(dead + e * in + col) ? 0.0f : __ldg(W + i);
  }
}

__global__ void __launch_bounds__(kGptqRows) gptq_kernel(float* __restrict__ Ww, const float* __restrict__ U,
                                                         const uint8_t* __restrict__ dead,
                                                         const float* __restrict__ blk,
                                                         const float* __restrict__ levels, int out, int in, int block,
                                                         int L, uint8_t* __restrict__ codes) {
  extern __shared__ float gsm[];
  float* rows = gsm;                                   // [kGptqRows][kGptqPitch]: values, then errors
  float* ub = gsm + kGptqRows * kGptqPitch;            // [kGptqCols][kGptqCols]: U block, then U panels
  __shared__ float lv[16], mids[16];
  const int e = blockIdx.y;
  const int r0 = blockIdx.x * kGptqRows;
  const int t = threadIdx.x;
  const int row = r0 + t;
  const bool live_row = row < out;
  if (t < L) lv[t] = __ldg(levels + static_cast<int64_t>(e) * L + t);
  __syncthreads();
  if (t < L - 1) mids[t] = __fdiv_rn(__fadd_rn(lv[t + 1], lv[t]), 2.0f);
  float* wrow = Ww + (static_cast<int64_t>(e) * out + (live_row ? row : 0)) * in;
  const float* ue = U + static_cast<int64_t>(e) * in * in;
  const float* srow = blk + (static_cast<int64_t>(e) * out + (live_row ? row : 0)) * (in / block);
  uint8_t* crow = codes + (static_cast<int64_t>(e) * out + (live_row ? row : 0)) * in;
  float* my = rows + t * kGptqPitch;
  for (int b0 = 0; b0 < in; b0 += kGptqCols) {
    const int bw = min(kGptqCols, in - b0);
    __syncthreads();
    for (int i = t; i < kGptqCols * kGptqCols; i += blockDim.x) {
      const int j = i / kGptqCols, c = i - j * kGptqCols;
      ub[i] = (j < bw && c < bw) ? __ldg(ue + static_cast<int64_t>(b0 + j) * in + b0 + c) : 0.0f;
    }
    for (int c = 0; c < bw; ++c) my[c] = live_row ? wrow[b0 + c] : 0.0f;
    __syncthreads();
    // the block's columns in order (each thread its own row)
    for (int j = 0; j < bw; ++j) {
      const float w = my[j];
      const float s = __ldg(srow + (b0 + j) / block);
      const float x = fminf(fmaxf(__fdiv_rn(w, s), -1.0f), 1.0f);
      int k = 0;
      for (int l = 0; l < L - 1; ++l) k += mids[l] < x ? 1 : 0;
      const float q = __fmul_rn(lv[k], s);
      const float err = __fdiv_rn(__fadd_rn(w, -q), ub[j * kGptqCols + j]);
      if (live_row) crow[b0 + j] = static_cast<uint8_t>(k);
      my[j] = err;
      const float* uj = ub + j * kGptqCols;
      for (int c = j + 1; c < bw; ++c) my[c] = __fmaf_rn(-err, uj[c], my[c]);
    }
    // the later columns: W[row, c] -= sum_j E[row, j] U[b0 + j, c], panels of 128 columns
    for (int p0 = b0 + bw; p0 < in; p0 += kGptqCols) {
      const int pw = min(kGptqCols, in - p0);
      __syncthreads();
      for (int i = t; i < kGptqCols * kGptqCols; i += blockDim.x) {
        const int j = i / kGptqCols, c = i - j * kGptqCols;
        ub[i] = (j < bw && c < pw) ? __ldg(ue + static_cast<int64_t>(b0 + j) * in + p0 + c) : 0.0f;
      }
      __syncthreads();
      for (int c0 = 0; c0 < pw; c0 += 32) {
        float acc[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) acc[c] = 0.0f;
        for (int j = 0; j < bw; ++j) {
          const float ej = my[j];
          const float4* u4 = reinterpret_cast<const float4*>(ub + j * kGptqCols + c0);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 v = u4[c];
            acc[4 * c] = __fmaf_rn(ej, v.x, acc[4 * c]);
            acc[4 * c + 1] = __fmaf_rn(ej, v.y, acc[4 * c + 1]);
            acc[4 * c + 2] = __fmaf_rn(ej, v.z, acc[4 * c + 2]);
            acc[4 * c + 3] = __fmaf_rn(ej, v.w, acc[4 * c + 3]);
          }
        }
        if (live_row) {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (c0 + c < pw) wrow[p0 + c0 + c] = __fadd_rn(wrow[p0 + c0 + c], -acc[c]);
        }
      }
    }
  }
  // dead inputs: Q = 0 there, so the nearest level of 0
  __syncthreads();
  if (live_row) {
    int k0 = 0;
    for (int l = 0; l < L - 1; ++l) k0 += mids[l] < 0.0f ? 1 : 0;
    const uint8_t* de = dead + static_cast<int64_t>(e) * in;
    for (int c = 0; c < in; ++c)
      if (__ldg(de + c)) crow[c] = static_cast<uint8_t>(k0);
  }
}

// Pack chosen codes u8 [n, out, in] as the layout's bit stream.
__global__ void quant_pack_codes_kernel(const uint8_t* __restrict__ codes, int64_t rows, int in, int bits,
                                        uint32_t* __restrict__ idx_out) {
  const int n32 = in / 32;
  const int64_t total = rows * n32;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / n32;
    const int c0 = static_cast<int>(i - r * n32) * 32;
    uint32_t words[4] = {0u, 0u, 0u, 0u};
    for (int j = 0; j < 32; ++j) {
      const uint32_t a = __ldg(codes + r * in + c0 + j);
      const int off = j * bits, wi = off >> 5, sh = off & 31;
      words[wi] |= a << sh;
      if (sh + bits > 32) words[wi + 1] |= a >> (32 - sh);
    }
    uint32_t* dst = idx_out + r * (n32 * bits) + static_cast<int64_t>(c0 / 32) * bits;
    for (int k = 0; k < bits; ++k) dst[k] = words[k];
  }
}

constexpr size_t kGptqSmem = sizeof(float) * (kGptqRows * kGptqPitch + kGptqCols * kGptqCols);

struct QuantLayout {
  size_t blk, xs, ws, sorted, off, temp, temp_bytes, gw, gcodes, total;
  int64_t ns;
};

size_t up256(size_t v) { return (v + 255) / 256 * 256; }

QuantLayout quant_layout(int n, int out, int in, int block, int64_t sample, bool weighted, bool gptq) {
  QuantLayout q{};
  const int64_t size = static_cast<int64_t>(out) * in;
  q.ns = sample > 0 && sample < size ? sample : size;
  size_t off = 0;
  q.blk = off; off = up256(off + sizeof(float) * static_cast<size_t>(n) * out * (in / block));
  q.xs = off; off = up256(off + sizeof(float) * static_cast<size_t>(n) * q.ns);
  q.ws = off; off = up256(off + (weighted ? sizeof(float) * static_cast<size_t>(n) * q.ns : 0));
  q.sorted = off; off = up256(off + sizeof(float) * static_cast<size_t>(n) * q.ns);
  q.off = off; off = up256(off + sizeof(int) * static_cast<size_t>(n + 1));
  size_t tb = 0;
  cub::DeviceSegmentedRadixSort::SortKeys(nullptr, tb, static_cast<const float*>(nullptr), static_cast<float*>(nullptr),
                                          static_cast<int>(n * q.ns), n, static_cast<const int*>(nullptr),
                                          static_cast<const int*>(nullptr) + 1);
  q.temp = off; q.temp_bytes = tb; off = up256(off + tb);
  const size_t nw = gptq ? static_cast<size_t>(n) * out * in : 0;
  q.gw = off; off = up256(off + sizeof(float) * nw);
  q.gcodes = off; off = up256(off + nw);
  q.total = off;
  return q;
}

int grid_for(int64_t work, int threads) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + threads - 1) / threads, 148 * 16)));
}

}  // namespace

}  // namespace hexmoe

using namespace hexmoe;

extern "C" {

size_t hexmoe_quantize_workspace_bytes(int32_t n, int32_t out, int32_t in, int32_t block, int64_t sample,
                                       int32_t weighted, int32_t gptq) {
  if (n <= 0 || out <= 0 || in <= 0 || (block != 32 && block != 128) || in % block) return 0;
  if (static_cast<int64_t>(n) * (sample > 0 ? sample : static_cast<int64_t>(out) * in) >= (1ll << 31)) return 0;
  return quant_layout(n, out, in, block, sample, weighted != 0, gptq != 0).total;
}

int hexmoe_quantize(const float* W, int32_t n, int32_t out, int32_t in, int32_t levels, int32_t block,
                    const float* energy, const int64_t* sample_idx, int64_t sample, int32_t iters,
                    const float* hinv_u, const uint8_t* dead, uint32_t* idx_out, uint8_t* block_scale_out,
                    float* expert_scale_out, float* levels_out, void* workspace, size_t workspace_bytes,
                    void* stream) {
  if (n <= 0 || out <= 0 || in <= 0) return report_error(HEXMOE_E_ARG, "hexmoe_quantize: n, out and in must be positive");
  if (levels != 8 && levels != 16) return report_error(HEXMOE_E_ARG, "hexmoe_quantize: levels must be 8 or 16");
  if (block != 32 && block != 128) return report_error(HEXMOE_E_ARG, "hexmoe_quantize: block must be 32 or 128");
  if (in % block) return report_error(HEXMOE_E_ARG, "hexmoe_quantize: in must be a multiple of the scale block");
  if (iters < 0) return report_error(HEXMOE_E_ARG, "hexmoe_quantize: iters must not be negative");
  if (sample_idx && sample <= 0) return report_error(HEXMOE_E_ARG, "hexmoe_quantize: sample_idx needs sample > 0");
  if (!sample_idx) sample = 0;
  const int64_t size = static_cast<int64_t>(out) * in;
  if (sample > size) return report_error(HEXMOE_E_ARG, "hexmoe_quantize: more sample positions than values");
  if (static_cast<int64_t>(n) * (sample > 0 ? sample : size) >= (1ll << 31))
    return report_error(HEXMOE_E_ARG, "hexmoe_quantize: n * sample (or n * out * in) must stay below 2^31");
  if (!W || !idx_out || !block_scale_out || !expert_scale_out || !levels_out || !workspace)
    return report_error(HEXMOE_E_ARG, "hexmoe_quantize: null pointer");
  if (reinterpret_cast<uintptr_t>(W) % 16 || reinterpret_cast<uintptr_t>(workspace) % 256)
    return report_error(HEXMOE_E_ARG, "hexmoe_quantize: W must be 16-byte and workspace 256-byte aligned");
  if ((hinv_u == nullptr) != (dead == nullptr))
    return report_error(HEXMOE_E_ARG, "hexmoe_quantize: hinv_u and dead go together");
  const QuantLayout q = quant_layout(n, out, in, block, sample, energy != nullptr, hinv_u != nullptr);
  if (workspace_bytes < q.total) return report_error(HEXMOE_E_ARG, "hexmoe_quantize: workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  float* blk = reinterpret_cast<float*>(ws + q.blk);
  float* xs = reinterpret_cast<float*>(ws + q.xs);
  float* wts = energy ? reinterpret_cast<float*>(ws + q.ws) : nullptr;
  float* sorted = reinterpret_cast<float*>(ws + q.sorted);
  int* off = reinterpret_cast<int*>(ws + q.off);
  const int bits = levels == 8 ? 3 : 4;
  quant_amax_kernel<<<n, kQuantThreads, 0, st>>>(W, size, expert_scale_out);
  const int64_t nb = static_cast<int64_t>(n) * out * (in / block);
  quant_scales_kernel<<<grid_for(nb, 256), 256, 0, st>>>(W, n, out, in, block, expert_scale_out, blk, block_scale_out);
  quant_sample_kernel<<<grid_for(static_cast<int64_t>(n) * q.ns, 256), 256, 0, st>>>(W, n, out, in, block, blk, energy,
                                                                                     sample_idx, q.ns, xs, wts);
  quant_offsets_kernel<<<1, 256, 0, st>>>(n, q.ns, off);
  size_t tb = q.temp_bytes;
  cudaError_t e = cub::DeviceSegmentedRadixSort::SortKeys(ws + q.temp, tb, xs, sorted, static_cast<int>(n * q.ns), n,
                                                          off, off + 1, 0, 32, st);
  if (e != cudaSuccess) return report_cuda_error(e, "hexmoe_quantize: sample sort");
  quant_fit_kernel<<<n, kFitThreads, 0, st>>>(xs, wts, sorted, q.ns, levels, iters, levels_out);
  const int64_t np32 = static_cast<int64_t>(n) * out * (in / 32);
  if (!hinv_u) {
    quant_pack_kernel<<<grid_for(np32, 128), 128, 0, st>>>(W, n, out, in, block, blk, levels_out, bits, idx_out);
  } else {
    float* gw = reinterpret_cast<float*>(ws + q.gw);
    uint8_t* gcodes = reinterpret_cast<uint8_t*>(ws + q.gcodes);
    gptq_init_kernel<<<grid_for(static_cast<int64_t>(n) * out * in, 256), 256, 0, st>>>(W, dead, n, out, in, gw);
    e = cudaFuncSetAttribute(gptq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kGptqSmem));
    if (e != cudaSuccess) return report_cuda_error(e, "hexmoe_quantize: GPTQ shared memory");
    gptq_kernel<<<dim3((out + kGptqRows - 1) / kGptqRows, n), kGptqRows, kGptqSmem, st>>>(
        gw, hinv_u, dead, blk, levels_out, out, in, block, levels, gcodes);
    quant_pack_codes_kernel<<<grid_for(np32, 128), 128, 0, st>>>(gcodes, static_cast<int64_t>(n) * out, in, bits,
                                                                 idx_out);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return report_cuda_error(e, "hexmoe_quantize: launch");
  return HEXMOE_OK;
}

}  // extern "C"
