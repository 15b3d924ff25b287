/*
 * CPU oracle for the fused DiT layer ops — TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this file's library; the product path (anima_flat_b200) never does.
 *
 * It restates the reference's per-row formulas (tan0210/anima-flat,
 * src/kernels/adaln.py, fp8.py, rope.py; cited per function) in plain C with
 * IEEE-754 binary32 arithmetic: compiled with -ffp-contract=off and without
 * -ffast-math, every + - * / sqrtf is one correctly rounded operation and
 * fmaf is used only where written.  Reductions follow the canonical order
 * (canonical_sum below), which fixes the association the reference leaves to
 * Triton's autotuned num_warps.  bf16 rounding is round-to-nearest-even;
 * e4m3 ("fn", max 448) rounding is round-to-nearest-even with saturation.
 *
 * ROUND_INTERP reproduces Triton's CPU interpreter instead
 * (triton/runtime/interpreter.py): bf16 casts truncate, the e4m3 cast is the
 * interpreter's (e4m3_interp), tl.sum is numpy's pairwise float32 sum
 * (numpy_sum), and GELU uses separate multiply/add and libm expf.  In that
 * mode the oracle can be compared with golden vectors produced by running the
 * reference's own Triton kernels under TRITON_INTERPRET=1.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ROUND_RNE 0
#define ROUND_INTERP 1

/* ---------------------------------------------------------------- bits -- */

static float f_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t bits_from_f(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float orc_bf16_to_f32(uint16_t h) { return f_from_bits((uint32_t)h << 16); }

uint16_t orc_f32_to_bf16(float f, int mode) {
  uint32_t u = bits_from_f(f);
  if (isnan(f)) return (uint16_t)(((u >> 16) & 0x8000u) | 0x7fc0u);
  if (mode == ROUND_INTERP) return (uint16_t)(u >> 16);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static float rbf(float f, int mode) { return orc_bf16_to_f32(orc_f32_to_bf16(f, mode)); }

/* The interpreter's fp32 -> e4m3 cast (interpreter.py _convert_float with
 * RTNE): keep 3 mantissa bits, add the first dropped bit, OR the (possibly
 * carried) mantissa into the exponent field.  Outputs below 2^-9 are not
 * modelled (returned as signed zero); callers compare them loosely. */
static uint8_t e4m3_interp(float f) {
  const uint32_t u = bits_from_f(f), sign = u >> 31, e = (u >> 23) & 0xffu, sig = u & 0x7fffffu;
  if (e == 0 && sig == 0) return (uint8_t)(sign << 7);
  int eo = (int)e - 127 + 7;
  if (eo < 0) eo = 0;
  if (eo > 15) eo = 15;
  uint32_t so = ((sig >> 20) & 7u) + ((sig & (1u << 19)) ? 1u : 0u);
  if (eo == 0) {
    const int shift = 121 - (int)e;
    so = (shift >= 1 && shift <= 3) ? ((so >> shift) | (1u << (3 - shift))) : 0u;
  }
  return (uint8_t)((sign << 7) | ((uint32_t)eo << 3) | so);
}

/* e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa bits; 0x7f is NaN, max
 * finite 448 = 1.75 * 2^8, subnormals are multiples of 2^-9. */
uint8_t orc_f32_to_e4m3(float f, int mode) {
  if (mode == ROUND_INTERP) return e4m3_interp(f);
  if (isnan(f)) return 0x7f;
  const uint8_t sign = signbit(f) ? 0x80 : 0x00;
  float a = fabsf(f);
  if (a >= 448.0f) return sign | 0x7e;
  int e2;
  (void)frexpf(a, &e2); /* a in [2^(e2-1), 2^e2) */
  int E = e2 - 1;
  if (a == 0.0f || E < -6) { /* subnormal grid, step 2^-9 */
    float r = nearbyintf(a * 512.0f); /* a * 512 is exact */
    return sign | (uint8_t)r; /* r == 8 encodes 2^-6, the smallest normal */
  }
  float r = nearbyintf(ldexpf(a, 3 - E)); /* argument in [8, 16), exact */
  if (r == 16.0f) { r = 8.0f; E += 1; }
  if (E > 8 || (E == 8 && r > 14.0f)) return sign | 0x7e; /* satfinite */
  return sign | (uint8_t)(((E + 7) << 3) | ((int)r - 8));
}

float orc_e4m3_to_f32(uint8_t b) {
  const float sign = (b & 0x80) ? -1.0f : 1.0f;
  const int E = (b >> 3) & 0xf, m = b & 7;
  if (E == 0xf && m == 7) return NAN;
  if (E == 0) return sign * ldexpf((float)m, -9);
  return sign * ldexpf((float)(8 + m), E - 10);
}

/* -------------------------------------------------------- canonical sum -- */

/* Sum of x[0..n) (n a multiple of 8) in the canonical order: zero-pad to
 * NVp = max(P, pow2ceil(n/8)) vectors of 8; halve the vector count by adding
 * vector v + NVp/2 into vector v until P remain; reduce each remaining vector
 * by the same stride rule, ((x0+x4)+(x2+x6))+((x1+x5)+(x3+x7)); halve the P
 * partials the same way. */
float orc_canonical_sum(const float* x, int64_t n, int P) {
  int64_t nv = n / 8, nvp = P;
  while (nvp < nv) nvp <<= 1;
  float* X = (float*)calloc((size_t)(nvp * 8), sizeof(float));
  memcpy(X, x, (size_t)n * sizeof(float));
  while (nvp > P) {
    const int64_t half = nvp / 2;
    for (int64_t v = 0; v < half; ++v)
      for (int k = 0; k < 8; ++k) X[v * 8 + k] = X[v * 8 + k] + X[(v + half) * 8 + k];
    nvp = half;
  }
  float* p = (float*)malloc((size_t)P * sizeof(float));
  for (int v = 0; v < P; ++v) {
    const float* q = X + (int64_t)v * 8;
    p[v] = ((q[0] + q[4]) + (q[2] + q[6])) + ((q[1] + q[5]) + (q[3] + q[7]));
  }
  for (int w = P; w > 1; w /= 2)
    for (int v = 0; v < w / 2; ++v) p[v] = p[v] + p[v + w / 2];
  const float r = p[0];
  free(p);
  free(X);
  return r;
}

/* numpy's float32 add.reduce order (pairwise with 8 accumulators, blocks of
 * 128), the order tl.sum takes under the Triton interpreter. */
float orc_numpy_sum(const float* a, int64_t n) {
  if (n < 8) {
    float r = 0.0f;
    for (int64_t i = 0; i < n; ++i) r = r + a[i];
    return r;
  }
  if (n <= 128) {
    float r[8];
    for (int j = 0; j < 8; ++j) r[j] = a[j];
    int64_t i = 8;
    for (; i < n - (n % 8); i += 8)
      for (int j = 0; j < 8; ++j) r[j] = r[j] + a[i + j];
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res = res + a[i];
    return res;
  }
  int64_t n2 = n / 2;
  n2 -= n2 % 8;
  return orc_numpy_sum(a, n2) + orc_numpy_sum(a + n2, n - n2);
}

static float row_sum(const float* x, int64_t n, int P, int mode) {
  return (mode == ROUND_INTERP) ? orc_numpy_sum(x, n) : orc_canonical_sum(x, n, P);
}

/* --------------------------------------------------------------- AdaLN -- */

/* src/kernels/adaln.py:26-46 (bf16 output) and src/kernels/fp8.py:73-97 (FP8
 * output).  One row of D: z = bf16(res + bf16(gate*x)) (has_x) or z = res;
 * mean, rstd of z; y = (d*rstd)*scale + shift; h = bf16(y) or
 * s = max(max|y|, 1e-12)/448, q = e4m3(clamp(y/s, +-448)). */
void orc_adaln_fwd(const uint16_t* x, const uint16_t* res, const uint16_t* gate,
                   const uint16_t* shift, const uint16_t* scale, uint16_t* h, uint16_t* z,
                   uint8_t* q, float* s, int64_t B, int64_t S, int64_t D, float eps, int has_x,
                   int fp8, int mode) {
  float* zf = (float*)malloc((size_t)D * sizeof(float));
  float* t = (float*)malloc((size_t)D * sizeof(float));
  float* y = (float*)malloc((size_t)D * sizeof(float));
  for (int64_t row = 0; row < B * S; ++row) {
    const int64_t b = row / S, o = row * D, po = b * D;
    for (int64_t i = 0; i < D; ++i) {
      const float r = orc_bf16_to_f32(res[o + i]);
      if (has_x) {
        const float p = rbf(orc_bf16_to_f32(gate[po + i]) * orc_bf16_to_f32(x[o + i]), mode);
        const uint16_t zb = orc_f32_to_bf16(r + p, mode);
        if (z) z[o + i] = zb;
        zf[i] = orc_bf16_to_f32(zb);
      } else {
        zf[i] = r;
      }
    }
    const float mean = row_sum(zf, D, 32, mode) / (float)D;
    for (int64_t i = 0; i < D; ++i) {
      const float d = zf[i] - mean;
      t[i] = d * d;
    }
    const float var = row_sum(t, D, 32, mode) / (float)D;
    const float rstd = 1.0f / sqrtf(var + eps);
    float amax = 0.0f;
    for (int64_t i = 0; i < D; ++i) {
      const float d = zf[i] - mean;
      y[i] = ((d * rstd) * orc_bf16_to_f32(scale[po + i])) + orc_bf16_to_f32(shift[po + i]);
      amax = fmaxf(amax, fabsf(y[i]));
    }
    if (!fp8) {
      for (int64_t i = 0; i < D; ++i) h[o + i] = orc_f32_to_bf16(y[i], mode);
    } else {
      const float sc = fmaxf(amax, 1e-12f) / 448.0f;
      s[row] = sc;
      for (int64_t i = 0; i < D; ++i)
        q[o + i] = orc_f32_to_e4m3(fminf(fmaxf(y[i] / sc, -448.0f), 448.0f), mode);
    }
  }
  free(zf);
  free(t);
  free(y);
}

/* ---------------------------------------------------------------- GELU -- */

/* exp(a), a <= 0: Cody-Waite reduction a = k ln2 + r (ln2 split in two parts),
 * degree-7 Taylor polynomial of exp(r) in Horner form with fmaf, times 2^k;
 * results below 2^-126 are scaled in two exact steps so that only the last
 * multiplication rounds. */
float orc_exp_nonpos(float a) {
  if (a < -104.0f) return 0.0f;
  const float k = rintf(a * 1.44269502162933349609375f);
  float r = fmaf(k, -0.693145751953125f, a);
  r = fmaf(k, -1.428606765330187e-06f, r);
  float p = 1.98412701138295233249664306640625e-04f; /* 1/7! */
  p = fmaf(p, r, 1.38888892251998186111450195312500e-03f); /* 1/6! */
  p = fmaf(p, r, 8.33333376795053482055664062500000e-03f); /* 1/5! */
  p = fmaf(p, r, 4.16666679084300994873046875000000e-02f); /* 1/4! */
  p = fmaf(p, r, 1.66666671633720397949218750000000e-01f); /* 1/3! */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ki = (int)k;
  if (ki >= -125) return p * ldexpf(1.0f, ki);
  return (p * ldexpf(1.0f, ki + 64)) * ldexpf(1.0f, -64);
}

/* exp(a) for every fp32 a: the reduction and polynomial of orc_exp_nonpos
 * (identical for a <= 0), two-step scaling above 2^127, overflow to infinity
 * beyond exp's range, NaN propagated.  Mirrors canonical_exp of the device. */
float orc_exp(float a) {
  if (a != a) return a + a;
  if (a < -104.0f) return 0.0f;
  if (a > 88.8f) return INFINITY;
  const float k = rintf(a * 1.44269502162933349609375f);
  float r = fmaf(k, -0.693145751953125f, a);
  r = fmaf(k, -1.428606765330187e-06f, r);
  float p = 1.98412701138295233249664306640625e-04f;
  p = fmaf(p, r, 1.38888892251998186111450195312500e-03f);
  p = fmaf(p, r, 8.33333376795053482055664062500000e-03f);
  p = fmaf(p, r, 4.16666679084300994873046875000000e-02f);
  p = fmaf(p, r, 1.66666671633720397949218750000000e-01f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ki = (int)k;
  if (ki > 127) return (p * ldexpf(1.0f, 64)) * ldexpf(1.0f, ki - 64);
  if (ki >= -125) return p * ldexpf(1.0f, ki);
  return (p * ldexpf(1.0f, ki + 64)) * ldexpf(1.0f, -64);
}

static void stride_tree_rows(const float* rows, int64_t n, int64_t cols, float* out);

/* Channel RMS norm + SiLU of the VAE (src/kernels/rms.py:20-123).  Rows are
 * pixels of C channels (channels last).  Lanes per row in the canonical
 * order: LPR = the smallest power of two with at most four 8-element vectors
 * per lane, at most 32; row sums are canonical sums with P = LPR. */
int orc_rms_lpr(int64_t C) {
  const int64_t nv = C / 8;
  int lpr = 1;
  while (lpr < 32 && (int64_t)lpr * 4 < nv) lpr <<= 1;
  return lpr;
}

/* Source offset of output row `row` (rms.py:20-32): with `shuf`, output pixel
 * (b, y, x) of an [B, H, W, C] grid reads the sub-pixel channels of
 * u[b, y/2, x/2, ((y%2)*2 + x%2)*C + c]. */
static int64_t rms_src(int64_t row, int64_t H, int64_t W, int64_t C, int shuf) {
  if (!shuf) return row * C;
  const int64_t hw = H * W, b = row / hw, rem = row - b * hw, y = rem / W, x = rem - y * W;
  return (((b * (H / 2) + y / 2) * (W / 2) + x / 2) * 4 + (y % 2) * 2 + x % 2) * C;
}

static float rms_sigmoid(float a, int mode) {
  const float e = mode == ROUND_INTERP ? expf(-a) : orc_exp(-a);
  return 1.0f / (1.0f + e);
}

/* Forward (rms.py:35-73): s = bf16(x + r) with r, the gathered x with shuf,
 * else x; rstd = sqrt(C) / max(sqrt(sum(s^2)), 1e-12); a = (s * rstd) * g;
 * y = bf16(a * sigmoid(a)).  s_out (when given) receives s. */
void orc_rms_silu_fwd(const uint16_t* x, const uint16_t* r, const float* g, uint16_t* s_out,
                      uint16_t* y, int64_t N, int64_t H, int64_t W, int64_t C, int shuf, int mode) {
  float* sv = (float*)malloc((size_t)C * sizeof(float));
  float* t = (float*)malloc((size_t)C * sizeof(float));
  const int P = orc_rms_lpr(C);
  const float sqrt_c = (float)sqrt((double)C);
  for (int64_t row = 0; row < N; ++row) {
    const int64_t src = rms_src(row, H, W, C, shuf), dst = row * C;
    for (int64_t c = 0; c < C; ++c) {
      float v = orc_bf16_to_f32(x[src + c]);
      if (r) v = orc_bf16_to_f32(orc_f32_to_bf16(v + orc_bf16_to_f32(r[dst + c]), mode));
      sv[c] = v;
      if (s_out) s_out[dst + c] = orc_f32_to_bf16(v, mode);
      t[c] = v * v;
    }
    const float ss = mode == ROUND_INTERP ? orc_numpy_sum(t, C) : orc_canonical_sum(t, C, P);
    const float nrm = sqrtf(ss);
    const float rstd = sqrt_c / (nrm > 1e-12f ? nrm : 1e-12f);
    for (int64_t c = 0; c < C; ++c) {
      const float a = (sv[c] * rstd) * g[c];
      y[dst + c] = orc_f32_to_bf16(a * rms_sigmoid(a, mode), mode);
    }
  }
  free(sv);
  free(t);
}

/* Backward (rms.py:76-125): per row, rstd of s as the forward; n = s * rstd;
 * a = n * g; sg = sigmoid(a); da = (dy * sg) * (1 + a * (1 - sg));
 * dn = da * g; ds = rstd * (dn - n * (sum(dn * n) / C)) (+ gs), stored at the
 * source offset; dg = sum over rows of da * n.  dg order: chunks of TPC tiles
 * of T = 32/P rows (TPC = 8, doubled until at most 32768 chunks remain);
 * within a chunk each row group (row index mod T) sums its rows in order
 * from zero, the T group sums go through a stride tree, the chunk partials
 * through a stride tree. */
int orc_rms_tiles_per_chunk(int64_t N, int64_t C) {
  const int64_t T = 32 / orc_rms_lpr(C);
  int tpc = 8;
  while ((N + tpc * T - 1) / (tpc * T) > 32768) tpc <<= 1;
  return tpc;
}


void orc_rms_silu_bwd(const uint16_t* s, const float* g, const uint16_t* dy, const uint16_t* gs,
                      uint16_t* ds, float* dg, int64_t N, int64_t H, int64_t W, int64_t C, int shuf,
                      int mode) {
  const int P = orc_rms_lpr(C);
  const int T = 32 / P;                      /* rows per tile */
  const int tpc = orc_rms_tiles_per_chunk(N, C);
  const int64_t chunk_rows = (int64_t)T * tpc;
  const int64_t chunks = (N + chunk_rows - 1) / chunk_rows;
  const float sqrt_c = (float)sqrt((double)C);
  float* n = (float*)malloc((size_t)C * sizeof(float));
  float* da = (float*)malloc((size_t)C * sizeof(float));
  float* t = (float*)malloc((size_t)C * sizeof(float));
  float* tile = (float*)malloc((size_t)T * C * sizeof(float));
  float* cs = (float*)malloc((size_t)(chunks > 0 ? chunks : 1) * C * sizeof(float));
  for (int64_t ch = 0; ch < chunks; ++ch) {
    for (int64_t i = 0; i < (int64_t)T * C; ++i) tile[i] = 0.0f; /* row-group sums */
    for (int tl = 0; tl < tpc; ++tl) {
      for (int k = 0; k < T; ++k) {
        const int64_t row = ch * chunk_rows + (int64_t)tl * T + k;
        if (row >= N) continue;
        const int64_t dst = row * C;
        for (int64_t c = 0; c < C; ++c) {
          const float v = orc_bf16_to_f32(s[dst + c]);
          t[c] = v * v;
        }
        const float ss = mode == ROUND_INTERP ? orc_numpy_sum(t, C) : orc_canonical_sum(t, C, P);
        const float nrm = sqrtf(ss);
        const float rstd = sqrt_c / (nrm > 1e-12f ? nrm : 1e-12f);
        for (int64_t c = 0; c < C; ++c) {
          n[c] = orc_bf16_to_f32(s[dst + c]) * rstd;
          const float a = n[c] * g[c];
          const float sg = rms_sigmoid(a, mode);
          da[c] = (orc_bf16_to_f32(dy[dst + c]) * sg) * (1.0f + a * (1.0f - sg));
          tile[(int64_t)k * C + c] = tile[(int64_t)k * C + c] + da[c] * n[c];
          t[c] = (da[c] * g[c]) * n[c];
        }
        const float sdn = mode == ROUND_INTERP ? orc_numpy_sum(t, C) : orc_canonical_sum(t, C, P);
        const float m = sdn / (float)C;
        const int64_t src = rms_src(row, H, W, C, shuf);
        for (int64_t c = 0; c < C; ++c) {
          float v = rstd * (da[c] * g[c] - n[c] * m);
          if (gs) v = v + orc_bf16_to_f32(gs[dst + c]);
          ds[src + c] = orc_f32_to_bf16(v, mode);
        }
      }
    }
    for (int w = T; w > 1; w /= 2) /* stride tree over the row groups */
      for (int k = 0; k < w / 2; ++k)
        for (int64_t c = 0; c < C; ++c) tile[(int64_t)k * C + c] = tile[(int64_t)k * C + c] + tile[(int64_t)(k + w / 2) * C + c];
    for (int64_t c = 0; c < C; ++c) cs[ch * C + c] = tile[c];
  }
  stride_tree_rows(cs, chunks, C, dg);
  free(n); free(da); free(t); free(tile); free(cs);
}

/* src/kernels/ctx_scale.py:8-37 and :61-100.  Per token s of batch b and head
 * h: gain = 1 / (1 + exp(ln_pad[b] - lse[b,h,s])); y = bf16(x * gain).
 * Backward: dout = bf16(dy * gain); dlse = (sum(dy * x) * gain) * (1 - gain),
 * the sum over the head's hd elements in canonical order (P = hd/8), or the
 * numpy order in INTERP mode.  out/dy/y/dout [B,S,H,hd] bf16, lse/dlse
 * [B,H,S] fp32, ln_pad [B] fp32.  In INTERP mode exp is the C library's expf,
 * standing in for the interpreter's numpy exp (last-bit differences remain). */
void orc_ctx_scale(const uint16_t* out, const float* lse, const float* ln_pad, const uint16_t* dy,
                   uint16_t* y, uint16_t* dout, float* dlse, int64_t B, int64_t S, int64_t H,
                   int64_t hd, int mode) {
  float* t = (float*)malloc((size_t)hd * sizeof(float));
  for (int64_t b = 0; b < B; ++b)
    for (int64_t s = 0; s < S; ++s)
      for (int64_t h = 0; h < H; ++h) {
        const int64_t li = (b * H + h) * S + s;
        const float a = ln_pad[b] - lse[li];
        const float e = mode == ROUND_INTERP ? expf(a) : orc_exp(a);
        const float gain = 1.0f / (1.0f + e);
        const int64_t o = ((b * S + s) * H + h) * hd;
        for (int64_t i = 0; i < hd; ++i) {
          const float x = orc_bf16_to_f32(out[o + i]);
          if (y) y[o + i] = orc_f32_to_bf16(x * gain, mode);
          if (dy) {
            const float g = orc_bf16_to_f32(dy[o + i]);
            dout[o + i] = orc_f32_to_bf16(g * gain, mode);
            t[i] = g * x;
          }
        }
        if (dy) {
          const float sum = mode == ROUND_INTERP ? orc_numpy_sum(t, hd) : orc_canonical_sum(t, hd, (int)(hd / 8));
          dlse[li] = (sum * gain) * (1.0f - gain);
        }
      }
  free(t);
}

/* GELU with the Abramowitz & Stegun 7.1.26 erf (src/kernels/fp8.py:260-270),
 * Horner steps as fmaf. */
float orc_gelu(float x) {
  const float z = x * 0.707106769084930419921875f;
  const float az = fabsf(z);
  const float t = 1.0f / (1.0f + 0.3275911f * az);
  float p = fmaf(1.061405429f, t, -1.453152027f);
  p = fmaf(p, t, 1.421413741f);
  p = fmaf(p, t, -0.284496736f);
  p = fmaf(p, t, 0.254829592f);
  p = p * t;
  const float e = orc_exp_nonpos(-(az * az));
  const float yv = fmaf(-p, e, 1.0f);
  const float erf = (z < 0.0f) ? -yv : yv;
  return (0.5f * x) * (1.0f + erf);
}

/* The same formula as the interpreter evaluates it: no fused multiply-add,
 * libm expf (the interpreter calls numpy's exp, which may differ in the last
 * bit). */
static float gelu_interp(float x) {
  const float z = x * 0.707106769084930419921875f;
  const float az = fabsf(z);
  const float t = 1.0f / (1.0f + 0.3275911f * az);
  const float p =
      ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t +
       0.254829592f) * t;
  const float yv = 1.0f - p * expf(-az * az);
  return 0.5f * x * (1.0f + ((z < 0.0f) ? -yv : yv));
}

static float gelu_mode(float x, int mode) { return mode == ROUND_INTERP ? gelu_interp(x) : orc_gelu(x); }

void orc_gelu_many(const uint16_t* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = orc_gelu(orc_bf16_to_f32(x[i]));
}

/* src/kernels/fp8.py:283-292: y = gelu(x) or x; s = max(max|y|,1e-12)/448;
 * q = e4m3(clamp(y/s, +-448)).  `y_out` (optional) receives y. */
void orc_rowquant(const uint16_t* x, uint8_t* q, float* s, float* y_out, int64_t rows, int64_t K,
                  int gelu, int mode) {
  float* y = (float*)malloc((size_t)K * sizeof(float));
  for (int64_t row = 0; row < rows; ++row) {
    float amax = 0.0f;
    for (int64_t i = 0; i < K; ++i) {
      const float v = orc_bf16_to_f32(x[row * K + i]);
      y[i] = gelu ? gelu_mode(v, mode) : v;
      amax = fmaxf(amax, fabsf(y[i]));
    }
    const float sc = fmaxf(amax, 1e-12f) / 448.0f;
    s[row] = sc;
    for (int64_t i = 0; i < K; ++i) {
      q[row * K + i] = orc_f32_to_e4m3(fminf(fmaxf(y[i] / sc, -448.0f), 448.0f), mode);
      if (y_out) y_out[row * K + i] = y[i];
    }
  }
  free(y);
}

/* -------------------------------------------------- q/k RMSNorm + RoPE -- */

/* One head (src/kernels/rope.py:39-58): rstd over hd dims (canonical sum with
 * P = hd/8 partials), a/b = bf16((x*rstd)*w), then optionally
 * a' = a*cos - b*sin, b' = b*cos + a*sin. */
static void head_fwd(const uint16_t* src, uint16_t* dst, const float* w, const float* cs,
                     const float* sn, int hd, float eps, int rotate, int mode, float* buf) {
  const int half = hd / 2;
  for (int i = 0; i < hd; ++i) {
    const float v = orc_bf16_to_f32(src[i]);
    buf[i] = v * v;
  }
  const float ss = (mode == ROUND_INTERP)
                       ? orc_numpy_sum(buf, half) + orc_numpy_sum(buf + half, half)
                       : orc_canonical_sum(buf, hd, hd / 8);
  const float rstd = 1.0f / sqrtf(ss / (float)hd + eps);
  for (int i = 0; i < hd; ++i) buf[i] = rbf((orc_bf16_to_f32(src[i]) * rstd) * w[i], mode);
  for (int i = 0; i < hd; ++i) {
    float o = buf[i];
    if (rotate) {
      const int j = i % half;
      o = (i < half) ? (buf[i] * cs[j]) - (buf[i + half] * sn[j])
                     : (buf[i] * cs[j]) + (buf[i - half] * sn[j]);
    }
    dst[i] = orc_f32_to_bf16(o, mode);
  }
}

/* src/kernels/rope.py:61-143.  qkv [B,S,3,H,hd]; q, k (and v if non-null)
 * [B,S,H,hd]; cos, sin [S, hd/2]; position = token % S. */
void orc_qkv_norm_rope(const uint16_t* qkv, const float* qw, const float* kw, const float* cs,
                       const float* sn, uint16_t* q, uint16_t* k, uint16_t* v, int64_t B,
                       int64_t S, int64_t H, int64_t hd, float eps, int mode) {
  float* buf = (float*)malloc((size_t)hd * sizeof(float));
  const int64_t width = H * hd;
  for (int64_t tok = 0; tok < B * S; ++tok) {
    const int64_t pos = tok % S;
    const uint16_t* row = qkv + tok * 3 * width;
    for (int64_t h = 0; h < H; ++h) {
      head_fwd(row + h * hd, q + tok * width + h * hd, qw, cs + pos * hd / 2, sn + pos * hd / 2,
               (int)hd, eps, 1, mode, buf);
      head_fwd(row + width + h * hd, k + tok * width + h * hd, kw, cs + pos * hd / 2,
               sn + pos * hd / 2, (int)hd, eps, 1, mode, buf);
    }
    if (v) memcpy(v + tok * width, row + 2 * width, (size_t)width * sizeof(uint16_t));
  }
  free(buf);
}

/* src/kernels/rope.py:146-172.  x [B,S,H*hd] -> y [B,S,H,hd]. */
void orc_head_norm(const uint16_t* x, const float* w, uint16_t* y, int64_t B, int64_t S,
                   int64_t H, int64_t hd, float eps, int mode) {
  float* buf = (float*)malloc((size_t)hd * sizeof(float));
  for (int64_t tok = 0; tok < B * S; ++tok)
    for (int64_t h = 0; h < H; ++h)
      head_fwd(x + (tok * H + h) * hd, y + (tok * H + h) * hd, w, NULL, NULL, (int)hd, eps, 0,
               mode, buf);
  free(buf);
}

/* ------------------------------------------------------------ backward -- */

/* Stride tree over n rows of `cols` floats (rows zero-padded to a power of
 * two); the result is written to out[0..cols). */
static void stride_tree_rows(const float* rows, int64_t n, int64_t cols, float* out) {
  int64_t np = 1;
  while (np < n) np <<= 1;
  float* t = (float*)calloc((size_t)(np * cols), sizeof(float));
  memcpy(t, rows, (size_t)(n * cols) * sizeof(float));
  for (int64_t h = np / 2; h >= 1; h /= 2)
    for (int64_t v = 0; v < h; ++v)
      for (int64_t c = 0; c < cols; ++c) t[v * cols + c] = t[v * cols + c] + t[(v + h) * cols + c];
  memcpy(out, t, (size_t)cols * sizeof(float));
  free(t);
}
/* src/kernels/adaln.py:133-217.  Per row: mean, rstd of z; xhat = d*rstd;
 * dxh = gh*scale; c1 = sum(dxh)/D; c2 = sum(dxh*xhat)/D, which the canonical
 * (RNE) mode forms as (sum(dxh*d) * rstd) / D: the same value up to
 * rounding, with a sum that needs only the mean, so the device computes it
 * together with the variance (INTERP mode keeps the reference's form);
 * dz = rstd*((dxh - c1) - xhat*c2) (+ gz) -> bf16; dx = bf16(dz*gate).
 * Parameter gradients (dshift = sum gh, dscale = sum gh*xhat,
 * dgate = sum dz*x) in the canonical order of the CUDA kernel: chunks of
 * `warps * rows_per_warp` rows; in a chunk warp w sums rows w, w+warps, ...;
 * the warp sums combine as a stride tree over warps (pairs w, w + warps/2
 * first), and the chunk sums combine by a stride tree over the chunk index
 * (zero-padded to a power of two); then bf16.  In INTERP mode the per-row
 * sums are numpy's; the parameter gradients keep the canonical order. */

void orc_adaln_bwd(const uint16_t* gh, const uint16_t* gz, const uint16_t* z, const uint16_t* x,
                   const uint16_t* gate, const uint16_t* scale, uint16_t* dz_out,
                   uint16_t* dx_out, uint16_t* dgate, uint16_t* dshift, uint16_t* dscale,
                   int64_t B, int64_t S, int64_t D, float eps, int warps, int rows_per_warp,
                   int mode) {
  const int has_x = x != NULL, nq = has_x ? 3 : 2;
  const int64_t chunk_rows = (int64_t)warps * rows_per_warp;
  const int64_t chunks = (S + chunk_rows - 1) / chunk_rows;
  float* zf = (float*)malloc((size_t)D * sizeof(float));
  float* t1 = (float*)malloc((size_t)D * sizeof(float));
  float* t2 = (float*)malloc((size_t)D * sizeof(float));
  float* wp = (float*)malloc((size_t)warps * nq * D * sizeof(float)); /* warp partials */
  float* cs = (float*)malloc((size_t)chunks * nq * D * sizeof(float)); /* chunk sums */
  float* tot = (float*)malloc((size_t)nq * D * sizeof(float));
  for (int64_t b = 0; b < B; ++b) {
    const int64_t po = b * D;
    for (int64_t c = 0; c < chunks; ++c) {
      for (int64_t i = 0; i < (int64_t)warps * nq * D; ++i) wp[i] = 0.0f;
      for (int r = 0; r < rows_per_warp; ++r) {
        for (int w = 0; w < warps; ++w) {
          const int64_t s = c * chunk_rows + (int64_t)r * warps + w;
          if (s >= S) continue;
          const int64_t o = (b * S + s) * D;
          for (int64_t i = 0; i < D; ++i) zf[i] = orc_bf16_to_f32(z[o + i]);
          const float mean = row_sum(zf, D, 32, mode) / (float)D;
          for (int64_t i = 0; i < D; ++i) {
            const float d = zf[i] - mean;
            t1[i] = d * d;
          }
          const float rstd = 1.0f / sqrtf(row_sum(t1, D, 32, mode) / (float)D + eps);
          for (int64_t i = 0; i < D; ++i) {
            const float xhat = (zf[i] - mean) * rstd;
            const float dxh = orc_bf16_to_f32(gh[o + i]) * orc_bf16_to_f32(scale[po + i]);
            t1[i] = dxh;
            t2[i] = mode == ROUND_INTERP ? dxh * xhat : dxh * (zf[i] - mean);
          }
          const float c1 = row_sum(t1, D, 32, mode) / (float)D;
          const float c2 = mode == ROUND_INTERP ? row_sum(t2, D, 32, mode) / (float)D
                                                : (row_sum(t2, D, 32, mode) * rstd) / (float)D;
          float* p = wp + (int64_t)w * nq * D;
          for (int64_t i = 0; i < D; ++i) {
            const float g = orc_bf16_to_f32(gh[o + i]);
            const float xhat = (zf[i] - mean) * rstd;
            const float dxh = g * orc_bf16_to_f32(scale[po + i]);
            float dz = rstd * ((dxh - c1) - xhat * c2);
            if (gz) dz = dz + orc_bf16_to_f32(gz[o + i]);
            dz_out[o + i] = orc_f32_to_bf16(dz, mode);
            p[i] = p[i] + g;
            p[D + i] = p[D + i] + g * xhat;
            if (has_x) {
              dx_out[o + i] = orc_f32_to_bf16(dz * orc_bf16_to_f32(gate[po + i]), mode);
              p[2 * D + i] = p[2 * D + i] + dz * orc_bf16_to_f32(x[o + i]);
            }
          }
        }
      }
      for (int span = warps; span > 1; span /= 2) /* stride tree over warps */
        for (int w = 0; w < span / 2; ++w)
          for (int64_t i = 0; i < nq * D; ++i)
            wp[(int64_t)w * nq * D + i] = wp[(int64_t)w * nq * D + i] + wp[(int64_t)(w + span / 2) * nq * D + i];
      memcpy(cs + c * nq * D, wp, (size_t)(nq * D) * sizeof(float));
    }
    stride_tree_rows(cs, chunks, nq * D, tot);
    for (int64_t i = 0; i < D; ++i) {
      dshift[po + i] = orc_f32_to_bf16(tot[i], ROUND_RNE);
      dscale[po + i] = orc_f32_to_bf16(tot[D + i], ROUND_RNE);
      if (has_x) dgate[po + i] = orc_f32_to_bf16(tot[2 * D + i], ROUND_RNE);
    }
  }
  free(zf); free(t1); free(t2); free(wp); free(cs); free(tot);
}

/* src/kernels/rope.py:223-383, :386-436.  Per token and head: undo the
 * rotation of the upstream gradient (da' = da*cos + db*sin,
 * db' = db*cos - da*sin), rstd of the forward input, xhat = x*rstd,
 * u = d'*w, c = sum(u*xhat)/hd, dx = bf16(rstd*(u - xhat*c)); dw += d'*xhat.
 * The canonical (RNE) mode forms c as (sum(u*x) * rstd)/hd: the same value
 * up to rounding, from a sum that needs no rstd, so the device reduces it
 * together with sum(x*x) (INTERP mode keeps the reference's form).
 * Weight-gradient order as the CUDA kernel: tokens in chunks of `warps`;
 * per token, lane group g (hpi = 32 / (hd/16) groups) sums heads
 * g, g + hpi, ... in increasing order from zero and the groups combine as a
 * stride tree; the token sums of a chunk combine as a stride tree over the
 * token index; the chunk sums as a stride tree over the chunk index.
 * src/dsrc rows are src_row wide with the normed sections at q_off/k_off
 * (nsec = 1 or 2) and, when dv is given, v at v_off. */
void orc_headnorm_bwd(const uint16_t* src, int64_t src_row, int64_t q_off, int64_t k_off,
                      int64_t v_off, const uint16_t* dq, const uint16_t* dk, const uint16_t* dv,
                      const float* wq, const float* wk, const float* cs, const float* sn,
                      uint16_t* dsrc, float* dw0, float* dw1, int64_t tokens, int64_t S,
                      int64_t H, int64_t hd, float eps, int rotate, int nsec, int warps,
                      int tok_per_warp, int mode) {
  (void)tok_per_warp;
  const int64_t half = hd / 2, hpi = 32 / (hd / 16);
  const int64_t chunks = (tokens + warps - 1) / warps;
  const int64_t ns = 2 * hd; /* per-token sums, both sections */
  float* x = (float*)malloc((size_t)hd * sizeof(float));
  float* d = (float*)malloc((size_t)hd * sizeof(float));
  float* t = (float*)malloc((size_t)hd * sizeof(float));
  float* grp = (float*)malloc((size_t)(hpi * ns) * sizeof(float));
  float* tokp = (float*)malloc((size_t)(warps * ns) * sizeof(float));
  float* chunkp = (float*)calloc((size_t)((chunks > 0 ? chunks : 1) * ns), sizeof(float));
  for (int64_t c = 0; c < chunks; ++c) {
    for (int w = 0; w < warps; ++w) {
      const int64_t tok = c * warps + w;
      for (int64_t i = 0; i < hpi * ns; ++i) grp[i] = 0.0f;
      if (tok < tokens) {
        const int64_t pos = tok % S;
        for (int sec = 0; sec < nsec; ++sec) {
          const uint16_t* in = src + tok * src_row + (sec ? k_off : q_off);
          uint16_t* out = dsrc + tok * src_row + (sec ? k_off : q_off);
          const uint16_t* go = (sec ? dk : dq) + tok * H * hd;
          const float* wv = sec ? wk : wq;
          for (int64_t h = 0; h < H; ++h) {
            float* acc = grp + (h % hpi) * ns + sec * hd;
            for (int64_t i = 0; i < hd; ++i) {
              x[i] = orc_bf16_to_f32(in[h * hd + i]);
              d[i] = orc_bf16_to_f32(go[h * hd + i]);
            }
            if (rotate)
              for (int64_t i = 0; i < half; ++i) {
                const float c0 = cs[pos * half + i], s0 = sn[pos * half + i];
                const float da = d[i], db = d[i + half];
                d[i] = (da * c0) + (db * s0);
                d[i + half] = (db * c0) - (da * s0);
              }
            for (int64_t i = 0; i < hd; ++i) t[i] = x[i] * x[i];
            const float ss = (mode == ROUND_INTERP)
                                 ? orc_numpy_sum(t, half) + orc_numpy_sum(t + half, half)
                                 : orc_canonical_sum(t, hd, (int)(hd / 8));
            const float rstd = 1.0f / sqrtf(ss / (float)hd + eps);
            float cc;
            if (mode == ROUND_INTERP) {
              for (int64_t i = 0; i < hd; ++i) t[i] = (d[i] * wv[i]) * (x[i] * rstd);
              cc = (orc_numpy_sum(t, half) + orc_numpy_sum(t + half, half)) / (float)hd;
            } else {
              for (int64_t i = 0; i < hd; ++i) t[i] = (d[i] * wv[i]) * x[i];
              cc = (orc_canonical_sum(t, hd, (int)(hd / 8)) * rstd) / (float)hd;
            }
            for (int64_t i = 0; i < hd; ++i) {
              const float xh = x[i] * rstd, u = d[i] * wv[i];
              out[h * hd + i] = orc_f32_to_bf16(rstd * (u - xh * cc), mode);
              acc[i] = acc[i] + d[i] * xh;
            }
          }
        }
        if (dv) memcpy(dsrc + tok * src_row + v_off, dv + tok * H * hd, (size_t)(H * hd) * 2);
      }
      stride_tree_rows(grp, hpi, ns, tokp + (int64_t)w * ns); /* over the lane groups */
    }
    stride_tree_rows(tokp, warps, ns, chunkp + c * ns); /* over the tokens of the chunk */
  }
  float tot[512];
  stride_tree_rows(chunkp, chunks > 0 ? chunks : 1, ns, tot); /* over the chunks */
  for (int64_t i = 0; i < hd; ++i) {
    dw0[i] = tot[i];
    if (nsec > 1) dw1[i] = tot[hd + i];
  }
  free(x); free(d); free(t); free(grp); free(tokp); free(chunkp);
}
