// Per-row FP8 e4m3 quantisation, optionally after GELU.
//
// Reference: src/kernels/fp8.py:273-292 (_rowquant_kernel) and :260-270
// (_gelu, Abramowitz & Stegun 7.1.26).  Per row of K elements:
//   y = gelu(x) if GELU else x                     (fp32)
//   s = max(max|y|, 1e-12) / 448;  q = e4m3(clamp(y / s, +-448))
//
// Layout: a group of GROUP warps owns a row (GROUP a power of two, 1..16,
// chosen so that a thread holds at most two chunks); thread t of the group
// holds the 16-element chunks ch = t + 32*GROUP*c (c < CPL), i.e. two 16-byte
// loads and one 16-byte FP8 store per chunk.  A block is max(GROUP, 4) warps
// (one or more rows).  The group's maxima are exchanged through shared memory
// with one barrier each.  The amax is a max, so the order of the reduction
// does not matter.
//
// Without GELU the codes and scales are exact: the codes come from products
// of y by RN(1/s) (1 -+ 2^-22) where they provably bracket the IEEE quotient,
// and from the IEEE division elsewhere (e4m3_quot8).  With GELU the
// per-element work would make the kernel compute-bound, so the codes use
// fast_gelu() and y * (1 / s); the scale stays
// exact: every element whose fast value lies within the fast_gelu error bound
// of the row's fast amax is recomputed with canonical_gelu() and the exact
// amax is the max over those candidates.  The codes can then differ from the
// canonical ones only where y / s lies within a few fp32 ulps of an e4m3
// rounding tie.
//
// CTX (the trimmed cross-attention's output path, src/model.py:457 with
// src/attention.py:180): rowquant(ctx_scale(out, lse, ln_pad)) in one pass.
// A row is one token's H * hd attention outputs; a 16-element chunk lies in
// one head h, whose gain ctx_gain(ln_pad[b], lse[b, h, s]) scales it, and the
// product is rounded to bf16 exactly as ctx_scale stores it.  The quantisation
// of those bf16 values is the exact non-GELU path, so the codes and scales are
// those of the two ops run one after the other, without writing and reading
// back the bf16 intermediate.
#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

// Out of line: the candidate branch is rare and the row loop is unrolled.
__device__ __noinline__ float canonical_gelu_call(float x) { return canonical_gelu(x); }

struct RowquantArgs {
  const uint16_t* x;  // [rows, K] bf16
  uint8_t* q;         // [rows, K] e4m3
  float* s;           // [rows] fp32
  int64_t rows;
  int K;
  // CTX only: x is out [B, S, H, hd] (rows = B*S, K = H*hd)
  const float* lse;     // [B, H, S]
  const float* ln_pad;  // [B]
  int64_t seq;
  DivU32 seqd;          // division by seq
  int heads;
  int hd_shift;         // log2(hd)
};

__host__ __device__ constexpr int rowquant_block_warps(int group) { return group > 4 ? group : 4; }

// The GELU kernel at K = 8192 (8 warps a row) asks for five CTAs per SM: 48
// registers without spills, 40 warps per SM to cover the row's barrier
// waits and SFU latency (measured 52.4 against 56.6 us with four CTAs of 64
// registers; six CTAs spill and take 55.3).
template <int CPL, int GROUP, bool GELU, bool CTX = false>
__global__ void __launch_bounds__(rowquant_block_warps(GROUP) * 32, (GELU && GROUP == 8) ? 5 : 1)
rowquant_kernel(const RowquantArgs a) {
  constexpr int BW = rowquant_block_warps(GROUP);
  __shared__ float red[2][BW];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int t = (warp % GROUP) * 32 + lane;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (BW / GROUP) + warp / GROUP;
  const bool row_ok = row < a.rows;
  const int K = a.K;
  const int64_t base = (row_ok ? row : 0) * K;

  // y as fp32 pairs: y2[c][j] holds elements (2j, 2j+1) of chunk c.
  f2_t y2[CPL][8];
  float amax = 0.0f;
  {
    uint4 xv[CPL][2];
    float lse[CPL], lnp = 0.0f;
    int64_t bb = 0, ss = 0;
    if (CTX && row_ok) {
      bb = div_u32(a.seqd, row);
      ss = row - bb * a.seq;
      lnp = __ldg(a.ln_pad + bb);
    }
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      const int e = (t + 32 * GROUP * c) * 16;
      const bool ok = row_ok && e < K;
      xv[c][0] = ok ? ld_stream(a.x + base + e) : make_uint4(0, 0, 0, 0);
      xv[c][1] = ok ? ld_stream(a.x + base + e + 8) : make_uint4(0, 0, 0, 0);
      if (CTX) lse[c] = ok ? __ldg(a.lse + (bb * a.heads + (e >> a.hd_shift)) * a.seq + ss) : 0.0f;
    }
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      // CTX: y = bf16(x * gain), ctx_scale's product and rounding (products only: packed)
      const f2_t g2 = splat2(CTX ? ctx_gain(lnp, lse[c]) : 1.0f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        f2_t v = bf2f2(word(xv[c][j >> 2], j & 3));
        if (CTX) v = bf2f2(f2bf2(mul2(v, g2)));
        y2[c][j] = GELU ? fast_gelu2(v) : v;
        amax = max_abs2(amax, f2lo(y2[c][j]), f2hi(y2[c][j]));
      }
    }
  }
  const float lamax = amax;

  // Group-wide max through red[buf].  Padding elements are zero and leave the
  // max unchanged.  The two exchanges of a row use different buffers.
  auto group_max = [&](float v, int buf) {
    v = warp_max(v);
    if (GROUP > 1) {
      if (lane == 0) red[buf][warp] = v;
      __syncthreads();
      const int w0 = (warp / GROUP) * GROUP;
#pragma unroll
      for (int w = 0; w < GROUP; ++w) v = fmaxf(v, red[buf][w0 + w]);
    }
    return v;
  };
  amax = group_max(amax, 0);

  if (GELU) {
    // Exact amax over the candidates (see the file comment).  A thread whose
    // own fast maximum is below the threshold holds no candidate; the rare
    // candidates re-read their input element.
    // A fast maximum of +inf comes from an input of +inf only (the fast GELU
    // of a finite input is finite, its exact value too), whose canonical GELU
    // is +inf: the exact maximum is +inf, and the threshold below would be
    // NaN.  amax is the group's, so the whole group takes the same branch.
    const bool inf_row = amax > 3.402823466e38f;
    const float margin = __fmaf_rn(amax, 0x1p-11f, 0x1p-19f);
    const float thresh = amax - margin;
    float exact = inf_row ? amax : 0.0f;
    // Only elements of the row are candidates: a chunk past the row's end
    // (e >= K) or a row past the last holds zeros, which pass a negative
    // threshold (a row of tiny values) but have no input to re-read.
    if (!inf_row && row_ok && lamax >= thresh) {
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int e = (t + 32 * GROUP * c) * 16;
        if (e >= K) continue;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const float yk = (k & 1) ? f2hi(y2[c][k >> 1]) : f2lo(y2[c][k >> 1]);
          if (fabsf(yk) >= thresh) {
            const float xk = __uint_as_float(static_cast<uint32_t>(__ldg(a.x + base + e + k)) << 16);
            exact = fmaxf(exact, fabsf(canonical_gelu_call(xk)));
          }
        }
      }
    }
    amax = group_max(exact, 1);
  }

  const float s = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
  const float r = __fdiv_rn(1.0f, s);
  const f2_t rb = e4m3_bracket(r);
  if (!row_ok) return;
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    const int e = (t + 32 * GROUP * c) * 16;
    if (e < K) {
      uint2 plo, phi;
      if (GELU) {
        const f2_t rr = f2(r, r);
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const f2_t q = mul2(y2[c][j], rr);
          w[j] = e4m3x2(clamp448(f2lo(q)), clamp448(f2hi(q)));
        }
        plo = make_uint2(w[0] | (w[1] << 16), w[2] | (w[3] << 16));
        phi = make_uint2(w[4] | (w[5] << 16), w[6] | (w[7] << 16));
      } else {
        float lo[8], hi[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          lo[2 * k] = f2lo(y2[c][k]);
          lo[2 * k + 1] = f2hi(y2[c][k]);
          hi[2 * k] = f2lo(y2[c][k + 4]);
          hi[2 * k + 1] = f2hi(y2[c][k + 4]);
        }
        plo = e4m3_quot8(lo, s, rb);
        phi = e4m3_quot8(hi, s, rb);
      }
      st16(a.q + base + e, make_uint4(plo.x, plo.y, phi.x, phi.y));
    }
  }
  if (t == 0) a.s[row] = s;
}

// Threads-per-row grouping and chunks per thread for a row of K elements:
// the smallest power-of-two group whose threads hold at most two chunks each.
static bool rowquant_shape(int64_t K, int* group, int* cpl) {
  const int64_t chunks = (K + 15) / 16;
  int g = 1;
  while (g < 16 && chunks > 64 * g) g <<= 1;
  if (chunks > 64 * g) return false;
  *group = g;
  *cpl = chunks > 32 * g ? 2 : 1;
  return true;
}

template <int GROUP, bool GELU, bool CTX>
static cudaError_t launch_rowquant_g(const RowquantArgs& a, int cpl, cudaStream_t st) {
  constexpr int BW = rowquant_block_warps(GROUP);
  const int rows_per_block = BW / GROUP;
  const dim3 grid(static_cast<unsigned>((a.rows + rows_per_block - 1) / rows_per_block));
  const dim3 block(BW * 32);
  return cpl == 1 ? launch_pdl(rowquant_kernel<1, GROUP, GELU, CTX>, grid, block, 0, st, a)
                  : launch_pdl(rowquant_kernel<2, GROUP, GELU, CTX>, grid, block, 0, st, a);
}

template <bool GELU, bool CTX = false>
static cudaError_t launch_rowquant(const RowquantArgs& a, cudaStream_t st) {
  int group = 0, cpl = 0;
  if (!rowquant_shape(a.K, &group, &cpl)) return cudaErrorInvalidValue;
  switch (group) {
    case 1: return launch_rowquant_g<1, GELU, CTX>(a, cpl, st);
    case 2: return launch_rowquant_g<2, GELU, CTX>(a, cpl, st);
    case 4: return launch_rowquant_g<4, GELU, CTX>(a, cpl, st);
    case 8: return launch_rowquant_g<8, GELU, CTX>(a, cpl, st);
    default: return launch_rowquant_g<16, GELU, CTX>(a, cpl, st);
  }
}

// Elementwise fast and canonical GELU, for checking the fast_gelu error bound
// that the GELU row kernel relies on.
// The fast values come from fast_gelu2, the pairwise form the row kernel runs.
__global__ void gelu_probe_kernel(const uint16_t* x, float* fast, float* canon, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = __uint_as_float(static_cast<uint32_t>(x[i]) << 16);
  const int64_t partner = (i ^ 1) < n ? (i ^ 1) : i;  // the other lane of the pair
  const float w = __uint_as_float(static_cast<uint32_t>(x[partner]) << 16);
  const f2_t g = fast_gelu2(f2(v, w));
  fast[i] = f2lo(g);
  canon[i] = canonical_gelu(v);
}

}  // namespace afb

using namespace afb;

extern "C" int afb_rowquant(const void* x, void* q, void* s, int64_t rows, int64_t K, int gelu,
                            void* stream) {
  ApiGuard g("afb_rowquant");
  int group = 0, cpl = 0;
  if (!check(rows >= 0, "rows must be >= 0") ||
      !check(K >= 16 && K % 16 == 0 && rowquant_shape(K, &group, &cpl),
             "K must be a multiple of 16 in [16, 16384], got " + std::to_string(K)) ||
      !check_ptrs({x, q}, {"x", "q"}) || !check_ptr4(s, "s"))
    return g.fail();
  if (rows == 0) return 0;
  RowquantArgs a{};
  a.x = static_cast<const uint16_t*>(x);
  a.q = static_cast<uint8_t*>(q);
  a.s = static_cast<float*>(s);
  a.rows = rows;
  a.K = static_cast<int>(K);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return g.done(gelu ? launch_rowquant<true>(a, st) : launch_rowquant<false>(a, st));
}

extern "C" int afb_ctx_scale_rowquant(const void* out, const void* lse, const void* ln_pad, void* q,
                                      void* s, int64_t batch, int64_t seq, int64_t heads,
                                      int64_t head_dim, void* stream) {
  ApiGuard g("afb_ctx_scale_rowquant");
  int group = 0, cpl = 0;
  if (!check(batch >= 0, "batch must be >= 0") || !check(seq >= 1, "seq must be >= 1") ||
      !check(head_dim == 64 || head_dim == 128 || head_dim == 256,
             "head_dim must be 64, 128 or 256, got " + std::to_string(head_dim)) ||
      !check(heads >= 1 && rowquant_shape(heads * head_dim, &group, &cpl),
             "heads * head_dim must be in [1, 16384], got " + std::to_string(heads * head_dim)) ||
      !check_ptrs({out, q}, {"out", "q"}) || !check_ptr4(lse, "lse") || !check_ptr4(ln_pad, "ln_pad") ||
      !check_ptr4(s, "s"))
    return g.fail();
  if (batch == 0) return 0;
  RowquantArgs a{};
  a.x = static_cast<const uint16_t*>(out);
  a.q = static_cast<uint8_t*>(q);
  a.s = static_cast<float*>(s);
  a.rows = batch * seq;
  a.K = static_cast<int>(heads * head_dim);
  a.lse = static_cast<const float*>(lse);
  a.ln_pad = static_cast<const float*>(ln_pad);
  a.seq = seq;
  a.seqd = make_divu32(seq);
  a.heads = static_cast<int>(heads);
  a.hd_shift = head_dim == 64 ? 6 : head_dim == 128 ? 7 : 8;
  return g.done(launch_rowquant<false, true>(a, static_cast<cudaStream_t>(stream)));
}

extern "C" int afb_gelu_probe(const void* x, void* fast, void* canon, int64_t n, void* stream) {
  ApiGuard g("afb_gelu_probe");
  if (!check(n >= 0, "n must be >= 0") || !check_ptrs({x, fast, canon}, {"x", "fast", "canon"}))
    return g.fail();
  if (n == 0) return 0;
  gelu_probe_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                      static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(x), static_cast<float*>(fast), static_cast<float*>(canon), n);
  return g.done(cudaGetLastError());
}
