// Channel RMS norm followed by SiLU (the VAE decoder's rms_silu family),
// forward and backward.
//
// Reference: src/kernels/rms.py:20-73 (_offset, _fwd_kernel), :76-125
// (_bwd_kernel), :157-335 (ops and autograd); called from src/vae.py:74,
// 258-278.  Rows are pixels of C channels, channels last.  Per row:
//   s = bf16(x + r) (add), the depth-to-space gather of u (shuffle), else x
//   rstd = sqrt(C) / max(sqrt(sum(s^2)), 1e-12)
//   a = (s * rstd) * g;   y = bf16(a * sigmoid(a)),  sigmoid(a) = 1 / (1 + exp(-a))
// Backward (s, dy, gs -> ds, dg):
//   n = s * rstd;  a = n * g;  sg = sigmoid(a);  da = (dy * sg) * (1 + a * (1 - sg))
//   ds = bf16(rstd * (da * g - n * (sum(da * g * n) / C)) (+ gs))  at the source offset
//   dg = sum over rows of da * n
// exp is canonical_exp (afb_device.cuh).
//
// Layout: a row is held by LPR lanes, the smallest power of two with at most
// four 8-element vectors per lane (C = 96: 4 lanes, 8 rows per warp); lane l
// of a row holds vectors l + LPR*k, k < NVP (NVP = pow2ceil(C/8) / LPR), so
// the canonical row sums (P = LPR) take their vector levels in the lane and
// an xor butterfly over the row's lanes.
// dg order: tiles of 32/LPR rows (one warp pass; a stride tree over the tile's
// rows by xor across the row groups), 32 tiles per chunk summed in order from
// zero (one warp per chunk), chunks by the stride tree of finalize.cu.
#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

constexpr int kRmsWarps = 4;
constexpr int kRmsTilesPerChunk = 32;
constexpr int kRmsMaxC = 1024;

struct RmsArgs {
  const uint16_t* x;    // fwd: x [rows, C] or u [B, H/2, W/2, 4C] (shuffle); bwd: s [rows, C]
  const uint16_t* r;    // fwd: residual [rows, C] (add)
  const float* g;       // [C] fp32
  const uint16_t* dy;   // bwd: [rows, C]
  const uint16_t* gs;   // bwd: gradient of s [rows, C] (add, shuffle) or null
  uint16_t* s;          // fwd: s [rows, C] (add, shuffle)
  uint16_t* y;          // fwd: y [rows, C]; bwd: ds (input layout)
  float* part;          // bwd: [chunks][C]
  int64_t rows;
  int64_t H, W;         // output grid of the shuffle
  int C;
  float sqrt_c;         // sqrt(C) rounded once to fp32
};

// Source offset of output row `row` (rms.py:20-32).
template <bool SHUF>
__device__ __forceinline__ int64_t rms_src(int64_t row, const RmsArgs& a) {
  if (!SHUF) return row * a.C;
  const int64_t hw = a.H * a.W;
  const int64_t b = row / hw, rem = row - b * hw, y = rem / a.W, x = rem - y * a.W;
  return (((b * (a.H / 2) + y / 2) * (a.W / 2) + x / 2) * 4 + (y % 2) * 2 + x % 2) * a.C;
}

__device__ __forceinline__ float rms_sigmoid(float a) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, canonical_exp(-a)));
}

// Canonical row sum of the lane's NVP vectors f[k][8] (P = LPR): vector tree
// in the lane, intra-vector tree, xor butterfly over the row's LPR lanes.
template <int LPR, int NVP>
__device__ __forceinline__ float rms_row_sum(float (&f)[NVP][8]) {
#pragma unroll
  for (int h = NVP / 2; h >= 1; h >>= 1)
#pragma unroll
    for (int k = 0; k < h; ++k)
#pragma unroll
      for (int e = 0; e < 8; ++e) f[k][e] = __fadd_rn(f[k][e], f[k + h][e]);
  float t = vec_sum8(f[0]);
#pragma unroll
  for (int o = LPR / 2; o >= 1; o >>= 1) t = __fadd_rn(t, __shfl_xor_sync(kFull, t, o));
  return t;
}

__device__ __forceinline__ float rms_rstd(float ss, float sqrt_c) {
  return __fdiv_rn(sqrt_c, fmaxf(__fsqrt_rn(ss), 1e-12f));
}

template <int LPR, int NVP, bool HAS_R, bool SHUF>
__global__ void __launch_bounds__(kRmsWarps * 32)
rms_fwd_kernel(const RmsArgs a) {
  constexpr int T = 32 / LPR;  // rows per warp pass
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int l = lane % LPR;
  const int gidx = lane / LPR;
  const int C = a.C;
  const int nv = C / 8;
  float gv[NVP][8];
#pragma unroll
  for (int k = 0; k < NVP; ++k) {
    const int v = l + LPR * k;
#pragma unroll
    for (int e = 0; e < 8; ++e) gv[k][e] = v < nv ? __ldg(a.g + v * 8 + e) : 0.0f;
  }
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kRmsWarps;
  for (int64_t base = (static_cast<int64_t>(blockIdx.x) * kRmsWarps + (threadIdx.x >> 5)) * T; base < a.rows;
       base += warps * T) {
    const int64_t row = base + gidx;
    const bool rok = row < a.rows;
    const int64_t src = rok ? rms_src<SHUF>(row, a) : 0;
    const int64_t dst = row * C;
    float sv[NVP][8], sq[NVP][8];
#pragma unroll
    for (int k = 0; k < NVP; ++k) {
      const int v = l + LPR * k;
      const bool ok = rok && v < nv;
      float f[8];
      unpack8(ok ? ld_stream(a.x + src + v * 8) : make_uint4(0, 0, 0, 0), f);
      if (HAS_R) {
        float rr[8];
        unpack8(ok ? ld_stream(a.r + dst + v * 8) : make_uint4(0, 0, 0, 0), rr);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = __fadd_rn(f[e], rr[e]);
        const uint4 sb = pack8_rn(f);
        unpack8(sb, f);  // s is the bf16-rounded sum
        if (ok) st16(a.s + dst + v * 8, sb);
      } else if (SHUF) {
        if (ok) st16(a.s + dst + v * 8, pack8_rn(f));
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        sv[k][e] = f[e];
        sq[k][e] = __fmul_rn(f[e], f[e]);
      }
    }
    const float rstd = rms_rstd(rms_row_sum<LPR, NVP>(sq), a.sqrt_c);
#pragma unroll
    for (int k = 0; k < NVP; ++k) {
      const int v = l + LPR * k;
      if (!rok || v >= nv) continue;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float av = __fmul_rn(__fmul_rn(sv[k][e], rstd), gv[k][e]);
        o[e] = __fmul_rn(av, rms_sigmoid(av));
      }
      st16(a.y + dst + v * 8, pack8_rn(o));
    }
  }
}

// One warp per chunk of kRmsTilesPerChunk tiles of T rows.
template <int LPR, int NVP, bool HAS_GS, bool SHUF>
__global__ void __launch_bounds__(kRmsWarps * 32)
rms_bwd_kernel(const RmsArgs a) {
  constexpr int T = 32 / LPR;
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int l = lane % LPR;
  const int gidx = lane / LPR;
  const int C = a.C;
  const int nv = C / 8;
  const int64_t chunk = static_cast<int64_t>(blockIdx.x) * kRmsWarps + (threadIdx.x >> 5);
  const int64_t chunk_rows = static_cast<int64_t>(T) * kRmsTilesPerChunk;
  if (chunk * chunk_rows >= a.rows) return;  // warp-uniform: no rows, no partial
  float gv[NVP][8], acc[NVP][8];
#pragma unroll
  for (int k = 0; k < NVP; ++k) {
    const int v = l + LPR * k;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      gv[k][e] = v < nv ? __ldg(a.g + v * 8 + e) : 0.0f;
      acc[k][e] = 0.0f;
    }
  }
  for (int tile = 0; tile < kRmsTilesPerChunk; ++tile) {
    const int64_t row = chunk * chunk_rows + static_cast<int64_t>(tile) * T + gidx;
    const bool rok = row < a.rows;
    const int64_t dst = row * C;
    uint4 sb[NVP], db[NVP];
#pragma unroll
    for (int k = 0; k < NVP; ++k) {
      const int v = l + LPR * k;
      const bool ok = rok && v < nv;
      sb[k] = ok ? ld_stream(a.x + dst + v * 8) : make_uint4(0, 0, 0, 0);
      db[k] = ok ? ld_stream(a.dy + dst + v * 8) : make_uint4(0, 0, 0, 0);
    }
    float f[NVP][8];
#pragma unroll
    for (int k = 0; k < NVP; ++k) {
      unpack8(sb[k], f[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[k][e] = __fmul_rn(f[k][e], f[k][e]);
    }
    const float rstd = rms_rstd(rms_row_sum<LPR, NVP>(f), a.sqrt_c);
    float n[NVP][8], da[NVP][8], t[NVP][8];
#pragma unroll
    for (int k = 0; k < NVP; ++k) {
      float sv[8], dv[8];
      unpack8(sb[k], sv);
      unpack8(db[k], dv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        n[k][e] = __fmul_rn(sv[e], rstd);
        const float av = __fmul_rn(n[k][e], gv[k][e]);
        const float sg = rms_sigmoid(av);
        da[k][e] = __fmul_rn(__fmul_rn(dv[e], sg), __fadd_rn(1.0f, __fmul_rn(av, __fsub_rn(1.0f, sg))));
        t[k][e] = __fmul_rn(__fmul_rn(da[k][e], gv[k][e]), n[k][e]);
      }
    }
    const float m = __fdiv_rn(rms_row_sum<LPR, NVP>(t), static_cast<float>(C));
#pragma unroll
    for (int k = 0; k < NVP; ++k) {
      const int v = l + LPR * k;
      float o[8], gsv[8];
      if (HAS_GS) unpack8(rok && v < nv ? ld_stream(a.gs + dst + v * 8) : make_uint4(0, 0, 0, 0), gsv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float vds = __fmul_rn(rstd, __fsub_rn(__fmul_rn(da[k][e], gv[k][e]), __fmul_rn(n[k][e], m)));
        if (HAS_GS) vds = __fadd_rn(vds, gsv[e]);
        o[e] = vds;
        // this row's dg term; rows past the end contribute zero (da = 0)
        float c = __fmul_rn(da[k][e], n[k][e]);
        // stride tree over the tile's T rows: xor across the row groups
#pragma unroll
        for (int off = 16; off >= LPR; off >>= 1) c = __fadd_rn(c, __shfl_xor_sync(kFull, c, off));
        acc[k][e] = __fadd_rn(acc[k][e], c);
      }
      if (rok && v < nv) st16(a.y + rms_src<SHUF>(row, a) + v * 8, pack8_rn(o));
    }
  }
  if (gidx == 0) {
    float* out = a.part + chunk * C;
#pragma unroll
    for (int k = 0; k < NVP; ++k) {
      const int v = l + LPR * k;
      if (v >= nv) continue;
      reinterpret_cast<float4*>(out + v * 8)[0] = make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
      reinterpret_cast<float4*>(out + v * 8)[1] = make_float4(acc[k][4], acc[k][5], acc[k][6], acc[k][7]);
    }
  }
}

// Lanes per row and vectors per lane for C channels (C % 8 == 0, C <= 1024).
static void rms_shape(int C, int* lpr, int* nvp) {
  const int nv = C / 8;
  int L = 1;
  while (L < 32 && L * 4 < nv) L <<= 1;
  int p2 = 1;
  while (p2 < nv) p2 <<= 1;
  *lpr = L;
  *nvp = p2 / L < 1 ? 1 : p2 / L;
}

#define AFB_RMS_DISPATCH(KERNEL, B1, B2, GO)          \
  switch (lpr * 8 + nvp) {                            \
    case 1 * 8 + 1: return GO(KERNEL<1, 1, B1, B2>);  \
    case 1 * 8 + 2: return GO(KERNEL<1, 2, B1, B2>);  \
    case 1 * 8 + 4: return GO(KERNEL<1, 4, B1, B2>);  \
    case 2 * 8 + 4: return GO(KERNEL<2, 4, B1, B2>);  \
    case 4 * 8 + 4: return GO(KERNEL<4, 4, B1, B2>);  \
    case 8 * 8 + 4: return GO(KERNEL<8, 4, B1, B2>);  \
    case 16 * 8 + 4: return GO(KERNEL<16, 4, B1, B2>); \
    case 32 * 8 + 4: return GO(KERNEL<32, 4, B1, B2>); \
    default: return cudaErrorInvalidValue;            \
  }

template <bool HAS_R, bool SHUF>
static cudaError_t launch_rms_fwd(const RmsArgs& a, cudaStream_t st) {
  const DeviceInfo& dev = device_info();
  if (dev.error != cudaSuccess) return dev.error;
  int lpr = 0, nvp = 0;
  rms_shape(a.C, &lpr, &nvp);
  const int64_t per_cta = static_cast<int64_t>(kRmsWarps) * (32 / lpr);
  const int64_t want = (a.rows + per_cta - 1) / per_cta;
  const int64_t cap = static_cast<int64_t>(dev.sms) * 16;
  const dim3 grid(static_cast<unsigned>(want < cap ? want : cap));
  auto go = [&](auto kern) { return launch_pdl(kern, grid, dim3(kRmsWarps * 32), 0, st, a); };
  AFB_RMS_DISPATCH(rms_fwd_kernel, HAS_R, SHUF, go)
}

template <bool HAS_GS, bool SHUF>
static cudaError_t launch_rms_bwd(const RmsArgs& a, int64_t chunks, cudaStream_t st) {
  int lpr = 0, nvp = 0;
  rms_shape(a.C, &lpr, &nvp);
  const dim3 grid(static_cast<unsigned>((chunks + kRmsWarps - 1) / kRmsWarps));
  auto go = [&](auto kern) { return launch_pdl(kern, grid, dim3(kRmsWarps * 32), 0, st, a); };
  AFB_RMS_DISPATCH(rms_bwd_kernel, HAS_GS, SHUF, go)
}
#undef AFB_RMS_DISPATCH

static int64_t rms_chunks(int64_t rows, int64_t C) {
  int lpr = 0, nvp = 0;
  rms_shape(static_cast<int>(C), &lpr, &nvp);
  const int64_t chunk_rows = static_cast<int64_t>(32 / lpr) * kRmsTilesPerChunk;
  return (rows + chunk_rows - 1) / chunk_rows;
}

static bool check_rms(int64_t rows, int64_t C, int shuffled, int64_t H, int64_t W) {
  return check(rows >= 0, "rows must be >= 0") &&
         check(C >= 8 && C <= kRmsMaxC && C % 8 == 0,
               "channels must be a multiple of 8 in [8, 1024], got " + std::to_string(C)) &&
         check(!shuffled || (H >= 2 && W >= 2 && H % 2 == 0 && W % 2 == 0 && rows % (H * W) == 0),
               "shuffle needs an even output grid H x W dividing the rows");
}

}  // namespace afb

using namespace afb;

extern "C" int afb_rms_silu(const void* x, const void* residual, const void* gamma, void* s, void* y,
                            int64_t rows, int64_t H, int64_t W, int64_t channels, int shuffled,
                            void* stream) {
  ApiGuard g("afb_rms_silu");
  if (!check_rms(rows, channels, shuffled, H, W) || !check_ptrs({x, y}, {"x", "y"}) ||
      !check_ptr4(gamma, "gamma") || (residual != nullptr && !check_ptrs({residual}, {"residual"})) ||
      ((residual != nullptr || shuffled) && !check_ptrs({s}, {"s"})) ||
      !check(!(residual != nullptr && shuffled), "the residual add and the shuffle do not combine"))
    return g.fail();
  if (rows == 0) return 0;
  RmsArgs a{};
  a.x = static_cast<const uint16_t*>(x);
  a.r = static_cast<const uint16_t*>(residual);
  a.g = static_cast<const float*>(gamma);
  a.s = static_cast<uint16_t*>(s);
  a.y = static_cast<uint16_t*>(y);
  a.rows = rows;
  a.H = H;
  a.W = W;
  a.C = static_cast<int>(channels);
  a.sqrt_c = static_cast<float>(std::sqrt(static_cast<double>(channels)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (residual) return g.done(launch_rms_fwd<true, false>(a, st));
  return g.done(shuffled ? launch_rms_fwd<false, true>(a, st) : launch_rms_fwd<false, false>(a, st));
}

extern "C" size_t afb_rms_silu_bwd_workspace(int64_t rows, int64_t channels) {
  if (rows <= 0 || channels < 8) return 0;
  return static_cast<size_t>(rms_chunks(rows, channels) * channels) * sizeof(float);
}

extern "C" int afb_rms_silu_bwd(const void* s, const void* gamma, const void* dy, const void* gs,
                                void* ds, void* dgamma, int64_t rows, int64_t H, int64_t W,
                                int64_t channels, int shuffled, void* workspace, size_t workspace_bytes,
                                void* stream) {
  ApiGuard g("afb_rms_silu_bwd");
  if (!check_rms(rows, channels, shuffled, H, W) || !check_ptrs({s, dy, ds}, {"s", "dy", "ds"}) ||
      !check_ptr4(gamma, "gamma") || !check_ptr4(dgamma, "dgamma") ||
      (gs != nullptr && !check_ptrs({gs}, {"gs"})) ||
      !check(finalize_fits(rows > 0 ? rms_chunks(rows, channels) : 1), "too many rows for one call") ||
      !check(rows == 0 || (workspace != nullptr && aligned(workspace, 16)), "workspace is null or misaligned") ||
      !check(workspace_bytes >= afb_rms_silu_bwd_workspace(rows, channels),
             "workspace too small: need " + std::to_string(afb_rms_silu_bwd_workspace(rows, channels)) +
                 " bytes"))
    return g.fail();
  if (rows == 0) return g.done(cudaMemsetAsync(dgamma, 0, channels * sizeof(float), static_cast<cudaStream_t>(stream)));
  RmsArgs a{};
  a.x = static_cast<const uint16_t*>(s);
  a.g = static_cast<const float*>(gamma);
  a.dy = static_cast<const uint16_t*>(dy);
  a.gs = static_cast<const uint16_t*>(gs);
  a.y = static_cast<uint16_t*>(ds);
  a.part = static_cast<float*>(workspace);
  a.rows = rows;
  a.H = H;
  a.W = W;
  a.C = static_cast<int>(channels);
  a.sqrt_c = static_cast<float>(std::sqrt(static_cast<double>(channels)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t chunks = rms_chunks(rows, channels);
  cudaError_t e;
  if (gs) e = shuffled ? launch_rms_bwd<true, true>(a, chunks, st) : launch_rms_bwd<true, false>(a, chunks, st);
  else e = shuffled ? launch_rms_bwd<false, true>(a, chunks, st) : launch_rms_bwd<false, false>(a, chunks, st);
  if (e != cudaSuccess) return g.done(e);
  FinalizeArgs f{};
  f.part = a.part;
  f.n = chunks;
  f.ncols = static_cast<int>(channels);
  f.seg = static_cast<int>(channels);
  f.out[0] = dgamma;
  f.bf16_out = 0;
  return g.done(launch_colsum_finalize(f, 1, st));
}
