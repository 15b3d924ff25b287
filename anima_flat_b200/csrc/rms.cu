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
// exp is canonical_exp and sigmoid canonical_sigmoid (afb_device.cuh).
//
// Row layout: a row is held by LPR lanes, the smallest power of two with at
// most four 8-element vectors per lane (C = 96: 4 lanes, T = 8 rows per warp
// pass); lane l of a row holds vectors l + LPR*k, k < NVP (NVP =
// pow2ceil(C/8) / LPR; slots at or past KV = ceil(C/8 / LPR) are zero for
// every lane and hold no registers), so the canonical row sums (P = LPR) take
// their vector levels in the lane and an xor butterfly over the row's lanes.
//
// Streaming: every warp owns a ring of shared-memory stages that its lane 0
// fills with bulk copies (TMA engine) completing on the stage's mbarrier, a
// unit of whole rows per stage, so the next unit's bytes are in flight while
// the warp computes.  Forward units go to warps round robin (any split gives
// the same per-row results); a shuffle unit is a run of source pixels (4
// output rows each), so every unit is one contiguous range of the input.
//
// Forward SiLU: fast_silu2 on the special-function unit; where silu_pair_bf16
// cannot vouch for the bf16 rounding (near a rounding midpoint, or |a| out of
// the fast range) the element is recomputed with canonical_silu.
//
// dg order (backward): chunks of TPC tiles of T rows, TPC = 8 doubled until
// at most kRmsMaxChunks chunks remain.  Within a chunk each row group (row
// index mod T) sums its rows' da * n in row order from +0; the T group sums
// are combined by a stride tree (an xor butterfly across the row groups), the
// chunk partials by the stride tree of finalize.cu.  A chunk is one warp's
// work; chunks go to warps round robin.  A sum that starts at +0 never becomes
// -0, so rows past the end may be skipped or added as zeros alike.
#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

constexpr int kRmsWarps = 8;     // warps per forward CTA
constexpr int kRmsBwdWarps = 6;  // warps per backward CTA: two CTAs per SM leave ~170 registers a thread
constexpr int kRmsBaseTilesPerChunk = 8;
constexpr int64_t kRmsMaxChunks = 32768;        // the finalize kernel's limit
constexpr int kRmsMaxC = 1024;
constexpr size_t kRmsStageTarget = 6 * 1024;    // forward bytes per stage
constexpr size_t kRmsCtaSmemFor2 = 110 * 1024;  // two CTAs per SM at or below this
constexpr int64_t kRmsMaxW = int64_t{1} << 30;  // shuffle width (32-bit column arithmetic)

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
  int tpc;              // bwd: tiles per chunk
  int ut;               // tiles per stage
  int nsw;              // stages per warp
  float sqrt_c;         // sqrt(C) rounded once to fp32
};

// Canonical row sum of the lane's slots f[k][8] (k < KV; slots KV..NVP-1 are
// +0): vector tree in the lane, intra-vector tree, xor butterfly over the
// row's LPR lanes.  The +0 slots are added, so every input, -0 included,
// gives the canonical result.
template <int LPR, int NVP, int KV>
__device__ __forceinline__ float rms_row_sum(float (&f)[KV][8]) {
  if (NVP == 4) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      f[0][e] = __fadd_rn(f[0][e], f[2][e]);
      f[1][e] = __fadd_rn(f[1][e], KV == 4 ? f[KV - 1][e] : 0.0f);
    }
  }
  if (NVP >= 2) {
#pragma unroll
    for (int e = 0; e < 8; ++e) f[0][e] = __fadd_rn(f[0][e], f[1][e]);
  }
  float t = vec_sum8(f[0]);
#pragma unroll
  for (int o = LPR / 2; o >= 1; o >>= 1) t = __fadd_rn(t, __shfl_xor_sync(kFull, t, o));
  return t;
}

__device__ __forceinline__ float rms_rstd(float ss, float sqrt_c) {
  return __fdiv_rn(sqrt_c, fmaxf(__fsqrt_rn(ss), 1e-12f));
}

__device__ __forceinline__ void load_g8(const float* g, bool ok, float (&f)[8]) {
  const float4 a = ok ? __ldg(reinterpret_cast<const float4*>(g)) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 b = ok ? __ldg(reinterpret_cast<const float4*>(g) + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// After a wait gave up: wait (bounded) for this warp's other copies in
// flight, stages j+1 .. j+nsw-1, so none lands after the CTA has exited.
template <typename F>
__device__ __forceinline__ void rms_drain(int64_t j, int nsw, const uint64_t* bars, F issued) {
  for (int64_t k = j + 1; k < j + nsw && issued(k); ++k)
    mbar_wait(smem_addr(&bars[k % nsw]), static_cast<uint32_t>((k / nsw) & 1));
}

template <int LPR, int NVP, int KV, bool HAS_R, bool SHUF>
__global__ void __launch_bounds__(kRmsWarps * 32, 2)
rms_fwd_kernel(const RmsArgs a) {
  constexpr int T = 32 / LPR;  // rows per warp pass
  constexpr int NIN = HAS_R ? 2 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int l = lane % LPR;
  const int gidx = lane / LPR;
  const int C = a.C;
  const bool last_ok = l + LPR * (KV - 1) < C / 8;  // slots below KV-1 are valid for every lane
  const int UR = a.ut * T;                          // rows per unit (a power of two)
  const uint32_t in_bytes = static_cast<uint32_t>(UR) * C * 2u;
  const uint32_t stage_bytes = in_bytes * NIN;
  const int nsw = a.nsw;
  uint8_t* ring = smem + static_cast<size_t>(warp) * nsw * stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(kRmsWarps) * nsw * stage_bytes) +
                   warp * nsw;
  if (lane == 0) {
    for (int s = 0; s < nsw; ++s) mbar_init(smem_addr(&bars[s]), 1);
    fence_mbar_init();
  }
  __syncwarp();
  pdl_wait();
  pdl_trigger();
  const int64_t N = a.rows;
  const int64_t units = (N + UR - 1) / UR;
  const int64_t W = static_cast<int64_t>(gridDim.x) * kRmsWarps;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kRmsWarps + warp;
  auto unit_of = [&](int64_t j) { return gw + j * W; };
  auto issued = [&](int64_t j) { return unit_of(j) < units; };
  auto issue = [&](int64_t j, int s) {  // unit j into stage s = j % nsw
    const int64_t r0 = unit_of(j) * UR;
    const int64_t nr = N - r0 < UR ? N - r0 : UR;
    const uint32_t bytes = static_cast<uint32_t>(nr) * C * 2u;
    const uint32_t bar = smem_addr(&bars[s]);
    uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    mbar_arrive_expect_tx(bar, bytes * NIN);
    // shuffle: unit rows [r0, r0 + nr) come from source pixels [r0/4, (r0+nr)/4),
    // the elements [r0*C, (r0+nr)*C) of u
    bulk_g2s(smem_addr(st), a.x + r0 * C, bytes, bar);
    if (HAS_R) bulk_g2s(smem_addr(st + in_bytes), a.r + r0 * C, bytes, bar);
  };
  if (lane == 0) {
    for (int j = 0; j < nsw && issued(j); ++j) issue(j, j);
  }
  float gv[KV][8];
#pragma unroll
  for (int k = 0; k < KV; ++k) load_g8(a.g + (l + LPR * k) * 8, k < KV - 1 || last_ok, gv[k]);
  const uint32_t w2 = static_cast<uint32_t>(a.W / 2);
  int s = 0;         // stage of unit j (j % nsw)
  uint32_t ph = 0;   // its phase parity ((j / nsw) & 1)
  for (int64_t j = 0; issued(j); ++j) {
    if (!mbar_wait(smem_addr(&bars[s]), ph)) {
      if (lane == 0) rms_drain(j, nsw, bars, issued);
      return;
    }
    const uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    const int64_t r0 = unit_of(j) * UR;
    const int64_t nr = N - r0 < UR ? N - r0 : UR;
    int64_t R0 = 0;  // shuffle: source image row (b * H/2 + i) and column of the unit's first pixel
    uint32_t j0 = 0;
    if (SHUF) {
      R0 = (r0 / 4) / w2;
      j0 = static_cast<uint32_t>(r0 / 4 - R0 * w2);
    }
    for (int p = 0; p < a.ut; ++p) {
      const int q = p * T + gidx;  // row of the unit
      int srow;                    // row of the stage, in rows of C elements
      int64_t orow;                // output row
      bool rok;
      if (SHUF) {
        // q = (aa, jj, bb): output row 2R + aa, column 2j + bb of the unit's pixel jj
        const int half = UR / 2;
        const int aa = q / half, rem = q % half, jj = rem >> 1, bb = rem & 1;
        srow = jj * 4 + aa * 2 + bb;
        rok = jj < nr / 4;
        const uint32_t t = j0 + static_cast<uint32_t>(jj);
        const uint32_t dq = t / w2;
        orow = (2 * (R0 + dq) + aa) * a.W + 2 * static_cast<int64_t>(t - dq * w2) + bb;
      } else {
        srow = q;
        rok = q < nr;
        orow = r0 + q;
      }
      const uint8_t* rp = st + static_cast<size_t>(srow) * C * 2;
      const int64_t dst = orow * C;
      float sv[KV][8], sq[KV][8];
#pragma unroll
      for (int k = 0; k < KV; ++k) {
        const int v = l + LPR * k;
        const bool ok = k < KV - 1 || last_ok;
        uint4 xb = ok ? lds16(rp + v * 16) : make_uint4(0, 0, 0, 0);
        if (HAS_R) {
          float f[8], rr[8];
          unpack8(xb, f);
          unpack8(ok ? lds16(rp + in_bytes + v * 16) : make_uint4(0, 0, 0, 0), rr);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = __fadd_rn(f[e], rr[e]);
          xb = pack8_rn(f);  // s is the bf16-rounded sum
        }
        if ((HAS_R || SHUF) && rok && ok) st16(a.s + dst + v * 8, xb);
        unpack8(xb, sv[k]);
#pragma unroll
        for (int e = 0; e < 8; ++e) sq[k][e] = __fmul_rn(sv[k][e], sv[k][e]);
      }
      const float rstd = rms_rstd(rms_row_sum<LPR, NVP, KV>(sq), a.sqrt_c);
      const f2_t rr = f2(rstd, rstd);
      f2_t av[KV][4];
      uint32_t o[KV][4];  // bf16 pairs of y
      uint32_t redo = 0;  // pairs whose fast value is not settled
#pragma unroll
      for (int k = 0; k < KV; ++k) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // a = (s * rstd) * g: products only, exact in packed form
          av[k][e] = mul2(mul2(f2(sv[k][2 * e], sv[k][2 * e + 1]), rr), f2(gv[k][2 * e], gv[k][2 * e + 1]));
          bool ok;
          o[k][e] = silu_pair_bf16(av[k][e], fast_silu2(av[k][e]), ok);
          if (!ok) redo |= 1u << (k * 4 + e);
        }
      }
      if (__any_sync(kFull, redo != 0)) {
#pragma unroll
        for (int k = 0; k < KV; ++k)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (redo & (1u << (k * 4 + e)))
              o[k][e] = pack2_rn(canonical_silu(f2lo(av[k][e])), canonical_silu(f2hi(av[k][e])));
      }
      if (rok) {
#pragma unroll
        for (int k = 0; k < KV; ++k)
          if (k < KV - 1 || last_ok)
            st16(a.y + dst + (l + LPR * k) * 8, make_uint4(o[k][0], o[k][1], o[k][2], o[k][3]));
      }
    }
    __syncwarp();
    if (lane == 0 && issued(j + nsw)) {
      fence_proxy_async_smem();
      issue(j + nsw, s);
    }
    if (++s == nsw) {
      s = 0;
      ph ^= 1u;
    }
  }
}

template <int LPR, int NVP, int KV, bool HAS_GS, bool SHUF>
__global__ void __launch_bounds__(kRmsBwdWarps * 32, 2)
rms_bwd_kernel(const RmsArgs a) {
  constexpr int T = 32 / LPR;
  constexpr int NIN = HAS_GS ? 3 : 2;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int l = lane % LPR;
  const int gidx = lane / LPR;
  const int C = a.C;
  const bool last_ok = l + LPR * (KV - 1) < C / 8;
  const int UR = a.ut * T;  // rows per stage; a.ut divides a.tpc
  const uint32_t in_bytes = static_cast<uint32_t>(UR) * C * 2u;
  const uint32_t stage_bytes = in_bytes * NIN;
  const int nsw = a.nsw;
  uint8_t* ring = smem + static_cast<size_t>(warp) * nsw * stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(kRmsBwdWarps) * nsw * stage_bytes) +
                   warp * nsw;
  if (lane == 0) {
    for (int s = 0; s < nsw; ++s) mbar_init(smem_addr(&bars[s]), 1);
    fence_mbar_init();
  }
  __syncwarp();
  pdl_wait();
  pdl_trigger();
  const int64_t N = a.rows;
  const int64_t chunk_rows = static_cast<int64_t>(a.tpc) * T;
  const int64_t chunks = (N + chunk_rows - 1) / chunk_rows;
  const int spc = a.tpc / a.ut;  // stages per chunk, a power of two
  const int lg_spc = __ffs(spc) - 1;
  const int64_t W = static_cast<int64_t>(gridDim.x) * kRmsBwdWarps;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kRmsBwdWarps + warp;
  // Stage j of this warp: chunk gw + (j / spc) * W, rows from (j % spc) * UR.
  // Only the last chunk can reach past the rows, and a warp's chunks come in
  // increasing order, so once a stage starts past the end no later one is
  // copied: the copied stages are a prefix of j and the ring's parity follows j.
  auto chunk_of = [&](int64_t j) { return gw + (j >> lg_spc) * W; };
  auto row0_of = [&](int64_t j) { return chunk_of(j) * chunk_rows + (j & (spc - 1)) * UR; };
  auto issued = [&](int64_t j) { return chunk_of(j) < chunks && row0_of(j) < N; };
  auto issue = [&](int64_t j, int s) {  // stage j into ring slot s = j % nsw
    const int64_t r0 = row0_of(j);
    const int64_t nr = N - r0 < UR ? N - r0 : UR;
    const uint32_t bytes = static_cast<uint32_t>(nr) * C * 2u;
    const uint32_t bar = smem_addr(&bars[s]);
    uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    mbar_arrive_expect_tx(bar, bytes * NIN);
    bulk_g2s(smem_addr(st), a.x + r0 * C, bytes, bar);
    bulk_g2s(smem_addr(st + in_bytes), a.dy + r0 * C, bytes, bar);
    if (HAS_GS) bulk_g2s(smem_addr(st + 2 * in_bytes), a.gs + r0 * C, bytes, bar);
  };
  if (lane == 0) {
    for (int j = 0; j < nsw && issued(j); ++j) issue(j, j);
  }
  float acc[KV][8];
#pragma unroll
  for (int k = 0; k < KV; ++k)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[k][e] = 0.0f;
  const uint32_t w2 = static_cast<uint32_t>(a.W / 2);
  const uint32_t Wd = static_cast<uint32_t>(a.W);
  int s = 0;        // ring slot of stage j (j % nsw)
  uint32_t ph = 0;  // its phase parity ((j / nsw) & 1)
  for (int64_t j = 0; chunk_of(j) < chunks; ++j) {
    if (issued(j)) {
      if (!mbar_wait(smem_addr(&bars[s]), ph)) {
        if (lane == 0) rms_drain(j, nsw, bars, issued);
        return;
      }
      const uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
      const int64_t r0 = row0_of(j);
      const int64_t nr = N - r0 < UR ? N - r0 : UR;
      int64_t rr0 = 0;  // shuffle: output image row and column of the stage's first row
      uint32_t xx0 = 0;
      if (SHUF) {
        rr0 = r0 / a.W;
        xx0 = static_cast<uint32_t>(r0 - rr0 * a.W);
      }
      for (int p = 0; p < a.ut; ++p) {
        const int q = p * T + gidx;
        const bool rok = q < nr;
        const uint8_t* rp = st + static_cast<size_t>(q) * C * 2;
        float f[KV][8];
#pragma unroll
        for (int k = 0; k < KV; ++k) {
          unpack8((k < KV - 1 || last_ok) ? lds16(rp + (l + LPR * k) * 16) : make_uint4(0, 0, 0, 0), f[k]);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[k][e] = __fmul_rn(f[k][e], f[k][e]);
        }
        const float rstd = rms_rstd(rms_row_sum<LPR, NVP, KV>(f), a.sqrt_c);
        const f2_t rr = f2(rstd, rstd);
        float dag[KV][8], t[KV][8];
#pragma unroll
        for (int k = 0; k < KV; ++k) {
          const int v = l + LPR * k;
          const bool ok = k < KV - 1 || last_ok;
          float sv[8], dv[8], gv[8];
          unpack8(ok ? lds16(rp + v * 16) : make_uint4(0, 0, 0, 0), sv);
          unpack8(ok ? lds16(rp + in_bytes + v * 16) : make_uint4(0, 0, 0, 0), dv);
          load_g8(a.g + v * 8, ok, gv);
          // n = s * rstd and a = n * g feed only products: packed.  The
          // sigmoid of |a| <= 87 takes the branch-free core; the rest (rare)
          // is redone with canonical_sigmoid.
          f2_t n2[4], av2[4], sg2[4];
          uint32_t out = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            n2[e] = mul2(f2(sv[2 * e], sv[2 * e + 1]), rr);
            av2[e] = mul2(n2[e], f2(gv[2 * e], gv[2 * e + 1]));
            // Out of the core's range the pair's values are meaningless (the
            // SFU and integer steps cannot fault) and are redone below.
            const bool in = fmaxf(fabsf(f2lo(av2[e])), fabsf(f2hi(av2[e]))) <= 87.0f;
            sg2[e] = sigmoid_core2(av2[e]);
            if (!in) out |= 1u << e;
          }
          if (__any_sync(kFull, out != 0)) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (out & (1u << e))
                sg2[e] = f2(canonical_sigmoid(f2lo(av2[e])), canonical_sigmoid(f2hi(av2[e])));
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            // da = (dy * sg) * (1 + a * (1 - sg)); a * (1 - sg) is added: scalar
            const f2_t u2 = sub2(splat2(1.0f), sg2[e]);
            const f2_t w2 = f2(__fadd_rn(1.0f, __fmul_rn(f2lo(av2[e]), f2lo(u2))),
                               __fadd_rn(1.0f, __fmul_rn(f2hi(av2[e]), f2hi(u2))));
            const f2_t da2 = mul2(mul2(f2(dv[2 * e], dv[2 * e + 1]), sg2[e]), w2);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int i = 2 * e + h;
              const float da = h ? f2hi(da2) : f2lo(da2);
              const float n = h ? f2hi(n2[e]) : f2lo(n2[e]);
              if (rok) acc[k][i] = __fadd_rn(acc[k][i], __fmul_rn(da, n));
              dag[k][i] = __fmul_rn(da, gv[i]);
              t[k][i] = __fmul_rn(dag[k][i], n);
            }
          }
        }
        const float m = __fdiv_rn(rms_row_sum<LPR, NVP, KV>(t), static_cast<float>(C));
        int64_t src = (r0 + q) * C;
        if (SHUF) {  // output row (R', x) reads source pixel (R'/2, x/2), sub-pixel (R'%2, x%2)
          const uint32_t tq = xx0 + static_cast<uint32_t>(q);
          const uint32_t dq = tq / Wd;
          const int64_t rr = rr0 + dq;
          const uint32_t xx = tq - dq * Wd;
          src = (((rr >> 1) * w2 + (xx >> 1)) * 4 + (rr & 1) * 2 + (xx & 1)) * C;
        }
#pragma unroll
        for (int k = 0; k < KV; ++k) {
          const int v = l + LPR * k;
          const bool ok = k < KV - 1 || last_ok;
          float sv[8], gsv[8], o[8];
          unpack8(ok ? lds16(rp + v * 16) : make_uint4(0, 0, 0, 0), sv);
          if (HAS_GS) unpack8(ok ? lds16(rp + 2 * in_bytes + v * 16) : make_uint4(0, 0, 0, 0), gsv);
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const f2_t n2 = mul2(f2(sv[e], sv[e + 1]), rr);  // the same n as above
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const float n = h ? f2hi(n2) : f2lo(n2);
              float vds = __fmul_rn(rstd, __fsub_rn(dag[k][e + h], __fmul_rn(n, m)));
              if (HAS_GS) vds = __fadd_rn(vds, gsv[e + h]);
              o[e + h] = vds;
            }
          }
          if (rok && ok) st16(a.y + src + v * 8, pack8_rn(o));
        }
      }
      __syncwarp();
      if (lane == 0 && issued(j + nsw)) {
        fence_proxy_async_smem();
        issue(j + nsw, s);
      }
    }
    if (++s == nsw) {
      s = 0;
      ph ^= 1u;
    }
    if (((j + 1) & (spc - 1)) == 0) {  // end of a chunk: stride tree over the row groups
      const int64_t chunk = chunk_of(j);
#pragma unroll
      for (int k = 0; k < KV; ++k)
#pragma unroll
        for (int e = 0; e < 8; ++e)
#pragma unroll
          for (int off = 16; off >= LPR; off >>= 1)
            acc[k][e] = __fadd_rn(acc[k][e], __shfl_xor_sync(kFull, acc[k][e], off));
      if (gidx == 0) {
        float* out = a.part + chunk * C;
#pragma unroll
        for (int k = 0; k < KV; ++k) {
          if (k == KV - 1 && !last_ok) continue;
          const int v = l + LPR * k;
          reinterpret_cast<float4*>(out + v * 8)[0] = make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
          reinterpret_cast<float4*>(out + v * 8)[1] = make_float4(acc[k][4], acc[k][5], acc[k][6], acc[k][7]);
        }
      }
#pragma unroll
      for (int k = 0; k < KV; ++k)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[k][e] = 0.0f;
    }
  }
}

// Every fp32 bit pattern through the forward's fast SiLU (fast_silu2,
// silu_pair_bf16 on neighbouring patterns as pairs) and the backward's
// sigmoid_core2, against canonical_silu and canonical_sigmoid.
// stats[0]: settled SiLU values whose bf16 differs from the canonical one
// (must be 0); stats[1]: SiLU values with |a| <= 8 left unsettled;
// stats[2 + sign * 256 + exponent]: the largest distance in fp32 steps
// between the fast and the canonical SiLU value (both finite, same sign);
// stats[514]: inputs with |a| <= 87 where sigmoid_core2 differs from
// canonical_sigmoid in any bit (must be 0).  Block b covers the patterns
// [b * 65536, (b + 1) * 65536): one sign, one exponent.
__global__ void __launch_bounds__(256) silu_probe_kernel(unsigned long long* stats) {
  __shared__ unsigned int red[4];
  if (threadIdx.x < 4) red[threadIdx.x] = 0;
  __syncthreads();
  const uint32_t base = static_cast<uint32_t>(blockIdx.x) << 16;
  unsigned int bad = 0, redo = 0, maxd = 0, core_bad = 0;
  for (uint32_t i = threadIdx.x * 2; i < 65536u; i += 2 * blockDim.x) {
    const float a0 = __uint_as_float(base + i), a1 = __uint_as_float(base + i + 1);
    const f2_t av2 = f2(a0, a1);
    const f2_t y = fast_silu2(av2);
    bool pair_ok;
    const uint32_t pb = silu_pair_bf16(av2, y, pair_ok);
    if (fabsf(a0) <= 87.0f && fabsf(a1) <= 87.0f) {
      const f2_t sg = sigmoid_core2(av2);
      core_bad += (__float_as_uint(f2lo(sg)) != __float_as_uint(canonical_sigmoid(a0)));
      core_bad += (__float_as_uint(f2hi(sg)) != __float_as_uint(canonical_sigmoid(a1)));
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float av = h ? a1 : a0;
      const float vf = h ? f2hi(y) : f2lo(y);
      const float vc = canonical_silu(av);
      const bool ok = pair_ok;
      const uint32_t bf = h ? pb >> 16 : pb & 0xffffu, bc = pack2_rn(vc, 0.0f) & 0xffffu;
      if (ok && bf != bc) ++bad;
      if (!ok && fabsf(av) <= 8.0f) ++redo;
      const uint32_t uf = __float_as_uint(vf), uc = __float_as_uint(vc);
      if (isfinite(vf) && isfinite(vc) && ((uf ^ uc) >> 31) == 0) {
        const uint32_t d = uf > uc ? uf - uc : uc - uf;
        maxd = d > maxd ? d : maxd;
      }
    }
  }
  atomicAdd(&red[0], bad);
  atomicAdd(&red[1], redo);
  atomicMax(&red[2], maxd);
  atomicAdd(&red[3], core_bad);
  __syncthreads();
  if (threadIdx.x == 0) {
    if (red[0]) atomicAdd(&stats[0], static_cast<unsigned long long>(red[0]));
    if (red[1]) atomicAdd(&stats[1], static_cast<unsigned long long>(red[1]));
    atomicMax(&stats[2 + (base >> 23)], static_cast<unsigned long long>(red[2]));
    if (red[3]) atomicAdd(&stats[514], static_cast<unsigned long long>(red[3]));
  }
}

// Lanes per row, padded vectors per lane and vectors per lane for C channels
// (C % 8 == 0, C <= 1024).
static void rms_shape(int C, int* lpr, int* nvp, int* kv) {
  const int nv = C / 8;
  int L = 1;
  while (L < 32 && L * 4 < nv) L <<= 1;
  int p2 = 1;
  while (p2 < nv) p2 <<= 1;
  *lpr = L;
  *nvp = p2 / L < 1 ? 1 : p2 / L;
  *kv = (nv + L - 1) / L;
}

static int rms_tiles_per_chunk(int64_t rows, int C) {
  int lpr = 0, nvp = 0, kv = 0;
  rms_shape(C, &lpr, &nvp, &kv);
  const int64_t T = 32 / lpr;
  int tpc = kRmsBaseTilesPerChunk;
  while ((rows + tpc * T - 1) / (tpc * T) > kRmsMaxChunks) tpc <<= 1;
  return tpc;
}

static int64_t rms_chunks(int64_t rows, int C) {
  int lpr = 0, nvp = 0, kv = 0;
  rms_shape(C, &lpr, &nvp, &kv);
  const int64_t chunk_rows = static_cast<int64_t>(32 / lpr) * rms_tiles_per_chunk(rows, C);
  return (rows + chunk_rows - 1) / chunk_rows;
}

#define AFB_RMS_DISPATCH(KERNEL, B1, B2, GO)                        \
  switch ((lpr * 8 + nvp) * 8 + kv) {                               \
    case (1 * 8 + 1) * 8 + 1: return GO(KERNEL<1, 1, 1, B1, B2>);   \
    case (1 * 8 + 2) * 8 + 2: return GO(KERNEL<1, 2, 2, B1, B2>);   \
    case (1 * 8 + 4) * 8 + 3: return GO(KERNEL<1, 4, 3, B1, B2>);   \
    case (1 * 8 + 4) * 8 + 4: return GO(KERNEL<1, 4, 4, B1, B2>);   \
    case (2 * 8 + 4) * 8 + 3: return GO(KERNEL<2, 4, 3, B1, B2>);   \
    case (2 * 8 + 4) * 8 + 4: return GO(KERNEL<2, 4, 4, B1, B2>);   \
    case (4 * 8 + 4) * 8 + 3: return GO(KERNEL<4, 4, 3, B1, B2>);   \
    case (4 * 8 + 4) * 8 + 4: return GO(KERNEL<4, 4, 4, B1, B2>);   \
    case (8 * 8 + 4) * 8 + 3: return GO(KERNEL<8, 4, 3, B1, B2>);   \
    case (8 * 8 + 4) * 8 + 4: return GO(KERNEL<8, 4, 4, B1, B2>);   \
    case (16 * 8 + 4) * 8 + 3: return GO(KERNEL<16, 4, 3, B1, B2>); \
    case (16 * 8 + 4) * 8 + 4: return GO(KERNEL<16, 4, 4, B1, B2>); \
    case (32 * 8 + 4) * 8 + 3: return GO(KERNEL<32, 4, 3, B1, B2>); \
    case (32 * 8 + 4) * 8 + 4: return GO(KERNEL<32, 4, 4, B1, B2>); \
    default: return cudaErrorInvalidValue;                          \
  }

static size_t rms_smem(size_t stage, int nsw, int warps = kRmsWarps) {
  return warps * (stage * nsw + nsw * sizeof(uint64_t));
}

template <bool HAS_R, bool SHUF>
static cudaError_t launch_rms_fwd(RmsArgs a, cudaStream_t st) {
  const DeviceInfo& dev = device_info();
  if (dev.error != cudaSuccess) return dev.error;
  int lpr = 0, nvp = 0, kv = 0;
  rms_shape(a.C, &lpr, &nvp, &kv);
  const int T = 32 / lpr;
  const size_t tile = static_cast<size_t>(T) * a.C * 2 * (HAS_R ? 2 : 1);
  // Up to four tiles per stage within the stage target; a shuffle unit needs
  // a multiple of four rows.
  a.ut = 4;
  while (a.ut > 1 && tile * a.ut > kRmsStageTarget) a.ut >>= 1;
  if (SHUF)
    while ((T * a.ut) % 4) a.ut <<= 1;
  a.nsw = 2;  // one unit computing, one in flight per warp
  const size_t stage = tile * a.ut;
  const size_t smem = rms_smem(stage, a.nsw);
  if (smem > dev.max_smem_optin) return cudaErrorInvalidValue;
  const int ctas = smem <= kRmsCtaSmemFor2 ? 2 : 1;
  const int64_t units = (a.rows + T * a.ut - 1) / (T * a.ut);
  const int64_t want = (units + kRmsWarps - 1) / kRmsWarps;
  const int64_t cap = static_cast<int64_t>(dev.sms) * ctas;
  const dim3 grid(static_cast<unsigned>(want < cap ? want : cap));
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e = ensure_smem(kern, smem, true);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, grid, dim3(kRmsWarps * 32), smem, st, a);
  };
  AFB_RMS_DISPATCH(rms_fwd_kernel, HAS_R, SHUF, go)
}

template <bool HAS_GS, bool SHUF>
static cudaError_t launch_rms_bwd(RmsArgs a, int64_t chunks, cudaStream_t st) {
  const DeviceInfo& dev = device_info();
  if (dev.error != cudaSuccess) return dev.error;
  int lpr = 0, nvp = 0, kv = 0;
  rms_shape(a.C, &lpr, &nvp, &kv);
  const int T = 32 / lpr;
  a.ut = 1;
  const size_t stage = static_cast<size_t>(T) * a.C * 2 * (HAS_GS ? 3 : 2);
  a.nsw = rms_smem(stage, 3, kRmsBwdWarps) <= kRmsCtaSmemFor2 ? 3 : 2;  // as deep as two CTAs per SM allow
  const size_t smem = rms_smem(stage, a.nsw, kRmsBwdWarps);
  if (smem > dev.max_smem_optin) return cudaErrorInvalidValue;
  const int ctas = smem <= kRmsCtaSmemFor2 ? 2 : 1;
  const int64_t want = (chunks + kRmsBwdWarps - 1) / kRmsBwdWarps;
  const int64_t cap = static_cast<int64_t>(dev.sms) * ctas;
  const dim3 grid(static_cast<unsigned>(want < cap ? want : cap));
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e = ensure_smem(kern, smem, true);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, grid, dim3(kRmsBwdWarps * 32), smem, st, a);
  };
  AFB_RMS_DISPATCH(rms_bwd_kernel, HAS_GS, SHUF, go)
}
#undef AFB_RMS_DISPATCH

static bool check_rms(int64_t rows, int64_t C, int shuffled, int64_t H, int64_t W) {
  return check(rows >= 0, "rows must be >= 0") &&
         check(C >= 8 && C <= kRmsMaxC && C % 8 == 0,
               "channels must be a multiple of 8 in [8, 1024], got " + std::to_string(C)) &&
         check(!shuffled || (H >= 2 && W >= 2 && H % 2 == 0 && W % 2 == 0 && W <= kRmsMaxW &&
                             rows % (H * W) == 0),
               "shuffle needs an even output grid H x W (W <= 2^30) dividing the rows");
}

cudaError_t read_status_rms(int* status, bool clear) { return tu_status(status, clear); }

}  // namespace afb

using namespace afb;

extern "C" int afb_rms_silu(const void* x, const void* residual, const void* gamma, void* s, void* y,
                            int64_t rows, int64_t H, int64_t W, int64_t channels, int shuffled,
                            void* stream) {
  ApiGuard g("afb_rms_silu");
  if (!check_rms(rows, channels, shuffled, H, W) || !check_ptrs({x, y}, {"x", "y"}) ||
      !check_ptrs({gamma}, {"gamma"}) || (residual != nullptr && !check_ptrs({residual}, {"residual"})) ||
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
  if (rows <= 0 || channels < 8 || channels > kRmsMaxC) return 0;
  return static_cast<size_t>(rms_chunks(rows, static_cast<int>(channels)) * channels) * sizeof(float);
}

extern "C" int afb_rms_silu_bwd(const void* s, const void* gamma, const void* dy, const void* gs,
                                void* ds, void* dgamma, int64_t rows, int64_t H, int64_t W,
                                int64_t channels, int shuffled, void* workspace, size_t workspace_bytes,
                                void* stream) {
  ApiGuard g("afb_rms_silu_bwd");
  if (!check_rms(rows, channels, shuffled, H, W) || !check_ptrs({s, dy, ds}, {"s", "dy", "ds"}) ||
      !check_ptrs({gamma}, {"gamma"}) || !check_ptr4(dgamma, "dgamma") ||
      (gs != nullptr && !check_ptrs({gs}, {"gs"})) ||
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
  a.tpc = rms_tiles_per_chunk(rows, a.C);
  a.sqrt_c = static_cast<float>(std::sqrt(static_cast<double>(channels)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t chunks = rms_chunks(rows, a.C);
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

extern "C" int afb_silu_probe(void* stats, void* stream) {
  ApiGuard g("afb_silu_probe");
  if (!check(stats != nullptr && aligned(stats, 8), "stats is null or misaligned")) return g.fail();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(stats, 0, (2 + 512 + 1) * sizeof(unsigned long long), st);
  if (e != cudaSuccess) return g.done(e);
  silu_probe_kernel<<<65536, 256, 0, st>>>(static_cast<unsigned long long*>(stats));
  return g.done(cudaGetLastError());
}
