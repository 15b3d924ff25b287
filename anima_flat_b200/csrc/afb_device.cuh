// Device-side building blocks shared by every kernel of the fused layer-op path.
//
// Numerics contract (the "canonical formulation").  The reference computes its
// row statistics with Triton's tl.sum, whose association order follows the
// autotuned num_warps (adaln.py:7, :41-43), so the reference fixes no single
// fp32 order.  These kernels fix one that does not depend on the launch shape:
//
//   canonical_sum(x[0..n), P):      n = 8*NV, NVp = max(P, pow2ceil(NV)),
//     vectors X[v] = x[8v .. 8v+8) (zero for v >= NV);
//     while NVp > P:  X[v] += X[v + NVp/2]  (v < NVp/2, elementwise);
//     p[v] = ((X0+X1)+(X2+X3)) + ((X4+X5)+(X6+X7))   for v < P;
//     while P > 1:    p[v] += p[v + P/2];
//     result p[0].
//
// A warp that keeps vector v = lane + 32*c in lane `lane` realises it exactly:
// an in-lane stride tree over c, the intra-vector tree, then an xor butterfly
// (strides 16..1), which pairs the same operands (addition commutes exactly).
// Every other operation is a single IEEE-754 fp32 operation (no contraction:
// the library is built with --fmad=false and uses __f*_rn intrinsics), bf16
// rounding is round-to-nearest-even, FP8 e4m3 rounding is RNE with
// saturation.  The CPU oracle in oracle/ follows the same definition, so
// forward outputs compare bit for bit.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace afb {

constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  Every kernel waits for its predecessor on
// the stream before touching global memory and then lets its own successor
// begin launching, so a chain of short bandwidth-bound kernels overlaps the
// launch latency of kernel i+1 with the tail of kernel i.  Without the launch
// attribute both instructions are no-ops.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// 16-byte global accesses.
// ---------------------------------------------------------------------------
// Streamed read-once activation: read-only path, no L1 allocation.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// Small per-call vectors (modulation rows, norm weights, rope tables) that
// every row re-reads: keep them in L1.
__device__ __forceinline__ uint4 ld_keep(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ float4 ld_keep_f4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
__device__ __forceinline__ void st16(void* p, uint4 v) {
  *reinterpret_cast<uint4*>(p) = v;
}
__device__ __forceinline__ void st8(void* p, uint2 v) {
  *reinterpret_cast<uint2*>(p) = v;
}

// ---------------------------------------------------------------------------
// bf16 <-> fp32 (bf16 widening is exact: the top 16 bits of an fp32).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
  f[0] = bf_lo(v.x); f[1] = bf_hi(v.x);
  f[2] = bf_lo(v.y); f[3] = bf_hi(v.y);
  f[4] = bf_lo(v.z); f[5] = bf_hi(v.z);
  f[6] = bf_lo(v.w); f[7] = bf_hi(v.w);
}
__device__ __forceinline__ float unpack_at(const uint4 v, int k) {
  const uint32_t w = (k < 2) ? v.x : (k < 4) ? v.y : (k < 6) ? v.z : v.w;
  return (k & 1) ? bf_hi(w) : bf_lo(w);
}
// Two fp32 -> packed bf16x2, round to nearest even (cvt.rn.bf16x2.f32).
__device__ __forceinline__ uint32_t pack2_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint4 pack8_rn(const float (&f)[8]) {
  uint4 r;
  r.x = pack2_rn(f[0], f[1]);
  r.y = pack2_rn(f[2], f[3]);
  r.z = pack2_rn(f[4], f[5]);
  r.w = pack2_rn(f[6], f[7]);
  return r;
}
// Round an fp32 to bf16 precision and widen it back.
__device__ __forceinline__ float round_bf(float x) {
  return bf_lo(pack2_rn(x, 0.0f));
}

// ---------------------------------------------------------------------------
// FP8 e4m3 (OCP "fn" variant, max 448): RNE with saturation to +-448.
// cvt.rn.satfinite.e4m3x2.f32 d, a, b puts a in the high byte, b in the low.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  unsigned short r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// Eight fp32 -> eight e4m3 bytes, element k in byte k (little endian).
__device__ __forceinline__ uint2 e4m3x8(const float (&f)[8]) {
  uint2 r;
  r.x = e4m3x2(f[0], f[1]) | (e4m3x2(f[2], f[3]) << 16);
  r.y = e4m3x2(f[4], f[5]) | (e4m3x2(f[6], f[7]) << 16);
  return r;
}

// ---------------------------------------------------------------------------
// Canonical sums.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float vec_sum8(const float (&f)[8]) {
  return __fadd_rn(__fadd_rn(__fadd_rn(f[0], f[1]), __fadd_rn(f[2], f[3])),
                   __fadd_rn(__fadd_rn(f[4], f[5]), __fadd_rn(f[6], f[7])));
}

// Warp-wide canonical sum (P = 32) of the vectors a lane holds at
// v = lane + 32*c, c < NC.  `f` is consumed.
template <int NC>
__device__ __forceinline__ float warp_canonical_sum(float (&f)[NC][8]) {
#pragma unroll
  for (int s = NC / 2; s >= 1; s >>= 1) {
#pragma unroll
    for (int c = 0; c < s; ++c) {
#pragma unroll
      for (int k = 0; k < 8; ++k) f[c][k] = __fadd_rn(f[c][k], f[c + s][k]);
    }
  }
  float p = vec_sum8(f[0]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) p = __fadd_rn(p, __shfl_xor_sync(kFull, p, o));
  return p;
}

// The same sum with the elements produced on demand by val(c, k): the first
// stride level is formed directly from val, so only NC/2 vectors are live.
template <int NC, typename F>
__device__ __forceinline__ float warp_canonical_sum_fn(F val) {
  constexpr int H = NC > 1 ? NC / 2 : 1;
  float f[H][8];
#pragma unroll
  for (int c = 0; c < H; ++c) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if constexpr (NC > 1) {
        f[c][k] = __fadd_rn(val(c, k), val(c + H, k));
      } else {
        f[c][k] = val(c, k);
      }
    }
  }
  return warp_canonical_sum<H>(f);
}

// Canonical sum over an aligned group of LPH lanes holding one vector each
// (P = LPH).  Used for per-head sums (head_dim = 8 * LPH).
template <int LPH>
__device__ __forceinline__ float group_canonical_sum(const float (&f)[8]) {
  float p = vec_sum8(f);
#pragma unroll
  for (int o = LPH / 2; o >= 1; o >>= 1) p = __fadd_rn(p, __shfl_xor_sync(kFull, p, o));
  return p;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// 1 / sqrt(v + eps) with two IEEE roundings (no rsqrt approximation).
__device__ __forceinline__ float canonical_rstd(float var, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

// ---------------------------------------------------------------------------
// GELU, Abramowitz & Stegun 7.1.26 erf (the formula of fp8.py:260-270).
// ---------------------------------------------------------------------------
// exp(a) for a <= 0 from IEEE fp32 operations only: Cody & Waite range
// reduction a = k*ln2 + r with a two-part ln2, then the degree-7 Taylor
// polynomial of exp(r) for |r| <= ln2/2 in Horner form, scaled by 2^k.  It is
// deterministic, so the CPU oracle reproduces it bit for bit.
__device__ __forceinline__ float canonical_exp_nonpos(float a) {
  if (a < -104.0f) return 0.0f;
  const float k = rintf(__fmul_rn(a, 1.44269502162933349609375f));
  float r = __fmaf_rn(k, -0.693145751953125f, a);
  r = __fmaf_rn(k, -1.428606765330187e-06f, r);
  float p = 1.98412701138295233249664306640625e-04f;
  p = __fmaf_rn(p, r, 1.38888892251998186111450195312500e-03f);
  p = __fmaf_rn(p, r, 8.33333376795053482055664062500000e-03f);
  p = __fmaf_rn(p, r, 4.16666679084300994873046875000000e-02f);
  p = __fmaf_rn(p, r, 1.66666671633720397949218750000000e-01f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ki = static_cast<int>(k);
  if (ki >= -125) return __fmul_rn(p, __int_as_float((ki + 127) << 23));
  // Subnormal result: one exact scaling, then one rounding.
  return __fmul_rn(__fmul_rn(p, __int_as_float((ki + 64 + 127) << 23)),
                   __int_as_float((-64 + 127) << 23));
}

__device__ __forceinline__ float canonical_gelu(float x) {
  const float z = __fmul_rn(x, 0.707106769084930419921875f);
  const float az = fabsf(z);
  const float t = __fdiv_rn(1.0f, __fadd_rn(1.0f, __fmul_rn(0.3275911f, az)));
  float p = __fmaf_rn(1.061405429f, t, -1.453152027f);
  p = __fmaf_rn(p, t, 1.421413741f);
  p = __fmaf_rn(p, t, -0.284496736f);
  p = __fmaf_rn(p, t, 0.254829592f);
  p = __fmul_rn(p, t);
  const float e = canonical_exp_nonpos(-__fmul_rn(az, az));
  const float y = __fmaf_rn(-p, e, 1.0f);
  const float erf = (z < 0.0f) ? -y : y;
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erf));
}

// The same formula on the special-function unit (rcp.approx, ex2.approx).
// Absolute error stays below 2^-20 + 2^-12 * |gelu(x)|; the row kernel uses it
// for the codes and recomputes the canonical value for amax candidates.
__device__ __forceinline__ float fast_gelu(float x) {
  const float z = x * 0.707106769084930419921875f;
  const float az = fabsf(z);
  float t;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(__fmaf_rn(0.3275911f, az, 1.0f)));
  float p = __fmaf_rn(1.061405429f, t, -1.453152027f);
  p = __fmaf_rn(p, t, 1.421413741f);
  p = __fmaf_rn(p, t, -0.284496736f);
  p = __fmaf_rn(p, t, 0.254829592f);
  p = p * t;
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-(az * az) * 1.44269502162933349609375f));
  const float y = __fmaf_rn(-p, e, 1.0f);
  const float erf = (z < 0.0f) ? -y : y;
  return (0.5f * x) * (1.0f + erf);
}

}  // namespace afb
