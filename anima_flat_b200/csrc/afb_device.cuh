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
//     p[v] = ((X0+X4)+(X2+X6)) + ((X1+X5)+(X3+X7))   for v < P;
//     while P > 1:    p[v] += p[v + P/2];
//     result p[0].
//
// (the intra-vector step is itself a stride tree, so that it maps onto packed
// fp32x2 adds).  A warp that keeps vector v = lane + 32*c in lane `lane`
// realises it exactly: an in-lane stride tree over c, the intra-vector tree,
// then an xor butterfly (strides 16..1), which pairs the same operands
// (addition commutes exactly).
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
// Division by a divisor fixed for a launch (the sequence length), by a
// multiply-high and two shifts instead of a 64-bit division in the row loop.
// The method is Granlund and Montgomery's ("Division by invariant integers
// using multiplication", PLDI 1994, unsigned case with N = 32): for
// 1 <= d <= 2^32 and 0 <= n < 2^32, with l = ceil(log2 d),
//   m = floor(2^32 (2^l - d) / d) + 1   (< 2^32),
//   t = mulhi(m, n),  q = (t + ((n - t) >> min(l, 1))) >> max(l - 1, 0).
// Dividends of 2^32 or more, and divisors above 2^32, take the 64-bit
// division.
// ---------------------------------------------------------------------------
struct DivU32 {
  int64_t d;
  uint32_t m;
  uint32_t s1, s2;
  uint32_t wide;  // d > 2^32: always the 64-bit division
};
__host__ inline DivU32 make_divu32(int64_t d) {
  DivU32 v{};
  v.d = d < 1 ? 1 : d;
  if (v.d > (int64_t{1} << 32)) {
    v.wide = 1;
    return v;
  }
  uint32_t l = 0;
  while ((int64_t{1} << l) < v.d) ++l;
  const unsigned __int128 num = (static_cast<unsigned __int128>(1) << 32) *
                                ((static_cast<unsigned __int128>(1) << l) - static_cast<uint64_t>(v.d));
  v.m = static_cast<uint32_t>(num / static_cast<uint64_t>(v.d) + 1);
  v.s1 = l < 1 ? l : 1;
  v.s2 = l > 1 ? l - 1 : 0;
  return v;
}
__device__ __forceinline__ int64_t div_u32(const DivU32& v, int64_t n) {
  if (v.wide || (static_cast<uint64_t>(n) >> 32) != 0) return n / v.d;
  const uint32_t n32 = static_cast<uint32_t>(n);
  const uint32_t t = __umulhi(v.m, n32);
  return static_cast<int64_t>((t + ((n32 - t) >> v.s1)) >> v.s2);
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
// The reference clamps to [-448, 448] before converting; satfinite already
// saturates every finite value and infinity, so clamp448 only has to map NaN
// to -448 as the clamp's max(NaN, -448) does.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float clamp448(float v) { return fmaxf(v, -448.0f); }
// max(a, |b|, |c|) in one three-input max (sm_100).  Like fmaxf, it returns
// the largest input that is not NaN.  Measured: residual_adaln_fp8 25.1 ->
// 24.3 us against two two-input maxima.
__device__ __forceinline__ float max_abs2(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(fabsf(b)), "f"(fabsf(c)));
  return r;
}
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
  return __fadd_rn(__fadd_rn(__fadd_rn(f[0], f[4]), __fadd_rn(f[2], f[6])),
                   __fadd_rn(__fadd_rn(f[1], f[5]), __fadd_rn(f[3], f[7])));
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
// Bulk asynchronous copies (TMA engine, non-tensor form) into shared memory,
// completing on an mbarrier.  No cluster multicast is used anywhere.
// ---------------------------------------------------------------------------
// Device-side status word of this translation unit: set when a bounded wait
// gives up (never expected).  Each .cu file that waits reports it through its
// own host reader (afb::read_status_* in afb_launch.h).
static __device__ int g_afb_device_status = 0;
constexpr int kStatusWaitTimeout = 1;
// Host side: this translation unit's status word, then (with `clear`) zero.
static inline cudaError_t tu_status(int* status, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_afb_device_status, sizeof(int));
  if (e == cudaSuccess && clear && *status != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_afb_device_status, &zero, sizeof(int));
  }
  return e;
}
// try_wait suspends for a hardware-defined interval per call; this bounds a
// wait to far beyond any real copy latency (seconds), then reports failure.
constexpr uint32_t kMaxWaitSpins = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// Make barrier initialisation visible to the async proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Order this thread's prior generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) writes to the same buffer.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Plain arrival (no transaction bytes): completes the phase of a count-1 barrier.
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// global -> shared bulk copy of `bytes` (multiple of 16, both ends 16-byte
// aligned), signalling `bar` with complete_tx.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
// Prefetch `bytes` (a multiple of 16, 16-byte aligned) from global memory
// into L2, without waiting.  It brings nothing into the SM, so it may run
// before griddepcontrol.wait: L2 is coherent for the whole GPU, and the
// bulk copies issued after the wait read the current data from it.
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// Wait for the phase of `bar` with the given parity to complete; false (and the
// device status set) if the bound of `limit` try_wait rounds is exhausted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t limit = kMaxWaitSpins) {
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
  }
  atomicOr(&g_afb_device_status, kStatusWaitTimeout);
  return false;
}
__device__ __forceinline__ uint4 lds16(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}
// Named CTA barrier `id` (1..15) over `threads` threads (a multiple of 32);
// orders the participants' shared-memory accesses like __syncthreads.
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------
// Packed arithmetic.  Blackwell executes two IEEE fp32 operations per
// instruction on a 64-bit register pair (add/sub/mul.rn.f32x2), and bf16x2
// multiply/add round the exact result once (RNE).
//
// Contraction rule.  With CUDA 12.9's ptxas, a mul.rn.f32x2 whose result
// feeds an add.rn.f32x2 can come out fused into one packed FMA (observed on
// B200: sums of packed squares differed by an ulp in ~9% of rows; exact with
// ptxas -O0, unchanged by -fmad=false).  Scalar mul.rn.f32 is never fused.
// So packed f32x2 is used only for adds/subs, for a sub feeding a multiply
// and for a multiply feeding a multiply; every product that is then added
// (squares in the variance, the scale product before + shift) is formed with
// scalar __fmul_rn.  A packed fma.rn.f32x2 with a -0 addend (exactly the
// rounded product) is folded into a following packed add the same way
// (observed: up to 30% of results differ), so it is no way around the rule.  For bf16 operands,
// add.rn.bf16x2(res, mul.rn.bf16x2(g, x)) equals bf16(fp32(res + bf16(g*x))):
// g*x of two bf16 is exact in fp32, and when res and the product are 17 or
// more binades apart the fp32 sum rounds to res's bf16 neighbourhood either
// way, so the double rounding of the fp32 route never differs.
// ---------------------------------------------------------------------------
typedef unsigned long long f2_t;  // two fp32 lanes {lo, hi}

__device__ __forceinline__ f2_t f2(float lo, float hi) {
  f2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float f2lo(f2_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2hi(f2_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ f2_t add2(f2_t a, f2_t b) {
  f2_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2_t sub2(f2_t a, f2_t b) {
  f2_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// Packed multiply: only where the result feeds another multiply or is rounded
// directly (see the contraction rule above).
__device__ __forceinline__ f2_t mul2(f2_t a, f2_t b) {
  f2_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// bf16 pair (packed in one 32-bit word) -> fp32 pair.
__device__ __forceinline__ f2_t bf2f2(uint32_t w) { return f2(bf_lo(w), bf_hi(w)); }
// fp32 pair -> bf16 pair, round to nearest even.
__device__ __forceinline__ uint32_t f2bf2(f2_t v) { return pack2_rn(f2lo(v), f2hi(v)); }

// e4m3 codes of clamp(RN(y[k] / s), +-448).  r = RN(1/s) has relative error
// at most 2^-24, and rl = RN(r * (1 - 2^-22)), rh = RN(r * (1 + 2^-22)) two
// more roundings of at most 2^-24 each, so as real numbers
//   |y| * rl <= |y/s| (1 + 2^-24)^2 (1 - 2^-22) < |y/s|  and  |y| * rh > |y/s|.
// RN is monotone, so RN(y * rl) and RN(y * rh) bracket the correctly
// rounded quotient Q = RN(y / s) in magnitude; e4m3 rounding (saturating)
// is monotone too, so when both ends give the same code, that is Q's code,
// and it is the result.  The lower end alone is clamped, so a NaN quotient
// (clamped to -448 by the reference) never matches and takes the exact
// path.  Where any pair of the vector is open, all eight codes come from the
// IEEE quotient.  e4m3_bracket gives (rl, rh) for r.
//
// e4m3_try8 forms the bracketed codes and clears `settled` where a pair is
// open, with no branch, so a kernel can form every vector's codes first and
// take one (rare) branch to e4m3_ieee8 after them all.
__device__ __forceinline__ f2_t e4m3_bracket(float r) {
  return f2(__fmul_rn(r, 1.0f - 0x1p-22f), __fmul_rn(r, 1.0f + 0x1p-22f));
}
__device__ __forceinline__ uint2 e4m3_try8(const float (&y)[8], f2_t rb, bool& settled) {
  const f2_t rl = f2(f2lo(rb), f2lo(rb)), rh = f2(f2hi(rb), f2hi(rb));
  uint32_t hi[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const f2_t v = f2(y[2 * j], y[2 * j + 1]);
    const f2_t a = mul2(v, rl);
    const f2_t b = mul2(v, rh);
    hi[j] = e4m3x2(f2lo(b), f2hi(b));
    settled = settled && e4m3x2(clamp448(f2lo(a)), clamp448(f2hi(a))) == hi[j];
  }
  return make_uint2(hi[0] | (hi[1] << 16), hi[2] | (hi[3] << 16));
}
__device__ __forceinline__ uint2 e4m3_ieee8(const float (&y)[8], float s) {
  float q[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) q[k] = clamp448(__fdiv_rn(y[k], s));
  return e4m3x8(q);
}
__device__ __forceinline__ uint2 e4m3_quot8(const float (&y)[8], float s, f2_t rb) {
  bool settled = true;
  const uint2 c = e4m3_try8(y, rb, settled);
  return settled ? c : e4m3_ieee8(y, s);
}

// Element-wise scalar products of two pairs, kept scalar so that they are never
// contracted into a following add.
__device__ __forceinline__ f2_t mul2_noc(f2_t a, f2_t b) {
  return f2(__fmul_rn(f2lo(a), f2lo(b)), __fmul_rn(f2hi(a), f2hi(b)));
}
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t badd2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t word(const uint4 v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}
// Exact fp32 products of the two bf16 pairs of a and b, elementwise: a bf16
// product has at most 16 significant bits, so fma.rn.f32.bf16 with a -0
// addend rounds exactly as the fp32 multiply of the widened operands does
// (the sign of a zero product included), without widening them first.
__device__ __forceinline__ f2_t bf16x2_mul(uint32_t a, uint32_t b) {
  float lo, hi;
  asm("{\n .reg .b16 al, ah, bl, bh;\n mov.b32 {al, ah}, %2;\n mov.b32 {bl, bh}, %3;\n"
      " fma.rn.f32.bf16 %0, al, bl, 0f80000000;\n fma.rn.f32.bf16 %1, ah, bh, 0f80000000;\n}"
      : "=f"(lo), "=f"(hi)
      : "r"(a), "r"(b));
  return f2(lo, hi);
}
// (lo(w) - m.lo, hi(w) - m.hi) and (lo(w) + m.lo, hi(w) + m.hi) for a bf16
// pair w and an fp32 pair m, each one IEEE fp32 operation on the exactly
// widened bf16 value (sub/add.rn.f32.bf16), without widening w first.
__device__ __forceinline__ f2_t bf16x2_sub_f2(uint32_t w, f2_t m) {
  float lo, hi;
  asm("{\n .reg .b16 wl, wh;\n mov.b32 {wl, wh}, %2;\n"
      " sub.rn.f32.bf16 %0, wl, %3;\n sub.rn.f32.bf16 %1, wh, %4;\n}"
      : "=f"(lo), "=f"(hi)
      : "r"(w), "f"(f2lo(m)), "f"(f2hi(m)));
  return f2(lo, hi);
}
__device__ __forceinline__ f2_t bf16x2_add_f2(uint32_t w, f2_t m) {
  float lo, hi;
  asm("{\n .reg .b16 wl, wh;\n mov.b32 {wl, wh}, %2;\n"
      " add.rn.f32.bf16 %0, wl, %3;\n add.rn.f32.bf16 %1, wh, %4;\n}"
      : "=f"(lo), "=f"(hi)
      : "r"(w), "f"(f2lo(m)), "f"(f2hi(m)));
  return f2(lo, hi);
}
__device__ __forceinline__ uint32_t& word_ref(uint4& v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

// Canonical warp sum (P = 32) of the 8-element vectors a lane holds at
// v = lane + 32*c, given as packed pairs p[c][j] = elements (2j, 2j+1).
// Consumes p.  Same operations as warp_canonical_sum.
template <int NC>
__device__ __forceinline__ float warp_canonical_sum2(f2_t (&p)[NC][4]) {
#pragma unroll
  for (int s = NC / 2; s >= 1; s >>= 1) {
#pragma unroll
    for (int c = 0; c < s; ++c) {
#pragma unroll
      for (int j = 0; j < 4; ++j) p[c][j] = add2(p[c][j], p[c + s][j]);
    }
  }
  // intra-vector stride tree: (e0+e4, e1+e5), (e2+e6, e3+e7), then pairs, then halves
  const f2_t q = add2(add2(p[0][0], p[0][2]), add2(p[0][1], p[0][3]));
  float r = __fadd_rn(f2lo(q), f2hi(q));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) r = __fadd_rn(r, __shfl_xor_sync(kFull, r, o));
  return r;
}

// The same with the pairs produced on demand by val(c, j); the first stride
// level is formed from val directly.
template <int NC, typename F>
__device__ __forceinline__ float warp_canonical_sum2_fn(F val) {
  constexpr int H = NC > 1 ? NC / 2 : 1;
  f2_t p[H][4];
#pragma unroll
  for (int c = 0; c < H; ++c) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (NC > 1) {
        p[c][j] = add2(val(c, j), val(c + H, j));
      } else {
        p[c][j] = val(c, j);
      }
    }
  }
  return warp_canonical_sum2<H>(p);
}

// Canonical sum (P = 32) of a row held by the two warps of a pair.  val(i, j)
// is the fp32 pair (2j, 2j+1) of the lane's i-th vector (vector index
// c = 2i + h when SPLIT, else i).  The stride tree over the NH local vectors
// runs in registers (first level fused with val); with SPLIT the last level
// adds the partner warp's vector from `xch` ([warp][pair][lane]) after the
// pair barrier.  Both warps return the same sum.
template <int NH, bool SPLIT, typename F>
__device__ __forceinline__ float pair_canonical_sum2(F val, f2_t* xch, int h, int lane, int bar_id) {
  constexpr int H = NH > 1 ? NH / 2 : 1;
  f2_t p[H][4];
#pragma unroll
  for (int i = 0; i < H; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (NH > 1) {
        p[i][j] = add2(val(i, j), val(i + H, j));
      } else {
        p[i][j] = val(i, j);
      }
    }
  }
#pragma unroll
  for (int s = H / 2; s >= 1; s >>= 1) {
#pragma unroll
    for (int i = 0; i < s; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) p[i][j] = add2(p[i][j], p[i + s][j]);
    }
  }
  if constexpr (SPLIT) {
#pragma unroll
    for (int j = 0; j < 4; ++j) xch[(h * 4 + j) * 32 + lane] = p[0][j];
    named_bar_sync(bar_id, 64);
#pragma unroll
    for (int j = 0; j < 4; ++j) p[0][j] = add2(p[0][j], xch[((h ^ 1) * 4 + j) * 32 + lane]);
  }
  const f2_t q = add2(add2(p[0][0], p[0][2]), add2(p[0][1], p[0][3]));
  float r = __fadd_rn(f2lo(q), f2hi(q));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) r = __fadd_rn(r, __shfl_xor_sync(kFull, r, o));
  return r;
}

// Two canonical sums at once (one exchange and one pair barrier): val(n, i, j)
// for n = 0, 1; `xch` holds 2 * (2 warps x 4 pairs x 32 lanes).  Same order as
// pair_canonical_sum2 for each sum.
template <int NH, bool SPLIT, typename F>
__device__ __forceinline__ void pair_canonical_sum2x2(F val, f2_t* xch, int h, int lane, int bar_id,
                                                      float& s0, float& s1) {
  constexpr int H = NH > 1 ? NH / 2 : 1;
  f2_t p[2][H][4];
#pragma unroll
  for (int n = 0; n < 2; ++n) {
#pragma unroll
    for (int i = 0; i < H; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (NH > 1) {
          p[n][i][j] = add2(val(n, i, j), val(n, i + H, j));
        } else {
          p[n][i][j] = val(n, i, j);
        }
      }
    }
#pragma unroll
    for (int s = H / 2; s >= 1; s >>= 1) {
#pragma unroll
      for (int i = 0; i < s; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) p[n][i][j] = add2(p[n][i][j], p[n][i + s][j]);
      }
    }
  }
  if constexpr (SPLIT) {
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) xch[((n * 2 + h) * 4 + j) * 32 + lane] = p[n][0][j];
    named_bar_sync(bar_id, 64);
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) p[n][0][j] = add2(p[n][0][j], xch[((n * 2 + (h ^ 1)) * 4 + j) * 32 + lane]);
  }
  float r[2];
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    const f2_t q = add2(add2(p[n][0][0], p[n][0][2]), add2(p[n][0][1], p[n][0][3]));
    r[n] = __fadd_rn(f2lo(q), f2hi(q));
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    r[0] = __fadd_rn(r[0], __shfl_xor_sync(kFull, r[0], o));
    r[1] = __fadd_rn(r[1], __shfl_xor_sync(kFull, r[1], o));
  }
  s0 = r[0];
  s1 = r[1];
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

// exp(a) for every fp32 a, by the same reduction and polynomial as
// canonical_exp_nonpos (identical results for a <= 0).  Above 2^127 the scale
// is applied in two exact steps; beyond exp's range the product overflows to
// infinity as IEEE multiplication does; NaN propagates.
//
// For |a| <= 87 the scale 2^k (|k| <= 126) is a normal number and one product
// applies it; at k = -126 that equals the two-step scaling below (its first
// step is exact), so the short path changes no result.
__device__ __forceinline__ float canonical_exp(float a) {
  if (fabsf(a) <= 87.0f) {
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
    return __fmul_rn(p, __int_as_float((static_cast<int>(k) + 127) << 23));
  }
  if (a != a) return a + a;
  if (a < -104.0f) return 0.0f;
  if (a > 88.8f) return __int_as_float(0x7f800000);
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
  if (ki > 127) return __fmul_rn(__fmul_rn(p, __int_as_float((64 + 127) << 23)), __int_as_float((ki - 64 + 127) << 23));
  if (ki >= -125) return __fmul_rn(p, __int_as_float((ki + 127) << 23));
  return __fmul_rn(__fmul_rn(p, __int_as_float((ki + 64 + 127) << 23)), __int_as_float((-64 + 127) << 23));
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
// It keeps the canonical formula's rounding structure where it matters: the
// erfc term is subtracted from 1 with one rounding (y = RN(1 - p*e)), and
// gelu = (x/2) * (1 +- y) is one FMA, RN(|x|/2 * y + x/2): for x < 0, where
// 1 - y cancels, that is RN((x/2) * (1 - y)) exactly as in the canonical
// formula, and for x >= 0 it skips the rounding of 1 + y.  1/sqrt2 is folded
// into the constants of t and of the exponent.  Absolute error stays below
// 2^-20 + 2^-12 * |gelu(x)|; the row kernel uses it for the codes and
// recomputes the canonical value for amax candidates.
__device__ __forceinline__ float fast_gelu(float x) {
  const float hx = 0.5f * x, hax = 0.5f * fabsf(x);
  float t;
  // hax * 2c == |x| * c exactly (a power-of-two scaling)
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(__fmaf_rn(hax, 2.0f * (0.3275911f * 0.707106769084930419921875f), 1.0f)));
  float n = __fmaf_rn(-1.061405429f, t, 1.453152027f);  // n = -p (see fast_gelu2)
  n = __fmaf_rn(n, t, -1.421413741f);
  n = __fmaf_rn(n, t, 0.284496736f);
  n = __fmaf_rn(n, t, -0.254829592f);
  n = n * t;
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"((x * x) * -0.721347520444481703680f));
  const float y = __fmaf_rn(n, e, 1.0f);
  return __fmaf_rn(hax, y, hx);
}

// fast_gelu on a pair of elements with packed fp32x2 arithmetic: the same
// operations lane by lane (fma.rn.f32x2 and mul.rn.f32x2 round like the
// scalar fma and mul; the reciprocal and the exponential stay scalar), so the
// result is bit-identical to fast_gelu on each element.  It has no product
// feeding an add, so the packed contraction rule does not apply.
__device__ __forceinline__ f2_t fma2(f2_t a, f2_t b, f2_t c) {
  f2_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ f2_t splat2(float v) { return f2(v, v); }
__device__ __forceinline__ f2_t fast_gelu2(f2_t x) {
  constexpr f2_t kAbs = 0x7fffffff7fffffffull;
  const f2_t hx = mul2(x, splat2(0.5f));
  const f2_t hax = hx & kAbs;  // |x / 2| = |x| / 2 exactly (halving rounds symmetrically)
  const f2_t den = fma2(hax, splat2(2.0f * (0.3275911f * 0.707106769084930419921875f)), splat2(1.0f));
  float t0, t1;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t0) : "f"(f2lo(den)));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t1) : "f"(f2hi(den)));
  const f2_t t = f2(t0, t1);
  // n = -p, from the negated coefficients: RN(-v) = -RN(v), so every step
  // is the exact negation of the canonical order's, and 1 - p*e = fma(n, e, 1).
  f2_t n = fma2(splat2(-1.061405429f), t, splat2(1.453152027f));
  n = fma2(n, t, splat2(-1.421413741f));
  n = fma2(n, t, splat2(0.284496736f));
  n = fma2(n, t, splat2(-0.254829592f));
  n = mul2(n, t);
  const f2_t arg = mul2(mul2(x, x), splat2(-0.721347520444481703680f));
  float e0, e1;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(f2lo(arg)));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(f2hi(arg)));
  const f2_t y = fma2(n, f2(e0, e1), splat2(1.0f));  // 1 - p*e
  return fma2(hax, y, hx);
}

// The trimmed cross-attention's gain (src/kernels/ctx_scale.py:8-37):
// 1 / (1 + exp(ln_pad - lse)), IEEE operations and canonical_exp.
__device__ __forceinline__ float ctx_gain(float ln_pad, float lse) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, canonical_exp(__fsub_rn(ln_pad, lse))));
}

// silu(a) = a * sigmoid(a) with sigmoid(a) = RN(1 / RN(1 + canonical_exp(-a))),
// every step an IEEE fp32 operation (the VAE's rms_silu, src/kernels/rms.py:74).
// 1/d correctly rounded is the same number whether formed by division or by
// the correctly rounded reciprocal.
__device__ __forceinline__ float canonical_sigmoid(float a) {
  return __frcp_rn(__fadd_rn(1.0f, canonical_exp(-a)));
}
__device__ __forceinline__ float canonical_silu(float a) { return __fmul_rn(a, canonical_sigmoid(a)); }

// silu on the special-function unit (ex2.approx, rcp.approx) for a pair of
// elements.  No product feeds an addition, so the packed operations round
// lane by lane like their scalar forms and no contraction can change them.
__device__ __forceinline__ f2_t fast_silu2(f2_t a) {
  const f2_t t = mul2(a, splat2(-1.44269502162933349609375f));
  float e0, e1, r0, r1;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(f2lo(t)));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(f2hi(t)));
  const f2_t d = add2(f2(e0, e1), splat2(1.0f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(f2lo(d)));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(f2hi(d)));
  return mul2(a, f2(r0, r1));
}

// The bf16 pair of fast_silu2's values v for a, with `settled` set when it
// is certainly the bf16 rounding of canonical_silu on both elements.  The
// fast and the canonical fp32 values lie at most 6 fp32 steps apart for
// |a| < 4 and 16 for |a| <= 8 (ex2's argument rounding grows with |a|), so
// when v * (1 - eps) and v * (1 + eps), eps = 2^-19 resp. 2^-17 (at least 15
// resp. 63 steps of v), round to the same bf16, so does the canonical value;
// that bf16 is the result.  An exhaustive check over every fp32 a, on the
// device, tests exactly this implication.  Outside |a| <= 8 (and where 1 + e
// overflows) and near a rounding midpoint the caller recomputes canonical_silu.
constexpr float kSiluFastRange = 8.0f;
__device__ __forceinline__ uint32_t silu_pair_bf16(f2_t a, f2_t v, bool& settled) {
  const float fa = fmaxf(fabsf(f2lo(a)), fabsf(f2hi(a)));
  const bool near = fa < 4.0f;
  const f2_t lo = mul2(v, splat2(near ? 1.0f - 0x1p-19f : 1.0f - 0x1p-17f));
  const f2_t hi = mul2(v, splat2(near ? 1.0f + 0x1p-19f : 1.0f + 0x1p-17f));
  const uint32_t bl = f2bf2(lo), bh = f2bf2(hi);
  settled = fa <= kSiluFastRange && bl == bh;
  return bh;
}

// canonical_sigmoid for a pair of elements with |a| <= 87, without branches,
// identical to canonical_sigmoid on every such fp32 a (an exhaustive device
// check tests this).  The steps are canonical_exp's: rint(x * log2e) as the
// sum with 1.5 * 2^23 (in [2^23, 2^24) the sum rounds to an integer, ties to
// even, and subtracting the constant back is exact), the same Cody & Waite
// reduction and polynomial (packed FMAs round like scalar ones), and 2^k from
// the integer bits of that sum (|k| <= 126, one product).  The correctly
// rounded reciprocal of d = 1 + e in [1, 2^126) is the special-function
// unit's estimate y refined by one Newton-Raphson step in Markstein's FMA
// form: r = 1 - d * y (exact), y + y * r.
__device__ __forceinline__ f2_t sigmoid_core2(f2_t a) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  // canonical_sigmoid takes exp(x) at x = -a.  The sign is carried by the
  // constants instead (RN(-v) = -RN(v)): the product x * log2e is a times
  // -log2e; m = -r is the reduction applied to a; and the polynomial in
  // r = -m runs as n1 = -p1, p2, n3 = -p3, ..., n7 = -p7 with every other
  // constant negated, so e' = n7 * 2^k = -e and d = 1 + e = 1 - e'.
  const float t0 = __fadd_rn(__fmul_rn(f2lo(a), -1.44269502162933349609375f), kRound);
  const float t1 = __fadd_rn(__fmul_rn(f2hi(a), -1.44269502162933349609375f), kRound);
  const f2_t k = sub2(f2(t0, t1), splat2(kRound));
  f2_t m = fma2(k, splat2(0.693145751953125f), a);
  m = fma2(k, splat2(1.428606765330187e-06f), m);
  f2_t p = fma2(splat2(1.98412701138295233249664306640625e-04f), m,
                splat2(-1.38888892251998186111450195312500e-03f));
  p = fma2(p, m, splat2(8.33333376795053482055664062500000e-03f));
  p = fma2(p, m, splat2(-4.16666679084300994873046875000000e-02f));
  p = fma2(p, m, splat2(1.66666671633720397949218750000000e-01f));
  p = fma2(p, m, splat2(-0.5f));
  p = fma2(p, m, splat2(1.0f));
  p = fma2(p, m, splat2(-1.0f));
  // bits of t = 0x4B400000 + k; 2^k = (k + 127) << 23
  constexpr int kBias = 127 - 0x4B400000;
  const float e0 = __fmul_rn(f2lo(p), __int_as_float((__float_as_int(t0) + kBias) << 23));
  const float e1 = __fmul_rn(f2hi(p), __int_as_float((__float_as_int(t1) + kBias) << 23));
  const float d0 = __fsub_rn(1.0f, e0), d1 = __fsub_rn(1.0f, e1);
  float y0, y1;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0) : "f"(d0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y1) : "f"(d1));
  const f2_t d = f2(d0, d1), y = f2(y0, y1);
  constexpr f2_t kSign = 0x8000000080000000ull;
  const f2_t rr = fma2(d ^ kSign, y, splat2(1.0f));
  return fma2(y, rr, y);
}

}  // namespace afb
