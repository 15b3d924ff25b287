// AdaLN modulate forward, with and without the gated residual, with bf16 or
// per-row FP8 e4m3 output.
//
// Reference: src/kernels/adaln.py:10-46 (_residual_adaln_kernel, HAS_X True
// for residual_adaln, False for adaln) and src/kernels/fp8.py:56-97
// (_residual_adaln_fp8_kernel).  Per row of D elements, with b = row / S:
//   p = bf16(gate[b] * x);  z = bf16(res + p)           (HAS_X; else z = res)
//   mean = sum(z) / D;  d = z - mean;  rstd = 1 / sqrt(sum(d*d) / D + eps)
//   y = (d * rstd) * scale[b] + shift[b]                 (fp32)
//   bf16 output:  h = bf16(y)
//   FP8 output:   s = max(max|y|, 1e-12) / 448;  q = e4m3(clamp(y / s, +-448))
//
// Layout: persistent CTAs, one per SM, of P warp pairs.  CTA c owns
// the contiguous rows [c*R/G, (c+1)*R/G) (R rows, G CTAs: every SM gets the
// same share within one row), and pair p of it the rows p, p + P, ...
// of that range.  Each pair keeps a private ring of `nsw` shared-memory stages;
// its leader lane streams each row's res (and x) into a stage with bulk copies
// (TMA engine) that complete on the stage's mbarrier, so up to nsw rows per
// pair are in flight while the pair computes.  The modulation vectors of the
// (at most two) batch entries a CTA's rows belong to are bulk-copied into
// shared memory first, ahead of the row stream, so no per-row global load
// waits behind it; a CTA whose rows span more batch entries (short sequences)
// reads them from global memory instead.  Both warps of a pair work on the same row: with
// NC = D/256 vectors of 8 elements per lane, warp h holds the vectors
// v = lane + 32*c for c = 2i + h (i < NC/2), so a row costs each warp half the
// instructions and half the latency.  The canonical sums keep their order:
// every level of the vector stride tree but the last pairs vectors of equal
// parity, inside one warp; the last level adds the two warps' vectors through
// shared memory (pair_canonical_sum2).  z and h (or q) are written straight
// from registers.  z = res + gate*x uses packed bf16x2 arithmetic; the
// statistics and the modulation use packed fp32x2 adds/subs under the
// contraction rule of afb_device.cuh.  In FP8 mode y stays in registers
// between the row max and the codes, and each code comes from products of y
// by RN(1/s) (1 -+ 2^-22) wherever they provably give the IEEE quotient's
// code (e4m3_try8).
#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

struct AdalnArgs {
  const uint16_t* x;      // [rows, D] bf16, only with HAS_X
  const uint16_t* res;    // [rows, D] bf16 (the z input of adaln)
  const uint16_t* gate;   // [B, D] bf16, only with HAS_X
  const uint16_t* shift;  // [B, D] bf16
  const uint16_t* scale;  // [B, D] bf16, already 1 + scale
  uint16_t* h;            // [rows, D] bf16 output (bf16 mode)
  uint16_t* z;            // [rows, D] bf16 output (HAS_X)
  uint8_t* q;             // [rows, D] e4m3 output (FP8 mode)
  float* s;               // [rows] fp32 row scales (FP8 mode)
  int64_t rows;
  int64_t seq;            // rows per batch entry: b = row / seq
  DivU32 seqd;            // division by seq
  int dim;
  float eps;
};

// Warp pairs per CTA.  The FP8 kernels at D = 2048 are bound by the latency
// of each row's chain of sums and run 12 pairs (80 registers, no spills; 24
// warps per SM): measured 4-5% faster than 8 pairs in short launches, though
// their row stage ring then has one stage.  Every other instantiation runs 8
// pairs (up to 128 registers); 12 pairs made plain adaln slower.
constexpr int kAdalnPairs = 8;
constexpr int kAdalnPairsFp8 = 12;
// Stages per pair.  A short launch (few rows per SM: config 2 has 27.7) is
// mostly ramp and tail, and more stages delay each pair's first row behind the
// others' copies, so it takes two (measured: adaln, whose 4 KiB stages would
// allow more, is slower with three or four; residual_adaln_fp8 at config 3
// takes 33.8 µs with three, 26.5 with two).  A long launch is a steady stream, where the
// bytes in flight bound the bandwidth, so it takes the deepest ring that fits,
// giving up the shared-memory modulation slots if that buys a stage.
constexpr int kAdalnShortStages = 2;
constexpr int kAdalnMaxStages = 4;
constexpr int64_t kAdalnLongRowsPerCta = 128;
// Per pair: two exchange buffers (one per sum of a row) of 2 warps x 4 pairs
// of fp32 x 32 lanes, then two floats for the FP8 row max (padded to 16 B).
constexpr size_t kAdalnXchF2 = 2 * 2 * 4 * 32;
constexpr size_t kAdalnPairXchBytes = kAdalnXchF2 * sizeof(f2_t) + 4 * sizeof(float);
// Modulation slots: the scale, shift (and gate) rows of up to two batch
// entries, bf16 in shared memory.  Slot layout: [scale D][shift D][gate D].
// (Widening them to fp32 once per CTA saves the per-row unpacking but doubles
// the shared-memory bytes read per row, and measured slower.)
constexpr int kAdalnModSlots = 2;
__host__ __device__ constexpr size_t adaln_slot_bytes(int64_t dim, bool has_x) {
  return static_cast<size_t>(dim) * (has_x ? 6 : 4);
}
__host__ __device__ constexpr size_t adaln_mod_bytes(int64_t dim, bool has_x) {
  return kAdalnModSlots * adaln_slot_bytes(dim, has_x);
}

// EXACT: dim == 256 * NC, so every lane owns NC full vectors (no masking).
// use_smods: the launch reserved shared memory for the modulation slots.
template <int P, int NC, bool HAS_X, bool FP8, bool EXACT>
__global__ void __launch_bounds__(P * 64, 1)
adaln_fwd_kernel(const AdalnArgs a, const int nsw, const int use_smods, const int early) {
  // SPLIT: the pair divides each lane's vectors; for NC == 1 both warps hold
  // the single vector and warp 0 writes the outputs.
  constexpr bool SPLIT = NC >= 2;
  constexpr int NH = SPLIT ? NC / 2 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int pair = warp >> 1;
  const int h = warp & 1;
  const int bar_id = 1 + pair;
  const bool leader = h == 0 && lane == 0;
  const bool writer = SPLIT || h == 0;
  const int D = EXACT ? NC * 256 : a.dim;
  const uint32_t row_bytes = static_cast<uint32_t>(D) * 2u;
  const uint32_t stage_bytes = (HAS_X ? 2u : 1u) * row_bytes;
  const size_t slot_bytes = adaln_slot_bytes(D, HAS_X);
  const size_t ring_all = static_cast<size_t>(P) * nsw * stage_bytes;
  uint8_t* ring = smem + static_cast<size_t>(pair) * nsw * stage_bytes;
  uint8_t* xbase = smem + ring_all + static_cast<size_t>(pair) * kAdalnPairXchBytes;
  f2_t* xch = reinterpret_cast<f2_t*>(xbase);
  float* xmax = reinterpret_cast<float*>(xbase + kAdalnXchF2 * sizeof(f2_t));
  uint8_t* mods = smem + ring_all + P * kAdalnPairXchBytes;
  uint64_t* bars0 = reinterpret_cast<uint64_t*>(mods + (use_smods ? adaln_mod_bytes(D, HAS_X) : 0));
  uint64_t* bars = bars0 + pair * nsw;
  uint64_t* modbar = bars0 + P * nsw;

  // This CTA's rows, and the batch entries they belong to.
  const int64_t r0 = a.rows * blockIdx.x / gridDim.x;
  const int64_t r1 = a.rows * (blockIdx.x + 1) / gridDim.x;
  const int64_t b_lo = r1 > r0 ? r0 / a.seq : 0;
  const int64_t b_hi = r1 > r0 ? (r1 - 1) / a.seq : 0;
  const bool smods = use_smods && r1 > r0 && b_hi - b_lo < kAdalnModSlots;
  const int nb = static_cast<int>(b_hi - b_lo + 1);
  if (leader) {
    for (int s = 0; s < nsw; ++s) mbar_init(smem_addr(&bars[s]), 1);
    if (pair == 0) mbar_init(smem_addr(modbar), 1);
    fence_mbar_init();
  }
  __syncthreads();  // barriers initialised before anyone waits on them
  // bf16 output: while the previous kernel on the stream finishes, pull the
  // first stage of each pair and the modulation rows into L2 (prefetch_l2).
  // Measured: the config-2 step 5.3% faster with every output kept, an
  // isolated launch unchanged; the FP8 instantiations lost 2 us isolated, so
  // they do not prefetch.
  if (!FP8 && lane == 0 && h == 0) {
    const int64_t row = r0 + pair;
    if (row < r1) {
      prefetch_l2(a.res + row * D, row_bytes);
      if (HAS_X) prefetch_l2(a.x + row * D, row_bytes);
    }
    if (pair == 0 && smods) {
      for (int k = 0; k < nb; ++k) {
        prefetch_l2(a.scale + (b_lo + k) * D, row_bytes);
        prefetch_l2(a.shift + (b_lo + k) * D, row_bytes);
        if (HAS_X) prefetch_l2(a.gate + (b_lo + k) * D, row_bytes);
      }
    }
  }
  pdl_wait();
  pdl_trigger();
  if (smods && threadIdx.x == 0) {
    // The modulation rows go first, ahead of every row stage.
    mbar_arrive_expect_tx(smem_addr(modbar), static_cast<uint32_t>(nb * (HAS_X ? 3 : 2)) * row_bytes);
    for (int k = 0; k < nb; ++k) {
      const int64_t pb = (b_lo + k) * D;
      uint8_t* slot = mods + k * slot_bytes;
      bulk_g2s(smem_addr(slot), a.scale + pb, row_bytes, smem_addr(modbar));
      bulk_g2s(smem_addr(slot + 2 * D), a.shift + pb, row_bytes, smem_addr(modbar));
      if (HAS_X) bulk_g2s(smem_addr(slot + 4 * D), a.gate + pb, row_bytes, smem_addr(modbar));
    }
  }
  if (smods) __syncthreads();

  auto row_of = [&](int64_t j) { return r0 + pair + j * P; };
  auto issue = [&](int64_t j, int s) {  // leader: stream row row_of(j) into stage s = j % nsw
    const int64_t row = row_of(j);
    uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    const uint32_t bar = smem_addr(&bars[s]);
    mbar_arrive_expect_tx(bar, stage_bytes);
    bulk_g2s(smem_addr(st), a.res + row * D, row_bytes, bar);
    if (HAS_X) bulk_g2s(smem_addr(st + row_bytes), a.x + row * D, row_bytes, bar);
  };
  if (leader) {
    for (int j = 0; j < nsw && row_of(j) < r1; ++j) issue(j, j);
  }
  auto col = [&](int i) { return (lane + 32 * (SPLIT ? 2 * i + h : i)) * 8; };
  auto ok = [&](int i) { return EXACT || col(i) < D; };

  // A wait that gives up (never expected) marks the warp dead: it keeps taking
  // the pair's barriers but stores nothing and issues no copy, and the leader
  // drains its copies in flight before the CTA exits.
  bool dead = false;
  int64_t jdead = 0;
  if (smods && !mbar_wait(smem_addr(modbar), 0)) dead = true;
  // fp32 pairs (2j, 2j+1) of modulation row v (0 scale, 1 shift) of batch
  // entry b at columns c .. c+7.
  auto mod8 = [&](int v, int64_t b, int c, f2_t (&m)[4]) {
    const uint4 w = smods ? lds16(mods + static_cast<size_t>(b - b_lo) * slot_bytes + v * 2 * D + c * 2)
                          : ld_keep((v == 0 ? a.scale : a.shift) + b * D + c);
    m[0] = bf2f2(w.x);
    m[1] = bf2f2(w.y);
    m[2] = bf2f2(w.z);
    m[3] = bf2f2(w.w);
  };
  // Modulation row v of batch entry b at columns c .. c+7, as bf16 words.
  auto modw = [&](int v, int64_t b, int c) {
    return smods ? lds16(mods + static_cast<size_t>(b - b_lo) * slot_bytes + v * 2 * D + c * 2)
                 : ld_keep((v == 0 ? a.scale : a.shift) + b * D + c);
  };
  auto gate8 = [&](int64_t b, int c) {
    return smods ? lds16(mods + static_cast<size_t>(b - b_lo) * slot_bytes + 4 * D + c * 2)
                 : ld_keep(a.gate + b * D + c);
  };

  // Stage s = j % nsw of row j and its phase parity (j / nsw) & 1, advanced
  // with j (no division in the loop).
  int s = 0;
  uint32_t ph = 0;
  for (int64_t j = 0; row_of(j) < r1; ++j) {
    const int64_t row = row_of(j);
    const uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    if (!dead && !mbar_wait(smem_addr(&bars[s]), ph)) {
      dead = true;
      jdead = j;
    }
    const bool store = writer && !dead;
    const int64_t b = div_u32(a.seqd, row);
    const int64_t base = row * D;

    // stage -> registers; z = bf16(res + bf16(gate * x)) in packed bf16x2;
    // zf = fp32(z) (zero for masked vectors), later d = z - mean in place.
    f2_t zf[NH][4];
    {
      uint4 zv[NH];
      uint4 xv[NH];
#pragma unroll
      for (int i = 0; i < NH; ++i) {
        zv[i] = ok(i) ? lds16(st + col(i) * 2) : make_uint4(0, 0, 0, 0);
        if (HAS_X) xv[i] = ok(i) ? lds16(st + row_bytes + col(i) * 2) : make_uint4(0, 0, 0, 0);
      }
      if (early) {  // refill as soon as both warps hold the row (long launches)
        named_bar_sync(bar_id, 64);
        if (leader && !dead && row_of(j + nsw) < r1) {
          fence_proxy_async_smem();
          issue(j + nsw, s);
        }
      }
      if (HAS_X) {
#pragma unroll
        for (int i = 0; i < NH; ++i) {
          if (ok(i)) {
            const uint4 g = gate8(b, col(i));
            zv[i].x = badd2(zv[i].x, bmul2(g.x, xv[i].x));
            zv[i].y = badd2(zv[i].y, bmul2(g.y, xv[i].y));
            zv[i].z = badd2(zv[i].z, bmul2(g.z, xv[i].z));
            zv[i].w = badd2(zv[i].w, bmul2(g.w, xv[i].w));
            if (store) st16(a.z + base + col(i), zv[i]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < NH; ++i) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) zf[i][jj] = bf2f2(word(zv[i], jj));
      }
    }

    // Statistics (canonical order, see afb_device.cuh), packed fp32x2.
    // x / D; for EXACT, D = 256 * NC is a power of two and x * (1/D) rounds identically
    auto div_d = [&](float x) {
      return EXACT ? __fmul_rn(x, 1.0f / (NC * 256)) : __fdiv_rn(x, static_cast<float>(D));
    };
    const float mean = div_d(pair_canonical_sum2<NH, SPLIT>(
        [&](int i, int jj) { return zf[i][jj]; }, xch, h, lane, bar_id));
    // Both warps have read the stage (the pair barrier above): refill it.
    if (!early) {
      if (!SPLIT) named_bar_sync(bar_id, 64);
      if (leader && !dead && row_of(j + nsw) < r1) {
        fence_proxy_async_smem();
        issue(j + nsw, s);
      }
    }
    const f2_t mm = f2(mean, mean);
#pragma unroll
    for (int i = 0; i < NH; ++i) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) zf[i][jj] = ok(i) ? sub2(zf[i][jj], mm) : 0ull;
    }
    const float var = div_d(pair_canonical_sum2<NH, SPLIT>(
        [&](int i, int jj) { return mul2_noc(zf[i][jj], zf[i][jj]); }, xch + 2 * 4 * 32, h, lane,
        bar_id));
    const float rstd = canonical_rstd(var, a.eps);
    const f2_t rr = f2(rstd, rstd);
    // y = ((z - mean) * rstd) * scale + shift for elements (2jj, 2jj+1) of
    // vector i.  ypair_w adds the shift in bf16 form (add.rn.f32.bf16 on the
    // exactly widened value: the same sum, without widening it first); the
    // FP8 kernels, whose y stays in registers for the codes, widen it (the
    // 12-pair kernel spills more with the bf16 words live).  Measured: adaln
    // 8.88 -> 8.77 us, the config-2 step 1.5644 -> 1.5616 ms.
    auto ypair = [&](int i, int jj, const f2_t (&sc)[4], const f2_t (&sh)[4]) {
      return add2(mul2_noc(mul2(zf[i][jj], rr), sc[jj]), sh[jj]);
    };
    auto ypair_w = [&](int i, int jj, const f2_t (&sc)[4], const uint4& sh) {
      return bf16x2_add_f2(word(sh, jj), mul2_noc(mul2(zf[i][jj], rr), sc[jj]));
    };

    if (!FP8) {
#pragma unroll
      for (int i = 0; i < NH; ++i) {
        if (ok(i) && store) {
          f2_t sc[4];
          mod8(0, b, col(i), sc);
          const uint4 sh = modw(1, b, col(i));
          uint4 o;
          o.x = f2bf2(ypair_w(i, 0, sc, sh));
          o.y = f2bf2(ypair_w(i, 1, sc, sh));
          o.z = f2bf2(ypair_w(i, 2, sc, sh));
          o.w = f2bf2(ypair_w(i, 3, sc, sh));
          st16(a.h + base + col(i), o);
        }
      }
    } else {
      // y is computed once and kept in registers for the amax and the codes.
      float y[NH][8];
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < NH; ++i) {
        if (ok(i)) {
          f2_t sc[4], sh[4];
          mod8(0, b, col(i), sc);
          mod8(1, b, col(i), sh);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const f2_t v = ypair(i, jj, sc, sh);
            y[i][2 * jj] = f2lo(v);
            y[i][2 * jj + 1] = f2hi(v);
            amax = max_abs2(amax, y[i][2 * jj], y[i][2 * jj + 1]);
          }
        }
      }
      amax = warp_max(amax);
      if (SPLIT) {
        if (lane == 0) xmax[h] = amax;
        named_bar_sync(bar_id, 64);
        amax = fmaxf(xmax[0], xmax[1]);
      }
      const float sc = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
      const f2_t rb = e4m3_bracket(__fdiv_rn(1.0f, sc));
      // Every vector's bracketed codes first (independent chains), then one
      // branch for the rare open pair.
      uint2 code[NH];
      bool settled = true;
#pragma unroll
      for (int i = 0; i < NH; ++i) code[i] = e4m3_try8(y[i], rb, settled);
      if (!settled) {
#pragma unroll
        for (int i = 0; i < NH; ++i) code[i] = e4m3_ieee8(y[i], sc);
      }
#pragma unroll
      for (int i = 0; i < NH; ++i) {
        if (ok(i) && store) st8(a.q + base + col(i), code[i]);
      }
      if (leader && !dead) a.s[row] = sc;
    }
    if (++s == nsw) {
      s = 0;
      ph ^= 1u;
    }
  }
  if (leader && dead) {
    // Drain the copies issued before the failed wait (bounded waits).
    for (int64_t k = jdead; k < jdead + nsw && row_of(k) < r1; ++k)
      mbar_wait(smem_addr(&bars[k % nsw]), static_cast<uint32_t>((k / nsw) & 1));
    if (pair == 0 && smods) mbar_wait(smem_addr(modbar), 0);
  }
}

// Launch plan: stages per pair, and whether the modulation slots fit in
// shared memory next to at least one stage per pair.
struct AdalnPlan {
  int nsw;
  int smods;
  int early;  // refill a stage right after the pair has read it (one more pair barrier per row)
  size_t smem;
};
static AdalnPlan adaln_plan(int64_t dim, bool has_x, size_t limit, bool long_launch, int pairs) {
  const size_t per = pairs * ((has_x ? 2 : 1) * static_cast<size_t>(dim) * 2 + sizeof(uint64_t));
  const size_t xch = pairs * kAdalnPairXchBytes + sizeof(uint64_t);
  const size_t mods = adaln_mod_bytes(dim, has_x);
  const int cap = long_launch ? kAdalnMaxStages : kAdalnShortStages;
  auto stages = [&](size_t fixed) {
    const int n = limit > fixed ? static_cast<int>((limit - fixed) / per) : 0;
    return n < cap ? n : cap;
  };
  AdalnPlan p{};
  const int with = stages(xch + mods), without = stages(xch);
  p.smods = with >= 1 && with >= without;
  p.nsw = p.smods ? with : (without < 1 ? 1 : without);
  p.smem = xch + (p.smods ? mods : 0) + p.nsw * per;
  p.early = long_launch && has_x;  // measured: helps the residual stream, not plain adaln
  return p;
}

template <bool HAS_X, bool FP8>
static cudaError_t launch_adaln(const AdalnArgs& a, cudaStream_t st) {
  const DeviceInfo& dev = device_info();
  if (dev.error != cudaSuccess) return dev.error;
  const int nc = row_chunks(a.dim);
  const bool exact = a.dim == 256 * nc;
  auto plan_for = [&](int pairs, dim3& grid) {
    const int64_t want = (a.rows + pairs - 1) / pairs;
    grid = dim3(static_cast<unsigned>(want < dev.sms ? want : dev.sms));
    return adaln_plan(a.dim, HAS_X, dev.max_smem_optin, a.rows >= kAdalnLongRowsPerCta * static_cast<int64_t>(grid.x),
                      pairs);
  };
  auto go = [&](auto kern, int pairs, const dim3& grid, const AdalnPlan& plan) -> cudaError_t {
    cudaError_t e = ensure_smem(kern, plan.smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, grid, dim3(pairs * 64), plan.smem, st, a, plan.nsw, plan.smods, plan.early);
  };
  dim3 grid;
  if constexpr (FP8) {
    if (exact && nc == 8) {
      // The 12-pair kernel for short launches whose stage fits (see kAdalnPairsFp8).
      const AdalnPlan p12 = plan_for(kAdalnPairsFp8, grid);
      const bool fits = p12.smem <= dev.max_smem_optin;
      if (fits && a.rows < kAdalnLongRowsPerCta * static_cast<int64_t>(grid.x))
        return go(adaln_fwd_kernel<kAdalnPairsFp8, 8, HAS_X, true, true>, kAdalnPairsFp8, grid, p12);
    }
  }
  const AdalnPlan plan = plan_for(kAdalnPairs, grid);
#define AFB_LAUNCH_ADALN(NC)                                                                     \
  return exact ? go(adaln_fwd_kernel<kAdalnPairs, NC, HAS_X, FP8, true>, kAdalnPairs, grid, plan) \
               : go(adaln_fwd_kernel<kAdalnPairs, NC, HAS_X, FP8, false>, kAdalnPairs, grid, plan)
  switch (nc) {
    case 1: AFB_LAUNCH_ADALN(1);
    case 2: AFB_LAUNCH_ADALN(2);
    case 4: AFB_LAUNCH_ADALN(4);
    case 8: AFB_LAUNCH_ADALN(8);
    case 16: AFB_LAUNCH_ADALN(16);
    default: return cudaErrorInvalidValue;
  }
#undef AFB_LAUNCH_ADALN
}

cudaError_t read_status_adaln_fwd(int* status, bool clear) { return tu_status(status, clear); }

}  // namespace afb

using namespace afb;

extern "C" int afb_residual_adaln(const void* x, const void* residual, const void* gate,
                                  const void* shift, const void* scale, void* h, void* z,
                                  int64_t batch, int64_t seq, int64_t dim, float eps,
                                  void* stream) {
  ApiGuard g("afb_residual_adaln");
  if (!check_rows(batch, seq, dim) ||
      !check_ptrs({x, residual, gate, shift, scale, h, z},
                  {"x", "residual", "gate", "shift", "scale", "h", "z"}))
    return g.fail();
  if (batch * seq == 0) return 0;
  AdalnArgs a{};
  a.x = static_cast<const uint16_t*>(x);
  a.res = static_cast<const uint16_t*>(residual);
  a.gate = static_cast<const uint16_t*>(gate);
  a.shift = static_cast<const uint16_t*>(shift);
  a.scale = static_cast<const uint16_t*>(scale);
  a.h = static_cast<uint16_t*>(h);
  a.z = static_cast<uint16_t*>(z);
  a.rows = batch * seq;
  a.seq = seq;
  a.seqd = make_divu32(seq);
  a.dim = static_cast<int>(dim);
  a.eps = eps;
  return g.done(launch_adaln<true, false>(a, static_cast<cudaStream_t>(stream)));
}

extern "C" int afb_adaln(const void* z, const void* shift, const void* scale, void* h,
                         int64_t batch, int64_t seq, int64_t dim, float eps, void* stream) {
  ApiGuard g("afb_adaln");
  if (!check_rows(batch, seq, dim) ||
      !check_ptrs({z, shift, scale, h}, {"z", "shift", "scale", "h"}))
    return g.fail();
  if (batch * seq == 0) return 0;
  AdalnArgs a{};
  a.res = static_cast<const uint16_t*>(z);
  a.shift = static_cast<const uint16_t*>(shift);
  a.scale = static_cast<const uint16_t*>(scale);
  a.h = static_cast<uint16_t*>(h);
  a.rows = batch * seq;
  a.seq = seq;
  a.seqd = make_divu32(seq);
  a.dim = static_cast<int>(dim);
  a.eps = eps;
  return g.done(launch_adaln<false, false>(a, static_cast<cudaStream_t>(stream)));
}

extern "C" int afb_residual_adaln_fp8(const void* x, const void* residual, const void* gate,
                                      const void* shift, const void* scale, void* q, void* s,
                                      void* z, int64_t batch, int64_t seq, int64_t dim,
                                      float eps, void* stream) {
  ApiGuard g("afb_residual_adaln_fp8");
  if (!check_rows(batch, seq, dim) ||
      !check_ptrs({x, residual, gate, shift, scale, z}, {"x", "residual", "gate", "shift", "scale", "z"}) ||
      !check_ptr8(q, "q") || !check_ptr4(s, "s"))
    return g.fail();
  if (batch * seq == 0) return 0;
  AdalnArgs a{};
  a.x = static_cast<const uint16_t*>(x);
  a.res = static_cast<const uint16_t*>(residual);
  a.gate = static_cast<const uint16_t*>(gate);
  a.shift = static_cast<const uint16_t*>(shift);
  a.scale = static_cast<const uint16_t*>(scale);
  a.q = static_cast<uint8_t*>(q);
  a.s = static_cast<float*>(s);
  a.z = static_cast<uint16_t*>(z);
  a.rows = batch * seq;
  a.seq = seq;
  a.seqd = make_divu32(seq);
  a.dim = static_cast<int>(dim);
  a.eps = eps;
  return g.done(launch_adaln<true, true>(a, static_cast<cudaStream_t>(stream)));
}

extern "C" int afb_adaln_fp8(const void* z, const void* shift, const void* scale, void* q,
                             void* s, int64_t batch, int64_t seq, int64_t dim, float eps,
                             void* stream) {
  ApiGuard g("afb_adaln_fp8");
  if (!check_rows(batch, seq, dim) ||
      !check_ptrs({z, shift, scale}, {"z", "shift", "scale"}) ||
      !check_ptr8(q, "q") || !check_ptr4(s, "s"))
    return g.fail();
  if (batch * seq == 0) return 0;
  AdalnArgs a{};
  a.res = static_cast<const uint16_t*>(z);
  a.shift = static_cast<const uint16_t*>(shift);
  a.scale = static_cast<const uint16_t*>(scale);
  a.q = static_cast<uint8_t*>(q);
  a.s = static_cast<float*>(s);
  a.rows = batch * seq;
  a.seq = seq;
  a.seqd = make_divu32(seq);
  a.dim = static_cast<int>(dim);
  a.eps = eps;
  return g.done(launch_adaln<false, true>(a, static_cast<cudaStream_t>(stream)));
}
