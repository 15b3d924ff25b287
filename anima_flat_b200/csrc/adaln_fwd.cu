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
// Layout: persistent CTAs, one per SM, of kAdalnWarps warps.  Warp g of the
// grid owns rows g, g + W, g + 2W, ... (W = warps in the grid) and keeps a
// private ring of `nsw` shared-memory stages; lane 0 streams each row's res
// (and x) into a stage with bulk copies (TMA engine) that complete on the
// stage's mbarrier, so up to nsw rows per warp are in flight while the warp
// computes.  A row moves from its stage into registers (lane l holds the
// 16-byte vectors v = l + 32*c, c < NC), the stage is refilled at once, and
// z and h (or q) are written straight from registers.  z = res + gate*x uses
// packed bf16x2 arithmetic; the statistics and the modulation use packed
// fp32x2 adds/subs under the contraction rule of afb_device.cuh.
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
  int dim;
  float eps;
};

constexpr int kAdalnWarps = 8;
constexpr int kAdalnMaxStages = 4;

// EXACT: dim == 256 * NC, so every lane owns NC full vectors (no masking).
template <int NC, bool HAS_X, bool FP8, bool EXACT>
__global__ void __launch_bounds__(kAdalnWarps * 32, 1)
adaln_fwd_kernel(const AdalnArgs a, const int nsw) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int D = EXACT ? NC * 256 : a.dim;
  const uint32_t row_bytes = static_cast<uint32_t>(D) * 2u;
  const uint32_t stage_bytes = (HAS_X ? 2u : 1u) * row_bytes;
  uint8_t* ring = smem + static_cast<size_t>(warp) * nsw * stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(kAdalnWarps) * nsw * stage_bytes) +
                   warp * nsw;
  if (lane == 0) {
    for (int s = 0; s < nsw; ++s) mbar_init(smem_addr(&bars[s]), 1);
    fence_mbar_init();
  }
  __syncwarp();
  pdl_wait();
  pdl_trigger();

  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kAdalnWarps + warp;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * kAdalnWarps;
  auto issue = [&](int64_t j) {  // lane 0: stream row gw + j*nw into stage j % nsw
    const int64_t row = gw + j * nw;
    const int s = static_cast<int>(j % nsw);
    uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    const uint32_t bar = smem_addr(&bars[s]);
    mbar_arrive_expect_tx(bar, stage_bytes);
    bulk_g2s(smem_addr(st), a.res + row * D, row_bytes, bar);
    if (HAS_X) bulk_g2s(smem_addr(st + row_bytes), a.x + row * D, row_bytes, bar);
  };
  if (lane == 0) {
    for (int j = 0; j < nsw && gw + j * nw < a.rows; ++j) issue(j);
  }
  auto ok = [&](int c) { return EXACT || (lane + 32 * c) * 8 < D; };
  auto col = [&](int c) { return (lane + 32 * c) * 8; };

  for (int64_t j = 0; gw + j * nw < a.rows; ++j) {
    const int64_t row = gw + j * nw;
    const int s = static_cast<int>(j % nsw);
    const uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    if (!mbar_wait(smem_addr(&bars[s]), static_cast<uint32_t>((j / nsw) & 1))) {
      // Never expected: drain this warp's other copies (bounded), then stop.
      for (int64_t k = j + 1; k < j + nsw && gw + k * nw < a.rows; ++k)
        mbar_wait(smem_addr(&bars[k % nsw]), static_cast<uint32_t>((k / nsw) & 1));
      return;
    }
    const int64_t b = row / a.seq;
    const int64_t base = row * D;
    const int64_t pbase = b * D;

    // stage -> registers; z = bf16(res + bf16(gate * x)) in packed bf16x2
    uint4 zv[NC];
    {
      uint4 xv[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        zv[c] = ok(c) ? lds16(st + col(c) * 2) : make_uint4(0, 0, 0, 0);
        if (HAS_X) xv[c] = ok(c) ? lds16(st + row_bytes + col(c) * 2) : make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
      if (lane == 0 && gw + (j + nsw) * nw < a.rows) {
        fence_proxy_async_smem();
        issue(j + nsw);
      }
      if (HAS_X) {
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          if (ok(c)) {
            const uint4 g = ld_keep(a.gate + pbase + col(c));
            zv[c].x = badd2(zv[c].x, bmul2(g.x, xv[c].x));
            zv[c].y = badd2(zv[c].y, bmul2(g.y, xv[c].y));
            zv[c].z = badd2(zv[c].z, bmul2(g.z, xv[c].z));
            zv[c].w = badd2(zv[c].w, bmul2(g.w, xv[c].w));
            st16(a.z + base + col(c), zv[c]);
          }
        }
      }
    }

    // Statistics (canonical order, see afb_device.cuh), packed fp32x2.
    // x / D; for EXACT, D = 256 * NC is a power of two and x * (1/D) rounds identically
    auto div_d = [&](float x) {
      return EXACT ? __fmul_rn(x, 1.0f / (NC * 256)) : __fdiv_rn(x, static_cast<float>(D));
    };
    const float mean = div_d(
        warp_canonical_sum2_fn<NC>([&](int c, int jj) { return bf2f2(word(zv[c], jj)); }));
    const f2_t mm = f2(mean, mean);
    const float var = div_d(warp_canonical_sum2_fn<NC>([&](int c, int jj) {
      const f2_t d = ok(c) ? sub2(bf2f2(word(zv[c], jj)), mm) : 0ull;
      return mul2_noc(d, d);
    }));
    const float rstd = canonical_rstd(var, a.eps);
    const f2_t rr = f2(rstd, rstd);
    // y = ((z - mean) * rstd) * scale + shift for elements (2jj, 2jj+1) of vector c
    auto ypair = [&](int c, int jj, const uint4& scv, const uint4& shv) {
      const f2_t d = sub2(bf2f2(word(zv[c], jj)), mm);
      return add2(mul2_noc(mul2(d, rr), bf2f2(word(scv, jj))), bf2f2(word(shv, jj)));
    };

    if (!FP8) {
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        if (ok(c)) {
          const uint4 scv = ld_keep(a.scale + pbase + col(c));
          const uint4 shv = ld_keep(a.shift + pbase + col(c));
          uint4 o;
          o.x = f2bf2(ypair(c, 0, scv, shv));
          o.y = f2bf2(ypair(c, 1, scv, shv));
          o.z = f2bf2(ypair(c, 2, scv, shv));
          o.w = f2bf2(ypair(c, 3, scv, shv));
          st16(a.h + base + col(c), o);
        }
      }
    } else {
      float amax = 0.0f;
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        if (ok(c)) {
          const uint4 scv = ld_keep(a.scale + pbase + col(c));
          const uint4 shv = ld_keep(a.shift + pbase + col(c));
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const f2_t y = ypair(c, jj, scv, shv);
            amax = fmaxf(amax, fmaxf(fabsf(f2lo(y)), fabsf(f2hi(y))));
          }
        }
      }
      amax = warp_max(amax);
      const float sc = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        if (ok(c)) {
          const uint4 scv = ld_keep(a.scale + pbase + col(c));
          const uint4 shv = ld_keep(a.shift + pbase + col(c));
          float qf[8];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const f2_t y = ypair(c, jj, scv, shv);
            qf[2 * jj] = fminf(fmaxf(__fdiv_rn(f2lo(y), sc), -448.0f), 448.0f);
            qf[2 * jj + 1] = fminf(fmaxf(__fdiv_rn(f2hi(y), sc), -448.0f), 448.0f);
          }
          st8(a.q + base + col(c), e4m3x8(qf));
        }
      }
      if (lane == 0) a.s[row] = sc;
    }
  }
}

// Stages per warp that fit the shared-memory budget (at least one).
static int adaln_stages(int64_t dim, bool has_x, size_t smem_limit) {
  const size_t stage = (has_x ? 2 : 1) * static_cast<size_t>(dim) * 2;
  const size_t per = kAdalnWarps * (stage + sizeof(uint64_t));
  const int n = static_cast<int>(smem_limit / per);
  return n < 1 ? 1 : (n > kAdalnMaxStages ? kAdalnMaxStages : n);
}

template <bool HAS_X, bool FP8>
static cudaError_t launch_adaln(const AdalnArgs& a, cudaStream_t st) {
  const DeviceInfo& dev = device_info();
  if (dev.error != cudaSuccess) return dev.error;
  const int nc = row_chunks(a.dim);
  const bool exact = a.dim == 256 * nc;
  const int nsw = adaln_stages(a.dim, HAS_X, dev.max_smem_optin);
  const size_t smem = static_cast<size_t>(kAdalnWarps) * nsw *
                      ((HAS_X ? 2 : 1) * static_cast<size_t>(a.dim) * 2 + sizeof(uint64_t));
  const int64_t want = (a.rows + kAdalnWarps - 1) / kAdalnWarps;
  const dim3 grid(static_cast<unsigned>(want < dev.sms ? want : dev.sms));
  const dim3 block(kAdalnWarps * 32);
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e = ensure_smem(kern, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, grid, block, smem, st, a, nsw);
  };
#define AFB_LAUNCH_ADALN(NC)                                            \
  return exact ? go(adaln_fwd_kernel<NC, HAS_X, FP8, true>) \
               : go(adaln_fwd_kernel<NC, HAS_X, FP8, false>)
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

cudaError_t read_status_adaln_fwd(int* status) {
  return cudaMemcpyFromSymbol(status, g_afb_device_status, sizeof(int));
}

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
  a.dim = static_cast<int>(dim);
  a.eps = eps;
  return g.done(launch_adaln<false, true>(a, static_cast<cudaStream_t>(stream)));
}
