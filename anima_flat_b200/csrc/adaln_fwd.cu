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
// Layout: one warp per row; lane l holds the 16-byte vectors v = l + 32*c of
// the row (c < NC), so each warp-wide access covers 512 contiguous bytes.  The
// row lives in registers between the statistics and the output pass: x and
// res are read once, z and h (or q) written once.
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

template <int NC, bool HAS_X, bool FP8>
__global__ void __launch_bounds__(kRowWarps * 32)
adaln_fwd_kernel(const AdalnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const int D = a.dim;
  const int64_t b = row / a.seq;
  const int64_t base = row * D;
  const int64_t pbase = b * D;

  uint4 zv[NC];
  {
    uint4 rv[NC];
    uint4 xv[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int e = (lane + 32 * c) * 8;
      const bool ok = e < D;
      rv[c] = ok ? ld_stream(a.res + base + e) : make_uint4(0, 0, 0, 0);
      if (HAS_X) xv[c] = ok ? ld_stream(a.x + base + e) : make_uint4(0, 0, 0, 0);
    }
    if (HAS_X) {
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int e = (lane + 32 * c) * 8;
        if (e < D) {
          float g[8], xf[8], rf[8], zf[8];
          unpack8(ld_keep(a.gate + pbase + e), g);
          unpack8(xv[c], xf);
          unpack8(rv[c], rf);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float p = round_bf(__fmul_rn(g[k], xf[k]));
            zf[k] = __fadd_rn(rf[k], p);
          }
          zv[c] = pack8_rn(zf);
          st16(a.z + base + e, zv[c]);
        } else {
          zv[c] = make_uint4(0, 0, 0, 0);
        }
      }
    } else {
#pragma unroll
      for (int c = 0; c < NC; ++c) zv[c] = rv[c];
    }
  }

  // Statistics (canonical order, see afb_device.cuh).
  const float fd = static_cast<float>(D);
  const float mean = __fdiv_rn(
      warp_canonical_sum_fn<NC>([&](int c, int k) { return unpack_at(zv[c], k); }), fd);
  const float var = __fdiv_rn(warp_canonical_sum_fn<NC>([&](int c, int k) {
                                const float d = ((lane + 32 * c) * 8 < D)
                                                    ? __fsub_rn(unpack_at(zv[c], k), mean)
                                                    : 0.0f;
                                return __fmul_rn(d, d);
                              }),
                              fd);
  const float rstd = canonical_rstd(var, a.eps);

  if (!FP8) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int e = (lane + 32 * c) * 8;
      if (e < D) {
        float sc[8], sh[8], y[8];
        unpack8(ld_keep(a.scale + pbase + e), sc);
        unpack8(ld_keep(a.shift + pbase + e), sh);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float d = __fsub_rn(unpack_at(zv[c], k), mean);
          y[k] = __fadd_rn(__fmul_rn(__fmul_rn(d, rstd), sc[k]), sh[k]);
        }
        st16(a.h + base + e, pack8_rn(y));
      }
    }
  } else {
    float y[NC][8];
    float amax = 0.0f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int e = (lane + 32 * c) * 8;
      if (e < D) {
        float sc[8], sh[8];
        unpack8(ld_keep(a.scale + pbase + e), sc);
        unpack8(ld_keep(a.shift + pbase + e), sh);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float d = __fsub_rn(unpack_at(zv[c], k), mean);
          y[c][k] = __fadd_rn(__fmul_rn(__fmul_rn(d, rstd), sc[k]), sh[k]);
          amax = fmaxf(amax, fabsf(y[c][k]));
        }
      }
    }
    amax = warp_max(amax);
    const float s = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int e = (lane + 32 * c) * 8;
      if (e < D) {
        float qf[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          qf[k] = fminf(fmaxf(__fdiv_rn(y[c][k], s), -448.0f), 448.0f);
        }
        st8(a.q + base + e, e4m3x8(qf));
      }
    }
    if (lane == 0) a.s[row] = s;
  }
}

template <bool HAS_X, bool FP8>
static cudaError_t launch_adaln(const AdalnArgs& a, cudaStream_t st) {
  const int nc = row_chunks(a.dim);
  const dim3 grid(static_cast<unsigned>((a.rows + kRowWarps - 1) / kRowWarps));
  const dim3 block(kRowWarps * 32);
  switch (nc) {
    case 1: return launch_pdl(adaln_fwd_kernel<1, HAS_X, FP8>, grid, block, 0, st, a);
    case 2: return launch_pdl(adaln_fwd_kernel<2, HAS_X, FP8>, grid, block, 0, st, a);
    case 4: return launch_pdl(adaln_fwd_kernel<4, HAS_X, FP8>, grid, block, 0, st, a);
    case 8: return launch_pdl(adaln_fwd_kernel<8, HAS_X, FP8>, grid, block, 0, st, a);
    case 16: return launch_pdl(adaln_fwd_kernel<16, HAS_X, FP8>, grid, block, 0, st, a);
    default: return cudaErrorInvalidValue;
  }
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
