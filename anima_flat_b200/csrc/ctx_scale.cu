// Trimmed-context gain of the cross attention, forward and backward.
//
// Reference: src/kernels/ctx_scale.py:8-37 (_ctx_scale_kernel) and :61-100
// (_ctx_scale_bwd_kernel); called from src/attention.py:180.  Per token s of
// batch entry b and head h, with lse [B, H, S] the attention log-sum-exp over
// the kept keys and ln_pad[b] the log of the number of removed padding keys:
//   gain = 1 / (1 + exp(ln_pad[b] - lse[b, h, s]))
//   y    = bf16(x * gain)                               (x = out [B, S, H, hd])
// Backward:
//   dout = bf16(dy * gain)
//   dlse = (sum(dy * x) * gain) * (1 - gain)            (sum over the head's hd)
// exp is canonical_exp (afb_device.cuh); the head sum is the canonical sum
// with P = hd/8 partials, as the head norms use.
//
// Layout: one token per warp at a time; warps of a CTA take consecutive tokens
// of the CTA's contiguous range, so the lse values of neighbouring tokens
// (contiguous in [B, H, S]) share L1 lines.  A head spans L = hd/16 lanes;
// lane l of a head holds dims [8l, 8l+8) and [hd/2 + 8l, hd/2 + 8l + 8), i.e.
// vectors l and l + L of the head's hd/8, so the canonical sum takes its first
// stride level in the lane and the rest as an xor butterfly over the L lanes.
// All of a token's loads are issued before any use.
#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

struct CtxScaleArgs {
  const uint16_t* out;   // [B, S, H, hd]
  const float* lse;      // [B, H, S]
  const float* ln_pad;   // [B]
  const uint16_t* dy;    // [B, S, H, hd] (backward)
  uint16_t* y;           // [B, S, H, hd] (forward)
  uint16_t* dout;        // [B, S, H, hd] (backward)
  float* dlse;           // [B, H, S] (backward)
  int64_t tokens;
  int64_t seq;
  DivU32 seqd;  // division by seq
  int heads;
};

constexpr int kCtxWarps = 16;

// MAXIT: the most head iterations a token needs (heads * hd <= 2048).
template <int HD, bool BWD>
__global__ void __launch_bounds__(kCtxWarps * 32)
ctx_scale_kernel(const CtxScaleArgs a) {
  constexpr int L = HD / 16;
  constexpr int HPI = 32 / L;
  constexpr int HALF = HD / 2;
  constexpr int MAXIT = 2048 / (HPI * HD);
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int l = lane % L;
  const int hsub = lane / L;
  const int H = a.heads;
  const int iters = (H + HPI - 1) / HPI;
  const int64_t t0 = a.tokens * blockIdx.x / gridDim.x;
  const int64_t t1 = a.tokens * (blockIdx.x + 1) / gridDim.x;
  for (int64_t tok = t0 + warp; tok < t1; tok += kCtxWarps) {
    const int64_t b = div_u32(a.seqd, tok);
    const int64_t s = tok - b * a.seq;
    const int64_t base = tok * static_cast<int64_t>(H) * HD;
    const float lnp = __ldg(a.ln_pad + b);
    uint4 xa[MAXIT], xb[MAXIT], ga[MAXIT], gb[MAXIT];
    float lse[MAXIT];
#pragma unroll
    for (int it = 0; it < MAXIT; ++it) {
      const int h = it * HPI + hsub;
      const bool hv = it < iters && h < H;
      const int64_t o = base + static_cast<int64_t>(h) * HD + 8 * l;
      xa[it] = hv ? ld_stream(a.out + o) : make_uint4(0, 0, 0, 0);
      xb[it] = hv ? ld_stream(a.out + o + HALF) : make_uint4(0, 0, 0, 0);
      if (BWD) {
        ga[it] = hv ? ld_stream(a.dy + o) : make_uint4(0, 0, 0, 0);
        gb[it] = hv ? ld_stream(a.dy + o + HALF) : make_uint4(0, 0, 0, 0);
      }
      lse[it] = hv ? __ldg(a.lse + (b * H + h) * a.seq + s) : 0.0f;
    }
#pragma unroll
    for (int it = 0; it < MAXIT; ++it) {
      if (it >= iters) break;  // warp-uniform
      const int h = it * HPI + hsub;
      const bool hv = h < H;
      const int64_t o = base + static_cast<int64_t>(h) * HD + 8 * l;
      const float gain = ctx_gain(lnp, lse[it]);
      float fa[8], fb[8];
      unpack8(xa[it], fa);
      unpack8(xb[it], fb);
      if (!BWD) {
        float oa[8], ob[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          oa[k] = __fmul_rn(fa[k], gain);
          ob[k] = __fmul_rn(fb[k], gain);
        }
        if (hv) {
          st16(a.y + o, pack8_rn(oa));
          st16(a.y + o + HALF, pack8_rn(ob));
        }
      } else {
        float da[8], db[8], pa[8], pb[8];
        unpack8(ga[it], da);
        unpack8(gb[it], db);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          pa[k] = __fmul_rn(da[k], fa[k]);
          pb[k] = __fmul_rn(db[k], fb[k]);
          fa[k] = __fmul_rn(da[k], gain);
          fb[k] = __fmul_rn(db[k], gain);
        }
        // canonical head sum: vectors l and l + L in the lane, then the lanes
        float sum = __fadd_rn(vec_sum8(pa), vec_sum8(pb));
#pragma unroll
        for (int off = L / 2; off >= 1; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(kFull, sum, off));
        if (hv) {
          st16(a.dout + o, pack8_rn(fa));
          st16(a.dout + o + HALF, pack8_rn(fb));
          if (l == 0) a.dlse[(b * H + h) * a.seq + s] = __fmul_rn(__fmul_rn(sum, gain), __fsub_rn(1.0f, gain));
        }
      }
    }
  }
}

template <bool BWD>
static cudaError_t launch_ctx_scale(const CtxScaleArgs& a, int hd, cudaStream_t st) {
  const DeviceInfo& dev = device_info();
  if (dev.error != cudaSuccess) return dev.error;
  // Every SM busy (two CTAs each), down to one token per warp.
  const int64_t want = (a.tokens + kCtxWarps - 1) / kCtxWarps;
  const int64_t cap = static_cast<int64_t>(dev.sms) * 2;
  const dim3 grid(static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap)));
  const dim3 block(kCtxWarps * 32);
  switch (hd) {
    case 64: return launch_pdl(ctx_scale_kernel<64, BWD>, grid, block, 0, st, a);
    case 128: return launch_pdl(ctx_scale_kernel<128, BWD>, grid, block, 0, st, a);
    case 256: return launch_pdl(ctx_scale_kernel<256, BWD>, grid, block, 0, st, a);
    default: return cudaErrorInvalidValue;
  }
}

static bool check_ctx(int64_t batch, int64_t seq, int64_t heads, int64_t hd) {
  return check(batch >= 0, "batch must be >= 0") && check(seq >= 1, "seq must be >= 1") &&
         check(heads >= 1 && heads * hd <= 2048,
               "heads * head_dim must be in [1, 2048], got " + std::to_string(heads * hd)) &&
         check(hd == 64 || hd == 128 || hd == 256,
               "head_dim must be 64, 128 or 256, got " + std::to_string(hd));
}

}  // namespace afb

using namespace afb;

extern "C" int afb_ctx_scale(const void* out, const void* lse, const void* ln_pad, void* y,
                             int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
                             void* stream) {
  ApiGuard g("afb_ctx_scale");
  if (!check_ctx(batch, seq, heads, head_dim) || !check_ptrs({out, y}, {"out", "y"}) ||
      !check_ptr4(lse, "lse") || !check_ptr4(ln_pad, "ln_pad"))
    return g.fail();
  if (batch * seq == 0) return 0;
  CtxScaleArgs a{};
  a.out = static_cast<const uint16_t*>(out);
  a.lse = static_cast<const float*>(lse);
  a.ln_pad = static_cast<const float*>(ln_pad);
  a.y = static_cast<uint16_t*>(y);
  a.tokens = batch * seq;
  a.seq = seq;
  a.seqd = make_divu32(seq);
  a.heads = static_cast<int>(heads);
  return g.done(launch_ctx_scale<false>(a, static_cast<int>(head_dim), static_cast<cudaStream_t>(stream)));
}

extern "C" int afb_ctx_scale_bwd(const void* out, const void* lse, const void* ln_pad, const void* dy,
                                 void* dout, void* dlse, int64_t batch, int64_t seq, int64_t heads,
                                 int64_t head_dim, void* stream) {
  ApiGuard g("afb_ctx_scale_bwd");
  if (!check_ctx(batch, seq, heads, head_dim) || !check_ptrs({out, dy, dout}, {"out", "dy", "dout"}) ||
      !check_ptr4(lse, "lse") || !check_ptr4(ln_pad, "ln_pad") || !check_ptr4(dlse, "dlse"))
    return g.fail();
  if (batch * seq == 0) return 0;
  CtxScaleArgs a{};
  a.out = static_cast<const uint16_t*>(out);
  a.lse = static_cast<const float*>(lse);
  a.ln_pad = static_cast<const float*>(ln_pad);
  a.dy = static_cast<const uint16_t*>(dy);
  a.dout = static_cast<uint16_t*>(dout);
  a.dlse = static_cast<float*>(dlse);
  a.tokens = batch * seq;
  a.seq = seq;
  a.seqd = make_divu32(seq);
  a.heads = static_cast<int>(heads);
  return g.done(launch_ctx_scale<true>(a, static_cast<int>(head_dim), static_cast<cudaStream_t>(stream)));
}
