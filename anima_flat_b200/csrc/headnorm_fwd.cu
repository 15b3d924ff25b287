// Per-head RMSNorm of q and k fused with the rotate-half 3D RoPE, and the
// plain per-head RMSNorm of the cross-attention queries.
//
// Reference: src/kernels/rope.py:12-58 (_section), :61-143
// (_qkv_norm_rope_kernel), :146-172 (_head_norm_kernel).  Per token and head,
// with a = dims [0, hd/2) and b = dims [hd/2, hd) of the head:
//   rstd = 1 / sqrt(sum(x*x) / hd + eps)
//   a = bf16((a * rstd) * w[:hd/2]);  b = bf16((b * rstd) * w[hd/2:])
//   rotate:  a' = bf16(a*cos - b*sin);  b' = bf16(b*cos + a*sin)
// with cos/sin rows [hd/2] fp32 taken at position = token % S (rope.py:80).
// qkv rows are [q | k | v], each heads*hd wide (rope.py:81-82); v is copied
// unchanged when requested (grad mode, rope.py:124-143).
//
// Layout: one warp per token.  A head spans LPH = hd/8 lanes holding 8
// contiguous dims each, so 32/LPH heads go per warp iteration, each warp-wide
// access covering 512 contiguous bytes; the rotation partner (dim +- hd/2) is
// the lane LPH/2 away in the same head.
#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

struct HeadNormArgs {
  const uint16_t* src;   // token rows of bf16
  int64_t src_row;       // elements per token row of src
  int64_t q_off;         // column of the first (normed) section
  int64_t k_off;         // column of the second normed section (WITH_K)
  int64_t v_off;         // column of the copied section (WITH_V)
  const float* wq;       // [hd] fp32
  const float* wk;       // [hd] fp32 (WITH_K)
  const float* cos;      // [S, hd/2] fp32 (ROTATE)
  const float* sin;      // [S, hd/2] fp32 (ROTATE)
  uint16_t* out_q;       // [tokens, heads, hd] bf16
  uint16_t* out_k;       // [tokens, heads, hd] bf16 (WITH_K)
  uint16_t* out_v;       // [tokens, heads, hd] bf16 (WITH_V)
  int64_t tokens;
  int64_t seq;
  int heads;
  float eps;
};

template <int HD, bool ROTATE, bool WITH_K, bool WITH_V>
__global__ void __launch_bounds__(kRowWarps * 32)
headnorm_fwd_kernel(const HeadNormArgs a) {
  constexpr int LPH = HD / 8;
  constexpr int HPI = 32 / LPH;
  constexpr int HALF = HD / 2;
  constexpr int UNR = 8;
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t tok = static_cast<int64_t>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5);
  if (tok >= a.tokens) return;
  const int j = lane % LPH;
  const int hsub = lane / LPH;
  const int H = a.heads;
  const int iters = (H + HPI - 1) / HPI;

  float cs[8], sn[8];
  if (ROTATE) {
    const int64_t pos = tok % a.seq;
    const float* cp = a.cos + pos * HALF + (8 * j) % HALF;
    const float* sp = a.sin + pos * HALF + (8 * j) % HALF;
    const float4 c0 = ld_keep_f4(cp), c1 = ld_keep_f4(cp + 4);
    const float4 s0 = ld_keep_f4(sp), s1 = ld_keep_f4(sp + 4);
    cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w;
    cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
    sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
    sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
  }

  const uint16_t* row = a.src + tok * a.src_row;
  const int64_t out_base = tok * static_cast<int64_t>(H) * HD;
#pragma unroll
  for (int sec = 0; sec < (WITH_K ? 2 : 1); ++sec) {
    const uint16_t* in = row + (sec ? a.k_off : a.q_off);
    uint16_t* out = (sec ? a.out_k : a.out_q) + out_base;
    float w[8];
    {
      const float* wp = (sec ? a.wk : a.wq) + 8 * j;
      const float4 w0 = ld_keep_f4(wp), w1 = ld_keep_f4(wp + 4);
      w[0] = w0.x; w[1] = w0.y; w[2] = w0.z; w[3] = w0.w;
      w[4] = w1.x; w[5] = w1.y; w[6] = w1.z; w[7] = w1.w;
    }
    for (int i0 = 0; i0 < iters; i0 += UNR) {
      uint4 v[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int h = (i0 + u) * HPI + hsub;
        v[u] = (i0 + u < iters && h < H) ? ld_stream(in + h * HD + 8 * j) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        if (i0 + u >= iters) break;  // warp-uniform
        const int h = (i0 + u) * HPI + hsub;
        float f[8], sq[8], n[8];
        unpack8(v[u], f);
#pragma unroll
        for (int k = 0; k < 8; ++k) sq[k] = __fmul_rn(f[k], f[k]);
        const float ss = group_canonical_sum<LPH>(sq);
        const float rstd = canonical_rstd(__fdiv_rn(ss, static_cast<float>(HD)), a.eps);
#pragma unroll
        for (int k = 0; k < 8; ++k) n[k] = round_bf(__fmul_rn(__fmul_rn(f[k], rstd), w[k]));
        uint4 packed = pack8_rn(n);  // exact: n is already bf16
        if (ROTATE) {
          uint4 pp;
          pp.x = __shfl_xor_sync(kFull, packed.x, LPH / 2);
          pp.y = __shfl_xor_sync(kFull, packed.y, LPH / 2);
          pp.z = __shfl_xor_sync(kFull, packed.z, LPH / 2);
          pp.w = __shfl_xor_sync(kFull, packed.w, LPH / 2);
          float pf[8], o[8];
          unpack8(pp, pf);
          const bool first = j < LPH / 2;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float mc = __fmul_rn(n[k], cs[k]);
            const float ps = __fmul_rn(pf[k], sn[k]);
            o[k] = first ? __fsub_rn(mc, ps) : __fadd_rn(mc, ps);
          }
          packed = pack8_rn(o);
        }
        if (h < H) st16(out + h * HD + 8 * j, packed);
      }
    }
  }

  if (WITH_V) {
    const uint16_t* in = row + a.v_off;
    uint16_t* out = a.out_v + out_base;
    const int nvec = H * HD / 8;
    for (int i0 = 0; i0 < nvec; i0 += 32 * UNR) {
      uint4 v[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int i = i0 + 32 * u + lane;
        v[u] = i < nvec ? ld_stream(in + 8 * i) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int i = i0 + 32 * u + lane;
        if (i < nvec) st16(out + 8 * i, v[u]);
      }
    }
  }
}

template <bool ROTATE, bool WITH_K, bool WITH_V>
static cudaError_t launch_headnorm(const HeadNormArgs& a, int hd, cudaStream_t st) {
  const dim3 grid(static_cast<unsigned>((a.tokens + kRowWarps - 1) / kRowWarps));
  const dim3 block(kRowWarps * 32);
  switch (hd) {
    case 64: return launch_pdl(headnorm_fwd_kernel<64, ROTATE, WITH_K, WITH_V>, grid, block, 0, st, a);
    case 128: return launch_pdl(headnorm_fwd_kernel<128, ROTATE, WITH_K, WITH_V>, grid, block, 0, st, a);
    case 256: return launch_pdl(headnorm_fwd_kernel<256, ROTATE, WITH_K, WITH_V>, grid, block, 0, st, a);
    default: return cudaErrorInvalidValue;
  }
}

inline bool check_heads(int64_t batch, int64_t seq, int64_t heads, int64_t hd) {
  return check(batch >= 0, "batch must be >= 0") && check(seq >= 1, "seq must be >= 1") &&
         check(heads >= 1 && heads <= 1024, "heads must be in [1, 1024]") &&
         check(hd == 64 || hd == 128 || hd == 256,
               "head_dim must be 64, 128 or 256, got " + std::to_string(hd));
}

}  // namespace afb

using namespace afb;

extern "C" int afb_qkv_norm_rope(const void* qkv, const void* q_weight, const void* k_weight,
                                 const void* cos, const void* sin, void* q, void* k, void* v,
                                 int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
                                 float eps, void* stream) {
  ApiGuard g("afb_qkv_norm_rope");
  if (!check_heads(batch, seq, heads, head_dim) ||
      !check_ptrs({qkv, q_weight, k_weight, cos, sin, q, k},
                  {"qkv", "q_weight", "k_weight", "cos", "sin", "q", "k"}) ||
      (v != nullptr && !check_ptrs({v}, {"v"})))
    return g.fail();
  if (batch * seq == 0) return 0;
  HeadNormArgs a{};
  const int64_t width = heads * head_dim;
  a.src = static_cast<const uint16_t*>(qkv);
  a.src_row = 3 * width;
  a.q_off = 0;
  a.k_off = width;
  a.v_off = 2 * width;
  a.wq = static_cast<const float*>(q_weight);
  a.wk = static_cast<const float*>(k_weight);
  a.cos = static_cast<const float*>(cos);
  a.sin = static_cast<const float*>(sin);
  a.out_q = static_cast<uint16_t*>(q);
  a.out_k = static_cast<uint16_t*>(k);
  a.out_v = static_cast<uint16_t*>(v);
  a.tokens = batch * seq;
  a.seq = seq;
  a.heads = static_cast<int>(heads);
  a.eps = eps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int hd = static_cast<int>(head_dim);
  return g.done(v ? launch_headnorm<true, true, true>(a, hd, st)
                  : launch_headnorm<true, true, false>(a, hd, st));
}

extern "C" int afb_head_norm(const void* x, const void* weight, void* y, int64_t batch,
                             int64_t seq, int64_t heads, int64_t head_dim, float eps,
                             void* stream) {
  ApiGuard g("afb_head_norm");
  if (!check_heads(batch, seq, heads, head_dim) ||
      !check_ptrs({x, weight, y}, {"x", "weight", "y"}))
    return g.fail();
  if (batch * seq == 0) return 0;
  HeadNormArgs a{};
  a.src = static_cast<const uint16_t*>(x);
  a.src_row = heads * head_dim;
  a.wq = static_cast<const float*>(weight);
  a.out_q = static_cast<uint16_t*>(y);
  a.tokens = batch * seq;
  a.seq = seq;
  a.heads = static_cast<int>(heads);
  a.eps = eps;
  return g.done(launch_headnorm<false, false, false>(a, static_cast<int>(head_dim),
                                                     static_cast<cudaStream_t>(stream)));
}
