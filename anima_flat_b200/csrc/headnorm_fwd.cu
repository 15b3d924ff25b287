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
// Layout: persistent CTAs, one per SM, of kHeadWarps warps; warp g of the grid
// owns tokens g, g + W, ... and keeps a private ring of shared-memory stages.
// Lane 0 streams each token's normed sections (q|k, contiguous in the qkv
// row; with v the whole row) into a stage with one bulk copy (TMA engine)
// completing on the stage's mbarrier.  A head spans L = hd/16 lanes; lane l
// of a head holds dims [8l, 8l+8) of the first half and the same dims of the
// second half, so the rotation pairs (i, i + hd/2) sit in one lane and the
// canonical per-head sum (P = hd/8 partials) takes its first stride level in
// the lane, then an xor butterfly over the L lanes.  32/L heads go per warp
// iteration; each shared-memory read and global store covers whole 128-byte
// lines of a head.
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

constexpr int kHeadWarps = 16;
constexpr int kHeadMaxStages = 4;
constexpr int kHeadUnroll = 4;

template <int HD, bool ROTATE, bool WITH_K, bool WITH_V>
__global__ void __launch_bounds__(kHeadWarps * 32, 1)
headnorm_fwd_kernel(const HeadNormArgs a, const int nsw) {
  constexpr int L = HD / 16;     // lanes per head
  constexpr int HPI = 32 / L;    // heads per warp iteration
  constexpr int HALF = HD / 2;
  constexpr int NSEC = WITH_K ? 2 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int l = lane % L;
  const int hsub = lane / L;
  const int H = a.heads;
  const int iters = (H + HPI - 1) / HPI;
  const uint32_t sec_bytes = static_cast<uint32_t>(H) * HD * 2u;
  // q (and k) are contiguous at the start of the row; with v the whole row.
  const uint32_t stage_bytes = sec_bytes * (NSEC + (WITH_V ? 1u : 0u));
  uint8_t* ring = smem + static_cast<size_t>(warp) * nsw * stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(kHeadWarps) * nsw * stage_bytes) +
                   warp * nsw;
  if (lane == 0) {
    for (int s = 0; s < nsw; ++s) mbar_init(smem_addr(&bars[s]), 1);
    fence_mbar_init();
  }
  __syncwarp();
  pdl_wait();
  pdl_trigger();

  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kHeadWarps + warp;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * kHeadWarps;
  auto issue = [&](int64_t t) {  // lane 0: stream token gw + t*nw into stage t % nsw
    const int64_t tok = gw + t * nw;
    const int s = static_cast<int>(t % nsw);
    const uint32_t bar = smem_addr(&bars[s]);
    mbar_arrive_expect_tx(bar, stage_bytes);
    bulk_g2s(smem_addr(ring + static_cast<size_t>(s) * stage_bytes), a.src + tok * a.src_row + a.q_off,
             stage_bytes, bar);
  };
  if (lane == 0) {
    for (int t = 0; t < nsw && gw + t * nw < a.tokens; ++t) issue(t);
  }

  for (int64_t t = 0; gw + t * nw < a.tokens; ++t) {
    const int64_t tok = gw + t * nw;
    const int s = static_cast<int>(t % nsw);
    const uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    float cs[8], sn[8];
    if (ROTATE) {  // issued before the wait: the tables do not depend on the stage
      const int64_t pos = tok % a.seq;
      const float* cp = a.cos + pos * HALF + 8 * l;
      const float* sp = a.sin + pos * HALF + 8 * l;
      const float4 c0 = ld_keep_f4(cp), c1 = ld_keep_f4(cp + 4);
      const float4 s0 = ld_keep_f4(sp), s1 = ld_keep_f4(sp + 4);
      cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w;
      cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
      sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
      sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
    }
    if (!mbar_wait(smem_addr(&bars[s]), static_cast<uint32_t>((t / nsw) & 1))) {
      for (int64_t k = t + 1; k < t + nsw && gw + k * nw < a.tokens; ++k)
        mbar_wait(smem_addr(&bars[k % nsw]), static_cast<uint32_t>((k / nsw) & 1));
      return;
    }
    const int64_t out_base = tok * static_cast<int64_t>(H) * HD;
#pragma unroll
    for (int sec = 0; sec < NSEC; ++sec) {
      const uint8_t* in = st + sec * sec_bytes;
      uint16_t* out = (sec ? a.out_k : a.out_q) + out_base;
      float wa[8], wb[8];
      {
        const float* wp = (sec ? a.wk : a.wq) + 8 * l;
        const float4 w0 = ld_keep_f4(wp), w1 = ld_keep_f4(wp + 4);
        const float4 w2 = ld_keep_f4(wp + HALF), w3 = ld_keep_f4(wp + HALF + 4);
        wa[0] = w0.x; wa[1] = w0.y; wa[2] = w0.z; wa[3] = w0.w;
        wa[4] = w1.x; wa[5] = w1.y; wa[6] = w1.z; wa[7] = w1.w;
        wb[0] = w2.x; wb[1] = w2.y; wb[2] = w2.z; wb[3] = w2.w;
        wb[4] = w3.x; wb[5] = w3.y; wb[6] = w3.z; wb[7] = w3.w;
      }
      for (int it0 = 0; it0 < iters; it0 += kHeadUnroll) {
        uint4 va[kHeadUnroll], vb[kHeadUnroll];
        float ss[kHeadUnroll];
#pragma unroll
        for (int u = 0; u < kHeadUnroll; ++u) {
          const int h = (it0 + u) * HPI + hsub;
          const bool hv = it0 + u < iters && h < H;
          va[u] = hv ? lds16(in + (h * HD + 8 * l) * 2) : make_uint4(0, 0, 0, 0);
          vb[u] = hv ? lds16(in + (h * HD + HALF + 8 * l) * 2) : make_uint4(0, 0, 0, 0);
          float fa[8], fb[8];
          unpack8(va[u], fa);
          unpack8(vb[u], fb);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            fa[k] = __fmul_rn(fa[k], fa[k]);
            fb[k] = __fmul_rn(fb[k], fb[k]);
          }
          ss[u] = __fadd_rn(vec_sum8(fa), vec_sum8(fb));  // partials v and v + L
        }
#pragma unroll
        for (int o = L / 2; o >= 1; o >>= 1) {
#pragma unroll
          for (int u = 0; u < kHeadUnroll; ++u) ss[u] = __fadd_rn(ss[u], __shfl_xor_sync(kFull, ss[u], o));
        }
#pragma unroll
        for (int u = 0; u < kHeadUnroll; ++u) {
          if (it0 + u >= iters) break;  // warp-uniform
          const int h = (it0 + u) * HPI + hsub;
          // ss / HD with HD a power of two: the product by 1/HD rounds identically
          const float rstd = canonical_rstd(__fmul_rn(ss[u], 1.0f / HD), a.eps);
          const f2_t rr = f2(rstd, rstd);
          uint4 na, nb;  // bf16((x * rstd) * w), exact pairs of bf16
          {
            float fa[8], fb[8];
            unpack8(va[u], fa);
            unpack8(vb[u], fb);
            uint32_t* pa = &na.x;
            uint32_t* pb = &nb.x;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              pa[k] = f2bf2(mul2(mul2(f2(fa[2 * k], fa[2 * k + 1]), rr), f2(wa[2 * k], wa[2 * k + 1])));
              pb[k] = f2bf2(mul2(mul2(f2(fb[2 * k], fb[2 * k + 1]), rr), f2(wb[2 * k], wb[2 * k + 1])));
            }
          }
          if (ROTATE) {
            float fa[8], fb[8], oa[8], ob[8];
            unpack8(na, fa);
            unpack8(nb, fb);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              oa[k] = __fsub_rn(__fmul_rn(fa[k], cs[k]), __fmul_rn(fb[k], sn[k]));
              ob[k] = __fadd_rn(__fmul_rn(fb[k], cs[k]), __fmul_rn(fa[k], sn[k]));
            }
            na = pack8_rn(oa);
            nb = pack8_rn(ob);
          }
          if (h < H) {
            st16(out + h * HD + 8 * l, na);
            st16(out + h * HD + HALF + 8 * l, nb);
          }
        }
      }
    }
    if (WITH_V) {
      const uint8_t* in = st + NSEC * sec_bytes;
      uint16_t* out = a.out_v + out_base;
      const int nvec = H * HD / 8;
      for (int v = lane; v < nvec; v += 32) st16(out + 8 * v, lds16(in + 16 * v));
    }
    __syncwarp();
    if (lane == 0 && gw + (t + nsw) * nw < a.tokens) {
      fence_proxy_async_smem();
      issue(t + nsw);
    }
  }
}

template <bool ROTATE, bool WITH_K, bool WITH_V>
static cudaError_t launch_headnorm(const HeadNormArgs& a, int hd, cudaStream_t st) {
  const DeviceInfo& dev = device_info();
  if (dev.error != cudaSuccess) return dev.error;
  const size_t stage = static_cast<size_t>(a.heads) * hd * 2 *
                       ((WITH_K ? 2 : 1) + (WITH_V ? 1 : 0));
  const size_t per = kHeadWarps * (stage + sizeof(uint64_t));
  int nsw = static_cast<int>(dev.max_smem_optin / per);
  if (nsw < 1) return cudaErrorInvalidValue;  // caller bounds heads * head_dim
  if (nsw > kHeadMaxStages) nsw = kHeadMaxStages;
  const size_t smem = per * nsw;
  const int64_t want = (a.tokens + kHeadWarps - 1) / kHeadWarps;
  const dim3 grid(static_cast<unsigned>(want < dev.sms ? want : dev.sms));
  const dim3 block(kHeadWarps * 32);
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e = ensure_smem(kern, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, grid, block, smem, st, a, nsw);
  };
  switch (hd) {
    case 64: return go(headnorm_fwd_kernel<64, ROTATE, WITH_K, WITH_V>);
    case 128: return go(headnorm_fwd_kernel<128, ROTATE, WITH_K, WITH_V>);
    case 256: return go(headnorm_fwd_kernel<256, ROTATE, WITH_K, WITH_V>);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t read_status_headnorm_fwd(int* status) {
  return cudaMemcpyFromSymbol(status, g_afb_device_status, sizeof(int));
}

inline bool check_heads(int64_t batch, int64_t seq, int64_t heads, int64_t hd) {
  return check(batch >= 0, "batch must be >= 0") && check(seq >= 1, "seq must be >= 1") &&
         check(heads >= 1 && heads * hd <= 2048,
               "heads * head_dim must be in [1, 2048], got " + std::to_string(heads * hd)) &&
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
