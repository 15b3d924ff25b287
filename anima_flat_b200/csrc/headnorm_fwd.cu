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
// Layout: persistent CTAs, one per SM, of kHeadWarps warps.  The work unit
// is one section of one token: its q or its k heads (normed, rotated), or its
// v (copied, grad mode); unit u is section u % NU of token u / NU.  Warp w of
// CTA c owns the units w*G + c + k*G*W (G CTAs of W warps: every SM gets the
// same share), with a private ring of shared-memory stages: two for a short
// launch (more delay each warp's first unit behind the others' copies), as
// many as fit for a long one (a steady stream, bound by the bytes in flight).  Lane 0 streams
// each unit into a stage with bulk copies (TMA engine) completing on the
// stage's mbarrier: the section, and for a rotated section the token's cos and
// sin rows, so no per-token global load sits on the critical path.  The norm
// weights are bulk-copied into shared memory first, ahead of every unit.  A head spans
// L = hd/16 lanes; lane l of a head holds dims [8l, 8l+8) of the first half
// and the same dims of the second half, so the rotation pairs (i, i + hd/2)
// sit in one lane and the canonical per-head sum (P = hd/8 partials) takes its
// first stride level in the lane, then an xor butterfly over the L lanes.
// 32/L heads go per warp iteration; each shared-memory read and global store
// covers whole 128-byte lines of a head.
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
  DivU32 seqd;           // division by seq
  int heads;
  float eps;
};

constexpr int kHeadWarps = 16;
constexpr int kHeadShortStages = 2;
constexpr int kHeadMaxStages = 4;
constexpr int64_t kHeadLongUnitsPerCta = 256;
constexpr int kHeadUnroll = 4;

template <int HD, bool ROTATE, bool WITH_K, bool WITH_V>
__global__ void __launch_bounds__(kHeadWarps * 32, 1)
headnorm_fwd_kernel(const HeadNormArgs a, const int nsw) {
  constexpr int L = HD / 16;     // lanes per head
  constexpr int HPI = 32 / L;    // heads per warp iteration
  constexpr int HALF = HD / 2;
  constexpr int NSEC = WITH_K ? 2 : 1;               // normed sections per token
  constexpr int NU = NSEC + (WITH_V ? 1 : 0);        // units per token
  constexpr uint32_t kTabBytes = ROTATE ? 2u * HALF * 4u : 0u;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int l = lane % L;
  const int hsub = lane / L;
  const int H = a.heads;
  const int iters = (H + HPI - 1) / HPI;
  const uint32_t sec_bytes = static_cast<uint32_t>(H) * HD * 2u;
  const uint32_t stage_bytes = sec_bytes + kTabBytes;
  uint8_t* ring = smem + static_cast<size_t>(warp) * nsw * stage_bytes;
  float* wsm = reinterpret_cast<float*>(smem + static_cast<size_t>(kHeadWarps) * nsw * stage_bytes);
  uint64_t* bars0 = reinterpret_cast<uint64_t*>(wsm + NSEC * HD);
  uint64_t* bars = bars0 + warp * nsw;
  uint64_t* wbar = bars0 + kHeadWarps * nsw;
  if (lane == 0) {
    for (int s = 0; s < nsw; ++s) mbar_init(smem_addr(&bars[s]), 1);
    if (warp == 0) mbar_init(smem_addr(wbar), 1);
    fence_mbar_init();
  }
  __syncthreads();  // the weight barrier is waited on by every warp
  // While the previous kernel on the stream finishes, pull each warp's first
  // unit (its section and table rows) and the norm weights into L2
  // (prefetch_l2).  Measured: the config-2 step 4.5% faster with every
  // output kept, an isolated launch unchanged.
  if (lane == 0) {
    const int64_t u = static_cast<int64_t>(warp) * gridDim.x + blockIdx.x;
    if (u < a.tokens * NU) {
      const int64_t tok = u / NU;
      const int sec = static_cast<int>(u % NU);
      const int64_t off = sec == 0 ? a.q_off : (sec == 1 && WITH_K) ? a.k_off : a.v_off;
      prefetch_l2(a.src + tok * a.src_row + off, sec_bytes);
      if (ROTATE && sec < NSEC) {
        const int64_t pos = tok - div_u32(a.seqd, tok) * a.seq;
        prefetch_l2(a.cos + pos * HALF, HALF * 4u);
        prefetch_l2(a.sin + pos * HALF, HALF * 4u);
      }
    }
    if (warp == 0) {
      prefetch_l2(a.wq, HD * 4u);
      if (WITH_K) prefetch_l2(a.wk, HD * 4u);
    }
  }
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) {
    // The norm weights go first, ahead of every unit.
    mbar_arrive_expect_tx(smem_addr(wbar), NSEC * HD * 4u);
    bulk_g2s(smem_addr(wsm), a.wq, HD * 4u, smem_addr(wbar));
    if (WITH_K) bulk_g2s(smem_addr(wsm + HD), a.wk, HD * 4u, smem_addr(wbar));
  }
  __syncthreads();

  const int64_t u1 = a.tokens * NU;  // units
  auto unit_of = [&](int64_t j) {
    return static_cast<int64_t>(warp) * gridDim.x + blockIdx.x + j * static_cast<int64_t>(gridDim.x) * kHeadWarps;
  };
  auto issue = [&](int64_t j, int s) {  // lane 0: stream unit unit_of(j) into stage s = j % nsw
    const int64_t u = unit_of(j);
    const int64_t tok = u / NU;
    const int sec = static_cast<int>(u % NU);
    uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    const uint32_t bar = smem_addr(&bars[s]);
    const bool tab = ROTATE && sec < NSEC;
    const int64_t off = sec == 0 ? a.q_off : (sec == 1 && WITH_K) ? a.k_off : a.v_off;
    mbar_arrive_expect_tx(bar, sec_bytes + (tab ? kTabBytes : 0u));
    bulk_g2s(smem_addr(st), a.src + tok * a.src_row + off, sec_bytes, bar);
    if (tab) {
      const int64_t pos = tok - div_u32(a.seqd, tok) * a.seq;
      bulk_g2s(smem_addr(st + sec_bytes), a.cos + pos * HALF, HALF * 4u, bar);
      bulk_g2s(smem_addr(st + sec_bytes + HALF * 4u), a.sin + pos * HALF, HALF * 4u, bar);
    }
  };
  if (lane == 0) {
    for (int j = 0; j < nsw && unit_of(j) < u1; ++j) issue(j, j);
  }
  if (!mbar_wait(smem_addr(wbar), 0)) {
    // Never expected: drain this warp's copies (bounded), then stop.
    for (int64_t k = 0; k < nsw && unit_of(k) < u1; ++k)
      mbar_wait(smem_addr(&bars[k % nsw]), 0);
    if (threadIdx.x == 0) mbar_wait(smem_addr(wbar), 0);
    return;
  }

  // Stage s = j % nsw of unit j and its phase parity (j / nsw) & 1, advanced
  // with j (no division in the loop).
  int s = 0;
  uint32_t ph = 0;
  for (int64_t j = 0; unit_of(j) < u1; ++j) {
    const int64_t u = unit_of(j);
    const int64_t tok = u / NU;
    const int sec = static_cast<int>(u % NU);
    const uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    if (!mbar_wait(smem_addr(&bars[s]), ph)) {
      for (int64_t k = j + 1; k < j + nsw && unit_of(k) < u1; ++k)
        mbar_wait(smem_addr(&bars[k % nsw]), static_cast<uint32_t>((k / nsw) & 1));
      return;
    }
    const int64_t out_base = tok * static_cast<int64_t>(H) * HD;
    if (WITH_V && sec == NSEC) {
      uint16_t* out = a.out_v + out_base;
      const int nvec = H * HD / 8;
      for (int v = lane; v < nvec; v += 32) st16(out + 8 * v, lds16(st + 16 * v));
    } else {
      uint16_t* out = (sec ? a.out_k : a.out_q) + out_base;
      float wa[8], wb[8], cs[8], sn[8];
      {
        const float4* wp = reinterpret_cast<const float4*>(wsm + sec * HD + 8 * l);
        const float4 w0 = wp[0], w1 = wp[1], w2 = wp[HALF / 4], w3 = wp[HALF / 4 + 1];
        wa[0] = w0.x; wa[1] = w0.y; wa[2] = w0.z; wa[3] = w0.w;
        wa[4] = w1.x; wa[5] = w1.y; wa[6] = w1.z; wa[7] = w1.w;
        wb[0] = w2.x; wb[1] = w2.y; wb[2] = w2.z; wb[3] = w2.w;
        wb[4] = w3.x; wb[5] = w3.y; wb[6] = w3.z; wb[7] = w3.w;
      }
      if (ROTATE) {
        const float4* cp = reinterpret_cast<const float4*>(st + sec_bytes) + 2 * l;
        const float4* sp = reinterpret_cast<const float4*>(st + sec_bytes + HALF * 4) + 2 * l;
        const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
        cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w;
        cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
        sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
        sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
      }
      for (int it0 = 0; it0 < iters; it0 += kHeadUnroll) {
        uint4 va[kHeadUnroll], vb[kHeadUnroll];
        float ss[kHeadUnroll];
#pragma unroll
        for (int uu = 0; uu < kHeadUnroll; ++uu) {
          const int h = (it0 + uu) * HPI + hsub;
          const bool hv = it0 + uu < iters && h < H;
          va[uu] = hv ? lds16(st + (h * HD + 8 * l) * 2) : make_uint4(0, 0, 0, 0);
          vb[uu] = hv ? lds16(st + (h * HD + HALF + 8 * l) * 2) : make_uint4(0, 0, 0, 0);
          float fa[8], fb[8];
          unpack8(va[uu], fa);
          unpack8(vb[uu], fb);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            fa[k] = __fmul_rn(fa[k], fa[k]);
            fb[k] = __fmul_rn(fb[k], fb[k]);
          }
          ss[uu] = __fadd_rn(vec_sum8(fa), vec_sum8(fb));  // partials v and v + L
        }
#pragma unroll
        for (int o = L / 2; o >= 1; o >>= 1) {
#pragma unroll
          for (int uu = 0; uu < kHeadUnroll; ++uu) ss[uu] = __fadd_rn(ss[uu], __shfl_xor_sync(kFull, ss[uu], o));
        }
#pragma unroll
        for (int uu = 0; uu < kHeadUnroll; ++uu) {
          if (it0 + uu >= iters) break;  // warp-uniform
          const int h = (it0 + uu) * HPI + hsub;
          // ss / HD with HD a power of two: the product by 1/HD rounds identically
          const float rstd = canonical_rstd(__fmul_rn(ss[uu], 1.0f / HD), a.eps);
          const f2_t rr = f2(rstd, rstd);
          uint4 na, nb;  // bf16((x * rstd) * w), exact pairs of bf16
          {
            float fa[8], fb[8];
            unpack8(va[uu], fa);
            unpack8(vb[uu], fb);
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
    __syncwarp();
    if (lane == 0 && unit_of(j + nsw) < u1) {
      fence_proxy_async_smem();
      issue(j + nsw, s);
    }
    if (++s == nsw) {
      s = 0;
      ph ^= 1u;
    }
  }
}

template <bool ROTATE, bool WITH_K, bool WITH_V>
static cudaError_t launch_headnorm(const HeadNormArgs& a, int hd, cudaStream_t st) {
  const DeviceInfo& dev = device_info();
  if (dev.error != cudaSuccess) return dev.error;
  const size_t stage = static_cast<size_t>(a.heads) * hd * 2 + (ROTATE ? static_cast<size_t>(hd) * 4 : 0);
  const size_t per = kHeadWarps * (stage + sizeof(uint64_t));
  const size_t fixed = static_cast<size_t>(WITH_K ? 2 : 1) * hd * sizeof(float) + sizeof(uint64_t);
  const int64_t units = a.tokens * ((WITH_K ? 2 : 1) + (WITH_V ? 1 : 0));
  const int64_t want = (units + kHeadWarps - 1) / kHeadWarps;
  const dim3 grid(static_cast<unsigned>(want < dev.sms ? want : dev.sms));
  const int cap = units >= kHeadLongUnitsPerCta * static_cast<int64_t>(grid.x) ? kHeadMaxStages : kHeadShortStages;
  int nsw = static_cast<int>((dev.max_smem_optin - fixed) / per);
  if (nsw < 1) return cudaErrorInvalidValue;  // caller bounds heads * head_dim
  if (nsw > cap) nsw = cap;
  const size_t smem = fixed + per * nsw;
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

cudaError_t read_status_headnorm_fwd(int* status, bool clear) { return tu_status(status, clear); }

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
  a.seqd = make_divu32(seq);
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
  a.seqd = make_divu32(seq);
  a.heads = static_cast<int>(heads);
  a.eps = eps;
  return g.done(launch_headnorm<false, false, false>(a, static_cast<int>(head_dim),
                                                     static_cast<cudaStream_t>(stream)));
}
