// Backward of the per-head RMSNorm (+ RoPE): qkv_norm_rope_bwd, head_norm_bwd.
//
// Reference: src/kernels/rope.py:223-274 (_section_bwd), :277-383
// (_qkv_norm_rope_bwd_kernel), :386-436 (_head_norm_bwd_kernel), :443-471 and
// :540-577 (weight-grad partials reduced with torch .sum((0, 1))).  Per token
// and head, with a/b the two halves of the forward input and da/db of the
// upstream gradient:
//   rotate back:  da' = da*cos + db*sin;  db' = db*cos - da*sin   (q and k)
//   rstd = 1 / sqrt(sum(x*x) / hd + eps);  xhat = x * rstd;  u = d' * w
//   c = sum(u * xhat) / hd;  dx = bf16(rstd * (u - xhat * c))
//   dw += d' * xhat   (fp32, per dim)
// c is formed as (sum(u * x) * rstd) / hd: the same value up to rounding, with
// a sum that does not wait for rstd, so both head sums share one butterfly.
// v's gradient is copied into the v third of dqkv (rope.py:304-326).
//
// Layout: persistent CTAs of kHnbWarps warps walk fixed chunks of kHnbWarps
// tokens; warp w takes token w of each chunk.  The unit of the warp's ring of
// shared-memory stages is one section of one token (q or k, or x): lane 0
// streams the section's forward input and its upstream gradient into a stage
// with bulk copies completing on an mbarrier, up to nsw units ahead, so the
// next section's bytes are in flight while the warp computes.  A head
// spans L = hd/16 lanes; lane l holds dims [8l, 8l+8) of both halves, so the
// rotation pairs are in the lane and the per-head sums follow the forward's
// canonical order.
//
// Weight-gradient order (deterministic, independent of the launch shape):
// per token, lane group g sums heads g, g + 32/L, ... in increasing order and
// the groups combine as a stride tree; the kHnbWarps token sums of a chunk
// combine as a stride tree over the token index; the chunk sums combine as a
// stride tree over the chunk index (finalize.cu).
#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

constexpr int kHnbWarps = 8;       // warps per CTA = tokens per chunk
constexpr int kHnbMaxStages = 3;
constexpr size_t kHnbCtaSmemFor2 = 110 * 1024;  // two CTAs per SM at or below this
constexpr int kHnbUnroll = 1;

struct HeadNormBwdArgs {
  const uint16_t* src;  // forward input rows (qkv or x)
  int64_t src_row;      // elements per token row of src and dsrc
  int64_t q_off, k_off, v_off;
  const uint16_t* dq;   // [tokens, heads, hd]
  const uint16_t* dk;   // (WITH_K)
  const uint16_t* dv;   // (WITH_V)
  const float* wq;
  const float* wk;
  const float* cos;
  const float* sin;
  uint16_t* dsrc;       // [tokens, src_row]
  float* part;          // [chunks][NSEC][hd] chunk sums of the weight gradient
  int64_t tokens;
  int64_t seq;
  DivU32 seqd;          // division by seq
  int heads;
  float eps;
};

template <int HD, bool ROTATE, bool WITH_K, bool WITH_V>
__global__ void __launch_bounds__(kHnbWarps * 32, 2)
headnorm_bwd_kernel(const HeadNormBwdArgs a, const int nsw) {
  constexpr int L = HD / 16;
  constexpr int HPI = 32 / L;
  constexpr int HALF = HD / 2;
  constexpr int NSEC = WITH_K ? 2 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int l = lane % L;
  const int grp = lane / L;
  const int H = a.heads;
  const int iters = (H + HPI - 1) / HPI;
  const uint32_t sec_bytes = static_cast<uint32_t>(H) * HD * 2u;
  // stage: one section's forward input, then its upstream gradient
  const uint32_t stage_bytes = 2u * sec_bytes;
  float* xch = reinterpret_cast<float*>(smem);  // [warps][NSEC][HD] token sums
  uint8_t* ring = smem + kHnbWarps * NSEC * HD * sizeof(float) +
                  static_cast<size_t>(warp) * nsw * stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kHnbWarps * NSEC * HD * sizeof(float) +
                                               static_cast<size_t>(kHnbWarps) * nsw * stage_bytes) +
                   warp * nsw;
  if (lane == 0) {
    for (int s = 0; s < nsw; ++s) mbar_init(smem_addr(&bars[s]), 1);
    fence_mbar_init();
  }
  __syncwarp();
  // While the previous kernel on the stream finishes, pull this warp's first
  // unit (section 0 of its first token and its gradient) into L2
  // (prefetch_l2).  Measured: head_norm_bwd 17.4 -> 15.9 us in a stream,
  // isolated unchanged.  (rowquant, whose CTAs hold one or two rows, lost
  // 1-2 us isolated with the same prefetch and does without it.)
  if (lane == 0) {
    const int64_t tok = static_cast<int64_t>(blockIdx.x) * kHnbWarps + warp;
    if (tok < a.tokens) {
      prefetch_l2(a.src + tok * a.src_row + a.q_off, sec_bytes);
      prefetch_l2(a.dq + tok * static_cast<int64_t>(H) * HD, sec_bytes);
    }
  }
  pdl_wait();
  pdl_trigger();

  const int64_t chunks = (a.tokens + kHnbWarps - 1) / kHnbWarps;
  // this warp's j-th token: token `warp` of chunk blockIdx.x + j*gridDim.x
  auto token_of = [&](int64_t j) {
    return (static_cast<int64_t>(blockIdx.x) + j * gridDim.x) * kHnbWarps + warp;
  };
  auto chunk_of = [&](int64_t j) { return static_cast<int64_t>(blockIdx.x) + j * gridDim.x; };
  // Unit u of this warp: section u % NSEC of its token u / NSEC.  Units of
  // tokens past the end are neither copied nor waited for; a warp's tokens
  // increase with u, so the copied units are a prefix and the ring's slot
  // (u % nsw) and phase ((u / nsw) & 1) follow u.
  auto unit_exists = [&](int64_t u) {
    const int64_t j = u / NSEC;
    return chunk_of(j) < chunks && token_of(j) < a.tokens;
  };
  auto issue = [&](int64_t u, int s) {  // lane 0: unit u into slot s
    const int64_t tok = token_of(u / NSEC);
    const int sec = static_cast<int>(u % NSEC);
    uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    const uint32_t bar = smem_addr(&bars[s]);
    mbar_arrive_expect_tx(bar, stage_bytes);
    bulk_g2s(smem_addr(st), a.src + tok * a.src_row + (sec ? a.k_off : a.q_off), sec_bytes, bar);
    bulk_g2s(smem_addr(st + sec_bytes), (sec ? a.dk : a.dq) + tok * static_cast<int64_t>(H) * HD, sec_bytes,
             bar);
  };
  auto prefetch = [&](int64_t u) {  // lane 0: unit u's section and gradient into L2
    const int64_t tok = token_of(u / NSEC);
    const int sec = static_cast<int>(u % NSEC);
    prefetch_l2(a.src + tok * a.src_row + (sec ? a.k_off : a.q_off), sec_bytes);
    prefetch_l2((sec ? a.dk : a.dq) + tok * static_cast<int64_t>(H) * HD, sec_bytes);
  };
  if (lane == 0) {
    for (int u = 0; u < nsw && unit_exists(u); ++u) issue(u, u);
  }
  int slot = 0;      // ring slot of the next unit
  uint32_t ph = 0;   // its phase parity

  bool dead = false;  // set if a bounded wait gave up: the warp then only joins the barriers
  int64_t u = 0;      // this warp's next unit
  for (int64_t j = 0; chunk_of(j) < chunks; ++j) {
    const int64_t tok = token_of(j);
    const bool has = tok < a.tokens && !dead;
    if (has) {
      float cs[8], sn[8];
      if (ROTATE) {
        const int64_t pos = tok - div_u32(a.seqd, tok) * a.seq;
        const float* cp = a.cos + pos * HALF + 8 * l;
        const float* sp = a.sin + pos * HALF + 8 * l;
        const float4 c0 = ld_keep_f4(cp), c1 = ld_keep_f4(cp + 4);
        const float4 s0 = ld_keep_f4(sp), s1 = ld_keep_f4(sp + 4);
        cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w;
        cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
        sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
        sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
      }
      if (WITH_V) {  // dqkv's v third is dv, unchanged
        const uint16_t* in = a.dv + tok * static_cast<int64_t>(H) * HD;
        uint16_t* out = a.dsrc + tok * a.src_row + a.v_off;
        for (int v = lane; v < H * HD / 8; v += 32) st16(out + 8 * v, ld_stream(in + 8 * v));
      }
#pragma unroll
      for (int sec = 0; sec < NSEC; ++sec) {
        const uint8_t* st = ring + static_cast<size_t>(slot) * stage_bytes;
        if (!mbar_wait(smem_addr(&bars[slot]), ph)) {
          // Never expected: wait (bounded) for the copies still in flight, then stop.
          for (int64_t k = u + 1; k < u + nsw && unit_exists(k); ++k)
            mbar_wait(smem_addr(&bars[k % nsw]), static_cast<uint32_t>((k / nsw) & 1));
          dead = true;
          break;
        }
        // The unit that will refill this slot after it: start pulling it into
        // L2 now, so that its bulk copy, issued once this unit is done, reads
        // L2 instead of waiting on DRAM.  Measured: qkv_norm_rope_bwd 33.9 ->
        // 31.9 us in a stream, 40.5 -> 38.4 us isolated; head_norm_bwd unchanged.
        if (lane == 0 && unit_exists(u + nsw)) prefetch(u + nsw);
        const uint8_t* xin = st;
        const uint8_t* gin = st + sec_bytes;
        // The section's norm weights (L1-resident) and its weight-gradient sums.
        float w[2][8], wacc[2][8];
        {
          const float* wp = (sec ? a.wk : a.wq) + 8 * l;
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const float4 w0 = ld_keep_f4(wp + hf * HALF), w1 = ld_keep_f4(wp + hf * HALF + 4);
            w[hf][0] = w0.x; w[hf][1] = w0.y; w[hf][2] = w0.z; w[hf][3] = w0.w;
            w[hf][4] = w1.x; w[hf][5] = w1.y; w[hf][6] = w1.z; w[hf][7] = w1.w;
#pragma unroll
            for (int k = 0; k < 8; ++k) wacc[hf][k] = 0.0f;
          }
        }
        uint16_t* out = a.dsrc + tok * a.src_row + (sec ? a.k_off : a.q_off);
        for (int it0 = 0; it0 < iters; it0 += kHnbUnroll) {
          uint4 xa[kHnbUnroll], xb[kHnbUnroll];
          float dpa[kHnbUnroll][8], dpb[kHnbUnroll][8];  // rotated-back gradient
          float ss[kHnbUnroll], cc[kHnbUnroll];  // sum(x * x), sum((d' * w) * x)
#pragma unroll
          for (int u = 0; u < kHnbUnroll; ++u) {
            const int h = (it0 + u) * HPI + grp;
            const bool hv = it0 + u < iters && h < H;
            const int o = (h * HD + 8 * l) * 2;
            xa[u] = hv ? lds16(xin + o) : make_uint4(0, 0, 0, 0);
            xb[u] = hv ? lds16(xin + o + HALF * 2) : make_uint4(0, 0, 0, 0);
            const uint4 ga = hv ? lds16(gin + o) : make_uint4(0, 0, 0, 0);
            const uint4 gb = hv ? lds16(gin + o + HALF * 2) : make_uint4(0, 0, 0, 0);
            float fa[8], fb[8];
            unpack8(ga, fa);
            unpack8(gb, fb);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              if (ROTATE) {
                dpa[u][k] = __fadd_rn(__fmul_rn(fa[k], cs[k]), __fmul_rn(fb[k], sn[k]));
                dpb[u][k] = __fsub_rn(__fmul_rn(fb[k], cs[k]), __fmul_rn(fa[k], sn[k]));
              } else {
                dpa[u][k] = fa[k];
                dpb[u][k] = fb[k];
              }
            }
            unpack8(xa[u], fa);
            unpack8(xb[u], fb);
            float ta[8], tb[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              ta[k] = __fmul_rn(__fmul_rn(dpa[u][k], w[0][k]), fa[k]);
              tb[k] = __fmul_rn(__fmul_rn(dpb[u][k], w[1][k]), fb[k]);
              fa[k] = __fmul_rn(fa[k], fa[k]);
              fb[k] = __fmul_rn(fb[k], fb[k]);
            }
            ss[u] = __fadd_rn(vec_sum8(fa), vec_sum8(fb));
            cc[u] = __fadd_rn(vec_sum8(ta), vec_sum8(tb));
          }
          // Both head sums in one butterfly: c = (sum((d' * w) * x) * rstd) / HD.
#pragma unroll
          for (int o = L / 2; o >= 1; o >>= 1) {
#pragma unroll
            for (int u = 0; u < kHnbUnroll; ++u) {
              ss[u] = __fadd_rn(ss[u], __shfl_xor_sync(kFull, ss[u], o));
              cc[u] = __fadd_rn(cc[u], __shfl_xor_sync(kFull, cc[u], o));
            }
          }
          float rstd[kHnbUnroll];
#pragma unroll
          for (int u = 0; u < kHnbUnroll; ++u) rstd[u] = canonical_rstd(__fmul_rn(ss[u], 1.0f / HD), a.eps);
#pragma unroll
          for (int u = 0; u < kHnbUnroll; ++u) {
            const int h = (it0 + u) * HPI + grp;
            if (it0 + u >= iters || h >= H) continue;
            const float c = __fmul_rn(__fmul_rn(cc[u], rstd[u]), 1.0f / HD);
            float fa[8], fb[8], oa[8], ob[8];
            unpack8(xa[u], fa);
            unpack8(xb[u], fb);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const float xha = __fmul_rn(fa[k], rstd[u]);
              const float xhb = __fmul_rn(fb[k], rstd[u]);
              const float ua = __fmul_rn(dpa[u][k], w[0][k]);
              const float ub = __fmul_rn(dpb[u][k], w[1][k]);
              oa[k] = __fmul_rn(rstd[u], __fsub_rn(ua, __fmul_rn(xha, c)));
              ob[k] = __fmul_rn(rstd[u], __fsub_rn(ub, __fmul_rn(xhb, c)));
              wacc[0][k] = __fadd_rn(wacc[0][k], __fmul_rn(dpa[u][k], xha));
              wacc[1][k] = __fadd_rn(wacc[1][k], __fmul_rn(dpb[u][k], xhb));
            }
            st16(out + h * HD + 8 * l, pack8_rn(oa));
            st16(out + h * HD + HALF + 8 * l, pack8_rn(ob));
          }
        }
        // the token's sum for this section: stride tree over the lane groups
        // (xor 16, then 8, ... down to L)
#pragma unroll
        for (int o = 16; o >= L; o >>= 1) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf)
#pragma unroll
            for (int k = 0; k < 8; ++k) wacc[hf][k] = __fadd_rn(wacc[hf][k], __shfl_xor_sync(kFull, wacc[hf][k], o));
        }
        if (grp == 0) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf)
#pragma unroll
            for (int k = 0; k < 8; ++k) xch[(warp * NSEC + sec) * HD + hf * HALF + 8 * l + k] = wacc[hf][k];
        }
        __syncwarp();  // the stage is read: refill it with unit u + nsw
        if (lane == 0 && unit_exists(u + nsw)) {
          fence_proxy_async_smem();
          issue(u + nsw, slot);
        }
        ++u;
        if (++slot == nsw) {
          slot = 0;
          ph ^= 1u;
        }
      }
    }
    if (!has) {  // a token past the end (or a stopped warp) adds zeros
      for (int i = lane; i < NSEC * HD; i += 32) xch[warp * NSEC * HD + i] = 0.0f;
    }
    __syncthreads();
    // chunk sum: stride tree over the warps (= tokens of the chunk)
    for (int i = threadIdx.x; i < NSEC * HD; i += kHnbWarps * 32) {
      float p[kHnbWarps];
#pragma unroll
      for (int t = 0; t < kHnbWarps; ++t) p[t] = xch[t * NSEC * HD + i];
#pragma unroll
      for (int hw = kHnbWarps / 2; hw >= 1; hw >>= 1)
#pragma unroll
        for (int t = 0; t < hw; ++t) p[t] = __fadd_rn(p[t], p[t + hw]);
      a.part[chunk_of(j) * NSEC * HD + i] = p[0];
    }
    __syncthreads();
  }
}

static int64_t hn_chunks(int64_t tokens) { return (tokens + kHnbWarps - 1) / kHnbWarps; }

size_t headnorm_bwd_workspace(int64_t tokens, int64_t hd, int nsec) {
  return static_cast<size_t>(hn_chunks(tokens) * nsec * hd) * sizeof(float);
}

template <bool ROTATE, bool WITH_K, bool WITH_V>
static cudaError_t launch_headnorm_bwd(const HeadNormBwdArgs& a, int hd, cudaStream_t st) {
  const DeviceInfo& dev = device_info();
  if (dev.error != cudaSuccess) return dev.error;
  constexpr int NSEC = WITH_K ? 2 : 1;
  const size_t stage = 2 * static_cast<size_t>(a.heads) * hd * 2;  // one section: input + gradient
  const size_t fixed = static_cast<size_t>(kHnbWarps) * NSEC * hd * sizeof(float);
  const size_t per = kHnbWarps * (stage + sizeof(uint64_t));
  // Two CTAs per SM (16 warps to hide the per-head dependency chains) with
  // as many stages as then fit; one CTA with a deeper ring otherwise.
  const size_t limit2 = kHnbCtaSmemFor2 > fixed ? kHnbCtaSmemFor2 - fixed : 0;
  int ctas = limit2 >= per ? 2 : 1;
  int nsw = static_cast<int>((ctas == 2 ? limit2 : dev.max_smem_optin - fixed) / per);
  if (nsw < 1) return cudaErrorInvalidValue;  // bounded by heads * head_dim <= 2048
  if (nsw > kHnbMaxStages) nsw = kHnbMaxStages;
  const size_t smem = fixed + per * nsw;
  const int64_t chunks = hn_chunks(a.tokens);
  const int64_t cap = static_cast<int64_t>(dev.sms) * ctas;
  const dim3 grid(static_cast<unsigned>(chunks < cap ? chunks : cap));
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e = ensure_smem(kern, smem, true);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, grid, dim3(kHnbWarps * 32), smem, st, a, nsw);
  };
  switch (hd) {
    case 64: return go(headnorm_bwd_kernel<64, ROTATE, WITH_K, WITH_V>);
    case 128: return go(headnorm_bwd_kernel<128, ROTATE, WITH_K, WITH_V>);
    case 256: return go(headnorm_bwd_kernel<256, ROTATE, WITH_K, WITH_V>);
    default: return cudaErrorInvalidValue;
  }
}

inline bool check_heads_bwd(int64_t batch, int64_t seq, int64_t heads, int64_t hd) {
  return check(batch >= 0, "batch must be >= 0") && check(seq >= 1, "seq must be >= 1") &&
         check(heads >= 1 && heads * hd <= 2048,
               "heads * head_dim must be in [1, 2048], got " + std::to_string(heads * hd)) &&
         check(hd == 64 || hd == 128 || hd == 256,
               "head_dim must be 64, 128 or 256, got " + std::to_string(hd)) &&
         check(finalize_fits(hn_chunks(batch * seq)),
               "backward supports batch * seq <= " + std::to_string(32768 * kHnbWarps));
}

static cudaError_t finalize(const HeadNormBwdArgs& a, void* dw0, void* dw1, int nsec, int hd,
                            cudaStream_t st) {
  FinalizeArgs f{};
  f.part = a.part;
  f.n = hn_chunks(a.tokens);
  f.ncols = nsec * hd;
  f.seg = hd;
  f.out[0] = dw0;
  f.out[1] = dw1;
  f.bf16_out = 0;
  if (f.n == 0) {  // no tokens: the gradients are zero
    cudaError_t e = cudaMemsetAsync(dw0, 0, hd * sizeof(float), st);
    if (e == cudaSuccess && nsec > 1) e = cudaMemsetAsync(dw1, 0, hd * sizeof(float), st);
    return e;
  }
  return launch_colsum_finalize(f, 1, st);
}

cudaError_t read_status_headnorm_bwd(int* status, bool clear) { return tu_status(status, clear); }

}  // namespace afb

using namespace afb;

extern "C" size_t afb_qkv_norm_rope_bwd_workspace(int64_t batch, int64_t seq, int64_t heads,
                                                  int64_t head_dim) {
  (void)heads;
  return headnorm_bwd_workspace(batch * seq, head_dim, 2);
}

extern "C" size_t afb_head_norm_bwd_workspace(int64_t batch, int64_t seq, int64_t heads,
                                              int64_t head_dim) {
  (void)heads;
  return headnorm_bwd_workspace(batch * seq, head_dim, 1);
}

extern "C" int afb_qkv_norm_rope_bwd(const void* qkv, const void* dq, const void* dk,
                                     const void* dv, const void* q_weight, const void* k_weight,
                                     const void* cos, const void* sin, void* dqkv, void* dqw,
                                     void* dkw, int64_t batch, int64_t seq, int64_t heads,
                                     int64_t head_dim, float eps, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  ApiGuard g("afb_qkv_norm_rope_bwd");
  const size_t need = headnorm_bwd_workspace(batch * seq, head_dim, 2);
  if (!check_heads_bwd(batch, seq, heads, head_dim) ||
      !check_ptrs({qkv, dq, dk, dv, q_weight, k_weight, cos, sin, dqkv, dqw, dkw},
                  {"qkv", "dq", "dk", "dv", "q_weight", "k_weight", "cos", "sin", "dqkv", "dqw",
                   "dkw"}) ||
      !check(workspace != nullptr && aligned(workspace, 16), "workspace is null or misaligned") ||
      !check(workspace_bytes >= need, "workspace too small: need " + std::to_string(need) + " bytes"))
    return g.fail();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  HeadNormBwdArgs a{};
  const int64_t width = heads * head_dim;
  a.src = static_cast<const uint16_t*>(qkv);
  a.src_row = 3 * width;
  a.q_off = 0;
  a.k_off = width;
  a.v_off = 2 * width;
  a.dq = static_cast<const uint16_t*>(dq);
  a.dk = static_cast<const uint16_t*>(dk);
  a.dv = static_cast<const uint16_t*>(dv);
  a.wq = static_cast<const float*>(q_weight);
  a.wk = static_cast<const float*>(k_weight);
  a.cos = static_cast<const float*>(cos);
  a.sin = static_cast<const float*>(sin);
  a.dsrc = static_cast<uint16_t*>(dqkv);
  a.part = static_cast<float*>(workspace);
  a.tokens = batch * seq;
  a.seq = seq;
  a.seqd = make_divu32(seq);
  a.heads = static_cast<int>(heads);
  a.eps = eps;
  const int hd = static_cast<int>(head_dim);
  if (a.tokens > 0) {
    cudaError_t e = launch_headnorm_bwd<true, true, true>(a, hd, st);
    if (e != cudaSuccess) return g.done(e);
  }
  return g.done(finalize(a, dqw, dkw, 2, hd, st));
}

extern "C" int afb_head_norm_bwd(const void* x, const void* dy, const void* weight, void* dx,
                                 void* dw, int64_t batch, int64_t seq, int64_t heads,
                                 int64_t head_dim, float eps, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  ApiGuard g("afb_head_norm_bwd");
  const size_t need = headnorm_bwd_workspace(batch * seq, head_dim, 1);
  if (!check_heads_bwd(batch, seq, heads, head_dim) ||
      !check_ptrs({x, dy, weight, dx, dw}, {"x", "dy", "weight", "dx", "dw"}) ||
      !check(workspace != nullptr && aligned(workspace, 16), "workspace is null or misaligned") ||
      !check(workspace_bytes >= need, "workspace too small: need " + std::to_string(need) + " bytes"))
    return g.fail();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  HeadNormBwdArgs a{};
  a.src = static_cast<const uint16_t*>(x);
  a.src_row = heads * head_dim;
  a.dq = static_cast<const uint16_t*>(dy);
  a.wq = static_cast<const float*>(weight);
  a.dsrc = static_cast<uint16_t*>(dx);
  a.part = static_cast<float*>(workspace);
  a.tokens = batch * seq;
  a.seq = seq;
  a.seqd = make_divu32(seq);
  a.heads = static_cast<int>(heads);
  a.eps = eps;
  const int hd = static_cast<int>(head_dim);
  if (a.tokens > 0) {
    cudaError_t e = launch_headnorm_bwd<false, false, false>(a, hd, st);
    if (e != cudaSuccess) return g.done(e);
  }
  return g.done(finalize(a, dw, dw, 1, hd, st));
}
