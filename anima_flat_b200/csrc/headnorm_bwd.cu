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
// v's gradient is copied into the v third of dqkv (rope.py:304-326).
//
// Layout as the forward: one warp per token, LPH = hd/8 lanes per head.
// Weight-gradient order (deterministic, independent of the launch shape):
// tokens are cut into chunks of kTokChunk; in a chunk, warp w takes tokens
// w, w + 4, ...; lane group g (lanes g*LPH .. g*LPH+LPH-1) takes heads
// g, g + 32/LPH, ...; each (chunk, warp, group) slot sums its (token, head)
// terms in that order starting from zero, and the finalize kernel adds the
// slots in increasing slot order.
#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

constexpr int kHnWarps = 4;
constexpr int kTokPerWarp = 4;
constexpr int kTokChunk = kHnWarps * kTokPerWarp;

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
  float* part;          // [slots][NSEC][hd], slots = chunks * kHnWarps * (32 / LPH)
  int64_t tokens;
  int64_t seq;
  int heads;
  float eps;
};

template <int HD, bool ROTATE, bool WITH_K, bool WITH_V>
__global__ void __launch_bounds__(kHnWarps * 32)
headnorm_bwd_kernel(const HeadNormBwdArgs a) {
  constexpr int LPH = HD / 8;
  constexpr int HPI = 32 / LPH;
  constexpr int HALF = HD / 2;
  constexpr int NSEC = WITH_K ? 2 : 1;
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int j = lane % LPH;
  const int grp = lane / LPH;
  const int H = a.heads;
  const int iters = (H + HPI - 1) / HPI;
  const int64_t chunk = blockIdx.x;
  const float fhd = static_cast<float>(HD);

  float wacc[NSEC][8];
  float w[NSEC][8];
#pragma unroll
  for (int sec = 0; sec < NSEC; ++sec) {
    const float* wp = (sec ? a.wk : a.wq) + 8 * j;
    const float4 w0 = ld_keep_f4(wp), w1 = ld_keep_f4(wp + 4);
    w[sec][0] = w0.x; w[sec][1] = w0.y; w[sec][2] = w0.z; w[sec][3] = w0.w;
    w[sec][4] = w1.x; w[sec][5] = w1.y; w[sec][6] = w1.z; w[sec][7] = w1.w;
#pragma unroll
    for (int k = 0; k < 8; ++k) wacc[sec][k] = 0.0f;
  }

  for (int i = 0; i < kTokPerWarp; ++i) {
    const int64_t tok = chunk * kTokChunk + i * kHnWarps + warp;
    if (tok >= a.tokens) break;  // warp-uniform
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
    uint16_t* drow = a.dsrc + tok * a.src_row;
    const int64_t gbase = tok * static_cast<int64_t>(H) * HD;
#pragma unroll
    for (int sec = 0; sec < NSEC; ++sec) {
      const uint16_t* in = row + (sec ? a.k_off : a.q_off);
      const uint16_t* dout = (sec ? a.dk : a.dq) + gbase;
      uint16_t* dst = drow + (sec ? a.k_off : a.q_off);
      for (int it = 0; it < iters; ++it) {
        const int h = it * HPI + grp;
        const bool hv = h < H;
        const uint4 xv = hv ? ld_stream(in + h * HD + 8 * j) : make_uint4(0, 0, 0, 0);
        const uint4 gv = hv ? ld_stream(dout + h * HD + 8 * j) : make_uint4(0, 0, 0, 0);
        float x[8], d[8];
        unpack8(xv, x);
        unpack8(gv, d);
        if (ROTATE) {
          uint4 pg;
          pg.x = __shfl_xor_sync(kFull, gv.x, LPH / 2);
          pg.y = __shfl_xor_sync(kFull, gv.y, LPH / 2);
          pg.z = __shfl_xor_sync(kFull, gv.z, LPH / 2);
          pg.w = __shfl_xor_sync(kFull, gv.w, LPH / 2);
          float p[8];
          unpack8(pg, p);
          const bool first = j < LPH / 2;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float mc = __fmul_rn(d[k], cs[k]);
            const float ps = __fmul_rn(p[k], sn[k]);
            d[k] = first ? __fadd_rn(mc, ps) : __fsub_rn(mc, ps);
          }
        }
        float t[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) t[k] = __fmul_rn(x[k], x[k]);
        const float rstd = canonical_rstd(__fdiv_rn(group_canonical_sum<LPH>(t), fhd), a.eps);
        float xh[8], u[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          xh[k] = __fmul_rn(x[k], rstd);
          u[k] = __fmul_rn(d[k], w[sec][k]);
          t[k] = __fmul_rn(u[k], xh[k]);
        }
        const float c = __fdiv_rn(group_canonical_sum<LPH>(t), fhd);
        float o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          o[k] = __fmul_rn(rstd, __fsub_rn(u[k], __fmul_rn(xh[k], c)));
          if (hv) wacc[sec][k] = __fadd_rn(wacc[sec][k], __fmul_rn(d[k], xh[k]));
        }
        if (hv) st16(dst + h * HD + 8 * j, pack8_rn(o));
      }
    }
    if (WITH_V) {
      const uint16_t* in = a.dv + gbase;
      uint16_t* out = drow + a.v_off;
      const int nvec = H * HD / 8;
      for (int v = lane; v < nvec; v += 32) st16(out + 8 * v, ld_stream(in + 8 * v));
    }
  }

  const int64_t slot = (chunk * kHnWarps + warp) * HPI + grp;
#pragma unroll
  for (int sec = 0; sec < NSEC; ++sec) {
    float* out = a.part + (slot * NSEC + sec) * HD + 8 * j;
    reinterpret_cast<float4*>(out)[0] = make_float4(wacc[sec][0], wacc[sec][1], wacc[sec][2], wacc[sec][3]);
    reinterpret_cast<float4*>(out)[1] = make_float4(wacc[sec][4], wacc[sec][5], wacc[sec][6], wacc[sec][7]);
  }
}

// dw[sec][dim] = sum over slots in increasing order.
__global__ void headnorm_bwd_finalize_kernel(const float* part, float* dw0, float* dw1,
                                             int64_t slots, int nsec, int hd) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nsec * hd) return;
  const float* p = part + i;
  const int64_t stride = static_cast<int64_t>(nsec) * hd;
  float s = 0.0f;
  int64_t k = 0;
  for (; k + 4 <= slots; k += 4) {
    const float v0 = p[(k + 0) * stride], v1 = p[(k + 1) * stride];
    const float v2 = p[(k + 2) * stride], v3 = p[(k + 3) * stride];
    s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v0), v1), v2), v3);
  }
  for (; k < slots; ++k) s = __fadd_rn(s, p[k * stride]);
  (i < hd ? dw0 : dw1)[i % hd] = s;
}

static int64_t hn_slots(int64_t tokens, int64_t hd) {
  const int64_t chunks = (tokens + kTokChunk - 1) / kTokChunk;
  return chunks * kHnWarps * (32 / (hd / 8));
}

size_t headnorm_bwd_workspace(int64_t tokens, int64_t hd, int nsec) {
  return static_cast<size_t>(hn_slots(tokens, hd) * nsec * hd) * sizeof(float);
}

template <bool ROTATE, bool WITH_K, bool WITH_V>
static cudaError_t launch_headnorm_bwd(const HeadNormBwdArgs& a, int hd, cudaStream_t st) {
  const dim3 grid(static_cast<unsigned>((a.tokens + kTokChunk - 1) / kTokChunk));
  const dim3 block(kHnWarps * 32);
  switch (hd) {
    case 64: return launch_pdl(headnorm_bwd_kernel<64, ROTATE, WITH_K, WITH_V>, grid, block, 0, st, a);
    case 128: return launch_pdl(headnorm_bwd_kernel<128, ROTATE, WITH_K, WITH_V>, grid, block, 0, st, a);
    case 256: return launch_pdl(headnorm_bwd_kernel<256, ROTATE, WITH_K, WITH_V>, grid, block, 0, st, a);
    default: return cudaErrorInvalidValue;
  }
}

inline bool check_heads_bwd(int64_t batch, int64_t seq, int64_t heads, int64_t hd) {
  return check(batch >= 0, "batch must be >= 0") && check(seq >= 1, "seq must be >= 1") &&
         check(heads >= 1 && heads <= 1024, "heads must be in [1, 1024]") &&
         check(hd == 64 || hd == 128 || hd == 256,
               "head_dim must be 64, 128 or 256, got " + std::to_string(hd));
}

static cudaError_t finalize(const HeadNormBwdArgs& a, void* dw0, void* dw1, int nsec, int hd,
                            cudaStream_t st) {
  const int64_t slots = hn_slots(a.tokens, hd);
  return launch_pdl(headnorm_bwd_finalize_kernel, dim3((nsec * hd + 127) / 128), dim3(128), 0, st,
                    static_cast<const float*>(a.part), static_cast<float*>(dw0),
                    static_cast<float*>(dw1), slots, nsec, hd);
}

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
  a.heads = static_cast<int>(heads);
  a.eps = eps;
  const int hd = static_cast<int>(head_dim);
  if (a.tokens > 0) {
    cudaError_t e = launch_headnorm_bwd<false, false, false>(a, hd, st);
    if (e != cudaSuccess) return g.done(e);
  }
  return g.done(finalize(a, dw, dw, 1, hd, st));
}
