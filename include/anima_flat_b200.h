/*
 * anima_flat_b200 — C ABI of the fused DiT layer ops for NVIDIA B200 (sm_100a).
 *
 * Each entry point replaces one Triton kernel launch of the reference
 * (tan0210/anima-flat, src/kernels/*.py) and takes what that launch takes:
 * raw device pointers, sizes, eps and the CUDA stream to launch on (a
 * cudaStream_t passed as void*; NULL is the legacy default stream).  All
 * launches are asynchronous on that stream; nothing allocates.
 *
 * Types.  Activations, modulation vectors (gate, shift, scale) and the
 * weight gradients of the modulation vectors are bf16 (uint16 bit patterns);
 * RMSNorm weights, RoPE tables, FP8 row scales and norm-weight gradients are
 * fp32; FP8 codes are OCP e4m3 "fn" bytes (max 448), the layout torch calls
 * float8_e4m3fn.  Every tensor is dense row-major; bf16 tensors must be
 * 16-byte aligned.  `scale` already includes the +1 (reference model.py:228).
 *
 * Errors.  Return 0 on success, otherwise a cudaError_t value
 * (cudaErrorInvalidValue = 1 for rejected arguments); afb_last_error()
 * returns this thread's message for the last failure.
 */
#ifndef ANIMA_FLAT_B200_H_
#define ANIMA_FLAT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ABI revision of this header. */
int afb_abi_version(void);

/* Message of this thread's last failed call ("" if none). */
const char* afb_last_error(void);
void afb_clear_error(void);

/* Device status of the current device: 0, or a bit set by a kernel whose
 * bounded wait on an asynchronous copy gave up (then the kernel stopped
 * early and its outputs are incomplete).  No reference counterpart. */
int afb_device_status(int* status);
/* The same status, after which every status word of the device is zeroed
 * (so a caller can report a failure once and carry on).  No reference
 * counterpart. */
int afb_take_device_status(int* status);

/* Failure-path probe of the bounded waits; no reference counterpart.  One
 * thread starts a 1 KiB bulk copy, then waits on an mbarrier that nothing
 * arrives on with a limit of `spins` try_wait rounds (1..65536): the wait
 * gives up and sets the device status word, as a kernel's wait on a copy
 * that never lands would, and the thread then drains the copy in flight and
 * returns.  result (device, 2 x int32): [0] = 1 if the wait gave up, [1] = 1
 * if the copy was drained.  It faults nothing; the status word stays set
 * until afb_take_device_status. */
int afb_wait_probe(uint32_t spins, void* result, void* stream);

/* Programmatic dependent launch on (1, default) or off (0).  Also read from
 * the environment variable AFB_PDL=0 at first use. */
void afb_set_pdl(int enabled);
int afb_get_pdl(void);

/* ----------------------------------------------------------------------- */
/* AdaLN modulate                                                           */
/* ----------------------------------------------------------------------- */

/* Gated residual + affine-free LayerNorm + modulate.
 * Replaces src/kernels/adaln.py:49-75 (anima_flat::residual_adaln launching
 * _residual_adaln_kernel, adaln.py:10-46, HAS_X=True).
 *   z = bf16(residual + bf16(gate * x));  h = bf16(LN(z) * scale + shift)
 * x, residual, h, z: [batch, seq, dim]; gate, shift, scale: [batch, dim]. */
int afb_residual_adaln(const void* x, const void* residual, const void* gate,
                       const void* shift, const void* scale, void* h, void* z,
                       int64_t batch, int64_t seq, int64_t dim, float eps,
                       void* stream);

/* LayerNorm + modulate without the residual.
 * Replaces src/kernels/adaln.py:83-103 (anima_flat::adaln, HAS_X=False). */
int afb_adaln(const void* z, const void* shift, const void* scale, void* h,
              int64_t batch, int64_t seq, int64_t dim, float eps, void* stream);

/* residual_adaln with the modulated output quantised to FP8 per row.
 * Replaces src/kernels/fp8.py:100-128 (anima_flat::residual_adaln_fp8
 * launching _residual_adaln_fp8_kernel, fp8.py:56-97, HAS_X=True).
 * q: [batch*seq, dim] e4m3; s: [batch*seq] fp32; z as above. */
int afb_residual_adaln_fp8(const void* x, const void* residual, const void* gate,
                           const void* shift, const void* scale, void* q, void* s,
                           void* z, int64_t batch, int64_t seq, int64_t dim,
                           float eps, void* stream);

/* adaln with FP8 output.  Replaces src/kernels/fp8.py:141-163
 * (anima_flat::adaln_fp8, HAS_X=False). */
int afb_adaln_fp8(const void* z, const void* shift, const void* scale, void* q,
                  void* s, int64_t batch, int64_t seq, int64_t dim, float eps,
                  void* stream);

/* ----------------------------------------------------------------------- */
/* FP8 row quantisation                                                     */
/* ----------------------------------------------------------------------- */

/* Per-row e4m3 quantisation, optionally after the A&S 7.1.26 GELU.
 * Replaces src/kernels/fp8.py:295-301 (anima_flat::rowquant launching
 * _rowquant_kernel, fp8.py:273-292).  x: [rows, K] bf16, K a multiple of 16
 * up to 16384; q: [rows, K] e4m3; s: [rows] fp32. */
int afb_rowquant(const void* x, void* q, void* s, int64_t rows, int64_t K, int gelu,
                 void* stream);

/* Test hook: fast and canonical GELU of n bf16 values (fp32 outputs).  The
 * GELU row quantisation relies on the bound between the two.  No reference
 * counterpart. */
int afb_gelu_probe(const void* x, void* fast, void* canon, int64_t n, void* stream);

/* ----------------------------------------------------------------------- */
/* q/k RMSNorm + 3D RoPE, head norm                                          */
/* ----------------------------------------------------------------------- */

/* Replaces src/kernels/rope.py:175-193 (anima_flat::qkv_norm_rope) and, with
 * v != NULL, rope.py:504-523 (anima_flat::qkv_norm_rope_v), both launching
 * _qkv_norm_rope_kernel (rope.py:61-143).
 * qkv: [batch, seq, 3*heads*head_dim] (q | k | v); q_weight, k_weight:
 * [head_dim] fp32; cos, sin: [seq, head_dim/2] fp32; q, k, v:
 * [batch, seq, heads, head_dim].  head_dim is 64, 128 or 256. */
int afb_qkv_norm_rope(const void* qkv, const void* q_weight, const void* k_weight,
                      const void* cos, const void* sin, void* q, void* k, void* v,
                      int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
                      float eps, void* stream);

/* Per-head RMSNorm without rotation (cross-attention queries).
 * Replaces src/kernels/rope.py:203-212 (anima_flat::head_norm launching
 * _head_norm_kernel, rope.py:146-172).  x: [batch, seq, heads*head_dim];
 * weight: [head_dim] fp32; y: [batch, seq, heads, head_dim]. */
int afb_head_norm(const void* x, const void* weight, void* y, int64_t batch,
                  int64_t seq, int64_t heads, int64_t head_dim, float eps,
                  void* stream);

/* Replaces src/kernels/ctx_scale.py:40-57 (anima_flat::ctx_scale, launching
 * _ctx_scale_kernel, ctx_scale.py:8-37), called from src/attention.py:180.
 * out, y [batch, seq, heads, head_dim] bf16; lse [batch, heads, seq] fp32;
 * ln_pad [batch] fp32.  y = bf16(out * gain), gain = 1 / (1 + exp(ln_pad -
 * lse)).  head_dim in {64, 128, 256}, heads * head_dim <= 2048. */
int afb_ctx_scale(const void* out, const void* lse, const void* ln_pad, void* y, int64_t batch,
                  int64_t seq, int64_t heads, int64_t head_dim, void* stream);

/* Replaces src/kernels/rms.py:157-197 (anima_flat::rms_silu, add_rms_silu,
 * shuffle_rms_silu, all launching _fwd_kernel, rms.py:35-73), called from
 * src/vae.py:74, 258-278.  Rows are pixels of `channels` channels, channels
 * last, bf16; gamma [channels] fp32, 16-byte aligned like every array.
 *   rms_silu:         residual NULL, shuffled 0; s unused (may be NULL).
 *   add_rms_silu:     residual [rows, C]; s = bf16(x + residual) is written.
 *   shuffle_rms_silu: shuffled 1, x = u [B, H/2, W/2, 4C], output grid
 *                     H x W (rows = B*H*W); s = the gathered x is written.
 * y = bf16(silu(s * sqrt(C) / max(|s|, 1e-12) * gamma)).  channels a
 * multiple of 8 in [8, 1024]; W <= 2^30 when shuffled. */
int afb_rms_silu(const void* x, const void* residual, const void* gamma, void* s, void* y,
                 int64_t rows, int64_t H, int64_t W, int64_t channels, int shuffled, void* stream);

/* Test hook: every fp32 input through the forward's fast SiLU and its
 * settle test against the canonical SiLU, and through the backward's
 * branch-free sigmoid against the canonical sigmoid.  stats: 515 uint64
 * counters, 8-byte aligned, overwritten: [0] settled inputs whose bf16 SiLU
 * differs from the canonical one (0 when the fast path is sound), [1]
 * unsettled inputs with |a| <= 8, [2 + sign*256 + exponent] the largest
 * fp32-step distance between the fast and canonical SiLU values, [514]
 * inputs with |a| <= 87 whose fast sigmoid differs from the canonical one in
 * any bit (0 when the backward's sigmoid is exact).  No reference counterpart. */
int afb_silu_probe(void* stats, void* stream);

/* ----------------------------------------------------------------------- */
/* Backward (LoRA training)                                                 */
/* ----------------------------------------------------------------------- */
/* Each backward entry point takes a caller-provided device workspace of at
 * least the size its *_workspace query returns (fp32 partial sums of the
 * parameter gradients); it is fully overwritten and needs no zeroing.  The
 * parameter gradients are summed in a fixed order, so they are reproducible
 * from run to run and across GPUs.  A workspace query returns SIZE_MAX for
 * sizes whose workspace does not fit in size_t. */

/* Replaces src/kernels/adaln.py:175-233 (_residual_adaln_bwd and the
 * anima_flat::residual_adaln_bwd op, launching _residual_adaln_bwd_kernel,
 * adaln.py:111-172).  gz may be NULL.  Outputs, in the op's order: dx, dres
 * [batch, seq, dim]; dgate, dshift, dscale [batch, dim] bf16.  dim <= 2048.
 * Workspace: batch * ceil(seq / 28) * 3 * dim * 4 bytes (chunk partials of
 * 28 rows). */
size_t afb_residual_adaln_bwd_workspace(int64_t batch, int64_t seq, int64_t dim);
int afb_residual_adaln_bwd(const void* gh, const void* gz, const void* z, const void* x,
                           const void* gate, const void* scale, void* dx, void* dres,
                           void* dgate, void* dshift, void* dscale, int64_t batch,
                           int64_t seq, int64_t dim, float eps, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Allocation-free variant of afb_residual_adaln_bwd, for callers that cannot
 * allocate device memory (a binding with no device allocator, or a process
 * that reserves all device memory up front and forbids allocation on the
 * hot path).  It has no counterpart in the reference.  Same arguments and
 * outputs, without the workspace: the partial sums live in a 16 MiB array
 * inside the library, which every GPU that loads the library holds until
 * exit.  Sizes needing more (batch * ceil(seq / 28) * 3 * dim * 4 bytes, the
 * workspace query's value) are rejected, overflowing sizes included.  The
 * first call on a device resolves the array's address and caches it, so make
 * it before any stream capture, and do not call cudaDeviceReset while the
 * library is loaded.  All calls share the array: calls that overlap on the
 * GPU race. */
int afb_residual_adaln_bwd_noalloc(const void* gh, const void* gz, const void* z,
                                   const void* x, const void* gate, const void* scale,
                                   void* dx, void* dres, void* dgate, void* dshift,
                                   void* dscale, int64_t batch, int64_t seq, int64_t dim,
                                   float eps, void* stream);

/* Replaces src/kernels/adaln.py:247-252 (anima_flat::adaln_bwd, HAS_X=False,
 * HAS_GZ=False): dz, dshift, dscale. */
size_t afb_adaln_bwd_workspace(int64_t batch, int64_t seq, int64_t dim);
int afb_adaln_bwd(const void* gh, const void* z, const void* scale, void* dz, void* dshift,
                  void* dscale, int64_t batch, int64_t seq, int64_t dim, float eps,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Replaces src/kernels/rope.py:540-593 (_qkv_norm_rope_bwd and the
 * anima_flat::qkv_norm_rope_bwd op, launching _qkv_norm_rope_bwd_kernel,
 * rope.py:277-383).  dq, dk, dv: [batch, seq, heads, head_dim]; dqkv like
 * qkv; dqw, dkw: [head_dim] fp32. */
size_t afb_qkv_norm_rope_bwd_workspace(int64_t batch, int64_t seq, int64_t heads,
                                       int64_t head_dim);
int afb_qkv_norm_rope_bwd(const void* qkv, const void* dq, const void* dk, const void* dv,
                          const void* q_weight, const void* k_weight, const void* cos,
                          const void* sin, void* dqkv, void* dqw, void* dkw, int64_t batch,
                          int64_t seq, int64_t heads, int64_t head_dim, float eps,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Replaces src/kernels/rope.py:443-478 (_head_norm_bwd and the
 * anima_flat::head_norm_bwd op, launching _head_norm_bwd_kernel,
 * rope.py:386-436).  dx like x; dw: [head_dim] fp32. */
size_t afb_head_norm_bwd_workspace(int64_t batch, int64_t seq, int64_t heads,
                                   int64_t head_dim);
int afb_head_norm_bwd(const void* x, const void* dy, const void* weight, void* dx, void* dw,
                      int64_t batch, int64_t seq, int64_t heads, int64_t head_dim, float eps,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Replaces src/kernels/ctx_scale.py:103-120 (anima_flat::ctx_scale_bwd,
 * launching _ctx_scale_bwd_kernel, ctx_scale.py:61-100): dout = bf16(dy *
 * gain) [batch, seq, heads, head_dim]; dlse = sum(dy * out) * gain *
 * (1 - gain) [batch, heads, seq] fp32. */
int afb_ctx_scale_bwd(const void* out, const void* lse, const void* ln_pad, const void* dy,
                      void* dout, void* dlse, int64_t batch, int64_t seq, int64_t heads,
                      int64_t head_dim, void* stream);

/* The trimmed cross-attention's output path of the FP8 forward in one pass:
 * replaces rowquant(ctx_scale(out, lse, ln_pad).flatten(2)), i.e.
 * src/model.py:457 after src/attention.py:180 (ctx_scale.py:8-37, then
 * fp8.py:273-301).  A fusion the reference does not have: q and s equal
 * those of the two entry points run one after the other, bit for bit, and
 * the bf16 intermediate is never written.  out [batch, seq, heads, head_dim]
 * bf16; lse [batch, heads, seq], ln_pad [batch] fp32 -> q [batch, seq,
 * heads*head_dim] e4m3, s [batch*seq] fp32.  head_dim 64, 128 or 256;
 * heads*head_dim <= 16384. */
int afb_ctx_scale_rowquant(const void* out, const void* lse, const void* ln_pad, void* q, void* s,
                           int64_t batch, int64_t seq, int64_t heads, int64_t head_dim,
                           void* stream);

/* Replaces src/kernels/rms.py:200-243 (anima_flat::rms_silu_bwd, launching
 * _bwd_kernel, rms.py:76-125; partials reduced here in a fixed order instead
 * of torch .sum).  s [rows, C] (the saved s or x); dy [rows, C]; gs (the
 * gradient of s for add/shuffle) or NULL; ds in the input layout (u's layout
 * when shuffled); dgamma [C] fp32.  Workspace from the query: C floats per
 * chunk of 8 * 32/L rows (L the lanes per row, the smallest power of two
 * with C <= 32 * L, at most 32), the chunk doubled until at most 32768
 * chunks remain. */
size_t afb_rms_silu_bwd_workspace(int64_t rows, int64_t channels);
int afb_rms_silu_bwd(const void* s, const void* gamma, const void* dy, const void* gs, void* ds,
                     void* dgamma, int64_t rows, int64_t H, int64_t W, int64_t channels,
                     int shuffled, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ANIMA_FLAT_B200_H_ */
