// Column sums of per-chunk partials, for the parameter gradients of the
// backward kernels (the reference reduces its partials with torch .sum,
// adaln.py:214-216 and rope.py:471, :575-576).
//
// Order: for each batch entry and column, the n chunk partials are summed by
// a stride tree over the chunk index, zero-padded to np = pow2ceil(n):
// p[s] += p[s + np/2], then np/4, ... down to p[0].  The tree runs in shared
// memory: a CTA holds np partials for COLS columns and halves them level by
// level, so the result does not depend on the launch shape.
#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

constexpr int kFinalizeThreads = 256;
constexpr int kFinalizeSmemFloats = 32768;  // 128 KiB

// grid: (ceil(ncols / COLS), batch); dynamic smem: np * COLS floats.  Thread t
// owns column t % COLS of the block and the partial rows t / COLS + k * RPI, so
// the index arithmetic is shifts and a warp's load covers whole lines.
template <int COLS>
__global__ void __launch_bounds__(kFinalizeThreads)
colsum_finalize_kernel(const FinalizeArgs f) {
  constexpr int RPI = kFinalizeThreads / COLS;  // partial rows per pass of the CTA
  constexpr int kBatch = 16;                    // loads in flight per thread
  extern __shared__ float sm[];
  pdl_wait();
  pdl_trigger();
  const int t = threadIdx.x;
  const int c = t % COLS;
  const int r = t / COLS;
  const int64_t b = blockIdx.y;
  const int col = blockIdx.x * COLS + c;
  const bool cok = col < f.ncols;
  const float* part = f.part + b * f.n * f.ncols + col;
  for (int s0 = r; s0 < f.np; s0 += kBatch * RPI) {
    float v[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int s = s0 + u * RPI;
      v[u] = (cok && s < f.n) ? __ldg(part + static_cast<int64_t>(s) * f.ncols) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int s = s0 + u * RPI;
      if (s < f.np) sm[s * COLS + c] = v[u];
    }
  }
  for (int h = f.np / 2; h >= 1; h >>= 1) {
    __syncthreads();
    for (int s = r; s < h; s += RPI) sm[s * COLS + c] = __fadd_rn(sm[s * COLS + c], sm[(s + h) * COLS + c]);
  }
  __syncthreads();
  if (r == 0 && cok) {
    const int seg = col / f.seg;
    const int64_t o = b * f.seg + col % f.seg;
    void* dst = seg == 0 ? f.out[0] : seg == 1 ? f.out[1] : f.out[2];  // no local copy of out[]
    if (f.bf16_out) {
      static_cast<uint16_t*>(dst)[o] = static_cast<uint16_t>(pack2_rn(sm[c], 0.0f) & 0xffffu);
    } else {
      static_cast<float*>(dst)[o] = sm[c];
    }
  }
}

bool finalize_fits(int64_t n) { return n >= 1 && n <= kFinalizeSmemFloats; }

cudaError_t launch_colsum_finalize(const FinalizeArgs& in, int64_t batch, cudaStream_t st) {
  FinalizeArgs f = in;
  int64_t np = 1;
  while (np < f.n) np <<= 1;
  if (np > kFinalizeSmemFloats) return cudaErrorInvalidValue;
  f.np = static_cast<int>(np);
  // 32 columns per CTA where they fit: a warp's load covers one 128-byte line
  // of a chunk's partial row.
  const int64_t fit = kFinalizeSmemFloats / np;
  auto go = [&](auto kern, int cols) -> cudaError_t {
    const size_t smem = static_cast<size_t>(np) * cols * sizeof(float);
    cudaError_t e = ensure_smem(kern, smem);
    if (e != cudaSuccess) return e;
    const dim3 grid(static_cast<unsigned>((f.ncols + cols - 1) / cols), static_cast<unsigned>(batch));
    return launch_pdl(kern, grid, dim3(kFinalizeThreads), smem, st, f);
  };
  if (fit >= 32) return go(colsum_finalize_kernel<32>, 32);
  if (fit >= 16) return go(colsum_finalize_kernel<16>, 16);
  if (fit >= 8) return go(colsum_finalize_kernel<8>, 8);
  if (fit >= 4) return go(colsum_finalize_kernel<4>, 4);
  if (fit >= 2) return go(colsum_finalize_kernel<2>, 2);
  return go(colsum_finalize_kernel<1>, 1);
}

}  // namespace afb
