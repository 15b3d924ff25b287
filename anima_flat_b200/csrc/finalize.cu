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

// grid: (ceil(ncols / cols), batch); dynamic smem: np * cols floats.
__global__ void __launch_bounds__(kFinalizeThreads)
colsum_finalize_kernel(const FinalizeArgs f, const int cols) {
  extern __shared__ float sm[];
  pdl_wait();
  pdl_trigger();
  const int t = threadIdx.x;
  const int64_t b = blockIdx.y;
  const int c0 = blockIdx.x * cols;
  const float* part = f.part + b * f.n * f.ncols;
  const int total = f.np * cols;
  for (int idx = t; idx < total; idx += kFinalizeThreads) {
    const int64_t s = idx / cols;
    const int c = c0 + idx % cols;
    sm[idx] = (s < f.n && c < f.ncols) ? part[s * f.ncols + c] : 0.0f;
  }
  for (int h = f.np / 2; h >= 1; h >>= 1) {
    __syncthreads();
    for (int idx = t; idx < h * cols; idx += kFinalizeThreads) sm[idx] = __fadd_rn(sm[idx], sm[idx + h * cols]);
  }
  __syncthreads();
  if (t < cols && c0 + t < f.ncols) {
    const int c = c0 + t;
    const int seg = c / f.seg;
    const int64_t o = b * f.seg + c % f.seg;
    if (f.bf16_out) {
      static_cast<uint16_t*>(f.out[seg])[o] = static_cast<uint16_t>(pack2_rn(sm[t], 0.0f) & 0xffffu);
    } else {
      static_cast<float*>(f.out[seg])[o] = sm[t];
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
  int cols = static_cast<int>(kFinalizeSmemFloats / np);
  if (cols > 16) cols = 16;
  const size_t smem = static_cast<size_t>(np) * cols * sizeof(float);
  cudaError_t e = ensure_smem(colsum_finalize_kernel, smem);
  if (e != cudaSuccess) return e;
  const dim3 grid(static_cast<unsigned>((f.ncols + cols - 1) / cols), static_cast<unsigned>(batch));
  return launch_pdl(colsum_finalize_kernel, grid, dim3(kFinalizeThreads), smem, st, f, cols);
}

}  // namespace afb
