// Column sums of per-chunk partials, for the parameter gradients of the
// backward kernels (the reference reduces its partials with torch .sum,
// adaln.py:214-216 and rope.py:471, :575-576).
//
// Order: for each batch entry and column, the n chunk partials are summed by
// a stride tree over the chunk index, zero-padded to np = pow2ceil(n):
// p[s] += p[s + np/2], then np/4, ... down to p[0].  The tree runs in shared
// memory: a CTA holds np partials for COLS columns and halves them level by
// level, so the result does not depend on the launch shape.
//
// Many chunks (np > kFinalizeDirect) go through two launches computing the
// same tree.  Its first log2(K) levels, K = np / Q, only ever combine
// partials whose chunk index agrees mod Q: for each s < Q they are the stride
// tree over the rows s + k*Q, k < K.  Seen as a [K][Q * ncols] matrix (row k
// = the Q contiguous partial rows from k*Q), that is this kernel's column
// reduction; it runs first and writes the Q subtree sums over partial rows
// [0, Q) in place (a CTA reads all of its columns before it writes them, and
// no other CTA reads them).  The second launch is the stride tree over those
// Q rows.  So a large reduction spreads over many CTAs instead of one CTA
// per column block.
#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

constexpr int kFinalizeThreads = 256;
constexpr int kFinalizeSmemFloats = 32768;  // 128 KiB
constexpr int64_t kFinalizeDirect = 1024;   // largest np reduced in one launch
constexpr int64_t kFinalizeSplit = 256;     // Q of the two-launch form

// grid: (ceil(ncols / COLS), batch); dynamic smem: np * COLS floats.  Thread t
// owns column t % COLS of the block and the partial rows t / COLS + k * RPI, so
// the index arithmetic is shifts and a warp's load covers whole lines.
template <int COLS>
__global__ void __launch_bounds__(kFinalizeThreads)
colsum_finalize_kernel(const FinalizeArgs f) {
  constexpr int RPI = kFinalizeThreads / COLS;  // partial rows per pass of the CTA
  constexpr int kBatch = 8;                     // loads in flight per thread
  extern __shared__ float sm[];
  pdl_wait();
  pdl_trigger();
  const int t = threadIdx.x;
  const int c = t % COLS;
  const int r = t / COLS;
  const int64_t b = blockIdx.y;
  const int col = blockIdx.x * COLS + c;
  const bool cok = col < f.ncols;
  // Rows s = r, r + RPI, ..., kBatch at a time with all their loads issued
  // before the stores into shared memory; rows past the end (and, in the
  // strided view, floats past the batch entry's partials) read as zero.
  const float* p = f.part + b * f.bstride;
  const int64_t step = static_cast<int64_t>(RPI) * f.ncols;
  int64_t at = static_cast<int64_t>(r) * f.ncols + col;  // flat index of (row s, this column)
  for (int s0 = r; s0 < f.np; s0 += kBatch * RPI) {
    float v[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int s = s0 + u * RPI;
      v[u] = (cok && s < f.n && at < f.nflat) ? __ldg(p + at) : 0.0f;
      at += step;
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
    const int64_t o = b * f.out_bstride + col % f.seg;
    void* dst = seg == 0 ? f.out[0] : seg == 1 ? f.out[1] : f.out[2];  // no local copy of out[]
    if (f.bf16_out) {
      static_cast<uint16_t*>(dst)[o] = static_cast<uint16_t>(pack2_rn(sm[c], 0.0f) & 0xffffu);
    } else {
      static_cast<float*>(dst)[o] = sm[c];
    }
  }
}

bool finalize_fits(int64_t n) { return n >= 1 && n <= kFinalizeSmemFloats; }

// One launch: f.n rows (np = pow2ceil) of f.ncols columns per batch entry.
static cudaError_t launch_finalize_one(FinalizeArgs f, int64_t batch, cudaStream_t st) {
  const DeviceInfo& dev = device_info();
  if (dev.error != cudaSuccess) return dev.error;
  int64_t np = 1;
  while (np < f.n) np <<= 1;
  if (np > kFinalizeSmemFloats) return cudaErrorInvalidValue;
  f.np = static_cast<int>(np);
  // Up to 32 columns per CTA (a warp's load covers a 128-byte line of a
  // partial row), fewer while that leaves under two CTAs per SM.
  const int64_t fit = kFinalizeSmemFloats / np;
  int cols = 32;
  while (cols > 1 && cols > fit) cols >>= 1;
  while (cols > 4 && ((f.ncols + cols - 1) / cols) * batch < 2 * static_cast<int64_t>(dev.sms)) cols >>= 1;
  auto go = [&](auto kern) -> cudaError_t {
    const size_t smem = static_cast<size_t>(np) * cols * sizeof(float);
    cudaError_t e = ensure_smem(kern, smem, true);
    if (e != cudaSuccess) return e;
    const dim3 grid(static_cast<unsigned>((f.ncols + cols - 1) / cols), static_cast<unsigned>(batch));
    return launch_pdl(kern, grid, dim3(kFinalizeThreads), smem, st, f);
  };
  switch (cols) {
    case 32: return go(colsum_finalize_kernel<32>);
    case 16: return go(colsum_finalize_kernel<16>);
    case 8: return go(colsum_finalize_kernel<8>);
    case 4: return go(colsum_finalize_kernel<4>);
    case 2: return go(colsum_finalize_kernel<2>);
    default: return go(colsum_finalize_kernel<1>);
  }
}

cudaError_t launch_colsum_finalize(const FinalizeArgs& in, int64_t batch, cudaStream_t st) {
  int64_t np = 1;
  while (np < in.n) np <<= 1;
  if (np > kFinalizeSmemFloats) return cudaErrorInvalidValue;
  const int64_t block = in.n * in.ncols;  // floats of a batch entry's partials
  if (np <= kFinalizeDirect) {
    FinalizeArgs f = in;
    f.bstride = block;
    f.nflat = block;
    f.out_bstride = f.seg;
    return launch_finalize_one(f, batch, st);
  }
  // The first log2(np / Q) levels: column reduction of the [K][Q * ncols]
  // view, written in place over partial rows [0, Q).
  const int64_t Q = kFinalizeSplit;
  FinalizeArgs a = in;
  a.n = np / Q;
  a.ncols = static_cast<int>(Q * in.ncols);
  a.seg = a.ncols;
  a.out[0] = const_cast<float*>(in.part);
  a.out[1] = a.out[2] = nullptr;
  a.bf16_out = 0;
  a.bstride = block;
  a.nflat = block;
  a.out_bstride = block;
  cudaError_t e = launch_finalize_one(a, batch, st);
  if (e != cudaSuccess) return e;
  // The last log2(Q) levels over those Q rows.
  FinalizeArgs b = in;
  b.n = Q;
  b.bstride = block;
  b.nflat = Q * in.ncols;
  b.out_bstride = b.seg;
  return launch_finalize_one(b, batch, st);
}

}  // namespace afb
