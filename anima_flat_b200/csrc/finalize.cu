// Column sums of per-chunk partials, for the parameter gradients of the
// backward kernels (the reference reduces its partials with torch .sum,
// adaln.py:214-216 and rope.py:471, :575-576).
//
// Order: for each batch entry and column, the n chunk partials are summed by
// a stride tree over the chunk index, zero-padded to np = pow2ceil(n):
// p[s] += p[s + np/2], then np/4, ... down to p[0], so the result does not
// depend on the launch shape.
//
// Many chunks (np > kFinalizeDirect) go through two launches computing the
// same tree.  Its first log2(K) levels, K = np / Q, only ever combine
// partials whose chunk index agrees mod Q: for each s < Q they are the stride
// tree over the rows s + k*Q, k < K.  Seen as a [K][Q * ncols] matrix (row k
// = the Q contiguous partial rows from k*Q), that is this kernel's column
// reduction; it runs first and writes the Q subtree sums over partial rows
// [0, Q) in place (a CTA reads all of its columns before it writes them, and
// no other CTA reads them).  The second launch is the stride tree over those
// Q rows.  So a large reduction spreads over many CTAs.
#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

constexpr int kFinalizeSmemFloats = 32768;  // largest np (finalize_fits)
constexpr int64_t kFinalizeDirect = 1024;   // largest np reduced in one launch
constexpr int64_t kFinalizeSplit = 256;     // Q of the two-launch form

// One CTA reduces 32 columns (lane = column) of one batch entry over np =
// RT * NW partial rows (NW warps).  Thread (w, lane) holds the rows
// w + NW * k, k < RT, in registers: the stride tree's levels with stride
// np/2 .. NW pair rows of equal w, so they run in the thread (a stride tree
// over k); the last log2(NW) levels (strides NW/2 .. 1) pair the warps' values
// through shared memory, in warp 0.  Same order as a stride tree over all np
// rows.  Loads of a warp cover whole 128-byte lines of a partial row.
template <int RT>
__global__ void __launch_bounds__(1024)
colsum_finalize_kernel(const FinalizeArgs f) {
  __shared__ float xs[32][33];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const int64_t b = blockIdx.y;
  const int col = blockIdx.x * 32 + lane;
  const bool cok = col < f.ncols;
  const float* p = f.part + b * f.bstride + col;
  float v[RT];
#pragma unroll
  for (int k = 0; k < RT; ++k) {
    const int64_t s = w + static_cast<int64_t>(nw) * k;
    const int64_t at = s * f.ncols + col;  // flat index of (row s, this column)
    v[k] = (cok && s < f.n && at < f.nflat) ? __ldg(p + s * f.ncols) : 0.0f;
  }
#pragma unroll
  for (int h = RT / 2; h >= 1; h >>= 1) {
#pragma unroll
    for (int k = 0; k < h; ++k) v[k] = __fadd_rn(v[k], v[k + h]);
  }
  xs[w][lane] = v[0];
  __syncthreads();
  if (w != 0 || !cok) return;
  // each lane combines its own column's warp values in place
  for (int h = nw / 2; h >= 1; h >>= 1)
    for (int u = 0; u < h; ++u) xs[u][lane] = __fadd_rn(xs[u][lane], xs[u + h][lane]);
  const float t0 = xs[0][lane];
  const int seg = col / f.seg;
  const int64_t o = b * f.out_bstride + col % f.seg;
  void* dst = seg == 0 ? f.out[0] : seg == 1 ? f.out[1] : f.out[2];  // no local copy of out[]
  if (f.bf16_out) {
    static_cast<uint16_t*>(dst)[o] = static_cast<uint16_t>(pack2_rn(t0, 0.0f) & 0xffffu);
  } else {
    static_cast<float*>(dst)[o] = t0;
  }
}

bool finalize_fits(int64_t n) { return n >= 1 && n <= kFinalizeSmemFloats; }

// One launch: f.n rows (np = pow2ceil <= kFinalizeDirect) of f.ncols columns
// per batch entry.  RT = np / NW rows per thread, NW <= 32 warps.
static cudaError_t launch_finalize_one(FinalizeArgs f, int64_t batch, cudaStream_t st) {
  int64_t np = 1;
  while (np < f.n) np <<= 1;
  if (np > kFinalizeDirect) return cudaErrorInvalidValue;
  f.np = static_cast<int>(np);
  int rt = static_cast<int>(np / 8);
  rt = rt < 1 ? 1 : rt > 32 ? 32 : rt;
  const int nw = static_cast<int>(np / rt);
  auto go = [&](auto kern) -> cudaError_t {
    const dim3 grid(static_cast<unsigned>((f.ncols + 31) / 32), static_cast<unsigned>(batch));
    return launch_pdl(kern, grid, dim3(nw * 32), 0, st, f);
  };
  switch (rt) {
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
