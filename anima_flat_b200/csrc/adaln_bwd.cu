// AdaLN modulate backward (LoRA training), with and without the gated
// residual.
//
// Reference: src/kernels/adaln.py:111-172 (_residual_adaln_bwd_kernel) and
// :175-217 (_residual_adaln_bwd; partials reduced with torch .sum(1), cast to
// the parameter dtype).  Per row, with b = row / S and z the saved residual
// stream:
//   mean, rstd of z (canonical order, as the forward);  xhat = d * rstd
//   dxh = gh * scale[b];  c1 = sum(dxh) / D;  c2 = sum(dxh * xhat) / D
//   dz = rstd * ((dxh - c1) - xhat * c2)  (+ gz)        -> bf16 (dres)
//   dx = bf16(dz * gate[b])                               (HAS_X)
//   dshift[b] += gh;  dscale[b] += gh * xhat;  dgate[b] += dz * x   (fp32)
//
// Parameter-gradient order (deterministic, independent of the launch shape):
// the rows of each batch entry are cut into chunks of kChunkRows; in a chunk,
// warp w sums rows w, w + 4, w + 8, ... in increasing order; the four warp
// sums combine as a stride tree, (p0 + p2) + (p1 + p3); the chunk sums combine
// by a stride tree over the chunk index (finalize.cu) and round to bf16.  The chunk sums live in
// a caller-provided fp32 workspace [B][chunks][NQ][D].
#include <map>
#include <mutex>

#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

constexpr int kBwdWarps = 4;
constexpr int kRowsPerWarp = 4;
constexpr int kChunkRows = kBwdWarps * kRowsPerWarp;

struct AdalnBwdArgs {
  const uint16_t* gh;     // [rows, D]
  const uint16_t* gz;     // [rows, D] or null
  const uint16_t* z;      // [rows, D]
  const uint16_t* x;      // [rows, D] (HAS_X)
  const uint16_t* gate;   // [B, D] (HAS_X)
  const uint16_t* scale;  // [B, D]
  uint16_t* dz;           // [rows, D]
  uint16_t* dx;           // [rows, D] (HAS_X)
  float* part;            // [B][chunks][NQ][D]
  int64_t seq;
  int64_t chunks;         // per batch entry
  int dim;
  float eps;
};

// Shared-memory words per warp: NQ accumulators per column.
template <bool HAS_X>
__host__ __device__ constexpr int bwd_nq() { return HAS_X ? 3 : 2; }

template <int NC, bool HAS_X, bool HAS_GZ>
__global__ void __launch_bounds__(kBwdWarps * 32)
adaln_bwd_kernel(const AdalnBwdArgs a) {
  constexpr int NQ = bwd_nq<HAS_X>();
  extern __shared__ float4 smem4[];
  float* acc_all = reinterpret_cast<float*>(smem4);
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int D = a.dim;
  const int64_t b = blockIdx.y;
  const int64_t chunk = blockIdx.x;
  const int64_t pbase = b * D;
  // Per-warp accumulators, NQ planes of NC*256 floats laid out [c][half][lane][4]
  // so that every warp-wide float4 access is 512 contiguous bytes.
  constexpr int kPlane = NC * 256;
  float* acc = acc_all + static_cast<int64_t>(warp) * NQ * kPlane;
  auto slot = [&](int q, int c, int half) {
    return reinterpret_cast<float4*>(acc + q * kPlane + ((c * 2 + half) * 32 + lane) * 4);
  };
  const float fd = static_cast<float>(D);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      *slot(q, c, 0) = make_float4(0.f, 0.f, 0.f, 0.f);
      *slot(q, c, 1) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }

  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int64_t s = chunk * kChunkRows + i * kBwdWarps + warp;
    if (s >= a.seq) break;  // warp-uniform
    const int64_t base = (b * a.seq + s) * D;
    uint4 zv[NC], gv[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int e = (lane + 32 * c) * 8;
      const bool ok = e < D;
      zv[c] = ok ? ld_stream(a.z + base + e) : make_uint4(0, 0, 0, 0);
      gv[c] = ok ? ld_stream(a.gh + base + e) : make_uint4(0, 0, 0, 0);
    }
    // statistics of z, exactly as the forward
    const float mean = __fdiv_rn(
        warp_canonical_sum_fn<NC>([&](int c, int k) { return unpack_at(zv[c], k); }), fd);
    const float rstd = canonical_rstd(
        __fdiv_rn(warp_canonical_sum_fn<NC>([&](int c, int k) {
                    const float d = ((lane + 32 * c) * 8 < D) ? __fsub_rn(unpack_at(zv[c], k), mean)
                                                              : 0.0f;
                    return __fmul_rn(d, d);
                  }),
                  fd),
        a.eps);
    // c1 = sum(dxh) / D, c2 = sum(dxh * xhat) / D
    uint4 scv[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int e = (lane + 32 * c) * 8;
      scv[c] = (e < D) ? ld_keep(a.scale + pbase + e) : make_uint4(0, 0, 0, 0);
    }
    const float c1 = __fdiv_rn(warp_canonical_sum_fn<NC>([&](int c, int k) {
                                 return __fmul_rn(unpack_at(gv[c], k), unpack_at(scv[c], k));
                               }),
                               fd);
    const float c2 = __fdiv_rn(warp_canonical_sum_fn<NC>([&](int c, int k) {
                                 if ((lane + 32 * c) * 8 >= D) return 0.0f;
                                 const float xhat =
                                     __fmul_rn(__fsub_rn(unpack_at(zv[c], k), mean), rstd);
                                 const float dxh = __fmul_rn(unpack_at(gv[c], k), unpack_at(scv[c], k));
                                 return __fmul_rn(dxh, xhat);
                               }),
                               fd);
    // dz, dx and the column accumulators
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int e = (lane + 32 * c) * 8;
      if (e >= D) continue;
      float sc[8], g8[8], gz8[8], x8[8], dzf[8];
      unpack8(scv[c], sc);
      if (HAS_GZ) unpack8(ld_stream(a.gz + base + e), gz8);
      if (HAS_X) {
        unpack8(ld_keep(a.gate + pbase + e), g8);
        unpack8(ld_stream(a.x + base + e), x8);
      }
      float sh_acc[8], sc_acc[8], g_acc[8];
      {
        const float4 p0 = *slot(0, c, 0), p1 = *slot(0, c, 1), q0 = *slot(1, c, 0), q1 = *slot(1, c, 1);
        sh_acc[0] = p0.x; sh_acc[1] = p0.y; sh_acc[2] = p0.z; sh_acc[3] = p0.w;
        sh_acc[4] = p1.x; sh_acc[5] = p1.y; sh_acc[6] = p1.z; sh_acc[7] = p1.w;
        sc_acc[0] = q0.x; sc_acc[1] = q0.y; sc_acc[2] = q0.z; sc_acc[3] = q0.w;
        sc_acc[4] = q1.x; sc_acc[5] = q1.y; sc_acc[6] = q1.z; sc_acc[7] = q1.w;
      }
      if (HAS_X) {
        const float4 r0 = *slot(2, c, 0), r1 = *slot(2, c, 1);
        g_acc[0] = r0.x; g_acc[1] = r0.y; g_acc[2] = r0.z; g_acc[3] = r0.w;
        g_acc[4] = r1.x; g_acc[5] = r1.y; g_acc[6] = r1.z; g_acc[7] = r1.w;
      }
      float dxf[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float gh = unpack_at(gv[c], k);
        const float xhat = __fmul_rn(__fsub_rn(unpack_at(zv[c], k), mean), rstd);
        const float dxh = __fmul_rn(gh, sc[k]);
        float dz = __fmul_rn(rstd, __fsub_rn(__fsub_rn(dxh, c1), __fmul_rn(xhat, c2)));
        if (HAS_GZ) dz = __fadd_rn(dz, gz8[k]);
        dzf[k] = dz;
        sh_acc[k] = __fadd_rn(sh_acc[k], gh);
        sc_acc[k] = __fadd_rn(sc_acc[k], __fmul_rn(gh, xhat));
        if (HAS_X) {
          dxf[k] = __fmul_rn(dz, g8[k]);
          g_acc[k] = __fadd_rn(g_acc[k], __fmul_rn(dz, x8[k]));
        }
      }
      st16(a.dz + base + e, pack8_rn(dzf));
      if (HAS_X) st16(a.dx + base + e, pack8_rn(dxf));
      *slot(0, c, 0) = make_float4(sh_acc[0], sh_acc[1], sh_acc[2], sh_acc[3]);
      *slot(0, c, 1) = make_float4(sh_acc[4], sh_acc[5], sh_acc[6], sh_acc[7]);
      *slot(1, c, 0) = make_float4(sc_acc[0], sc_acc[1], sc_acc[2], sc_acc[3]);
      *slot(1, c, 1) = make_float4(sc_acc[4], sc_acc[5], sc_acc[6], sc_acc[7]);
      if (HAS_X) {
        *slot(2, c, 0) = make_float4(g_acc[0], g_acc[1], g_acc[2], g_acc[3]);
        *slot(2, c, 1) = make_float4(g_acc[4], g_acc[5], g_acc[6], g_acc[7]);
      }
    }
  }

  // Chunk partial: stride tree over the warps, (p0 + p2) + (p1 + p3).
  __syncthreads();
  float* out = a.part + ((b * a.chunks + chunk) * NQ) * D;
  const int stride = NQ * kPlane;
  for (int i = threadIdx.x; i < NQ * kPlane; i += blockDim.x) {
    const int q = i / kPlane, r = i % kPlane;
    const int kk = r & 3, ln = (r >> 2) & 31, half = (r >> 7) & 1, c = r >> 8;
    const int col = (ln + 32 * c) * 8 + half * 4 + kk;
    if (col >= D) continue;
    const float p0 = acc_all[i], p1 = acc_all[stride + i];
    const float p2 = acc_all[2 * stride + i], p3 = acc_all[3 * stride + i];
    out[q * D + col] = __fadd_rn(__fadd_rn(p0, p2), __fadd_rn(p1, p3));
  }
}

template <bool HAS_X, bool HAS_GZ>
static cudaError_t launch_adaln_bwd(const AdalnBwdArgs& a, int64_t batch, cudaStream_t st) {
  constexpr int NQ = bwd_nq<HAS_X>();
  const size_t smem = static_cast<size_t>(kBwdWarps) * NQ * row_chunks(a.dim) * 256 * sizeof(float);
  const dim3 grid(static_cast<unsigned>(a.chunks), static_cast<unsigned>(batch));
  const dim3 block(kBwdWarps * 32);
  cudaError_t e = cudaErrorInvalidValue;
  auto go = [&](auto kern) {
    cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (r != cudaSuccess) return r;
    return launch_pdl(kern, grid, block, smem, st, a);
  };
  switch (row_chunks(a.dim)) {
    case 1: e = go(adaln_bwd_kernel<1, HAS_X, HAS_GZ>); break;
    case 2: e = go(adaln_bwd_kernel<2, HAS_X, HAS_GZ>); break;
    case 4: e = go(adaln_bwd_kernel<4, HAS_X, HAS_GZ>); break;
    case 8: e = go(adaln_bwd_kernel<8, HAS_X, HAS_GZ>); break;
    default: e = cudaErrorInvalidValue; break;
  }
  return e;
}

size_t adaln_bwd_workspace(int64_t batch, int64_t seq, int64_t dim, bool has_x) {
  const int64_t chunks = (seq + kChunkRows - 1) / kChunkRows;
  return static_cast<size_t>(batch * chunks * (has_x ? 3 : 2) * dim) * sizeof(float);
}

// Shared implementation of the two entry points (and of the workspace-free
// variant): validates, then launches the row kernel and the finalize kernel.
int adaln_bwd_impl(const char* name, const void* gh, const void* gz, const void* z,
                   const void* x, const void* gate, const void* scale, void* dz, void* dx,
                   void* dgate, void* dshift, void* dscale, int64_t batch, int64_t seq,
                   int64_t dim, float eps, void* workspace, size_t workspace_bytes,
                   cudaStream_t st) {
  ApiGuard g(name);
  const bool has_x = x != nullptr;
  if (!check_rows(batch, seq, dim) ||
      !check(dim <= 2048, "backward supports dim <= 2048, got " + std::to_string(dim)) ||
      !check(finalize_fits((seq + kChunkRows - 1) / kChunkRows),
             "backward supports seq <= " + std::to_string(32768 * kChunkRows)) ||
      !check_ptrs({gh, z, scale, dz, dshift, dscale}, {"gh", "z", "scale", "dz", "dshift", "dscale"}) ||
      (gz != nullptr && !check_ptrs({gz}, {"gz"})) ||
      (has_x && !check_ptrs({gate, dx, dgate}, {"gate", "dx", "dgate"})) ||
      !check(workspace != nullptr && aligned(workspace, 16), "workspace is null or misaligned") ||
      !check(workspace_bytes >= adaln_bwd_workspace(batch, seq, dim, has_x),
             "workspace too small: need " + std::to_string(adaln_bwd_workspace(batch, seq, dim, has_x)) +
                 " bytes"))
    return g.fail();
  if (batch == 0) return 0;
  AdalnBwdArgs a{};
  a.gh = static_cast<const uint16_t*>(gh);
  a.gz = static_cast<const uint16_t*>(gz);
  a.z = static_cast<const uint16_t*>(z);
  a.x = static_cast<const uint16_t*>(x);
  a.gate = static_cast<const uint16_t*>(gate);
  a.scale = static_cast<const uint16_t*>(scale);
  a.dz = static_cast<uint16_t*>(dz);
  a.dx = static_cast<uint16_t*>(dx);
  a.part = static_cast<float*>(workspace);
  a.seq = seq;
  a.chunks = (seq + kChunkRows - 1) / kChunkRows;
  a.dim = static_cast<int>(dim);
  a.eps = eps;
  cudaError_t e;
  if (has_x) e = gz ? launch_adaln_bwd<true, true>(a, batch, st) : launch_adaln_bwd<true, false>(a, batch, st);
  else e = gz ? launch_adaln_bwd<false, true>(a, batch, st) : launch_adaln_bwd<false, false>(a, batch, st);
  if (e != cudaSuccess) return g.done(e);
  FinalizeArgs f{};
  f.part = static_cast<const float*>(workspace);
  f.n = a.chunks;
  f.ncols = (has_x ? 3 : 2) * static_cast<int>(dim);
  f.seg = static_cast<int>(dim);
  f.out[0] = dshift;
  f.out[1] = dscale;
  f.out[2] = dgate;
  f.bf16_out = 1;
  return g.done(launch_colsum_finalize(f, batch, st));
}

// ---------------------------------------------------------------------------
// Scratch for afb_residual_adaln_bwd_noalloc: some callers of this library
// cannot allocate device memory at all (a host binding with no device
// allocator of its own, or a serving process whose device memory is fully
// reserved at start-up and which forbids allocation on the hot path).  For
// them the parameter-gradient partials live in this file-scope array
// instead of a caller-provided workspace.  Every GPU that loads the library
// holds these 16 MiB until the process exits.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of the scratch array for the current device.  The name of
// the array is only a host-side stand-in; the address is looked up once per
// device (with that device current) and cached.
static cudaError_t noalloc_scratch(void** ptr) {
  static std::mutex mu;
  static std::map<int, void*> cache;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) {
    *ptr = it->second;
    return cudaSuccess;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return e;
  cache.emplace(dev, p);
  *ptr = p;
  return cudaSuccess;
}

}  // namespace afb

using namespace afb;

// Allocation-free variant of afb_residual_adaln_bwd (see the scratch comment
// above).  The first call on a device looks up the scratch address; make that
// first call before any stream capture.  The partial sums it keeps there are
// fully overwritten by every call, so nothing needs clearing, but all calls
// share the one array: calls that overlap on the GPU (other streams, other
// threads) race.  Sizes whose partials exceed 16 MiB are rejected.
extern "C" int afb_residual_adaln_bwd_noalloc(const void* gh, const void* gz, const void* z,
                                              const void* x, const void* gate, const void* scale,
                                              void* dx, void* dres, void* dgate, void* dshift,
                                              void* dscale, int64_t batch, int64_t seq,
                                              int64_t dim, float eps, void* stream) {
  const char* name = "afb_residual_adaln_bwd_noalloc";
  if (batch >= 0 && seq >= 1 && dim >= 1 &&
      adaln_bwd_workspace(batch, seq, dim, true) > kNoAllocScratchBytes) {
    set_error(std::string(name) + ": this size needs " +
              std::to_string(adaln_bwd_workspace(batch, seq, dim, true)) +
              " bytes of scratch, more than the " + std::to_string(kNoAllocScratchBytes) +
              " bytes this entry point holds; use afb_residual_adaln_bwd with a workspace");
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (x == nullptr) {
    set_error(std::string(name) + ": x is null");
    return static_cast<int>(cudaErrorInvalidValue);
  }
  void* scratch = nullptr;
  const cudaError_t e = noalloc_scratch(&scratch);
  if (e != cudaSuccess) {
    set_error(std::string(name) + ": cannot resolve the scratch array: " + cudaGetErrorString(e));
    return static_cast<int>(e);
  }
  return adaln_bwd_impl(name, gh, gz, z, x, gate, scale, dres, dx, dgate, dshift, dscale, batch,
                        seq, dim, eps, scratch, kNoAllocScratchBytes,
                        static_cast<cudaStream_t>(stream));
}

extern "C" size_t afb_residual_adaln_bwd_workspace(int64_t batch, int64_t seq, int64_t dim) {
  return adaln_bwd_workspace(batch, seq, dim, true);
}

extern "C" size_t afb_adaln_bwd_workspace(int64_t batch, int64_t seq, int64_t dim) {
  return adaln_bwd_workspace(batch, seq, dim, false);
}

extern "C" int afb_residual_adaln_bwd(const void* gh, const void* gz, const void* z, const void* x,
                                      const void* gate, const void* scale, void* dx, void* dres,
                                      void* dgate, void* dshift, void* dscale, int64_t batch,
                                      int64_t seq, int64_t dim, float eps, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  if (x == nullptr) {
    set_error("afb_residual_adaln_bwd: x is null");
    return static_cast<int>(cudaErrorInvalidValue);
  }
  return adaln_bwd_impl("afb_residual_adaln_bwd", gh, gz, z, x, gate, scale, dres, dx, dgate,
                        dshift, dscale, batch, seq, dim, eps, workspace, workspace_bytes,
                        static_cast<cudaStream_t>(stream));
}

extern "C" int afb_adaln_bwd(const void* gh, const void* z, const void* scale, void* dz,
                             void* dshift, void* dscale, int64_t batch, int64_t seq, int64_t dim,
                             float eps, void* workspace, size_t workspace_bytes, void* stream) {
  return adaln_bwd_impl("afb_adaln_bwd", gh, nullptr, z, nullptr, nullptr, scale, dz, nullptr,
                        nullptr, dshift, dscale, batch, seq, dim, eps, workspace, workspace_bytes,
                        static_cast<cudaStream_t>(stream));
}
