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
// the rows of each batch entry are cut into chunks of kChunkRows = 16; in a
// chunk, stream w (w < 4) sums rows w, w + 4, w + 8, w + 12 in increasing
// order from zero; the four stream sums combine as a stride tree,
// (p0 + p2) + (p1 + p3); the chunk sums combine by a stride tree over the
// chunk index (finalize.cu) and round to bf16.
//
// Two passes, so that no thread needs a whole row's parameter sums:
//  1. adaln_bwd_stats_kernel, one row per warp pair as in the forward kernel
//     (bulk-copied z and gh, scale rows in shared memory): the row scalars
//     mean, rstd, c1, c2 (canonical sums) into the workspace.
//  2. adaln_bwd_cols_kernel, one 8-column vector per thread and one chunk per
//     CTA: the thread walks the chunk's rows in stream order, forms dz and dx
//     from the row scalars, stores them, and keeps its columns' stream sums in
//     registers.  z and gh were just read by pass 1 and are normally still in
//     the L2, so the DRAM traffic stays close to one pass.
// Workspace: [rows][4] fp32 row scalars, then the [B][chunks][NQ][D] fp32
// chunk sums.
#include <map>
#include <mutex>

#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

constexpr int kStreams = 4;
constexpr int kRowsPerStream = 4;
constexpr int kChunkRows = kStreams * kRowsPerStream;

// ---------------------------------------------------------------------------
// Pass 1: row scalars.
// ---------------------------------------------------------------------------
constexpr int kStatPairs = 8;
constexpr int kStatWarps = 2 * kStatPairs;
constexpr int kStatStages = 2;
constexpr int kStatModSlots = 2;
// Per pair: exchange buffers A (mean), B (variance) of 2 warps x 4 pairs x 32
// lanes, and C (c1 and c2 together) of twice that.
constexpr size_t kStatXchF2 = 4 * 2 * 4 * 32;

struct AdalnStatsArgs {
  const uint16_t* gh;     // [rows, D]
  const uint16_t* z;      // [rows, D]
  const uint16_t* scale;  // [B, D]
  float4* stats;          // [rows] (mean, rstd, c1, c2)
  int64_t rows;
  int64_t seq;
  int dim;
  float eps;
};

template <int NC, bool EXACT>
__global__ void __launch_bounds__(kStatWarps * 32, 1)
adaln_bwd_stats_kernel(const AdalnStatsArgs a, const int use_smods) {
  constexpr bool SPLIT = NC >= 2;
  constexpr int NH = SPLIT ? NC / 2 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int pair = warp >> 1;
  const int h = warp & 1;
  const int bar_id = 1 + pair;
  const bool leader = h == 0 && lane == 0;
  const int D = EXACT ? NC * 256 : a.dim;
  const uint32_t row_bytes = static_cast<uint32_t>(D) * 2u;
  const uint32_t stage_bytes = 2u * row_bytes;  // z | gh
  const size_t ring_all = static_cast<size_t>(kStatPairs) * kStatStages * stage_bytes;
  uint8_t* ring = smem + static_cast<size_t>(pair) * kStatStages * stage_bytes;
  f2_t* xch = reinterpret_cast<f2_t*>(smem + ring_all) + pair * kStatXchF2;
  uint8_t* mods = smem + ring_all + kStatPairs * kStatXchF2 * sizeof(f2_t);
  uint64_t* bars0 = reinterpret_cast<uint64_t*>(mods + (use_smods ? kStatModSlots * row_bytes : 0u));
  uint64_t* bars = bars0 + pair * kStatStages;
  uint64_t* modbar = bars0 + kStatPairs * kStatStages;

  const int64_t r0 = a.rows * blockIdx.x / gridDim.x;
  const int64_t r1 = a.rows * (blockIdx.x + 1) / gridDim.x;
  const int64_t b_lo = r1 > r0 ? r0 / a.seq : 0;
  const int64_t b_hi = r1 > r0 ? (r1 - 1) / a.seq : 0;
  const bool smods = use_smods && r1 > r0 && b_hi - b_lo < kStatModSlots;
  if (leader) {
    for (int s = 0; s < kStatStages; ++s) mbar_init(smem_addr(&bars[s]), 1);
    if (pair == 0) mbar_init(smem_addr(modbar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  if (smods && threadIdx.x == 0) {  // the scale rows go first, ahead of every row stage
    const int nb = static_cast<int>(b_hi - b_lo + 1);
    mbar_arrive_expect_tx(smem_addr(modbar), static_cast<uint32_t>(nb) * row_bytes);
    for (int k = 0; k < nb; ++k)
      bulk_g2s(smem_addr(mods + k * row_bytes), a.scale + (b_lo + k) * D, row_bytes, smem_addr(modbar));
  }
  if (smods) __syncthreads();

  auto row_of = [&](int64_t j) { return r0 + pair + j * kStatPairs; };
  auto issue = [&](int64_t j) {
    const int64_t row = row_of(j);
    const int s = static_cast<int>(j % kStatStages);
    uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    const uint32_t bar = smem_addr(&bars[s]);
    mbar_arrive_expect_tx(bar, stage_bytes);
    bulk_g2s(smem_addr(st), a.z + row * D, row_bytes, bar);
    bulk_g2s(smem_addr(st + row_bytes), a.gh + row * D, row_bytes, bar);
  };
  if (leader) {
    for (int j = 0; j < kStatStages && row_of(j) < r1; ++j) issue(j);
  }
  auto col = [&](int i) { return (lane + 32 * (SPLIT ? 2 * i + h : i)) * 8; };
  auto ok = [&](int i) { return EXACT || col(i) < D; };
  auto div_d = [&](float x) {
    return EXACT ? __fmul_rn(x, 1.0f / (NC * 256)) : __fdiv_rn(x, static_cast<float>(D));
  };

  bool dead = false;
  int64_t jdead = 0;
  if (smods && !mbar_wait(smem_addr(modbar), 0)) dead = true;
  for (int64_t j = 0; row_of(j) < r1; ++j) {
    const int64_t row = row_of(j);
    const int s = static_cast<int>(j % kStatStages);
    const uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    if (!dead && !mbar_wait(smem_addr(&bars[s]), static_cast<uint32_t>((j / kStatStages) & 1))) {
      dead = true;
      jdead = j;
    }
    const int64_t b = row / a.seq;
    f2_t zf[NH][4];
    uint4 gv[NH];
#pragma unroll
    for (int i = 0; i < NH; ++i) {
      const uint4 zv = ok(i) ? lds16(st + col(i) * 2) : make_uint4(0, 0, 0, 0);
      gv[i] = ok(i) ? lds16(st + row_bytes + col(i) * 2) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) zf[i][jj] = bf2f2(word(zv, jj));
    }
    // dxh = gh * scale (fp32 pairs)
    f2_t dxh[NH][4];
#pragma unroll
    for (int i = 0; i < NH; ++i) {
      const uint4 scv = !ok(i) ? make_uint4(0, 0, 0, 0)
                        : smods ? lds16(mods + static_cast<size_t>(b - b_lo) * row_bytes + col(i) * 2)
                                : ld_keep(a.scale + b * D + col(i));
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) dxh[i][jj] = mul2_noc(bf2f2(word(gv[i], jj)), bf2f2(word(scv, jj)));
    }
    // Round 1: sum(z) and sum(dxh), which need nothing else.
    float mean, c1;
    pair_canonical_sum2x2<NH, SPLIT>([&](int n, int i, int jj) { return n == 0 ? zf[i][jj] : dxh[i][jj]; }, xch, h,
                                     lane, bar_id, mean, c1);
    mean = div_d(mean);
    c1 = div_d(c1);
    if (!SPLIT) named_bar_sync(bar_id, 64);
    if (leader && !dead && row_of(j + kStatStages) < r1) {  // both warps have read the stage
      fence_proxy_async_smem();
      issue(j + kStatStages);
    }
    const f2_t mm = f2(mean, mean);
#pragma unroll
    for (int i = 0; i < NH; ++i) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) zf[i][jj] = ok(i) ? sub2(zf[i][jj], mm) : 0ull;  // d = z - mean
    }
    // Round 2: sum(d * d) and sum(dxh * d); c2 = (sum(dxh * d) * rstd) / D.
    float var, e;
    pair_canonical_sum2x2<NH, SPLIT>(
        [&](int n, int i, int jj) { return mul2_noc(n == 0 ? zf[i][jj] : dxh[i][jj], zf[i][jj]); },
        xch + 2 * 2 * 4 * 32, h, lane, bar_id, var, e);
    const float rstd = canonical_rstd(div_d(var), a.eps);
    const float c2 = div_d(__fmul_rn(e, rstd));
    if (leader && !dead) a.stats[row] = make_float4(mean, rstd, c1, c2);
  }
  if (leader && dead) {
    for (int64_t k = jdead; k < jdead + kStatStages && row_of(k) < r1; ++k)
      mbar_wait(smem_addr(&bars[k % kStatStages]), static_cast<uint32_t>((k / kStatStages) & 1));
    if (pair == 0 && smods) mbar_wait(smem_addr(modbar), 0);
  }
}

// ---------------------------------------------------------------------------
// Pass 2: dz, dx and the chunk sums of the parameter gradients.  Lane group w
// (lanes 8w .. 8w+7) of a warp runs stream w of one chunk for 8 consecutive
// 8-column vectors: its four rows are loaded at once, so a thread makes one
// round trip.  The stream sums combine by xor shuffles in the canonical order:
// (p0 + p2) and (p1 + p3) across lane distance 16, then their sum across 8.
// ---------------------------------------------------------------------------
constexpr int kColWarps = 4;
constexpr int kColVecsPerWarp = 8;                                   // 64 columns per warp
constexpr int kColCols = kColWarps * kColVecsPerWarp * 8;             // 256 columns per CTA

struct AdalnColsArgs {
  const uint16_t* gh;     // [rows, D]
  const uint16_t* gz;     // [rows, D] or null
  const uint16_t* z;      // [rows, D]
  const uint16_t* x;      // [rows, D] (HAS_X)
  const uint16_t* gate;   // [B, D] (HAS_X)
  const uint16_t* scale;  // [B, D]
  const float4* stats;    // [rows]
  uint16_t* dz;           // [rows, D]
  uint16_t* dx;           // [rows, D] (HAS_X)
  float* part;            // [B][chunks][NQ][D]
  int64_t seq;
  int64_t chunks;
  int dim;
};

template <bool HAS_X>
__host__ __device__ constexpr int bwd_nq() { return HAS_X ? 3 : 2; }

// grid (ceil(D / 256), chunks, B)
template <bool HAS_X, bool HAS_GZ>
__global__ void __launch_bounds__(kColWarps * 32, 4)
adaln_bwd_cols_kernel(const AdalnColsArgs a) {
  constexpr int NQ = bwd_nq<HAS_X>();
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int w = lane >> 3;  // stream
  const int64_t ch = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int D = a.dim;
  const int col = ((blockIdx.x * kColWarps + warp) * kColVecsPerWarp + (lane & 7)) * 8;
  const bool cok = col < D;
  const int64_t s0 = ch * kChunkRows;

  float acc[NQ][8];
#pragma unroll
  for (int q = 0; q < NQ; ++q)
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[q][k] = 0.0f;
  if (cok) {
    uint4 zv[kRowsPerStream], gv[kRowsPerStream], gzv[kRowsPerStream], xv[kRowsPerStream];
    float4 t[kRowsPerStream];
#pragma unroll
    for (int r = 0; r < kRowsPerStream; ++r) {  // the stream's rows, all in flight at once
      const int64_t s = s0 + r * kStreams + w;
      if (s < a.seq) {
        const int64_t o = (b * a.seq + s) * D + col;
        zv[r] = ld_stream(a.z + o);
        gv[r] = ld_stream(a.gh + o);
        if (HAS_GZ) gzv[r] = ld_stream(a.gz + o);
        if (HAS_X) xv[r] = ld_stream(a.x + o);
        t[r] = a.stats[b * a.seq + s];  // mean, rstd, c1, c2
      }
    }
    float sc[8], gt[8];
    unpack8(ld_keep(a.scale + b * D + col), sc);
    if (HAS_X) unpack8(ld_keep(a.gate + b * D + col), gt);
#pragma unroll
    for (int r = 0; r < kRowsPerStream; ++r) {
      const int64_t s = s0 + r * kStreams + w;
      if (s >= a.seq) break;
      const int64_t o = (b * a.seq + s) * D + col;
      float dzf[8], dxf[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float g = unpack_at(gv[r], k);
        const float xhat = __fmul_rn(__fsub_rn(unpack_at(zv[r], k), t[r].x), t[r].y);
        const float dxh = __fmul_rn(g, sc[k]);
        float dz = __fmul_rn(t[r].y, __fsub_rn(__fsub_rn(dxh, t[r].z), __fmul_rn(xhat, t[r].w)));
        if (HAS_GZ) dz = __fadd_rn(dz, unpack_at(gzv[r], k));
        dzf[k] = dz;
        acc[0][k] = __fadd_rn(acc[0][k], g);
        acc[1][k] = __fadd_rn(acc[1][k], __fmul_rn(g, xhat));
        if (HAS_X) {
          dxf[k] = __fmul_rn(dz, gt[k]);
          acc[2][k] = __fadd_rn(acc[2][k], __fmul_rn(dz, unpack_at(xv[r], k)));
        }
      }
      st16(a.dz + o, pack8_rn(dzf));
      if (HAS_X) st16(a.dx + o, pack8_rn(dxf));
    }
  }
  // (p0 + p2) + (p1 + p3): lane groups 0/2 and 1/3 are 16 lanes apart, then
  // groups 0/1 are 8 apart.  Commutative adds give the same bits in every lane.
#pragma unroll
  for (int q = 0; q < NQ; ++q)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float v = __fadd_rn(acc[q][k], __shfl_xor_sync(kFull, acc[q][k], 16));
      acc[q][k] = __fadd_rn(v, __shfl_xor_sync(kFull, v, 8));
    }
  if (cok && w == 0) {
    float* out = a.part + ((b * a.chunks + ch) * NQ) * D + col;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      float4* o4 = reinterpret_cast<float4*>(out + q * D);
      o4[0] = make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]);
      o4[1] = make_float4(acc[q][4], acc[q][5], acc[q][6], acc[q][7]);
    }
  }
}

// Pass-1 launch plan: shared memory for the rings, exchange buffers, and (when
// they fit) the scale slots.
static cudaError_t launch_adaln_bwd_stats(const AdalnStatsArgs& a, cudaStream_t st) {
  const DeviceInfo& dev = device_info();
  if (dev.error != cudaSuccess) return dev.error;
  const size_t row = static_cast<size_t>(a.dim) * 2;
  const size_t base = static_cast<size_t>(kStatPairs) * kStatStages * 2 * row + kStatPairs * kStatXchF2 * sizeof(f2_t) +
                      (kStatPairs * kStatStages + 1) * sizeof(uint64_t);
  const int smods = base + kStatModSlots * row <= dev.max_smem_optin;
  const size_t smem = base + (smods ? kStatModSlots * row : 0);
  if (smem > dev.max_smem_optin) return cudaErrorInvalidValue;
  const int nc = row_chunks(a.dim);
  const bool exact = a.dim == 256 * nc;
  const int64_t want = (a.rows + kStatPairs - 1) / kStatPairs;
  const dim3 grid(static_cast<unsigned>(want < dev.sms ? want : dev.sms));
  auto go = [&](auto kern) -> cudaError_t {
    cudaError_t e = ensure_smem(kern, smem, true);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, grid, dim3(kStatWarps * 32), smem, st, a, smods);
  };
#define AFB_LAUNCH_STATS(NC) \
  return exact ? go(adaln_bwd_stats_kernel<NC, true>) : go(adaln_bwd_stats_kernel<NC, false>)
  switch (nc) {
    case 1: AFB_LAUNCH_STATS(1);
    case 2: AFB_LAUNCH_STATS(2);
    case 4: AFB_LAUNCH_STATS(4);
    case 8: AFB_LAUNCH_STATS(8);
    default: return cudaErrorInvalidValue;
  }
#undef AFB_LAUNCH_STATS
}

template <bool HAS_X, bool HAS_GZ>
static cudaError_t launch_adaln_bwd_cols(const AdalnColsArgs& a, int64_t batch, cudaStream_t st) {
  const dim3 grid(static_cast<unsigned>((a.dim + kColCols - 1) / kColCols), static_cast<unsigned>(a.chunks),
                  static_cast<unsigned>(batch));
  // The same shared-memory carveout as the stats and finalize kernels around
  // it, so consecutive launches need no reconfiguration of the SMs.
  cudaError_t e = ensure_smem(adaln_bwd_cols_kernel<HAS_X, HAS_GZ>, 0, true);
  if (e != cudaSuccess) return e;
  return launch_pdl(adaln_bwd_cols_kernel<HAS_X, HAS_GZ>, grid, dim3(kColWarps * 32), 0, st, a);
}

cudaError_t read_status_adaln_bwd(int* status) {
  return cudaMemcpyFromSymbol(status, g_afb_device_status, sizeof(int));
}

static size_t adaln_bwd_stats_bytes(int64_t batch, int64_t seq) {
  return static_cast<size_t>(batch * seq) * sizeof(float4);
}

size_t adaln_bwd_workspace(int64_t batch, int64_t seq, int64_t dim, bool has_x) {
  const int64_t chunks = (seq + kChunkRows - 1) / kChunkRows;
  return adaln_bwd_stats_bytes(batch, seq) +
         static_cast<size_t>(batch * chunks * (has_x ? 3 : 2) * dim) * sizeof(float);
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
  const int64_t chunks = (seq + kChunkRows - 1) / kChunkRows;
  float4* stats = static_cast<float4*>(workspace);
  float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + adaln_bwd_stats_bytes(batch, seq));
  AdalnStatsArgs sa{};
  sa.gh = static_cast<const uint16_t*>(gh);
  sa.z = static_cast<const uint16_t*>(z);
  sa.scale = static_cast<const uint16_t*>(scale);
  sa.stats = stats;
  sa.rows = batch * seq;
  sa.seq = seq;
  sa.dim = static_cast<int>(dim);
  sa.eps = eps;
  cudaError_t e = launch_adaln_bwd_stats(sa, st);
  if (e != cudaSuccess) return g.done(e);
  AdalnColsArgs a{};
  a.gh = sa.gh;
  a.gz = static_cast<const uint16_t*>(gz);
  a.z = sa.z;
  a.x = static_cast<const uint16_t*>(x);
  a.gate = static_cast<const uint16_t*>(gate);
  a.scale = sa.scale;
  a.stats = stats;
  a.dz = static_cast<uint16_t*>(dz);
  a.dx = static_cast<uint16_t*>(dx);
  a.part = part;
  a.seq = seq;
  a.chunks = chunks;
  a.dim = static_cast<int>(dim);
  if (has_x) e = gz ? launch_adaln_bwd_cols<true, true>(a, batch, st) : launch_adaln_bwd_cols<true, false>(a, batch, st);
  else e = gz ? launch_adaln_bwd_cols<false, true>(a, batch, st) : launch_adaln_bwd_cols<false, false>(a, batch, st);
  if (e != cudaSuccess) return g.done(e);
  FinalizeArgs f{};
  f.part = part;
  f.n = chunks;
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
// them the workspace (row statistics and parameter-gradient partials) lives
// in this file-scope array instead of a caller-provided one.  Every GPU that loads the library
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
// first call before any stream capture.  What it keeps there is fully
// overwritten by every call, so nothing needs clearing, but all calls share
// the one array: calls that overlap on the GPU (other streams, other threads)
// race.  Sizes whose workspace exceeds 16 MiB are rejected.
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
