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
// the rows of each batch entry are cut into chunks of kChunkRows = 28; in a
// chunk every column sums its 28 rows in increasing order from zero; the
// chunk sums combine by a stride tree over the chunk index (finalize.cu) and
// round to bf16.
//
// One persistent kernel does all the per-row work.  A CTA (one per SM) owns
// the chunks blockIdx.x, blockIdx.x + gridDim.x, ... and streams them through
// a ring of shared-memory stages, kStageRows = 2 rows of every input tensor
// (z, gh, and gz, x where present) per stage, filled by bulk copies (TMA
// engine) that complete on the stage's mbarrier, and the chunk's scale (and
// gate) rows in two modulation slots, whose copies complete on a barrier of
// their own per slot.  So every input byte crosses HBM once and is then read
// from shared memory by three warp roles:
//  - a producer warp issues the bulk copies of each stage once the column
//    warps have released its slot (an issuing thread can block for a
//    microsecond on a full copy queue, so no compute warp issues them);
//  - 4 row pairs (8 warps) in two groups taking alternate stages, one row
//    of the stage per pair: the row scalars mean,
//    rstd, c1, c2 as canonical sums (P = 32) over the shared-memory row, the
//    row split over the pair as in the forward kernel and kept in registers
//    for both rounds, into a per-stage slot; an mbarrier tells the column
//    warps they are there;
//  - 4 column warps, two 8-column vectors per thread: dz and dx from the row
//    scalars, stored straight from registers, and the chunk's parameter
//    sums in registers, written once per chunk as [B][chunks][NQ][D] fp32
//    partials; then each warp releases the stage to the producer.
// The partials are then reduced by the finalize kernel (launched behind this
// one with programmatic dependent launch).  Workspace: the partials only.
#include <map>
#include <mutex>

#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

// Rows per chunk, the unit of a CTA's work and of the parameter-gradient
// order.  28 rather than 32: a 4096-row sequence then makes 147 chunks and
// keeps 147 of the 148 SMs busy (32-row chunks: 128), and a CTA's share
// shrinks to 28 rows.  Measured: adaln_bwd 21.75 -> 20.06 us,
// residual_adaln_bwd 27.2 -> 25.0 us at config 4.
constexpr int kChunkRows = 28;
// Rows per ring stage.  Small stages keep more of the ring in flight: a
// slot is refilled only once both roles are done with it, and a bulk copy
// takes about 2 us to land under load, so 4-row stages left about one stage
// (64 KiB) per SM in flight; one-row stages cost more in per-stage
// bookkeeping than they gain (measured: 2 rows per stage is fastest, and 4,
// 6 or 8 stages of 2 rows time the same).
constexpr int kStageRows = 2;
constexpr int kStagesPerChunk = kChunkRows / kStageRows;
// Row pairs (8 warps), two groups of two taking the stages in turn.  With the
// 4 column warps and the producer warp that makes 13 warps, at most 4 per SM
// sub-partition, so each may hold 128 registers (5 warps on one sub-partition
// would leave 96 each).  The row scalars are the critical path (a pair's
// row takes about a microsecond of dependent sums), so the warps go to row
// pairs rather than column warps: measured with 2 pairs and 8 column warps
// of one vector each, adaln_bwd 23.2 us against 21.7, residual_adaln_bwd
// 27.3 against 27.0.
constexpr int kBwdPairs = 4;
static_assert(kBwdPairs % kStageRows == 0, "pairs per stage");
constexpr int kBwdRowGroups = kBwdPairs / kStageRows;  // pair groups, taking stages in turn
constexpr int kBwdRowWarps = 2 * kBwdPairs;
constexpr int kBwdColWarps = 4;
constexpr int kColVecs = 2;  // 8-column vectors per column thread: D <= 2048
// One more warp streams the stages in: a bulk copy can block the issuing
// thread for a microsecond when the copy engine's queue is full, so no
// compute warp issues them.
constexpr int kBwdProducerWarp = kBwdRowWarps + kBwdColWarps;
constexpr int kBwdThreads = (kBwdProducerWarp + 1) * 32;
// Stages: a multiple of kBwdRowGroups, so that every slot serves one pair
// group only (each group then waits on every phase of its slots in order),
// and at most kStagesPerChunk: the modulation slot of chunk k is refilled for
// chunk k + 2 when stage SPC(k + 2) is issued, after the column warps
// finished stage SPC(k + 2) - ns, which for ns <= SPC lies past chunk k.
constexpr int kBwdMaxStages = 6;
static_assert(kBwdMaxStages <= kStagesPerChunk && kBwdMaxStages % kBwdRowGroups == 0, "stage count");
constexpr int kBwdModSlots = 2;
// Per row pair: one exchange buffer of 2 sums x 2 warps x 4 fp32 pairs x 32
// lanes.  The two rounds of a row share it: in round 2 each warp writes the
// half it read in round 1 (pair_canonical_sum2x2 called with h ^ 1), so no
// warp overwrites data its partner has yet to read.
constexpr size_t kBwdXchF2 = 2 * 2 * 4 * 32;
constexpr size_t kBwdXchBytes = kBwdPairs * kBwdXchF2 * sizeof(f2_t);

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
  int64_t chunks;         // chunks per batch entry
  int64_t units;          // B * chunks
  int dim;
  float eps;
};

template <bool HAS_X>
__host__ __device__ constexpr int bwd_nq() { return HAS_X ? 3 : 2; }
template <bool HAS_X, bool HAS_GZ>
__host__ __device__ constexpr int bwd_tensors() { return 2 + (HAS_GZ ? 1 : 0) + (HAS_X ? 1 : 0); }

// Shared memory: ns stages of kStageRows rows of each input tensor; two
// modulation slots (the scale row, and the gate row with HAS_X, of a chunk's
// batch entry); the row scalars of each stage; the row pairs' exchange
// buffers; three mbarriers per stage (data full, scalars ready, stage
// empty) and one per modulation slot (rows landed).
__host__ __device__ constexpr size_t bwd_stage_bytes(int64_t dim, int nt) {
  return static_cast<size_t>(nt) * kStageRows * static_cast<size_t>(dim) * 2;
}
__host__ __device__ constexpr size_t bwd_slot_bytes(int64_t dim, bool has_x) {
  return static_cast<size_t>(dim) * 2 * (has_x ? 2 : 1);
}
__host__ __device__ constexpr size_t bwd_smem(int64_t dim, int nt, bool has_x, int ns) {
  return static_cast<size_t>(ns) * (bwd_stage_bytes(dim, nt) + kStageRows * sizeof(float4) + 3 * sizeof(uint64_t)) +
         kBwdModSlots * sizeof(uint64_t) +
         kBwdModSlots * bwd_slot_bytes(dim, has_x) + kBwdXchBytes;
}

// Walks a CTA's stages in order: stage j is stage i = j % SPC of the CTA's
// chunk k = j / SPC (SPC = kStagesPerChunk), the chunk unit blockIdx.x +
// k * gridDim.x, rows [s0, s0 + n) of batch entry b (n < kStageRows only at
// the end of a sequence, 0 for the unused stages of a short chunk); slot
// j % ns of the ring with phase parity (j / ns) & 1.  Incremental, so no
// 64-bit division per stage.
struct BwdCursor {
  int64_t unit, b, row0;
  int n, i, k, slot;
  uint32_t parity;
  __device__ void chunk_start(const AdalnBwdArgs& a) {
    unit = blockIdx.x + static_cast<int64_t>(k) * gridDim.x;
    b = unit / a.chunks;
    row0 = b * a.seq + (unit - b * a.chunks) * kChunkRows;
  }
  __device__ void rows(const AdalnBwdArgs& a) {
    const int64_t left = (b + 1) * a.seq - row0;
    n = left <= 0 ? 0 : left < kStageRows ? static_cast<int>(left) : kStageRows;
  }
  __device__ void init(const AdalnBwdArgs& a) {
    i = k = slot = 0;
    parity = 0;
    chunk_start(a);
    rows(a);
  }
  __device__ void next(const AdalnBwdArgs& a, int ns) {
    if (++slot == ns) {
      slot = 0;
      parity ^= 1u;
    }
    if (++i == kStagesPerChunk) {
      i = 0;
      ++k;
      chunk_start(a);
    } else {
      row0 += kStageRows;
    }
    rows(a);
  }
};

// EXACT: dim == 256 * NC (no masked vectors in the row pairs).  ns: stages.
template <int NC, bool EXACT, bool HAS_X, bool HAS_GZ>
__global__ void __launch_bounds__(kBwdThreads, 1)
adaln_bwd_kernel(const AdalnBwdArgs a, const int ns) {
  constexpr int NT = bwd_tensors<HAS_X, HAS_GZ>();
  constexpr int NQ = bwd_nq<HAS_X>();
  extern __shared__ __align__(128) uint8_t smem[];
  const int D = EXACT ? NC * 256 : a.dim;
  const uint32_t tensor_bytes = static_cast<uint32_t>(kStageRows * D * 2);  // one tensor of a stage
  const uint32_t stage_bytes = NT * tensor_bytes;
  const uint32_t slot_bytes = static_cast<uint32_t>(bwd_slot_bytes(D, HAS_X));
  uint8_t* mods = smem + static_cast<size_t>(ns) * stage_bytes;                    // [2][scale | gate]
  float4* scal = reinterpret_cast<float4*>(mods + kBwdModSlots * slot_bytes);      // [ns][rows]
  f2_t* xch_all = reinterpret_cast<f2_t*>(scal + ns * kStageRows);
  uint64_t* full = reinterpret_cast<uint64_t*>(xch_all + kBwdPairs * kBwdXchF2);
  uint64_t* ready = full + ns;
  uint64_t* empty = ready + ns;
  // The modulation rows of chunk k land in slot k & 1 on mfull[k & 1], whose
  // phase for chunk k has parity (k >> 1) & 1.  Both row-pair groups wait on
  // it once per chunk before reading the slot: the rows are issued with the
  // chunk's first stage, which one group does not take (the groups take
  // alternate stages), so that stage's barrier cannot carry them.  The
  // column warps are ordered after it through the first stage's ready.
  uint64_t* mfull = empty + ns;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t my_units =
      a.units > static_cast<int64_t>(blockIdx.x) ? (a.units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t nstages = my_units * kStagesPerChunk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&ready[s]), 2 * kStageRows);  // the warps of one pair group
      mbar_init(smem_addr(&empty[s]), kBwdColWarps);
    }
    for (int m = 0; m < kBwdModSlots; ++m) mbar_init(smem_addr(&mfull[m]), 1);
    fence_mbar_init();
  }
  __syncthreads();
  // While the previous kernel on the stream finishes, pull this CTA's first
  // stage and its chunk's modulation rows into L2 (prefetch_l2).  Measured:
  // the config-4 backward step 5% faster, isolated launches 2 us faster.
  if (warp == kBwdProducerWarp && lane == 0 && nstages > 0) {
    BwdCursor c0;
    c0.init(a);
    const uint32_t bytes = static_cast<uint32_t>(c0.n * D * 2);
    const int64_t off = c0.row0 * D;
    if (bytes > 0) {
      prefetch_l2(a.z + off, bytes);
      prefetch_l2(a.gh + off, bytes);
      if (HAS_GZ) prefetch_l2(a.gz + off, bytes);
      if (HAS_X) prefetch_l2(a.x + off, bytes);
    }
    prefetch_l2(a.scale + c0.b * D, static_cast<uint32_t>(D * 2));
    if (HAS_X) prefetch_l2(a.gate + c0.b * D, static_cast<uint32_t>(D * 2));
  }
  pdl_wait();
  pdl_trigger();

  BwdCursor cur;
  cur.init(a);
  if (warp < kBwdRowWarps) {
    // ---------------- row pairs: the row scalars -----------------------------
    // Pair p takes row p % kStageRows of the stages j with
    // j % kBwdRowGroups == p / kStageRows.  As the forward kernel: with
    // NC = D/256 vectors of 8 elements per lane, warp h of the pair holds the
    // vectors v = lane + 32 * c for c = 2i + h, and the last level of the
    // canonical vector tree crosses the pair through shared memory
    // (pair_canonical_sum2x2).
    constexpr bool SPLIT = NC >= 2;
    constexpr int NH = SPLIT ? NC / 2 : 1;
    const int pair = warp >> 1;
    const int h = warp & 1;
    const int prow = pair % kStageRows;
    const int group = pair / kStageRows;
    const int bar_id = 2 + pair;
    f2_t* xch = xch_all + pair * kBwdXchF2;
    auto col = [&](int i) { return (lane + 32 * (SPLIT ? 2 * i + h : i)) * 8; };
    auto ok = [&](int i) { return EXACT || col(i) < D; };
    auto div_d = [&](float v) {
      return EXACT ? __fmul_rn(v, 1.0f / (NC * 256)) : __fdiv_rn(v, static_cast<float>(D));
    };
    bool dead = false;
    int mchunk = -1;  // the chunk whose modulation rows this warp has waited for
    for (int64_t j = 0; j < nstages; ++j, cur.next(a, ns)) {
      if (static_cast<int>(j % kBwdRowGroups) != group) continue;
      const int s = cur.slot;
      if (!dead && !mbar_wait(smem_addr(&full[s]), cur.parity)) dead = true;
      if (!dead && cur.k != mchunk) {
        if (!mbar_wait(smem_addr(&mfull[cur.k & 1]), static_cast<uint32_t>((cur.k >> 1) & 1))) dead = true;
        mchunk = cur.k;
      }
      if (dead) continue;  // no arrival: the column warps' bounded waits give up too
      if (prow < cur.n) {
        const uint8_t* zr = smem + static_cast<size_t>(s) * stage_bytes + static_cast<size_t>(prow) * D * 2;
        const uint8_t* gr = zr + tensor_bytes;
        const uint8_t* sc = mods + (cur.k & 1) * slot_bytes;
        f2_t zf[NH][4], dxh[NH][4];
#pragma unroll
        for (int i = 0; i < NH; ++i) {
          const uint4 zv = ok(i) ? lds16(zr + col(i) * 2) : make_uint4(0, 0, 0, 0);
          const uint4 gv = ok(i) ? lds16(gr + col(i) * 2) : make_uint4(0, 0, 0, 0);
          const uint4 sv = ok(i) ? lds16(sc + col(i) * 2) : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            zf[i][jj] = bf2f2(word(zv, jj));
            dxh[i][jj] = bf16x2_mul(word(gv, jj), word(sv, jj));  // gh * scale, exact
          }
        }
        // Round 1: sum(z) and sum(dxh).
        float mean, c1;
        pair_canonical_sum2x2<NH, SPLIT>([&](int n, int i, int jj) { return n == 0 ? zf[i][jj] : dxh[i][jj]; },
                                         xch, h, lane, bar_id, mean, c1);
        mean = div_d(mean);
        c1 = div_d(c1);
        // Round 2: sum(d * d) and sum(dxh * d), d = z - mean (zero where masked).
        const f2_t mm = f2(mean, mean);
#pragma unroll
        for (int i = 0; i < NH; ++i) {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) zf[i][jj] = ok(i) ? sub2(zf[i][jj], mm) : 0ull;
        }
        float var, e;
        pair_canonical_sum2x2<NH, SPLIT>(
            [&](int n, int i, int jj) { return mul2_noc(n == 0 ? zf[i][jj] : dxh[i][jj], zf[i][jj]); },
            xch, h ^ 1, lane, bar_id, var, e);
        const float rstd = canonical_rstd(div_d(var), a.eps);
        const float c2 = div_d(__fmul_rn(e, rstd));
        if (h == 0 && lane == 0) scal[s * kStageRows + prow] = make_float4(mean, rstd, c1, c2);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&ready[s]));
    }
    return;
  }

  if (warp == kBwdProducerWarp) {
    // ---------------- producer: stream the stages into the ring ------------
    // Stage j goes into slot j % ns once the column warps have released the
    // stage that held it before (j - ns); a chunk's modulation rows go
    // with its first stage, on their own barrier (mfull).
    if (lane != 0) return;
    bool dead = false;
    int mod_k = -1;  // the last chunk whose modulation rows were issued
    int64_t j = 0;
    for (; j < nstages; ++j, cur.next(a, ns)) {
      const uint32_t bar = smem_addr(&full[cur.slot]);
      if (j >= ns) {
        if (!mbar_wait(smem_addr(&empty[cur.slot]), cur.parity ^ 1u)) {
          dead = true;
          break;
        }
        fence_proxy_async_smem();
      }
      if (cur.n == 0) {  // nothing to copy: complete the phase with a plain arrival
        mbar_arrive(bar);
        continue;
      }
      const uint32_t bytes = static_cast<uint32_t>(cur.n * D * 2);
      const uint32_t row_bytes = static_cast<uint32_t>(D * 2);
      const uint32_t dst = smem_addr(smem + static_cast<size_t>(cur.slot) * stage_bytes);
      const int64_t off = cur.row0 * D;
      if (cur.i == 0) {  // a chunk's first stage: its modulation rows, on their own barrier
        const uint32_t mb = smem_addr(&mfull[cur.k & 1]);
        const uint32_t slot = smem_addr(mods + (cur.k & 1) * slot_bytes);
        mbar_arrive_expect_tx(mb, (HAS_X ? 2u : 1u) * row_bytes);
        bulk_g2s(slot, a.scale + cur.b * D, row_bytes, mb);
        if (HAS_X) bulk_g2s(slot + row_bytes, a.gate + cur.b * D, row_bytes, mb);
        mod_k = cur.k;
      }
      mbar_arrive_expect_tx(bar, NT * bytes);
      bulk_g2s(dst, a.z + off, bytes, bar);
      bulk_g2s(dst + tensor_bytes, a.gh + off, bytes, bar);
      if (HAS_GZ) bulk_g2s(dst + 2 * tensor_bytes, a.gz + off, bytes, bar);
      if (HAS_X) bulk_g2s(dst + (HAS_GZ ? 3 : 2) * tensor_bytes, a.x + off, bytes, bar);
    }
    if (dead) {  // drain the copies issued before the failed wait (bounded waits)
      for (int64_t k = j - ns; k < j; ++k)
        if (k >= 0) mbar_wait(smem_addr(&full[k % ns]), static_cast<uint32_t>((k / ns) & 1));
      for (int k = mod_k - 1; k <= mod_k; ++k)
        if (k >= 0) mbar_wait(smem_addr(&mfull[k & 1]), static_cast<uint32_t>((k >> 1) & 1));
    }
    return;
  }

  // ---------------- column warps: dz, dx and the chunk sums ---------------
  const int t = threadIdx.x - kBwdRowWarps * 32;
  auto colv = [&](int v) { return (t + v * kBwdColWarps * 32) * 8; };
  bool dead = false;
  f2_t acc[kColVecs][NQ][4];
  // The modulation rows: held in registers for a chunk, or (HAS_X, where
  // the registers are short) re-read from the shared-memory slot per row.
  constexpr bool kModRegs = !HAS_X;
  f2_t sc[kColVecs][4], gt[kColVecs][4];
  for (int64_t j = 0; j < nstages; ++j, cur.next(a, ns)) {
    const int s = cur.slot;
    if (!dead && !(mbar_wait(smem_addr(&full[s]), cur.parity) && mbar_wait(smem_addr(&ready[s]), cur.parity)))
      dead = true;
    // The chunk's modulation rows need no wait of their own here: the first
    // stage's row pair group waits for them (mfull) before its arrival on
    // ready, which this warp has just waited for.
    if (cur.i == 0) {
#pragma unroll
      for (int v = 0; v < kColVecs; ++v) {
#pragma unroll
        for (int q = 0; q < NQ; ++q)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) acc[v][q][jj] = 0ull;
        if (kModRegs && colv(v) < D && !dead) {
          const uint8_t* slot = mods + (cur.k & 1) * slot_bytes + colv(v) * 2;
          const uint4 w = lds16(slot);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) sc[v][jj] = bf2f2(word(w, jj));
          if (HAS_X) {
            const uint4 g = lds16(slot + D * 2);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) gt[v][jj] = bf2f2(word(g, jj));
          }
        }
      }
    }
    if (!dead) {
      auto do_row = [&](int r) {
        const float4 k = scal[s * kStageRows + r];  // mean, rstd, c1, c2
        const f2_t mm = f2(k.x, k.x), rr = f2(k.y, k.y), cc1 = f2(k.z, k.z), cc2 = f2(k.w, k.w);
        const uint8_t* row = smem + static_cast<size_t>(s) * stage_bytes + static_cast<size_t>(r) * D * 2;
        const int64_t o0 = (cur.row0 + r) * D;
#pragma unroll
        for (int v = 0; v < kColVecs; ++v) {
          const int col = colv(v);
          if (col >= D) continue;
          const uint4 zv = lds16(row + col * 2);
          const uint4 gv = lds16(row + tensor_bytes + col * 2);
          uint4 gzv = make_uint4(0, 0, 0, 0), xv = make_uint4(0, 0, 0, 0);
          if (HAS_GZ) gzv = lds16(row + 2 * tensor_bytes + col * 2);
          if (HAS_X) xv = lds16(row + (HAS_GZ ? 3 : 2) * tensor_bytes + col * 2);
          f2_t scv[4], gtv[4];
          if (kModRegs) {
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              scv[jj] = sc[v][jj];
              gtv[jj] = gt[v][jj];
            }
          } else {
            const uint8_t* slot = mods + (cur.k & 1) * slot_bytes + col * 2;
            const uint4 w = lds16(slot);
            const uint4 g = HAS_X ? lds16(slot + D * 2) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              scv[jj] = bf2f2(word(w, jj));
              gtv[jj] = bf2f2(word(g, jj));
            }
          }
          uint4 dzo, dxo;
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const f2_t g = bf2f2(word(gv, jj));
            const f2_t xhat = mul2(bf16x2_sub_f2(word(zv, jj), mm), rr);
            const f2_t dxh = mul2_noc(g, scv[jj]);
            const f2_t tt = sub2(sub2(dxh, cc1), mul2_noc(xhat, cc2));
            f2_t dz;
            if (HAS_GZ) {
              dz = bf16x2_add_f2(word(gzv, jj), mul2_noc(rr, tt));
            } else {
              dz = mul2(rr, tt);  // feeds multiplies only
            }
            word_ref(dzo, jj) = f2bf2(dz);
            acc[v][0][jj] = add2(acc[v][0][jj], g);
            acc[v][1][jj] = add2(acc[v][1][jj], mul2_noc(g, xhat));
            if (HAS_X) {
              word_ref(dxo, jj) = f2bf2(mul2(dz, gtv[jj]));
              acc[v][2][jj] = add2(acc[v][2][jj], mul2_noc(dz, bf2f2(word(xv, jj))));
            }
          }
          st16(a.dz + o0 + col, dzo);
          if (HAS_X) st16(a.dx + o0 + col, dxo);
        }
      };
      if (cur.n == kStageRows) {  // a full stage: every row, unguarded
#pragma unroll
        for (int r = 0; r < kStageRows; ++r) do_row(r);
      } else {
        for (int r = 0; r < cur.n; ++r) do_row(r);
      }
    }
    // The warp is done with the stage (and, through the ready barrier, so
    // are the row warps): release it to the producer.
    __syncwarp();
    if (lane == 0 && !dead) mbar_arrive(smem_addr(&empty[s]));
    if (cur.i == kStagesPerChunk - 1 && !dead) {
#pragma unroll
      for (int v = 0; v < kColVecs; ++v) {
        if (colv(v) >= D) continue;
        float* out = a.part + cur.unit * NQ * D + colv(v);
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
          float4* o4 = reinterpret_cast<float4*>(out + q * D);
          o4[0] = make_float4(f2lo(acc[v][q][0]), f2hi(acc[v][q][0]), f2lo(acc[v][q][1]), f2hi(acc[v][q][1]));
          o4[1] = make_float4(f2lo(acc[v][q][2]), f2hi(acc[v][q][2]), f2lo(acc[v][q][3]), f2hi(acc[v][q][3]));
        }
      }
    }
  }
}

// Stages that fit the shared memory (at most kBwdMaxStages).
static int bwd_stages(int64_t dim, int nt, bool has_x, size_t limit) {
  int n = kBwdMaxStages;
  while (n > 0 && bwd_smem(dim, nt, has_x, n) > limit) n -= kBwdRowGroups;
  return n;
}

template <bool HAS_X, bool HAS_GZ>
static cudaError_t launch_adaln_bwd(const AdalnBwdArgs& a, cudaStream_t st) {
  const DeviceInfo& dev = device_info();
  if (dev.error != cudaSuccess) return dev.error;
  constexpr int NT = bwd_tensors<HAS_X, HAS_GZ>();
  const int ns = bwd_stages(a.dim, NT, HAS_X, dev.max_smem_optin);
  if (ns < 2 * kBwdRowGroups) return cudaErrorInvalidValue;
  const size_t smem = bwd_smem(a.dim, NT, HAS_X, ns);
  const int nc = row_chunks(a.dim);
  const bool exact = a.dim == 256 * nc;
  const dim3 grid(static_cast<unsigned>(a.units < dev.sms ? a.units : dev.sms));
  auto go = [&](auto kern) -> cudaError_t {
    // The same shared-memory carveout as the finalize kernel behind it.
    cudaError_t e = ensure_smem(kern, smem, true);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, grid, dim3(kBwdThreads), smem, st, a, ns);
  };
#define AFB_LAUNCH_BWD(NC)                                                \
  return exact ? go(adaln_bwd_kernel<NC, true, HAS_X, HAS_GZ>) \
               : go(adaln_bwd_kernel<NC, false, HAS_X, HAS_GZ>)
  switch (nc) {
    case 1: AFB_LAUNCH_BWD(1);
    case 2: AFB_LAUNCH_BWD(2);
    case 4: AFB_LAUNCH_BWD(4);
    case 8: AFB_LAUNCH_BWD(8);
    default: return cudaErrorInvalidValue;
  }
#undef AFB_LAUNCH_BWD
}

cudaError_t read_status_adaln_bwd(int* status, bool clear) { return tu_status(status, clear); }

// Workspace bytes (the [B][chunks][NQ][D] fp32 partials), or false when the
// product does not fit in size_t (absurd sizes are rejected, not wrapped).
static bool adaln_bwd_workspace_checked(int64_t batch, int64_t seq, int64_t dim, bool has_x, size_t* out) {
  if (batch < 0 || seq < 1 || dim < 1) {
    *out = 0;
    return true;
  }
  const unsigned __int128 chunks = static_cast<unsigned __int128>((seq + kChunkRows - 1) / kChunkRows);
  const unsigned __int128 bytes = static_cast<unsigned __int128>(batch) * chunks * (has_x ? 3 : 2) *
                                  static_cast<unsigned __int128>(dim) * sizeof(float);
  if (bytes > static_cast<unsigned __int128>(SIZE_MAX)) return false;
  *out = static_cast<size_t>(bytes);
  return true;
}

size_t adaln_bwd_workspace(int64_t batch, int64_t seq, int64_t dim, bool has_x) {
  size_t n = 0;
  return adaln_bwd_workspace_checked(batch, seq, dim, has_x, &n) ? n : SIZE_MAX;
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
  float* part = static_cast<float*>(workspace);
  AdalnBwdArgs a{};
  a.gh = static_cast<const uint16_t*>(gh);
  a.gz = static_cast<const uint16_t*>(gz);
  a.z = static_cast<const uint16_t*>(z);
  a.x = static_cast<const uint16_t*>(x);
  a.gate = static_cast<const uint16_t*>(gate);
  a.scale = static_cast<const uint16_t*>(scale);
  a.dz = static_cast<uint16_t*>(dz);
  a.dx = static_cast<uint16_t*>(dx);
  a.part = part;
  a.seq = seq;
  a.chunks = chunks;
  a.units = batch * chunks;
  a.dim = static_cast<int>(dim);
  a.eps = eps;
  cudaError_t e;
  if (has_x) e = gz ? launch_adaln_bwd<true, true>(a, st) : launch_adaln_bwd<true, false>(a, st);
  else e = launch_adaln_bwd<false, false>(a, st);
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
// them the workspace (the parameter-gradient partials) lives in this
// file-scope array instead of a caller-provided one.  Every GPU that loads the library
// holds these 16 MiB until the process exits.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of the scratch array for the current device.  The name of
// the array is only a host-side stand-in; the address is looked up once per
// device (with that device current) and cached, so cudaDeviceReset is not
// supported while the library is loaded.
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
  size_t need = 0;
  const bool fits = adaln_bwd_workspace_checked(batch, seq, dim, true, &need);
  if (!fits || need > kNoAllocScratchBytes) {
    set_error(std::string(name) + ": this size needs " +
              (fits ? std::to_string(need) : std::string("more than SIZE_MAX")) +
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
