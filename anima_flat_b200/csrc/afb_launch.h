// Host-side helpers shared by the C-ABI entry points: argument validation,
// the per-thread error message, and kernel launch with programmatic
// dependent launch (PDL).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <initializer_list>
#include <string>
#include <utility>

namespace afb {

// Warps (rows) per CTA of the warp-per-row kernels.
constexpr int kRowWarps = 4;
// Largest row width the warp-per-row kernels hold in registers.
constexpr int64_t kMaxRowDim = 4096;

// Properties of the current device, read once per device.
struct DeviceInfo {
  int sms = 0;
  size_t max_smem_optin = 0;  // dynamic shared memory a CTA may opt into
  cudaError_t error = cudaSuccess;
};
const DeviceInfo& device_info();

// Opt a kernel into `bytes` of dynamic shared memory (cached per kernel).
// max_shared: also prefer the largest shared-memory carveout, for kernels
// that rely on several CTAs' rings sharing an SM (without it the driver may
// keep a large L1 and fit one CTA per SM).
cudaError_t ensure_smem_raw(const void* kernel, size_t bytes, bool max_shared);
template <typename K>
cudaError_t ensure_smem(K kernel, size_t bytes, bool max_shared = false) {
  return ensure_smem_raw(reinterpret_cast<const void*>(kernel), bytes, max_shared);
}

// Set by afb_set_pdl(); defaults to on unless AFB_PDL=0 is in the environment.
bool pdl_enabled();

// Host readers of the per-file device status words (OR-ed by
// afb_device_status; `clear` zeroes a word after reading it).
cudaError_t read_status_adaln_fwd(int* status, bool clear);
cudaError_t read_status_headnorm_fwd(int* status, bool clear);
cudaError_t read_status_headnorm_bwd(int* status, bool clear);
cudaError_t read_status_adaln_bwd(int* status, bool clear);
cudaError_t read_status_rms(int* status, bool clear);
cudaError_t read_status_probe(int* status, bool clear);

// Column sums of chunk partials part[batch][n][ncols] (fp32) by a stride tree
// over the chunk index (finalize.cu); column c goes to out[c / seg][b*seg +
// c % seg], rounded to bf16 (RNE) or kept fp32.
struct FinalizeArgs {
  const float* part;
  int64_t n;
  int ncols;
  int seg;
  void* out[3];
  int bf16_out;
  int np;               // set by the launcher
  int64_t bstride;      // set by the launcher: floats between batch entries of part
  int64_t nflat;        // set by the launcher: valid floats of a batch entry of part
  int64_t out_bstride;  // set by the launcher: elements between batch entries of out
};
bool finalize_fits(int64_t n);
cudaError_t launch_colsum_finalize(const FinalizeArgs& f, int64_t batch, cudaStream_t st);

// Records `msg` as this thread's last error (read by afb_last_error()).
void set_error(const std::string& msg);
const std::string& last_error();

// 16-byte vectors per warp lane for a row of `dim` elements: the canonical
// tree pads the row to max(32, pow2ceil(dim / 8)) vectors.
inline int row_chunks(int64_t dim) {
  int64_t nv = (dim + 7) / 8;
  int64_t p = 32;
  while (p < nv) p <<= 1;
  return static_cast<int>(p / 32);
}

// Validation failures carry cudaErrorInvalidValue.  The guard names the entry
// point in every message.
class ApiGuard {
 public:
  explicit ApiGuard(const char* name) : name_(name) {}
  int fail() const {
    set_error(std::string(name_) + ": " + last_error());
    return static_cast<int>(cudaErrorInvalidValue);
  }
  int done(cudaError_t e) const {
    if (e != cudaSuccess) {
      set_error(std::string(name_) + ": " + cudaGetErrorName(e) + ": " + cudaGetErrorString(e));
    }
    return static_cast<int>(e);
  }
  const char* name() const { return name_; }

 private:
  const char* name_;
};

inline bool check(bool ok, const std::string& msg) {
  if (!ok) set_error(msg);
  return ok;
}

// Row-kernel shape check: batch >= 0, seq >= 1, dim a multiple of 8 up to
// kMaxRowDim.
inline bool check_rows(int64_t batch, int64_t seq, int64_t dim) {
  return check(batch >= 0, "batch must be >= 0") && check(seq >= 1, "seq must be >= 1") &&
         check(dim >= 8 && dim % 8 == 0 && dim <= kMaxRowDim,
               "dim must be a multiple of 8 in [8, " + std::to_string(kMaxRowDim) + "], got " +
                   std::to_string(dim));
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Non-null, 16-byte aligned device pointers.
inline bool check_ptrs(std::initializer_list<const void*> ps, std::initializer_list<const char*> names) {
  auto n = names.begin();
  for (const void* p : ps) {
    const char* nm = (n != names.end()) ? *n++ : "pointer";
    if (!check(p != nullptr, std::string(nm) + " is null")) return false;
    if (!check(aligned(p, 16), std::string(nm) + " is not 16-byte aligned")) return false;
  }
  return true;
}
inline bool check_ptr8(const void* p, const char* nm) {
  return check(p != nullptr, std::string(nm) + " is null") &&
         check(aligned(p, 8), std::string(nm) + " is not 8-byte aligned");
}
inline bool check_ptr4(const void* p, const char* nm) {
  return check(p != nullptr, std::string(nm) + " is null") &&
         check(aligned(p, 4), std::string(nm) + " is not 4-byte aligned");
}

// Launch on `st`, with the programmatic-stream-serialization attribute when
// PDL is on.  Every kernel of this library begins with griddepcontrol.wait,
// so it never reads its predecessor's output early.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args&&... args) {
  if (grid.x == 0 || grid.y == 0 || grid.z == 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace afb
