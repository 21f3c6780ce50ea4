// extern "C" entry points of liblocalcorr_b200.so (declared in
// include/localcorr_b200.h): argument validation, engine selection and
// error reporting around the kernels.
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

#include "lc_common.cuh"

namespace lcb200 {

// Engines (defined in corr_simt.cu, corr_tc.cu, layout.cu, spatial.cu).
// (H1, W1) is the pixel grid of fmap1/coords/corr, (H2, W2) the level-0 size
// of the map fmap2_packed was built from.
bool simt_forward(const void*, const void*, const void*, void*, int B, int H1, int W1, int H2,
                  int W2, int C, int r, int levels, int dil, int dtype, int cdtype, bool ymajor,
                  float scale, cudaStream_t);
bool simt_backward(const void*, const void*, const void*, const void*, void*, float*, int B,
                   int H1, int W1, int H2, int W2, int C, int r, int levels, int dil, int dtype,
                   int cdtype, bool ymajor, float scale, bool acc1, bool add_f2, cudaStream_t);
bool tc_det_pull_ok(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
                    int dilation, std::string* why);
size_t tc_det_pull_bytes(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels);
bool tc_det_f2_pull(const void* f1, const void* co, const void* gout, float* f2g, int B, int H1,
                    int W1, int H2, int W2, int C, int radius, int levels, int dtype, int cdtype,
                    bool ymajor, float scale, void* ws, size_t ws_bytes, cudaStream_t s);
bool tc_eligible(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
                 int dilation, int dtype, std::string* why);
size_t tc_workspace_bytes(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
                          bool backward);
bool tc_forward(const void*, const void*, const void*, void*, int B, int H1, int W1, int H2,
                int W2, int C, int radius, int levels, int cdtype, bool ymajor, float scale,
                void* sort_ws, void*, size_t, cudaStream_t);
bool tc_backward(const void*, const void*, const void*, const void*, void*, float*, int B,
                 int H1, int W1, int H2, int W2, int C, int radius, int levels, int cdtype,
                 bool ymajor, float scale, bool acc_f1, void* sort_ws, void*, size_t,
                 cudaStream_t);
size_t tc_sort_state_bytes(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels);
bool tc_backward_fmap1(const void* f1, const void* f2, const void* co, const void* gout,
                       void* f1g, int B, int H1, int W1, int H2, int W2, int C, int radius,
                       int levels, int cdtype, bool ymajor, float scale, bool acc_f1,
                       void* sort_ws, void* ws, size_t ws_bytes, void* records,
                       size_t records_bytes, cudaStream_t s);
size_t tc_records_bytes(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels);
bool tc_pull_lookups(const void* const* sort_states, const void* const* records, int n,
                     float* f2g, int B, int H1, int W1, int H2, int W2, int C, int radius,
                     int levels, float scale, void* ws, size_t ws_bytes, cudaStream_t s);
bool tc_bwd_eligible(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
                     int dilation, int dtype, std::string* why);
int tc_device_status(bool reset);
bool layout_nchw_to_nhwc(const void*, void*, int, int, int, int, cudaStream_t);
bool layout_nhwc_to_nchw(const void*, void*, int, int, int, int, cudaStream_t);
bool layout_pyramid_build(const void*, void*, int, int, int, int, int, int, cudaStream_t);
bool layout_pyramid_build_grad(const void*, bool, void*, int, int, int, int, int, int,
                               cudaStream_t);
bool spatial_forward(const void*, const void*, void*, int, int, int, int, int, int, int, float,
                     cudaStream_t);
bool spatial_backward(const void*, const void*, const void*, void*, void*, int, int, int, int,
                      int, int, int, float, cudaStream_t);

namespace {
thread_local std::string g_last_error;
// every host thread's launches (autograd runs backward passes on its own
// worker threads)
std::atomic<long long> g_launches{0};
std::atomic<int> g_deterministic{0};
}  // namespace

// NVTX range around an entry point's host work and launches (shows up in
// Nsight Systems / ncu --nvtx; free when no tool is attached).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

bool deterministic_mode() { return g_deterministic.load(std::memory_order_relaxed) != 0; }

bool bounds_read_tc(unsigned long long out[3], bool reset);
bool bounds_read_simt(unsigned long long out[3], bool reset);
bool bounds_read_spatial(unsigned long long out[3], bool reset);

#ifdef LC_BOUNDS_CHECK
namespace {
std::atomic<long long> g_bounds_total{0};
const char* const kSiteNames[kSiteCount] = {
    "none",
    "tc_hist (sort bin)",
    "tc_scatter (sorted position)",
    "tc_rank_fix (bin member)",
    "tc_gather_rows (fmap1 row)",
    "tc_fwd (chunk range)",
    "tc_fwd (member pixel)",
    "tc_unsort (sorted position)",
    "tc_gint (sorted position)",
    "tc_bwd1 (pixel)",
    "tc_bwd2 (candidate position)",
    "simt forward (fmap2 element)",
    "simt backward (fmap2 element)",
    "spatial (in2 element)",
};
}  // namespace
#endif

bool bounds_finish(bool ok, cudaStream_t s) {
#ifdef LC_BOUNDS_CHECK
  if (!ok) return false;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) return check_launch("bounds check");
  if (cs != cudaStreamCaptureStatusNone) return true;  // nothing has run yet
  if (cudaStreamSynchronize(s) != cudaSuccess) return check_launch("bounds check");
  unsigned long long total = 0, site = 0, idx = 0;
  for (auto rd : {bounds_read_tc, bounds_read_simt, bounds_read_spatial}) {
    unsigned long long r[3];
    if (!rd(r, true)) return check_launch("bounds check: reading the device record");
    if (r[0] && !total) { site = r[1]; idx = r[2]; }
    total += r[0];
  }
  if (!total) return true;
  g_bounds_total.fetch_add((long long)total);
  set_error("bounds check: " + std::to_string(total) + " out-of-range index(es), first at " +
            (site < (unsigned long long)kSiteCount ? kSiteNames[site] : "?") + ", index " +
            std::to_string((long long)idx));
  return false;
#else
  (void)s;
  return ok;
#endif
}

long long bounds_total(bool reset) {
#ifdef LC_BOUNDS_CHECK
  return reset ? g_bounds_total.exchange(0) : g_bounds_total.load();
#else
  (void)reset;
  return -1;
#endif
}

void set_error(const std::string& msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return true;
  set_error(std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
  return false;
}

int max_dyn_smem() {
  int dev = 0;
  cudaGetDevice(&dev);
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    v = 48 * 1024;
  return v;
}

bool ensure_smem_attr(const void* func, size_t bytes) {
  if (bytes <= 48 * 1024) return true;
  // (kernel, device) -> largest size already granted. Small fixed table: the
  // library has a bounded number of kernels that opt in.
  struct Entry { const void* f; int dev; size_t bytes; };
  static Entry table[256];
  static int n = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n; ++i)
    if (table[i].f == func && table[i].dev == dev && table[i].bytes >= bytes) return true;
  const cudaError_t e =
      cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) {
    set_error(std::string("cudaFuncSetAttribute(MaxDynamicSharedMemorySize=") +
              std::to_string(bytes) + "): " + cudaGetErrorString(e));
    return false;
  }
  for (int i = 0; i < n; ++i)
    if (table[i].f == func && table[i].dev == dev) { table[i].bytes = bytes; return true; }
  if (n < 256) table[n++] = Entry{func, dev, bytes};
  return true;
}

namespace {

// Validation shared by all pyramid launchers, mirroring the reference
// launchers (cuda_pyramid/localcorr_cuda_pyramid_kernel.cu:1420-1435) plus the
// checks the reference leaves implicit (non-negative radius, positive C,
// 32-bit index ranges).
bool validate_pyramid(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
                      int dilation, int dtype, bool* empty) {
  *empty = false;
  if ((long long)H1 * W1 <= 0 || B <= 0) { *empty = true; return true; }
  if (levels < 1 || levels > kMaxLevels) {
    set_error("levels must be in [1, 8] (got " + std::to_string(levels) + ")");
    return false;
  }
  if (dilation < 1) {
    set_error("dilation must be >= 1 (got " + std::to_string(dilation) + ")");
    return false;
  }
  if (radius < 0) {
    set_error("radius must be >= 0 (got " + std::to_string(radius) + ")");
    return false;
  }
  if (C <= 0) {
    set_error("C must be positive (got " + std::to_string(C) + ")");
    return false;
  }
  if (dtype != LCB200_F32 && dtype != LCB200_F16) {
    set_error("dtype must be LCB200_F32 (0) or LCB200_F16 (1)");
    return false;
  }
  for (int l = 0; l < levels; ++l) {
    if ((H2 >> l) < 1 || (W2 >> l) < 1) {
      set_error("level " + std::to_string(l) + " of a " + std::to_string(H2) + "x" +
                std::to_string(W2) + " map is empty");
      return false;
    }
  }
  if ((long long)H1 * W1 > (1ll << 30) || (long long)H2 * W2 > (1ll << 30)) {
    set_error("H1*W1 or H2*W2 too large");
    return false;
  }
  return true;
}

// Library-owned scratch for the reference-compatible launchers, which take no
// workspace argument. One buffer per device, shared by every stream:
//  * a call on stream s first makes s wait for the event recorded after the
//    previous call's kernels (on whatever stream they ran), so two calls
//    never use the buffer at the same time and a buffer is only freed after
//    its last user has finished;
//  * growing it frees the old buffer (cudaFreeAsync) and allocates the new
//    one (cudaMallocAsync) on s, after that wait;
//  * the lease holds the lock from the wait until the event is recorded
//    behind the call's kernels, so host threads cannot interleave.
struct DeviceScratch {
  void* ptr = nullptr;
  size_t bytes = 0;
  cudaEvent_t done = nullptr;  // recorded after the last call that used ptr
  cudaStream_t last = nullptr;
  bool used = false;
};
std::mutex g_scratch_mu;
DeviceScratch g_scratch[64];

class ScratchLease {
 public:
  ScratchLease(size_t bytes, cudaStream_t s) : lock_(g_scratch_mu), s_(s) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
      cudaGetLastError();
      set_error("no current CUDA device for the library scratch");
      return;
    }
    d_ = &g_scratch[dev];
    if (!d_->done && cudaEventCreateWithFlags(&d_->done, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      d_->done = nullptr;
      set_error("could not create the library scratch event");
      d_ = nullptr;
      return;
    }
    if (d_->used && d_->last != s &&
        cudaStreamWaitEvent(s, d_->done, 0) != cudaSuccess) {
      check_launch("wait for the previous user of the library scratch");
      d_ = nullptr;
      return;
    }
    if (bytes > d_->bytes) {
      if (d_->ptr) cudaFreeAsync(d_->ptr, s);
      d_->ptr = nullptr;
      d_->bytes = 0;
      void* p = nullptr;
      if (cudaMallocAsync(&p, bytes, s) != cudaSuccess) {
        cudaGetLastError();
        set_error("could not allocate " + std::to_string(bytes) + " B of scratch");
        d_ = nullptr;
        return;
      }
      d_->ptr = p;
      d_->bytes = bytes;
    }
    ptr_ = d_->ptr;
  }
  // Record the event behind everything this call enqueued on s.
  ~ScratchLease() {
    if (!d_) return;
    if (cudaEventRecord(d_->done, s_) == cudaSuccess) {
      d_->used = true;
      d_->last = s_;
    } else {
      cudaGetLastError();
    }
  }
  void* ptr() const { return ptr_; }
  bool ok() const { return d_ != nullptr; }

 private:
  std::lock_guard<std::mutex> lock_;
  cudaStream_t s_;
  DeviceScratch* d_ = nullptr;
  void* ptr_ = nullptr;
};

bool use_tc(int engine, int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
            int dilation,
            int dtype, bool* ok, bool backward = false, const void* p1 = nullptr,
            const void* p2 = nullptr) {
  *ok = true;
  if (engine == LCB200_ENGINE_SIMT) return false;
  std::string why;
  bool elig = backward
                  ? tc_bwd_eligible(B, H1, W1, H2, W2, C, radius, levels, dilation, dtype, &why)
                  : tc_eligible(B, H1, W1, H2, W2, C, radius, levels, dilation, dtype, &why);
  // TMA and 16-byte cp.async need 16-byte aligned map bases.
  if (elig && ((reinterpret_cast<uintptr_t>(p1) | reinterpret_cast<uintptr_t>(p2)) & 15)) {
    elig = false;
    why = "maps not 16-byte aligned";
  }
  if (engine == LCB200_ENGINE_TC && !elig) {
    set_error("tensor-core engine not eligible: " + why);
    *ok = false;
    return false;
  }
  if (engine != LCB200_ENGINE_AUTO && engine != LCB200_ENGINE_TC) {
    set_error("unknown engine " + std::to_string(engine));
    *ok = false;
    return false;
  }
  return elig;
}

// sort_ws (tensor-core engine only, may be null): keep the pixel sort there
// for a later backward (...KeepSort); ws then holds only the rest.
bool pyramid_forward_impl(const void* f1, const void* f2, const void* co, void* out, int B,
                          int H1, int W1, int H2, int W2, int C, int radius, int levels, int dil,
                          int dtype, int cdtype, bool ymajor, float scale, int engine, void* ws,
                          size_t ws_bytes, bool lib_ws, cudaStream_t s, void* sort_ws,
                          size_t sort_bytes) {
  clear_error();
  bool empty = false;
  if (!validate_pyramid(B, H1, W1, H2, W2, C, radius, levels, dil, dtype, &empty)) return false;
  if (empty) return true;
  if (cdtype != LCB200_F32 && cdtype != LCB200_F16) {
    set_error("coords dtype must be LCB200_F32 (0) or LCB200_F16 (1)");
    return false;
  }
  bool ok = true;
  if (use_tc(engine, B, H1, W1, H2, W2, C, radius, levels, dil, dtype, &ok, false, f1, f2)) {
    size_t need = tc_workspace_bytes(B, H1, W1, H2, W2, C, radius, levels, false);
    if (lib_ws) {
      ScratchLease lease(need, s);
      if (!lease.ok()) return false;
      return tc_forward(f1, f2, co, out, B, H1, W1, H2, W2, C, radius, levels, cdtype, ymajor,
                        scale, nullptr, lease.ptr(), need, s);
    }
    if (sort_ws) {
      const size_t sb = tc_sort_state_bytes(B, H1, W1, H2, W2, C, radius, levels);
      if (sort_bytes < sb) {
        set_error("sort state too small: need " + std::to_string(sb) + " B, got " +
                  std::to_string(sort_bytes));
        return false;
      }
      need -= sb;
    }
    if (ws_bytes < need || (need && ws == nullptr)) {
      set_error("workspace too small: need " + std::to_string(need) + " B, got " +
                std::to_string(ws_bytes));
      return false;
    }
    return tc_forward(f1, f2, co, out, B, H1, W1, H2, W2, C, radius, levels, cdtype, ymajor,
                      scale, sort_ws, ws, ws_bytes, s);
  }
  if (!ok) return false;
  return simt_forward(f1, f2, co, out, B, H1, W1, H2, W2, C, radius, levels, dil, dtype, cdtype,
                      ymajor, scale, s);
}

// sort_ws (tensor-core engine only, may be null): the sort a ...KeepSort
// forward of the same coords left there; ws then holds only the rest.
bool pyramid_backward_impl(const void* f1, const void* f2, const void* co, const void* gout,
                           void* f1g, float* f2g, int B, int H1, int W1, int H2, int W2, int C,
                           int radius, int levels, int dil, int dtype, int cdtype, bool ymajor,
                           float scale, int accumulate, int engine, void* ws, size_t ws_bytes,
                           bool lib_ws, cudaStream_t s, const void* sort_ws, size_t sort_bytes) {
  clear_error();
  bool empty = false;
  if (!validate_pyramid(B, H1, W1, H2, W2, C, radius, levels, dil, dtype, &empty)) return false;
  if (empty) return true;
  if (cdtype != LCB200_F32 && cdtype != LCB200_F16) {
    set_error("coords dtype must be LCB200_F32 (0) or LCB200_F16 (1)");
    return false;
  }
  const bool acc1 = (accumulate & LCB200_ACC_FMAP1) != 0;
  if (!(accumulate & LCB200_ACC_FMAP2)) {
    const PyrGeom g = make_geom(H2, W2, C, levels);
    if (cudaMemsetAsync(f2g, 0, sizeof(float) * (size_t)B * g.batch_elems, s) != cudaSuccess)
      return check_launch("memset fmap2_grad");
  }
  bool ok = true;
  if (use_tc(engine, B, H1, W1, H2, W2, C, radius, levels, dil, dtype, &ok, true, f1, f2)) {
    size_t need = tc_workspace_bytes(B, H1, W1, H2, W2, C, radius, levels, true);
    if (lib_ws) {
      ScratchLease lease(need, s);
      if (!lease.ok()) return false;
      return tc_backward(f1, f2, co, gout, f1g, f2g, B, H1, W1, H2, W2, C, radius, levels,
                         cdtype, ymajor, scale, acc1, nullptr, lease.ptr(), need, s);
    }
    if (sort_ws) {
      const size_t sb = tc_sort_state_bytes(B, H1, W1, H2, W2, C, radius, levels);
      if (sort_bytes < sb) {
        set_error("sort state too small: need " + std::to_string(sb) + " B, got " +
                  std::to_string(sort_bytes));
        return false;
      }
      need -= sb;
    }
    if (ws_bytes < need || (need && ws == nullptr)) {
      set_error("workspace too small: need " + std::to_string(need) + " B, got " +
                std::to_string(ws_bytes));
      return false;
    }
    return tc_backward(f1, f2, co, gout, f1g, f2g, B, H1, W1, H2, W2, C, radius, levels, cdtype,
                       ymajor, scale, acc1, const_cast<void*>(sort_ws), ws, ws_bytes, s);
  }
  if (!ok) return false;
  if (deterministic_mode()) {
    // grad_fmap1 from the CUDA-core kernel without its scattered fmap2
    // adds; grad_fmap2 pulled per output position over the sorted pixels
    std::string why;
    if (!tc_det_pull_ok(B, H1, W1, H2, W2, C, radius, levels, dil, &why)) {
      set_error("deterministic mode: the CUDA-core backward's deterministic grad_fmap2 needs " +
                why);
      return false;
    }
    const size_t need = tc_det_pull_bytes(B, H1, W1, H2, W2, C, radius, levels);
    if (!simt_backward(f1, f2, co, gout, f1g, f2g, B, H1, W1, H2, W2, C, radius, levels, dil,
                       dtype, cdtype, ymajor, scale, acc1, false, s))
      return false;
    if (lib_ws) {
      ScratchLease lease(need, s);
      if (!lease.ok()) return false;
      return tc_det_f2_pull(f1, co, gout, f2g, B, H1, W1, H2, W2, C, radius, levels, dtype,
                            cdtype, ymajor, scale, lease.ptr(), need, s);
    }
    if (ws_bytes < need || ws == nullptr) {
      set_error("workspace too small: need " + std::to_string(need) + " B, got " +
                std::to_string(ws_bytes));
      return false;
    }
    return tc_det_f2_pull(f1, co, gout, f2g, B, H1, W1, H2, W2, C, radius, levels, dtype,
                          cdtype, ymajor, scale, ws, ws_bytes, s);
  }
  return simt_backward(f1, f2, co, gout, f1g, f2g, B, H1, W1, H2, W2, C, radius, levels, dil,
                       dtype, cdtype, ymajor, scale, acc1, true, s);
}

bool pyramid_forward(const void* f1, const void* f2, const void* co, void* out, int B, int H1,
                     int W1, int H2, int W2, int C, int radius, int levels, int dil, int dtype,
                     int cdtype, bool ymajor, float scale, int engine, void* ws, size_t ws_bytes,
                     bool lib_ws, cudaStream_t s, void* sort_ws = nullptr,
                     size_t sort_bytes = 0) {
  NvtxRange range("localcorr_b200 pyramid forward");
  return bounds_finish(
      pyramid_forward_impl(f1, f2, co, out, B, H1, W1, H2, W2, C, radius, levels, dil, dtype,
                           cdtype, ymajor, scale, engine, ws, ws_bytes, lib_ws, s, sort_ws,
                           sort_bytes),
      s);
}

bool pyramid_backward(const void* f1, const void* f2, const void* co, const void* gout,
                      void* f1g, float* f2g, int B, int H1, int W1, int H2, int W2, int C,
                      int radius, int levels, int dil, int dtype, int cdtype, bool ymajor,
                      float scale, int accumulate, int engine, void* ws, size_t ws_bytes,
                      bool lib_ws, cudaStream_t s, const void* sort_ws = nullptr,
                      size_t sort_bytes = 0) {
  NvtxRange range("localcorr_b200 pyramid backward");
  return bounds_finish(
      pyramid_backward_impl(f1, f2, co, gout, f1g, f2g, B, H1, W1, H2, W2, C, radius, levels,
                            dil, dtype, cdtype, ymajor, scale, accumulate, engine, ws, ws_bytes,
                            lib_ws, s, sort_ws, sort_bytes),
      s);
}

bool validate_layout(int B, int C, int H, int W, int dtype) {
  if (dtype != LCB200_F32 && dtype != LCB200_F16) {
    set_error("dtype must be LCB200_F32 (0) or LCB200_F16 (1)");
    return false;
  }
  if (C <= 0 || H < 0 || W < 0 || B < 0) {
    set_error("invalid shape");
    return false;
  }
  return true;
}

}  // namespace
}  // namespace lcb200

using namespace lcb200;

extern "C" {

bool launchLocalCorrCudaPyramidForward(const void* fmap1, const void* fmap2_packed,
                                       const void* coords, void* corr, int B, int H1, int W1,
                                       int C, int radius, int levels, int dilation, bool isHalf,
                                       bool ymajor, cudaStream_t stream) {
  return pyramid_forward(fmap1, fmap2_packed, coords, corr, B, H1, W1, H1, W1, C, radius,
                         levels, dilation, isHalf ? LCB200_F16 : LCB200_F32,
                         isHalf ? LCB200_F16 : LCB200_F32, ymajor, 1.0f, LCB200_ENGINE_AUTO,
                         nullptr, 0, true, stream);
}

bool launchLocalCorrCudaPyramidBackward(const void* fmap1, const void* fmap2_packed,
                                        const void* coords, const void* corr_grad,
                                        void* fmap1_grad, float* fmap2_grad, int B, int H1,
                                        int W1, int C, int radius, int levels, int dilation,
                                        bool isHalf, bool ymajor, cudaStream_t stream) {
  return pyramid_backward(fmap1, fmap2_packed, coords, corr_grad, fmap1_grad, fmap2_grad, B, H1,
                          W1, H1, W1, C, radius, levels, dilation,
                          isHalf ? LCB200_F16 : LCB200_F32,
                          isHalf ? LCB200_F16 : LCB200_F32, ymajor, 1.0f, LCB200_ACC_FMAP2,
                          LCB200_ENGINE_AUTO, nullptr, 0, true, stream);
}

size_t localCorrB200PyramidWorkspaceBytesMapDims(int B, int H1, int W1, int H2, int W2, int C,
                                                 int radius, int levels, int dilation,
                                                 int dtype, int engine) {
  bool empty = false;
  clear_error();
  if (!validate_pyramid(B, H1, W1, H2, W2, C, radius, levels, dilation, dtype, &empty) || empty)
    return 0;
  bool ok = true;
  const bool f = use_tc(engine, B, H1, W1, H2, W2, C, radius, levels, dilation, dtype, &ok);
  ok = true;
  const bool b =
      use_tc(engine, B, H1, W1, H2, W2, C, radius, levels, dilation, dtype, &ok, true);
  if (!b && deterministic_mode() &&
      tc_det_pull_ok(B, H1, W1, H2, W2, C, radius, levels, dilation, nullptr)) {
    // the CUDA-core backward's deterministic grad_fmap2 sorts the pixels
    const size_t d = tc_det_pull_bytes(B, H1, W1, H2, W2, C, radius, levels);
    return f ? std::max(d, tc_workspace_bytes(B, H1, W1, H2, W2, C, radius, levels, false)) : d;
  }
  if (!f && !b) return 0;
  return tc_workspace_bytes(B, H1, W1, H2, W2, C, radius, levels, b);
}

size_t localCorrB200PyramidSortStateBytes(int B, int H1, int W1, int H2, int W2, int C,
                                          int radius, int levels, int dilation, int dtype,
                                          int engine) {
  bool empty = false;
  clear_error();
  if (!validate_pyramid(B, H1, W1, H2, W2, C, radius, levels, dilation, dtype, &empty) || empty)
    return 0;
  bool ok = true;
  // the backward's eligibility: a sort is only kept for a tensor-core pair
  if (!use_tc(engine, B, H1, W1, H2, W2, C, radius, levels, dilation, dtype, &ok, true))
    return 0;
  return tc_sort_state_bytes(B, H1, W1, H2, W2, C, radius, levels);
}

bool launchLocalCorrB200PyramidForwardKeepSort(
    const void* fmap1, const void* fmap2_packed, const void* coords, void* corr, int B, int H1,
    int W1, int H2, int W2, int C, int radius, int levels, int dilation, int dtype,
    int coords_dtype, bool ymajor, float scale, int engine, void* sort_state,
    size_t sort_state_bytes, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return pyramid_forward(fmap1, fmap2_packed, coords, corr, B, H1, W1, H2, W2, C, radius,
                         levels, dilation, dtype, coords_dtype, ymajor, scale, engine, workspace,
                         workspace_bytes, false, stream, sort_state, sort_state_bytes);
}

bool launchLocalCorrB200PyramidBackwardWithSort(
    const void* fmap1, const void* fmap2_packed, const void* coords, const void* corr_grad,
    void* fmap1_grad, float* fmap2_grad_f32, int B, int H1, int W1, int H2, int W2, int C,
    int radius, int levels, int dilation, int dtype, int coords_dtype, bool ymajor, float scale,
    int accumulate, int engine, const void* sort_state, size_t sort_state_bytes,
    void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return pyramid_backward(fmap1, fmap2_packed, coords, corr_grad, fmap1_grad, fmap2_grad_f32, B,
                          H1, W1, H2, W2, C, radius, levels, dilation, dtype, coords_dtype,
                          ymajor, scale, accumulate, engine, workspace, workspace_bytes, false,
                          stream, sort_state, sort_state_bytes);
}

size_t localCorrB200PyramidRecordsBytes(int B, int H1, int W1, int H2, int W2, int C, int radius,
                                        int levels) {
  clear_error();
  bool empty = false;
  if (!validate_pyramid(B, H1, W1, H2, W2, C, radius, levels, 1, LCB200_F16, &empty) || empty)
    return 0;
  std::string why;
  if (!tc_bwd_eligible(B, H1, W1, H2, W2, C, radius, levels, 1, LCB200_F16, &why)) return 0;
  return tc_records_bytes(B, H1, W1, H2, W2, C, radius, levels);
}

bool launchLocalCorrB200PyramidBackwardFmap1(
    const void* fmap1, const void* fmap2_packed, const void* coords, const void* corr_grad,
    void* fmap1_grad, int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
    int coords_dtype, bool ymajor, float scale, int accumulate, const void* sort_state,
    size_t sort_state_bytes, void* records, size_t records_bytes, void* workspace,
    size_t workspace_bytes, cudaStream_t stream) {
  NvtxRange range("localcorr_b200 pyramid backward (grad_fmap1, records kept)");
  clear_error();
  bool empty = false;
  if (!validate_pyramid(B, H1, W1, H2, W2, C, radius, levels, 1, LCB200_F16, &empty))
    return false;
  if (empty) return true;
  if (coords_dtype != LCB200_F32 && coords_dtype != LCB200_F16) {
    set_error("coords dtype must be LCB200_F32 (0) or LCB200_F16 (1)");
    return false;
  }
  bool ok = true;
  if (!use_tc(LCB200_ENGINE_TC, B, H1, W1, H2, W2, C, radius, levels, 1, LCB200_F16, &ok, true,
              fmap1, fmap2_packed))
    return false;
  const size_t sb = tc_sort_state_bytes(B, H1, W1, H2, W2, C, radius, levels);
  if (!sort_state || sort_state_bytes < sb) {
    set_error("sort state missing or too small: need " + std::to_string(sb) + " B");
    return false;
  }
  const size_t need = tc_workspace_bytes(B, H1, W1, H2, W2, C, radius, levels, true) - sb;
  if (workspace_bytes < need || (need && workspace == nullptr)) {
    set_error("workspace too small: need " + std::to_string(need) + " B, got " +
              std::to_string(workspace_bytes));
    return false;
  }
  return bounds_finish(
      tc_backward_fmap1(fmap1, fmap2_packed, coords, corr_grad, fmap1_grad, B, H1, W1, H2, W2,
                        C, radius, levels, coords_dtype, ymajor, scale,
                        (accumulate & LCB200_ACC_FMAP1) != 0, const_cast<void*>(sort_state),
                        workspace, workspace_bytes, records, records_bytes, stream),
      stream);
}

bool launchLocalCorrB200PyramidBackwardFmap2Pull(
    const void* const* sort_states, const void* const* records, int nlookups,
    float* fmap2_grad_f32, int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
    float scale, int accumulate, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  NvtxRange range("localcorr_b200 pyramid backward (grad_fmap2 of kept lookups)");
  clear_error();
  bool empty = false;
  if (!validate_pyramid(B, H1, W1, H2, W2, C, radius, levels, 1, LCB200_F16, &empty))
    return false;
  if (empty) return true;
  if (nlookups < 0 || (nlookups > 0 && (!sort_states || !records))) {
    set_error("grad_fmap2 pull: nlookups sort states and records required");
    return false;
  }
  if (!(accumulate & LCB200_ACC_FMAP2)) {
    const PyrGeom g = make_geom(H2, W2, C, levels);
    if (cudaMemsetAsync(fmap2_grad_f32, 0, sizeof(float) * (size_t)B * g.batch_elems, stream) !=
        cudaSuccess)
      return check_launch("memset fmap2_grad");
  }
  return bounds_finish(
      tc_pull_lookups(sort_states, records, nlookups, fmap2_grad_f32, B, H1, W1, H2, W2, C,
                      radius, levels, scale, workspace, workspace_bytes, stream),
      stream);
}

size_t localCorrB200PyramidWorkspaceBytes(int B, int H1, int W1, int C, int radius, int levels,
                                          int dilation, int dtype, int engine) {
  return localCorrB200PyramidWorkspaceBytesMapDims(B, H1, W1, H1, W1, C, radius, levels,
                                                   dilation, dtype, engine);
}

bool launchLocalCorrB200PyramidForward(const void* fmap1, const void* fmap2_packed,
                                       const void* coords, void* corr, int B, int H1, int W1,
                                       int C, int radius, int levels, int dilation, int dtype,
                                       int coords_dtype, bool ymajor, float scale, int engine,
                                       void* workspace, size_t workspace_bytes,
                                       cudaStream_t stream) {
  return pyramid_forward(fmap1, fmap2_packed, coords, corr, B, H1, W1, H1, W1, C, radius,
                         levels, dilation, dtype, coords_dtype, ymajor, scale, engine, workspace,
                         workspace_bytes, false, stream);
}

bool launchLocalCorrB200PyramidForwardMapDims(const void* fmap1, const void* fmap2_packed,
                                              const void* coords, void* corr, int B, int H1,
                                              int W1, int H2, int W2, int C, int radius,
                                              int levels, int dilation, int dtype,
                                              int coords_dtype, bool ymajor, float scale,
                                              int engine, void* workspace,
                                              size_t workspace_bytes, cudaStream_t stream) {
  return pyramid_forward(fmap1, fmap2_packed, coords, corr, B, H1, W1, H2, W2, C, radius,
                         levels, dilation, dtype, coords_dtype, ymajor, scale, engine, workspace,
                         workspace_bytes, false, stream);
}

bool launchLocalCorrB200PyramidBackward(const void* fmap1, const void* fmap2_packed,
                                        const void* coords, const void* corr_grad,
                                        void* fmap1_grad, float* fmap2_grad_f32, int B, int H1,
                                        int W1, int C, int radius, int levels, int dilation,
                                        int dtype, int coords_dtype, bool ymajor, float scale,
                                        int accumulate, int engine, void* workspace,
                                        size_t workspace_bytes, cudaStream_t stream) {
  return pyramid_backward(fmap1, fmap2_packed, coords, corr_grad, fmap1_grad, fmap2_grad_f32, B,
                          H1, W1, H1, W1, C, radius, levels, dilation, dtype, coords_dtype,
                          ymajor, scale, accumulate, engine, workspace, workspace_bytes, false,
                          stream);
}

bool launchLocalCorrB200PyramidBackwardMapDims(
    const void* fmap1, const void* fmap2_packed, const void* coords, const void* corr_grad,
    void* fmap1_grad, float* fmap2_grad_f32, int B, int H1, int W1, int H2, int W2, int C,
    int radius, int levels, int dilation, int dtype, int coords_dtype, bool ymajor, float scale,
    int accumulate, int engine, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return pyramid_backward(fmap1, fmap2_packed, coords, corr_grad, fmap1_grad, fmap2_grad_f32, B,
                          H1, W1, H2, W2, C, radius, levels, dilation, dtype, coords_dtype,
                          ymajor, scale, accumulate, engine, workspace, workspace_bytes, false,
                          stream);
}

bool launchLocalCorrB200PyramidBuild(const void* fmap2_nchw, void* fmap2_packed, int B, int C,
                                     int H, int W, int levels, int dtype, cudaStream_t stream) {
  clear_error();
  bool empty = false;
  if (!validate_pyramid(B, H, W, H, W, C, 0, levels, 1, dtype, &empty)) return false;
  if (empty) return true;
  NvtxRange range("localcorr_b200 pyramid build");
  return layout_pyramid_build(fmap2_nchw, fmap2_packed, B, C, H, W, levels, dtype, stream);
}

bool launchLocalCorrB200PyramidBuildBackward(const void* grad_packed, bool grad_is_f32,
                                             void* grad_fmap2_nchw, int B, int C, int H, int W,
                                             int levels, int dtype, cudaStream_t stream) {
  clear_error();
  bool empty = false;
  if (!validate_pyramid(B, H, W, H, W, C, 0, levels, 1, dtype, &empty)) return false;
  if (empty) return true;
  NvtxRange range("localcorr_b200 pyramid build backward");
  return layout_pyramid_build_grad(grad_packed, grad_is_f32, grad_fmap2_nchw, B, C, H, W,
                                   levels, dtype, stream);
}

bool launchLocalCorrB200NchwToNhwc(const void* in, void* out, int B, int C, int HW, int dtype,
                                   cudaStream_t stream) {
  clear_error();
  if (!validate_layout(B, C, HW, 1, dtype)) return false;
  if (B == 0 || HW == 0) return true;
  return layout_nchw_to_nhwc(in, out, B, C, HW, dtype, stream);
}

bool launchLocalCorrB200NhwcToNchw(const void* in, void* out, int B, int C, int HW, int dtype,
                                   cudaStream_t stream) {
  clear_error();
  if (!validate_layout(B, C, HW, 1, dtype)) return false;
  if (B == 0 || HW == 0) return true;
  return layout_nhwc_to_nchw(in, out, B, C, HW, dtype, stream);
}

bool launchLocalCorrB200SpatialForward(const void* in1, const void* in2, void* out, int B, int C,
                                       int H, int W, int radius, int dilation, int dtype,
                                       float scale, cudaStream_t stream) {
  clear_error();
  if (!validate_layout(B, C, H, W, dtype)) return false;
  if (radius < 0 || dilation < 1) {
    set_error("spatial correlation needs radius >= 0 and dilation >= 1");
    return false;
  }
  if (B == 0 || H == 0 || W == 0) return true;
  NvtxRange range("localcorr_b200 spatial forward");
  return bounds_finish(
      spatial_forward(in1, in2, out, B, C, H, W, radius, dilation, dtype, scale, stream), stream);
}

bool launchLocalCorrB200SpatialBackward(const void* in1, const void* in2, const void* grad_out,
                                        void* grad_in1, void* grad_in2, int B, int C, int H,
                                        int W, int radius, int dilation, int dtype, float scale,
                                        cudaStream_t stream) {
  clear_error();
  if (!validate_layout(B, C, H, W, dtype)) return false;
  if (radius < 0 || dilation < 1) {
    set_error("spatial correlation needs radius >= 0 and dilation >= 1");
    return false;
  }
  if (B == 0 || H == 0 || W == 0) return true;
  NvtxRange range("localcorr_b200 spatial backward");
  return bounds_finish(
      spatial_backward(in1, in2, grad_out, grad_in1, grad_in2, B, C, H, W, radius, dilation,
                          dtype, scale, stream),
      stream);
}

const char* localCorrB200GetLastError(void) { return g_last_error.c_str(); }

int localCorrB200DeviceStatus(int reset) { return tc_device_status(reset != 0); }

int localCorrB200Version(void) { return 100; }

long long localCorrB200LaunchCount(int reset) {
  return reset ? g_launches.exchange(0) : g_launches.load();
}

void localCorrB200SetDeterministic(int on) { g_deterministic.store(on ? 1 : 0); }

int localCorrB200GetDeterministic(void) { return g_deterministic.load(); }

long long localCorrB200BoundsViolations(int reset) { return bounds_total(reset != 0); }

}  // extern "C"
