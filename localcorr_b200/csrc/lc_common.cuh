// Shared device/host helpers of the localcorr_b200 CUDA library.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "localcorr_b200.h"

namespace lcb200 {

constexpr int kMaxLevels = 8;  // same bound as the reference launchers

// ---- element conversion -------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

template <typename T>
__device__ __forceinline__ float ldf(const T* p) { return Elem<T>::to_f(*p); }
template <typename T>
__device__ __forceinline__ void stf(T* p, float v) { *p = Elem<T>::from_f(v); }

// ---- pyramid geometry ----------------------------------------------------
// Per-level dims (floor-halved) and element offsets inside one batch row of
// the packed fmap2 buffer.
struct PyrGeom {
  int levels;
  int h[kMaxLevels];
  int w[kMaxLevels];
  long long off[kMaxLevels];   // element offset of level l inside a batch row
  long long batch_elems;       // C * sum_l h_l * w_l
};

inline PyrGeom make_geom(int H1, int W1, int C, int levels) {
  PyrGeom g{};
  g.levels = levels;
  long long acc = 0;
  for (int l = 0; l < levels; ++l) {
    g.h[l] = H1 >> l;
    g.w[l] = W1 >> l;
    g.off[l] = acc;
    acc += (long long)C * g.h[l] * g.w[l];
  }
  g.batch_elems = acc;
  return g;
}

// ---- error reporting -----------------------------------------------------
void set_error(const std::string& msg);
void clear_error();
bool check_launch(const char* what);
void count_launch(int n = 1);

// Process-wide deterministic mode (localCorrB200SetDeterministic): the
// tensor-core engine sorts pixels in a fixed order and reduces grad_fmap2
// with one add per position, so repeated calls give identical bits.
bool deterministic_mode();

// Bounds-check build: after a successful call, synchronise s, read the device
// records and fail with the first violation's site; the normal build returns
// ok unchanged.
bool bounds_finish(bool ok, cudaStream_t s);

// Largest dynamic shared memory a CTA may opt into on the current device.
int max_dyn_smem();

// Raise a kernel's dynamic shared-memory limit once per (kernel, device);
// later calls with a smaller or equal size do nothing.
bool ensure_smem_attr(const void* func, size_t bytes);

// ---- bounds-check build (-DLC_BOUNDS_CHECK) -------------------------------
// Every data-dependent global index of the kernels goes through LCB_IN(cond,
// site, index): in a checked build a false condition counts a violation in
// a device record (first site and index kept), the access is skipped, and
// the entry point that launched the kernel synchronises its stream, reads
// the records and fails with the site's name. In the normal build LCB_IN is
// the constant true and the condition is not evaluated. Sites:
enum BoundsSite : int {
  kSiteNone = 0,
  kSiteTcHist,       // sort bin of a pixel
  kSiteTcScatter,    // sorted position of a pixel
  kSiteTcRankFix,    // pixel index of a bin member
  kSiteTcGather,     // fmap1 row of a sorted position (sorted fmap1 copy)
  kSiteTcFwdWork,    // forward chunk: sorted range and scratch rows
  kSiteTcFwdRow,     // forward chunk: fmap1 row of a member pixel
  kSiteTcUnsort,     // sorted position of an output pixel
  kSiteTcGint,       // sorted position of a pixel's gradient records
  kSiteTcBwd1,       // grad_fmap1 chunk: pixel of a sorted position
  kSiteTcBwd2,       // grad_fmap2 item: candidate's sorted position
  kSiteSimtFwd,      // CUDA-core forward: fmap2 element of a grid sample
  kSiteSimtBwd,      // CUDA-core backward: fmap2 element read and added
  kSiteSpatial,      // spatial correlation: in2 element of a shifted row
  kSiteCount
};

#ifdef LC_BOUNDS_CHECK
// One record per translation unit (the library is built without
// relocatable device code): [0] violations, [1] first site, [2] its index.
static __device__ unsigned long long lcb_bounds_rec[3];

__device__ __forceinline__ bool lcb_in(bool ok, int site, long long idx) {
  if (!ok && atomicAdd(&lcb_bounds_rec[0], 1ull) == 0ull) {
    lcb_bounds_rec[1] = (unsigned long long)site;
    lcb_bounds_rec[2] = (unsigned long long)idx;
  }
  return ok;
}
#define LCB_IN(cond, site, idx) ::lcb200::lcb_in((cond), (site), (long long)(idx))

// Reads (and with reset clears) this translation unit's record.
static inline bool lcb_read_bounds(unsigned long long out[3], bool reset) {
  if (cudaMemcpyFromSymbol(out, lcb_bounds_rec, sizeof(unsigned long long) * 3) != cudaSuccess)
    return false;
  if (reset && out[0]) {
    const unsigned long long z[3] = {0, 0, 0};
    if (cudaMemcpyToSymbol(lcb_bounds_rec, z, sizeof(z)) != cudaSuccess) return false;
  }
  return true;
}
#define LCB_BOUNDS_READER(name) \
  bool name(unsigned long long out[3], bool reset) { return lcb_read_bounds(out, reset); }
#else
#define LCB_IN(cond, site, idx) true
#define LCB_BOUNDS_READER(name) \
  bool name(unsigned long long out[3], bool) { out[0] = out[1] = out[2] = 0; return true; }
#endif

// Warp helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Reduce 8 per-lane partial sums across the warp. On return, lane L holds the
// full sum of value index (L >> 2) & 7 (one shuffle per value on average).
__device__ __forceinline__ float warp_reduce8(const float (&v)[8], int lane) {
  float w[4];
  const bool b4 = lane & 16;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b4 ? v[i] : v[i + 4];
    const float keep = b4 ? v[i + 4] : v[i];
    w[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float u[2];
  const bool b3 = lane & 8;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b3 ? w[i] : w[i + 2];
    const float keep = b3 ? w[i + 2] : w[i];
    u[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  const bool b2 = lane & 4;
  const float send = b2 ? u[0] : u[1];
  const float keep = b2 ? u[1] : u[0];
  float t = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  t += __shfl_xor_sync(0xffffffffu, t, 2);
  t += __shfl_xor_sync(0xffffffffu, t, 1);
  return t;
}

}  // namespace lcb200
