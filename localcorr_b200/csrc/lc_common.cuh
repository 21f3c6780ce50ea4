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

// Largest dynamic shared memory a CTA may opt into on the current device.
int max_dyn_smem();

// Raise a kernel's dynamic shared-memory limit once per (kernel, device);
// later calls with a smaller or equal size do nothing.
bool ensure_smem_attr(const void* func, size_t bytes);

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
