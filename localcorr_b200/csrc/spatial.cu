// Spatial (PWC-Net) correlation, forward and backward, on NCHW inputs:
//   out[b, iy, ix, h, w] = scale * sum_c in1[b,c,h,w] * in2[b,c,h+dil(iy-r),w+dil(ix-r)]
// (zero outside the image). The reference runs this through its pyramid
// launcher with levels=1, y-major order and identity coordinates after two
// NHWC copies (blocks.py:649-668, spatial_corr.py:275-298); here the integer
// shifts are exploited directly: a CTA owns an 8x32 output tile, stages
// channel slabs of both inputs (plus the halo) in shared memory, and each
// thread keeps an 8-pixel x RD-displacement register block, sliding the
// shifted row through registers (dilation 1), so a shared-memory load feeds
// several FMAs. The backward is two gathers (no atomics):
//   grad_in1[c,p] = scale * sum_d g[d,p]     * in2[c,p+delta_d]
//   grad_in2[c,q] = scale * sum_d g[d,q-delta_d] * in1[c,q-delta_d]
#include <initializer_list>

#include "lc_common.cuh"

namespace lcb200 {
namespace {

constexpr int kTH = 8, kTW = 32, kPX = 8;

__host__ __device__ constexpr int odd_up(int v) { return v | 1; }

// ---- forward -------------------------------------------------------------
template <typename T, int RD, bool DIL1>
__global__ void __launch_bounds__(32 * RD)
spatial_fwd_kernel(const T* __restrict__ in1, const T* __restrict__ in2, T* __restrict__ out,
                   int C, int H, int W, int dil, float scale) {
  constexpr int CK = 8;
  constexpr int S1 = kTW + 1;  // odd row stride: conflict-free column reads
  extern __shared__ float smem[];
  const int R = (RD / 2) * dil;
  const int TR2 = kTH + 2 * R;
  const int TC2 = kTW + 2 * R;
  const int S2 = odd_up(TC2);
  float* in1s = smem;                    // [CK][kTH][S1]
  float* in2s = in1s + CK * kTH * S1;    // [CK][TR2][S2]

  const int b = blockIdx.z;
  const int tiles_x = (W + kTW - 1) / kTW;
  const int h0 = (blockIdx.x / tiles_x) * kTH;
  const int w0 = (blockIdx.x % tiles_x) * kTW;
  const int t = threadIdx.x;
  const int iy = t >> 5;
  const int s = t & 31;
  const int py = s >> 2;
  const int px0 = (s & 3) * kPX;
  const long long HW = (long long)H * W;
  const T* i1b = in1 + (long long)b * C * HW;
  const T* i2b = in2 + (long long)b * C * HW;

  float acc[kPX][RD];
#pragma unroll
  for (int i = 0; i < kPX; ++i)
#pragma unroll
    for (int j = 0; j < RD; ++j) acc[i][j] = 0.f;

  for (int c0 = 0; c0 < C; c0 += CK) {
    __syncthreads();
    for (int i = t; i < CK * kTH * kTW; i += blockDim.x) {
      const int x = i % kTW, y = (i / kTW) % kTH, cc = i / (kTW * kTH);
      const int gy = h0 + y, gx = w0 + x, c = c0 + cc;
      float v = 0.f;
      if (c < C && gy < H && gx < W) v = ldf(i1b + c * HW + (long long)gy * W + gx);
      in1s[(cc * kTH + y) * S1 + x] = v;
    }
    for (int i = t; i < CK * TR2 * TC2; i += blockDim.x) {
      const int x = i % TC2, y = (i / TC2) % TR2, cc = i / (TC2 * TR2);
      const int gy = h0 - R + y, gx = w0 - R + x, c = c0 + cc;
      float v = 0.f;
      if (c < C && gy >= 0 && gy < H && gx >= 0 && gx < W)
        v = ldf(i2b + c * HW + (long long)gy * W + gx);
      in2s[(cc * TR2 + y) * S2 + x] = v;
    }
    __syncthreads();
#pragma unroll 2
    for (int cc = 0; cc < CK; ++cc) {
      float a[kPX];
#pragma unroll
      for (int i = 0; i < kPX; ++i) a[i] = in1s[(cc * kTH + py) * S1 + px0 + i];
      const float* row = in2s + (cc * TR2 + py + dil * iy) * S2 + px0;
      if constexpr (DIL1) {
        float v[kPX + RD - 1];
#pragma unroll
        for (int j = 0; j < kPX + RD - 1; ++j) v[j] = row[j];
#pragma unroll
        for (int i = 0; i < kPX; ++i)
#pragma unroll
          for (int ix = 0; ix < RD; ++ix) acc[i][ix] = fmaf(a[i], v[i + ix], acc[i][ix]);
      } else {
#pragma unroll
        for (int i = 0; i < kPX; ++i)
#pragma unroll
          for (int ix = 0; ix < RD; ++ix) acc[i][ix] = fmaf(a[i], row[i + dil * ix], acc[i][ix]);
      }
    }
  }

  const int gy = h0 + py;
  if (gy >= H) return;
#pragma unroll
  for (int ix = 0; ix < RD; ++ix) {
    T* o = out + (((long long)b * RD + iy) * RD + ix) * HW + (long long)gy * W + w0 + px0;
#pragma unroll
    for (int i = 0; i < kPX; ++i)
      if (w0 + px0 + i < W) stf(o + i, acc[i][ix] * scale);
  }
}

// ---- backward ------------------------------------------------------------
// SHIFTED=false: grad_in1 (G at p, X = in2 at p+delta)
// SHIFTED=true : grad_in2 (G and X = in1 both at q-delta)
template <typename T, int RD, bool DIL1, bool SHIFTED>
__global__ void __launch_bounds__(128)
spatial_bwd_kernel(const T* __restrict__ gout, const T* __restrict__ X, T* __restrict__ gx,
                   int C, int H, int W, int dil, float scale) {
  constexpr int CKt = 8;   // channels per thread
  constexpr int CK = 32;   // channels per CTA
  extern __shared__ float smem[];
  const int r = RD / 2;
  const int R = r * dil;
  const int TC2 = kTW + 2 * R;
  const int SX = odd_up(TC2);
  const int GW = SHIFTED ? TC2 : kTW;       // G slab width
  const int SG = odd_up(GW);
  float* Gs = smem;                         // [RD][kTH][SG]
  float* Xs = Gs + RD * kTH * SG;           // [CK][kTH][SX]

  const int b = blockIdx.z;
  const int c0 = blockIdx.y * CK;
  const int tiles_x = (W + kTW - 1) / kTW;
  const int h0 = (blockIdx.x / tiles_x) * kTH;
  const int w0 = (blockIdx.x % tiles_x) * kTW;
  const int t = threadIdx.x;
  const int cg = t >> 5;
  const int s = t & 31;
  const int py = s >> 2;
  const int px0 = (s & 3) * kPX;
  const long long HW = (long long)H * W;
  const T* gb = gout + (long long)b * RD * RD * HW;
  const T* xb = X + (long long)b * C * HW;

  float acc[CKt][kPX];
#pragma unroll
  for (int c = 0; c < CKt; ++c)
#pragma unroll
    for (int i = 0; i < kPX; ++i) acc[c][i] = 0.f;

  for (int iy = 0; iy < RD; ++iy) {
    const int sy = dil * (iy - r);              // row shift of this displacement row
    const int grow0 = SHIFTED ? h0 - sy : h0;   // first global row of the G slab
    const int xrow0 = SHIFTED ? h0 - sy : h0 + sy;
    __syncthreads();
    for (int i = t; i < RD * kTH * GW; i += blockDim.x) {
      const int x = i % GW, y = (i / GW) % kTH, ix = i / (GW * kTH);
      const int gy = grow0 + y;
      const int gxx = SHIFTED ? w0 - R + x : w0 + x;
      float v = 0.f;
      if (gy >= 0 && gy < H && gxx >= 0 && gxx < W)
        v = ldf(gb + ((long long)iy * RD + ix) * HW + (long long)gy * W + gxx);
      Gs[(ix * kTH + y) * SG + x] = v;
    }
    for (int i = t; i < CK * kTH * TC2; i += blockDim.x) {
      const int x = i % TC2, y = (i / TC2) % kTH, cc = i / (TC2 * kTH);
      const int gy = xrow0 + y, gxx = w0 - R + x, c = c0 + cc;
      float v = 0.f;
      if (c < C && gy >= 0 && gy < H && gxx >= 0 && gxx < W)
        v = ldf(xb + c * HW + (long long)gy * W + gxx);
      Xs[(cc * kTH + y) * SX + x] = v;
    }
    __syncthreads();
    // G register block for this displacement row.
    float gv[RD][kPX];
#pragma unroll
    for (int ix = 0; ix < RD; ++ix)
#pragma unroll
      for (int i = 0; i < kPX; ++i) {
        // grad_in1: G at the output pixel; grad_in2: at q - delta, which is
        // slab column px + 2R - dil*ix.
        const int col = SHIFTED ? px0 + i + 2 * R - dil * ix : px0 + i;
        gv[ix][i] = Gs[(ix * kTH + py) * SG + col];
      }
#pragma unroll
    for (int cc = 0; cc < CKt; ++cc) {
      const float* xr = Xs + ((cg * CKt + cc) * kTH + py) * SX + px0;
      if constexpr (DIL1) {
        float v[kPX + RD - 1];
#pragma unroll
        for (int j = 0; j < kPX + RD - 1; ++j) v[j] = xr[j];
#pragma unroll
        for (int ix = 0; ix < RD; ++ix)
#pragma unroll
          for (int i = 0; i < kPX; ++i) {
            // grad_in1: X column px + ix; grad_in2: px + (RD-1) - ix.
            const float xv = SHIFTED ? v[i + RD - 1 - ix] : v[i + ix];
            acc[cc][i] = fmaf(gv[ix][i], xv, acc[cc][i]);
          }
      } else {
#pragma unroll
        for (int ix = 0; ix < RD; ++ix)
#pragma unroll
          for (int i = 0; i < kPX; ++i) {
            const int col = SHIFTED ? i + 2 * R - dil * ix : i + dil * ix;
            acc[cc][i] = fmaf(gv[ix][i], xr[col], acc[cc][i]);
          }
      }
    }
  }

  const int gy = h0 + py;
  if (gy >= H) return;
#pragma unroll
  for (int cc = 0; cc < CKt; ++cc) {
    const int c = c0 + cg * CKt + cc;
    if (c >= C) continue;
    T* o = gx + ((long long)b * C + c) * HW + (long long)gy * W + w0 + px0;
#pragma unroll
    for (int i = 0; i < kPX; ++i)
      if (w0 + px0 + i < W) stf(o + i, acc[cc][i] * scale);
  }
}

// ---- tiled path: dilation 1, W % 4 == 0, aligned bases -------------------
// Inputs stream into shared memory as units of 4 elements (16 B in float32,
// 8 B in float16) with cp.async, zero-filled outside the image; a unit is
// wholly inside or outside because W % 4 == 0 and units start on multiples
// of 4. The next slab is copied while the current one is used (double
// buffer). Shared rows are padded to a multiple of 4 elements plus 4, so the
// 4-element reads of a warp's 8 pixel quads hit distinct banks.
template <typename T>
__device__ __forceinline__ void cp4(T* dst, const T* src, bool valid) {
  if constexpr (sizeof(T) == 4) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(valid ? 16u : 0u)
                 : "memory");
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(valid ? 8u : 0u)
                 : "memory");
  }
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Four consecutive shared elements (4-element aligned) as floats.
__device__ __forceinline__ void ld4(const float* p, float* o) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}
__device__ __forceinline__ void ld4(const __half* p, float* o) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
  o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
}
// n consecutive shared elements starting at p (aligned to 4 when ALIGNED)
template <int N, bool ALIGNED, typename T>
__device__ __forceinline__ void ldn(const T* p, float* o) {
  if constexpr (ALIGNED) {
#pragma unroll
    for (int j = 0; j < N; j += 4) ld4(p + j, o + j);
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) o[j] = ldf(p + j);
  }
}
__device__ __forceinline__ void st4(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void st4(__half* p, const float* v) {
  __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

template <int RD>
struct TiledShape {
  static constexpr int R = RD / 2;
  static constexpr int R4 = (R + 3) / 4 * 4;  // halo in whole 4-element units
  static constexpr int OFF = R4 - R;          // slab column of pixel 0's first tap
  static constexpr int NV = (4 + RD - 1 + 3) / 4 * 4;  // shifted row values per quad
};

// Forward: CTA = 4 x 32 output pixels, warp iy = displacement row, lane =
// (pixel row, quad of 4 columns); each thread accumulates its 4 pixels x RD
// column displacements over 16-channel slabs: per channel one 4-element
// read of in1 and NV/4 of the shifted in2 row feed 4*RD FMAs.
constexpr int kFTH = 4, kFTW = 32, kFCK = 8;

template <int RD>
struct FwdTiled {
  using S = TiledShape<RD>;
  static constexpr int TR2 = kFTH + 2 * S::R;
  static constexpr int TC2 = kFTW + 2 * S::R4;
  static constexpr int S1 = kFTW + 4, S2 = TC2 + 4;
  static constexpr int SL1 = kFCK * kFTH * S1, SL2 = kFCK * TR2 * S2;
  template <typename T>
  static constexpr size_t smem() { return sizeof(T) * 2 * (SL1 + SL2); }
};

template <typename T, int RD>
__global__ void __launch_bounds__(32 * RD, 3)
spatial_fwd_tiled(const T* __restrict__ in1, const T* __restrict__ in2, T* __restrict__ out,
                  int C, int H, int W, float scale) {
  using S = TiledShape<RD>;
  using F = FwdTiled<RD>;
  extern __shared__ __align__(16) uint8_t sraw[];
  T* s1 = reinterpret_cast<T*>(sraw);
  T* s2 = s1 + 2 * F::SL1;
  const int b = blockIdx.z;
  const int tiles_x = (W + kFTW - 1) / kFTW;
  const int h0 = (blockIdx.x / tiles_x) * kFTH;
  const int w0 = (blockIdx.x % tiles_x) * kFTW;
  const int t = threadIdx.x;
  const int iy = t >> 5, lane = t & 31;
  const int q = lane & 7, py = lane >> 3;
  const long long HW = (long long)H * W;
  const T* i1b = in1 + (long long)b * C * HW;
  const T* i2b = in2 + (long long)b * C * HW;

  auto stage = [&](int buf, int c0) {
    constexpr int U1 = kFTW / 4, U2 = F::TC2 / 4;
    for (int u = t; u < kFCK * kFTH * U1; u += 32 * RD) {
      const int ux = u % U1, row = (u / U1) % kFTH, cc = u / (U1 * kFTH);
      const int c = c0 + cc, gy = h0 + row, gx = w0 + 4 * ux;
      const bool v = c < C && gy < H && gx < W;
      cp4(s1 + buf * F::SL1 + (cc * kFTH + row) * F::S1 + 4 * ux,
          v ? i1b + c * HW + (long long)gy * W + gx : in1, v);
    }
    for (int u = t; u < kFCK * F::TR2 * U2; u += 32 * RD) {
      const int ux = u % U2, row = (u / U2) % F::TR2, cc = u / (U2 * F::TR2);
      const int c = c0 + cc, gy = h0 - S::R + row, gx = w0 - S::R4 + 4 * ux;
      const bool v = c < C && gy >= 0 && gy < H && gx >= 0 && gx < W &&
                     LCB_IN(c * HW + (long long)gy * W + gx + 4 <= (long long)C * HW,
                            kSiteSpatial, c * HW + (long long)gy * W + gx);
      cp4(s2 + buf * F::SL2 + (cc * F::TR2 + row) * F::S2 + 4 * ux,
          v ? i2b + c * HW + (long long)gy * W + gx : in2, v);
    }
    cp_commit();
  };

  float acc[RD][4];
#pragma unroll
  for (int ix = 0; ix < RD; ++ix)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[ix][i] = 0.f;
  const int nch = (C + kFCK - 1) / kFCK;
  stage(0, 0);
  for (int k = 0; k < nch; ++k) {
    if (k + 1 < nch) {
      stage((k + 1) & 1, (k + 1) * kFCK);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const T* a_s = s1 + (k & 1) * F::SL1 + py * F::S1 + 4 * q;
    const T* v_s = s2 + (k & 1) * F::SL2 + (py + iy) * F::S2 + 4 * q + S::OFF;
#pragma unroll 2
    for (int cc = 0; cc < kFCK; ++cc) {
      float a[4], v[S::NV];
      ld4(a_s + cc * kFTH * F::S1, a);
      ldn<S::NV, S::OFF % 4 == 0>(v_s + cc * F::TR2 * F::S2, v);
#pragma unroll
      for (int ix = 0; ix < RD; ++ix)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[ix][i] = fmaf(a[i], v[i + ix], acc[ix][i]);
    }
    __syncthreads();
  }
  const int gy = h0 + py, gx = w0 + 4 * q;
  if (gy >= H || gx >= W) return;
#pragma unroll
  for (int ix = 0; ix < RD; ++ix) {
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = acc[ix][i] * scale;
    st4(out + (((long long)b * RD + iy) * RD + ix) * HW + (long long)gy * W + gx, o);
  }
}

// Backward (two gathers, no atomics): CTA = 8 x 32 pixels x 16 channels,
// 128 threads = 64 pixel quads x 2 groups of 8 channels. The CTA's channel
// slab of X (in2 for grad_in1, in1 for grad_in2) with its halo rows and
// columns is copied once; the incoming gradients are copied one
// displacement row at a time (RD maps, double-buffered). For displacement
// row iy each thread holds the RD x 4 gradients of its pixels and, per
// channel, reads one shifted X row segment: 4*RD FMAs per NV/4 reads.
//   grad_in1[c,p] = scale * sum_d g[d,p] * in2[c,p+delta_d]
//   grad_in2[c,q] = scale * sum_d g[d,q-delta_d] * in1[c,q-delta_d]
constexpr int kBTH = 8, kBTW = 32, kBCK = 16;

template <int RD, bool SHIFTED>
struct BwdTiled {
  using S = TiledShape<RD>;
  static constexpr int XR = kBTH + 2 * S::R;
  static constexpr int XC = kBTW + 2 * S::R4;
  static constexpr int SX = XC + 4;
  static constexpr int GC = SHIFTED ? XC : kBTW;
  static constexpr int SG = GC + 4;
  static constexpr int XSL = kBCK * XR * SX;
  static constexpr int GSL = RD * kBTH * SG;
  template <typename T>
  static constexpr size_t smem() { return sizeof(T) * (XSL + 2 * GSL); }
};

template <typename T, int RD, bool SHIFTED>
__global__ void __launch_bounds__(128)
spatial_bwd_tiled(const T* __restrict__ gout, const T* __restrict__ X, T* __restrict__ gx,
                  int C, int H, int W, float scale) {
  using S = TiledShape<RD>;
  using Bt = BwdTiled<RD, SHIFTED>;
  extern __shared__ __align__(16) uint8_t sraw[];
  T* Xs = reinterpret_cast<T*>(sraw);
  T* Gs = Xs + Bt::XSL;
  const int b = blockIdx.z;
  const int c0 = blockIdx.y * kBCK;
  const int tiles_x = (W + kBTW - 1) / kBTW;
  const int h0 = (blockIdx.x / tiles_x) * kBTH;
  const int w0 = (blockIdx.x % tiles_x) * kBTW;
  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int q = lane & 7, py = (warp & 1) * 4 + (lane >> 3), cg = warp >> 1;
  const long long HW = (long long)H * W;
  const T* gb = gout + (long long)b * RD * RD * HW;
  const T* xb = X + (long long)b * C * HW;

  {
    constexpr int UX = Bt::XC / 4;
    for (int u = t; u < kBCK * Bt::XR * UX; u += 128) {
      const int ux = u % UX, row = (u / UX) % Bt::XR, cc = u / (UX * Bt::XR);
      const int c = c0 + cc, gy = h0 - S::R + row, gxx = w0 - S::R4 + 4 * ux;
      const bool v = c < C && gy >= 0 && gy < H && gxx >= 0 && gxx < W &&
                     LCB_IN(c * HW + (long long)gy * W + gxx + 4 <= (long long)C * HW,
                            kSiteSpatial, c * HW + (long long)gy * W + gxx);
      cp4(Xs + (cc * Bt::XR + row) * Bt::SX + 4 * ux,
          v ? xb + c * HW + (long long)gy * W + gxx : X, v);
    }
  }
  auto stage_g = [&](int buf, int iy) {
    constexpr int UG = Bt::GC / 4;
    // grad_in1: the gradients at the tile's pixels; grad_in2: at q - delta,
    // i.e. rows shifted by -(iy - r) and the column halo
    const int grow0 = SHIFTED ? h0 - (iy - S::R) : h0;
    const int gcol0 = SHIFTED ? w0 - S::R4 : w0;
    for (int u = t; u < RD * kBTH * UG; u += 128) {
      const int ux = u % UG, row = (u / UG) % kBTH, ix = u / (UG * kBTH);
      const int gy = grow0 + row, gxx = gcol0 + 4 * ux;
      const bool v = gy >= 0 && gy < H && gxx >= 0 && gxx < W;
      cp4(Gs + buf * Bt::GSL + (ix * kBTH + row) * Bt::SG + 4 * ux,
          v ? gb + ((long long)iy * RD + ix) * HW + (long long)gy * W + gxx : gout, v);
    }
    cp_commit();
  };

  float acc[8][4];
#pragma unroll
  for (int cc = 0; cc < 8; ++cc)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[cc][i] = 0.f;
  stage_g(0, 0);  // commits the X slab with it
  for (int iy = 0; iy < RD; ++iy) {
    if (iy + 1 < RD) {
      stage_g((iy + 1) & 1, iy + 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    float gv[RD][4];
    const T* g_s = Gs + (iy & 1) * Bt::GSL + py * Bt::SG + 4 * q;
#pragma unroll
    for (int ix = 0; ix < RD; ++ix) {
      if constexpr (SHIFTED)
        ldn<4, false>(g_s + ix * kBTH * Bt::SG + S::R4 + S::R - ix, gv[ix]);
      else
        ld4(g_s + ix * kBTH * Bt::SG, gv[ix]);
    }
    const int xrow = SHIFTED ? py + 2 * S::R - iy : py + iy;
    const T* x_s = Xs + ((cg * 8) * Bt::XR + xrow) * Bt::SX + 4 * q + S::OFF;
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
      float v[S::NV];
      ldn<S::NV, S::OFF % 4 == 0>(x_s + cc * Bt::XR * Bt::SX, v);
#pragma unroll
      for (int ix = 0; ix < RD; ++ix)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          acc[cc][i] = fmaf(gv[ix][i], SHIFTED ? v[i + RD - 1 - ix] : v[i + ix], acc[cc][i]);
    }
    __syncthreads();
  }
  const int gy = h0 + py, gxx = w0 + 4 * q;
  if (gy >= H || gxx >= W) return;
#pragma unroll
  for (int cc = 0; cc < 8; ++cc) {
    const int c = c0 + cg * 8 + cc;
    if (c >= C) break;
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = acc[cc][i] * scale;
    st4(gx + ((long long)b * C + c) * HW + (long long)gy * W + gxx, o);
  }
}

// The tiled kernels need dilation 1, W % 4 == 0 and bases aligned to a
// 4-element unit.
bool tiled_ok(int W, int dil, size_t esize, std::initializer_list<const void*> ptrs) {
  if (dil != 1 || W % 4 != 0) return false;
  for (const void* p : ptrs)
    if (p && reinterpret_cast<uintptr_t>(p) % (4 * esize)) return false;
  return true;
}

template <typename T, int RD>
bool fwd_rd(const void* in1, const void* in2, void* out, int B, int C, int H, int W, int dil,
            float scale, cudaStream_t s) {
  if (tiled_ok(W, dil, sizeof(T), {in1, in2, out})) {
    const size_t smem = FwdTiled<RD>::template smem<T>();
    const int tiles = ((H + kFTH - 1) / kFTH) * ((W + kFTW - 1) / kFTW);
    auto k = spatial_fwd_tiled<T, RD>;
    if (!ensure_smem_attr((const void*)k, smem)) return false;
    k<<<dim3(tiles, 1, B), 32 * RD, smem, s>>>((const T*)in1, (const T*)in2, (T*)out, C, H, W,
                                                scale);
    count_launch();
    return check_launch("spatial_fwd_tiled");
  }
  const int R = (RD / 2) * dil;
  const size_t smem = sizeof(float) * (8 * kTH * (kTW + 1) +
                                       (size_t)8 * (kTH + 2 * R) * odd_up(kTW + 2 * R));
  const int tiles = ((H + kTH - 1) / kTH) * ((W + kTW - 1) / kTW);
  dim3 grid(tiles, 1, B);
  if (dil == 1) {
    auto k = spatial_fwd_kernel<T, RD, true>;
    if (!ensure_smem_attr((const void*)k, smem)) return false;
    k<<<grid, 32 * RD, smem, s>>>((const T*)in1, (const T*)in2, (T*)out, C, H, W, dil, scale);
  } else {
    auto k = spatial_fwd_kernel<T, RD, false>;
    if (!ensure_smem_attr((const void*)k, smem)) return false;
    k<<<grid, 32 * RD, smem, s>>>((const T*)in1, (const T*)in2, (T*)out, C, H, W, dil, scale);
  }
  count_launch();
  return check_launch("spatial_fwd");
}

template <typename T, int RD, bool SHIFTED>
bool bwd_one(const void* g, const void* X, void* gx, int B, int C, int H, int W, int dil,
             float scale, cudaStream_t s) {
  if (tiled_ok(W, dil, sizeof(T), {g, X, gx})) {
    const size_t smem = BwdTiled<RD, SHIFTED>::template smem<T>();
    const int tiles = ((H + kBTH - 1) / kBTH) * ((W + kBTW - 1) / kBTW);
    auto k = spatial_bwd_tiled<T, RD, SHIFTED>;
    if (!ensure_smem_attr((const void*)k, smem)) return false;
    k<<<dim3(tiles, (C + kBCK - 1) / kBCK, B), 128, smem, s>>>((const T*)g, (const T*)X, (T*)gx,
                                                              C, H, W, scale);
    count_launch();
    return check_launch(SHIFTED ? "spatial_bwd_tiled_in2" : "spatial_bwd_tiled_in1");
  }
  const int R = (RD / 2) * dil;
  const int TC2 = kTW + 2 * R;
  const int GW = SHIFTED ? TC2 : kTW;
  const size_t smem = sizeof(float) * ((size_t)RD * kTH * odd_up(GW) +
                                       (size_t)32 * kTH * odd_up(TC2));
  const int tiles = ((H + kTH - 1) / kTH) * ((W + kTW - 1) / kTW);
  dim3 grid(tiles, (C + 31) / 32, B);
  if (dil == 1) {
    auto k = spatial_bwd_kernel<T, RD, true, SHIFTED>;
    if (!ensure_smem_attr((const void*)k, smem)) return false;
    k<<<grid, 128, smem, s>>>((const T*)g, (const T*)X, (T*)gx, C, H, W, dil, scale);
  } else {
    auto k = spatial_bwd_kernel<T, RD, false, SHIFTED>;
    if (!ensure_smem_attr((const void*)k, smem)) return false;
    k<<<grid, 128, smem, s>>>((const T*)g, (const T*)X, (T*)gx, C, H, W, dil, scale);
  }
  count_launch();
  return check_launch(SHIFTED ? "spatial_bwd_in2" : "spatial_bwd_in1");
}

template <typename T, int RD>
bool bwd_rd(const void* in1, const void* in2, const void* g, void* g1, void* g2, int B,
            int C, int H, int W, int dil, float scale, cudaStream_t s) {
  if (g1 && !bwd_one<T, RD, false>(g, in2, g1, B, C, H, W, dil, scale, s)) return false;
  if (g2 && !bwd_one<T, RD, true>(g, in1, g2, B, C, H, W, dil, scale, s)) return false;
  return true;
}

}  // namespace

constexpr int kSpatialMaxRadius = 4;

bool spatial_forward(const void* in1, const void* in2, void* out, int B, int C, int H, int W,
                     int radius, int dil, int dtype, float scale, cudaStream_t s) {
  const bool h = dtype == LCB200_F16;
  switch (radius) {
#define LCB_CASE(RAD)                                                                     \
  case RAD:                                                                               \
    return h ? fwd_rd<__half, 2 * RAD + 1>(in1, in2, out, B, C, H, W, dil, scale, s)     \
             : fwd_rd<float, 2 * RAD + 1>(in1, in2, out, B, C, H, W, dil, scale, s);
    LCB_CASE(0) LCB_CASE(1) LCB_CASE(2) LCB_CASE(3) LCB_CASE(4)
#undef LCB_CASE
    default:
      set_error("spatial correlation kernel supports radius <= " +
                std::to_string(kSpatialMaxRadius) + " (got " + std::to_string(radius) + ")");
      return false;
  }
}

bool spatial_backward(const void* in1, const void* in2, const void* g, void* g1, void* g2,
                      int B, int C, int H, int W, int radius, int dil, int dtype, float scale,
                      cudaStream_t s) {
  const bool h = dtype == LCB200_F16;
  switch (radius) {
#define LCB_CASE(RAD)                                                                         \
  case RAD:                                                                                   \
    return h ? bwd_rd<__half, 2 * RAD + 1>(in1, in2, g, g1, g2, B, C, H, W, dil, scale, s)   \
             : bwd_rd<float, 2 * RAD + 1>(in1, in2, g, g1, g2, B, C, H, W, dil, scale, s);
    LCB_CASE(0) LCB_CASE(1) LCB_CASE(2) LCB_CASE(3) LCB_CASE(4)
#undef LCB_CASE
    default:
      set_error("spatial correlation kernel supports radius <= " +
                std::to_string(kSpatialMaxRadius) + " (got " + std::to_string(radius) + ")");
      return false;
  }
}

LCB_BOUNDS_READER(bounds_read_spatial)

}  // namespace lcb200
