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
#pragma unroll 2
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

template <typename T, int RD>
bool fwd_rd(const void* in1, const void* in2, void* out, int B, int C, int H, int W, int dil,
            float scale, cudaStream_t s) {
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

}  // namespace lcb200
