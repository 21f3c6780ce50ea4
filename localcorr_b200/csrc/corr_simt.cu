// CUDA-core (SIMT) engine of the pyramid local correlation: every dtype,
// channel count, radius, dilation and level count the C ABI accepts.
//
// Formulation (linearity of the bilinear tap, the same identity the
// reference's standard-ops path uses, onnx_generic.py:11-21): for a pixel and
// a level, the dot products of fmap1 with the fmap2 samples on the integer
// grid covered by the window are computed once,
//     D[j][k] = <fmap1[p], fmap2_l[y_j][x_k]>,
// and every output is the bilinear combination of its four grid neighbours,
//     out(iy, ix) = wa*D[j0][k0] + wb*D[j0][k1] + wc*D[j1][k0] + wd*D[j1][k1].
// With dilation 1 neighbouring taps share grid columns/rows, so a level costs
// (2r+2)^2 dot products instead of the 4*(2r+1)^2 corner reads per channel of
// the tap-by-tap form (cuda_pyramid/localcorr_cuda_pyramid_kernel.cu:53-282).
//
// Work split: a CTA owns PG = 8*PPW consecutive output pixels of one batch
// image; each warp owns PPW of them, lanes split the channels. Outputs of a
// level are staged in shared memory and written plane by plane, so the
// [B, L, RD*RD, H, W] stores are coalesced along W.
#include <initializer_list>

#include "lc_common.cuh"

namespace lcb200 {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

// Grid column k of the window in level coordinates (xb = x0 - r*dil).
__device__ __forceinline__ int grid_pos(int base, int k, int dil) {
  return dil == 1 ? base + k : base + dil * (k >> 1) + (k & 1);
}

// Four consecutive channels of a map row as floats (16-byte load in
// float32, 8-byte load in float16); p is 4-element aligned.
__device__ __forceinline__ float4 ld4g(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4g(const __half* p) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// Dot products of one fmap1 row (fp32 in shared memory) with NX fmap2
// samples of grid row y; lane-split channels, 8 columns per warp reduction.
// V4: C % 4 == 0 and aligned rows, each lane reads 4 consecutive channels
// per load (a warp covers 128 channels per step).
template <typename T, bool V4>
__device__ void dots_row(const float* __restrict__ f1q, const T* __restrict__ f2l,
                         int y, int hl, int wl, int xb, int dil, int NX, int C,
                         float* __restrict__ dst, int lane) {
  const bool rowok = (y >= 0) && (y < hl);
  for (int k0 = 0; k0 < NX; k0 += 8) {
    const T* ptr[8];
    bool ok[8];
    bool any = false;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int x = grid_pos(xb, k0 + k, dil);
      ok[k] = rowok && (k0 + k < NX) && x >= 0 && x < wl;
      const long long e = ((long long)(ok[k] ? y : 0) * wl + (ok[k] ? x : 0)) * C;
      if (ok[k] && !LCB_IN(e >= 0 && e + C <= (long long)hl * wl * C, kSiteSimtFwd, e))
        ok[k] = false;
      ptr[k] = f2l + e;
      any |= ok[k];
    }
    if (!any) {
      if (lane < 8 && k0 + lane < NX) dst[k0 + lane] = 0.f;
      continue;
    }
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
    if constexpr (V4) {
      for (int c = 4 * lane; c < C; c += 128) {
        const float4 f = *reinterpret_cast<const float4*>(f1q + c);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (ok[k]) {
            const float4 v = ld4g(ptr[k] + c);
            acc[k] = fmaf(f.x, v.x, fmaf(f.y, v.y, fmaf(f.z, v.z, fmaf(f.w, v.w, acc[k]))));
          }
      }
    } else {
      for (int c = lane; c < C; c += 32) {
        const float f = f1q[c];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (ok[k]) acc[k] = fmaf(f, ldf(ptr[k] + c), acc[k]);
      }
    }
    const float red = warp_reduce8(acc, lane);
    const int kk = k0 + ((lane >> 2) & 7);
    if ((lane & 3) == 0 && kk < NX) dst[kk] = red;
  }
}

template <typename T, typename TC, int PPW, bool V4>
__global__ void __launch_bounds__(kThreads)
corr_fwd_simt_kernel(const T* __restrict__ fmap1, const T* __restrict__ fmap2p,
                     const TC* __restrict__ coords, T* __restrict__ corr,
                     int H1, int W1, int C, int r, int dil, bool ymajor,
                     float scale, PyrGeom g) {
  constexpr int PG = kWarps * PPW;
  extern __shared__ float smem[];
  const int RD = 2 * r + 1;
  const int RD2 = RD * RD;
  const int NX = (dil == 1) ? RD + 1 : 2 * RD;
  float* f1s = smem;                   // [PG][C]
  float* stage = f1s + PG * C;         // [RD2][PG]
  float* rows = stage + RD2 * PG;      // [kWarps][2][NX]

  const int b = blockIdx.y;
  const int HW = H1 * W1;
  const int p0 = blockIdx.x * PG;
  const int npix = min(PG, HW - p0);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  for (int i = threadIdx.x; i < PG * C; i += kThreads) {
    const int q = i / C;
    const int c = i - q * C;
    f1s[i] = q < npix ? ldf(fmap1 + ((long long)b * HW + p0 + q) * C + c) : 0.f;
  }
  __syncthreads();

  float* rowA = rows + warp * 2 * NX;
  float* rowB = rowA + NX;
  const T* f2b = fmap2p + (long long)b * g.batch_elems;

  // small problems spread the levels over blockIdx.z
  for (int lvl = blockIdx.z; lvl < g.levels; lvl += gridDim.z) {
    const int hl = g.h[lvl], wl = g.w[lvl];
    const T* f2l = f2b + g.off[lvl];
    const float inv = 1.f / (float)(1 << lvl);
    for (int pi = 0; pi < PPW; ++pi) {
      const int q = warp * PPW + pi;
      if (q >= npix) break;
      const int p = p0 + q;
      const float cx = ldf(coords + (long long)b * 2 * HW + p);
      const float cy = ldf(coords + (long long)b * 2 * HW + HW + p);
      // Level coordinates and bilinear weights, as in the reference kernel
      // (cuda_pyramid/localcorr_cuda_pyramid_kernel.cu:139-153).
      const float clx = cx * inv, cly = cy * inv;
      const float x0f = floorf(clx), y0f = floorf(cly);
      const float dx = clx - x0f, dy = cly - y0f;
      const int xb = (int)x0f - r * dil;
      const int yb = (int)y0f - r * dil;
      const float wa = (1.f - dx) * (1.f - dy), wb = dx * (1.f - dy);
      const float wc = (1.f - dx) * dy, wd = dx * dy;
      const float* f1q = f1s + q * C;
      float* A = rowA;
      float* Bv = rowB;
      for (int iy = 0; iy < RD; ++iy) {
        const int y = yb + dil * iy;
        if (iy == 0 || dil != 1) dots_row<T, V4>(f1q, f2l, y, hl, wl, xb, dil, NX, C, A, lane);
        dots_row<T, V4>(f1q, f2l, y + 1, hl, wl, xb, dil, NX, C, Bv, lane);
        __syncwarp();
        for (int ix = lane; ix < RD; ix += 32) {
          const int k0 = (dil == 1) ? ix : 2 * ix;
          const float v = wa * A[k0] + wb * A[k0 + 1] + wc * Bv[k0] + wd * Bv[k0 + 1];
          const int d = ymajor ? (ix + RD * iy) : (iy + RD * ix);
          stage[d * PG + q] = v;
        }
        __syncwarp();
        if (dil == 1) { float* t = A; A = Bv; Bv = t; }
      }
    }
    __syncthreads();
    T* outl = corr + ((long long)b * g.levels + lvl) * RD2 * HW + p0;
    for (int i = threadIdx.x; i < RD2 * PG; i += kThreads) {
      const int d = i / PG;
      const int q = i - d * PG;
      if (q < npix) stf(outl + (long long)d * HW + q, stage[i] * scale);
    }
    __syncthreads();
  }
}

template <typename T, typename TC, int PPW, bool V4>
__global__ void __launch_bounds__(kThreads)
corr_bwd_simt_kernel(const T* __restrict__ fmap1, const T* __restrict__ fmap2p,
                     const TC* __restrict__ coords, const T* __restrict__ corr_grad,
                     T* __restrict__ fmap1_grad, float* __restrict__ fmap2_grad,
                     int H1, int W1, int C, int r, int dil, bool ymajor,
                     float scale, bool acc1, bool add_f2, PyrGeom g) {
  constexpr int PG = kWarps * PPW;
  extern __shared__ float smem[];
  const int RD = 2 * r + 1;
  const int RD2 = RD * RD;
  const int NX = (dil == 1) ? RD + 1 : 2 * RD;
  float* f1s = smem;                 // [PG][C] fmap1 rows
  float* f1g = f1s + PG * C;         // [PG][C] fmap1 gradient accumulators
  float* stage = f1g + PG * C;       // [RD2][PG] incoming gradient of a level
  float* grow = stage + RD2 * PG;    // [kWarps][NX] one grid row of weights

  const int b = blockIdx.y;
  const int HW = H1 * W1;
  const int p0 = blockIdx.x * PG;
  const int npix = min(PG, HW - p0);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  for (int i = threadIdx.x; i < PG * C; i += kThreads) {
    const int q = i / C;
    const int c = i - q * C;
    f1s[i] = q < npix ? ldf(fmap1 + ((long long)b * HW + p0 + q) * C + c) : 0.f;
    f1g[i] = 0.f;
  }

  float* Gr = grow + warp * NX;
  const T* f2b = fmap2p + (long long)b * g.batch_elems;
  float* g2b = fmap2_grad + (long long)b * g.batch_elems;
  const int NY = NX;

  for (int lvl = 0; lvl < g.levels; ++lvl) {
    __syncthreads();
    const T* gl = corr_grad + ((long long)b * g.levels + lvl) * RD2 * HW + p0;
    for (int i = threadIdx.x; i < RD2 * PG; i += kThreads) {
      const int d = i / PG;
      const int q = i - d * PG;
      stage[i] = q < npix ? ldf(gl + (long long)d * HW + q) * scale : 0.f;
    }
    __syncthreads();
    const int hl = g.h[lvl], wl = g.w[lvl];
    const T* f2l = f2b + g.off[lvl];
    float* g2l = g2b + g.off[lvl];
    const float inv = 1.f / (float)(1 << lvl);
    for (int pi = 0; pi < PPW; ++pi) {
      const int q = warp * PPW + pi;
      if (q >= npix) break;
      const int p = p0 + q;
      const float cx = ldf(coords + (long long)b * 2 * HW + p);
      const float cy = ldf(coords + (long long)b * 2 * HW + HW + p);
      const float clx = cx * inv, cly = cy * inv;
      const float x0f = floorf(clx), y0f = floorf(cly);
      const float dx = clx - x0f, dy = cly - y0f;
      const int xb = (int)x0f - r * dil;
      const int yb = (int)y0f - r * dil;
      const float w[2][2] = {{(1.f - dx) * (1.f - dy), dx * (1.f - dy)},
                             {(1.f - dx) * dy, dx * dy}};
      auto gval = [&](int iy, int ix) -> float {
        if (iy < 0 || iy >= RD || ix < 0 || ix >= RD) return 0.f;
        const int d = ymajor ? (ix + RD * iy) : (iy + RD * ix);
        return stage[d * PG + q];
      };
      const float* f1q = f1s + q * C;
      float* f1gq = f1g + q * C;
      for (int j = 0; j < NY; ++j) {
        const int y = (dil == 1) ? yb + j : yb + dil * (j >> 1) + (j & 1);
        if (y < 0 || y >= hl) continue;
        // Grid-row weights: each tap spreads its gradient to its 4 corners.
        for (int k = lane; k < NX; k += 32) {
          float v;
          if (dil == 1) {
            v = gval(j, k) * w[0][0] + gval(j, k - 1) * w[0][1] +
                gval(j - 1, k) * w[1][0] + gval(j - 1, k - 1) * w[1][1];
          } else {
            v = gval(j >> 1, k >> 1) * w[j & 1][k & 1];
          }
          Gr[k] = v;
        }
        __syncwarp();
        const long long rowoff = (long long)y * wl;
        if constexpr (V4) {
          // four channels per lane: one vector load of fmap2 and one 4-wide
          // float32 reduction into its gradient per grid sample
          for (int c = 4 * lane; c < C; c += 128) {
            const float4 f1v = *reinterpret_cast<const float4*>(f1q + c);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int k = 0; k < NX; ++k) {
              const int x = grid_pos(xb, k, dil);
              const float gk = Gr[k];
              if (x < 0 || x >= wl || gk == 0.f) continue;
              const long long e = (rowoff + x) * C + c;
              if (!LCB_IN(e >= 0 && e + 4 <= (long long)hl * wl * C, kSiteSimtBwd, e)) continue;
              const float4 v = ld4g(f2l + e);
              acc.x = fmaf(gk, v.x, acc.x); acc.y = fmaf(gk, v.y, acc.y);
              acc.z = fmaf(gk, v.z, acc.z); acc.w = fmaf(gk, v.w, acc.w);
              if (add_f2)
                asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(g2l + e),
                             "f"(gk * f1v.x), "f"(gk * f1v.y), "f"(gk * f1v.z), "f"(gk * f1v.w)
                             : "memory");
            }
            float4* fg = reinterpret_cast<float4*>(f1gq + c);
            float4 o = *fg;
            o.x += acc.x; o.y += acc.y; o.z += acc.z; o.w += acc.w;
            *fg = o;
          }
        } else {
          for (int c = lane; c < C; c += 32) {
            const float f1v = f1q[c];
            float acc = 0.f;
            for (int k = 0; k < NX; ++k) {
              const int x = grid_pos(xb, k, dil);
              const float gk = Gr[k];
              if (x < 0 || x >= wl || gk == 0.f) continue;
              const long long e = (rowoff + x) * C + c;
              if (!LCB_IN(e >= 0 && e < (long long)hl * wl * C, kSiteSimtBwd, e)) continue;
              acc = fmaf(gk, ldf(f2l + e), acc);
              if (add_f2) atomicAdd(g2l + e, gk * f1v);
            }
            f1gq[c] += acc;
          }
        }
        __syncwarp();
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < PG * C; i += kThreads) {
    const int q = i / C;
    const int c = i - q * C;
    if (q < npix) {
      T* dst = fmap1_grad + ((long long)b * HW + p0 + q) * C + c;
      stf(dst, acc1 ? ldf(dst) + f1g[i] : f1g[i]);
    }
  }
}

size_t fwd_smem(int PG, int C, int RD, int NX) {
  return sizeof(float) * ((size_t)PG * C + (size_t)RD * RD * PG + (size_t)kWarps * 2 * NX);
}
size_t bwd_smem(int PG, int C, int RD, int NX) {
  return sizeof(float) * ((size_t)2 * PG * C + (size_t)RD * RD * PG + (size_t)kWarps * NX);
}

int num_sms_simt() {
  int dev = 0, v = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  return v > 0 ? v : 1;
}

// 4-channel vector path: C % 4 == 0 and 4-element aligned map bases
bool simt_v4(int C, size_t esize, std::initializer_list<const void*> ptrs) {
  if (C % 4) return false;
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) % (4 * esize)) return false;
  return true;
}

template <typename T, typename TC, int PPW>
bool launch_fwd(const void* f1, const void* f2, const void* co, void* out, int B,
                int H1, int W1, int C, int r, int dil, bool ymajor, float scale,
                const PyrGeom& g, size_t smem, cudaStream_t s) {
  auto k = simt_v4(C, sizeof(T), {f1, f2}) ? corr_fwd_simt_kernel<T, TC, PPW, true>
                                           : corr_fwd_simt_kernel<T, TC, PPW, false>;
  if (!ensure_smem_attr((const void*)k, smem)) return false;
  const int PG = kWarps * PPW;
  dim3 grid((H1 * W1 + PG - 1) / PG, B);
  // fewer CTAs than a few per SM: one CTA per (pixel group, level)
  if ((long long)grid.x * grid.y < 4ll * num_sms_simt()) grid.z = g.levels;
  k<<<grid, kThreads, smem, s>>>((const T*)f1, (const T*)f2, (const TC*)co, (T*)out,
                                 H1, W1, C, r, dil, ymajor, scale, g);
  count_launch();
  return check_launch("corr_fwd_simt");
}

template <typename T, typename TC, int PPW>
bool launch_bwd(const void* f1, const void* f2, const void* co, const void* gout,
                void* f1g, float* f2g, int B, int H1, int W1, int C, int r, int dil,
                bool ymajor, float scale, bool acc1, bool add_f2, const PyrGeom& g, size_t smem,
                cudaStream_t s) {
  auto k = simt_v4(C, sizeof(T), {f1, f2, f2g}) ? corr_bwd_simt_kernel<T, TC, PPW, true>
                                                 : corr_bwd_simt_kernel<T, TC, PPW, false>;
  if (!ensure_smem_attr((const void*)k, smem)) return false;
  const int PG = kWarps * PPW;
  dim3 grid((H1 * W1 + PG - 1) / PG, B);
  k<<<grid, kThreads, smem, s>>>((const T*)f1, (const T*)f2, (const TC*)co, (const T*)gout,
                                 (T*)f1g, f2g, H1, W1, C, r, dil, ymajor, scale, acc1, add_f2, g);
  count_launch();
  return check_launch("corr_bwd_simt");
}

}  // namespace

// Host entry: forward of the SIMT engine. Chooses 4 pixels per warp when the
// shared-memory footprint allows it, else 1.
bool simt_forward(const void* f1, const void* f2, const void* co, void* out, int B,
                  int H1, int W1, int H2, int W2, int C, int r, int levels, int dil, int dtype,
                  int cdtype, bool ymajor, float scale, cudaStream_t s) {
  const PyrGeom g = make_geom(H2, W2, C, levels);
  const int RD = 2 * r + 1;
  const int NX = (dil == 1) ? RD + 1 : 2 * RD;
  const size_t lim = (size_t)max_dyn_smem();
  int ppw = 4;
  // 4 pixels per warp unless that leaves fewer CTAs than a few per SM
  if (fwd_smem(kWarps * 4, C, RD, NX) > lim ||
      (long long)B * ((H1 * W1 + kWarps * 4 - 1) / (kWarps * 4)) < 4ll * num_sms_simt())
    ppw = 1;
  const size_t smem = fwd_smem(kWarps * ppw, C, RD, NX);
  if (smem > lim) {
    set_error("pyramid forward: shared-memory footprint " + std::to_string(smem) +
              " B exceeds the device limit for C=" + std::to_string(C) +
              ", radius=" + std::to_string(r));
    return false;
  }
#define LCB_FWD(T, TC)                                                                        \
  return ppw == 4                                                                             \
             ? launch_fwd<T, TC, 4>(f1, f2, co, out, B, H1, W1, C, r, dil, ymajor, scale, g,   \
                                    smem, s)                                                   \
             : launch_fwd<T, TC, 1>(f1, f2, co, out, B, H1, W1, C, r, dil, ymajor, scale, g,   \
                                    smem, s);
  if (dtype == LCB200_F32) {
    if (cdtype == LCB200_F32) { LCB_FWD(float, float) }
    LCB_FWD(float, __half)
  }
  if (cdtype == LCB200_F32) { LCB_FWD(__half, float) }
  LCB_FWD(__half, __half)
#undef LCB_FWD
}

bool simt_backward(const void* f1, const void* f2, const void* co, const void* gout,
                   void* f1g, float* f2g, int B, int H1, int W1, int H2, int W2, int C,
                   int r, int levels, int dil, int dtype, int cdtype, bool ymajor, float scale,
                   bool acc1, bool add_f2, cudaStream_t s) {
  const PyrGeom g = make_geom(H2, W2, C, levels);
  const int RD = 2 * r + 1;
  const int NX = (dil == 1) ? RD + 1 : 2 * RD;
  const size_t lim = (size_t)max_dyn_smem();
  int ppw = 4;
  if (bwd_smem(kWarps * 4, C, RD, NX) > lim ||
      (long long)B * ((H1 * W1 + kWarps * 4 - 1) / (kWarps * 4)) < 4ll * num_sms_simt())
    ppw = 1;
  const size_t smem = bwd_smem(kWarps * ppw, C, RD, NX);
  if (smem > lim) {
    set_error("pyramid backward: shared-memory footprint " + std::to_string(smem) +
              " B exceeds the device limit for C=" + std::to_string(C) +
              ", radius=" + std::to_string(r));
    return false;
  }
#define LCB_BWD(T, TC)                                                                        \
  return ppw == 4 ? launch_bwd<T, TC, 4>(f1, f2, co, gout, f1g, f2g, B, H1, W1, C, r, dil,    \
                                         ymajor, scale, acc1, add_f2, g, smem, s)              \
                  : launch_bwd<T, TC, 1>(f1, f2, co, gout, f1g, f2g, B, H1, W1, C, r, dil,    \
                                         ymajor, scale, acc1, add_f2, g, smem, s);
  if (dtype == LCB200_F32) {
    if (cdtype == LCB200_F32) { LCB_BWD(float, float) }
    LCB_BWD(float, __half)
  }
  if (cdtype == LCB200_F32) { LCB_BWD(__half, float) }
  LCB_BWD(__half, __half)
#undef LCB_BWD
}

LCB_BOUNDS_READER(bounds_read_simt)

}  // namespace lcb200
