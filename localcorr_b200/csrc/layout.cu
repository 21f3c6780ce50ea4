// Layout preparation kernels of the RAFT-style block:
//  * NCHW <-> NHWC transposes (fmap1 and its gradient),
//  * the fused pyramid build: fmap2 NCHW -> packed batch-major NHWC pyramid,
//    all 2x2 average-pooled levels of an 8x32 level-0 tile in one pass,
//  * its gradient: packed level gradients -> NCHW fmap2 gradient in one pass.
// They replace the torch permute/avg_pool2d/cat chain of the reference block
// constructor (blocks.py:369-383) and its autograd backward.
#include "lc_common.cuh"

namespace lcb200 {
namespace {

// ---- [B, C, HW] <-> [B, HW, C] ---------------------------------------------
// 32x32 tiles through shared memory; both global sides coalesced.
template <typename T>
__global__ void transpose_kernel(const T* __restrict__ in, T* __restrict__ out,
                                 int R, int Ccols) {
  // in: [B][R][Ccols] -> out: [B][Ccols][R]
  __shared__ float tile[32][33];
  const long long bo = (long long)blockIdx.z * R * Ccols;
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int rr = r0 + i, cc = c0 + threadIdx.x;
    if (rr < R && cc < Ccols) tile[i][threadIdx.x] = ldf(in + bo + (long long)rr * Ccols + cc);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int cc = c0 + i, rr = r0 + threadIdx.x;
    if (rr < R && cc < Ccols) stf(out + bo + (long long)cc * R + rr, tile[threadIdx.x][i]);
  }
}

template <typename T>
bool launch_transpose(const void* in, void* out, int B, int R, int Ccols, cudaStream_t s) {
  dim3 grid((Ccols + 31) / 32, (R + 31) / 32, B);
  transpose_kernel<T><<<grid, dim3(32, 8), 0, s>>>((const T*)in, (T*)out, R, Ccols);
  count_launch();
  return check_launch("transpose");
}

// ---- fused pyramid build -----------------------------------------------------
// CTA = one 8x32 tile of level-0 pixels (aligned, so its level-l footprint is
// the (8>>l)x(32>>l) aligned tile of level l) and CC channels. Levels are
// pooled from the previous level's dtype-rounded values in the order
// (y0,x0),(y0,x1),(y1,x0),(y1,x1), then divided by 4, matching avg_pool2d.
constexpr int kTY = 8, kTX = 32;
constexpr int kFusedLevels = 4;  // levels 0..3 in the fused kernel

template <typename T, int CC>
__global__ void __launch_bounds__(256)
pyramid_build_kernel(const T* __restrict__ in, T* __restrict__ packed, int C, int H,
                     int W, PyrGeom g, int nlev) {
  // s[l] holds level l of the tile as [ty][tx][CC+1] (one padding word per
  // pixel keeps both the x-fastest NCHW side and the channel-fastest NHWC
  // side free of bank conflicts), fp32 values equal to the dtype-rounded
  // level values.
  constexpr int CP = CC + 1;
  __shared__ float s0[kTY * kTX * CP];
  __shared__ float s1[(kTY / 2) * (kTX / 2) * CP];
  const int b = blockIdx.z;
  const int c0 = blockIdx.y * CC;
  const int tiles_x = (W + kTX - 1) / kTX;
  const int ty0 = (blockIdx.x / tiles_x) * kTY;
  const int tx0 = (blockIdx.x % tiles_x) * kTX;
  const int nc = min(CC, C - c0);

  // Load the NCHW tile (coalesced along x).
  for (int i = threadIdx.x; i < CC * kTY * kTX; i += blockDim.x) {
    const int x = i % kTX;
    const int y = (i / kTX) % kTY;
    const int c = i / (kTX * kTY);
    const int gy = ty0 + y, gx = tx0 + x;
    float v = 0.f;
    if (c < nc && gy < H && gx < W)
      v = ldf(in + (((long long)b * C + c0 + c) * H + gy) * W + gx);
    s0[(y * kTX + x) * CP + c] = v;
  }
  __syncthreads();

  T* pb = packed + (long long)b * g.batch_elems;
  // Level 0: NHWC write, channel-fastest (coalesced along c).
  for (int i = threadIdx.x; i < CC * kTY * kTX; i += blockDim.x) {
    const int c = i % CC;
    const int x = (i / CC) % kTX;
    const int y = i / (CC * kTX);
    const int gy = ty0 + y, gx = tx0 + x;
    if (c < nc && gy < H && gx < W)
      stf(pb + g.off[0] + ((long long)gy * W + gx) * C + c0 + c, s0[(y * kTX + x) * CP + c]);
  }

  float* src = s0;
  float* dst = s1;
  int sy = kTY, sx = kTX;
  for (int l = 1; l < nlev && l < kFusedLevels; ++l) {
    const int ny = sy / 2, nx = sx / 2;
    __syncthreads();
    for (int i = threadIdx.x; i < CC * ny * nx; i += blockDim.x) {
      const int c = i % CC;
      const int x = (i / CC) % nx;
      const int y = i / (CC * nx);
      const float* q = src + ((2 * y) * sx + 2 * x) * CP + c;
      float acc = q[0];
      acc += q[CP];
      acc += q[sx * CP];
      acc += q[sx * CP + CP];
      // Round to the storage dtype so the next level pools rounded values.
      dst[(y * nx + x) * CP + c] = Elem<T>::to_f(Elem<T>::from_f(acc / 4.f));
    }
    __syncthreads();
    const int hl = g.h[l], wl = g.w[l];
    const int oy = ty0 >> l, ox = tx0 >> l;
    for (int i = threadIdx.x; i < CC * ny * nx; i += blockDim.x) {
      const int c = i % CC;
      const int x = (i / CC) % nx;
      const int y = i / (CC * nx);
      const int gy = oy + y, gx = ox + x;
      if (c < nc && gy < hl && gx < wl)
        stf(pb + g.off[l] + ((long long)gy * wl + gx) * C + c0 + c, dst[(y * nx + x) * CP + c]);
    }
    // Ping-pong: level l becomes the source of level l+1. s0 is free after
    // level 1 has been computed from it, so levels alternate s1 -> s0 -> s1.
    float* t = src; src = dst; dst = t;
    sy = ny; sx = nx;
  }
}

// Levels >= 4: pool level l-1 of the packed buffer into level l (NHWC).
template <typename T>
__global__ void pool_level_kernel(T* __restrict__ packed, int C, PyrGeom g, int l) {
  const int hl = g.h[l], wl = g.w[l];
  const int hp = g.h[l - 1], wp = g.w[l - 1];
  (void)hp;
  const long long n = (long long)hl * wl * C;
  const int b = blockIdx.y;
  T* pb = packed + (long long)b * g.batch_elems;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const long long pix = i / C;
    const int x = (int)(pix % wl), y = (int)(pix / wl);
    const T* q = pb + g.off[l - 1] + ((long long)(2 * y) * wp + 2 * x) * C + c;
    float acc = ldf(q);
    acc += ldf(q + C);
    acc += ldf(q + (long long)wp * C);
    acc += ldf(q + (long long)wp * C + C);
    stf(pb + g.off[l] + i, acc / 4.f);
  }
}

// ---- pyramid build gradient ----------------------------------------------------
// grad_nchw[b,c,y,x] = sum_l [y>>l < h_l && x>>l < w_l] * gp_l[b,y>>l,x>>l,c] / 4^l
// CTA = 8x32 level-0 tile x CC channels; level reads are channel-fastest
// (coalesced NHWC), the NCHW write goes through shared memory (coalesced x).
template <typename T, typename G, int CC>
__global__ void __launch_bounds__(256)
pyramid_grad_kernel(const G* __restrict__ gp, T* __restrict__ out, int C, int H, int W,
                    PyrGeom g) {
  constexpr int CP = CC + 1;  // [ty][tx][CC+1]: conflict-free on both sides
  __shared__ float acc[kTY * kTX * CP];
  const int b = blockIdx.z;
  const int c0 = blockIdx.y * CC;
  const int tiles_x = (W + kTX - 1) / kTX;
  const int ty0 = (blockIdx.x / tiles_x) * kTY;
  const int tx0 = (blockIdx.x % tiles_x) * kTX;
  const int nc = min(CC, C - c0);
  const G* gb = gp + (long long)b * g.batch_elems;
  for (int i = threadIdx.x; i < CC * kTY * kTX; i += blockDim.x) {
    const int c = i % CC;
    const int x = (i / CC) % kTX;
    const int y = i / (CC * kTX);
    const int gy = ty0 + y, gx = tx0 + x;
    float v = 0.f;
    if (c < nc && gy < H && gx < W) {
      float sc = 1.f;
      for (int l = 0; l < g.levels; ++l) {
        const int ly = gy >> l, lx = gx >> l;
        if (ly < g.h[l] && lx < g.w[l])
          v += sc * ldf(gb + g.off[l] + ((long long)ly * g.w[l] + lx) * C + c0 + c);
        sc *= 0.25f;
      }
    }
    acc[(y * kTX + x) * CP + c] = v;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < CC * kTY * kTX; i += blockDim.x) {
    const int x = i % kTX;
    const int y = (i / kTX) % kTY;
    const int c = i / (kTX * kTY);
    const int gy = ty0 + y, gx = tx0 + x;
    if (c < nc && gy < H && gx < W)
      stf(out + (((long long)b * C + c0 + c) * H + gy) * W + gx, acc[(y * kTX + x) * CP + c]);
  }
}

template <typename T>
bool launch_build(const void* in, void* packed, int B, int C, int H, int W, int levels,
                  cudaStream_t s) {
  const PyrGeom g = make_geom(H, W, C, levels);
  constexpr int CC = 32;  // 40 KB of static shared memory per CTA
  const int tiles = ((H + kTY - 1) / kTY) * ((W + kTX - 1) / kTX);
  dim3 grid(tiles, (C + CC - 1) / CC, B);
  pyramid_build_kernel<T, CC><<<grid, 256, 0, s>>>((const T*)in, (T*)packed, C, H, W, g,
                                                   levels);
  count_launch();
  if (!check_launch("pyramid_build")) return false;
  for (int l = kFusedLevels; l < levels; ++l) {
    const long long n = (long long)g.h[l] * g.w[l] * C;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 4096);
    pool_level_kernel<T><<<dim3(blocks, B), 256, 0, s>>>((T*)packed, C, g, l);
    count_launch();
    if (!check_launch("pyramid_pool_level")) return false;
  }
  return true;
}

template <typename T, typename G>
bool launch_build_grad(const void* gp, void* out, int B, int C, int H, int W, int levels,
                       cudaStream_t s) {
  const PyrGeom g = make_geom(H, W, C, levels);
  constexpr int CC = 32;
  const int tiles = ((H + kTY - 1) / kTY) * ((W + kTX - 1) / kTX);
  dim3 grid(tiles, (C + CC - 1) / CC, B);
  pyramid_grad_kernel<T, G, CC><<<grid, 256, 0, s>>>((const G*)gp, (T*)out, C, H, W, g);
  count_launch();
  return check_launch("pyramid_build_grad");
}

}  // namespace

bool layout_nchw_to_nhwc(const void* in, void* out, int B, int C, int HW, int dtype,
                         cudaStream_t s) {
  return dtype == LCB200_F32 ? launch_transpose<float>(in, out, B, C, HW, s)
                             : launch_transpose<__half>(in, out, B, C, HW, s);
}

bool layout_nhwc_to_nchw(const void* in, void* out, int B, int C, int HW, int dtype,
                         cudaStream_t s) {
  return dtype == LCB200_F32 ? launch_transpose<float>(in, out, B, HW, C, s)
                             : launch_transpose<__half>(in, out, B, HW, C, s);
}

bool layout_pyramid_build(const void* in, void* packed, int B, int C, int H, int W,
                          int levels, int dtype, cudaStream_t s) {
  return dtype == LCB200_F32 ? launch_build<float>(in, packed, B, C, H, W, levels, s)
                             : launch_build<__half>(in, packed, B, C, H, W, levels, s);
}

bool layout_pyramid_build_grad(const void* gp, bool grad_is_f32, void* out, int B, int C,
                               int H, int W, int levels, int dtype, cudaStream_t s) {
  if (dtype == LCB200_F32)
    return launch_build_grad<float, float>(gp, out, B, C, H, W, levels, s);
  return grad_is_f32 ? launch_build_grad<__half, float>(gp, out, B, C, H, W, levels, s)
                     : launch_build_grad<__half, __half>(gp, out, B, C, H, W, levels, s);
}

}  // namespace lcb200
