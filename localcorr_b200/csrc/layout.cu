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

// float16 with even R and Ccols: 64x64 tiles, each thread moving half2
// pairs on both sides (4-byte accesses, 128 bytes per warp access).
__global__ void transpose_h2_kernel(const __half* __restrict__ in, __half* __restrict__ out,
                                    int R, int Ccols) {
  __shared__ __half tile[64][66];
  const long long bo = (long long)blockIdx.z * R * Ccols;
  const int c0 = blockIdx.x * 64, r0 = blockIdx.y * 64;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int i = ty; i < 64; i += 8) {
    const int rr = r0 + i, cc = c0 + 2 * tx;
    __half2 v = __floats2half2_rn(0.f, 0.f);
    if (rr < R && cc < Ccols) v = *reinterpret_cast<const __half2*>(in + bo + (long long)rr * Ccols + cc);
    tile[i][2 * tx] = __low2half(v);
    tile[i][2 * tx + 1] = __high2half(v);
  }
  __syncthreads();
  for (int i = ty; i < 64; i += 8) {
    const int cc = c0 + i, rr = r0 + 2 * tx;
    if (cc < Ccols && rr < R)
      *reinterpret_cast<__half2*>(out + bo + (long long)cc * R + rr) =
          __halves2half2(tile[2 * tx][i], tile[2 * tx + 1][i]);
  }
}

template <typename T>
bool launch_transpose(const void* in, void* out, int B, int R, int Ccols, cudaStream_t s) {
  if (std::is_same<T, __half>::value && R % 2 == 0 && Ccols % 2 == 0 &&
      ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 3) == 0) {
    dim3 grid((Ccols + 63) / 64, (R + 63) / 64, B);
    transpose_h2_kernel<<<grid, dim3(32, 8), 0, s>>>((const __half*)in, (__half*)out, R, Ccols);
    count_launch();
    return check_launch("transpose");
  }
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
// float16 pyramid build with half2 accesses: CTA = 8x32 level-0 tile x 64
// channels, levels kept in shared memory as float16 [y][x][64+2] (the stored
// values are the dtype-rounded level values that the next level pools). The
// NCHW tile is read as x pairs; every NHWC row of 64 channels (128 bytes) is
// written by one warp as channel pairs. Needs C % 64 == 0 and W even.
constexpr int kHC = 64, kHP = kHC + 2;
__global__ void __launch_bounds__(256)
pyramid_build_h_kernel(const __half* __restrict__ in, __half* __restrict__ packed, int C, int H,
                       int W, PyrGeom g, int nlev) {
  __shared__ __align__(16) __half s0[kTY * kTX * kHP];
  __shared__ __align__(16) __half s1[(kTY / 2) * (kTX / 2) * kHP];
  const int b = blockIdx.z;
  const int c0 = blockIdx.y * kHC;
  const int tiles_x = (W + kTX - 1) / kTX;
  const int ty0 = (blockIdx.x / tiles_x) * kTY;
  const int tx0 = (blockIdx.x % tiles_x) * kTX;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // NCHW tile: item = (c, y, x pair)
  for (int i = tid; i < kHC * kTY * (kTX / 2); i += 256) {
    const int xp = i % (kTX / 2), rest = i / (kTX / 2);
    const int y = rest % kTY, c = rest / kTY;
    const int gy = ty0 + y, gx = tx0 + 2 * xp;
    __half2 v = __floats2half2_rn(0.f, 0.f);
    if (gy < H && gx < W)
      v = *reinterpret_cast<const __half2*>(in + (((long long)b * C + c0 + c) * H + gy) * W + gx);
    s0[(y * kTX + 2 * xp) * kHP + c] = __low2half(v);
    s0[(y * kTX + 2 * xp + 1) * kHP + c] = __high2half(v);
  }
  __syncthreads();
  __half* pb = packed + (long long)b * g.batch_elems;
  // level 0: one position per warp step, lanes = channel pairs
  for (int p0 = warp; p0 < kTY * kTX; p0 += 8) {
    const int y = p0 / kTX, x = p0 % kTX;
    const int gy = ty0 + y, gx = tx0 + x;
    if (gy < H && gx < W)
      *reinterpret_cast<__half2*>(pb + g.off[0] + ((long long)gy * W + gx) * C + c0 + 2 * lane) =
          *reinterpret_cast<const __half2*>(s0 + p0 * kHP + 2 * lane);
  }
  __half* src = s0;
  __half* dst = s1;
  int sx = kTX, sy = kTY;
  for (int l = 1; l < nlev && l < kFusedLevels; ++l) {
    const int ny = sy / 2, nx = sx / 2;
    __syncthreads();
    for (int i = tid; i < ny * nx * (kHC / 2); i += 256) {
      const int cp = i % (kHC / 2), pp = i / (kHC / 2);
      const int y = pp / nx, x = pp % nx;
      const __half* q = src + ((2 * y) * sx + 2 * x) * kHP + 2 * cp;
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(q));
      const float2 bq = __half22float2(*reinterpret_cast<const __half2*>(q + kHP));
      const float2 cq = __half22float2(*reinterpret_cast<const __half2*>(q + sx * kHP));
      const float2 dq = __half22float2(*reinterpret_cast<const __half2*>(q + sx * kHP + kHP));
      float ax = a.x, ay = a.y;
      ax += bq.x; ay += bq.y;
      ax += cq.x; ay += cq.y;
      ax += dq.x; ay += dq.y;
      *reinterpret_cast<__half2*>(dst + pp * kHP + 2 * cp) = __floats2half2_rn(ax / 4.f, ay / 4.f);
    }
    __syncthreads();
    const int hl = g.h[l], wl = g.w[l];
    const int oy = ty0 >> l, ox = tx0 >> l;
    for (int pp = warp; pp < ny * nx; pp += 8) {
      const int y = pp / nx, x = pp % nx;
      const int gy = oy + y, gx = ox + x;
      if (gy < hl && gx < wl)
        *reinterpret_cast<__half2*>(pb + g.off[l] + ((long long)gy * wl + gx) * C + c0 + 2 * lane) =
            *reinterpret_cast<const __half2*>(dst + pp * kHP + 2 * lane);
    }
    __half* t = src; src = dst; dst = t;
    sy = ny; sx = nx;
  }
}

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

// Gradient of the pyramid build for float32 level gradients and a float16
// NCHW result (the path the block's autograd takes): CTA = 16x32 level-0
// tile x 32 channels. The coarse levels collapse first into the tile's
// level-1 footprint, c1 = g1 + (g2 + g3/4)/4 (16 KB of shared memory, 16-byte
// channel-quad loads), then out = g0 + c1/4 per level-0 pixel, staged as
// [channel][pixel] float16 and written along x in 8-byte pieces.
// Needs C % 32 == 0, W % 4 == 0 and at most 4 levels.
constexpr int kGY = 16, kGX = 32, kGC = 32;
constexpr int kGS = kGY * kGX + 4;  // staging row stride in halves (8-byte aligned rows)
constexpr size_t kGradSmem = (size_t)(kGY / 2) * (kGX / 2) * kGC * 4 + (size_t)kGC * kGS * 2;

__global__ void __launch_bounds__(256)
pyramid_grad_f32_kernel(const float* __restrict__ gp, __half* __restrict__ out, int C, int H,
                        int W, PyrGeom g) {
  extern __shared__ __align__(16) uint8_t gsm[];
  float4* c1 = reinterpret_cast<float4*>(gsm);  // [(kGY/2)*(kGX/2)][kGC/4]
  __half* st = reinterpret_cast<__half*>(gsm + (size_t)(kGY / 2) * (kGX / 2) * kGC * 4);
  const int b = blockIdx.z;
  const int c0 = blockIdx.y * kGC;
  const int tiles_x = (W + kGX - 1) / kGX;
  const int ty0 = (blockIdx.x / tiles_x) * kGY;
  const int tx0 = (blockIdx.x % tiles_x) * kGX;
  const float* gb = gp + (long long)b * g.batch_elems + c0;
  auto lvl = [&](int l, int y, int x, int cq) -> float4 {  // level-l quad, zero off the level
    if (l >= g.levels || y >= g.h[l] || x >= g.w[l]) return make_float4(0.f, 0.f, 0.f, 0.f);
    return *reinterpret_cast<const float4*>(gb + g.off[l] + ((long long)y * g.w[l] + x) * C +
                                            4 * cq);
  };
  const int tid = threadIdx.x;
  if (g.levels > 1) {
    for (int i = tid; i < (kGY / 2) * (kGX / 2) * (kGC / 4); i += 256) {
      const int cq = i % (kGC / 4), p1 = i / (kGC / 4);
      const int y1 = ty0 / 2 + p1 / (kGX / 2), x1 = tx0 / 2 + p1 % (kGX / 2);
      float4 v = lvl(1, y1, x1, cq);
      if (g.levels > 2) {
        float4 v2 = lvl(2, y1 >> 1, x1 >> 1, cq);
        if (g.levels > 3) {
          const float4 v3 = lvl(3, y1 >> 2, x1 >> 2, cq);
          v2.x += 0.25f * v3.x; v2.y += 0.25f * v3.y; v2.z += 0.25f * v3.z; v2.w += 0.25f * v3.w;
        }
        v.x += 0.25f * v2.x; v.y += 0.25f * v2.y; v.z += 0.25f * v2.z; v.w += 0.25f * v2.w;
      }
      c1[p1 * (kGC / 4) + cq] = v;
    }
    __syncthreads();
  }
  for (int i = tid; i < kGY * kGX * (kGC / 4); i += 256) {
    const int cq = i % (kGC / 4), p0 = i / (kGC / 4);
    const int y = p0 / kGX, x = p0 % kGX;
    const int gy = ty0 + y, gx = tx0 + x;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (gy < H && gx < W) {
      v = *reinterpret_cast<const float4*>(gb + ((long long)gy * W + gx) * C + 4 * cq);
      if (g.levels > 1) {
        const float4 u = c1[((y >> 1) * (kGX / 2) + (x >> 1)) * (kGC / 4) + cq];
        v.x += 0.25f * u.x; v.y += 0.25f * u.y; v.z += 0.25f * u.z; v.w += 0.25f * u.w;
      }
    }
    __half* d = st + (4 * cq) * kGS + p0;
    d[0] = __float2half_rn(v.x);
    d[kGS] = __float2half_rn(v.y);
    d[2 * kGS] = __float2half_rn(v.z);
    d[3 * kGS] = __float2half_rn(v.w);
  }
  __syncthreads();
  for (int i = tid; i < kGC * kGY * (kGX / 4); i += 256) {
    const int xq = i % (kGX / 4), rest = i / (kGX / 4);
    const int y = rest % kGY, c = rest / kGY;
    const int gy = ty0 + y, gx = tx0 + 4 * xq;
    if (gy >= H || gx >= W) continue;
    const __half* src = st + c * kGS + y * kGX + 4 * xq;
    __half* dst = out + (((long long)b * C + c0 + c) * H + gy) * W + gx;
    if (gx + 3 < W) {
      *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(src);
    } else {
      for (int e = 0; gx + e < W; ++e) dst[e] = src[e];
    }
  }
}

template <typename T>
bool launch_build(const void* in, void* packed, int B, int C, int H, int W, int levels,
                  cudaStream_t s) {
  const PyrGeom g = make_geom(H, W, C, levels);
  constexpr int CC = 32;  // 40 KB of static shared memory per CTA
  const int tiles = ((H + kTY - 1) / kTY) * ((W + kTX - 1) / kTX);
  if (std::is_same<T, __half>::value && C % kHC == 0 && W % 2 == 0 &&
      ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(packed)) & 3) == 0) {
    dim3 grid(tiles, C / kHC, B);
    pyramid_build_h_kernel<<<grid, 256, 0, s>>>((const __half*)in, (__half*)packed, C, H, W, g,
                                                levels);
  } else {
    dim3 grid(tiles, (C + CC - 1) / CC, B);
    pyramid_build_kernel<T, CC><<<grid, 256, 0, s>>>((const T*)in, (T*)packed, C, H, W, g,
                                                     levels);
  }
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
  if (std::is_same<T, __half>::value && std::is_same<G, float>::value && C % kGC == 0 &&
      W % 4 == 0 && levels <= 4 && (reinterpret_cast<uintptr_t>(gp) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(out) & 7) == 0) {
    if (!ensure_smem_attr((const void*)pyramid_grad_f32_kernel, kGradSmem)) return false;
    const int tiles = ((H + kGY - 1) / kGY) * ((W + kGX - 1) / kGX);
    dim3 grid(tiles, C / kGC, B);
    pyramid_grad_f32_kernel<<<grid, 256, kGradSmem, s>>>((const float*)gp, (__half*)out, C, H,
                                                         W, g);
    count_launch();
    return check_launch("pyramid_build_grad");
  }
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
