// Tensor-core (tcgen05 + TMA + TMEM) engine of the pyramid local correlation,
// float16 maps, dilation 1, up to 4 levels, 64 <= C <= 256 (C % 64 == 0).
//
// Why a sort: every pixel needs the dot products of its fmap1 row with the
// (2r+2)^2 fmap2 samples of its window, at every level. With arbitrary flow
// the windows of neighbouring source pixels need not overlap, so a tile of
// source pixels shares no fmap2 data and the work is a gather-GEMV. Bucketing
// the pixels by where their windows land makes the sharing explicit:
//
//  1. sort    pixels are counting-sorted into anchor cells of 8x16 level-0
//             base positions (floor of the level-0 coordinate). Cells are
//             aligned to multiples of 8 (y) and 16 (x), so the level-l bases
//             of a cell span (8>>l)x(16>>l) positions and the union of the
//             cell's windows at level l is a fixed (8>>l)+2r+1 by
//             (16>>l)+2r+1 box. Pixels whose windows miss the map at every
//             level are dropped (their outputs are exact zeros).
//  2. forward per chunk of <= 128 pixels of one cell: A = the chunk's fmap1
//             rows (M=128, K=C), B = each level's union box of fmap2 loaded
//             by TMA (N = union positions, K = C; out-of-map taps are the
//             TMA zero fill, which is the reference's zero padding).
//             tcgen05.mma accumulates S = A*B^T (fp32) in TMEM; TMEM lane m
//             holds pixel m's row, so the epilogue thread of pixel m reads
//             its window rows from TMEM and combines neighbouring grid
//             samples with its bilinear weights:
//               out(iy,ix) = wa*S[j][k] + wb*S[j][k+1] + wc*S[j+1][k] + wd*S[j+1][k+1]
//             which equals the reference's tap-by-tap bilinear dot product
//             (cuda_pyramid/localcorr_cuda_pyramid_kernel.cu:139-272) by
//             linearity. Outputs go to a scratch in sorted order.
//  3. unsort  scratch rows are written to [B, L, RD^2, H, W] (coalesced
//             along W), zeros for dropped pixels.
//
// Warp roles of the forward kernel (persistent, one CTA per SM):
//   warp 0      producer: TMA loads of the B boxes
//   warp 1      TMEM owner and MMA issuer (one thread)
//   warps 2..13 epilogue: three groups of four warps (TMEM lane quadrant =
//               warp % 4) that share out the rows of each part and stage
//               each level's outputs in shared memory
//   then        gather warps (cp.async of the A tile: the chunk's fmap1 rows)
//               and copier warps (staged outputs -> the sorted scratch, one
//               staging buffer behind the epilogue, so the epilogue never
//               waits for the copy while the other buffer is free)
// Every mbarrier wait is bounded (2 s); on timeout the kernel records an
// error status, all roles wind down, TMEM is freed and the kernel returns.
#include <cub/block/block_scan.cuh>
#include <cudaTypedefs.h>
#include <climits>

#include <mutex>
#include <string>

#include "lc_common.cuh"
#include "tc_ptx.cuh"

namespace lcb200 {

__device__ int g_tc_status = 0;

namespace {

constexpr int kCellY = 8, kCellX = 16, kTile = 128;
constexpr int kColBins = kCellX;  // sort bins per cell: the level-0 base column in the cell
// Work counters of the persistent kernels' dynamic schedulers: [0] grad_fmap2
// items; zeroed by the gradient-record kernel that precedes their user.
constexpr int kWorkCounters = 4;
constexpr int kMaxTcLevels = 4;
constexpr int kBwd1Threads = 64 + 256 + 128;  // grad_fmap1: producer, MMA, 2 x 4 builder warps, 4 epilogue warps
constexpr int kFwdEG = 3;          // forward epilogue warp groups
// forward fmap1 row gather (A tile): 4 warps, 1 at radius 8, whose
// epilogue needs the registers of a block of at most 512 threads
constexpr int fwd_gather_warps(int radius) { return radius > 4 ? 1 : 4; }
// staged-output copier warps
constexpr int fwd_copy_warps(int radius) { return radius > 4 ? 1 : 2; }
constexpr int fwd_threads(int radius) {
  return 64 + 128 * kFwdEG + 32 * (fwd_gather_warps(radius) + fwd_copy_warps(radius));
}

// out[i] = v[rx + i] for rx in [0, 2^SD), a select network of SD stages on
// the bits of rx (no dynamic register indexing).
template <int NW, int NV, int SD>
struct WindowSelect {
  static_assert(NV >= NW + (1 << SD) - 1, "window source too short");
  __device__ __forceinline__ static void run(const float* v, int rx, float (&out)[NW]) {
    constexpr int H = 1 << (SD - 1);
    float t[NW + H - 1];
#pragma unroll
    for (int i = 0; i < NW + H - 1; ++i) t[i] = (rx & H) ? v[i + H] : v[i];
    WindowSelect<NW, NW + H - 1, SD - 1>::run(t, rx, out);
  }
};
template <int NW, int NV>
struct WindowSelect<NW, NV, 0> {
  __device__ __forceinline__ static void run(const float* v, int, float (&out)[NW]) {
#pragma unroll
    for (int i = 0; i < NW; ++i) out[i] = v[i];
  }
};

// TMEM columns a forward window row is read in: the least of 16, 32, 64
// holding the window (2r+2) plus the anchor offsets within a level-l cell
// column span (16 >> l).
__host__ __device__ constexpr int fwd_row_cols(int radius, int l) {
  return (2 * radius + 2) + (kCellX >> l) - 1 <= 16 ? 16
         : (2 * radius + 2) + (kCellX >> l) - 1 <= 32 ? 32 : 64;
}
__host__ __device__ constexpr int fwd_select_depth(int l) { return 4 - l; }

struct TcGeom {
  int B, H, W, C, r, L, RD, RD2, RDP, KC, HW;
  int ylo, xlo, yhi, xhi, ncy, ncx, ncell;
  int h[kMaxTcLevels], w[kMaxTcLevels];
  long long off[kMaxTcLevels];
  long long batch_elems;
  int UH[kMaxTcLevels], UW[kMaxTcLevels], R[kMaxTcLevels], nparts[kMaxTcLevels],
      npad[kMaxTcLevels];
  int maxN, nld, RS;
  long long npix;  // B*HW
  // backward: integer-grid weights per pixel/level ((RD+1)^2, padded), the
  // union row groups of <= 64 positions (grad_fmap1 K chunks), and the
  // output-tile work decomposition of grad_fmap2
  int NG;
  int NU;  // 16-byte units of one pre-shifted grid row (grad_fmap2 records)
  int UWb[kMaxTcLevels];  // grad_fmap1 box width: 8-aligned origin, multiple of 8
  int Rg[kMaxTcLevels], ngroups[kMaxTcLevels];
  int nqy[kMaxTcLevels], nqx[kMaxTcLevels], rpi[kMaxTcLevels], qgroups[kMaxTcLevels];
  long long items_before[kMaxTcLevels + 1];  // grad_fmap2 items of one image, coarse levels first
};

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline int round_up(int a, int b) { return ceil_div(a, b) * b; }

bool make_tc_geom(int B, int H, int W, int H2, int W2, int C, int r, int L, TcGeom* g,
                  std::string* why) {
  TcGeom t{};
  t.B = B; t.H = H; t.W = W; t.C = C; t.r = r; t.L = L;
  t.RD = 2 * r + 1;
  t.RD2 = t.RD * t.RD;
  t.RDP = round_up(t.RD2, 8);
  t.KC = C / 64;
  t.HW = H * W;
  t.npix = (long long)B * H * W;
  const int s = 1 << (L - 1);
  // Bases outside [lo, hi) have windows outside the map at every level.
  t.ylo = -round_up((r + 2) * s, kCellY);
  t.xlo = -round_up((r + 2) * s, kCellX);
  t.yhi = H2 + (r + 1) * s;
  t.xhi = W2 + (r + 1) * s;
  t.ncy = ceil_div(t.yhi - t.ylo, kCellY);
  t.ncx = ceil_div(t.xhi - t.xlo, kCellX);
  t.ncell = t.ncy * t.ncx;
  long long acc = 0;
  for (int l = 0; l < L; ++l) {
    t.h[l] = H2 >> l;
    t.w[l] = W2 >> l;
    t.off[l] = acc;
    acc += (long long)C * t.h[l] * t.w[l];
  }
  t.batch_elems = acc;
  t.UW[0] = kCellX + 2 * r + 1;
  t.nld = ceil_div(t.UW[0], 32);
  t.RS = 32 * t.nld + 4;
  t.maxN = 0;
  for (int l = 0; l < L; ++l) {
    t.UH[l] = (kCellY >> l) + 2 * r + 1;
    t.UW[l] = (kCellX >> l) + 2 * r + 1;
    // Rows per part: the part must fit one 256-column TMEM buffer, including
    // the 32*nld-column window read of its last row.
    const int rmax = std::min(256 / t.UW[l], (256 - 32 * t.nld) / t.UW[l] + 1);
    if (rmax < 2) {
      if (why) *why = "union rows too wide for a TMEM buffer";
      return false;
    }
    int np = std::max(1, ceil_div(t.UH[l] - 1, rmax - 1));
    int R = ceil_div(t.UH[l] - 1, np) + 1;
    if (R > t.UH[l]) R = t.UH[l];
    t.nparts[l] = np;
    t.R[l] = R;
    t.npad[l] = round_up(R * t.UW[l], 16);
    t.maxN = std::max(t.maxN, t.npad[l]);
  }
  t.NG = t.RD + 1;
  t.NU = ceil_div(t.NG + 7, 8);
  for (int l = 0; l < L; ++l) {
    // grad_fmap1 boxes start at the 8-aligned column at or left of the union
    // origin (cell_x0 >> l) - r, so that record units (8-aligned positions)
    // land on whole 16-byte units of the box rows.
    int shift = 0;
    for (int m = 0; m < 8; ++m) {
      const int x0 = ((t.xlo + m * kCellX) >> l) - r;
      shift = std::max(shift, x0 - (x0 & ~7));
    }
    t.UWb[l] = round_up(t.UW[l] + shift, 8);
    if (t.UWb[l] > 64) {
      if (why) *why = "union rows wider than 64 positions";
      return false;
    }
    t.Rg[l] = 64 / t.UWb[l];
    t.ngroups[l] = ceil_div(t.UH[l], t.Rg[l]);
    // grad_fmap2 tiles of 8x16 level-l positions; a tile pulls the pixels of
    // the anchor cells whose level-l windows can reach it, split into items
    // of rpi cell rows.
    t.nqy[l] = ceil_div(t.h[l], 8);
    t.nqx[l] = ceil_div(t.w[l], 16);
    const int span_y = (8 + 2 * r + 1) << l;   // level-0 rows of bases that can touch a tile
    const int span_x = (16 + 2 * r + 1) << l;
    const int rows = span_y / kCellY + 2;
    const int cols = span_x / kCellX + 2;
    // Deterministic mode: one item per tile (all its cell rows), so every
    // position gets exactly one add per call.
    t.rpi[l] = deterministic_mode() ? rows : std::max(1, 16 / cols);
    t.qgroups[l] = ceil_div(rows, t.rpi[l]);
  }
  t.items_before[0] = 0;
  for (int i = 0; i < L; ++i) {
    const int l = L - 1 - i;  // coarse levels first (longest items first)
    t.items_before[i + 1] =
        t.items_before[i] + (long long)t.nqy[l] * t.nqx[l] * t.qgroups[l];
  }
  *g = t;
  return true;
}

struct alignas(64) TcFwdParams {
  CUtensorMap tmap[kMaxTcLevels];
  const __half* fmap1;
  const void* coords;
  const int* sorted;
  const int4* work;
  const int* work_count;
  __half* scratch;
  float scale;
  int coords_f32;
  int ymajor;
  int nstage;
  int nsb;  // output staging buffers (1 or 2)
  uint32_t stage_bytes;
  TcGeom g;
};

// ---------------------------------------------------------------------------
// sort: histogram -> scan (+ work list) -> scatter
// ---------------------------------------------------------------------------
// Sort bin of pixel gid and its rank in the bin (atomic count), or key -1
// when its windows miss every level.
template <typename TC>
__device__ __forceinline__ void hist_pixel(const TC* __restrict__ coords, int* __restrict__ counts,
                                           int2* __restrict__ keyrank, const TcGeom& g,
                                           long long gid) {
  const int b = (int)(gid / g.HW);
  const int p = (int)(gid - (long long)b * g.HW);
  const float cx = ldf(coords + (long long)b * 2 * g.HW + p);
  const float cy = ldf(coords + (long long)b * 2 * g.HW + g.HW + p);
  const float fx = floorf(cx), fy = floorf(cy);
  int2 kr = make_int2(-1, 0);
  if (fx >= (float)g.xlo && fx < (float)g.xhi && fy >= (float)g.ylo && fy < (float)g.yhi) {
    const int bx = (int)fx, by = (int)fy;
    const int cell = ((by - g.ylo) / kCellY) * g.ncx + (bx - g.xlo) / kCellX;
    const int key = cell * kColBins + (bx - g.xlo) % kCellX;  // (cell, column in cell)
    if (LCB_IN(key >= 0 && key < g.ncell * kColBins, kSiteTcHist, key)) {
      kr.x = key;
      kr.y = atomicAdd(counts + (long long)b * g.ncell * kColBins + key, 1);
    }
  }
  keyrank[gid] = kr;
}

template <typename TC>
__global__ void tc_hist_kernel(const TC* __restrict__ coords, int* __restrict__ counts,
                               int2* __restrict__ keyrank, TcGeom g) {
  const long long gid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (gid < g.npix) hist_pixel(coords, counts, keyrank, g, gid);
}

// Scan of the sort bins, three passes over the cells (all blocks busy
// instead of one): per-cell totals (pixels; 128-pixel chunks = work
// entries) scanned within blocks of kScanBlock cells, the block totals
// scanned, then every (cell, column) bin offset into the sorted order (bins
// in order, so a cell's pixels are sorted by their base column), a final
// entry = number of sorted pixels, and the work list
// {b, cell, first sorted index, pixel count <= 128}.
constexpr int kScanBlock = 256;
struct PairSum {
  __device__ int2 operator()(int2 a, int2 b) const { return make_int2(a.x + b.x, a.y + b.y); }
};

template <bool L2 = false>
__device__ __forceinline__ void load_cell_bins(const int* __restrict__ counts, int i,
                                               int (&bins)[kColBins]) {
  const int4* src = reinterpret_cast<const int4*>(counts + (long long)i * kColBins);
#pragma unroll
  for (int q = 0; q < kColBins / 4; ++q) {
    const int4 v = L2 ? __ldcg(src + q) : src[q];
    bins[4 * q] = v.x; bins[4 * q + 1] = v.y; bins[4 * q + 2] = v.z; bins[4 * q + 3] = v.w;
  }
}

__global__ void __launch_bounds__(kScanBlock)
tc_cellscan_kernel(const int* __restrict__ counts, int2* __restrict__ cellpre,
                   int2* __restrict__ bsum, int ncell_total) {
  using Scan = cub::BlockScan<int2, kScanBlock>;
  __shared__ typename Scan::TempStorage tmp;
  const int i = blockIdx.x * kScanBlock + threadIdx.x;
  int cnt = 0;
  if (i < ncell_total) {
    int bins[kColBins];
    load_cell_bins(counts, i, bins);
#pragma unroll
    for (int q = 0; q < kColBins; ++q) cnt += bins[q];
  }
  int2 ex, tot;
  Scan(tmp).ExclusiveScan(make_int2(cnt, (cnt + kTile - 1) / kTile), ex, make_int2(0, 0),
                          PairSum(), tot);
  if (i < ncell_total) cellpre[i] = ex;
  if (threadIdx.x == 0) bsum[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(1024)
tc_blockscan_kernel(int2* __restrict__ bsum, int nblocks, int* __restrict__ total,
                    int* __restrict__ work_count) {
  using Scan = cub::BlockScan<int2, 1024>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ int2 carry;
  if (threadIdx.x == 0) carry = make_int2(0, 0);
  __syncthreads();
  for (int base = 0; base < nblocks; base += 1024) {
    const int i = base + threadIdx.x;
    const int2 v = i < nblocks ? bsum[i] : make_int2(0, 0);
    int2 ex, tot;
    Scan(tmp).ExclusiveScan(v, ex, make_int2(0, 0), PairSum(), tot);
    const int2 c = carry;
    if (i < nblocks) bsum[i] = make_int2(c.x + ex.x, c.y + ex.y);
    __syncthreads();
    if (threadIdx.x == 0) carry = make_int2(c.x + tot.x, c.y + tot.y);
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    *total = carry.x;
    *work_count = carry.y;
  }
}

__global__ void __launch_bounds__(kScanBlock)
tc_cellwrite_kernel(const int* __restrict__ counts, const int2* __restrict__ cellpre,
                    const int2* __restrict__ bsum, int* __restrict__ offsets,
                    int4* __restrict__ work, int ncell_total, int ncell) {
  const int i = blockIdx.x * kScanBlock + threadIdx.x;
  if (i >= ncell_total) return;
  int bins[kColBins];
  load_cell_bins(counts, i, bins);
  const int2 pre = cellpre[i], bo = bsum[blockIdx.x];
  const int off = bo.x + pre.x, coff = bo.y + pre.y;
  int acc = off;
  int4* dst = reinterpret_cast<int4*>(offsets + (long long)i * kColBins);
#pragma unroll
  for (int q = 0; q < kColBins / 4; ++q) {
    int4 v;
    v.x = acc; acc += bins[4 * q];
    v.y = acc; acc += bins[4 * q + 1];
    v.z = acc; acc += bins[4 * q + 2];
    v.w = acc; acc += bins[4 * q + 3];
    dst[q] = v;
  }
  const int cnt = acc - off;
  const int nch = (cnt + kTile - 1) / kTile;
  const int b = i / ncell;
  const int cell = i - b * ncell;
  for (int j = 0; j < nch; ++j)
    work[coff + j] = make_int4(b, cell, off + j * kTile, min(kTile, cnt - j * kTile));
}

// Small problems (one or two images): the histogram and the whole scan in
// one launch. Blocks of 1024 threads count their pixels; the last block to
// finish (a ticket counter after a fence, no waiting) scans all the bins,
// up to kSmallScanCpt cells per thread, where the three-pass form's
// launches would cost more than the scan itself.
constexpr int kSmallScanCpt = 4;
template <typename TC>
__global__ void __launch_bounds__(1024)
tc_hist_scan_kernel(const TC* __restrict__ coords, int* __restrict__ counts,
                    int2* __restrict__ keyrank, int* __restrict__ done,
                    int* __restrict__ offsets, int4* __restrict__ work, int* __restrict__ total,
                    int* __restrict__ work_count, TcGeom g) {
  using Scan = cub::BlockScan<int2, 1024>;
  __shared__ typename Scan::TempStorage tmp;
  __shared__ int is_last;
  const long long gid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (gid < g.npix) hist_pixel(coords, counts, keyrank, g, gid);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();  // this block's counts before its ticket
    is_last = atomicAdd(done, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();  // every block's counts (read from L2 below)
  const int ncell_total = g.B * g.ncell;
  const int ncell = g.ncell;
  // consecutive cells per thread: as few as the cell count allows (one
  // cell per thread up to 1024 cells: whole 64-byte bin rows per lane)
  const int cpt = (ncell_total + 1023) / 1024;
  const int c0 = threadIdx.x * cpt;
  int2 mine = make_int2(0, 0);
#pragma unroll
  for (int k = 0; k < kSmallScanCpt; ++k) {
    const int i = c0 + k;
    if (k < cpt && i < ncell_total) {
      int bins[kColBins];
      load_cell_bins<true>(counts, i, bins);
      int cnt = 0;
#pragma unroll
      for (int q = 0; q < kColBins; ++q) cnt += bins[q];
      mine.x += cnt;
      mine.y += (cnt + kTile - 1) / kTile;
    }
  }
  int2 ex, tot;
  Scan(tmp).ExclusiveScan(mine, ex, make_int2(0, 0), PairSum(), tot);
  int acc = ex.x, coff = ex.y;
  for (int k = 0; k < cpt; ++k) {
    const int i = c0 + k;
    if (i >= ncell_total) break;
    int bins[kColBins];
    load_cell_bins<true>(counts, i, bins);
    const int off = acc;
    int4* dst = reinterpret_cast<int4*>(offsets + (long long)i * kColBins);
#pragma unroll
    for (int q = 0; q < kColBins / 4; ++q) {
      int4 v;
      v.x = acc; acc += bins[4 * q];
      v.y = acc; acc += bins[4 * q + 1];
      v.z = acc; acc += bins[4 * q + 2];
      v.w = acc; acc += bins[4 * q + 3];
      dst[q] = v;
    }
    const int cnt = acc - off;
    const int nch = (cnt + kTile - 1) / kTile;
    const int b = i / ncell;
    const int cell = i - b * ncell;
    for (int j = 0; j < nch; ++j)
      work[coff + j] = make_int4(b, cell, off + j * kTile, min(kTile, cnt - j * kTile));
    coff += nch;
  }
  if (threadIdx.x == 0) {
    *total = tot.x;
    *work_count = tot.y;
  }
}

__global__ void tc_scatter_kernel(const int2* __restrict__ keyrank, const int* __restrict__ offsets,
                                  int* __restrict__ sorted, int* __restrict__ inv, TcGeom g) {
  const long long gid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (gid >= g.npix) return;
  const int2 kr = keyrank[gid];
  if (kr.x < 0) {
    inv[gid] = -1;
    return;
  }
  const int b = (int)(gid / g.HW);
  const int pos = offsets[(long long)b * g.ncell * kColBins + kr.x] + kr.y;
  if (!LCB_IN(pos >= 0 && pos < g.npix, kSiteTcScatter, pos)) return;
  sorted[pos] = (int)gid;
  inv[gid] = pos;
}

// Deterministic order within the sort bins. The histogram's ranks come from
// atomics, so a bin's pixels land in thread-timing order; this pass gives
// each pixel of a bin the rank = number of the bin's pixels with a smaller
// index (one warp per bin, bins of any size), and the scatter then runs
// again with those ranks.
__global__ void tc_rank_fix_kernel(const int* __restrict__ offsets, const int* __restrict__ sorted,
                                   int2* __restrict__ keyrank, long long nbins, long long npix) {
  const long long bin = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (bin >= nbins) return;  // warp-uniform
  const int s0 = offsets[bin];
  const int n = offsets[bin + 1] - s0;
  if (n < 2) return;
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int mine = i0 + lane < n ? sorted[s0 + i0 + lane] : INT_MAX;
    int rank = 0;
    for (int j0 = 0; j0 < n; j0 += 32) {
      const int other = j0 + lane < n ? sorted[s0 + j0 + lane] : INT_MAX;
#pragma unroll 8
      for (int m = 0; m < 32; ++m) rank += __shfl_sync(0xffffffffu, other, m) < mine;
    }
    if (i0 + lane < n && LCB_IN(mine >= 0 && mine < npix, kSiteTcRankFix, mine))
      keyrank[mine].y = rank;
  }
}

// Sorted copy of fmap1 for the grad_fmap2 pull: row i = fmap1 row sorted[i]
// for the sorted pixels, zeros for the rows past them (their A rows are zero
// but the TMA tiles read them). One warp per kGatherRows rows, whose loads
// are all issued before the stores.
constexpr int kGatherRows = 4;
__global__ void tc_gather_rows_kernel(const __half* __restrict__ fmap1, const int* __restrict__ sorted,
                                      const int* __restrict__ nsorted, __half* __restrict__ f1s,
                                      TcGeom g) {
  const long long row0 =
      ((long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5)) * kGatherRows;
  const int lane = threadIdx.x & 31;
  const int ns = *nsorted;
  const int units = g.C / 8;  // 16-byte units per row (<= 32)
  if (lane >= units) return;
  uint4 v[kGatherRows];
#pragma unroll
  for (int k = 0; k < kGatherRows; ++k) {
    const long long row = row0 + k;
    v[k] = make_uint4(0, 0, 0, 0);
    if (row < ns) {
      const int src = sorted[row];
      if (LCB_IN(src >= 0 && src < g.npix, kSiteTcGather, src))
        v[k] = reinterpret_cast<const uint4*>(fmap1 + (long long)src * g.C)[lane];
    }
  }
#pragma unroll
  for (int k = 0; k < kGatherRows; ++k) {
    const long long row = row0 + k;
    if (row < g.npix) reinterpret_cast<uint4*>(f1s + row * g.C)[lane] = v[k];
  }
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
// One epilogue pass over union rows [ua, ub] of a forward part, level l
// (select depth and TMEM read width fixed per level): the window rows of this
// lane's pixel are picked out of each union row, bilinearly combined with the
// previous one and the RD outputs of window row iy staged in orow.
template <int RADIUS, int LVL>
__device__ __forceinline__ void fwd_part_rows(uint32_t taddr, int UW, int U0, int ua, int ub,
                                              int ry, int rx, bool valid, float wa, float wb,
                                              float wc, float wd, bool ymajor, __half* orow) {
  constexpr int RD = 2 * RADIUS + 1;
  constexpr int NW = RD + 1;
  constexpr int NC = fwd_row_cols(RADIUS, LVL);
  float prev[NW];
#pragma unroll
  for (int k2 = 0; k2 < NW; ++k2) prev[k2] = 0.f;
  for (int u = ua; u <= ub; ++u) {
    float v[NC];
    if constexpr (NC == 16) {
      tc::tmem_ld16(taddr + u * UW, *reinterpret_cast<float(*)[16]>(v));
    } else {
#pragma unroll
      for (int c = 0; c < NC / 32; ++c)
        tc::tmem_ld32(taddr + u * UW + 32 * c, *reinterpret_cast<float(*)[32]>(v + 32 * c));
    }
    tc::tmem_ld_wait();
    const int j = U0 + u - ry;  // window row of this grid row
    if (valid && j >= 0 && j <= RD) {
      float cur[NW];
      WindowSelect<NW, NC, fwd_select_depth(LVL)>::run(v, rx, cur);
      if (u > ua && j >= 1) {
        const int iy = j - 1;
        const int dbase = ymajor ? RD * iy : iy;
        const int dstep = ymajor ? 1 : RD;
#pragma unroll
        for (int ix = 0; ix < RD; ++ix) {
          const float val = wa * prev[ix] + wb * prev[ix + 1] + wc * cur[ix] + wd * cur[ix + 1];
          orow[dbase + dstep * ix] = __float2half_rn(val);
        }
      }
#pragma unroll
      for (int k2 = 0; k2 < NW; ++k2) prev[k2] = cur[k2];
    }
  }
}

template <int RADIUS>
__global__ void __launch_bounds__(fwd_threads(RADIUS), 1) tc_fwd_kernel(const __grid_constant__ TcFwdParams p) {
  constexpr int GW = fwd_gather_warps(RADIUS);
  constexpr int GROWS = kTile / GW / 4;  // 4-row copy groups per gather warp
  extern __shared__ uint8_t smem_raw[];
  __shared__ int abort_flag;
  const TcGeom& g = p.g;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + g.KC * 16384;
  constexpr int NCW = fwd_copy_warps(RADIUS);
  const int NST = p.nstage;
  const int NSB = p.nsb;
  const int RDPS = g.RDP / 2 + 1;  // smem output row stride in 32-bit words (odd)
  const int stage_words = kTile * RDPS;
  uint32_t* sOut = reinterpret_cast<uint32_t*>(sB + (size_t)NST * p.stage_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + NSB * stage_words);
  uint64_t* full = bars;
  uint64_t* empty = bars + NST;
  uint64_t* a_full = bars + 2 * NST;
  uint64_t* a_empty = a_full + 1;
  uint64_t* t_full = a_full + 2;   // [2]
  uint64_t* t_empty = a_full + 4;  // [2]
  uint64_t* s_full = a_full + 6;   // [2] a level's outputs are staged
  uint64_t* s_empty = a_full + 8;  // [2] a staging buffer has been copied out
  uint64_t* fin_bar = a_full + 10; // all MMAs of this CTA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(a_full + 11);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) { tc::mbar_init(full + s, 1); tc::mbar_init(empty + s, 1); }
    tc::mbar_init(a_full, 32 * GW);
    tc::mbar_init(a_empty, 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(t_full + i, 1);
      tc::mbar_init(t_empty + i, kTile * kFwdEG);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(s_full + i, kTile * kFwdEG);
      tc::mbar_init(s_empty + i, 32 * NCW);
    }
    tc::mbar_init(fin_bar, 1);
    tc::fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nwork = *p.work_count;
  volatile int* abort = &abort_flag;

  if (warp >= 2 + 4 * kFwdEG + GW) {
    // ---------------- copier: staged level outputs -> sorted scratch ----------------
    // Walks the same chunks and levels as the epilogue; staging buffer
    // (chunk-level index) % NSB. The scratch rows are contiguous, so the
    // copy is a flat run of 16-byte units (a row of RDP halves holds UPR of
    // them); each thread loads four units' words from shared memory before
    // storing them.
    const int ct = threadIdx.x - (64 + 128 * kFwdEG + 32 * GW);
    constexpr int NCT = 32 * NCW;
    constexpr int RDP = ((2 * RADIUS + 1) * (2 * RADIUS + 1) + 7) / 8 * 8;
    constexpr int UPR = RDP / 8;  // 16-byte units per scratch row
    uint32_t li = 0;
    bool ok = true;
    for (int wi = blockIdx.x; wi < nwork && ok; wi += gridDim.x) {
      const int4 wk = p.work[wi];
      const int start = wk.z, n = wk.w;
      for (int l = 0; l < g.L; ++l, ++li) {
        const int sbuf = (int)(li % (uint32_t)NSB);
        const uint32_t suse = li / (uint32_t)NSB;
        if (!tc::mbar_wait(s_full + sbuf, suse & 1, abort)) { ok = false; break; }
        const uint32_t* src = sOut + sbuf * stage_words;
        uint4* dst = reinterpret_cast<uint4*>(p.scratch + ((long long)l * g.npix + start) * RDP);
        const int nunits =
            LCB_IN(start >= 0 && n >= 0 && start + n <= g.npix, kSiteTcFwdWork, start) ? n * UPR : 0;
        for (int u0 = ct; u0 < nunits; u0 += 4 * NCT) {
          uint4 v[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int u = u0 + k * NCT;
            if (u < nunits) {
              const int row = u / UPR;
              const uint32_t* sp = src + row * RDPS + (u - row * UPR) * 4;
              v[k] = make_uint4(sp[0], sp[1], sp[2], sp[3]);
            }
          }
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (u0 + k * NCT < nunits) dst[u0 + k * NCT] = v[k];
        }
        tc::mbar_arrive(s_empty + sbuf);
      }
    }
  } else if (warp >= 2 + 4 * kFwdEG) {
    // ---------------- A tile: the chunk's fmap1 rows ----------------
    // 128 rows x C fp16, K-major SWIZZLE_128B, 64-channel slabs. Warp gw
    // owns rows [gw * 128 / GW, (gw + 1) * 128 / GW); one copy instruction covers 4 rows x
    // 128 contiguous bytes (8 lanes per row), so every request is whole
    // 32-byte sectors. The chunk's pixel ids are loaded before the wait for
    // the previous chunk's MMAs, and the B tiles of the chunk are requested
    // by the TMA warp independently of this gather.
    const int gw = warp - (2 + 4 * kFwdEG);
    const int sub = lane & 7, rr = lane >> 3;
    int it = 0;
    for (int wi = blockIdx.x; wi < nwork; wi += gridDim.x, ++it) {
      const int4 wk = p.work[wi];
      const int start = wk.z, n = wk.w;
      int rid[GROWS];
#pragma unroll
      for (int i = 0; i < GROWS; ++i) {
        const int t = gw * 4 * GROWS + 4 * i + rr;
        rid[i] = t < n ? p.sorted[start + t] : -1;
        if (!LCB_IN(rid[i] >= -1 && rid[i] < g.npix, kSiteTcFwdRow, rid[i])) rid[i] = -1;
      }
      // Bring the rows into L2 while the previous chunk's MMAs still need
      // the A tile (lanes 0..3 of a row: one 128-byte line per 64 channels).
#pragma unroll
      for (int i = 0; i < GROWS; ++i)
        if (rid[i] >= 0 && sub < g.KC)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(p.fmap1 + (long long)rid[i] * g.C + sub * 64));
      if (!tc::mbar_wait(a_empty, (it & 1) ^ 1, abort)) break;
      for (int kc = 0; kc < g.KC; ++kc) {
#pragma unroll
        for (int i = 0; i < GROWS; ++i) {
          const int t = gw * 4 * GROWS + 4 * i + rr;
          uint8_t* dst = sA + kc * 16384 + t * 128 + ((sub ^ (t & 7)) << 4);
          if (rid[i] >= 0)
            tc::cp_async_16(dst, p.fmap1 + (long long)rid[i] * g.C + kc * 64 + sub * 8, 16);
          else
            tc::cp_async_16(dst, p.fmap1, 0);
        }
      }
      tc::cp_async_mbar_arrive_noinc(a_full);
    }
    // Copies still in flight complete before the kernel's final barrier.
    tc::cp_async_wait_all();
  } else if (warp == 0) {
    // ---------------- B tiles (TMA) ----------------
    uint32_t gs = 0;
    for (int wi = blockIdx.x; wi < nwork; wi += gridDim.x) {
      const int4 wk = p.work[wi];
      const int b = wk.x, cell = wk.y;
      const int cy = cell / g.ncx, cx = cell - cy * g.ncx;
      const int cell_y0 = g.ylo + cy * kCellY, cell_x0 = g.xlo + cx * kCellX;
      bool ok = true;
      for (int l = 0; l < g.L && ok; ++l) {
        const int X0 = (cell_x0 >> l) - RADIUS;
        const int Y0 = (cell_y0 >> l) - RADIUS;
        const uint32_t box = 128u * g.UW[l] * g.R[l];
        for (int k = 0; k < g.nparts[l] && ok; ++k) {
          for (int kc = 0; kc < g.KC; ++kc, ++gs) {
            const int s = gs % NST;
            const uint32_t use = gs / NST;
            if (lane == 0) {
              if (!tc::mbar_wait(empty + s, (use & 1) ^ 1, abort)) { ok = false; }
              else {
                tc::mbar_arrive_expect_tx(full + s, box);
                tc::tma_load_4d(sB + (size_t)s * p.stage_bytes, &p.tmap[l], full + s, kc * 64,
                                X0, Y0 + k * (g.R[l] - 1), b);
              }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
          }
        }
      }
      if (!ok) break;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t pc = 0;
      int s = 0;          // B stage ring position and its fill phase
      uint32_t ph = 0;
      int it = 0;
      // descriptors: A slab kc at +kc*16 KB, B stage s at +s*stage_bytes
      // (start-address units of 16 bytes), K steps of 32 bytes (+2)
      const uint64_t a_desc0 = tc::smem_desc_sw128(tc::smem_u32(sA), 16, 1024);
      const uint64_t b_desc0 = tc::smem_desc_sw128(tc::smem_u32(sB), 16, 1024);
      const uint32_t b_stage_units = p.stage_bytes >> 4;
      bool ok = true;
      for (int wi = blockIdx.x; wi < nwork && ok; wi += gridDim.x, ++it) {
        if (!tc::mbar_wait(a_full, it & 1, abort)) break;
        // A rows arrive through cp.async completion: make their
        // shared-memory writes visible to the tensor core's proxy.
        tc::fence_proxy_async_smem();
        tc::tc_fence_after();
        for (int l = 0; l < g.L && ok; ++l) {
          const uint32_t idesc = tc::idesc_f16_f32(128, g.npad[l], false, false);
          for (int k = 0; k < g.nparts[l] && ok; ++k, ++pc) {
            const int buf = pc & 1;
            if (!tc::mbar_wait(t_empty + buf, ((pc >> 1) & 1) ^ 1, abort)) { ok = false; break; }
            tc::tc_fence_after();
            const uint32_t d = tmem + buf * 256;
            for (int kc = 0; kc < g.KC; ++kc) {
              const int cs = s;
              const uint32_t cph = ph;
              if (++s == NST) { s = 0; ph ^= 1; }
              const uint64_t ad = a_desc0 + (uint64_t)(kc * 1024);
              const uint64_t bd = b_desc0 + (uint64_t)(cs * b_stage_units);
              if (!tc::mbar_wait(full + cs, cph, abort)) { ok = false; break; }
              tc::tc_fence_after();
              tc::mma_f16_ss_n(d, ad, 2, bd, 2, idesc, kc != 0, 4);
              tc::mma_commit(empty + cs);
            }
            if (!ok) break;
            tc::mma_commit(t_full + buf);
          }
        }
        if (ok) tc::mma_commit(a_empty);
      }
      // Drain: TMEM is freed only after every issued MMA has completed.
      tc::mma_commit(fin_bar);
      tc::mbar_wait(fin_bar, 0, abort);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue ----------------
    // kFwdEG groups of 4 warps; each group covers all 128 TMEM lanes (warp %
    // 4 = lane quadrant) and takes a contiguous slice of every part's union
    // rows, overlapping the next slice by one row (a slice's first row only
    // seeds the bilinear pair), so the output rows are split without overlap.
    const int q = warp & 3;               // TMEM lane quadrant of this warp
    const int ge = (warp - 2) >> 2;       // epilogue group
    const int t = q * 32 + lane;          // tile row = pixel slot
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
    uint32_t pc = 0, li = 0;
    bool ok = true;
    for (int wi = blockIdx.x; wi < nwork && ok; wi += gridDim.x) {
      const int4 wk = p.work[wi];
      const int b = wk.x, cell = wk.y, start = wk.z, n = wk.w;
      const bool valid = t < n;
      float cx = 0.f, cy = 0.f;
      if (valid) {
        const int gid = p.sorted[start + t];
        int pix = gid - b * g.HW;
        if (!LCB_IN(pix >= 0 && pix < g.HW, kSiteTcFwdRow, gid)) pix = 0;
        if (p.coords_f32) {
          const float* co = reinterpret_cast<const float*>(p.coords) + (long long)b * 2 * g.HW + pix;
          cx = co[0]; cy = co[g.HW];
        } else {
          const __half* co = reinterpret_cast<const __half*>(p.coords) + (long long)b * 2 * g.HW + pix;
          cx = __half2float(co[0]); cy = __half2float(co[g.HW]);
        }
      }
      const int ccy = cell / g.ncx, ccx = cell - ccy * g.ncx;
      const int cell_y0 = g.ylo + ccy * kCellY, cell_x0 = g.xlo + ccx * kCellX;
      for (int l = 0; l < g.L && ok; ++l, ++li) {
        const int sbuf = (int)(li % (uint32_t)NSB);
        const uint32_t suse = li / (uint32_t)NSB;
        // the staging buffer's previous level has been copied out
        if (!tc::mbar_wait(s_empty + sbuf, (suse & 1) ^ 1, abort)) { ok = false; break; }
        const float inv = 1.f / (float)(1 << l);
        const float clx = cx * inv, cly = cy * inv;
        const float x0f = floorf(clx), y0f = floorf(cly);
        const float dx = clx - x0f, dy = cly - y0f;
        const float wa = (1.f - dx) * (1.f - dy) * p.scale, wb = dx * (1.f - dy) * p.scale;
        const float wc = (1.f - dx) * dy * p.scale, wd = dx * dy * p.scale;
        const int rx = (int)x0f - (cell_x0 >> l);   // 0..15
        const int ry = (int)y0f - (cell_y0 >> l);
        const int UW = g.UW[l], UH = g.UH[l], R = g.R[l];
        __half* orow = reinterpret_cast<__half*>(sOut + sbuf * stage_words + t * RDPS);
        for (int k = 0; k < g.nparts[l]; ++k, ++pc) {
          const int buf = pc & 1;
          if (!tc::mbar_wait(t_full + buf, (pc >> 1) & 1, abort)) { ok = false; break; }
          tc::tc_fence_after();
          const int U0 = k * (R - 1);
          const int reff = min(R, UH - U0);            // rows of this part inside the union
          const int rs = reff > 1 ? (reff - 2) / kFwdEG + 1 : 1;
          const int ua = ge * rs;
          const int ub = min(reff - 1, (ge + 1) * rs);
          const uint32_t taddr = lane_addr + buf * 256;
          const bool ym = p.ymajor != 0;
          // rx < 16 >> l: the select depth and read width of the level
          if (l == 0)
            fwd_part_rows<RADIUS, 0>(taddr, UW, U0, ua, ub, ry, rx, valid, wa, wb, wc, wd, ym, orow);
          else if (l == 1)
            fwd_part_rows<RADIUS, 1>(taddr, UW, U0, ua, ub, ry, rx, valid, wa, wb, wc, wd, ym, orow);
          else if (l == 2)
            fwd_part_rows<RADIUS, 2>(taddr, UW, U0, ua, ub, ry, rx, valid, wa, wb, wc, wd, ym, orow);
          else
            fwd_part_rows<RADIUS, 3>(taddr, UW, U0, ua, ub, ry, rx, valid, wa, wb, wc, wd, ym, orow);
          tc::tc_fence_before();
          tc::mbar_arrive(t_empty + buf);
        }
        if (!ok) break;
        // Level complete for this chunk: hand the staged rows to the copier.
        tc::mbar_arrive(s_full + sbuf);
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && abort_flag) atomicExch(&g_tc_status, 1);
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
// The gradient of one tap spreads over its four grid corners, so per pixel
// and level the incoming gradient collapses onto the (RD+1)^2 integer grid:
//   G[j][k] = scale * ( g(j,k)*wa + g(j,k-1)*wb + g(j-1,k)*wc + g(j-1,k-1)*wd )
// (terms with an index outside [0, RD) omitted). Then
//   grad_fmap1[p]  = sum_l sum_{j,k} G_l[p][j][k] * fmap2_l[y0-r+j][x0-r+k]
//   grad_fmap2_l[q] = sum_p G_l[p][q - (y0-r, x0-r)] * fmap1[p]
// which are the reference backward's per-tap sums
// (cuda_pyramid/localcorr_cuda_pyramid_kernel.cu:887-916) regrouped.

// Source-order pass over 128-pixel runs of one (batch, level): the run's
// incoming gradients (RD^2 rows of 128 pixels) are staged in shared memory
// with 16-byte loads, each thread collapses its pixel's onto the (RD+1)^2
// grid one grid row at a time (separable weights: a horizontal lerp of two
// tap rows, then a vertical one), and writes the pixel's record
//   gsh[l][idx][NG][NU] (16-byte units, sorted order): grid row j shifted
//   right by a = (x0 - r) mod 8 halves inside NU*8 zero-padded halves,
// so a record unit covers the 8 positions [X + 8u, X + 8u + 8) with
// X = (x0 - r) - a, a multiple of 8; grad_fmap2 and grad_fmap1 builders
// copy these units into 8-aligned position units with cp.async as they are.
// Records go out through a per-warp shared staging area, RC grid rows at a
// time, as contiguous runs. It also records the packed level bases and
// zeroes grad_fmap1 of pixels dropped by the sort (windows off the map at
// every level).
template <int RADIUS>
struct GintShape {
  static constexpr int RD = 2 * RADIUS + 1;
  static constexpr int NG = RD + 1;
  static constexpr int NU = (NG + 14) / 8;                 // units per shifted row
  static constexpr int RC = (16 / NU) < NG ? 16 / NU : NG;  // grid rows per staged chunk
  static constexpr int SU = (RC * NU) % 2 ? RC * NU : RC * NU + 1;  // odd unit stride
  static constexpr size_t tile_bytes = (size_t)RD * RD * 128 * 2;
  static constexpr size_t stage_bytes = (size_t)4 * 32 * SU * 16;
  static constexpr size_t smem_bytes = tile_bytes + stage_bytes;
  // persistent form: two 1024-aligned tiles (TMA double buffer) + staging
  static constexpr size_t tile_pad = (tile_bytes + 1023) / 1024 * 1024;
  static constexpr size_t tma_smem_bytes = 1024 + 2 * tile_pad + stage_bytes;
  static constexpr bool tma_ok = RD * RD <= 256;  // one TMA box per tile
};

// One 128-pixel run (pixels pix0.., level l, image b) whose incoming
// gradients are in `tile` ([RD*RD][128] halves): the per-pixel prologue
// (sorted index, level base, dropped-pixel zeroing) and the records.
template <int RADIUS>
__device__ __forceinline__ void gint_tile(const __half* __restrict__ tile, uint4* stage, int pix0,
                                          int l, int b, const void* __restrict__ coords,
                                          int coords_f32, const int* __restrict__ inv,
                                          uint4* __restrict__ gsh, int* __restrict__ sbase,
                                          __half* __restrict__ grad_f1, int ymajor, int acc_f1,
                                          const TcGeom& g) {
  using S = GintShape<RADIUS>;
  constexpr int RD = S::RD, NG = S::NG, NU = S::NU, RC = S::RC, SU = S::SU;
  constexpr unsigned FULL = 0xffffffffu;
  const int t = threadIdx.x, lane = t & 31;
  const int pix = pix0 + t;
  int idx = -1;
  float dx = 0.f, dy = 0.f;
  int x0 = 0;
  if (pix < g.HW) {
    const long long gid = (long long)b * g.HW + pix;
    idx = inv[gid];
    if (!LCB_IN(idx >= -1 && idx < g.npix, kSiteTcGint, idx)) idx = -1;
    if (idx < 0) {
      if (l == 0 && !acc_f1) {
        uint4* row = reinterpret_cast<uint4*>(grad_f1 + gid * g.C);
        for (int i = 0; i < g.C / 8; ++i) row[i] = make_uint4(0, 0, 0, 0);
      }
    } else {
      float cx, cy;
      if (coords_f32) {
        const float* co = reinterpret_cast<const float*>(coords) + (long long)b * 2 * g.HW + pix;
        cx = co[0]; cy = co[g.HW];
      } else {
        const __half* co = reinterpret_cast<const __half*>(coords) + (long long)b * 2 * g.HW + pix;
        cx = __half2float(co[0]); cy = __half2float(co[g.HW]);
      }
      const float inv_s = 1.f / (float)(1 << l);
      const float clx = cx * inv_s, cly = cy * inv_s;
      dx = clx - floorf(clx);
      dy = cly - floorf(cly);
      x0 = (int)floorf(clx);
      const int y0 = (int)floorf(cly);
      // Level-l integer base of the window, packed (x low, y high, int16
      // each), in sorted order: the grad_fmap2 pull reads it per candidate.
      sbase[(long long)l * g.npix + idx] = (x0 & 0xFFFF) | (y0 << 16);
    }
  }
  // Shift by a halves: one byte permute (odd part) and two word selects.
  const int a = (x0 - RADIUS) & 7;
  const uint32_t sel = (a & 1) ? 0x5432u : 0x7654u;
  const bool s1 = (a & 2) != 0, s2 = (a & 4) != 0;
  // The output scale is applied in float32 by the GEMM epilogues, not here:
  // the float16 records keep the magnitude of the incoming gradient.
  const float ex = 1.f - dx, ey = 1.f - dy, fy = dy;
  auto tap = [&](int iy, int ix) -> float {
    return __half2float(tile[(ymajor ? (ix + RD * iy) : (iy + RD * ix)) * 128 + t]);
  };
  float hp[NG];
#pragma unroll
  for (int k = 0; k < NG; ++k) hp[k] = 0.f;
#pragma unroll
  for (int j0 = 0; j0 < NG; j0 += RC) {
#pragma unroll
    for (int j = j0; j < j0 + RC && j < NG; ++j) {
      float hc[NG];
      if (j < RD) {
        float tr[RD];
#pragma unroll
        for (int k = 0; k < RD; ++k) tr[k] = tap(j, k);
#pragma unroll
        for (int k = 0; k < NG; ++k)
          hc[k] = (k < RD ? ex * tr[k] : 0.f) + (k >= 1 ? dx * tr[k - 1] : 0.f);
      } else {
#pragma unroll
        for (int k = 0; k < NG; ++k) hc[k] = 0.f;
      }
      uint32_t q[4 * NU];
#pragma unroll
      for (int k = 0; k < 4 * NU; ++k) {
        uint32_t w[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c = 2 * k + h;
          w[h] = c < NG ? (uint32_t)__half_as_ushort(__float2half_rn(ey * hc[c] + fy * hp[c])) : 0u;
        }
        q[k] = w[0] | (w[1] << 16);
      }
#pragma unroll
      for (int k = 4 * NU - 1; k >= 0; --k) q[k] = __byte_perm(k >= 1 ? q[k - 1] : 0u, q[k], sel);
#pragma unroll
      for (int k = 4 * NU - 1; k >= 0; --k) q[k] = s1 ? (k >= 1 ? q[k - 1] : 0u) : q[k];
#pragma unroll
      for (int k = 4 * NU - 1; k >= 0; --k) q[k] = s2 ? (k >= 2 ? q[k - 2] : 0u) : q[k];
#pragma unroll
      for (int u = 0; u < NU; ++u)
        stage[lane * SU + (j - j0) * NU + u] = make_uint4(q[4 * u], q[4 * u + 1], q[4 * u + 2], q[4 * u + 3]);
#pragma unroll
      for (int k = 0; k < NG; ++k) hp[k] = hc[k];
    }
    __syncwarp();
    // the warp's 32 records, rows [j0, j0 + RC): contiguous runs per pixel
    constexpr int CU0 = RC * NU;
    const int CU = (j0 + RC <= NG ? RC : NG - j0) * NU;
    for (int f = lane; f < 32 * CU0; f += 32) {
      const int k = f / CU0, v = f - k * CU0;
      const int idk = __shfl_sync(FULL, idx, k);
      if (idk >= 0 && v < CU)
        gsh[((long long)l * g.npix + idk) * (NG * NU) + j0 * NU + v] = stage[k * SU + v];
    }
    __syncwarp();
  }
}


template <int RADIUS>
__global__ void __launch_bounds__(128)
tc_gint_kernel(const __half* __restrict__ corr_grad, const void* __restrict__ coords,
               int coords_f32, const int* __restrict__ inv, uint4* __restrict__ gsh,
               int* __restrict__ sbase, __half* __restrict__ grad_f1, int ymajor,
               int vec_ok, int acc_f1, int* __restrict__ wctr, TcGeom g) {
  if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x < kWorkCounters)
    wctr[threadIdx.x] = 0;
  using S = GintShape<RADIUS>;
  constexpr int RD = S::RD, SU = S::SU;
  extern __shared__ __align__(16) uint8_t gsm[];
  __half* tile = reinterpret_cast<__half*>(gsm);
  const int t = threadIdx.x, warp = t >> 5;
  uint4* stage = reinterpret_cast<uint4*>(gsm + S::tile_bytes) + warp * 32 * SU;
  const int pix0 = blockIdx.x * 128;
  const int l = blockIdx.y;
  const int b = blockIdx.z;
  const int npx = min(128, g.HW - pix0);
  const __half* src = corr_grad + ((long long)b * g.L + l) * RD * RD * g.HW + pix0;
  if (vec_ok && npx == 128) {
#pragma unroll 4
    for (int i = t; i < RD * RD * 16; i += 128) {
      const int d = i >> 4, c = i & 15;
      reinterpret_cast<uint4*>(tile)[i] =
          *reinterpret_cast<const uint4*>(src + (long long)d * g.HW + c * 8);
    }
  } else {
    for (int i = t; i < RD * RD * 128; i += 128) {
      const int d = i >> 7, c = i & 127;
      tile[i] = c < npx ? src[(long long)d * g.HW + c] : __float2half(0.f);
    }
  }
  __syncthreads();
  gint_tile<RADIUS>(tile, stage, pix0, l, b, coords, coords_f32, inv, gsh, sbase, grad_f1,
                    ymajor, acc_f1, g);
}

// Persistent form for 16-byte aligned gradient rows: each block walks runs
// blockIdx.x, +gridDim.x, ... and a TMA 2D load ([RD*RD rows][128 pixels]
// of corr_grad viewed as [B*L*RD*RD][HW], zero past HW) brings the next
// run's gradients in while the current one is turned into records.
template <int RADIUS>
__global__ void __launch_bounds__(128)
tc_gint_tma_kernel(const __grid_constant__ CUtensorMap tmap_g, const void* __restrict__ coords,
                   int coords_f32, const int* __restrict__ inv, uint4* __restrict__ gsh,
                   int* __restrict__ sbase, __half* __restrict__ grad_f1,
                   int ymajor, int acc_f1, int nblk, int nruns, int* __restrict__ wctr,
                   TcGeom g) {
  if (blockIdx.x == 0 && threadIdx.x < kWorkCounters) wctr[threadIdx.x] = 0;
  using S = GintShape<RADIUS>;
  constexpr int RD = S::RD;
  constexpr int SU = S::SU;
  extern __shared__ uint8_t gsm_raw[];
  __shared__ uint64_t full[2];
  __shared__ int abort_flag;
  uint8_t* gsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
  const int t = threadIdx.x, warp = t >> 5;
  uint4* stage = reinterpret_cast<uint4*>(gsm + 2 * S::tile_pad) + warp * 32 * SU;
  if (t == 0) {
    tc::mbar_init(full, 1);
    tc::mbar_init(full + 1, 1);
    tc::fence_mbar_init();
    abort_flag = 0;
  }
  __syncthreads();
  volatile int* abort = &abort_flag;
  // run k: pixel block k % nblk of (image, level) = k / nblk (image major)
  auto issue = [&](int k, int buf) {
    const int bl = k / nblk;
    const int pb = k - bl * nblk;
    const int b = bl / g.L, l = bl - b * g.L;
    tc::fence_proxy_async_smem();
    tc::mbar_arrive_expect_tx(full + buf, (uint32_t)S::tile_bytes);
    tc::tma_load_2d(gsm + buf * S::tile_pad, &tmap_g, full + buf, pb * 128,
                    (b * g.L + l) * RD * RD);
  };
  if (t == 0 && (int)blockIdx.x < nruns) issue(blockIdx.x, 0);
  int i = 0;
  bool pending_next = false;
  for (int k = blockIdx.x; k < nruns; k += gridDim.x, ++i) {
    const int buf = i & 1;
    const int kn = k + gridDim.x;
    // the other buffer was last read by run i-1, which every thread
    // finished before the barrier that ended iteration i-1
    pending_next = kn < nruns;
    if (t == 0 && pending_next) issue(kn, buf ^ 1);
    if (!tc::mbar_wait(full + buf, (i >> 1) & 1, abort)) break;
    const int bl = k / nblk;
    const int pb = k - bl * nblk;
    const int b = bl / g.L, l = bl - b * g.L;
    gint_tile<RADIUS>(reinterpret_cast<const __half*>(gsm + buf * S::tile_pad), stage, pb * 128,
                      l, b, coords, coords_f32, inv, gsh, sbase, grad_f1, ymajor, acc_f1, g);
    __syncthreads();
    pending_next = false;
  }
  if (abort_flag) {
    // copies still in flight land before the block's shared memory goes
    if (t == 0) {
      tc::mbar_wait_drain(full + (i & 1), (i >> 1) & 1);
      if (pending_next) tc::mbar_wait_drain(full + ((i + 1) & 1), ((i + 1) >> 1) & 1);
      atomicExch(&g_tc_status, 1);
    }
  }
}

struct alignas(64) TcBwdParams {
  CUtensorMap tmap[kMaxTcLevels];
  CUtensorMap tmap_f1s;  // sorted fmap1 copy [npix rows][C], 64-channel x 64-row SW128 boxes
  const void* coords;
  const int* sorted;
  const int* counts;
  const int* offsets;
  const int4* work;
  const int* work_count;
  const uint4* gsh;
  const int* sbase;
  const __half* fmap1;
  __half* grad_f1;
  float* grad_f2;
  int coords_f32;
  int nstage;
  uint32_t stage_bytes;
  long long nitems;
  int* item_next;  // grad_fmap2 item counter (zeroed by the gradient-record kernel)
  int nbg;     // grad_fmap1 builder groups (1 or 2)
  int acc_f1;  // add grad_fmap1 into the existing rows instead of overwriting them
  float scale; // output scale, applied to the float32 accumulators
  TcGeom g;
};

// grad_fmap2 pull over one or more lookups of the same maps (a RAFT block's
// iterations): each lookup brings its own sort, sorted fmap1 copy and
// gradient records; an output tile sums the candidates of every lookup in
// one accumulator and is added to the float32 gradient once.
constexpr int kMaxPull = 12;
struct alignas(64) TcPullParams {
  CUtensorMap tmap_f1s[kMaxPull];  // per lookup: sorted fmap1 copy, 64-channel x 64-row boxes
  const int* offsets[kMaxPull];    // per lookup: sort bin offsets
  const uint4* gsh[kMaxPull];      // per lookup: pre-shifted gradient records
  const int* sbase[kMaxPull];      // per lookup: packed level bases (sorted order)
  int nlook;
  float* grad_f2;
  int nstage;
  uint32_t stage_bytes;
  long long nitems;
  int* item_next;  // item counter, zero at launch
  float scale;     // output scale, applied to the float32 accumulators
  TcGeom g;
};

__device__ __forceinline__ void pixel_coords(const TcBwdParams& p, int b, int pix, float& cx,
                                             float& cy) {
  const TcGeom& g = p.g;
  if (p.coords_f32) {
    const float* co = reinterpret_cast<const float*>(p.coords) + (long long)b * 2 * g.HW + pix;
    cx = co[0]; cy = co[g.HW];
  } else {
    const __half* co = reinterpret_cast<const __half*>(p.coords) + (long long)b * 2 * g.HW + pix;
    cx = __half2float(co[0]); cy = __half2float(co[g.HW]);
  }
}

// A grad_fmap1 row group (box rows gi*Rg.. of level l for the cell at
// (cell_y0, cell_x0)) takes part only if it overlaps the level's map: outside
// it the boxes are TMA zero fill and contribute nothing.
__device__ __forceinline__ bool b1_group_live(const TcGeom& g, int l, int gi, int cell_y0,
                                              int cell_x0, int radius) {
  const int X0 = ((cell_x0 >> l) - radius) & ~7;
  if (X0 >= g.w[l] || X0 + g.UWb[l] <= 0) return false;
  const int Y0 = (cell_y0 >> l) - radius;
  const int ra = Y0 + gi * g.Rg[l];
  const int rb = min(ra + g.Rg[l], Y0 + g.UH[l]);
  return ra < g.h[l] && rb > 0;
}

// grad_fmap1, per 128-pixel chunk: D[128 px x C] += G[128 px x 64 pos] *
// F2[64 pos x C] over every union row group of every level; D lives in TMEM
// for the whole chunk, so each pixel row is written once (no atomics).
// A (G rows, K-major, SWIZZLE_128B) is built by the builder warps from the
// pixel's pre-shifted grid records: the group's boxes start at an 8-aligned
// column and have a width that is a multiple of 8, so every 16-byte A unit is
// one record unit (cp.async) or zeros. B is the union row group loaded by
// TMA and read as an MN-major operand (channels contiguous).
template <int RADIUS>
__global__ void __launch_bounds__(kBwd1Threads, 1) tc_bwd1_kernel(const __grid_constant__ TcBwdParams p) {
  constexpr int RD = 2 * RADIUS + 1;
  constexpr int NG = RD + 1;
  constexpr int NU = (NG + 14) / 8;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int abort_flag;
  const TcGeom& g = p.g;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NST = p.nstage;
  const uint32_t SB = p.stage_bytes;  // 16 KB of A + KC * 8 KB of B
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)NST * SB);
  // full[s]: the stage's B boxes (TMA bytes, one producer arrival) and its A
  // rows (one arrival per builder thread when its copies have landed)
  uint64_t* full = bars;
  uint64_t* empty = bars + 2 * NST;
  uint64_t* acc_full = bars + 3 * NST;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* fin_bar = acc_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 5);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Zero every stage once: the rows of a B stage past the current box (and
  // never loaded yet) must hold finite values for the padded K positions.
  for (int i = threadIdx.x; i < (int)(NST * SB / 16); i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  tc::fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      tc::mbar_init(full + s, kTile + 1);
      tc::mbar_init(empty + s, 1);
    }
    for (int i = 0; i < 2; ++i) { tc::mbar_init(acc_full + i, 1); tc::mbar_init(acc_empty + i, kTile); }
    tc::mbar_init(fin_bar, 1);
    tc::fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nwork = *p.work_count;
  volatile int* abort = &abort_flag;

  if (warp == 0) {
    // ---------------- producer: B = union row groups ----------------
    if (lane == 0) {
      uint32_t gs = 0;
      bool ok = true;
      for (int wi = blockIdx.x; wi < nwork && ok; wi += gridDim.x) {
        const int4 wk = p.work[wi];
        const int b = wk.x, cell = wk.y;
        const int cy = cell / g.ncx, cx = cell - cy * g.ncx;
        const int cell_y0 = g.ylo + cy * kCellY, cell_x0 = g.xlo + cx * kCellX;
        for (int l = 0; l < g.L && ok; ++l) {
          const int X0 = ((cell_x0 >> l) - RADIUS) & ~7;
          const int Y0 = (cell_y0 >> l) - RADIUS;
          const uint32_t box = 128u * g.UWb[l] * g.Rg[l];
          for (int gi = 0; gi < g.ngroups[l]; ++gi) {
            if (!b1_group_live(g, l, gi, cell_y0, cell_x0, RADIUS)) continue;
            const int s = gs % NST;
            const uint32_t use = gs / NST;
            ++gs;
            if (!tc::mbar_wait(empty + s, (use & 1) ^ 1, abort)) { ok = false; break; }
            tc::mbar_arrive_expect_tx(full + s, box * g.KC);
            uint8_t* sb = smem + (size_t)s * SB + 16384;
            for (int kc = 0; kc < g.KC; ++kc)
              tc::tma_load_4d(sb + kc * 8192, &p.tmap[l], full + s, kc * 64, X0,
                              Y0 + gi * g.Rg[l], b);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int s = 0;          // stage ring position and its fill phase
      uint32_t ph = 0;
      int it = 0;
      // descriptors: stage s at +s*SB, its B at +16 KB; K steps of 32 bytes
      // in A (+2), of 16 rows x 128 bytes in B (+128)
      const uint64_t a_desc0 = tc::smem_desc_sw128(tc::smem_u32(smem), 16, 1024);
      const uint64_t b_desc0 = tc::smem_desc_sw128(tc::smem_u32(smem) + 16384, 8192, 1024);
      const uint32_t stage_units = SB >> 4;
      const uint32_t idesc = tc::idesc_f16_f32(128, g.C, false, true);
      bool ok = true;
      int next_cell = blockIdx.x < nwork ? p.work[blockIdx.x].y : 0;
      for (int wi = blockIdx.x; wi < nwork && ok; wi += gridDim.x, ++it) {
        const int buf = it & 1;
        const int cell = next_cell;  // loaded one chunk ahead
        if (wi + (int)gridDim.x < nwork) next_cell = p.work[wi + gridDim.x].y;
        const int mcy = cell / g.ncx, mcx = cell - mcy * g.ncx;
        const int m_y0 = g.ylo + mcy * kCellY, m_x0 = g.xlo + mcx * kCellX;
        if (!tc::mbar_wait(acc_empty + buf, ((it >> 1) & 1) ^ 1, abort)) break;
        tc::tc_fence_after();
        bool first = true;
        for (int l = 0; l < g.L && ok; ++l) {
          // K positions actually in the group's boxes: whole 16-row MMA steps
          const int nkk = (g.UWb[l] * g.Rg[l] + 15) / 16;
          for (int gi = 0; gi < g.ngroups[l]; ++gi) {
            if (!b1_group_live(g, l, gi, m_y0, m_x0, RADIUS)) continue;
            const int cs = s;
            const uint32_t cph = ph;
            if (++s == NST) { s = 0; ph ^= 1; }
            const uint64_t ad = a_desc0 + (uint64_t)(cs * stage_units);
            const uint64_t bd = b_desc0 + (uint64_t)(cs * stage_units);
            if (!tc::mbar_wait(full + cs, cph, abort)) { ok = false; break; }
            // A rows arrive through cp.async completion: make their
            // shared-memory writes visible to the tensor core's proxy.
            tc::fence_proxy_async_smem();
            tc::tc_fence_after();
            tc::mma_f16_ss_n(tmem + buf * 256, ad, 2, bd, 128, idesc, first ? 0u : 1u, nkk);
            first = false;
            tc::mma_commit(empty + cs);
          }
        }
        if (ok) tc::mma_commit(acc_full + buf);
      }
      tc::mma_commit(fin_bar);
      tc::mbar_wait(fin_bar, 0, abort);
    }
    __syncwarp();
  } else if (warp < 2 + 4 * p.nbg) {
    // ---------------- builders ----------------
    // Groups of 4 warps (one thread per A row = pixel of the chunk): group
    // gb builds the A tiles of the stages with (stage index % nbg) == gb.
    const int q = warp & 3;
    const int gb = (warp - 2) >> 2;
    const int t = q * 32 + lane;
    uint32_t gs = 0;
    bool ok = true;
    for (int wi = blockIdx.x; wi < nwork && ok; wi += gridDim.x) {
      const int4 wk = p.work[wi];
      const int b = wk.x, cell = wk.y, start = wk.z, n = wk.w;
      const int idx = start + t;
      const bool valid = t < n && LCB_IN(idx >= 0 && idx < g.npix, kSiteTcBwd1, idx);
      float cx = 0.f, cy = 0.f;
      if (valid) {
        int pix = p.sorted[idx] - b * g.HW;
        if (!LCB_IN(pix >= 0 && pix < g.HW, kSiteTcBwd1, pix)) pix = 0;
        pixel_coords(p, b, pix, cx, cy);
      }
      const int ccy = cell / g.ncx, ccx = cell - ccy * g.ncx;
      const int cell_y0 = g.ylo + ccy * kCellY, cell_x0 = g.xlo + ccx * kCellX;
      for (int l = 0; l < g.L && ok; ++l) {
        const float inv = 1.f / (float)(1 << l);
        const int bxl = (int)floorf(cx * inv), byl = (int)floorf(cy * inv);
        const int ry = byl - (cell_y0 >> l);                          // window row 0 in the box
        const int X0 = ((cell_x0 >> l) - RADIUS) & ~7;                // box column 0
        const int cu = (((bxl - RADIUS) & ~7) - X0) >> 3;             // box unit of record unit 0
        const int UPR = g.UWb[l] >> 3, Rg = g.Rg[l];
        const int nunit = 2 * ((g.UWb[l] * Rg + 15) / 16);  // A units the MMA reads
        const uint4* rec = p.gsh + ((long long)l * g.npix + idx) * (NG * NU);
        for (int gi = 0; gi < g.ngroups[l]; ++gi) {
          if (!b1_group_live(g, l, gi, cell_y0, cell_x0, RADIUS)) continue;
          const uint32_t my = gs++;
          if ((int)(my % (uint32_t)p.nbg) != gb) continue;
          const int s = my % NST;
          const uint32_t use = my / NST;
          if (!tc::mbar_wait(empty + s, (use & 1) ^ 1, abort)) { ok = false; break; }
          // A row of this pixel: 8 units of 8 K positions (box row br, unit
          // uc of that row); each a record unit (cp.async) or zeros.
          uint8_t* arow = smem + (size_t)s * SB + t * 128;
          int br = 0, uc = 0;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            if (k >= nunit) break;  // past the MMA's K steps: never read
            const int jj = gi * Rg + br - ry;
            const int u = uc - cu;
            uint8_t* dst = arow + ((k ^ (t & 7)) << 4);
            if (valid && br < Rg && (unsigned)jj < (unsigned)NG && (unsigned)u < (unsigned)NU)
              tc::cp_async_16(dst, rec + jj * NU + u, 16);
            else
              *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
            if (++uc == UPR) { uc = 0; ++br; }
          }
          tc::fence_proxy_async_smem();
          tc::cp_async_mbar_arrive_noinc(full + s);
        }
      }
    }
    // Copies still in flight complete before the kernel's final barrier.
    tc::cp_async_wait_all();
  } else {
    // ---------------- epilogue: TMEM row t = pixel t's grad_fmap1 ----------------
    const int q = warp & 3;
    const int t = q * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
    int it = 0;
    for (int wi = blockIdx.x; wi < nwork; wi += gridDim.x, ++it) {
      const int4 wk = p.work[wi];
      const int buf = it & 1;
      bool valid = t < wk.w;
      int gid = valid ? p.sorted[wk.z + t] : 0;
      if (!LCB_IN(gid >= 0 && gid < g.npix, kSiteTcBwd1, gid)) { gid = 0; valid = false; }
      // A chunk whose boxes all lie off the map issued no MMA: its
      // accumulator holds a previous chunk's values and its gradient is zero.
      bool live = false;
      {
        const int ecy = wk.y / g.ncx, ecx = wk.y - ecy * g.ncx;
        const int e_y0 = g.ylo + ecy * kCellY, e_x0 = g.xlo + ecx * kCellX;
        for (int l = 0; l < g.L && !live; ++l)
          for (int gi = 0; gi < g.ngroups[l] && !live; ++gi)
            live = b1_group_live(g, l, gi, e_y0, e_x0, RADIUS);
      }
      if (!tc::mbar_wait(acc_full + buf, (it >> 1) & 1, abort)) break;
      tc::tc_fence_after();
      for (int c0 = 0; c0 < g.C; c0 += 32) {
        float v[32];
        tc::tmem_ld32(lane_addr + buf * 256 + c0, v);
        tc::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = live ? v[i] * p.scale : 0.f;
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(p.grad_f1 + (long long)gid * g.C + c0);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (p.acc_f1) {
              // add the existing row (in its float16 storage type, as a sum
              // of per-lookup float16 gradients would be)
              const uint4 old = dst[i];
              const __half2* o2 = reinterpret_cast<const __half2*>(&old);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 of = __half22float2(o2[e]);
                v[8 * i + 2 * e] += of.x;
                v[8 * i + 2 * e + 1] += of.y;
              }
            }
            __align__(16) __half2 h2[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) h2[e] = __floats2half2_rn(v[8 * i + 2 * e], v[8 * i + 2 * e + 1]);
            dst[i] = *reinterpret_cast<const uint4*>(h2);
          }
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(acc_empty + buf);
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && abort_flag) atomicExch(&g_tc_status, 1);
}

// grad_fmap2, pulled per output tile Q of 8x16 level-l positions:
//   D[128 pos x C] = sum over the pixels whose windows reach Q of
//                    G^T[pos x px] * fmap1[px x C]
// The candidates of an item are, per anchor-cell row, one contiguous range
// of the sorted order: the cells are sorted by (cell, level-0 base column
// within the cell), so the columns of the boundary cells whose bases can
// reach Q are a sub-range and a cell row's candidates are one range. Every
// candidate is a K row (non-touching ones get an all-zero A row): A rows
// (MN-major, the pixel's G restricted to Q) are built by the builders from
// the pre-shifted records with cp.async, B rows are the candidates' fmap1
// rows, loaded by TMA as 64-row tiles of the sorted fmap1 copy. D is
// double-buffered in TMEM; the epilogue adds it to the float32 gradient with
// red.global.add.v4.f32 (items may cover only part of Q's cells).
constexpr int kB2Rows = 64;                       // K rows per stage
constexpr int kBwd2Builders = 256;                // builder threads (warps 2..9)
constexpr int kB2Groups = kBwd2Builders / kB2Rows;  // stage gs is built by group gs % 4
constexpr int kBwd2Threads = 64 + kBwd2Builders + 128;  // MMA warp, TMA warp, builders, epilogue

struct Bwd2Item {
  int l, b, qy0, qx0, ra, rb, ca, cb;  // level, batch, tile origin, cell rows/cols
  int bx_lo, bx_hi;                    // level-0 base columns that can reach Q
  bool empty;
};

__device__ __forceinline__ Bwd2Item decode_item(const TcGeom& g, long long it, int radius) {
  // Items run image by image (the CTAs then share one image's fmap1 rows and
  // records in L2), coarse levels first within an image (longest first).
  Bwd2Item r{};
  const long long per_image = g.items_before[g.L];
  const int b = (int)(it / per_image);
  long long rem = it - (long long)b * per_image;
  int li = 0;
  while (li + 1 < g.L && rem >= g.items_before[li + 1]) ++li;
  const int l = g.L - 1 - li;
  rem -= g.items_before[li];
  const int grp = (int)(rem % g.qgroups[l]);
  rem /= g.qgroups[l];
  const int qtx = (int)(rem % g.nqx[l]);
  const int qty = (int)(rem / g.nqx[l]);
  r.l = l;
  r.b = b;
  r.qy0 = qty * 8;
  r.qx0 = qtx * 16;
  const int s = 1 << l;
  // level-l bases that can touch Q, then the level-0 base range, then cells
  const int by_lo = (r.qy0 - radius - 1) * s, by_hi = (r.qy0 + 7 + radius) * s + s - 1;
  const int bx_lo = (r.qx0 - radius - 1) * s, bx_hi = (r.qx0 + 15 + radius) * s + s - 1;
  int ra = (by_lo - g.ylo) >= 0 ? (by_lo - g.ylo) / kCellY : 0;
  int rb = (by_hi - g.ylo) >= 0 ? (by_hi - g.ylo) / kCellY : -1;
  int ca = (bx_lo - g.xlo) >= 0 ? (bx_lo - g.xlo) / kCellX : 0;
  int cb = (bx_hi - g.xlo) >= 0 ? (bx_hi - g.xlo) / kCellX : -1;
  rb = min(rb, g.ncy - 1);
  cb = min(cb, g.ncx - 1);
  ra = ra + grp * g.rpi[l];
  rb = min(rb, ra + g.rpi[l] - 1);
  r.ra = ra; r.rb = rb; r.ca = ca; r.cb = cb;
  r.bx_lo = bx_lo; r.bx_hi = bx_hi;
  r.empty = ra > rb || ca > cb;
  return r;
}

// Sorted range [s0, s1) of the item's candidates in cell row k (k < nranges).
__device__ __forceinline__ int2 item_range(const TcGeom& g, const int* __restrict__ fine_off,
                                           const Bwd2Item& it, int k) {
  const int cyr = it.ra + k;
  const long long row0 = ((long long)it.b * g.ncell + (long long)cyr * g.ncx) * kColBins;
  const int la = max(0, it.bx_lo - (g.xlo + it.ca * kCellX));
  const int lb = min(kColBins - 1, it.bx_hi - (g.xlo + it.cb * kCellX));
  const int s0 = fine_off[row0 + (long long)it.ca * kColBins + la];
  const int s1 = fine_off[row0 + (long long)it.cb * kColBins + lb + 1];
  return make_int2(s0, max(s0, s1));
}

// Stages (64 sorted rows each) of an item over its nr cell-row ranges (0
// for an item without candidates: the producer skips it).
__device__ __forceinline__ int item_stages(const TcGeom& g, const int* __restrict__ fine_off,
                                           const Bwd2Item& it, int nr) {
  int total = 0;
  for (int k = 0; k < nr; ++k) {
    const int2 rg = item_range(g, fine_off, it, k);
    total += (rg.y - rg.x + kB2Rows - 1) / kB2Rows;
  }
  return total;
}

// Range kk (< nlook * nr) of an item over its lookups: lookup kk / nr, cell
// row kk % nr; (0, 0) past the last.
__device__ __forceinline__ int2 pull_range(const TcPullParams& p, const Bwd2Item& it, int kk,
                                           int nr) {
  return kk < nr * p.nlook ? item_range(p.g, p.offsets[kk / nr], it, kk % nr) : make_int2(0, 0);
}

__device__ __forceinline__ int pull_stages(const TcPullParams& p, const Bwd2Item& it, int nr) {
  int total = 0;
  for (int look = 0; look < p.nlook; ++look) total += item_stages(p.g, p.offsets[look], it, nr);
  return total;
}

template <int RADIUS>
__global__ void __launch_bounds__(kBwd2Threads, 1) tc_bwd2_kernel(const __grid_constant__ TcPullParams p) {
  constexpr int RD = 2 * RADIUS + 1;
  constexpr int NG = RD + 1;
  constexpr int NU = (NG + 14) / 8;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int abort_flag;
  // stages of each item, written by the TMA producer before the item's first
  // stage is released (ring of 16 > the most items the producer can lead by)
  __shared__ int item_nst[16];
  // Items are taken dynamically: the TMA producer takes the next item index
  // from a global counter (coarse, long items first) and publishes it in a
  // 16-slot ring with one mbarrier per slot; the MMA thread, the builders
  // and the epilogue read the same sequence (-1 ends it). No role lags the
  // producer by 16 items (at most the stage count plus the two accumulator
  // buffers), so a slot is read by all before it is reused.
  __shared__ int item_ring[16];
  __shared__ __align__(8) uint64_t item_bar[16];
  const TcGeom& g = p.g;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NST = p.nstage;
  const uint32_t SB = p.stage_bytes;  // A: 2 x 8 KB (position halves), B: KC x 8 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)NST * SB);
  // full[s]: the stage's B tile (TMA bytes, one producer arrival) and its A
  // rows (one arrival per builder thread when its copies have landed)
  uint64_t* full = bars;
  uint64_t* empty = bars + 2 * NST;
  uint64_t* acc_full = bars + 3 * NST;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* fin_bar = acc_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 5);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < (int)(NST * SB / 16); i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  tc::fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      tc::mbar_init(full + s, kB2Rows + 1);
      tc::mbar_init(empty + s, 1);
    }
    for (int i = 0; i < 2; ++i) { tc::mbar_init(acc_full + i, 1); tc::mbar_init(acc_empty + i, kTile); }
    tc::mbar_init(fin_bar, 1);
    for (int i = 0; i < 16; ++i) tc::mbar_init(item_bar + i, 1);
    tc::fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  volatile int* abort = &abort_flag;
  const long long nitems = p.nitems;
  const uint32_t bbytes = (uint32_t)g.KC * kB2Rows * 128;

  if (warp == 0) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t ac = 0;
      int s = 0;          // stage ring position and its fill phase
      uint32_t ph = 0;
      // descriptors: stage s at +s*SB (A), its B at +2*kB2Rows*128; K steps
      // of 16 rows x 128 bytes (+128) in both
      const uint64_t a_desc0 = tc::smem_desc_sw128(tc::smem_u32(smem), kB2Rows * 128, 1024);
      const uint64_t b_desc0 =
          tc::smem_desc_sw128(tc::smem_u32(smem) + 2 * kB2Rows * 128, kB2Rows * 128, 1024);
      const uint32_t stage_units = SB >> 4;
      const uint32_t idesc = tc::idesc_f16_f32(128, g.C, true, true);
      bool ok = true;
      for (;; ++ac) {
        if (!tc::mbar_wait(item_bar + (ac & 15), (ac >> 4) & 1, abort)) break;
        if (item_ring[ac & 15] < 0) break;
        const int buf = ac & 1;
        if (!tc::mbar_wait(acc_empty + buf, ((ac >> 1) & 1) ^ 1, abort)) break;
        tc::tc_fence_after();
        int nst = 1;
        for (int q = 0; q < nst; ++q) {
          const int cs = s;
          const uint32_t cph = ph;
          if (++s == NST) { s = 0; ph ^= 1; }
          if (!tc::mbar_wait(full + cs, cph, abort)) { ok = false; break; }
          if (q == 0) nst = item_nst[ac & 15];
          // A rows arrive through cp.async completion: make their
          // shared-memory writes visible to the tensor core's proxy.
          tc::fence_proxy_async_smem();
          tc::tc_fence_after();
          static_assert(kB2Rows / 16 == 4, "one 4-MMA batch per stage");
          tc::mma_f16_ss_n(tmem + buf * 256, a_desc0 + (uint64_t)(cs * stage_units), 128,
                           b_desc0 + (uint64_t)(cs * stage_units), 128, idesc, q ? 1u : 0u, 4);
          tc::mma_commit(empty + cs);
        }
        if (!ok) break;
        tc::mma_commit(acc_full + buf);
      }
      tc::mma_commit(fin_bar);
      tc::mbar_wait(fin_bar, 0, abort);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- TMA producer: B = 64-row tiles of sorted fmap1 ----------------
    // Same stage sequence as the builders: the item's ranges cut into 64-row
    // stages (items without candidates are never published). Rows past a
    // range's end belong to other cells (or are zero fill past the end);
    // their A rows are zero.
    if (lane == 0) {
      uint32_t gs = 0, ic = 0;
      bool ok = true;
      for (; ok; ++ic) {
        // the next item with candidates (an item without any adds nothing:
        // it is not published)
        int it, nr = 0, nst = 0;
        Bwd2Item item{};
        for (;;) {
          it = atomicAdd(p.item_next, 1);
          if (it >= nitems) break;
          item = decode_item(g, it, RADIUS);
          nr = item.empty ? 0 : item.rb - item.ra + 1;
          nst = pull_stages(p, item, nr);
          if (nst > 0) break;
        }
        item_ring[ic & 15] = it < nitems ? it : -1;
        tc::mbar_arrive(item_bar + (ic & 15));
        if (it >= nitems) break;
        const int last = nst - 1;
        const int nrt = nr * p.nlook;  // ranges over all lookups
        int k = 0, j = 0;
        int2 rg = pull_range(p, item, 0, nr);
        for (int q = 0; q <= last && ok; ++q, ++gs) {
          while (k < nrt && j * kB2Rows >= rg.y - rg.x) {
            ++k;
            j = 0;
            rg = pull_range(p, item, k, nr);
          }
          const int look = min(k / nr, p.nlook - 1);
          const int row = rg.x + (j++) * kB2Rows;
          const int s = gs % NST;
          const uint32_t use = gs / NST;
          if (!tc::mbar_wait(empty + s, (use & 1) ^ 1, abort)) { ok = false; break; }
          // the item's stage count, released with its first stage
          if (q == 0) item_nst[ic & 15] = last + 1;
          tc::mbar_arrive_expect_tx(full + s, bbytes);
          uint8_t* sb = smem + (size_t)s * SB + 2 * kB2Rows * 128;
          for (int kc = 0; kc < g.KC; ++kc)
            tc::tma_load_2d(sb + kc * kB2Rows * 128, &p.tmap_f1s[look], full + s, kc * 64, row);
        }
      }
    }
    __syncwarp();
  } else if (warp < 2 + kBwd2Builders / 32) {
    // ---------------- builders ----------------
    // Group gb (two warps, one thread per row) builds the A tiles of the
    // stages with gs % 4 == gb: row t is candidate s0 + 64 j + t of the
    // stage's range, its G restricted to Q as 8 tile rows x two 16-byte
    // units, each a cp.async of a pre-shifted record unit or zeros (rows
    // past the range and non-touching candidates come out all zero). Each
    // builder's arrival on the stage's full barrier fires when its copies
    // have landed (cp.async.mbarrier.arrive.noinc).
    const int bt = threadIdx.x - 64;
    const int gb = bt / kB2Rows;
    const int t = bt % kB2Rows;
    uint32_t gs = 0;
    bool ok = true;
    for (uint32_t ic = 0; ok; ++ic) {
      if (!tc::mbar_wait(item_bar + (ic & 15), (ic >> 4) & 1, abort)) break;
      const int it = item_ring[ic & 15];
      if (it < 0) break;
      const Bwd2Item item = decode_item(g, it, RADIUS);
      const int l = item.l;
      const int nr = item.empty ? 0 : item.rb - item.ra + 1;
      const int last = pull_stages(p, item, nr) - 1;
      const int nrt = nr * p.nlook;
      int k = 0, j = 0;  // range (over all lookups) and stage within it of item stage q
      int2 rg = pull_range(p, item, 0, nr);
      for (int q = 0; q <= last && ok; ++q, ++gs) {
        while (k < nrt && j * kB2Rows >= rg.y - rg.x) {
          ++k;
          j = 0;
          rg = pull_range(p, item, k, nr);
        }
        const int look = min(k / nr, p.nlook - 1);
        const int* sb_l = p.sbase[look] + (long long)l * g.npix;
        const uint4* gsh_l = p.gsh[look] + (long long)l * g.npix * (NG * NU);
        const int s0 = rg.x;
        const int s1 = rg.y;
        const int jj0 = j++;
        if ((int)(gs % kB2Groups) != gb) continue;
        const int pos = s0 + jj0 * kB2Rows + t;
        const bool valid = pos < s1 && LCB_IN(pos >= 0 && pos < g.npix, kSiteTcBwd2, pos);
        int pk = 0;
        if (valid) pk = sb_l[pos];
        const int s = gs % NST;
        const uint32_t use = gs / NST;
        if (!tc::mbar_wait(empty + s, (use & 1) ^ 1, abort)) { ok = false; break; }
        uint8_t* A = smem + (size_t)s * SB;
        const int sw = t & 7;  // 16-byte units XOR-swizzled by row (SW128)
        const int x0 = (int)(short)(pk & 0xFFFF), y0 = pk >> 16;
        const uint4* rec = gsh_l + (long long)pos * (NG * NU);
        const int dy = valid ? item.qy0 - y0 + RADIUS : -64;          // grid row of tile row 0
        const int cu = (((x0 - RADIUS) & ~7) - item.qx0) >> 3;        // tile unit of record unit 0
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int jr = i + dy;
          const bool rv = (unsigned)jr < (unsigned)NG;
#pragma unroll
          for (int d = 0; d < 2; ++d) {
            const int u = d - cu;
            uint8_t* dst = A + (i >> 2) * (kB2Rows * 128) + t * 128 + (((((i & 3) << 1) | d) ^ sw) << 4);
            if (rv && (unsigned)u < (unsigned)NU)
              tc::cp_async_16(dst, rec + jr * NU + u, 16);
            else
              *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
          }
        }
        tc::fence_proxy_async_smem();
        tc::cp_async_mbar_arrive_noinc(full + s);
      }
    }
    // Copies still in flight complete before the kernel's final barrier.
    tc::cp_async_wait_all();
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const int t = q * 32 + lane;   // D row = position in Q
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
    uint32_t ac = 0;
    for (;; ++ac) {
      if (!tc::mbar_wait(item_bar + (ac & 15), (ac >> 4) & 1, abort)) break;
      const int it = item_ring[ac & 15];
      if (it < 0) break;
      const int buf = ac & 1;
      if (!tc::mbar_wait(acc_full + buf, (ac >> 1) & 1, abort)) break;
      tc::tc_fence_after();
      const Bwd2Item item = decode_item(g, it, RADIUS);
      const int l = item.l;
      const int qy = item.qy0 + (t >> 4), qx = item.qx0 + (t & 15);
      const bool inmap = !item.empty && qy < g.h[l] && qx < g.w[l];
      float* dst = p.grad_f2 + (long long)item.b * g.batch_elems + g.off[l] +
                   ((long long)qy * g.w[l] + qx) * g.C;
      for (int c0 = 0; c0 < g.C; c0 += 32) {
        float v[32];
        tc::tmem_ld32(lane_addr + buf * 256 + c0, v);
        tc::tmem_ld_wait();
        if (inmap) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= p.scale;
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            if (v[i] != 0.f || v[i + 1] != 0.f || v[i + 2] != 0.f || v[i + 3] != 0.f)
              asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + c0 + i),
                           "f"(v[i]), "f"(v[i + 1]), "f"(v[i + 2]), "f"(v[i + 3])
                           : "memory");
          }
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(acc_empty + buf);
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && abort_flag) atomicExch(&g_tc_status, 1);
}

// Deterministic grad_fmap2 of the CUDA-core engine (deterministic mode): the
// pull of tc_bwd2_kernel on CUDA cores in float32, for maps of any dtype and
// channel count. One block per output tile Q (8x16 level-l positions, one
// item per tile in deterministic mode) and 32-channel slice; thread t owns
// position t of Q and sums, over the tile's candidates in sorted order
// (fixed in deterministic mode), G_p(q) * fmap1[p][c0 .. c0+31], where
// G_p(q) is the pixel's scaled incoming gradient spread onto its (RD+1)^2
// grid by the four-corner rule of corr_bwd_simt_kernel. Each position is
// written by one thread, after the candidates in a fixed order.
template <typename T, typename TC>
__global__ void __launch_bounds__(128)
det_f2_pull_kernel(const T* __restrict__ fmap1, const TC* __restrict__ coords,
                   const T* __restrict__ corr_grad, const int* __restrict__ sorted,
                   const int* __restrict__ offsets, float* __restrict__ grad_f2, int radius,
                   int ymajor, float scale, TcGeom g) {
  const int RD = 2 * radius + 1;
  const Bwd2Item item = decode_item(g, blockIdx.x, radius);
  const int c0 = blockIdx.y * 32;
  const int nc = min(32, g.C - c0);
  const int t = threadIdx.x;
  const int l = item.l;
  const int qy = item.qy0 + (t >> 4), qx = item.qx0 + (t & 15);
  const bool inmap = !item.empty && qy < g.h[l] && qx < g.w[l];
  const float inv = 1.f / (float)(1 << l);
  const int nr = item.empty ? 0 : item.rb - item.ra + 1;
  float acc[32];
#pragma unroll
  for (int c = 0; c < 32; ++c) acc[c] = 0.f;
  const TC* cxb = coords + (long long)item.b * 2 * g.HW;
  const T* gl = corr_grad + ((long long)item.b * g.L + l) * RD * RD * g.HW;
  for (int k = 0; k < nr; ++k) {
    const int2 rg = item_range(g, offsets, item, k);
    for (int pos = rg.x; pos < rg.y; ++pos) {
      const int gid = sorted[pos];
      int pix = gid - item.b * g.HW;
      if (!LCB_IN(pix >= 0 && pix < g.HW, kSiteTcBwd2, gid)) continue;
      const float clx = ldf(cxb + pix) * inv, cly = ldf(cxb + g.HW + pix) * inv;
      const float x0f = floorf(clx), y0f = floorf(cly);
      const float dx = clx - x0f, dy = cly - y0f;
      const int jx = qx - ((int)x0f - radius), jy = qy - ((int)y0f - radius);
      float G = 0.f;
      if (inmap && jx >= 0 && jx <= RD && jy >= 0 && jy <= RD) {
        auto gv = [&](int iy, int ix) -> float {
          if (iy < 0 || iy >= RD || ix < 0 || ix >= RD) return 0.f;
          const int d = ymajor ? ix + RD * iy : iy + RD * ix;
          return ldf(gl + (long long)d * g.HW + pix);
        };
        G = (gv(jy, jx) * ((1.f - dx) * (1.f - dy)) + gv(jy, jx - 1) * (dx * (1.f - dy)) +
             gv(jy - 1, jx) * ((1.f - dx) * dy) + gv(jy - 1, jx - 1) * (dx * dy)) *
            scale;
      }
      if (G != 0.f) {
        const T* f1 = fmap1 + (long long)gid * g.C + c0;
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (c < nc) acc[c] = fmaf(G, ldf(f1 + c), acc[c]);
      }
    }
  }
  if (inmap) {
    float* dst = grad_f2 + (long long)item.b * g.batch_elems + g.off[l] +
                 ((long long)qy * g.w[l] + qx) * g.C + c0;
#pragma unroll
    for (int c = 0; c < 32; ++c)
      if (c < nc) dst[c] += acc[c];
  }
}

// scratch [L][npix][RDP] (sorted order) -> out [B][L][RD2][H][W]. Each thread
// moves one pixel's row: its 16-byte units are loaded in batches of up to 12,
// all of a batch before any of its stores (the row sits at a random sorted
// position, so the loads' latency is what bounds the kernel), then written
// plane by plane (consecutive pixels -> coalesced stores).
template <int RADIUS>
__global__ void tc_unsort_kernel(const __half* __restrict__ scratch, const int* __restrict__ inv,
                                 __half* __restrict__ out, TcGeom g) {
  constexpr int RD2 = (2 * RADIUS + 1) * (2 * RADIUS + 1);
  constexpr int NL = (RD2 + 7) / 8;  // 16-byte units of a scratch row (RDP / 8)
  constexpr int NB = NL < 12 ? NL : 12;
  const int pix = blockIdx.x * blockDim.x + threadIdx.x;
  const int l = blockIdx.y;
  const int b = blockIdx.z;
  if (pix >= g.HW) return;
  const long long gid = (long long)b * g.HW + pix;
  int idx = inv[gid];
  if (!LCB_IN(idx >= -1 && idx < g.npix, kSiteTcUnsort, idx)) idx = -1;
  const __half* src = scratch + ((long long)l * g.npix + (idx < 0 ? 0 : idx)) * (NL * 8);
  __half* dst = out + ((long long)b * g.L + l) * RD2 * g.HW + pix;
#pragma unroll
  for (int k0 = 0; k0 < NL; k0 += NB) {
    uint4 v[NB];
#pragma unroll
    for (int k = 0; k < NB; ++k)
      v[k] = (idx >= 0 && 8 * (k0 + k) < g.RD2)
                 ? *reinterpret_cast<const uint4*>(src + 8 * (k0 + k))
                 : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const int d0 = 8 * (k0 + k);
      if (d0 >= g.RD2) break;
      const __half* hv = reinterpret_cast<const __half*>(&v[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (d0 + e < g.RD2) dst[(long long)(d0 + e) * g.HW] = hv[e];
    }
  }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

int num_sms() {
  int dev = 0, v = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  return v > 0 ? v : 1;
}

// Workspace regions, in one offset space: the sort state [0, sort_total)
// (bin offsets, sorted pixel ids, inverse permutation, chunk work list) that
// a backward can reuse from its forward, then the per-call scratch. With one
// buffer both parts are contiguous; the ...KeepSort / ...WithSort entry
// points put the sort state in a buffer of its own.
struct WsLayout {
  size_t counts, offsets, keyrank, sorted, inv, work, work_count, cellpre, bsum, sbase, scratch,
      gsh, f1s, wctr;
  size_t sort_total;        // bytes of the sort state
  size_t fwd_total, total;  // bytes the forward / the backward need (both parts)
  long long max_work;
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

WsLayout ws_layout(const TcGeom& g) {
  WsLayout w{};
  size_t o = 0;
  const size_t ncells = (size_t)g.B * g.ncell;
  w.max_work = (g.npix + kTile - 1) / kTile + (long long)ncells;
  w.offsets = o; o = align256(o + (ncells * kColBins + 1) * 4);
  w.sorted = o; o = align256(o + (size_t)g.npix * 4);
  w.inv = o; o = align256(o + (size_t)g.npix * 4);
  w.work = o; o = align256(o + (size_t)w.max_work * 16);
  w.work_count = o; o = align256(o + 4);
  w.sort_total = o;
  w.counts = o; o = align256(o + (ncells * kColBins + 1) * 4);
  w.keyrank = o; o = align256(o + (size_t)g.npix * 8);
  w.cellpre = o; o = align256(o + ncells * 8);
  w.bsum = o; o = align256(o + (ncells + kScanBlock - 1) / kScanBlock * 8);
  w.sbase = o; o = align256(o + (size_t)g.L * g.npix * 4);
  w.wctr = o; o = align256(o + kWorkCounters * 4);
  w.scratch = o; o = align256(o + (size_t)g.L * g.npix * g.RDP * 2);
  w.fwd_total = o;
  // the backward's records reuse the forward's output scratch
  w.gsh = w.scratch;
  w.f1s = align256(w.gsh + (size_t)g.L * g.npix * g.NG * g.NU * 16);
  w.total = std::max(o, align256(w.f1s + (size_t)g.npix * g.C * 2));
  return w;
}

struct TcWs {
  int* counts;
  int* offsets;
  int2* keyrank;
  int* sorted;
  int* inv;
  int4* work;
  int* work_count;
  int2* cellpre;
  int2* bsum;
  int* sbase;
  __half* scratch;
  uint4* gsh;
  __half* f1s;
  int* wctr;  // dynamic work counters (kWorkCounters)
};

// sort_ws: the sort state (or nullptr: it is the first sort_total bytes of
// ws, the single-buffer layout); ws: the rest.
TcWs ws_pointers(void* sort_ws, void* ws, const WsLayout& L) {
  uint8_t* st = static_cast<uint8_t*>(sort_ws ? sort_ws : ws);
  // regions past the sort state sit at (their offset - sort_total) in a
  // separate rest buffer
  const uintptr_t wb = reinterpret_cast<uintptr_t>(ws) - (sort_ws ? L.sort_total : 0);
  uint8_t* w = reinterpret_cast<uint8_t*>(wb);
  TcWs p;
  p.offsets = reinterpret_cast<int*>(st + L.offsets);
  p.sorted = reinterpret_cast<int*>(st + L.sorted);
  p.inv = reinterpret_cast<int*>(st + L.inv);
  p.work = reinterpret_cast<int4*>(st + L.work);
  p.work_count = reinterpret_cast<int*>(st + L.work_count);
  p.counts = reinterpret_cast<int*>(w + L.counts);
  p.keyrank = reinterpret_cast<int2*>(w + L.keyrank);
  p.cellpre = reinterpret_cast<int2*>(w + L.cellpre);
  p.bsum = reinterpret_cast<int2*>(w + L.bsum);
  p.sbase = reinterpret_cast<int*>(w + L.sbase);
  p.scratch = reinterpret_cast<__half*>(w + L.scratch);
  p.gsh = reinterpret_cast<uint4*>(w + L.gsh);
  p.f1s = reinterpret_cast<__half*>(w + L.f1s);
  p.wctr = reinterpret_cast<int*>(w + L.wctr);
  return p;
}

// Counting sort of the pixels into anchor cells + the chunk work list.
bool tc_sort(const TcWs& W, const TcGeom& g, const void* co, int cdtype, cudaStream_t s) {
  // the counts and, after them, the small path's block ticket
  if (cudaMemsetAsync(W.counts, 0, sizeof(int) * ((size_t)g.B * g.ncell * kColBins + 1), s) !=
      cudaSuccess)
    return check_launch("memset counts");
  const int threads = 256;
  const int blocks = (int)((g.npix + threads - 1) / threads);
  const int ncells = g.B * g.ncell;
  if (ncells <= 1024 * kSmallScanCpt) {
    const unsigned hb = (unsigned)((g.npix + 1023) / 1024);
    int* done = W.counts + (size_t)ncells * kColBins;  // zeroed with the counts
    int* total = W.offsets + (size_t)ncells * kColBins;
    if (cdtype == LCB200_F32)
      tc_hist_scan_kernel<float><<<hb, 1024, 0, s>>>((const float*)co, W.counts, W.keyrank, done,
                                                      W.offsets, W.work, total, W.work_count, g);
    else
      tc_hist_scan_kernel<__half><<<hb, 1024, 0, s>>>((const __half*)co, W.counts, W.keyrank,
                                                       done, W.offsets, W.work, total,
                                                       W.work_count, g);
    count_launch();
    if (!check_launch("tc_hist_scan")) return false;
  } else {
    if (cdtype == LCB200_F32)
      tc_hist_kernel<float><<<blocks, threads, 0, s>>>((const float*)co, W.counts, W.keyrank, g);
    else
      tc_hist_kernel<__half><<<blocks, threads, 0, s>>>((const __half*)co, W.counts, W.keyrank, g);
    count_launch();
    if (!check_launch("tc_hist")) return false;
    const int nsb = (ncells + kScanBlock - 1) / kScanBlock;
    tc_cellscan_kernel<<<nsb, kScanBlock, 0, s>>>(W.counts, W.cellpre, W.bsum, ncells);
    count_launch();
    if (!check_launch("tc_cellscan")) return false;
    tc_blockscan_kernel<<<1, 1024, 0, s>>>(W.bsum, nsb, W.offsets + (size_t)ncells * kColBins,
                                           W.work_count);
    count_launch();
    if (!check_launch("tc_blockscan")) return false;
    tc_cellwrite_kernel<<<nsb, kScanBlock, 0, s>>>(W.counts, W.cellpre, W.bsum, W.offsets,
                                                   W.work, ncells, g.ncell);
    count_launch();
    if (!check_launch("tc_cellwrite")) return false;
  }
  tc_scatter_kernel<<<blocks, threads, 0, s>>>(W.keyrank, W.offsets, W.sorted, W.inv, g);
  count_launch();
  if (!check_launch("tc_scatter")) return false;
  if (!deterministic_mode()) return true;
  const long long nbins = (long long)ncells * kColBins;
  tc_rank_fix_kernel<<<(unsigned)((nbins * 32 + 255) / 256), 256, 0, s>>>(W.offsets, W.sorted,
                                                                        W.keyrank, nbins, g.npix);
  count_launch();
  if (!check_launch("tc_rank_fix")) return false;
  tc_scatter_kernel<<<blocks, threads, 0, s>>>(W.keyrank, W.offsets, W.sorted, W.inv, g);
  count_launch();
  return check_launch("tc_scatter");
}

size_t fwd_smem_bytes(const TcGeom& g, int nstage, int nsb, uint32_t* stage_bytes) {
  const uint32_t sb = (uint32_t)g.maxN * 128;
  if (stage_bytes) *stage_bytes = sb;
  const size_t rdps = g.RDP / 2 + 1;
  const size_t need = 1024 /*alignment slack*/ + (size_t)g.KC * 16384 + (size_t)nstage * sb +
                      (size_t)nsb * kTile * rdps * 4 + (2 * nstage + 12) * 8 + 16;
  // At least half of the SM's shared memory: one CTA per SM, so the
  // 512-column TMEM allocation never waits on a co-resident CTA.
  return std::max<size_t>(need, 120 * 1024);
}

bool radius_supported(int r) { return r == 3 || r == 4 || r == 8; }

// Forward pipeline depth: two output staging buffers when that still leaves
// three B stages, else one; then as many B stages (<= 4) as fit.
bool fwd_pipeline(const TcGeom& g, int* nstage, int* nsb) {
  const size_t lim = (size_t)max_dyn_smem();
  for (int sb = 2; sb >= 1; --sb) {
    int nst = 4;
    while (nst >= 2 && fwd_smem_bytes(g, nst, sb, nullptr) > lim) --nst;
    if (nst >= (sb == 2 ? 3 : 2)) {
      *nstage = nst;
      *nsb = sb;
      return true;
    }
  }
  return false;
}

bool eligible(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
              int dilation, int dtype, std::string* why, TcGeom* out_geom,
              int* out_nstage, int* out_nsb = nullptr) {
  auto no = [&](const char* m) { if (why) *why = m; return false; };
  if (dtype != LCB200_F16) return no("tensor-core engine needs float16 maps");
  if (dilation != 1) return no("tensor-core engine needs dilation 1");
  if (levels < 1 || levels > kMaxTcLevels) return no("tensor-core engine supports 1..4 levels");
  if (C % 64 != 0 || C < 64 || C > 256) return no("tensor-core engine needs C in {64,128,192,256}");
  if (!radius_supported(radius)) return no("tensor-core engine radius not instantiated");
  TcGeom g;
  if (!make_tc_geom(B, H1, W1, H2, W2, C, radius, levels, &g, why)) return false;
  if ((long long)B * H1 * W1 >= (1ll << 31)) return no("too many pixels");
  int nst = 0, nsb = 0;
  if (!fwd_pipeline(g, &nst, &nsb)) return no("tensor-core engine shared-memory budget exceeded");
  if (out_geom) *out_geom = g;
  if (out_nstage) *out_nstage = nst;
  if (out_nsb) *out_nsb = nsb;
  return true;
}

template <int RADIUS>
bool launch_fwd_kernel(const TcFwdParams& prm, size_t smem, cudaStream_t s) {
  auto k = tc_fwd_kernel<RADIUS>;
  if (!ensure_smem_attr((const void*)k, smem)) return false;
  k<<<num_sms(), fwd_threads(RADIUS), smem, s>>>(prm);
  count_launch();
  return check_launch("tc_fwd");
}

}  // namespace

bool tc_eligible(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
                 int dilation, int dtype, std::string* why) {
  return eligible(B, H1, W1, H2, W2, C, radius, levels, dilation, dtype, why, nullptr, nullptr);
}

size_t tc_workspace_bytes(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
                          bool backward) {
  TcGeom g;
  if (!make_tc_geom(B, H1, W1, H2, W2, C, radius, levels, &g, nullptr)) return 0;
  const WsLayout L = ws_layout(g);
  return backward ? L.total : L.fwd_total;
}

size_t tc_sort_state_bytes(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels) {
  TcGeom g;
  if (!make_tc_geom(B, H1, W1, H2, W2, C, radius, levels, &g, nullptr)) return 0;
  return ws_layout(g).sort_total;
}

// Deterministic CUDA-core grad_fmap2 (det_f2_pull_kernel): needs the pixel
// sort, hence dilation 1, 1..4 levels and a radius whose anchor-cell
// geometry exists. Workspace: the sort's buffers (everything the layout puts
// before the forward scratch).
bool tc_det_pull_ok(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
                    int dilation, std::string* why) {
  if (dilation != 1) { if (why) *why = "dilation 1"; return false; }
  if (levels < 1 || levels > kMaxTcLevels) { if (why) *why = "1..4 levels"; return false; }
  TcGeom g;
  std::string w;
  if (!make_tc_geom(B, H1, W1, H2, W2, C, radius, levels, &g, &w)) {
    if (why) *why = w;
    return false;
  }
  return true;
}

size_t tc_det_pull_bytes(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels) {
  TcGeom g;
  if (!make_tc_geom(B, H1, W1, H2, W2, C, radius, levels, &g, nullptr)) return 0;
  return ws_layout(g).scratch;
}

bool tc_det_f2_pull(const void* f1, const void* co, const void* gout, float* f2g, int B, int H1,
                    int W1, int H2, int W2, int C, int radius, int levels, int dtype, int cdtype,
                    bool ymajor, float scale, void* ws, size_t ws_bytes, cudaStream_t s) {
  TcGeom g;
  std::string why;
  if (!make_tc_geom(B, H1, W1, H2, W2, C, radius, levels, &g, &why)) {
    set_error("deterministic backward: " + why);
    return false;
  }
  const WsLayout L = ws_layout(g);
  if (ws_bytes < L.scratch || ws == nullptr) {
    set_error("deterministic backward: workspace too small");
    return false;
  }
  TcWs W = ws_pointers(nullptr, ws, L);
  if (!tc_sort(W, g, co, cdtype, s)) return false;
  const dim3 grid((unsigned)((long long)B * g.items_before[levels]), (unsigned)((C + 31) / 32));
#define LCB_PULL(T, TC)                                                                       \
  det_f2_pull_kernel<T, TC><<<grid, 128, 0, s>>>((const T*)f1, (const TC*)co, (const T*)gout, \
                                                 W.sorted, W.offsets, f2g, radius,            \
                                                 ymajor ? 1 : 0, scale, g)
  if (dtype == LCB200_F32) {
    if (cdtype == LCB200_F32) LCB_PULL(float, float);
    else LCB_PULL(float, __half);
  } else {
    if (cdtype == LCB200_F32) LCB_PULL(__half, float);
    else LCB_PULL(__half, __half);
  }
#undef LCB_PULL
  count_launch();
  return check_launch("det_f2_pull");
}

// sort_ws == nullptr: ws holds the whole workspace (sort state first);
// otherwise sort_ws receives the sort state and ws holds the rest.
bool tc_forward(const void* f1, const void* f2, const void* co, void* out, int B, int H1, int W1,
                int H2, int W2, int C, int radius, int levels, int cdtype, bool ymajor, float scale,
                void* sort_ws, void* ws, size_t ws_bytes, cudaStream_t s) {
  TcGeom g;
  int nst = 0, nsb = 0;
  std::string why;
  if (!eligible(B, H1, W1, H2, W2, C, radius, levels, 1, LCB200_F16, &why, &g, &nst, &nsb)) {
    set_error("tensor-core forward: " + why);
    return false;
  }
  const WsLayout L = ws_layout(g);
  if (ws_bytes < L.fwd_total - (sort_ws ? L.sort_total : 0)) {
    set_error("tensor-core forward: workspace too small");
    return false;
  }
  auto encode = get_encode_fn();
  if (!encode) {
    set_error("cuTensorMapEncodeTiled unavailable from the driver");
    return false;
  }
  TcWs W = ws_pointers(sort_ws, ws, L);
  if (!tc_sort(W, g, co, cdtype, s)) return false;
  int* sorted = W.sorted;
  int* inv = W.inv;
  int4* work = W.work;
  int* work_count = W.work_count;
  __half* scratch = W.scratch;

  TcFwdParams prm;
  memset(&prm, 0, sizeof(prm));
  for (int l = 0; l < levels; ++l) {
    const __half* base = static_cast<const __half*>(f2) + g.off[l];
    cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)g.w[l], (cuuint64_t)g.h[l], (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)C * 2, (cuuint64_t)g.w[l] * C * 2,
                             (cuuint64_t)g.batch_elems * 2};
    cuuint32_t box[4] = {64, (cuuint32_t)g.UW[l], (cuuint32_t)g.R[l], 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = encode(&prm.tmap[l], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, (void*)base, dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled failed for level " + std::to_string(l) + " (CUresult " +
                std::to_string((int)r) + ")");
      return false;
    }
  }
  prm.fmap1 = static_cast<const __half*>(f1);
  prm.coords = co;
  prm.sorted = sorted;
  prm.work = work;
  prm.work_count = work_count;
  prm.scratch = scratch;
  prm.scale = scale;
  prm.coords_f32 = cdtype == LCB200_F32;
  prm.ymajor = ymajor ? 1 : 0;
  prm.nstage = nst;
  prm.nsb = nsb;
  prm.g = g;
  const size_t smem = fwd_smem_bytes(g, nst, nsb, &prm.stage_bytes);
  bool ok = false;
  switch (radius) {
    case 3: ok = launch_fwd_kernel<3>(prm, smem, s); break;
    case 4: ok = launch_fwd_kernel<4>(prm, smem, s); break;
    case 8: ok = launch_fwd_kernel<8>(prm, smem, s); break;
    default: set_error("radius not instantiated"); return false;
  }
  if (!ok) return false;
  dim3 ug((g.HW + 127) / 128, levels, B);
  __half* o = static_cast<__half*>(out);
  switch (radius) {
    case 3: tc_unsort_kernel<3><<<ug, 128, 0, s>>>(scratch, inv, o, g); break;
    case 4: tc_unsort_kernel<4><<<ug, 128, 0, s>>>(scratch, inv, o, g); break;
    default: tc_unsort_kernel<8><<<ug, 128, 0, s>>>(scratch, inv, o, g); break;
  }
  count_launch();
  return check_launch("tc_unsort");
}

namespace {

size_t bwd1_stage_bytes(const TcGeom& g) { return 16384 + (size_t)g.KC * 8192; }
// A: two 64-position halves of 64 rows; B: KC 64-channel chunks of 64 rows
size_t bwd2_stage_bytes(const TcGeom& g) { return (size_t)(2 + g.KC) * kB2Rows * 128; }
constexpr size_t kBwd2Extra = 512;  // barriers after the stages
size_t bwd2_smem_bytes(int nstage, size_t stage) { return 1024 + (size_t)nstage * stage + kBwd2Extra; }

int pick_stages(size_t stage, size_t extra, int maxst) {
  const size_t lim = (size_t)max_dyn_smem();
  int n = maxst;
  while (n >= 2 && 1024 + n * stage + extra > lim) --n;
  return n;
}

bool bwd_eligible(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
                  int dilation, int dtype, std::string* why, TcGeom* out, int* nst1,
                  int* nst2) {
  TcGeom g;
  int nf = 0;
  if (!eligible(B, H1, W1, H2, W2, C, radius, levels, dilation, dtype, why, &g, &nf)) return false;
  const int nbg = 2;
  const int n1 = pick_stages(bwd1_stage_bytes(g), 256, 4);
  const int n2 = pick_stages(bwd2_stage_bytes(g), kBwd2Extra, 8);
  if (n1 < 2 || n2 < 2) {
    if (why) *why = "tensor-core backward shared-memory budget exceeded";
    return false;
  }
  if (out) *out = g;
  if (nst1) *nst1 = n1 * 4 + nbg;  // packed: stages, builder groups
  if (nst2) *nst2 = n2;
  return true;
}

template <int RADIUS>
bool launch_pull(const TcPullParams& p2, cudaStream_t s) {
  const size_t smem2 = std::max<size_t>(bwd2_smem_bytes(p2.nstage, p2.stage_bytes), 120 * 1024);
  auto k2 = tc_bwd2_kernel<RADIUS>;
  if (!ensure_smem_attr((const void*)k2, smem2)) return false;
  k2<<<num_sms(), kBwd2Threads, smem2, s>>>(p2);
  count_launch();
  return check_launch("tc_bwd2");
}

template <int RADIUS>
bool launch_bwd_kernels(const TcBwdParams& p1, const TcPullParams& p2, const __half* corr_grad,
                        const int* inv, uint4* gsh, float scale, int ymajor, bool pull,
                        cudaStream_t s) {
  const TcGeom& g = p1.g;
  using GS = GintShape<RADIUS>;
  // 16-byte loads (and TMA rows) of the incoming gradient need HW % 8 == 0
  // and an aligned base
  const int vec_ok = (g.HW % 8 == 0) && (reinterpret_cast<uintptr_t>(corr_grad) % 16 == 0);
  auto encode = get_encode_fn();
  CUtensorMap gmap;
  bool tma = false;
  if (vec_ok && GS::tma_ok && encode) {
    // corr_grad as [B*L*RD*RD rows][HW], boxes of RD*RD rows x 128 pixels
    cuuint64_t dims[2] = {(cuuint64_t)g.HW, (cuuint64_t)g.B * g.L * g.RD2};
    cuuint64_t strides[1] = {(cuuint64_t)g.HW * 2};
    cuuint32_t box[2] = {128, (cuuint32_t)g.RD2};
    cuuint32_t estr[2] = {1, 1};
    tma = encode(&gmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)corr_grad, dims, strides, box,
                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  if (tma) {
    auto k0 = tc_gint_tma_kernel<RADIUS>;
    const size_t smem0 = GS::tma_smem_bytes;
    if (!ensure_smem_attr((const void*)k0, smem0)) return false;
    const int nblk = (g.HW + 127) / 128;
    const int nruns = nblk * g.L * g.B;
    const int per_sm = std::max(1, (int)((size_t)max_dyn_smem() / (smem0 + 1024)));
    const int grid = std::min(nruns, num_sms() * per_sm);
    k0<<<grid, 128, smem0, s>>>(gmap, p1.coords, p1.coords_f32, inv, gsh,
                                const_cast<int*>(p1.sbase), p1.grad_f1, ymajor, p1.acc_f1, nblk,
                                nruns, p2.item_next, g);
  } else {
    dim3 ug((g.HW + 127) / 128, g.L, g.B);
    auto k0 = tc_gint_kernel<RADIUS>;
    const size_t smem0 = GS::smem_bytes;
    if (!ensure_smem_attr((const void*)k0, smem0)) return false;
    k0<<<ug, 128, smem0, s>>>(corr_grad, p1.coords, p1.coords_f32, inv, gsh,
                              const_cast<int*>(p1.sbase), p1.grad_f1, ymajor, vec_ok, p1.acc_f1,
                              p2.item_next, g);
  }
  count_launch();
  if (!check_launch("tc_gint")) return false;
  const size_t smem1 = 1024 + (size_t)p1.nstage * p1.stage_bytes + 256;
  auto k1 = tc_bwd1_kernel<RADIUS>;
  if (!ensure_smem_attr((const void*)k1, smem1)) return false;
  k1<<<num_sms(), 64 + 128 * p1.nbg + 128, smem1, s>>>(p1);
  count_launch();
  if (!check_launch("tc_bwd1")) return false;
  return pull ? launch_pull<RADIUS>(p2, s) : true;
}

}  // namespace

bool tc_bwd_eligible(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
                     int dilation, int dtype, std::string* why) {
  return bwd_eligible(B, H1, W1, H2, W2, C, radius, levels, dilation, dtype, why, nullptr, nullptr,
                      nullptr);
}

// sort_ws == nullptr: sort the coords into ws (single-buffer layout);
// otherwise sort_ws holds the sort a forward made of the same coords and
// geometry (tc_forward with that buffer) and ws holds the rest.
// A lookup's grad_fmap2 records kept for a later multi-lookup pull: the
// sorted fmap1 copy, the packed level bases and the pre-shifted records.
struct RecLayout {
  size_t f1s, sbase, gsh, total;
};
RecLayout rec_layout(const TcGeom& g) {
  RecLayout r{};
  size_t o = 0;
  r.f1s = o; o = align256(o + (size_t)g.npix * g.C * 2);
  r.sbase = o; o = align256(o + (size_t)g.L * g.npix * 4);
  r.gsh = o; o = align256(o + (size_t)g.L * g.npix * g.NG * g.NU * 16);
  r.total = o;
  return r;
}

// records == nullptr: the whole backward. Else grad_fmap1 only; the sorted
// fmap1 copy, level bases and gradient records go to `records` for
// tc_pull_lookups.
bool tc_backward_impl(const void* f1, const void* f2, const void* co, const void* gout, void* f1g,
                      float* f2g, int B, int H1, int W1, int H2, int W2, int C, int radius,
                      int levels, int cdtype, bool ymajor, float scale, bool acc_f1, void* sort_ws,
                      void* ws, size_t ws_bytes, void* records, size_t records_bytes,
                      cudaStream_t s) {
  TcGeom g;
  int n1 = 0, n2 = 0;
  std::string why;
  if (!bwd_eligible(B, H1, W1, H2, W2, C, radius, levels, 1, LCB200_F16, &why, &g, &n1, &n2)) {
    set_error("tensor-core backward: " + why);
    return false;
  }
  const WsLayout L = ws_layout(g);
  if (ws_bytes < L.total - (sort_ws ? L.sort_total : 0)) {
    set_error("tensor-core backward: workspace too small");
    return false;
  }
  auto encode = get_encode_fn();
  if (!encode) {
    set_error("cuTensorMapEncodeTiled unavailable from the driver");
    return false;
  }
  TcWs W = ws_pointers(sort_ws, ws, L);
  if (records) {
    const RecLayout R = rec_layout(g);
    if (records_bytes < R.total || (reinterpret_cast<uintptr_t>(records) & 255)) {
      set_error("tensor-core backward: records buffer too small or not 256-byte aligned");
      return false;
    }
    uint8_t* rb = static_cast<uint8_t*>(records);
    W.f1s = reinterpret_cast<__half*>(rb + R.f1s);
    W.sbase = reinterpret_cast<int*>(rb + R.sbase);
    W.gsh = reinterpret_cast<uint4*>(rb + R.gsh);
  }
  if (!sort_ws && !tc_sort(W, g, co, cdtype, s)) return false;
  {
    // 8 warps per block, kGatherRows rows per warp
    const int rows_per_block = 8 * kGatherRows;
    const long long nb = (g.npix + rows_per_block - 1) / rows_per_block;
    tc_gather_rows_kernel<<<(unsigned)nb, 256, 0, s>>>(
        static_cast<const __half*>(f1), W.sorted, W.offsets + (size_t)g.B * g.ncell * kColBins, W.f1s, g);
    count_launch();
    if (!check_launch("tc_gather_rows")) return false;
  }

  TcBwdParams p1;
  memset(&p1, 0, sizeof(p1));
  for (int l = 0; l < levels; ++l) {
    const __half* base = static_cast<const __half*>(f2) + g.off[l];
    cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)g.w[l], (cuuint64_t)g.h[l], (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)C * 2, (cuuint64_t)g.w[l] * C * 2,
                             (cuuint64_t)g.batch_elems * 2};
    cuuint32_t box[4] = {64, (cuuint32_t)g.UWb[l], (cuuint32_t)g.Rg[l], 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = encode(&p1.tmap[l], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, (void*)base, dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled failed for level " + std::to_string(l));
      return false;
    }
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)C, (cuuint64_t)g.npix};
    cuuint64_t strides[1] = {(cuuint64_t)C * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)kB2Rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&p1.tmap_f1s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)W.f1s, dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled failed for the sorted fmap1 copy");
      return false;
    }
  }
  p1.coords = co;
  p1.coords_f32 = cdtype == LCB200_F32;
  p1.sorted = W.sorted;
  p1.counts = W.counts;
  p1.offsets = W.offsets;
  p1.work = W.work;
  p1.work_count = W.work_count;
  p1.gsh = W.gsh;
  p1.sbase = W.sbase;
  p1.fmap1 = static_cast<const __half*>(f1);
  p1.grad_f1 = static_cast<__half*>(f1g);
  p1.grad_f2 = f2g;
  p1.acc_f1 = acc_f1 ? 1 : 0;
  p1.scale = scale;
  p1.g = g;
  p1.nitems = (long long)B * g.items_before[levels];
  p1.item_next = W.wctr;
  TcPullParams p2;
  memset(&p2, 0, sizeof(p2));
  p2.tmap_f1s[0] = p1.tmap_f1s;
  p2.offsets[0] = p1.offsets;
  p2.gsh[0] = p1.gsh;
  p2.sbase[0] = p1.sbase;
  p2.nlook = 1;
  p2.grad_f2 = f2g;
  p2.nstage = n2;
  p2.stage_bytes = (uint32_t)bwd2_stage_bytes(g);
  p2.nitems = p1.nitems;
  p2.item_next = p1.item_next;
  p2.scale = scale;
  p2.g = g;
  p1.nstage = n1 / 4;
  p1.nbg = n1 % 4;
  p1.stage_bytes = (uint32_t)bwd1_stage_bytes(g);
  const __half* cg = static_cast<const __half*>(gout);
  const bool pull = records == nullptr;
  switch (radius) {
    case 3: return launch_bwd_kernels<3>(p1, p2, cg, W.inv, W.gsh, scale, ymajor, pull, s);
    case 4: return launch_bwd_kernels<4>(p1, p2, cg, W.inv, W.gsh, scale, ymajor, pull, s);
    case 8: return launch_bwd_kernels<8>(p1, p2, cg, W.inv, W.gsh, scale, ymajor, pull, s);
    default: set_error("radius not instantiated"); return false;
  }
}

bool tc_backward(const void* f1, const void* f2, const void* co, const void* gout, void* f1g,
                 float* f2g, int B, int H1, int W1, int H2, int W2, int C, int radius,
                 int levels, int cdtype, bool ymajor, float scale, bool acc_f1, void* sort_ws,
                 void* ws, size_t ws_bytes, cudaStream_t s) {
  return tc_backward_impl(f1, f2, co, gout, f1g, f2g, B, H1, W1, H2, W2, C, radius, levels,
                          cdtype, ymajor, scale, acc_f1, sort_ws, ws, ws_bytes, nullptr, 0, s);
}

bool tc_backward_fmap1(const void* f1, const void* f2, const void* co, const void* gout,
                       void* f1g, int B, int H1, int W1, int H2, int W2, int C, int radius,
                       int levels, int cdtype, bool ymajor, float scale, bool acc_f1,
                       void* sort_ws, void* ws, size_t ws_bytes, void* records,
                       size_t records_bytes, cudaStream_t s) {
  if (!records) {
    set_error("grad_fmap1 backward: records buffer required");
    return false;
  }
  return tc_backward_impl(f1, f2, co, gout, f1g, nullptr, B, H1, W1, H2, W2, C, radius, levels,
                          cdtype, ymajor, scale, acc_f1, sort_ws, ws, ws_bytes, records,
                          records_bytes, s);
}

size_t tc_records_bytes(int B, int H1, int W1, int H2, int W2, int C, int radius, int levels) {
  TcGeom g;
  if (!make_tc_geom(B, H1, W1, H2, W2, C, radius, levels, &g, nullptr)) return 0;
  return rec_layout(g).total;
}

// grad_fmap2 of n lookups of one pair of maps, from their kept sorts and
// records: passes of up to kMaxPull lookups, each one grad_fmap2 kernel whose
// output tiles sum every lookup's candidates before one add.
bool tc_pull_lookups(const void* const* sort_states, const void* const* records, int n,
                     float* f2g, int B, int H1, int W1, int H2, int W2, int C, int radius,
                     int levels, float scale, void* ws, size_t ws_bytes, cudaStream_t s) {
  TcGeom g;
  int n1 = 0, n2 = 0;
  std::string why;
  if (!bwd_eligible(B, H1, W1, H2, W2, C, radius, levels, 1, LCB200_F16, &why, &g, &n1, &n2)) {
    set_error("grad_fmap2 pull: " + why);
    return false;
  }
  if (n <= 0) return true;
  if (!ws || ws_bytes < 256 || (reinterpret_cast<uintptr_t>(ws) & 255)) {
    set_error("grad_fmap2 pull: workspace of 256 aligned bytes required");
    return false;
  }
  auto encode = get_encode_fn();
  if (!encode) {
    set_error("cuTensorMapEncodeTiled unavailable from the driver");
    return false;
  }
  const WsLayout L = ws_layout(g);
  const RecLayout R = rec_layout(g);
  for (int i0 = 0; i0 < n; i0 += kMaxPull) {
    const int m = std::min(kMaxPull, n - i0);
    TcPullParams p;
    memset(&p, 0, sizeof(p));
    for (int j = 0; j < m; ++j) {
      const uint8_t* st = static_cast<const uint8_t*>(sort_states[i0 + j]);
      const uint8_t* rb = static_cast<const uint8_t*>(records[i0 + j]);
      if (!st || !rb || ((reinterpret_cast<uintptr_t>(st) | reinterpret_cast<uintptr_t>(rb)) & 255)) {
        set_error("grad_fmap2 pull: sort states and records must be 256-byte aligned buffers");
        return false;
      }
      p.offsets[j] = reinterpret_cast<const int*>(st + L.offsets);
      p.sbase[j] = reinterpret_cast<const int*>(rb + R.sbase);
      p.gsh[j] = reinterpret_cast<const uint4*>(rb + R.gsh);
      cuuint64_t dims[2] = {(cuuint64_t)C, (cuuint64_t)g.npix};
      cuuint64_t strides[1] = {(cuuint64_t)C * 2};
      cuuint32_t box[2] = {64, (cuuint32_t)kB2Rows};
      cuuint32_t estr[2] = {1, 1};
      CUresult r = encode(&p.tmap_f1s[j], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                          const_cast<uint8_t*>(rb + R.f1s), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed for a kept sorted fmap1 copy");
        return false;
      }
    }
    p.nlook = m;
    p.grad_f2 = f2g;
    p.nstage = n2;
    p.stage_bytes = (uint32_t)bwd2_stage_bytes(g);
    p.nitems = (long long)B * g.items_before[levels];
    p.item_next = static_cast<int*>(ws);
    p.scale = scale;
    p.g = g;
    if (cudaMemsetAsync(ws, 0, sizeof(int), s) != cudaSuccess) return check_launch("memset");
    bool ok = false;
    switch (radius) {
      case 3: ok = launch_pull<3>(p, s); break;
      case 4: ok = launch_pull<4>(p, s); break;
      case 8: ok = launch_pull<8>(p, s); break;
      default: set_error("radius not instantiated"); return false;
    }
    if (!ok) return false;
  }
  return true;
}

int tc_device_status(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int));
  if (reset) {
    const int z = 0;
    cudaMemcpyToSymbol(g_tc_status, &z, sizeof(int));
  }
  return v;
}

LCB_BOUNDS_READER(bounds_read_tc)

}  // namespace lcb200

// ---------------------------------------------------------------------------
// Allocation-free forward: the tensor-core forward with its scratch in a
// fixed device array instead of a caller workspace or an allocator, for
// callers that may not allocate while they run (TensorRT enqueue, CUDA graph
// capture, runtimes with memory fixed at start-up).
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[LCB200_NOALLOC_SCRATCH_BYTES];

namespace lcb200 {
namespace {
// Device address of g_noalloc_scratch on the current device (the host-side
// name is only a stand-in). Looked up on every call, so a context that was
// torn down and re-created (cudaDeviceReset) never sees a stale address.
void* noalloc_scratch_ptr() {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    set_error(std::string("no-alloc forward: cudaGetSymbolAddress failed: ") +
              cudaGetErrorString(e));
    return nullptr;
  }
  return p;
}
}  // namespace

}  // namespace lcb200

extern "C" bool launchLocalCorrB200PyramidForwardNoAlloc(
    const void* fmap1, const void* fmap2_packed, const void* coords, void* corr, int B, int H1,
    int W1, int C, int radius, int levels, int dtype, int coords_dtype, bool ymajor, float scale,
    cudaStream_t stream) {
  using namespace lcb200;
  clear_error();
  if (B <= 0 || (long long)H1 * W1 <= 0) return true;
  if (levels < 1 || levels > kMaxTcLevels) {
    set_error("no-alloc forward: levels must be in [1, 4] (got " + std::to_string(levels) + ")");
    return false;
  }
  for (int l = 0; l < levels; ++l) {
    if ((H1 >> l) < 1 || (W1 >> l) < 1) {
      set_error("level " + std::to_string(l) + " of a " + std::to_string(H1) + "x" +
                std::to_string(W1) + " map is empty");
      return false;
    }
  }
  if (coords_dtype != LCB200_F32 && coords_dtype != LCB200_F16) {
    set_error("coords dtype must be LCB200_F32 (0) or LCB200_F16 (1)");
    return false;
  }
  std::string why;
  if (!tc_eligible(B, H1, W1, H1, W1, C, radius, levels, 1, dtype, &why)) {
    set_error("no-alloc forward supports only tensor-core configurations: " + why);
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(fmap1) | reinterpret_cast<uintptr_t>(fmap2_packed)) & 15) {
    set_error("no-alloc forward: maps must be 16-byte aligned");
    return false;
  }
  const size_t need = tc_workspace_bytes(B, H1, W1, H1, W1, C, radius, levels, false);
  if (need > LCB200_NOALLOC_SCRATCH_BYTES) {
    set_error("no-alloc forward: this problem needs " + std::to_string(need) +
              " bytes of scratch, more than the fixed " +
              std::to_string((unsigned long long)LCB200_NOALLOC_SCRATCH_BYTES) +
              " bytes the allocation-free entry point holds; use "
              "launchLocalCorrB200PyramidForward with a workspace");
    return false;
  }
  void* ws = noalloc_scratch_ptr();
  if (!ws) return false;
  return bounds_finish(tc_forward(fmap1, fmap2_packed, coords, corr, B, H1, W1, H1, W1, C,
                                  radius, levels, coords_dtype, ymajor, scale, nullptr, ws,
                                  LCB200_NOALLOC_SCRATCH_BYTES, stream),
                       stream);
}
