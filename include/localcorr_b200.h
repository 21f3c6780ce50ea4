/*
 * localcorr_b200 — C ABI of the B200 (sm_100a) local-correlation library
 * (liblocalcorr_b200.so).
 *
 * Tensor contract shared by every pyramid entry point (identical to the
 * contract of the reference library's launchers):
 *   fmap1        [B, H1, W1, C]           contiguous, NHWC
 *   fmap2_packed [B, C * sum_l h_l * w_l] contiguous, batch-major; level l of
 *                batch b starts at b*P + C*sum_{j<l} h_j*w_j and is NHWC;
 *                h_l = H1 >> l, w_l = W1 >> l
 *   coords       [B, 2, H1, W1]           contiguous, planar (x, then y),
 *                                         level-0 pixel units
 *   corr         [B, levels, RD*RD, H1, W1], RD = 2*radius+1
 *   corr[b,l,d,h,w] = sum_c fmap1[b,h,w,c] *
 *        bilinear(fmap2_l[b], coords[b,:,h,w]/2^l + dilation*(ix-r, iy-r))[c]
 *   with zero padding outside fmap2_l, d = iy + RD*ix (ymajor=false, RAFT
 *   order) or d = ix + RD*iy (ymajor=true, spatial-sampler order).
 *
 * All launchers are asynchronous on `stream`, never synchronise the host and
 * return true on success (or for an empty problem: B <= 0 or H1*W1 <= 0) and
 * false for an invalid configuration or a launch error; the reason is then
 * available from localCorrB200GetLastError() (thread-local).
 *
 * dtype codes: LCB200_F32 = 0 (float32), LCB200_F16 = 1 (float16).
 */
#ifndef LOCALCORR_B200_H
#define LOCALCORR_B200_H

#include <stddef.h>
#include <stdbool.h>
#include <cuda_runtime.h>

#if defined(__GNUC__)
#define LCB200_API __attribute__((visibility("default")))
#else
#define LCB200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LCB200_F32 0
#define LCB200_F16 1

/* Engine selection for the extended pyramid launchers. */
#define LCB200_ENGINE_AUTO 0    /* tensor-core engine when eligible, else CUDA-core */
#define LCB200_ENGINE_SIMT 1    /* CUDA-core engine, every configuration */
#define LCB200_ENGINE_TC 2      /* tensor-core engine; fails if not eligible */

/* ---- Reference-compatible entry points ------------------------------------
 * Same symbol names, argument order, argument meaning and error behaviour as
 * the reference library, so its ctypes loader (blocks.py:74-131) and its
 * TensorRT plugin enqueue (cuda_pyramid/localcorr_cuda_pyramid_plugin.cpp:
 * 164-199) bind to this library unchanged.
 */

/* Replaces launchLocalCorrCudaPyramidForward,
 * cuda_pyramid/localcorr_cuda_pyramid_kernel.h:39-53. isHalf selects float16
 * for every pointer. Scratch, when the tensor-core engine needs it, comes from
 * one buffer per device owned by the library (grown on demand with
 * cudaMallocAsync/cudaFreeAsync); a call on another stream than the previous
 * call first waits, on the GPU, for that call's kernels (an event), so calls
 * from several streams or threads are safe and run one after the other. */
LCB200_API bool launchLocalCorrCudaPyramidForward(
    const void* fmap1, const void* fmap2_packed, const void* coords, void* corr,
    int B, int H1, int W1, int C, int radius, int levels, int dilation,
    bool isHalf, bool ymajor, cudaStream_t stream);

/* Replaces launchLocalCorrCudaPyramidBackward,
 * cuda_pyramid/localcorr_cuda_pyramid_kernel.h:82-98. fmap1_grad is written
 * in the input dtype; fmap2_grad must be a zero-initialised float32 buffer
 * with fmap2_packed's element count and receives the fmap2 gradient
 * (accumulated, so several calls may share it). coords get no gradient. */
LCB200_API bool launchLocalCorrCudaPyramidBackward(
    const void* fmap1, const void* fmap2_packed, const void* coords,
    const void* corr_grad, void* fmap1_grad, float* fmap2_grad,
    int B, int H1, int W1, int C, int radius, int levels, int dilation,
    bool isHalf, bool ymajor, cudaStream_t stream);

/* ---- Extended pyramid entry points (no reference counterpart beyond the
 * launchers above: they add an output scale, an engine choice and a
 * caller-provided workspace) ------------------------------------------------ */

/* Bytes of workspace the pyramid forward/backward need for this shape and
 * engine (0 when the engine needs none). */
LCB200_API size_t localCorrB200PyramidWorkspaceBytes(
    int B, int H1, int W1, int C, int radius, int levels, int dilation,
    int dtype, int engine);

/* corr = scale * (the reference forward). The 1/sqrt(C) of the RAFT block
 * (blocks.py:411) is passed as scale instead of a separate division pass.
 * coords_dtype may differ from dtype (float32 coords with float16 maps keep
 * sub-pixel precision at large coordinates).
 * workspace may be NULL when localCorrB200PyramidWorkspaceBytes() is 0;
 * otherwise it must hold at least that many bytes (256-byte aligned). */
LCB200_API bool launchLocalCorrB200PyramidForward(
    const void* fmap1, const void* fmap2_packed, const void* coords, void* corr,
    int B, int H1, int W1, int C, int radius, int levels, int dilation,
    int dtype, int coords_dtype, bool ymajor, float scale, int engine,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Backward of launchLocalCorrB200PyramidForward (gradient of the scaled
 * output). accumulate is a set of flags:
 *   LCB200_ACC_FMAP2: add into fmap2_grad_f32 (float32, fmap2_packed's element
 *                     count) instead of overwriting it;
 *   LCB200_ACC_FMAP1: add into fmap1_grad (dtype) instead of overwriting it.
 * (1 = LCB200_ACC_FMAP2 keeps the meaning of a plain `true`.) Accumulating
 * both lets the lookups of one pair of maps share one pair of gradient
 * buffers instead of summing per-lookup gradients afterwards. */
#define LCB200_ACC_FMAP2 1
#define LCB200_ACC_FMAP1 2
LCB200_API bool launchLocalCorrB200PyramidBackward(
    const void* fmap1, const void* fmap2_packed, const void* coords,
    const void* corr_grad, void* fmap1_grad, float* fmap2_grad_f32,
    int B, int H1, int W1, int C, int radius, int levels, int dilation,
    int dtype, int coords_dtype, bool ymajor, float scale, int accumulate, int engine,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* ---- Separate map size (no reference counterpart: the reference derives the
 * pyramid from fmap1's H1 x W1) ---------------------------------------------
 * The three calls above with the pixel grid (fmap1, coords, corr, corr_grad:
 * H1 x W1) decoupled from the level-0 size of the map fmap2_packed was built
 * from (H2 x W2; level l is (H2 >> l) x (W2 >> l)). coords stay in level-0
 * pixels of the map. A row band of a large frame (rows [y0, y1) of fmap1 and
 * coords, H1 = y1 - y0) against the whole frame's pyramid (H2 = H) gives
 * exactly rows [y0, y1) of the whole-frame output, which is how one frame is
 * split over several GPUs. With H2 = H1 and W2 = W1 they are the calls
 * above. */
LCB200_API size_t localCorrB200PyramidWorkspaceBytesMapDims(
    int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
    int dilation, int dtype, int engine);
LCB200_API bool launchLocalCorrB200PyramidForwardMapDims(
    const void* fmap1, const void* fmap2_packed, const void* coords, void* corr,
    int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
    int dilation, int dtype, int coords_dtype, bool ymajor, float scale,
    int engine, void* workspace, size_t workspace_bytes, cudaStream_t stream);
LCB200_API bool launchLocalCorrB200PyramidBackwardMapDims(
    const void* fmap1, const void* fmap2_packed, const void* coords,
    const void* corr_grad, void* fmap1_grad, float* fmap2_grad_f32,
    int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
    int dilation, int dtype, int coords_dtype, bool ymajor, float scale,
    int accumulate, int engine, void* workspace, size_t workspace_bytes,
    cudaStream_t stream);

/* ---- Sort reuse between a forward and its backward (no reference
 * counterpart: the reference has no per-call state) -------------------------
 * The tensor-core engine sorts the pixels by where their windows land before
 * every forward and every backward. A training step runs the backward of each
 * lookup with the coordinates of its forward, so the sort can be made once:
 * ...ForwardKeepSort writes it to a caller buffer (sort_state, at least
 * localCorrB200PyramidSortStateBytes() bytes, a few MB per lookup) and the
 * matching ...BackwardWithSort reads it instead of sorting again. Arguments
 * are those of the ...MapDims calls; `workspace` then needs only
 * localCorrB200PyramidWorkspaceBytesMapDims() - SortStateBytes() bytes
 * (the sort state is not part of it). The backward must get the same coords,
 * geometry and engine as the forward that filled sort_state, and sort_state
 * must be left untouched in between. When the configuration runs on the
 * CUDA-core engine SortStateBytes() is 0 and sort_state is ignored. */
LCB200_API size_t localCorrB200PyramidSortStateBytes(
    int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
    int dilation, int dtype, int engine);
LCB200_API bool launchLocalCorrB200PyramidForwardKeepSort(
    const void* fmap1, const void* fmap2_packed, const void* coords, void* corr,
    int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
    int dilation, int dtype, int coords_dtype, bool ymajor, float scale,
    int engine, void* sort_state, size_t sort_state_bytes, void* workspace,
    size_t workspace_bytes, cudaStream_t stream);
LCB200_API bool launchLocalCorrB200PyramidBackwardWithSort(
    const void* fmap1, const void* fmap2_packed, const void* coords,
    const void* corr_grad, void* fmap1_grad, float* fmap2_grad_f32,
    int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
    int dilation, int dtype, int coords_dtype, bool ymajor, float scale,
    int accumulate, int engine, const void* sort_state, size_t sort_state_bytes,
    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* ---- Allocation-free forward (no counterpart in the reference) -------------
 * Some callers may not allocate device memory at the time they run the
 * correlation: a TensorRT plugin's enqueue (the engine's memory is fixed when
 * it is built), code recorded while a CUDA graph is being captured, or a
 * serving runtime that reserves all of its memory at start-up. This entry
 * point computes the same result as launchLocalCorrB200PyramidForward with
 * the tensor-core engine, but takes its scratch from a fixed array that the
 * library holds on every GPU that loads it (LCB200_NOALLOC_SCRATCH_BYTES, kept
 * until the process exits) instead of from the caller or an allocator; it
 * calls no cudaMalloc/cudaFree.
 *  - Only tensor-core configurations: float16 maps, dilation 1, 1..4 levels,
 *    C in {64,128,192,256}, radius in {3,4,8}; coords float16 or float32.
 *  - Problems whose scratch (localCorrB200PyramidWorkspaceBytes) exceeds
 *    LCB200_NOALLOC_SCRATCH_BYTES are rejected (false, message says so).
 *  - Every call looks up the array's device address on the current device
 *    (cudaGetSymbolAddress, no allocation); the first call on a device may
 *    also load the library's device code, so make that first call before
 *    any stream capture.
 *  - All calls on a device share the one array: calls that can overlap on
 *    the GPU (different streams, no ordering) race and must be serialised by
 *    the caller. Each call starts from a cleared state (no carry-over). */
#define LCB200_NOALLOC_SCRATCH_BYTES (32ull << 20)
LCB200_API bool launchLocalCorrB200PyramidForwardNoAlloc(
    const void* fmap1, const void* fmap2_packed, const void* coords, void* corr,
    int B, int H1, int W1, int C, int radius, int levels,
    int dtype, int coords_dtype, bool ymajor, float scale, cudaStream_t stream);

/* ---- Layout preparation (replaces the torch permute/avg_pool2d/cat chain of
 * LocalCorrCudaPyramidBlock.__init__, blocks.py:369-383) ------------------- */

/* fmap2 [B,C,H,W] (NCHW) -> fmap2_packed (layout above), levels built by 2x2
 * average pooling with floor-halved dims, each level pooled from the previous
 * level's dtype-rounded values as torch's avg_pool2d chain does. */
LCB200_API bool launchLocalCorrB200PyramidBuild(
    const void* fmap2_nchw, void* fmap2_packed,
    int B, int C, int H, int W, int levels, int dtype, cudaStream_t stream);

/* Gradient of launchLocalCorrB200PyramidBuild: grad_packed (float32 when
 * grad_is_f32, else dtype) -> grad_fmap2_nchw (dtype, overwritten). */
LCB200_API bool launchLocalCorrB200PyramidBuildBackward(
    const void* grad_packed, bool grad_is_f32, void* grad_fmap2_nchw,
    int B, int C, int H, int W, int levels, int dtype, cudaStream_t stream);

/* [B, C, HW] <-> [B, HW, C] layout transposes (fmap1 NCHW <-> NHWC). */
LCB200_API bool launchLocalCorrB200NchwToNhwc(const void* in, void* out, int B, int C,
                                   int HW, int dtype, cudaStream_t stream);
LCB200_API bool launchLocalCorrB200NhwcToNchw(const void* in, void* out, int B, int C,
                                   int HW, int dtype, cudaStream_t stream);

/* ---- Spatial (PWC-Net) correlation ---------------------------------------
 * Replaces the sampler path LocalCorrCudaSpatialSampler (blocks.py:671-694)
 * / LocalCorrCudaPyramidSampler (spatial_corr.py:328-376), which runs the
 * pyramid launcher with levels=1, ymajor and identity coords:
 *   out[b, iy, ix, h, w] = scale * sum_c in1[b,c,h,w] *
 *                          in2[b, c, h + dil*(iy-r), w + dil*(ix-r)]
 * (zero outside), in1/in2 [B,C,H,W] NCHW, out [B, RD, RD, H, W]. */
LCB200_API bool launchLocalCorrB200SpatialForward(
    const void* in1, const void* in2, void* out,
    int B, int C, int H, int W, int radius, int dilation, int dtype,
    float scale, cudaStream_t stream);

/* Gradients of the spatial correlation; grad_in1/grad_in2 (dtype, NCHW) are
 * overwritten. Either may be NULL to skip it. */
LCB200_API bool launchLocalCorrB200SpatialBackward(
    const void* in1, const void* in2, const void* grad_out,
    void* grad_in1, void* grad_in2,
    int B, int C, int H, int W, int radius, int dilation, int dtype,
    float scale, cudaStream_t stream);

/* ---- Diagnostics ---------------------------------------------------------- */

/* Message of the last failed call on this thread ("" if none). */
LCB200_API const char* localCorrB200GetLastError(void);

/* Error status raised on the device by the tensor-core kernels (0 = none;
 * 1 = a pipeline wait timed out and the kernel stopped early). Synchronises
 * with the current device; reset clears it. */
LCB200_API int localCorrB200DeviceStatus(int reset);

/* Library ABI version (major*10000 + minor*100 + patch). */
LCB200_API int localCorrB200Version(void);

/* Number of kernel launches issued by this library in this process (all
 * host threads) since the last reset (diagnostics for launch accounting in
 * benchmarks). */
LCB200_API long long localCorrB200LaunchCount(int reset);

/* ---- Deferred grad_fmap2 for many lookups of one pair of maps -------------
 * No reference counterpart (the reference runs one backward per lookup).
 * A RAFT block runs many lookups against the same fmap1/fmap2. Instead of
 * adding every lookup's grad_fmap2 into the float32 gradient pyramid (one
 * read-modify-write of the whole pyramid per lookup), a training step can
 * (1) per lookup, with the sort its ...ForwardKeepSort left, compute grad_fmap1
 * and keep the lookup's grad_fmap2 records in a caller buffer of
 * localCorrB200PyramidRecordsBytes(...) bytes, then (2) once, pull
 * grad_fmap2 over all those lookups: every output tile sums the candidates
 * of up to 12 lookups in one accumulator before one add. Tensor-core
 * engine only (float16 maps, dilation 1); buffers 256-byte aligned.
 * ...BackwardFmap1: workspace as for ...BackwardWithSort; accumulate:
 * LCB200_ACC_FMAP1. ...BackwardFmap2Pull: sort_states[i] / records[i] are
 * device pointers (a host array of nlookups each); workspace >= 256 bytes;
 * accumulate: LCB200_ACC_FMAP2 adds into fmap2_grad_f32, else it is
 * overwritten. The maps, scale and channel order are those of the lookups. */
LCB200_API size_t localCorrB200PyramidRecordsBytes(int B, int H1, int W1, int H2, int W2, int C,
                                                   int radius, int levels);
LCB200_API bool launchLocalCorrB200PyramidBackwardFmap1(
    const void* fmap1, const void* fmap2_packed, const void* coords, const void* corr_grad,
    void* fmap1_grad, int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
    int coords_dtype, bool ymajor, float scale, int accumulate, const void* sort_state,
    size_t sort_state_bytes, void* records, size_t records_bytes, void* workspace,
    size_t workspace_bytes, cudaStream_t stream);
LCB200_API bool launchLocalCorrB200PyramidBackwardFmap2Pull(
    const void* const* sort_states, const void* const* records, int nlookups,
    float* fmap2_grad_f32, int B, int H1, int W1, int H2, int W2, int C, int radius, int levels,
    float scale, int accumulate, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* ---- Deterministic mode ---------------------------------------------------
 * No reference counterpart (the reference's backward adds grad_fmap2 with
 * float atomics, cuda_pyramid/localcorr_cuda_pyramid_kernel.cu:909-916).
 * When on (process-wide, off by default), the tensor-core engine sorts the
 * pixels of a lookup in a fixed order (forward and backward) and adds every
 * grad_fmap2 position once per call, so repeated calls on the same inputs
 * give bitwise identical results. The CUDA-core engine's backward then
 * replaces its scattered float adds by a pull over the same sort (one writer
 * per grad_fmap2 position, candidates in a fixed order); that needs
 * dilation 1 and 1..4 levels, other configurations fail with an error, and
 * its workspace (localCorrB200PyramidWorkspaceBytes* queried while the mode
 * is on) is the sort's. Set it before the forward whose sort a
 * ...BackwardWithSort reuses. */
LCB200_API void localCorrB200SetDeterministic(int on);
LCB200_API int localCorrB200GetDeterministic(void);

/* ---- Bounds-check build ---------------------------------------------------
 * liblocalcorr_b200_checked.so (python -m localcorr_b200.csrc.build
 * --bounds-check) is the same library compiled with LC_BOUNDS_CHECK: every
 * data-dependent global index in the kernels is checked on the device, an
 * out-of-range access is skipped and recorded, and the entry point that
 * launched the kernel synchronises its stream and returns false with the
 * site in localCorrB200GetLastError(). Returns the violations recorded since
 * the last reset, or -1 in the normal build. */
LCB200_API long long localCorrB200BoundsViolations(int reset);

#ifdef __cplusplus
}
#endif

#endif /* LOCALCORR_B200_H */
