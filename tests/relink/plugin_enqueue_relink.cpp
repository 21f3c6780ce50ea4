// Relink check of the TensorRT plugin path against liblocalcorr_b200.so.
//
// The reference's TensorRT plugin (cuda_pyramid/localcorr_cuda_pyramid_plugin.cpp)
// computes the custom_ops::LocalCorrCudaPyramid node in enqueue() by calling
// launchLocalCorrCudaPyramidForward (plugin.cpp:164-199): B, H1, W1, C from
// input 0's dims [B, H1, W1, C], isHalf from input 0's type, radius/levels/
// dilation/ymajor from the node's attributes, and returns 0 on success, 1 on
// failure. The function below makes that call with the same argument
// expressions, against include/localcorr_b200.h and the types of a TensorRT
// enqueue (stand-ins, TensorRT is absent), so a plugin that includes the new
// header in place of localcorr_cuda_pyramid_kernel.h and links the new
// library compiles, links and runs unchanged.
//
// Built by tests/test_relink_cpu.py (and the GPU test) as a shared library and
// driven through ctypes.
#include "localcorr_b200.h"
#include "trt_stand_in.h"

using namespace nvinfer1;

namespace {

struct PyramidNodeAttrs {
  int radius_;
  int levels_;
  int dilation_;
  int ymajor_;

  int32_t enqueue(PluginTensorDesc const* inputDesc, PluginTensorDesc const* outputDesc,
                  void const* const* inputs, void* const* outputs, void* workspace,
                  cudaStream_t stream) const noexcept {
    (void)outputDesc;
    (void)workspace;
    Dims const& fmap1Dims = inputDesc[0].dims;
    Dims const& coordsDims = inputDesc[2].dims;
    if (fmap1Dims.nbDims != 4 || coordsDims.nbDims != 4) return 1;
    const int batch = static_cast<int>(fmap1Dims.d[0]);
    const int h1 = static_cast<int>(fmap1Dims.d[1]);
    const int w1 = static_cast<int>(fmap1Dims.d[2]);
    const int channels = static_cast<int>(fmap1Dims.d[3]);
    const bool isHalf = inputDesc[0].type == DataType::kHALF;
    const bool ok = launchLocalCorrCudaPyramidForward(
        inputs[0], inputs[1], inputs[2], outputs[0], batch, h1, w1, channels, radius_,
        levels_, dilation_, isHalf, ymajor_ != 0, stream);
    return ok ? 0 : 1;
  }
};

}  // namespace

// One enqueue of a LocalCorrCudaPyramid node: fmap1 [B, H1, W1, C], packed
// pyramid, coords [B, 2, H1, W1], output; dtype 1 = float16, 0 = float32.
extern "C" int relink_enqueue(const void* fmap1, const void* fmap2_packed, const void* coords,
                              void* corr, int B, int H1, int W1, int C, int dtype, int radius,
                              int levels, int dilation, int ymajor, void* stream) {
  PluginTensorDesc in[3] = {};
  in[0].dims.nbDims = 4;
  in[0].dims.d[0] = B; in[0].dims.d[1] = H1; in[0].dims.d[2] = W1; in[0].dims.d[3] = C;
  in[0].type = dtype == 1 ? DataType::kHALF : DataType::kFLOAT;
  in[2].dims.nbDims = 4;
  in[2].dims.d[0] = B; in[2].dims.d[1] = 2; in[2].dims.d[2] = H1; in[2].dims.d[3] = W1;
  in[2].type = in[0].type;
  PluginTensorDesc out = {};
  out.type = in[0].type;
  const void* inputs[3] = {fmap1, fmap2_packed, coords};
  void* outputs[1] = {corr};
  const PyramidNodeAttrs node{radius, levels, dilation, ymajor};
  return node.enqueue(in, &out, inputs, outputs, nullptr, static_cast<cudaStream_t>(stream));
}
