// Tensor-core engine of the pyramid local correlation (placeholder until the
// tcgen05 path lands: reports itself ineligible, so AUTO uses the SIMT engine).
#include "lc_common.cuh"

namespace lcb200 {

bool tc_eligible(int, int, int, int, int, int, int, int, std::string* why) {
  if (why) *why = "tensor-core engine not built";
  return false;
}

size_t tc_workspace_bytes(int, int, int, int, int, int) { return 0; }

bool tc_forward(const void*, const void*, const void*, void*, int, int, int, int, int, int,
                int, bool, float, void*, size_t, cudaStream_t) {
  set_error("tensor-core engine not built");
  return false;
}

bool tc_backward(const void*, const void*, const void*, const void*, void*, float*, int, int,
                 int, int, int, int, int, bool, float, void*, size_t, cudaStream_t) {
  set_error("tensor-core engine not built");
  return false;
}

}  // namespace lcb200
