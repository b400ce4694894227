// Tensor-core (tcgen05) E-step kernels -- placeholder until the fast path lands.
#include "fgmm_internal.cuh"

namespace fgmm {

bool tc_supported(int, const EstepArgs&, std::string* why) {
  if (why) *why = "tensor-core path not built";
  return false;
}
size_t tc_workspace_bytes(int, int64_t, int, int) { return 0; }
cudaError_t tc_estep(int, const EstepArgs&) { return cudaErrorNotSupported; }

}  // namespace fgmm
