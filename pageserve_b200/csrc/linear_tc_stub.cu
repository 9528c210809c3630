// Placeholder until the tcgen05 kernel lands: no tensor-core configuration.
#include "linear.cuh"
namespace ps_host {
int linear_tc(void*, const void*, const void*, int, const float*, const void*, const void*, int, int, int, int,
              void*, size_t, cudaStream_t) {
  return PS_ERR_UNSUPPORTED;
}
size_t linear_tc_workspace(int, int, int) { return 0; }
}  // namespace ps_host
