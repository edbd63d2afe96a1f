// ca_sm100.cu -- sm_100a tensor-core (tcgen05 / TMEM / TMA) kernels.
#include "ca_common.cuh"
#include "ca_internal.h"

namespace ca {

// Status word written by kernels whose bounded waits gave up (CA_ERR_DEVICE_TIMEOUT).
__device__ int g_device_status = 0;

cudaError_t read_device_status(int* out, bool reset) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return e;
  e = cudaMemcpyFromSymbol(out, g_device_status, sizeof(int));
  if (e != cudaSuccess || !reset) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
}

namespace sm100 {
bool forward_supported(const FwdArgs&) { return false; }
bool backward_supported(const BwdArgs&) { return false; }
int forward_launches(const FwdArgs&) { return 0; }
int backward_launches(const BwdArgs&) { return 0; }
cudaError_t forward(const FwdArgs&) { return cudaErrorNotSupported; }
cudaError_t backward(const BwdArgs&, const BwdWorkspace&) { return cudaErrorNotSupported; }
}  // namespace sm100

}  // namespace ca
