// dcn_tc.cu -- tensor-core (tcgen05 / TMEM) kernels for sm_100a.
#include "dcn_tc.h"

namespace dcn {

// Device status word: set by a kernel whose bounded wait expired.
__device__ int g_dcn_status = 0;

bool tc_supported(const dcn_conv_desc&, const Geom&) { return false; }
size_t tc_forward_workspace(const dcn_conv_desc&, const Geom&) { return 0; }
size_t tc_backward_workspace(const dcn_conv_desc&, const Geom&) { return 0; }
cudaError_t tc_forward(const dcn_conv_desc&, const Geom&, const void*, const void*, const void*,
                       const void*, const void*, void*, void*, cudaStream_t) {
  return cudaErrorNotSupported;
}
cudaError_t tc_backward(const dcn_conv_desc&, const Geom&, const void*, const void*, const void*,
                        const void*, const void*, void*, void*, void*, void*, void*, void*,
                        cudaStream_t) {
  return cudaErrorNotSupported;
}

cudaError_t tc_read_and_clear_status(int* out, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_dcn_status, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(g_dcn_status, &zero, sizeof(int));
}

}  // namespace dcn
