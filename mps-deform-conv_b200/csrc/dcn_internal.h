// dcn_internal.h -- declarations shared by the kernel files and the C ABI layer.
#pragma once

#include "dcn_common.cuh"

namespace dcn {

// Scratch buffers of the SIMT backward (all fp32, caller-provided).
struct SimtBackwardWs {
  float* gcol = nullptr;          // [C*T][P] column gradient
  float* gin32 = nullptr;         // [B][C][H][W] fp32 grad_input accumulator (NULL when T is float)
  float* gacc = nullptr;          // [B][H][W][C] fp32 channels-last grad_input accumulator, or NULL
  float* gw32 = nullptr;          // [Co][C/G*T] fp32 grad_weight accumulator (NULL when T is float)
  void* goff_scratch = nullptr;   // offset-grad sink when the caller wants only grad_mask
  const float* cols = nullptr;    // the forward's fp32 columns [C*T][P] (training state), or NULL
};

// Forward workspace: the K-split partial sums when the output tiles alone
// would not fill one wave of the 148 SMs (0 otherwise).
size_t simt_forward_workspace(const Geom& g);
// Training state of the SIMT path: the forward's fp32 columns [C*T][P] of the
// whole batch, kept for the weight-gradient GEMM, when they fit the forward's
// single column slice (1 GiB); 0 otherwise.
size_t simt_saved_columns_bytes(const Geom& g);
template <typename T>
cudaError_t simt_forward(const Geom& g, const T* x, const T* w, const T* off, const T* msk,
                         const T* bias, T* out, void* workspace, cudaStream_t st);
template <typename T>
cudaError_t simt_im2col(const Geom& g, const T* x, const T* off, const T* msk, T* cols,
                        cudaStream_t st);
template <typename TC, typename T>
cudaError_t simt_col2im(const Geom& g, const TC* gcol, const T* off, const T* msk, float* gin32,
                        cudaStream_t st);
template <typename TC, typename T>
cudaError_t simt_col2im_coord(const Geom& g, const TC* gcol, const T* x, const T* off,
                              const T* msk, T* goff, T* gmsk, cudaStream_t st);
template <typename T>
cudaError_t convert_f32(const float* src, T* dst, long long n, cudaStream_t st);
template <typename T>
cudaError_t simt_backward(const Geom& g, const T* go, const T* x, const T* w, const T* off,
                          const T* msk, T* gin, T* gw, T* goff, T* gmsk, T* gb,
                          const SimtBackwardWs& ws, cudaStream_t st);

// Allocation-free input gradient (dcn_noalloc.cu): largest grad_input it
// accepts, and the launcher that uses the library's fixed device array.
long long noalloc_max_elems();
cudaError_t noalloc_backward_input_dispatch(int dtype, const Geom& g, const void* gcol,
                                            const void* off, const void* msk, void* gin,
                                            cudaStream_t st);

// Device address of a __device__ variable on the current device.  `symbol` is
// the variable's host-side stand-in (its name in host code), which is not a
// device address.  The address is looked up with cudaGetSymbolAddress, with
// the device current, the first time a (device, CUDA context) pair asks, and
// cached per device; a different current context on that device (a new
// primary context after cudaDeviceReset) gets a fresh lookup.  Thread-safe.
struct DeviceSymbolCache {
  static constexpr int kMaxDevices = 64;
  void* ctx[kMaxDevices] = {};
  void* ptr[kMaxDevices] = {};
};
cudaError_t device_symbol_address(DeviceSymbolCache& cache, const void* symbol, void** out);

// Counts kernel launches made by this library (dcn_launch_count()).
void note_launch(int n = 1);

// Scope around one kernel launch: counts it and, while profiling is enabled
// (dcn_profile_enable), records a CUDA event pair on the launching stream so
// the launch's device time can be read back per kernel name.
class KernelScope {
 public:
  KernelScope(const char* name, cudaStream_t st);
  ~KernelScope();
  KernelScope(const KernelScope&) = delete;
  KernelScope& operator=(const KernelScope&) = delete;

 private:
  const char* name_;
  cudaStream_t st_;
  cudaEvent_t start_ = nullptr;
};

// Round a byte count up to the 256-byte workspace alignment.
inline size_t ws_align(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace dcn
