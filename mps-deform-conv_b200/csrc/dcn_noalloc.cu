// dcn_noalloc.cu -- input gradient from a column gradient without any device
// allocation, for callers that cannot allocate.
//
// Some callers hold only their input and output buffers: plugin interfaces of
// inference and training runtimes whose enqueue step hands a kernel library
// pointers but no allocator, and real-time loops that forbid device
// allocation after start-up because cudaMalloc can block and synchronise the
// whole device.  dcn_deform_conv2d_backward_input needs a caller-provided
// fp32 workspace for fp16/bf16 data; this variant keeps that fp32
// accumulator in a fixed array in device memory instead.
//
// The array is a file-scope __device__ array of NOALLOC_MAX_ELEMS floats
// (8 MiB).  Every GPU that loads this library holds it until the process
// exits.  Host code cannot use the array's name as a device address (in host
// code it names a host-side stand-in), so the device address is looked up
// with cudaGetSymbolAddress, once per device, with that device current, on
// the first fp16/bf16 call made on that device (and again after the device's
// context was reset).  fp32 data accumulates straight into grad_input and
// never uses the array, so fp32 problems have no size limit here.
#include <type_traits>

#include "dcn_internal.h"

namespace dcn {

constexpr long long NOALLOC_MAX_ELEMS = 2LL * 1024 * 1024;  // grad_input elements (8 MiB of fp32)

static __device__ __align__(256) float g_noalloc_accum[NOALLOC_MAX_ELEMS];

// Device address of the accumulator on the current device: looked up on the
// first call made on a device (with that device current) and again whenever
// the device's CUDA context has changed since (cudaDeviceReset).
static cudaError_t noalloc_accum_ptr(float** out) {
  static DeviceSymbolCache cache;
  void* p = nullptr;
  const cudaError_t e = device_symbol_address(cache, &g_noalloc_accum, &p);
  *out = static_cast<float*>(p);
  return e;
}

long long noalloc_max_elems() { return NOALLOC_MAX_ELEMS; }

template <typename T>
static cudaError_t noalloc_backward_input(const Geom& g, const T* gcol, const T* off,
                                          const T* msk, T* gin, float* accum, cudaStream_t st) {
  const long long n = (long long)g.B * g.C * g.H * g.W;
  // fp32 data accumulates straight into grad_input; fp16/bf16 use the array.
  float* acc = std::is_same<T, float>::value ? reinterpret_cast<float*>(gin) : accum;
  // The array keeps the previous call's contents: clear the part this call uses.
  cudaError_t e = cudaMemsetAsync(acc, 0, sizeof(float) * (size_t)n, st);
  if (e != cudaSuccess) return e;
  if ((e = simt_col2im<T, T>(g, gcol, off, msk, acc, st)) != cudaSuccess) return e;
  if (!std::is_same<T, float>::value) e = convert_f32<T>(acc, gin, n, st);
  return e;
}

cudaError_t noalloc_backward_input_dispatch(int dtype, const Geom& g, const void* gcol,
                                            const void* off, const void* msk, void* gin,
                                            cudaStream_t st) {
  float* accum = nullptr;
  if (dtype != DCN_FLOAT32) {
    const cudaError_t e = noalloc_accum_ptr(&accum);
    if (e != cudaSuccess) return e;
  }
  switch (dtype) {
    case DCN_FLOAT32:
      return noalloc_backward_input<float>(g, (const float*)gcol, (const float*)off,
                                           (const float*)msk, (float*)gin, accum, st);
    case DCN_FLOAT16:
      return noalloc_backward_input<__half>(g, (const __half*)gcol, (const __half*)off,
                                            (const __half*)msk, (__half*)gin, accum, st);
    default:
      return noalloc_backward_input<__nv_bfloat16>(g, (const __nv_bfloat16*)gcol,
                                                   (const __nv_bfloat16*)off,
                                                   (const __nv_bfloat16*)msk,
                                                   (__nv_bfloat16*)gin, accum, st);
  }
}

}  // namespace dcn
