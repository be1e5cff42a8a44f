// dcn_debug.cuh -- optional bounds checks on the gather and scatter index math.
//
// Built with -DDCN_DEBUG_BOUNDS (build.py --bounds, libdcn_b200_bounds.so),
// every checked index is compared with the extent of the tensor it addresses
// before the access.  An index outside [0, extent - width] is recorded (a
// count, and the site, index and extent of the first one) in the translation
// unit's record and replaced by 0, so the access stays inside the tensor: the
// check never traps, faults or stops the kernel.  dcn_debug_bounds_read()
// (dcn_abi.cu) sums the records of all kernel files.  Without the define,
// DCN_BOUND(i, ...) is i and nothing is recorded.
#pragma once

#include <cuda_runtime.h>

namespace dcn {

// Where a checked index was computed.
enum DebugSite : int {
  DBG_CORNER = 1,        // corners_of: in-plane corner index vs H*W
  DBG_COORD_CORNER,      // coord_corners_of: in-plane corner index vs H*W
  DBG_TC_GATHER_X,       // tensor-core producers: corner vector of the channels-last input
  DBG_TC_GATHER_OFF,     // tensor-core producers: offset element
  DBG_TC_GATHER_MSK,     // tensor-core producers: mask element
  DBG_TC_GATHER_QUAD,    // corner-quad producer: 32-byte half of a record
  DBG_DG_CORNER_X,       // dgrad epilogue: corner vector of the input
  DBG_DG_SCATTER,        // dgrad epilogue: fp32 grad_input reduction target
  DBG_DG_QUAD_SCATTER,   // dgrad corner-quad epilogue: fp32 record reduction target
  DBG_DG_COORD,          // dgrad epilogue: offset / mask gradient element
  DBG_SIMT_COL2IM,       // SIMT col2im: fp32 grad_input element
  DBG_SIMT_COL2IM_NHWC,  // SIMT col2im_nhwc4: channels-last fp32 reduction target
  DBG_SIMT_IM2COL,       // SIMT im2col_og: column element written
  DBG_SITES
};

// One translation unit's record (also the summed record dcn_debug_bounds_read returns).
struct DebugBounds {
  unsigned long long count;
  long long index, extent;
  int site, width;
};

#ifdef DCN_DEBUG_BOUNDS
static __device__ DebugBounds dcn_debug_rec;

__device__ __noinline__ inline void debug_violation(int site, long long idx, long long width, long long extent) {
  if (atomicAdd(&dcn_debug_rec.count, 1ull) == 0ull) {
    dcn_debug_rec.site = site;
    dcn_debug_rec.index = idx;
    dcn_debug_rec.extent = extent;
    dcn_debug_rec.width = (int)width;
  }
}

// idx if [idx, idx + width) lies inside [0, extent), else 0 (recorded).
template <typename I>
__device__ __forceinline__ I debug_bound(I idx, long long width, long long extent, int site) {
  const long long v = (long long)idx;
  if (v < 0 || v + width > extent) {
    debug_violation(site, v, width, extent);
    return I(0);
  }
  return idx;
}
#define DCN_BOUND(idx, width, extent, site) ::dcn::debug_bound((idx), (long long)(width), (long long)(extent), (site))

// Host side of one kernel file: add its record to *acc and optionally clear
// it.  Defined once per file by DCN_DEBUG_BOUNDS_TU(name).
#define DCN_DEBUG_BOUNDS_TU(name)                                                            \
  cudaError_t debug_bounds_collect_##name(DebugBounds* acc, bool reset) {                    \
    DebugBounds r;                                                                           \
    cudaError_t e = cudaMemcpyFromSymbol(&r, dcn_debug_rec, sizeof(r));                      \
    if (e != cudaSuccess) return e;                                                          \
    if (r.count && !acc->count) {                                                            \
      acc->site = r.site;                                                                    \
      acc->index = r.index;                                                                  \
      acc->extent = r.extent;                                                                \
      acc->width = r.width;                                                                  \
    }                                                                                        \
    acc->count += r.count;                                                                   \
    if (reset) {                                                                             \
      const DebugBounds z = {};                                                              \
      e = cudaMemcpyToSymbol(dcn_debug_rec, &z, sizeof(z));                                  \
    }                                                                                        \
    return e;                                                                                \
  }
#else
#define DCN_BOUND(idx, width, extent, site) (idx)
#define DCN_DEBUG_BOUNDS_TU(name)                                               \
  cudaError_t debug_bounds_collect_##name(DebugBounds*, bool) { return cudaSuccess; }
#endif

// The collectors of the kernel files with checked kernels.
cudaError_t debug_bounds_collect_tc(DebugBounds* acc, bool reset);
cudaError_t debug_bounds_collect_tc_bwd(DebugBounds* acc, bool reset);
cudaError_t debug_bounds_collect_simt(DebugBounds* acc, bool reset);

}  // namespace dcn
