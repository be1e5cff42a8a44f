// dcn_layout.cuh -- vectorized HBM-bound layout passes between the NCHW
// tensors of the public interface and the channels-last / pixel-major
// operands of the tensor-core kernels, for 16-bit element types.
//
// Each CTA moves one tile of 64 channels x 64 pixels of one image through
// shared memory.  The tile holds 32-bit pairs (two channels of one pixel, or
// two pixels of one channel) in rows of 33 words, and every shared-memory
// access pattern below maps a warp onto 32 distinct banks.  Global loads and
// stores are 4, 8 or 16 bytes wide and cover whole 32-byte sectors.
//
// Both passes are pure data movement (plus a round-to-nearest fp32 -> 16-bit
// conversion in from_channels_last_f32_16), so their results are bit-identical
// to the scalar kernels that serve the shapes these do not take.
#pragma once

#include "dcn_tc_common.cuh"

namespace dcn {
namespace layout {

using tcc::Vec;

constexpr int TP = 64;              // tile edge: 64 channels x 64 pixels
constexpr int LAYOUT_THREADS = 256;

// to_channels_last16 loads pixel pairs as 32-bit words and stores 16 bytes
// (8 channels) per pixel row.
inline bool to_channels_last_vec_ok(const void* src, const void* dst, long long C, long long HW) {
  return C % 8 == 0 && HW % 2 == 0 && reinterpret_cast<uintptr_t>(src) % 4 == 0 &&
         reinterpret_cast<uintptr_t>(dst) % 16 == 0;
}
// from_channels_last_f32_16 loads 4 fp32 channels (16 bytes) and stores 4
// pixels (8 bytes).
inline bool from_channels_last_vec_ok(const void* src, const void* dst, long long C, long long HW) {
  return C % 4 == 0 && HW % 4 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(dst) % 8 == 0;
}

inline dim3 tile_grid(long long C, long long HW, long long B) {
  return dim3((unsigned)((HW + TP - 1) / TP), (unsigned)((C + TP - 1) / TP), (unsigned)B);
}

// src [B][C][HW] -> dst [B][HW][C] (16-bit T, bits copied).  With SUM,
// gsum[c] += sum over the tile's pixels of src[c][hw] in fp32 (the bias
// gradient when src is grad_output).
template <typename T, bool SUM>
__global__ void __launch_bounds__(LAYOUT_THREADS)
to_channels_last16_kernel(const T* __restrict__ src, T* __restrict__ dst, float* __restrict__ gsum,
                          int C, int HW) {
  static_assert(sizeof(T) == 2, "16-bit element types only");
  __shared__ uint32_t tile[TP][TP / 2 + 1];  // [pixel][channel pair]
  __shared__ float csum[TP];
  const int b = blockIdx.z, c0 = blockIdx.y * TP, hw0 = blockIdx.x * TP;
  if (SUM) {
    if (threadIdx.x < TP) csum[threadIdx.x] = 0.f;
    __syncthreads();
  }
  // 32 channel pairs x 32 pixel pairs; a warp takes 2 channel pairs x 16
  // pixel pairs (two 64-byte row segments per channel).
  const uint32_t* s32 = reinterpret_cast<const uint32_t*>(src + (long long)b * C * HW);
  constexpr int ITERS = (TP / 2) * (TP / 2) / LAYOUT_THREADS;
  uint32_t va[ITERS], vb[ITERS];
#pragma unroll
  for (int it = 0; it < ITERS; ++it) {
    const int e = threadIdx.x + it * LAYOUT_THREADS, w = e >> 5, lane = e & 31;
    const int cp = (w & 15) * 2 + (lane >> 4), hp = (w >> 4) * 16 + (lane & 15);
    const int c = c0 + 2 * cp, hw = hw0 + 2 * hp;
    va[it] = vb[it] = 0u;
    if (c < C && hw < HW) {  // C even and HW even: the pair is whole
      va[it] = s32[((long long)c * HW + hw) >> 1];
      vb[it] = s32[((long long)(c + 1) * HW + hw) >> 1];
    }
  }
#pragma unroll
  for (int it = 0; it < ITERS; ++it) {
    const int e = threadIdx.x + it * LAYOUT_THREADS, w = e >> 5, lane = e & 31;
    const int cp = (w & 15) * 2 + (lane >> 4), hp = (w >> 4) * 16 + (lane & 15);
    // word 66*hp + cp: bank 2*(lane&15) + (lane>>4) + const, distinct per lane
    tile[2 * hp][cp] = __byte_perm(va[it], vb[it], 0x5410);      // pixel hw:   (c, c+1)
    tile[2 * hp + 1][cp] = __byte_perm(va[it], vb[it], 0x7632);  // pixel hw+1: (c, c+1)
    if (SUM) {
      const float2 fa = Vec<T>::unpack(va[it]), fb = Vec<T>::unpack(vb[it]);
      float sa = fa.x + fa.y, sb = fb.x + fb.y;
#pragma unroll
      for (int o = 8; o; o >>= 1) {
        sa += __shfl_xor_sync(0xffffffffu, sa, o);
        sb += __shfl_xor_sync(0xffffffffu, sb, o);
      }
      if ((lane & 15) == 0) {
        atomicAdd(&csum[2 * cp], sa);
        atomicAdd(&csum[2 * cp + 1], sb);
      }
    }
  }
  __syncthreads();
  // 64 pixel rows x 8 vectors of 8 channels; word 33*r + 4*j + k: bank
  // r + 4*j + k over 4 consecutive r and j = 0..7, distinct per lane.
  T* d = dst + (long long)b * HW * C;
#pragma unroll
  for (int it = 0; it < TP * 8 / LAYOUT_THREADS; ++it) {
    const int e = threadIdx.x + it * LAYOUT_THREADS, r = e >> 3, j = e & 7;
    const int hw = hw0 + r, c = c0 + 8 * j;
    if (hw < HW && c < C) {
      const uint4 v = make_uint4(tile[r][4 * j], tile[r][4 * j + 1], tile[r][4 * j + 2], tile[r][4 * j + 3]);
      *reinterpret_cast<uint4*>(d + (long long)hw * C + c) = v;
    }
  }
  if (SUM && threadIdx.x < TP && c0 + (int)threadIdx.x < C) atomicAdd(gsum + c0 + threadIdx.x, csum[threadIdx.x]);
}

// Reader of a channels-last fp32 tensor [B][HW][C]: channels c..c+3 of pixel
// hw of image b as one float4.
struct NhwcF32Reader {
  const float* src;
  int C, HW;
  __device__ __forceinline__ float4 operator()(int b, int hw, int c) const {
    return *reinterpret_cast<const float4*>(src + ((long long)b * HW + hw) * C + c);
  }
};

// fp32 [B][HW][C] (read through rd, e.g. NhwcF32Reader) -> dst [B][C][HW]
// in 16-bit T (round to nearest).
template <typename T, class RD>
__global__ void __launch_bounds__(LAYOUT_THREADS)
from_channels_last_f32_16_kernel(const RD rd, T* __restrict__ dst, int C, int HW) {
  static_assert(sizeof(T) == 2, "16-bit element types only");
  __shared__ uint32_t tile[TP][TP / 2 + 1];  // [channel][pixel pair]
  const int b = blockIdx.z, c0 = blockIdx.y * TP, hw0 = blockIdx.x * TP;
  // 32 pixel pairs x 16 groups of 4 channels; a warp takes 4 pixel pairs x
  // 8 groups (128 contiguous bytes of each of 8 pixel rows).
  constexpr int ITERS = (TP / 2) * (TP / 4) / LAYOUT_THREADS;
  float4 v0[ITERS], v1[ITERS];
#pragma unroll
  for (int it = 0; it < ITERS; ++it) {
    const int e = threadIdx.x + it * LAYOUT_THREADS, w = e >> 5, lane = e & 31;
    const int hp = (w >> 1) * 4 + (lane & 3), q = (w & 1) * 8 + (lane >> 2);
    const int hw = hw0 + 2 * hp, c = c0 + 4 * q;
    v0[it] = v1[it] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (hw < HW && c < C) {  // C % 4 == 0 and HW even: both vectors are whole
      v0[it] = rd(b, hw, c);
      v1[it] = rd(b, hw + 1, c);
    }
  }
#pragma unroll
  for (int it = 0; it < ITERS; ++it) {
    const int e = threadIdx.x + it * LAYOUT_THREADS, w = e >> 5, lane = e & 31;
    const int hp = (w >> 1) * 4 + (lane & 3), q = (w & 1) * 8 + (lane >> 2);
    // word 33*(4q+i) + hp: bank 4*(lane>>2) + (lane&3) + i + const, distinct per lane
    tile[4 * q + 0][hp] = Vec<T>::pack(v0[it].x, v1[it].x);
    tile[4 * q + 1][hp] = Vec<T>::pack(v0[it].y, v1[it].y);
    tile[4 * q + 2][hp] = Vec<T>::pack(v0[it].z, v1[it].z);
    tile[4 * q + 3][hp] = Vec<T>::pack(v0[it].w, v1[it].w);
  }
  __syncthreads();
  // 64 channel rows x 16 vectors of 4 pixels; word 33*r + 2*j + k: bank
  // r + 2*j + k over 2 consecutive r and j = 0..15, distinct per lane.
  T* d = dst + (long long)b * C * HW;
#pragma unroll
  for (int it = 0; it < TP * 16 / LAYOUT_THREADS; ++it) {
    const int e = threadIdx.x + it * LAYOUT_THREADS, r = e >> 4, j = e & 15;
    const int c = c0 + r, hw = hw0 + 4 * j;
    if (c < C && hw < HW)
      *reinterpret_cast<uint2*>(d + (long long)c * HW + hw) = make_uint2(tile[r][2 * j], tile[r][2 * j + 1]);
  }
}

}  // namespace layout
}  // namespace dcn
