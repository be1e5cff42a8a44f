// dcn_tc_common.cuh -- pieces shared by the tensor-core kernels: tile
// constants, packed 16-bit conversions, the bilinear gather producer that
// writes one 128-byte-swizzled row of a [pixels][64 channels] operand tile,
// and 2-D TMA tensor maps.
#pragma once

#include <cuda.h>
#include <type_traits>

#include "dcn_sm100.cuh"
#include "dcn_tc.h"

namespace dcn {
namespace tcc {

using namespace sm100;

constexpr int BM = 128;                     // pixels per tile (MMA M for pixel-major tiles)
constexpr int BK = 64;                      // channels per K chunk (one 128-byte row)
constexpr int A_STAGE_BYTES = BM * BK * 2;  // one [128][64] 16-bit tile: 16 KB

template <typename T> struct Vec;
template <> struct Vec<__nv_bfloat16> {
  static __device__ __forceinline__ float2 unpack(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Vec<__half> {
  static __device__ __forceinline__ float2 unpack(uint32_t w) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    return __half22float2(h);
  }
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// ---------------------------------------------------------------- producer
// Gathers one K chunk (tap t, 64 channels starting at c_abs0) of pixel row r
// for this thread's 4 channel vectors [v0, v0+4) into the swizzled A row.
template <typename T>
__device__ __forceinline__ void gather_row(const Geom& g, const T* __restrict__ xh,
                                           const T* __restrict__ off, const T* __restrict__ msk,
                                           uint8_t* arow, int r, int v0, bool valid, int b, int p,
                                           int t, int c_abs0) {
  uint4 vals[4][4];
  float wts[4][4];
  int cur_o = -1;
  float w4[4] = {0.f, 0.f, 0.f, 0.f};
  long long base4[4] = {0, 0, 0, 0};
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const int c_abs = c_abs0 + (v0 + v) * 8;
    if (valid) {
      const int o = c_abs / g.cpo;
      if (o != cur_o) {
        cur_o = o;
        float y, x, m;
        sample_point(g, off, msk, b, o, t, p, &y, &x, &m);
        const Corners cs = corners_of(y, x, g.H, g.W);
        const long long img = (long long)b * g.H * g.W;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          w4[k] = cs.w[k] * m;
          base4[k] = (img + cs.idx[k]) * g.C;
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        wts[v][k] = w4[k];
        vals[v][k] = (w4[k] != 0.f) ? __ldg(reinterpret_cast<const uint4*>(xh + base4[k] + c_abs))
                                    : make_uint4(0, 0, 0, 0);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        wts[v][k] = 0.f;
        vals[v][k] = make_uint4(0, 0, 0, 0);
      }
    }
  }
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const uint32_t* q0 = reinterpret_cast<const uint32_t*>(&vals[v][0]);
    const uint32_t* q1 = reinterpret_cast<const uint32_t*>(&vals[v][1]);
    const uint32_t* q2 = reinterpret_cast<const uint32_t*>(&vals[v][2]);
    const uint32_t* q3 = reinterpret_cast<const uint32_t*>(&vals[v][3]);
    uint32_t o4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f0 = Vec<T>::unpack(q0[e]), f1 = Vec<T>::unpack(q1[e]);
      const float2 f2 = Vec<T>::unpack(q2[e]), f3 = Vec<T>::unpack(q3[e]);
      const float lo = wts[v][0] * f0.x + wts[v][1] * f1.x + wts[v][2] * f2.x + wts[v][3] * f3.x;
      const float hi = wts[v][0] * f0.y + wts[v][1] * f1.y + wts[v][2] * f2.y + wts[v][3] * f3.y;
      o4[e] = Vec<T>::pack(lo, hi);
    }
    const int chunk = v0 + v;
    uint4* dst = reinterpret_cast<uint4*>(arow + ((chunk ^ (r & 7)) << 4));
    *dst = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
}

// ---------------------------------------------------------------- TMA (tensor)
// 2-D tiled load (no multicast): box at (x = inner coordinate, y) of the
// tensor described by `tmap` into shared memory at `dst`, completing as
// transaction bytes on `bar`.  x * element size must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tmap, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Shared-memory descriptor of an MN-major operand with 128-byte swizzle:
// 64 contiguous MN elements per 128-byte row, rows along K 128 bytes apart,
// 8-row groups `sbo` = 1024 bytes apart, 64-element MN blocks `lbo` apart.
__device__ __forceinline__ uint64_t desc_mnmajor_sw128(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kind::f16 instruction descriptor with explicit operand majors
// (a_mn / b_mn: operand is MN-major instead of K-major).
__host__ __device__ constexpr uint32_t idesc_f16_major(int M, int N, bool ab_bf16, bool a_mn, bool b_mn) {
  return idesc_f16(M, N, ab_bf16) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16);
}

}  // namespace tcc

// Host: encode a 2-D tiled tensor map over a row-major [rows][cols] 16-bit
// matrix with a box of box_cols x box_rows and 128-byte swizzle; rows beyond
// `rows` read as zero.  Returns false when the driver entry point is missing
// or the encode fails.
bool make_tmap_2d(CUtensorMap* map, const void* base, bool bf16, uint64_t rows, uint64_t cols,
                  uint32_t box_rows, uint32_t box_cols);

// Host: device address of the status word (null on failure).
int* tc_status_ptr();

}  // namespace dcn
