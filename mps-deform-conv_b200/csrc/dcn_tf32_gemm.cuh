// dcn_tf32_gemm.cuh -- fp32 GEMM on the tensor cores (tcgen05, kind::tf32)
// with the three-term split that keeps fp32 accuracy (3xTF32).
//
// The fp32 path composes the reference's way (deform_conv2d_mps.mm:679-800,
// __init__.py:245-322): materialised columns, three GEMMs (forward W x cols,
// grad_weight gO x cols^T, column gradient W^T x gO) and the scatter kernels.
// Here the three GEMMs run on tcgen05 MMAs instead of CUDA-core FMAs:
//
//   D[r][c] = sum_k R(k, r) * C(k, c)       r: 128-row tile = TMEM lanes
//                                            c: BN-column tile = TMEM columns
//
// Operands are read through loader functors (ld(g, k, mn) -> float), so any
// layout and any size works; out-of-range elements are zero.  Each value x is
// split into hi = tf32(x) (round to nearest) and lo = tf32(x - hi), and every
// 8-deep K step issues three MMAs into the same fp32 TMEM accumulator:
//   R_hi C_hi + R_hi C_lo + R_lo C_hi.
// The dropped R_lo C_lo term and the rounding of the lo parts are below
// 2^-21 of each product, so the result carries fp32 accuracy (fp16/bf16
// values have lo = 0 and give exact products).
//
// Warp roles (288 threads): warps 0-7 fill the operand tiles of each K chunk
// of 32 values (hi and lo tiles, K-major, 128-byte swizzle: row r of a tile is
// 128 bytes, its 16-byte chunk j stored at chunk j ^ (r % 8)) and after the
// main loop read the accumulator back (tcgen05.ld) into the epilogue functor;
// warp 8 lane 0 issues the MMAs.  STAGES chunks are in flight.  Every
// mbarrier wait is bounded (dcn_sm100.cuh).
#pragma once

#include "dcn_sm100.cuh"

namespace dcn {

cudaError_t tc_status_ptr(int** out);

namespace tf32g {

using namespace sm100;

constexpr int BM = 128;                      // tile rows (TMEM lanes)
constexpr int BKF = 32;                      // fp32 K values per 128-byte row
constexpr int PROD_WARPS = 8;
constexpr int NPROD = PROD_WARPS * 32;
constexpr int MMA_WARP = PROD_WARPS;
constexpr int NTHREADS = NPROD + 32;
constexpr int STAGES = 3;
constexpr uint32_t R_TILE = BM * 128;        // one 16 KB row-operand tile (hi or lo)

// status codes recorded on a wait that expired
constexpr int ST_G_PROD = 41, ST_G_MMA = 42, ST_G_EPI = 43, ST_G_DRAIN = 44;

struct Smem {
  uint32_t r, c, bar, total;
};
// [stage][hi, lo] row-operand tiles, [stage][hi, lo] column-operand tiles,
// then full[S], empty[S], acc_full, drain, the TMEM slot and the abort flag.
__host__ __device__ inline Smem smem_layout(int bn) {
  Smem L;
  L.r = 0;
  L.c = L.r + STAGES * 2 * R_TILE;
  L.bar = L.c + STAGES * 2 * (uint32_t)bn * 128u;
  L.total = L.bar + (2 * STAGES + 2) * 8 + 16;
  return L;
}

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// Rows [0, ROWS) x K values [k0, k0 + 32) of one operand, loaded into
// registers (load) and then written as hi = tf32(x), lo = tf32(x - hi) into
// the tile pair (store).  The items a thread owns depend on the loader's
// contiguity (L::kContig):
//   2 (rows contiguous): item = (4-row group, 4-value K chunk): four float4
//     reads (one per k) of 4 consecutive rows, written as 4 row chunks;
//     consecutive threads take consecutive row groups (coalesced);
//   1 (K contiguous): item = (row, chunk), one float4 read; 8 consecutive
//     threads read one row's 32 values;
//   0: item = (row, chunk), four element reads; KFAST picks the thread order
//     (8 threads per row, or consecutive rows).
// Reads fall back to elements at the tile's edges or when L::vec is unset.
template <int ROWS, bool KFAST, class L>
struct Fill {
  static constexpr int C = L::kContig;
  static constexpr int NITEMS = C == 2 ? ROWS * 2 : ROWS * 8;
  static constexpr int NI = (NITEMS + NPROD - 1) / NPROD;
  static constexpr int NV = C == 2 ? 16 : 4;
  static_assert(ROWS % 32 == 0 && (NITEMS % NPROD == 0 || NITEMS < NPROD), "tile rows");
  float v[NI][NV];

  __device__ __forceinline__ static void item(int it, int& r, int& j) {
    if (C == 2) { r = 4 * (it % (ROWS / 4)); j = it / (ROWS / 4); }
    else if (C == 1 || KFAST) { r = it >> 3; j = it & 7; }
    else { r = it % ROWS; j = it / ROWS; }
  }

  __device__ __forceinline__ void load(const L& ld, int g, int k0, int kend, int mn0, int mnend, int tid) {
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int it = tid + i * NPROD;
      if (it >= NITEMS) break;
      int r, j;
      item(it, r, j);
      const int mn = mn0 + r, kq = k0 + 4 * j;
      if (C == 2) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = kq + e;
          if (ld.vec && k < kend && mn + 3 < mnend) {
            const float4 f = ld.ld4(g, k, mn);
            v[i][4 * e] = f.x; v[i][4 * e + 1] = f.y; v[i][4 * e + 2] = f.z; v[i][4 * e + 3] = f.w;
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) v[i][4 * e + q] = (k < kend && mn + q < mnend) ? ld(g, k, mn + q) : 0.0f;
          }
        }
      } else if (C == 1 && ld.vec && kq + 3 < kend && mn < mnend) {
        const float4 f = ld.ld4(g, kq, mn);
        v[i][0] = f.x; v[i][1] = f.y; v[i][2] = f.z; v[i][3] = f.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[i][e] = (kq + e < kend && mn < mnend) ? ld(g, kq + e, mn) : 0.0f;
      }
    }
  }

  __device__ __forceinline__ static void put(uint8_t* hi, uint8_t* lo, int r, int j, float a, float b, float c,
                                             float d) {
    const float x[4] = {a, b, c, d};
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      h[e] = to_tf32(x[e]);
      l[e] = to_tf32(x[e] - __uint_as_float(h[e]));
    }
    const uint32_t off = (uint32_t)r * 128u + ((uint32_t)(j ^ (r & 7)) << 4);
    *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
  }

  __device__ __forceinline__ void store(uint8_t* hi, uint8_t* lo, int tid) const {
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int it = tid + i * NPROD;
      if (it >= NITEMS) break;
      int r, j;
      item(it, r, j);
      if (C == 2) {
        // the 4 rows in an order rotated by rot = (r / 8) % 4, so that the 8
        // lanes of a store phase write rows of 8 distinct (row % 8), i.e.
        // 8 distinct chunk positions (no bank conflicts)
        const int rot = (r >> 3) & 3;
        float a[4][4];  // a[e][q] = v[4e + (q + rot) % 4]
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float a0 = v[i][4 * e], a1 = v[i][4 * e + 1], a2 = v[i][4 * e + 2], a3 = v[i][4 * e + 3];
          if (rot & 1) { const float t = a0; a0 = a1; a1 = a2; a2 = a3; a3 = t; }
          if (rot & 2) { float t = a0; a0 = a2; a2 = t; t = a1; a1 = a3; a3 = t; }
          a[e][0] = a0; a[e][1] = a1; a[e][2] = a2; a[e][3] = a3;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) put(hi, lo, r + ((q + rot) & 3), j, a[0][q], a[1][q], a[2][q], a[3][q]);
      } else {
        put(hi, lo, r, j, v[i][0], v[i][1], v[i][2], v[i][3]);
      }
    }
  }
};

// grid (ceil(Ccols / BN), ceil(Rrows / BM), groups * splits); blockIdx.z =
// group * splits + split, the split owning K range [split*kps, +kps).
// Epilogue: ep(g, c, r, value) for every in-range element (column index
// first: the callers' GEMMs are M = columns, N = rows).
template <int BN, bool R_KFAST, bool C_KFAST, class LR, class LC, class EP>
__global__ void __launch_bounds__(NTHREADS, 1)
tf32x3_gemm_kernel(const LR lr, const LC lc, const EP ep, int Rrows, int Ccols, int K, int splits, int kps,
                   int* status) {
  static_assert(BN == 64 || BN == 128, "column tile");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Smem L = smem_layout(BN);
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bar0 = sbase + L.bar;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
  const uint32_t acc_full = bar0 + 8u * (2 * STAGES);
  const uint32_t drain = bar0 + 8u * (2 * STAGES + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + (2 * STAGES + 2) * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.bar + (2 * STAGES + 2) * 8 + 8);
  constexpr uint32_t C_TILE = (uint32_t)BN * 128u;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.z / splits, sp = blockIdx.z - (blockIdx.z / splits) * splits;
  const int r0 = blockIdx.y * BM, c0 = blockIdx.x * BN;
  const int kbeg = sp * kps;
  const int kend = min(K, kbeg + kps);
  const int nk = kend > kbeg ? (kend - kbeg + BKF - 1) / BKF : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), NPROD);
      mbar_init(empty(s), 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(smem_addr(tmem_slot), BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < PROD_WARPS) {
    // ------------------------------------------------ operand producers
    // chunks i+1 and i+2 have their loads in flight while chunk i is split
    // and stored (three register sets, used in rotation)
    using FR = Fill<BM, R_KFAST, LR>;
    using FC = Fill<BN, C_KFAST, LC>;
    const int tid = threadIdx.x;
    FR fr0, fr1, fr2;
    FC fc0, fc1, fc2;
    auto load = [&](int i, FR& fr, FC& fc) {
      if (i >= nk) return;
      const int k0 = kbeg + i * BKF;
      fr.load(lr, g, k0, kend, r0, Rrows, tid);
      fc.load(lc, g, k0, kend, c0, Ccols, tid);
    };
    auto store = [&](int i, const FR& fr, const FC& fc) {
      const int s = i % STAGES;
      if (!mbar_wait(empty(s), ((i / STAGES) & 1) ^ 1, abort_flag, status, ST_G_PROD)) return false;
      uint8_t* rt = smem + L.r + (uint32_t)s * 2 * R_TILE;
      uint8_t* ct = smem + L.c + (uint32_t)s * 2 * C_TILE;
      fr.store(rt, rt + R_TILE, tid);
      fc.store(ct, ct + C_TILE, tid);
      fence_async_shared();
      mbar_arrive(full(s));
      return true;
    };
    bool ok = true;
    load(0, fr0, fc0);
    load(1, fr1, fc1);
    for (int i = 0; i < nk; i += 3) {
      load(i + 2, fr2, fc2);
      if (!(ok = store(i, fr0, fc0)) || i + 1 >= nk) break;
      load(i + 3, fr0, fc0);
      if (!(ok = store(i + 1, fr1, fc1)) || i + 2 >= nk) break;
      load(i + 4, fr1, fc1);
      if (!(ok = store(i + 2, fr2, fc2))) break;
    }
    // ------------------------------------------------ epilogue
    // warp w reads TMEM lanes 32 (w % 4) .. +31 (its quadrant), column
    // blocks of 16 starting at 16 (w / 4), every 32 columns
    const bool acc_ready = ok && (nk == 0 || mbar_wait(acc_full, 0, abort_flag, status, ST_G_EPI));
    if (__all_sync(0xffffffffu, acc_ready)) {
      tc_fence_after();
      const int q = warp & 3, half = warp >> 2;
      const int r = r0 + q * 32 + lane;
      for (int cb = half * 16; cb < BN && c0 + cb < Ccols; cb += 32) {
        uint32_t acc[16];
        if (nk > 0) {
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)cb, acc);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] = 0u;
        }
        if (r < Rrows) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + cb + j < Ccols) ep(g, c0 + cb + j, r, __uint_as_float(acc[j]));
        }
      }
    }
  } else if (lane == 0) {
    // ------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_tf32(BM, BN);
    bool ok = true;
    int issued = 0;
    for (int i = 0; i < nk && ok; ++i) {
      const int s = i % STAGES;
      ok = mbar_wait(full(s), (i / STAGES) & 1, abort_flag, status, ST_G_MMA);
      if (!ok) break;
      tc_fence_after();
      const uint32_t rh = sbase + L.r + (uint32_t)s * 2 * R_TILE, rl = rh + R_TILE;
      const uint32_t ch = sbase + L.c + (uint32_t)s * 2 * C_TILE, cl = ch + C_TILE;
#pragma unroll
      for (int kk = 0; kk < BKF / 8; ++kk) {
        const uint32_t o = (uint32_t)kk * 32u;
        mma_tf32(tmem, desc_kmajor_sw128(rh + o), desc_kmajor_sw128(ch + o), idesc, (i > 0 || kk > 0) ? 1u : 0u);
        mma_tf32(tmem, desc_kmajor_sw128(rh + o), desc_kmajor_sw128(cl + o), idesc, 1u);
        mma_tf32(tmem, desc_kmajor_sw128(rl + o), desc_kmajor_sw128(ch + o), idesc, 1u);
      }
      mma_commit(empty(s));
      ++issued;
    }
    if (ok && nk > 0) {
      mma_commit(acc_full);
    } else if (issued > 0) {
      // let the MMAs already issued finish before TMEM is released
      mma_commit(drain);
      mbar_wait(drain, 0, abort_flag, status, ST_G_DRAIN);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

// Column tile width and K splits for a GEMM of Rrows x Ccols per group:
// 128 columns when that alone gives a wave of CTAs (148 SMs), else 64; K is
// split (auto_split) until about two waves are in flight, keeping at least 4
// K chunks per split.
struct Plan {
  int bn, splits, kps;
};
inline Plan plan(int Rrows, int Ccols, int K, int groups, bool auto_split) {
  Plan p;
  const long long rt = (Rrows + BM - 1) / BM;
  p.bn = rt * ((Ccols + 127) / 128) * groups >= 148 ? 128 : 64;
  const long long tiles = rt * ((Ccols + p.bn - 1) / p.bn) * groups;
  const int nchunks = K > 0 ? (K + BKF - 1) / BKF : 1;
  int splits = 1;
  if (auto_split && tiles > 0 && tiles < 2 * 148) {
    splits = (int)((2 * 148 + tiles - 1) / tiles);
    if (splits > nchunks / 4) splits = nchunks / 4;
    if (splits < 1) splits = 1;
  }
  const int cps = (nchunks + splits - 1) / splits;  // chunks per split
  p.kps = cps * BKF;
  p.splits = (nchunks + cps - 1) / cps;  // every split non-empty
  if (p.splits < 1) p.splits = 1;
  return p;
}

// Launch: the callers' GEMM C[m][n] = sum_k A(k, m) B(k, n) (A: M x K via
// la(g, k, m), B: via lb(g, k, n)), as D[r = n][c = m]; ep(g, m, n, value).
// auto_split: the epilogue accumulates (atomics), so K may be split.
template <bool A_KFAST, bool B_KFAST, class LA, class LB, class EP>
cudaError_t launch_tf32x3(const LA& la, const LB& lb, const EP& ep, int M, int N, int K, int groups,
                          bool auto_split, cudaStream_t st) {
  if (M <= 0 || N <= 0 || groups <= 0) return cudaSuccess;
  int* status = nullptr;
  cudaError_t e = tc_status_ptr(&status);
  if (e != cudaSuccess) return e;
  const Plan p = plan(N, M, K, groups, auto_split);
  const dim3 grid((unsigned)((M + p.bn - 1) / p.bn), (unsigned)((N + BM - 1) / BM), (unsigned)(groups * p.splits));
  const int smem = (int)smem_layout(p.bn).total + 1024;
  if (p.bn == 128) {
    auto kern = tf32x3_gemm_kernel<128, B_KFAST, A_KFAST, LB, LA, EP>;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
    kern<<<grid, NTHREADS, smem, st>>>(lb, la, ep, N, M, K, p.splits, p.kps, status);
  } else {
    auto kern = tf32x3_gemm_kernel<64, B_KFAST, A_KFAST, LB, LA, EP>;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
    kern<<<grid, NTHREADS, smem, st>>>(lb, la, ep, N, M, K, p.splits, p.kps, status);
  }
  return cudaGetLastError();
}

}  // namespace tf32g
}  // namespace dcn
