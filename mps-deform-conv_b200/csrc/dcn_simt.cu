// dcn_simt.cu -- general-purpose CUDA-core kernels for deformable convolution.
//
// These handle every dtype and every shape (any channel count, kernel size,
// group split) with fp32 accumulation, and they implement the reference's
// column-buffer interface (im2col / col2im / col2im_coord).  The tensor-core
// kernels in dcn_tc.cu take over the shapes they support for fp16/bf16.
//
//   im2col        reference deformable_im2col_*      deform_conv2d_mps.mm:105-340
//   col2im        reference deformable_col2im_fp32   deform_conv2d_mps.mm:344-417
//   col2im_coord  reference deformable_col2im_coord  deform_conv2d_mps.mm:423-519
//   gemm kernels  reference at::mm / at::bmm / torch.mm (mm:765-782,
//                 __init__.py:281, :289-290), with the gather fused into the
//                 operand loader so no column buffer is needed for fwd/wgrad.
#include "dcn_internal.h"

namespace dcn {

// ---------------------------------------------------------------- gather
// Column value col[c*T + t][b*HWo + p] computed on the fly.
template <typename T>
__device__ __forceinline__ float column_value(const Geom& g, const T* __restrict__ input,
                                              const T* __restrict__ offset,
                                              const T* __restrict__ mask, int b, int c, int t,
                                              int p) {
  float m;
  const SamplePos sp = sample_point(g, offset, mask, b, c / g.cpo, t, p, &m);
  const Corners cs = corners_of(sp, g.H, g.W);
  const T* plane = input + ((long long)b * g.C + c) * g.H * g.W;
  return m * bilinear(plane, cs);
}

// ---------------------------------------------------------------- SIMT GEMM
// C[M][N] = sum_k A(k, m) * B(k, n), per group g = blockIdx.z / splits, with
// the K range split `splits` ways (blockIdx.z % splits).  64x64x16 tiles, 256
// threads, 4x4 accumulators per thread.  Loaders are functors
// float operator()(g, k, mn); A_KFAST / B_KFAST pick which index varies
// fastest across threads during the load (the contiguous one in memory).
constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 16, SG_THREADS = 256;

template <bool KFAST, class L>
__device__ __forceinline__ void sg_load_tile(float (*S)[SG_BM + 4], const L& ld, int g, int k0,
                                             int kend, int mn0, int mnend, int tid) {
#pragma unroll
  for (int r = 0; r < (SG_BK * SG_BM) / SG_THREADS; ++r) {
    const int e = tid + r * SG_THREADS;
    int kk, mn;
    if (KFAST) { kk = e % SG_BK; mn = e / SG_BK; }
    else       { mn = e % SG_BM; kk = e / SG_BM; }
    const int k = k0 + kk, j = mn0 + mn;
    S[kk][mn] = (k < kend && j < mnend) ? ld(g, k, j) : 0.0f;
  }
}

template <bool A_KFAST, bool B_KFAST, class LA, class LB, class EP>
__global__ void __launch_bounds__(SG_THREADS)
simt_gemm_kernel(LA la, LB lb, EP ep, int M, int N, int K, int splits, int k_per_split) {
  __shared__ __align__(16) float As[SG_BK][SG_BM + 4];
  __shared__ __align__(16) float Bs[SG_BK][SG_BN + 4];
  const int tid = threadIdx.x;
  const int g = blockIdx.z / splits, s = blockIdx.z % splits;
  const int m0 = blockIdx.y * SG_BM, n0 = blockIdx.x * SG_BN;
  const int kbeg = s * k_per_split;
  const int kend = min(K, kbeg + k_per_split);
  const int tx = tid % 16, ty = tid / 16;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  for (int k0 = kbeg; k0 < kend; k0 += SG_BK) {
    sg_load_tile<A_KFAST>(As, la, g, k0, kend, m0, M, tid);
    sg_load_tile<B_KFAST>(Bs, lb, g, k0, kend, n0, N, tid);
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SG_BK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < M && n < N) ep(g, m, n, acc[i][j]);
    }
}

// The same GEMM with 128 x 128 x 8 tiles, 8 x 8 accumulators per thread
// (four times the FMAs per shared-memory load of the 64 x 64 kernel) and the
// next K tile's global loads in registers while the current tile computes
// (double-buffered shared memory, one barrier per K tile).  Thread (tx, ty)
// owns rows {4ty..4ty+3, 64+4ty..64+4ty+3} and the same pattern of columns,
// so its operand reads are two float4 per matrix per k, broadcast or on
// distinct banks.
constexpr int BG_BM = 128, BG_BN = 128, BG_BK = 8, BG_THREADS = 256;

template <bool KFAST, int BMN, class L>
__device__ __forceinline__ void bg_load_regs(float (&r)[4], const L& ld, int g, int k0, int kend, int mn0,
                                             int mnend, int tid) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int e = tid + i * BG_THREADS;
    int kk, mn;
    if (KFAST) { kk = e % BG_BK; mn = e / BG_BK; }
    else       { mn = e % BMN; kk = e / BMN; }
    const int k = k0 + kk, j = mn0 + mn;
    r[i] = (k < kend && j < mnend) ? ld(g, k, j) : 0.0f;
  }
}
template <bool KFAST, int BMN>
__device__ __forceinline__ void bg_store_regs(float (*S)[BMN + 4], const float (&r)[4], int tid) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int e = tid + i * BG_THREADS;
    int kk, mn;
    if (KFAST) { kk = e % BG_BK; mn = e / BG_BK; }
    else       { mn = e % BMN; kk = e / BMN; }
    S[kk][mn] = r[i];
  }
}

template <bool A_KFAST, bool B_KFAST, class LA, class LB, class EP>
__global__ void __launch_bounds__(BG_THREADS)
simt_gemm_big_kernel(LA la, LB lb, EP ep, int M, int N, int K, int splits, int k_per_split) {
  __shared__ __align__(16) float As[2][BG_BK][BG_BM + 4];
  __shared__ __align__(16) float Bs[2][BG_BK][BG_BN + 4];
  const int tid = threadIdx.x;
  const int g = blockIdx.z / splits, s = blockIdx.z % splits;
  const int m0 = blockIdx.y * BG_BM, n0 = blockIdx.x * BG_BN;
  const int kbeg = s * k_per_split;
  const int kend = min(K, kbeg + k_per_split);
  const int tx = tid % 16, ty = tid / 16;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  float ra[4], rb[4];
  if (kbeg < kend) {
    bg_load_regs<A_KFAST, BG_BM>(ra, la, g, kbeg, kend, m0, M, tid);
    bg_load_regs<B_KFAST, BG_BN>(rb, lb, g, kbeg, kend, n0, N, tid);
    bg_store_regs<A_KFAST, BG_BM>(As[0], ra, tid);
    bg_store_regs<B_KFAST, BG_BN>(Bs[0], rb, tid);
  }
  __syncthreads();
  int buf = 0;
  for (int k0 = kbeg; k0 < kend; k0 += BG_BK) {
    const bool more = k0 + BG_BK < kend;
    if (more) {  // the next tile's loads are in flight during this tile's FMAs
      bg_load_regs<A_KFAST, BG_BM>(ra, la, g, k0 + BG_BK, kend, m0, M, tid);
      bg_load_regs<B_KFAST, BG_BN>(rb, lb, g, k0 + BG_BK, kend, n0, N, tid);
    }
#pragma unroll
    for (int kk = 0; kk < BG_BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) {
      bg_store_regs<A_KFAST, BG_BM>(As[buf ^ 1], ra, tid);
      bg_store_regs<B_KFAST, BG_BN>(Bs[buf ^ 1], rb, tid);
    }
    __syncthreads();
    buf ^= 1;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
      const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (m < M && n < N) ep(g, m, n, acc[i][j]);
    }
}

// 128 x 128 tiles when they alone give at least a wave of CTAs (148 SMs),
// else 64 x 64 tiles.
template <bool A_KFAST, bool B_KFAST, class LA, class LB, class EP>
static cudaError_t launch_simt_gemm(const char* name, const LA& la, const LB& lb, const EP& ep,
                                    int M, int N, int K, int groups, int splits, cudaStream_t st) {
  if (M <= 0 || N <= 0 || groups <= 0) return cudaSuccess;
  const long long big_ctas = (long long)((N + BG_BN - 1) / BG_BN) * ((M + BG_BM - 1) / BG_BM) * groups * splits;
  KernelScope ks(name, st);
  if (big_ctas >= 148) {
    const int kps = ((K + splits - 1) / splits + BG_BK - 1) / BG_BK * BG_BK;
    dim3 grid((N + BG_BN - 1) / BG_BN, (M + BG_BM - 1) / BG_BM, groups * splits);
    simt_gemm_big_kernel<A_KFAST, B_KFAST><<<grid, BG_THREADS, 0, st>>>(la, lb, ep, M, N, K, splits, kps);
  } else {
    const int kps = ((K + splits - 1) / splits + SG_BK - 1) / SG_BK * SG_BK;
    dim3 grid((N + SG_BN - 1) / SG_BN, (M + SG_BM - 1) / SG_BM, groups * splits);
    simt_gemm_kernel<A_KFAST, B_KFAST><<<grid, SG_THREADS, 0, st>>>(la, lb, ep, M, N, K, splits, kps);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- functors
template <typename T>
struct WeightRowLoader {  // A(k, m) = W[g*Cog + m][k]   (forward)
  const T* w; int Cog, Kg;
  __device__ float operator()(int g, int k, int m) const {
    return to_f(w[(long long)(g * Cog + m) * Kg + k]);
  }
};
template <typename T>
struct WeightColLoader {  // A(co, m=k) = W[g*Cog + co][k]   (dgrad)
  const T* w; int Cog, Kg;
  __device__ float operator()(int g, int co, int k) const {
    return to_f(w[(long long)(g * Cog + co) * Kg + k]);
  }
};
template <typename T>
struct ColumnLoader {  // B(k, n) = col[(g*Cig + k/T)*T + k%T][n]   (forward)
  Geom geo; const T* x; const T* off; const T* msk;
  __device__ float operator()(int g, int k, int n) const {
    const int b = n / geo.HWo, p = n - b * geo.HWo;
    const int cl = k / geo.T, t = k - cl * geo.T;
    return column_value(geo, x, off, msk, b, g * geo.Cig + cl, t, p);
  }
};
// n / d for 0 <= n: a float-reciprocal quotient corrected to the exact one
// (n < 2^24), else the integer division.
__device__ __forceinline__ int div_rcp(int n, int d, float rcp) {
  if (n >= (1 << 24)) return n / d;
  int q = __float2int_rz((float)n * rcp);
  const int r = n - q * d;
  if (r < 0) --q;
  else if (r >= d) ++q;
  return q;
}
template <typename T>
struct GradOutLoaderCN {  // B(co, n=px) = gO[b][g*Cog + co][p]   (dgrad)
  Geom geo; const T* go; float rcp_hwo;
  __device__ float operator()(int g, int co, int n) const {
    const int b = div_rcp(n, geo.HWo, rcp_hwo), p = n - b * geo.HWo;
    return to_f(go[((long long)b * geo.Co + g * geo.Cog + co) * geo.HWo + p]);
  }
};
template <typename T>
struct GradOutLoaderPM {  // A(px, m=co) = gO[b][g*Cog + co][p]   (wgrad)
  Geom geo; const T* go; float rcp_hwo;
  __device__ float operator()(int g, int px, int co) const {
    const int b = div_rcp(px, geo.HWo, rcp_hwo), p = px - b * geo.HWo;
    return to_f(go[((long long)b * geo.Co + g * geo.Cog + co) * geo.HWo + p]);
  }
};
struct ColumnBufferLoader {  // B(k, n) = cols[(g*Kg + k)][n]   (forward, materialized columns)
  const float* cols; int Kg; long long P;
  __device__ float operator()(int g, int k, int n) const { return cols[((long long)g * Kg + k) * P + n]; }
};
struct ColumnBufferLoaderPK {  // B(px, n=k) = cols[(g*Kg + k)][px]   (wgrad, materialized columns)
  const float* cols; int Kg; long long P;
  __device__ float operator()(int g, int px, int k) const { return cols[((long long)g * Kg + k) * P + px]; }
};
template <typename T>
struct ForwardEpilogue {  // out[b][g*Cog + m][p] = acc + bias
  Geom geo; const T* bias; T* out;
  __device__ void operator()(int g, int m, int n, float acc) const {
    const int b = n / geo.HWo, p = n - b * geo.HWo;
    const int oc = g * geo.Cog + m;
    if (bias) acc += to_f(bias[oc]);
    out[((long long)b * geo.Co + oc) * geo.HWo + p] = from_f<T>(acc);
  }
};
struct ColumnStoreEpilogue {  // gcol[(g*Kg + m)][n] = acc
  float* gcol; int Kg; long long P;
  __device__ void operator()(int g, int m, int n, float acc) const {
    gcol[(long long)(g * Kg + m) * P + n] = acc;
  }
};
struct AtomicWeightEpilogue {  // gW32[(g*Cog + m)*Kg + n] += acc
  float* gw; int Cog, Kg;
  __device__ void operator()(int g, int m, int n, float acc) const {
    atomicAdd(&gw[(long long)(g * Cog + m) * Kg + n], acc);
  }
};

// ---------------------------------------------------------------- kernels
// Column buffer with one sample per (pixel, tap, offset group): thread e
// = (o, t, n) computes the sampling point once and writes the rows
// (o*cpo + c)*T + t of all the group's channels (coalesced over pixels n).
template <typename T, typename TC>
__global__ void im2col_og_kernel(Geom g, const T* __restrict__ x, const T* __restrict__ off,
                                 const T* __restrict__ msk, TC* __restrict__ cols) {
  const long long total = (long long)g.OG * g.T * g.P;
  const long long row_stride = (long long)g.T * g.P;  // channel c -> c + 1
  const long long plane = (long long)g.H * g.W;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long r = e / g.P, n = e - r * g.P;
    const int o = (int)(r / g.T), t = (int)(r - (long long)o * g.T);
    const int b = (int)(n / g.HWo), p = (int)(n - (long long)b * g.HWo);
    float m;
    const SamplePos sp = sample_point(g, off, msk, b, o, t, p, &m);
    const Corners cs = corners_of(sp, g.H, g.W);
    const T* src = x + ((long long)b * g.C + (long long)o * g.cpo) * plane;
    TC* dst = cols + ((long long)o * g.cpo * g.T + t) * g.P + n;
    for (int c = 0; c < g.cpo; ++c)
      dst[DCN_BOUND((long long)c * row_stride, 1, (long long)g.C * g.T * g.P - (dst - cols), DBG_SIMT_IM2COL)] =
          from_f<TC>(m * bilinear(src + (long long)c * plane, cs));
  }
}

// grad_input (fp32, zeroed) += col2im(gcol); gcol in the column layout.
template <typename TC, typename T>
__global__ void col2im_kernel(Geom g, const TC* __restrict__ gcol, const T* __restrict__ off,
                              const T* __restrict__ msk, float* __restrict__ gin) {
  const long long total = (long long)g.C * g.T * g.P;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long row = e / g.P, n = e - row * g.P;
    const int c = (int)(row / g.T), t = (int)(row - (long long)c * g.T);
    const int b = (int)(n / g.HWo), p = (int)(n - (long long)b * g.HWo);
    float m;
    const SamplePos sp = sample_point(g, off, msk, b, c / g.cpo, t, p, &m);
    const Corners cs = corners_of(sp, g.H, g.W);
    const float v = m * to_f(gcol[e]);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (cs.w[k] != 0.0f)
        atomicAdd(gin + DCN_BOUND(((long long)b * g.C + c) * g.H * g.W + cs.idx[k], 1, (long long)g.B * g.C * g.H * g.W,
                                  DBG_SIMT_COL2IM),
                  cs.w[k] * v);
  }
}

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// grad_input (channels-last fp32 [B][H][W][C], zeroed) += col2im(gcol), four
// channels of one sample per thread: the sampling point once for the four,
// and one 16-byte red.global.add.v4.f32 per corner (a quarter of
// col2im_kernel's reduction requests).  C and the channels per offset group
// are multiples of 4; acc is 16-byte aligned.
template <typename TC, typename T>
__global__ void col2im_nhwc4_kernel(Geom g, const TC* __restrict__ gcol, const T* __restrict__ off,
                                    const T* __restrict__ msk, float* __restrict__ acc) {
  const long long total = (long long)(g.C / 4) * g.T * g.P;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long row = e / g.P, n = e - row * g.P;  // row = (c/4)*T + t
    const int c4 = (int)(row / g.T), t = (int)(row - (long long)c4 * g.T);
    const int c = 4 * c4;
    const int b = (int)(n / g.HWo), p = (int)(n - (long long)b * g.HWo);
    float m;
    const SamplePos sp = sample_point(g, off, msk, b, c / g.cpo, t, p, &m);
    const Corners cs = corners_of(sp, g.H, g.W);
    const long long rs = (long long)g.T * g.P;  // channel c -> c + 1 in the column layout
    const TC* src = gcol + ((long long)c * g.T + t) * g.P + n;
    const float v0 = m * to_f(src[0]), v1 = m * to_f(src[rs]), v2 = m * to_f(src[2 * rs]), v3 = m * to_f(src[3 * rs]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float w = cs.w[k];
      if (w != 0.0f)
        red_add_v4(acc + DCN_BOUND(((long long)b * g.H * g.W + cs.idx[k]) * g.C + c, 4, (long long)g.B * g.H * g.W * g.C,
                                   DBG_SIMT_COL2IM_NHWC),
                   w * v0, w * v1, w * v2, w * v3);
    }
  }
}

// channels-last fp32 [B][HW][C] -> NCHW T [B][C][HW], 32 x 32 tiles through
// shared memory (33-word rows).  grid (HW/32, C/32, B), 256 threads.
template <typename T>
__global__ void nhwc_f32_to_nchw_kernel(const float* __restrict__ src, T* __restrict__ dst, int C, int HW) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z, c0 = blockIdx.y * 32, hw0 = blockIdx.x * 32;
  const float* s = src + (long long)b * HW * C;
  T* d = dst + (long long)b * C * HW;
  for (int e = threadIdx.x; e < 32 * 32; e += blockDim.x) {
    const int hh = e >> 5, cc = e & 31;
    if (hw0 + hh < HW && c0 + cc < C) tile[cc][hh] = s[(long long)(hw0 + hh) * C + c0 + cc];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 32 * 32; e += blockDim.x) {
    const int cc = e >> 5, hh = e & 31;
    if (hw0 + hh < HW && c0 + cc < C) d[(long long)(c0 + cc) * HW + hw0 + hh] = from_f<T>(tile[cc][hh]);
  }
}

// grad_offset / grad_mask, one thread per (b, offset group, tap, pixel).
template <typename TC, typename T>
__global__ void col2im_coord_kernel(Geom g, const TC* __restrict__ gcol, const T* __restrict__ x,
                                    const T* __restrict__ off, const T* __restrict__ msk,
                                    T* __restrict__ goff, T* __restrict__ gmsk) {
  const long long total = (long long)g.B * g.OG * g.T * g.HWo;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(e % g.HWo);
    long long r = e / g.HWo;
    const int t = (int)(r % g.T); r /= g.T;
    const int o = (int)(r % g.OG);
    const int b = (int)(r / g.OG);
    float m;
    const SamplePos sp = sample_point(g, off, msk, b, o, t, p, &m);
    const CoordCorners cc = coord_corners_of(sp, g.H, g.W);
    const Corners cs = corners_of(sp, g.H, g.W);
    float gy = 0.f, gx = 0.f, gm = 0.f;
    for (int cl = 0; cl < g.cpo; ++cl) {
      const int c = o * g.cpo + cl;
      const T* plane = x + ((long long)b * g.C + c) * g.H * g.W;
      const float v = to_f(gcol[((long long)c * g.T + t) * g.P + (long long)b * g.HWo + p]);
      const float v00 = cc.v[0] ? to_f(plane[cc.idx[0]]) : 0.f;
      const float v01 = cc.v[1] ? to_f(plane[cc.idx[1]]) : 0.f;
      const float v10 = cc.v[2] ? to_f(plane[cc.idx[2]]) : 0.f;
      const float v11 = cc.v[3] ? to_f(plane[cc.idx[3]]) : 0.f;
      float dy, dx;
      coord_grads(cc, v00, v01, v10, v11, &dy, &dx);
      gy += m * dy * v;
      gx += m * dx * v;
      if (g.use_mask) gm += v * bilinear(plane, cs);
    }
    const long long ob = ((long long)(b * g.OG + o) * 2 * g.T + 2 * t) * g.HWo + p;
    goff[ob] = from_f<T>(gy);
    goff[ob + g.HWo] = from_f<T>(gx);
    if (g.use_mask && gmsk) gmsk[((long long)(b * g.OG + o) * g.T + t) * g.HWo + p] = from_f<T>(gm);
  }
}

// grad_bias[co] = sum over (b, p) of grad_out[b][co][p]; one block per co.
template <typename T, typename TO>
__global__ void bias_grad_kernel(Geom g, const T* __restrict__ go, TO* __restrict__ gb) {
  const int co = blockIdx.x;
  float s = 0.f;
  for (int b = 0; b < g.B; ++b) {
    const T* row = go + ((long long)b * g.Co + co) * g.HWo;
    for (int p = threadIdx.x; p < g.HWo; p += blockDim.x) s += to_f(row[p]);
  }
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) gb[co] = from_f<TO>(s);
  }
}

template <typename T>
__global__ void f32_to_kernel(const float* __restrict__ src, T* __restrict__ dst, long long n) {
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x)
    dst[e] = from_f<T>(src[e]);
}

static inline int grid_for(long long n, int threads = 256) {
  long long b = (n + threads - 1) / threads;
  const long long cap = 148LL * 32;  // 148 SMs x 32 resident blocks of 256 max
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

// Forward K-split: split s of the reduction stores its partial output
// part[s][g*Cog + m][n] (n = b*HWo + p); simt_fwd_reduce adds the splits in
// order, plus bias, so the result does not depend on scheduling.
struct SplitPartialEpilogue {
  float* part; int splits, Co, Cog; long long P;
  __device__ void operator()(int g, int m, int n, float acc) const {
    const int s = blockIdx.z % splits;
    part[((long long)s * Co + g * Cog + m) * P + n] = acc;
  }
};

template <typename T>
__global__ void simt_fwd_reduce_kernel(Geom g, const float* __restrict__ part, int splits,
                                       const T* __restrict__ bias, T* __restrict__ out) {
  const long long total = (long long)g.Co * g.P;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int oc = (int)(e / g.P);
    const long long n = e - (long long)oc * g.P;
    float acc = bias ? to_f(bias[oc]) : 0.f;
    for (int s = 0; s < splits; ++s) acc += part[(long long)s * total + e];
    const int b = (int)(n / g.HWo), p = (int)(n - (long long)b * g.HWo);
    out[((long long)b * g.Co + oc) * g.HWo + p] = from_f<T>(acc);
  }
}

static int simt_fwd_splits(const Geom& g) {
  const long long tiles = ((g.P + SG_BN - 1) / SG_BN) * ((g.Cog + SG_BM - 1) / SG_BM) * g.G;
  if (tiles == 0) return 1;  // empty batch
  // the 128 x 128 tiles of launch_simt_gemm: split K until they make a wave
  const long long big = ((g.P + BG_BN - 1) / BG_BN) * ((g.Cog + BG_BM - 1) / BG_BM) * g.G;
  if (big >= 148) return 1;
  const int big_ksteps = (g.Cig * g.T + BG_BK - 1) / BG_BK;
  int splits = (int)((148 + big - 1) / big);
  if (splits > big_ksteps / 8) splits = big_ksteps / 8;  // at least 8 K steps per split
  if (splits >= 2 && big * splits >= 148) return splits;
  // else the 64 x 64 tiles: a wave of them, at least 4 K steps per split
  if (tiles >= 148) return 1;
  const int ksteps = (g.Cig * g.T + SG_BK - 1) / SG_BK;
  splits = (int)((148 + tiles - 1) / tiles);
  if (splits > ksteps / 4) splits = ksteps / 4;
  return splits < 2 ? 1 : splits;
}

// The forward materializes fp32 columns (one sample per pixel, tap and offset
// group, im2col_og_kernel) when that kernel has at least a wave of threads
// (148 x 256) and the columns take at most 1 GiB; other problems gather inside
// the GEMM's operand loader.
static size_t simt_fwd_cols_bytes(const Geom& g) {
  const size_t b = sizeof(float) * (size_t)g.C * g.T * (size_t)g.P;
  const long long threads = (long long)g.OG * g.T * g.P;
  return (threads >= 148 * 256 && b <= (size_t(1) << 30)) ? b : 0;
}

size_t simt_forward_workspace(const Geom& g) {
  const int splits = simt_fwd_splits(g);
  return ws_align(simt_fwd_cols_bytes(g)) + (splits > 1 ? sizeof(float) * (size_t)splits * g.Co * g.P : 0);
}

// ---------------------------------------------------------------- host side
template <typename T>
cudaError_t simt_forward(const Geom& g, const T* x, const T* w, const T* off, const T* msk,
                         const T* bias, T* out, void* workspace, cudaStream_t st) {
  const int Kg = g.Cig * g.T;
  WeightRowLoader<T> la{w, g.Cog, Kg};
  const size_t cols_bytes = workspace ? simt_fwd_cols_bytes(g) : 0;
  float* cols = cols_bytes ? static_cast<float*>(workspace) : nullptr;
  const int splits = workspace ? simt_fwd_splits(g) : 1;
  float* part = splits > 1 ? reinterpret_cast<float*>(static_cast<char*>(workspace) + ws_align(cols_bytes)) : nullptr;
  cudaError_t e;
  if (cols) {
    KernelScope ks("im2col_og", st);
    im2col_og_kernel<T, float><<<grid_for((long long)g.OG * g.T * g.P), 256, 0, st>>>(g, x, off, msk, cols);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  auto gemm = [&](const auto& ep, int nsplit) {
    if (cols) {
      ColumnBufferLoader lb{cols, Kg, g.P};
      return launch_simt_gemm<false, false>("simt_fwd_gemm", la, lb, ep, g.Cog, (int)g.P, Kg, g.G, nsplit, st);
    }
    ColumnLoader<T> lb{g, x, off, msk};
    return launch_simt_gemm<false, false>("simt_fwd_gemm", la, lb, ep, g.Cog, (int)g.P, Kg, g.G, nsplit, st);
  };
  if (!part) return gemm(ForwardEpilogue<T>{g, bias, out}, 1);
  if ((e = gemm(SplitPartialEpilogue{part, splits, g.Co, g.Cog, g.P}, splits)) != cudaSuccess) return e;
  KernelScope ks("simt_fwd_reduce", st);
  simt_fwd_reduce_kernel<T><<<grid_for((long long)g.Co * g.P), 256, 0, st>>>(g, part, splits, bias, out);
  return cudaGetLastError();
}

template <typename T>
cudaError_t simt_im2col(const Geom& g, const T* x, const T* off, const T* msk, T* cols,
                        cudaStream_t st) {
  const long long total = (long long)g.C * g.T * g.P;
  if (total == 0) return cudaSuccess;
  KernelScope ks("im2col", st);
  im2col_og_kernel<T, T><<<grid_for((long long)g.OG * g.T * g.P), 256, 0, st>>>(g, x, off, msk, cols);
  return cudaGetLastError();
}

template <typename TC, typename T>
cudaError_t simt_col2im(const Geom& g, const TC* gcol, const T* off, const T* msk, float* gin32,
                        cudaStream_t st) {
  const long long total = (long long)g.C * g.T * g.P;
  if (total == 0) return cudaSuccess;
  KernelScope ks("col2im", st);
  col2im_kernel<TC, T><<<grid_for(total), 256, 0, st>>>(g, gcol, off, msk, gin32);
  return cudaGetLastError();
}

template <typename TC, typename T>
cudaError_t simt_col2im_coord(const Geom& g, const TC* gcol, const T* x, const T* off,
                              const T* msk, T* goff, T* gmsk, cudaStream_t st) {
  const long long total = (long long)g.B * g.OG * g.T * g.HWo;
  if (total == 0) return cudaSuccess;
  KernelScope ks("col2im_coord", st);
  col2im_coord_kernel<TC, T><<<grid_for(total), 256, 0, st>>>(g, gcol, x, off, msk, goff, gmsk);
  return cudaGetLastError();
}

template <typename T>
cudaError_t convert_f32(const float* src, T* dst, long long n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  KernelScope ks("f32_convert", st);
  f32_to_kernel<T><<<grid_for(n), 256, 0, st>>>(src, dst, n);
  return cudaGetLastError();
}

// Full backward on the SIMT kernels.  Workspace: gcol (fp32 columns), plus
// fp32 accumulators for grad_input / grad_weight when T is not float.
template <typename T>
cudaError_t simt_backward(const Geom& g, const T* go, const T* x, const T* w, const T* off,
                          const T* msk, T* gin, T* gw, T* goff, T* gmsk, T* gb,
                          const SimtBackwardWs& ws, cudaStream_t st) {
  cudaError_t e = cudaSuccess;
  const int Kg = g.Cig * g.T;
  if (gb) {
    {
      KernelScope ks("bias_grad", st);
      bias_grad_kernel<T, T><<<g.Co, 256, 0, st>>>(g, go, gb);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (gw) {
    float* gw32 = ws.gw32 ? ws.gw32 : reinterpret_cast<float*>(gw);
    if ((e = cudaMemsetAsync(gw32, 0, sizeof(float) * (size_t)g.Co * Kg, st)) != cudaSuccess) return e;
    // split the pixel reduction so that ~2 waves of CTAs are in flight
    const long long tiles = (long long)((g.Cog + 63) / 64) * ((Kg + 63) / 64) * g.G;
    long long splits = (2 * 148 * 4 + tiles - 1) / tiles;
    const long long max_splits = (g.P + 255) / 256;
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
    GradOutLoaderPM<T> la{g, go, 1.f / (float)g.HWo};
    AtomicWeightEpilogue ep{gw32, g.Cog, Kg};
    // the columns, one sample per (pixel, tap, offset group), in the column
    // gradient's buffer (free until the dgrad GEMM below writes it)
    {
      KernelScope ks("im2col_og", st);
      im2col_og_kernel<T, float><<<grid_for((long long)g.OG * g.T * g.P), 256, 0, st>>>(g, x, off, msk, ws.gcol);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    ColumnBufferLoaderPK lb{ws.gcol, Kg, g.P};
    if ((e = launch_simt_gemm<true, true>("simt_wgrad_gemm", la, lb, ep, g.Cog, Kg, (int)g.P, g.G, (int)splits, st)) != cudaSuccess)
      return e;
    if (ws.gw32 && (e = convert_f32<T>(ws.gw32, gw, (long long)g.Co * Kg, st)) != cudaSuccess) return e;
  }
  if (gin || goff || gmsk) {
    WeightColLoader<T> la{w, g.Cog, Kg};
    GradOutLoaderCN<T> lb{g, go, 1.f / (float)g.HWo};
    ColumnStoreEpilogue ep{ws.gcol, Kg, g.P};
    if ((e = launch_simt_gemm<false, false>("simt_dgrad_gemm", la, lb, ep, Kg, (int)g.P, g.Cog, g.G, 1, st)) != cudaSuccess)
      return e;
    if (gin) {
      const long long n = (long long)g.B * g.C * g.H * g.W;
      if (ws.gacc && g.C % 4 == 0 && g.cpo % 4 == 0 && n > 0) {
        // four channels per thread into a channels-last accumulator, then NCHW
        if ((e = cudaMemsetAsync(ws.gacc, 0, sizeof(float) * (size_t)n, st)) != cudaSuccess) return e;
        {
          KernelScope ks("col2im_nhwc4", st);
          col2im_nhwc4_kernel<float, T><<<grid_for((long long)(g.C / 4) * g.T * g.P), 256, 0, st>>>(
              g, ws.gcol, off, msk, ws.gacc);
        }
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        KernelScope ks("nhwc_f32_to_nchw", st);
        const dim3 grid((unsigned)((g.H * g.W + 31) / 32), (unsigned)((g.C + 31) / 32), (unsigned)g.B);
        nhwc_f32_to_nchw_kernel<T><<<grid, 256, 0, st>>>(ws.gacc, gin, g.C, g.H * g.W);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
      } else {
        float* gin32 = ws.gin32 ? ws.gin32 : reinterpret_cast<float*>(gin);
        if ((e = cudaMemsetAsync(gin32, 0, sizeof(float) * (size_t)n, st)) != cudaSuccess) return e;
        if ((e = simt_col2im<float, T>(g, ws.gcol, off, msk, gin32, st)) != cudaSuccess) return e;
        if (ws.gin32 && (e = convert_f32<T>(ws.gin32, gin, n, st)) != cudaSuccess) return e;
      }
    }
    if (goff || gmsk) {
      T* goff_t = goff ? goff : reinterpret_cast<T*>(ws.goff_scratch);
      if ((e = simt_col2im_coord<float, T>(g, ws.gcol, x, off, msk, goff_t, gmsk, st)) != cudaSuccess)
        return e;
    }
  }
  return cudaSuccess;
}

// ---------------------------------------------------------------- instances
#define DCN_SIMT_INSTANCES(T)                                                                    \
  template cudaError_t simt_forward<T>(const Geom&, const T*, const T*, const T*, const T*,      \
                                       const T*, T*, void*, cudaStream_t);                       \
  template cudaError_t simt_im2col<T>(const Geom&, const T*, const T*, const T*, T*,            \
                                      cudaStream_t);                                             \
  template cudaError_t simt_col2im<T, T>(const Geom&, const T*, const T*, const T*, float*,     \
                                         cudaStream_t);                                          \
  template cudaError_t simt_col2im_coord<T, T>(const Geom&, const T*, const T*, const T*,       \
                                               const T*, T*, T*, cudaStream_t);                  \
  template cudaError_t convert_f32<T>(const float*, T*, long long, cudaStream_t);               \
  template cudaError_t simt_backward<T>(const Geom&, const T*, const T*, const T*, const T*,    \
                                        const T*, T*, T*, T*, T*, T*, const SimtBackwardWs&,     \
                                        cudaStream_t);

DCN_SIMT_INSTANCES(float)
DCN_SIMT_INSTANCES(__half)
DCN_SIMT_INSTANCES(__nv_bfloat16)

DCN_DEBUG_BOUNDS_TU(simt)

}  // namespace dcn
