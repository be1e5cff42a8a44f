// dcn_tc_bwd.cu -- tensor-core (tcgen05 / TMEM) backward for sm_100a.
//
// The reference's backward (mps_deform_conv/__init__.py:245-322) recomputes the
// column buffer, runs two torch.mm GEMMs and two scatter/reduce kernels
// (deform_conv2d_mps.mm:344-519).  Here:
//
//   prep        grad_output NCHW -> pixel-major gOt[P][Co] (+ grad_bias sums),
//               input -> channels-last, weight -> W^T tiles for dgrad.
//   dgrad       (dcn_dgrad_tc_kernel) per 128-pixel tile: gcol = gOt . W^T on
//               tcgen05 into TMEM, one 64-channel K chunk (tap, channels) at a
//               time; the epilogue reads each gcol tile from TMEM and, without
//               writing it anywhere, (a) gathers the 4 bilinear corners of the
//               input to reduce the offset and mask gradients over channels
//               (col2im_coord, mm:423-519) and (b) scatters mask * weight *
//               gcol into an fp32 channels-last grad_input with vector
//               red.global.add.v4.f32 (col2im, mm:344-417).
//   wgrad       (dcn_wgrad_tc_kernel) gW[co][k] = sum_p gOt[p][co] col[p][k]:
//               the forward's gather producer rebuilds col tiles in shared
//               memory as the MN-major B operand, gOt tiles arrive by TMA as
//               the MN-major A operand; each CTA owns a few K chunks and a
//               range of pixel tiles, accumulates in TMEM and adds its partial
//               gW into an fp32 buffer.
//   finalize    fp32 accumulators -> caller dtype / NCHW.
#include <cmath>

#include "dcn_layout.cuh"
#include "dcn_tc_common.cuh"

namespace dcn {

using namespace sm100;
using namespace tcc;

namespace {

constexpr int ST_W_PROD = 21, ST_W_MMA = 22, ST_W_LOAD = 23, ST_W_EPI = 24, ST_W_DRAIN = 25;
constexpr int ST_D_MMA = 31, ST_D_LOAD = 32, ST_D_EPI = 33, ST_D_DRAIN = 34;

// ================================================================ wgrad
constexpr int W_NPROD_WARPS = GATHER_WARPS;
constexpr int W_NPROD = GATHER_THREADS;
constexpr int W_MMA_WARP = W_NPROD_WARPS;
constexpr int W_NTHREADS = (W_NPROD_WARPS + 2) * 32;

struct WgradArgs {
  const void* xh;
  const void* off;
  const void* msk;
  float* gwp;      // per-split partial gW [splits][Co][nkc][64] fp32 (kc in gather order)
  int* status;
  Geom g;
  int nkc;         // K chunks per group, kc = t * (Cig/64) + cc (gather order)
  int nkg;         // K chunks per CTA
  int mh;          // M halves of 128 output channels
  int ncb;         // 64-channel blocks of grad_output loaded per tile
  int tiles_per_cta;
  int n_tiles;
  int a_stages, b_stages;
  uint32_t idesc;
  uint32_t tmem_cols;
};

// One 16-column TMEM load of the gW accumulator (row co, channels c16*16 ..
// c16*16+15 of K chunk kc) into this CTA's split of the partial buffer: plain
// 16-byte stores, every element written by exactly one CTA.
__device__ __forceinline__ void store_wgrad_partial(const WgradArgs& a, int co, int kc, int c16,
                                                    const uint32_t (&v)[16]) {
  const Geom& g = a.g;
  float4* dst = reinterpret_cast<float4*>(
      a.gwp + ((((size_t)blockIdx.z * g.Co + (size_t)blockIdx.y * g.Cog + co) * a.nkc + kc) * 64 + c16 * 16));
#pragma unroll
  for (int i = 0; i < 4; ++i)
    dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]), __uint_as_float(v[4 * i + 2]),
                         __uint_as_float(v[4 * i + 3]));
}

struct WgradSmem {
  uint32_t a, a_stage, b, bar, total;
};
__host__ __device__ inline WgradSmem wgrad_smem(int mh, int a_stages, int b_stages) {
  WgradSmem L;
  L.a = 0;
  L.a_stage = (uint32_t)(2 * mh) * A_STAGE_BYTES;
  L.b = L.a + a_stages * L.a_stage;
  L.bar = L.b + b_stages * A_STAGE_BYTES;
  L.total = L.bar + (2 * a_stages + 2 * b_stages + 2) * 8 + 16;
  return L;
}

// LOGIT = a.g.msk_logit (mask logits of the DCNv2 head layout)
template <typename T, bool LOGIT>
__global__ void __launch_bounds__(W_NTHREADS, 1)
dcn_wgrad_tc_kernel(const WgradArgs a, const __grid_constant__ CUtensorMap tmap_go) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Geom& g = a.g;
  const int AS = a.a_stages, BS = a.b_stages;
  const WgradSmem L = wgrad_smem(a.mh, AS, BS);
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bar0 = sbase + L.bar;
  auto a_full = [&](int s) { return bar0 + 8u * s; };
  auto a_empty = [&](int s) { return bar0 + 8u * (AS + s); };
  auto b_full = [&](int s) { return bar0 + 8u * (2 * AS + s); };
  auto b_empty = [&](int s) { return bar0 + 8u * (2 * AS + BS + s); };
  const uint32_t d_full = bar0 + 8u * (2 * AS + 2 * BS);
  const uint32_t drain = d_full + 8u;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + (2 * AS + 2 * BS + 2) * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(tmem_slot) + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = blockIdx.y;
  const int k0 = blockIdx.x * a.nkg;
  const int nk = min(a.nkg, a.nkc - k0);
  const int t0 = blockIdx.z * a.tiles_per_cta;
  const int nt = max(0, min(a.tiles_per_cta, a.n_tiles - t0));

  if (threadIdx.x == 0) {
    for (int s = 0; s < AS; ++s) { mbar_init(a_full(s), 1); mbar_init(a_empty(s), 1); }
    for (int s = 0; s < BS; ++s) { mbar_init(b_full(s), W_NPROD); mbar_init(b_empty(s), 1); }
    mbar_init(d_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == W_MMA_WARP) {
    tmem_alloc(smem_addr(tmem_slot), a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const T* xh = static_cast<const T*>(a.xh);
  const T* off = static_cast<const T*>(a.off);
  const T* msk = static_cast<const T*>(a.msk);

  if (warp < W_NPROD_WARPS) {
    // -------------------------------------------- col-tile producers
    const int r0 = warp * 8 + (lane >> 3), q = lane & 7;
    bool ok = true;
    Ring ring{0, BS, 0u};  // continues across the CTA's pixel tiles
    for (int li = 0; li < nt && ok; ++li) {
      const PixelCtx pc[2] = {pixel_ctx(g, (long long)(t0 + li) * BM + r0),
                              pixel_ctx(g, (long long)(t0 + li) * BM + r0 + 4)};
      auto stage_of = [&](int s, uint8_t*& t, uint32_t& eb, uint32_t& fb) {
        t = smem + L.b + s * A_STAGE_BYTES;
        eb = b_empty(s);
        fb = b_full(s);
      };
      ok = gather_run<T, LOGIT>(g, xh, off, msk, pc, r0, q, grp * g.Cig, k0, nk, ring, abort_flag, a.status,
                                ST_W_PROD, stage_of);
    }
    // -------------------------------------------- epilogue: TMEM -> this split's partial gW
    const bool ready = nt > 0 && ok && mbar_wait(d_full, 0, abort_flag, a.status, ST_W_EPI);
    if (__all_sync(0xffffffffu, ready)) {
      tc_fence_after();
      const int q = warp & 3, quarter = warp >> 2;
      for (int blk = quarter; blk < a.mh * nk; blk += W_NPROD_WARPS / 4) {
        const int h = blk / nk, kcl = blk % nk;
        const int co = h * BM + q * 32 + lane;
        const uint32_t col = (uint32_t)((h * a.nkg + kcl) * 64);
#pragma unroll 1
        for (int c16 = 0; c16 < 4; ++c16) {
          uint32_t v[16];
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + col + c16 * 16, v);
          tmem_ld_wait();
          if (co < g.Cog) store_wgrad_partial(a, co, k0 + kcl, c16, v);
        }
      }
    }
  } else if (warp == W_MMA_WARP) {
    // -------------------------------------------- MMA issuer
    if (lane == 0 && nt > 0) {
      bool ok = true;
      int committed = 0;
      for (int li = 0; li < nt && ok; ++li) {
        const int as = li % AS;
        ok = mbar_wait(a_full(as), (li / AS) & 1, abort_flag, a.status, ST_W_MMA);
        if (!ok) break;
        const uint32_t abase = sbase + L.a + as * L.a_stage;
        for (int kcl = 0; kcl < nk && ok; ++kcl) {
          const int j = li * nk + kcl;
          const int s = j % BS;
          ok = mbar_wait(b_full(s), (j / BS) & 1, abort_flag, a.status, ST_W_MMA);
          if (!ok) break;
          tc_fence_after();
          const uint32_t bbase = sbase + L.b + s * A_STAGE_BYTES;
          for (int h = 0; h < a.mh; ++h) {
            const uint32_t dcol = (uint32_t)((h * a.nkg + kcl) * 64);
#pragma unroll
            for (int kk = 0; kk < BM / 16; ++kk) {
              const uint64_t ad = desc_mnmajor_sw128(abase + h * 2 * A_STAGE_BYTES + kk * 2048, A_STAGE_BYTES);
              const uint64_t bd = desc_mnmajor_sw128(bbase + kk * 2048, A_STAGE_BYTES);
              mma_f16(tmem + dcol, ad, bd, a.idesc, (li > 0 || kk > 0) ? 1u : 0u);
            }
          }
          mma_commit(b_empty(s));
          ++committed;
        }
        if (ok) mma_commit(a_empty(as));
      }
      if (ok) {
        mma_commit(d_full);
      } else if (committed > 0) {
        mma_commit(drain);
        mbar_wait(drain, 0, abort_flag, a.status, ST_W_DRAIN);
      }
    }
  } else {
    // -------------------------------------------- grad_output tiles by TMA
    if (lane == 0 && nt > 0) {
      int issued = 0;
      const uint32_t bytes = (uint32_t)a.ncb * A_STAGE_BYTES;
      for (int li = 0; li < nt; ++li) {
        const int s = li % AS;
        if (!mbar_wait(a_empty(s), ((li / AS) & 1) ^ 1, abort_flag, a.status, ST_W_LOAD)) break;
        mbar_arrive_expect_tx(a_full(s), bytes);
        const uint32_t dst = sbase + L.a + s * L.a_stage;
        for (int cb = 0; cb < a.ncb; ++cb)
          tma_load_2d(dst + cb * A_STAGE_BYTES, &tmap_go, grp * g.Cog + cb * 64, (t0 + li) * BM, a_full(s));
        ++issued;
      }
      for (int li = (issued > AS ? issued - AS : 0); li < issued; ++li)
        mbar_wait(a_full(li % AS), (li / AS) & 1, abort_flag, a.status, ST_W_LOAD);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == W_MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, a.tmem_cols);
  }
}

// ---------------------------------------------------------------- wgrad from saved columns
// Same GEMM as dcn_wgrad_tc_kernel, but the column tiles are the forward's
// (saved in their shared-memory image) and arrive by bulk copy: no gather.
// The reduction over pixels runs in 64-pixel slices; one stage holds the
// slice of grad_output (A, MN-major [64 px][Cog]) and the same slice of all
// nk column tiles of the CTA side by side (B, MN-major [64 px][nk*64]), so
// each MMA is M=128 x N=64*nk x K=16 and reads few operand bytes per FLOP.
// Warps 0-3 epilogue, warp 4 MMA, warp 5 loader.
constexpr int WC_EPI_WARPS = 4;
constexpr int WC_MMA_WARP = 4;
constexpr int WC_NTHREADS = 192;
constexpr int WC_SLICE = 64;                        // pixels per stage
constexpr int WC_HALF_TILE = WC_SLICE * 128;        // 8 KB: 64 rows of 128 bytes

struct WgradColsSmem {
  uint32_t stage, a_bytes, b_bytes, bar, total;
  int stages;
};
__host__ __device__ inline WgradColsSmem wgrad_cols_smem(int ncb_pad, int nkg, int stages) {
  WgradColsSmem L;
  L.a_bytes = (uint32_t)ncb_pad * WC_HALF_TILE;     // [64 px][64 co] blocks, ncb_pad = 2*mh
  L.b_bytes = (uint32_t)nkg * WC_HALF_TILE;         // [64 px][64 ch] per K chunk
  L.stage = L.a_bytes + L.b_bytes;
  L.stages = stages;
  L.bar = stages * L.stage;
  L.total = L.bar + (2 * stages + 2) * 8 + 16;
  return L;
}

template <typename T>
__global__ void __launch_bounds__(WC_NTHREADS, 1)
dcn_wgrad_cols_tc_kernel(const WgradArgs a, const void* __restrict__ cols,
                         const __grid_constant__ CUtensorMap tmap_go64) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Geom& g = a.g;
  const int S = a.b_stages;
  const WgradColsSmem L = wgrad_cols_smem(2 * a.mh, a.nkg, S);
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bar0 = sbase + L.bar;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (S + s); };
  const uint32_t d_full = bar0 + 8u * (2 * S);
  const uint32_t drain = d_full + 8u;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + (2 * S + 2) * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(tmem_slot) + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = blockIdx.y;
  const int k0 = blockIdx.x * a.nkg;
  const int nk = min(a.nkg, a.nkc - k0);
  const int t0 = blockIdx.z * a.tiles_per_cta;
  const int nt = max(0, min(a.tiles_per_cta, a.n_tiles - t0));
  const int nslices = nt * (BM / WC_SLICE);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(full(s), 1); mbar_init(empty(s), 1); }
    mbar_init(d_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == WC_MMA_WARP) {
    tmem_alloc(smem_addr(tmem_slot), a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < WC_EPI_WARPS) {
    // -------------------------------------------- epilogue: TMEM -> this split's partial gW
    const bool ready = nslices > 0 && mbar_wait(d_full, 0, abort_flag, a.status, ST_W_EPI);
    if (__all_sync(0xffffffffu, ready)) {
      tc_fence_after();
      const int q = warp;
      for (int blk = 0; blk < a.mh * nk; ++blk) {
        const int h = blk / nk, kcl = blk % nk;
        const int co = h * BM + q * 32 + lane;
        const uint32_t col = (uint32_t)(h * a.nkg * 64 + kcl * 64);
#pragma unroll 1
        for (int c16 = 0; c16 < 4; ++c16) {
          uint32_t v[16];
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + col + c16 * 16, v);
          tmem_ld_wait();
          if (co < g.Cog) store_wgrad_partial(a, co, k0 + kcl, c16, v);
        }
      }
    }
  } else if (warp == WC_MMA_WARP) {
    // -------------------------------------------- MMA issuer
    if (lane == 0 && nslices > 0) {
      // up to 4 K chunks (N = 256) per MMA; a 5th..8th chunk goes to a second MMA
      const int nsub = (nk + 3) / 4;
      const uint32_t idesc0 = idesc_f16_major(BM, 64 * min(nk, 4), a.idesc != 0, true, true);
      const uint32_t idesc1 = idesc_f16_major(BM, 64 * max(nk - 4, 1), a.idesc != 0, true, true);
      bool ok = true;
      int committed = 0;
      for (int i = 0; i < nslices && ok; ++i) {
        const int s = i % S;
        ok = mbar_wait(full(s), (i / S) & 1, abort_flag, a.status, ST_W_MMA);
        if (!ok) break;
        tc_fence_after();
        const uint32_t abase = sbase + s * L.stage;
        const uint32_t bbase = abase + L.a_bytes;
        for (int h = 0; h < a.mh; ++h) {
          for (int sub = 0; sub < nsub; ++sub) {
#pragma unroll
            for (int kk = 0; kk < WC_SLICE / 16; ++kk) {
              const uint64_t ad = desc_mnmajor_sw128(abase + h * 2 * WC_HALF_TILE + kk * 2048, WC_HALF_TILE);
              const uint64_t bd = desc_mnmajor_sw128(bbase + sub * 4 * WC_HALF_TILE + kk * 2048, WC_HALF_TILE);
              mma_f16(tmem + (uint32_t)(h * a.nkg * 64 + sub * 256), ad, bd, sub ? idesc1 : idesc0,
                      (i > 0 || kk > 0) ? 1u : 0u);
            }
          }
        }
        mma_commit(empty(s));
        ++committed;
      }
      if (ok) {
        mma_commit(d_full);
      } else if (committed > 0) {
        mma_commit(drain);
        mbar_wait(drain, 0, abort_flag, a.status, ST_W_DRAIN);
      }
    }
  } else {
    // -------------------------------------------- loader
    if (lane == 0 && nslices > 0) {
      const uint32_t bytes = (uint32_t)a.ncb * WC_HALF_TILE + (uint32_t)nk * WC_HALF_TILE;
      int issued = 0;
      for (int i = 0; i < nslices; ++i) {
        const int s = i % S;
        if (!mbar_wait(empty(s), ((i / S) & 1) ^ 1, abort_flag, a.status, ST_W_LOAD)) break;
        mbar_arrive_expect_tx(full(s), bytes);
        const int tile = t0 + i / (BM / WC_SLICE), half = i % (BM / WC_SLICE);
        const uint32_t dst = sbase + s * L.stage;
        for (int cb = 0; cb < a.ncb; ++cb)
          tma_load_2d(dst + cb * WC_HALF_TILE, &tmap_go64, grp * g.Cog + cb * 64, tile * BM + half * WC_SLICE,
                      full(s));
        const uint8_t* src = static_cast<const uint8_t*>(cols) +
                             (((size_t)grp * a.n_tiles + tile) * a.nkc + k0) * (size_t)A_STAGE_BYTES +
                             (size_t)half * WC_HALF_TILE;
        for (int kcl = 0; kcl < nk; ++kcl)
          bulk_g2s(dst + L.a_bytes + kcl * WC_HALF_TILE, src + (size_t)kcl * A_STAGE_BYTES, WC_HALF_TILE,
                   full(s));
        ++issued;
      }
      for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
        mbar_wait(full(i % S), (i / S) & 1, abort_flag, a.status, ST_W_LOAD);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == WC_MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, a.tmem_cols);
  }
}

// ================================================================ dgrad
constexpr int D_EPI_WARPS = 16;      // 4 groups of 4 warps, one group per TMEM buffer
constexpr int D_MMA_WARP = 16;
constexpr int D_LOAD_WARP = 17;
constexpr int D_NTHREADS = (D_LOAD_WARP + 1) * 32;  // 576: epilogue warps, MMA warp, loader warp
constexpr int D_NBUF = 4;            // TMEM gcol buffers of 64 columns

struct DgradArgs {
  const void* xh;
  const void* off;
  const void* msk;
  const void* wdt;   // W^T tiles [G][NKC][KB][64 ch][64 co], 128-byte swizzled rows
  float* gi32;       // channels-last [B][H][W][C], zeroed
  float* goff32;     // [B][OG*2T][HWo], zeroed
  float* gmsk32;     // [B][OG*T][HWo], zeroed (null without mask)
  const void* xq;    // quad epilogue (SW = 8): corner-quad records of the input
  void* goff_t;      // quad epilogue: grad_offset / grad_mask in the caller's dtype, written
  void* gmsk_t;      //   directly (each value has one writer); null when not wanted
  float* gq32;       // quad epilogue: fp32 corner-quad accumulator, zeroed (null: no grad_input)
  int* status;
  Geom g;
  int nkc;           // K chunks per group, kc = cc*T + t
  int kb;            // 64-channel blocks of the reduction over output channels
  int b_stages;
  uint32_t idesc;
  int tpc;           // pixel tiles per CTA, run back to back (>1 only for SW = 8)
  int ntiles;        // pixel tiles of the problem
};

// Per-warp epilogue scratch: a 16-channel gcol slab of the warp's 32 rows and
// the rows' sample table (2 eight-channel segments x 16 words: corner pixel
// indices, bilinear weights, fy, fx, mask, corner-valid bits, partial sums).
// Row strides of 20 and 36 words keep the 16-byte accesses aligned and
// spread over the banks.
struct DgWarpSmem {
  float slab[32][16];    // 16-byte chunk k of row r stored at chunk k ^ ((r >> 1) & 3)
  uint32_t tab[32][36];
};

// Chunk position in a slab row: conflict-free both for the row owner's
// 16-byte stores (8 rows per phase) and for the 4-lanes-per-row loads.
__device__ __forceinline__ int slab_pos(int r, int k) { return (k ^ ((r >> 1) & 3)) * 4; }

// Per-warp epilogue scratch of the 32-channel-slab variant (offset groups of
// a multiple of 32 channels, so a slab has one sample per pixel): the slab of
// 32 rows x 32 channels (16-byte chunk k of row r at chunk k ^ (r & 7), so
// that 8 rows' stores and 8 lanes' loads of one row both hit distinct banks)
// and one sample per row (corner pixel indices, bilinear weights, fy, fx,
// mask, valid bits; 48-byte rows: 4 rows read together hit distinct banks).
struct DgWarpSmem32 {
  float slab[32][32];
  uint32_t tab[32][12];
};

// 64-channel-slab variant (offset groups of a multiple of 64 channels, so a
// whole K chunk has one sample per pixel): the chunk's gcol row as 16-bit
// pairs (the precision of the reference's own 16-bit GEMM output), 16-byte
// chunk k of row r at chunk k ^ (r & 7), and the same per-row sample table.
struct DgWarpSmem64 {
  uint32_t slab[32][32];
  uint32_t tab[32][12];
};

// Per-warp epilogue scratch of the quad variant (offset groups of 8
// channels): the chunk's gcol rows as 16-bit pairs (as DgWarpSmem64), the
// warp's 32 pixels (image or -1, pixel, y and x base), and a staging area
// where each lane leaves its sample's 32 fp32 contributions (a corner-quad
// record, corner-major) and the record's index (-1: none) so that each
// reduction instruction can cover four whole records.
struct DgWarpSmemQ {
  uint32_t slab[32][32];
  int4 pix[32];
  float stage[32][32];
  int rec[32];
};

// Shared memory: the whole gOt tile [128 px][KB*64 co] stays resident; W^T
// streams through b_stages stages of one 8 KB K block ([64 ch][64 co]) each;
// then the epilogue warps' scratch.
struct DgradSmem {
  uint32_t a, b, b_stage, epi, bar, total;
};
__host__ __device__ inline DgradSmem dgrad_smem(int kb, int b_stages, int sw) {
  DgradSmem L;
  L.a = 0;
  L.b = (uint32_t)kb * A_STAGE_BYTES;
  L.b_stage = 8192u;
  L.epi = L.b + b_stages * L.b_stage;
  L.bar = L.epi + D_EPI_WARPS * (uint32_t)(sw == 64   ? sizeof(DgWarpSmem64)
                                            : sw == 32 ? sizeof(DgWarpSmem32)
                                            : sw == 8  ? sizeof(DgWarpSmemQ)
                                                       : sizeof(DgWarpSmem));
  L.total = L.bar + (1 + 2 * b_stages + 2 * D_NBUF + 2) * 8 + 16;
  return L;
}

__device__ __forceinline__ void red_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// SW = channels per epilogue pass: 64 when the offset groups are a multiple
// of 64 channels and B*H*W*C < 2^31 (one pass per K chunk, gcol held as
// 16-bit pairs, 16-byte corner loads); 32 when they are a multiple of 32
// channels (8 lanes x 4 channels per pixel: each corner's 32 fp32 gradients
// are one 128-byte line, half the lines per byte of SW = 16; 32-bit element
// offsets); 8 for offset groups of exactly 8 channels with 32-bit corner-quad
// offsets (one lane per (pixel, offset group): the sample's four corners
// from one corner-quad record, its offset and mask gradients complete in the
// lane, and its 32 contributions added to an fp32 corner-quad accumulator
// as one 128-byte line); else 16 (4 lanes x 4 channels, up to 2 offset
// groups per slab).
template <typename T, int SW>
__global__ void __launch_bounds__(D_NTHREADS, 1)
dcn_dgrad_tc_kernel(const DgradArgs a, const __grid_constant__ CUtensorMap tmap_go) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Geom& g = a.g;
  const int S = a.b_stages;
  const DgradSmem L = dgrad_smem(a.kb, S, SW);
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bar0 = sbase + L.bar;
  const uint32_t a_full = bar0;
  auto b_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto b_empty = [&](int s) { return bar0 + 8u * (1 + S + s); };
  auto d_full = [&](int e) { return bar0 + 8u * (1 + 2 * S + e); };
  auto d_empty = [&](int e) { return bar0 + 8u * (1 + 2 * S + D_NBUF + e); };
  const uint32_t drain = bar0 + 8u * (1 + 2 * S + 2 * D_NBUF);
  const uint32_t a_empty = bar0 + 8u * (2 + 2 * S + 2 * D_NBUF);  // a tile's MMAs are done with A
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + (1 + 2 * S + 2 * D_NBUF + 2) * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(reinterpret_cast<uint8_t*>(tmem_slot) + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // pixel tiles blockIdx.x + tl * gridDim.x (tl < ntile), one after the
  // other: chunk i of the CTA is K chunk kc_lo + i % nkc_cta of the CTA's
  // tile i / nkc_cta (the TMEM buffers keep cycling across the tiles, so the
  // epilogue groups stay evenly loaded when a tile has few chunks).  The CTAs
  // of a wave work on neighbouring tiles at any one time, as with one tile
  // per CTA, which keeps the scatter's target lines in L2.
  const int tile0 = blockIdx.x, grp = blockIdx.y;
  const int ntile = min(a.tpc, (a.ntiles - tile0 + (int)gridDim.x - 1) / (int)gridDim.x);
  auto tile_of = [&](int tl) { return tile0 + tl * (int)gridDim.x; };
  const int tile = tile0;  // single-tile epilogues (tpc = 1)
  // this CTA's share of the K chunks (several CTAs per tile balance the waves
  // when there are few tiles)
  const int kc_lo = (int)(((long long)a.nkc * blockIdx.z) / gridDim.z);
  const int nkc_cta = (int)(((long long)a.nkc * (blockIdx.z + 1)) / gridDim.z) - kc_lo;
  const int nchunks = ntile * nkc_cta;

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    for (int s = 0; s < S; ++s) { mbar_init(b_full(s), 1); mbar_init(b_empty(s), 1); }
    for (int e = 0; e < D_NBUF; ++e) { mbar_init(d_full(e), 1); mbar_init(d_empty(e), 4); }  // one per warp
    mbar_init(drain, 1);
    mbar_init(a_empty, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == D_MMA_WARP) {
    tmem_alloc(smem_addr(tmem_slot), 64 * D_NBUF);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < D_EPI_WARPS && SW == 64) {
    // -------------------------------------------- epilogue, one 64-channel pass per K chunk
    //  (1) row owner (lane = TMEM row = pixel): its 64 gcol values to the
    //      slab as 16-bit pairs (the TMEM buffer is then free for the next
    //      MMA) and the sample of the chunk's offset group into the table;
    //  (2) 8 lanes per pixel, 4 pixels per step: each lane loads 8
    //      consecutive channels of the 4 corners (16 bytes: one instruction
    //      covers 4 whole 128-byte lines) for the offset/mask dot products,
    //      and scatters channels 4j..4j+3 and 32+4j..32+4j+3 with two
    //      red.global.add.v4.f32 per corner (again whole lines); its partial
    //      sums go to the slab chunk it has consumed, and the row owner adds
    //      its row's 8 chunks to global memory once per (pixel, K chunk).
    const T* xh = static_cast<const T*>(a.xh);
    const T* off = static_cast<const T*>(a.off);
    const T* msk = static_cast<const T*>(a.msk);
    const int e = warp >> 2, q = warp & 3;
    DgWarpSmem64* ws = reinterpret_cast<DgWarpSmem64*>(smem + L.epi) + warp;
    const PixelCtx pc = pixel_ctx(g, (long long)tile * BM + q * 32 + lane);
    const int j8 = lane & 7, rsub = lane >> 3;
    bool ok = true;
    for (int i = e; i < nkc_cta; i += D_NBUF) {
      const bool ready = ok && mbar_wait(d_full(e), (i / D_NBUF) & 1, abort_flag, a.status, ST_D_EPI);
      ok = __all_sync(0xffffffffu, ready);
      if (!ok) break;
      tc_fence_after();
      KWalk kw;
      kw.start(g, kc_lo + i);
      const int cbase = grp * g.Cig + kw.cc * BK;
      // ---- phase 1: row owner
      {
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(e * 64);
        uint32_t* srow = ws->slab[lane];
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // channels 32h .. 32h+31 = chunks 4h .. 4h+3
          uint32_t a0[16], a1[16];
          tmem_ld16(taddr + h * 32, a0);
          tmem_ld16(taddr + h * 32 + 16, a1);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            *reinterpret_cast<uint4*>(srow + (((4 * h + k) ^ (lane & 7)) << 2)) = make_uint4(
                Vec<T>::pack(__uint_as_float(a0[8 * k]), __uint_as_float(a0[8 * k + 1])),
                Vec<T>::pack(__uint_as_float(a0[8 * k + 2]), __uint_as_float(a0[8 * k + 3])),
                Vec<T>::pack(__uint_as_float(a0[8 * k + 4]), __uint_as_float(a0[8 * k + 5])),
                Vec<T>::pack(__uint_as_float(a0[8 * k + 6]), __uint_as_float(a0[8 * k + 7])));
            *reinterpret_cast<uint4*>(srow + (((4 * h + 2 + k) ^ (lane & 7)) << 2)) = make_uint4(
                Vec<T>::pack(__uint_as_float(a1[8 * k]), __uint_as_float(a1[8 * k + 1])),
                Vec<T>::pack(__uint_as_float(a1[8 * k + 2]), __uint_as_float(a1[8 * k + 3])),
                Vec<T>::pack(__uint_as_float(a1[8 * k + 4]), __uint_as_float(a1[8 * k + 5])),
                Vec<T>::pack(__uint_as_float(a1[8 * k + 6]), __uint_as_float(a1[8 * k + 7])));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty(e));  // TMEM buffer read completely
      }
      const int o = cbase / g.cpo;  // one offset group per chunk
      float tab_m;
      {
        const RawSample<T> raw = load_raw(g, off, msk, pc, o, kw.t);
        const SamplePos sp = sample_pos(pc.y0 + kw.ti * g.dh, pc.x0 + kw.tj * g.dw, to_f(raw.dy), to_f(raw.dx));
        const Corners cs = corners_of(sp, g.H, g.W);
        const CoordCorners c4 = coord_corners_of(sp, g.H, g.W);
        uint32_t cvb = 0;
        int cidx[4];
        float cw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const bool v = pc.valid && c4.v[k];
          cvb |= (v ? 1u : 0u) << k;
          cidx[k] = v ? (int)((pc.img + c4.idx[k]) * g.C) : 0;  // element offset, B*H*W*C < 2^31
          cw[k] = pc.valid ? cs.w[k] : 0.f;
        }
        tab_m = pc.valid ? mask_of(g, to_f(raw.m)) : 0.f;
        uint32_t* trow = ws->tab[lane];
        *reinterpret_cast<uint4*>(trow) = make_uint4(cidx[0], cidx[1], cidx[2], cidx[3]);
        *reinterpret_cast<uint4*>(trow + 4) = make_uint4(__float_as_uint(cw[0]), __float_as_uint(cw[1]),
                                                         __float_as_uint(cw[2]), __float_as_uint(cw[3]));
        *reinterpret_cast<uint4*>(trow + 8) =
            make_uint4(__float_as_uint(c4.fy), __float_as_uint(c4.fx), __float_as_uint(tab_m), cvb);
      }
      __syncwarp();
      // ---- phase 2: 8 lanes per pixel, 4 pixels per step
      const uint32_t cl = (uint32_t)(cbase + j8 * 8);                 // dot-product channels
      const uint32_t cr0 = (uint32_t)(cbase + j8 * 4), cr1 = cr0 + 32;  // scattered channels
#pragma unroll 1
      for (int it = 0; it < 8; ++it) {
        const int rr = it * 4 + rsub;
        const uint32_t* tr = ws->tab[rr];
        const uint4 tb = *reinterpret_cast<const uint4*>(tr);
        const uint4 tw = *reinterpret_cast<const uint4*>(tr + 4);
        const uint4 tx = *reinterpret_cast<const uint4*>(tr + 8);
        uint32_t* srow = ws->slab[rr];
        const int sw7 = rr & 7;
        const uint4 gd = *reinterpret_cast<const uint4*>(srow + ((j8 ^ sw7) << 2));
        const uint2 gr0 = *reinterpret_cast<const uint2*>(srow + (((j8 >> 1) ^ sw7) << 2) + (j8 & 1) * 2);
        const uint2 gr1 = *reinterpret_cast<const uint2*>(srow + (((4 + (j8 >> 1)) ^ sw7) << 2) + (j8 & 1) * 2);
        const uint32_t cof[4] = {tb.x, tb.y, tb.z, tb.w};
        const float w[4] = {__uint_as_float(tw.x), __uint_as_float(tw.y), __uint_as_float(tw.z),
                            __uint_as_float(tw.w)};
        const float fy = __uint_as_float(tx.x), fx = __uint_as_float(tx.y), m = __uint_as_float(tx.z);
        const uint32_t cv = tx.w;
        uint4 xv[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          xv[k] = (cv >> k & 1u) ? __ldg(reinterpret_cast<const uint4*>(
                                       xh + DCN_BOUND(cof[k] + cl, 8, (long long)g.B * g.H * g.W * g.C, DBG_DG_CORNER_X)))
                                 : make_uint4(0, 0, 0, 0);
        const float2 g01 = Vec<T>::unpack(gd.x), g23 = Vec<T>::unpack(gd.y), g45 = Vec<T>::unpack(gd.z),
                     g67 = Vec<T>::unpack(gd.w);
        float d[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 x01 = Vec<T>::unpack(xv[k].x), x23 = Vec<T>::unpack(xv[k].y), x45 = Vec<T>::unpack(xv[k].z),
                       x67 = Vec<T>::unpack(xv[k].w);
          d[k] = g01.x * x01.x + g01.y * x01.y + g23.x * x23.x + g23.y * x23.y + g45.x * x45.x + g45.y * x45.y +
                 g67.x * x67.x + g67.y * x67.y;
        }
        const float pgm = w[0] * d[0] + w[1] * d[1] + w[2] * d[2] + w[3] * d[3];
        const float pgy = m * (fx * (d[3] - d[1]) + (1.f - fx) * (d[2] - d[0]));
        const float pgx = m * (fy * (d[3] - d[2]) + (1.f - fy) * (d[1] - d[0]));
        const float2 r01 = Vec<T>::unpack(gr0.x), r23 = Vec<T>::unpack(gr0.y);
        const float2 r45 = Vec<T>::unpack(gr1.x), r67 = Vec<T>::unpack(gr1.y);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float wk = w[k] * m;
          if (wk != 0.f) {
            red_v4(a.gi32 + DCN_BOUND(cof[k] + cr0, 4, (long long)g.B * g.H * g.W * g.C, DBG_DG_SCATTER), wk * r01.x, wk * r01.y, wk * r23.x,
                   wk * r23.y);
            red_v4(a.gi32 + DCN_BOUND(cof[k] + cr1, 4, (long long)g.B * g.H * g.W * g.C, DBG_DG_SCATTER), wk * r45.x, wk * r45.y, wk * r67.x,
                   wk * r67.y);
          }
        }
        __syncwarp();  // every lane has read this step's rows: the consumed chunks take the partial sums
        *reinterpret_cast<float4*>(srow + ((j8 ^ sw7) << 2)) = make_float4(pgy, pgx, pgm, 0.f);
      }
      __syncwarp();
      // ---- row owner: sum the 8 lanes' partials of its row, once per chunk
      {
        const uint32_t* srow = ws->slab[lane];
        float gy = 0.f, gx = 0.f, gm = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float4 pv = *reinterpret_cast<const float4*>(srow + ((k ^ (lane & 7)) << 2));
          gy += pv.x;
          gx += pv.y;
          gm += pv.z;
        }
        if (pc.valid) {
          const long long ob = DCN_BOUND((long long)pc.b * g.off_bs + (long long)(o * 2 * g.T + 2 * kw.t) * g.HWo + pc.p,
                                         g.HWo + 1, g.B * g.off_bs, DBG_DG_COORD);
          atomicAdd(a.goff32 + ob, gy);
          atomicAdd(a.goff32 + ob + g.HWo, gx);
          if (g.use_mask)  // d/dlogit = m (1 - m) d/dm for a mask stored as logits
            atomicAdd(a.gmsk32 + DCN_BOUND((long long)pc.b * g.msk_bs + (long long)(o * g.T + kw.t) * g.HWo + pc.p, 1,
                                           g.B * g.msk_bs, DBG_DG_COORD),
                      g.msk_logit ? gm * tab_m * (1.f - tab_m) : gm);
        }
      }
      __syncwarp();  // the next chunk's phase 1 rewrites the rows
    }
  } else if (warp < D_EPI_WARPS && SW == 8) {
    // -------------------------------------------- epilogue, corner-quad (offset groups of 8 channels)
    //  (1) row owner (lane = TMEM row = pixel): its 64 gcol values to the
    //      slab as 16-bit pairs; the TMEM buffer is then free;
    //  (2) lane = (pixel rr, offset group j8 of the chunk), 4 pixels per
    //      step: the sample from the offsets and mask, the four corners from
    //      its corner-quad record (two 256-bit loads), the offset and mask
    //      gradients (all 8 channels of the group are in the lane: plain
    //      stores, each (pixel, group, tap) is produced once), and the 32
    //      contributions mask * w_k * gcol_c to the warp's staging area;
    //      then 8 rounds in which 8 lanes add the 8 16-byte pieces of one
    //      record with red.global.add.v4.f32, four whole records (128-byte
    //      lines) per instruction.
    const T* xq = static_cast<const T*>(a.xq);
    const T* off = static_cast<const T*>(a.off);
    const T* msk = static_cast<const T*>(a.msk);
    const int e = warp >> 2, q = warp & 3;
    DgWarpSmemQ* ws = reinterpret_cast<DgWarpSmemQ*>(smem + L.epi) + warp;
    const int j8 = lane & 7, rsub = lane >> 3;
    const int W1 = g.W + 1, OG = g.C / 8;
    bool ok = true;
    int cur_tile = -1;
    for (int i = e; i < nchunks; i += D_NBUF) {
      const bool ready = ok && mbar_wait(d_full(e), (i / D_NBUF) & 1, abort_flag, a.status, ST_D_EPI);
      ok = __all_sync(0xffffffffu, ready);
      if (!ok) break;
      tc_fence_after();
      if (i / nkc_cta != cur_tile) {
        // the warp's 32 pixels of this chunk's tile (the previous chunk's
        // reads of them ended at its closing __syncwarp)
        cur_tile = i / nkc_cta;
        const PixelCtx pc = pixel_ctx(g, (long long)tile_of(cur_tile) * BM + q * 32 + lane);
        ws->pix[lane] = make_int4(pc.valid ? pc.b : -1, pc.p, pc.y0, pc.x0);
      }
      KWalk kw;
      kw.start(g, kc_lo + i % nkc_cta);
      const int cbase = grp * g.Cig + kw.cc * BK;
      const int o = cbase / 8 + j8;  // the lane's offset group
      // ---- phase 1: row owner
      {
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(e * 64);
        uint32_t* srow = ws->slab[lane];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t a0[16], a1[16];
          tmem_ld16(taddr + h * 32, a0);
          tmem_ld16(taddr + h * 32 + 16, a1);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            *reinterpret_cast<uint4*>(srow + (((4 * h + k) ^ (lane & 7)) << 2)) = make_uint4(
                Vec<T>::pack(__uint_as_float(a0[8 * k]), __uint_as_float(a0[8 * k + 1])),
                Vec<T>::pack(__uint_as_float(a0[8 * k + 2]), __uint_as_float(a0[8 * k + 3])),
                Vec<T>::pack(__uint_as_float(a0[8 * k + 4]), __uint_as_float(a0[8 * k + 5])),
                Vec<T>::pack(__uint_as_float(a0[8 * k + 6]), __uint_as_float(a0[8 * k + 7])));
            *reinterpret_cast<uint4*>(srow + (((4 * h + 2 + k) ^ (lane & 7)) << 2)) = make_uint4(
                Vec<T>::pack(__uint_as_float(a1[8 * k]), __uint_as_float(a1[8 * k + 1])),
                Vec<T>::pack(__uint_as_float(a1[8 * k + 2]), __uint_as_float(a1[8 * k + 3])),
                Vec<T>::pack(__uint_as_float(a1[8 * k + 4]), __uint_as_float(a1[8 * k + 5])),
                Vec<T>::pack(__uint_as_float(a1[8 * k + 6]), __uint_as_float(a1[8 * k + 7])));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty(e));  // TMEM buffer read completely
      }
      __syncwarp();
      // ---- phase 2: lane = (pixel, offset group), 4 pixels per step.  The
      // record of step it+1 is in flight while step it is processed, and the
      // offsets and mask of step it+2 while step it+1's record is requested.
      auto load_sample = [&](int row, T& dy, T& dx, T& mr) {
        const int4 p4 = ws->pix[row];
        if (p4.x >= 0) {
          const long long ob = DCN_BOUND((long long)p4.x * g.off_bs + (long long)(o * 2 * g.T + 2 * kw.t) * g.HWo + p4.y,
                                         g.HWo + 1, g.B * g.off_bs, DBG_TC_GATHER_OFF);
          dy = off[ob];
          dx = off[ob + g.HWo];
          mr = g.use_mask ? msk[DCN_BOUND((long long)p4.x * g.msk_bs + (long long)(o * g.T + kw.t) * g.HWo + p4.y, 1,
                                          g.B * g.msk_bs, DBG_TC_GATHER_MSK)]
                          : from_f<T>(1.f);
        }
      };
      // the sample's corner-quad record (two 256-bit loads) when its floor
      // lies in [-1, H-1] x [-1, W-1] (other samples have no corner in the
      // image); returns the record index, or -1 with zeros
      auto fetch = [&](int row, T dy, T dx, uint4 (&xv)[4]) {
#pragma unroll
        for (int k = 0; k < 4; ++k) xv[k] = make_uint4(0, 0, 0, 0);
        const int4 p4 = ws->pix[row];
        if (p4.x < 0) return -1;
        const SamplePos sp = sample_pos(p4.z + kw.ti * g.dh, p4.w + kw.tj * g.dw, to_f(dy), to_f(dx));
        if (!(sp.y0 >= -1 && sp.y0 < g.H && sp.x0 >= -1 && sp.x0 < g.W)) return -1;
        const int rec = ((p4.x * (g.H + 1) + sp.y0 + 1) * W1 + sp.x0 + 1) * OG + o;
        const T* r = xq + DCN_BOUND((uint32_t)rec * 32u, 32, quad_elems(g), DBG_TC_GATHER_QUAD);
        ldg256(r, xv[0], xv[1]);
        ldg256(r + 16, xv[2], xv[3]);
        return rec;
      };
      T cdy = from_f<T>(0.f), cdx = from_f<T>(0.f), cmr = from_f<T>(1.f);  // step it
      T ndy = from_f<T>(0.f), ndx = from_f<T>(0.f), nmr = from_f<T>(1.f);  // step it+1
      load_sample(rsub, cdy, cdx, cmr);
      load_sample(rsub + 4, ndy, ndx, nmr);
      uint4 xc[4], xn[4];
      int crec = fetch(rsub, cdy, cdx, xc);
#pragma unroll 1
      for (int it = 0; it < 8; ++it) {
        const int rr = it * 4 + rsub;
        int nrec = -1;
        T n2dy = from_f<T>(0.f), n2dx = from_f<T>(0.f), n2mr = from_f<T>(1.f);
        if (it + 1 < 8) nrec = fetch(rr + 4, ndy, ndx, xn);
        if (it + 2 < 8) load_sample(rr + 8, n2dy, n2dx, n2mr);
        const int4 px = ws->pix[rr];
        const uint4 gd = *reinterpret_cast<const uint4*>(ws->slab[rr] + ((j8 ^ (rr & 7)) << 2));
        float gc[8];
        {
          const float2 g01 = Vec<T>::unpack(gd.x), g23 = Vec<T>::unpack(gd.y), g45 = Vec<T>::unpack(gd.z),
                       g67 = Vec<T>::unpack(gd.w);
          gc[0] = g01.x; gc[1] = g01.y; gc[2] = g23.x; gc[3] = g23.y;
          gc[4] = g45.x; gc[5] = g45.y; gc[6] = g67.x; gc[7] = g67.y;
        }
        int rec = -1;
        float wm[4] = {0.f, 0.f, 0.f, 0.f};
        if (px.x >= 0) {
          const long long ob = DCN_BOUND((long long)px.x * g.off_bs + (long long)(o * 2 * g.T + 2 * kw.t) * g.HWo + px.y,
                                         g.HWo + 1, g.B * g.off_bs, DBG_DG_COORD);
          const float m = g.use_mask ? mask_of(g, to_f(cmr)) : 1.f;
          const SamplePos sp = sample_pos(px.z + kw.ti * g.dh, px.w + kw.tj * g.dw, to_f(cdy), to_f(cdx));
          const Corners cs = corners_of(sp, g.H, g.W);
          rec = crec;
          float d[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 x01 = Vec<T>::unpack(xc[k].x), x23 = Vec<T>::unpack(xc[k].y),
                         x45 = Vec<T>::unpack(xc[k].z), x67 = Vec<T>::unpack(xc[k].w);
            d[k] = gc[0] * x01.x + gc[1] * x01.y + gc[2] * x23.x + gc[3] * x23.y + gc[4] * x45.x + gc[5] * x45.y +
                   gc[6] * x67.x + gc[7] * x67.y;
          }
          // coordinate derivative: corners outside the image hold zeros in the
          // record, as get_coordinate_weight's per-corner validity does
          const float gy = m * (sp.fx * (d[3] - d[1]) + (1.f - sp.fx) * (d[2] - d[0]));
          const float gx = m * (sp.fy * (d[3] - d[2]) + (1.f - sp.fy) * (d[1] - d[0]));
          const float gm = cs.w[0] * d[0] + cs.w[1] * d[1] + cs.w[2] * d[2] + cs.w[3] * d[3];
          if (a.goff_t) {
            T* go_ = static_cast<T*>(a.goff_t);
            go_[ob] = from_f<T>(gy);
            go_[ob + g.HWo] = from_f<T>(gx);
          }
          if (a.gmsk_t)  // d/dlogit = m (1 - m) d/dm for a mask stored as logits
            static_cast<T*>(a.gmsk_t)[DCN_BOUND((long long)px.x * g.msk_bs + (long long)(o * g.T + kw.t) * g.HWo + px.y,
                                                1, g.B * g.msk_bs, DBG_DG_COORD)] =
                from_f<T>(g.msk_logit ? gm * m * (1.f - m) : gm);
#pragma unroll
          for (int k = 0; k < 4; ++k) wm[k] = cs.w[k] * m;
          if (wm[0] == 0.f && wm[1] == 0.f && wm[2] == 0.f && wm[3] == 0.f) rec = -1;
        }
        if (a.gq32) {
          // the lane's record of contributions, corner-major; 16-byte piece p
          // at position p ^ (lane & 7), so that stores and loads of the rounds
          // below take the minimum 4 wavefronts
          float* st = ws->stage[lane];
          const int sw = lane & 7;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            *reinterpret_cast<float4*>(st + 4 * ((2 * k) ^ sw)) =
                make_float4(wm[k] * gc[0], wm[k] * gc[1], wm[k] * gc[2], wm[k] * gc[3]);
            *reinterpret_cast<float4*>(st + 4 * ((2 * k + 1) ^ sw)) =
                make_float4(wm[k] * gc[4], wm[k] * gc[5], wm[k] * gc[6], wm[k] * gc[7]);
          }
          ws->rec[lane] = rec;
          __syncwarp();
          // 8 rounds: lanes 8s..8s+7 add the 8 pieces of record (4j + s)
#pragma unroll 2
          for (int j = 0; j < 8; ++j) {
            const int src = 4 * j + (lane >> 3);
            const int rs = ws->rec[src];
            if (rs >= 0) {
              const float4 v = *reinterpret_cast<const float4*>(ws->stage[src] + 4 * (j8 ^ (src & 7)));
              red_v4(a.gq32 + DCN_BOUND((uint32_t)rs * 32u + 4 * j8, 4, quad_elems(g), DBG_DG_QUAD_SCATTER), v.x, v.y,
                     v.z, v.w);
            }
          }
          __syncwarp();  // the staging area is rewritten by the next step
        }
        // rotate: step it+1 becomes current
        cdy = ndy; cdx = ndx; cmr = nmr;
        ndy = n2dy; ndx = n2dx; nmr = n2mr;
#pragma unroll
        for (int k = 0; k < 4; ++k) xc[k] = xn[k];
        crec = nrec;
      }
      __syncwarp();  // the next chunk's phase 1 rewrites the slab
    }
  } else if (warp < D_EPI_WARPS && SW == 32) {
    // -------------------------------------------- epilogue, 32-channel slabs
    // Per slab of a gcol tile (one offset group):
    //  (1) row owner (lane = TMEM row = pixel): reads its 32 gcol values from
    //      TMEM into the warp's slab and, when the offset group changes,
    //      computes the sample's corners into its table row;
    //  (2) 8 lanes per pixel, 4 channels per lane, 4 pixels per instruction:
    //      corner loads and red.global.add.v4.f32 scatters cover whole lines;
    //      each lane leaves its offset/mask partial sums in the slab chunk it
    //      has just consumed, and the row owner sums its row's 8 chunks and
    //      adds the result to global memory once per (pixel, offset group,
    //      K chunk).
    const T* xh = static_cast<const T*>(a.xh);
    const T* off = static_cast<const T*>(a.off);
    const T* msk = static_cast<const T*>(a.msk);
    const int e = warp >> 2, q = warp & 3;
    DgWarpSmem32* ws = reinterpret_cast<DgWarpSmem32*>(smem + L.epi) + warp;
    const PixelCtx pc = pixel_ctx(g, (long long)tile * BM + q * 32 + lane);
    const int j8 = lane & 7, rsub = lane >> 3;
    bool ok = true;
    for (int i = e; i < nkc_cta; i += D_NBUF) {
      const bool ready = ok && mbar_wait(d_full(e), (i / D_NBUF) & 1, abort_flag, a.status, ST_D_EPI);
      ok = __all_sync(0xffffffffu, ready);
      if (!ok) break;
      tc_fence_after();
      KWalk kw;
      kw.start(g, kc_lo + i);
      const int cbase = grp * g.Cig + kw.cc * BK;
      int tab_o = -1, acc_o = -1;
      float tab_m = 0.f, acc_m = 0.f;  // mask values of the table's and the running sums' offset group
      float run_gy = 0.f, run_gx = 0.f, run_gm = 0.f;
      auto flush = [&]() {
        if (acc_o >= 0 && pc.valid) {
          const long long ob =
              DCN_BOUND((long long)pc.b * g.off_bs + (long long)(acc_o * 2 * g.T + 2 * kw.t) * g.HWo + pc.p,
                        g.HWo + 1, g.B * g.off_bs, DBG_DG_COORD);
          atomicAdd(a.goff32 + ob, run_gy);
          atomicAdd(a.goff32 + ob + g.HWo, run_gx);
          if (g.use_mask)  // d/dlogit = m (1 - m) d/dm for a mask stored as logits
            atomicAdd(a.gmsk32 + DCN_BOUND((long long)pc.b * g.msk_bs + (long long)(acc_o * g.T + kw.t) * g.HWo + pc.p,
                                           1, g.B * g.msk_bs, DBG_DG_COORD),
                      g.msk_logit ? run_gm * acc_m * (1.f - acc_m) : run_gm);
        }
        run_gy = run_gx = run_gm = 0.f;
      };
#pragma unroll 1
      for (int sl = 0; sl < 2; ++sl) {
        // ---- phase 1: row owner
        {
          uint32_t acc0[16], acc1[16];
          const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(e * 64 + sl * 32);
          tmem_ld16(taddr, acc0);
          tmem_ld16(taddr + 16, acc1);
          tmem_ld_wait();
          if (sl == 1) {  // last read of this TMEM buffer: let the MMA reuse it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(d_empty(e));
          }
          float* srow = ws->slab[lane];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            *reinterpret_cast<uint4*>(srow + ((k ^ (lane & 7)) << 2)) =
                make_uint4(acc0[4 * k], acc0[4 * k + 1], acc0[4 * k + 2], acc0[4 * k + 3]);
            *reinterpret_cast<uint4*>(srow + (((k + 4) ^ (lane & 7)) << 2)) =
                make_uint4(acc1[4 * k], acc1[4 * k + 1], acc1[4 * k + 2], acc1[4 * k + 3]);
          }
        }
        const int o = (cbase + sl * 32) / g.cpo;  // warp-uniform
        if (o != tab_o) {
          tab_o = o;
          const RawSample<T> raw = load_raw(g, off, msk, pc, o, kw.t);
          const SamplePos sp = sample_pos(pc.y0 + kw.ti * g.dh, pc.x0 + kw.tj * g.dw, to_f(raw.dy), to_f(raw.dx));
          const Corners cs = corners_of(sp, g.H, g.W);
          const CoordCorners c4 = coord_corners_of(sp, g.H, g.W);
          uint32_t cvb = 0;
          int cidx[4];
          float cw[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const bool v = pc.valid && c4.v[k];
            cvb |= (v ? 1u : 0u) << k;
            cidx[k] = v ? (int)((pc.img + c4.idx[k]) * g.C) : 0;  // element offset, B*H*W*C < 2^31
            cw[k] = pc.valid ? cs.w[k] : 0.f;
          }
          tab_m = pc.valid ? mask_of(g, to_f(raw.m)) : 0.f;
          uint32_t* trow = ws->tab[lane];
          *reinterpret_cast<uint4*>(trow) = make_uint4(cidx[0], cidx[1], cidx[2], cidx[3]);
          *reinterpret_cast<uint4*>(trow + 4) = make_uint4(__float_as_uint(cw[0]), __float_as_uint(cw[1]),
                                                           __float_as_uint(cw[2]), __float_as_uint(cw[3]));
          *reinterpret_cast<uint4*>(trow + 8) =
              make_uint4(__float_as_uint(c4.fy), __float_as_uint(c4.fx), __float_as_uint(tab_m), cvb);
        }
        if (o != acc_o) {
          flush();
          acc_o = o;
          acc_m = tab_m;
        }
        __syncwarp();
        // ---- phase 2: 8 lanes per pixel, 4 pixels per step
        const int cslab = cbase + sl * 32 + j8 * 4;
#pragma unroll 1
        for (int it = 0; it < 8; ++it) {
          const int rr = it * 4 + rsub;
          const uint32_t* tr = ws->tab[rr];
          const uint4 tb = *reinterpret_cast<const uint4*>(tr);
          const uint4 tw = *reinterpret_cast<const uint4*>(tr + 4);
          const uint4 tx = *reinterpret_cast<const uint4*>(tr + 8);
          const float4 gv = *reinterpret_cast<const float4*>(ws->slab[rr] + ((j8 ^ (rr & 7)) << 2));
          const uint32_t eo[4] = {tb.x + (uint32_t)cslab, tb.y + (uint32_t)cslab, tb.z + (uint32_t)cslab,
                                  tb.w + (uint32_t)cslab};
          const float w[4] = {__uint_as_float(tw.x), __uint_as_float(tw.y), __uint_as_float(tw.z),
                              __uint_as_float(tw.w)};
          const float fy = __uint_as_float(tx.x), fx = __uint_as_float(tx.y), m = __uint_as_float(tx.z);
          const uint32_t cv = tx.w;
          uint2 xv[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            xv[k] = (cv >> k & 1u) ? __ldg(reinterpret_cast<const uint2*>(
                                         xh + DCN_BOUND(eo[k], 4, (long long)g.B * g.H * g.W * g.C, DBG_DG_CORNER_X)))
                                   : make_uint2(0, 0);
          // d[k] = sum over the lane's 4 channels of gcol * x at corner k; the
          // mask, offset-y and offset-x partial sums are linear in them
          float d[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 lo = Vec<T>::unpack(xv[k].x), hi = Vec<T>::unpack(xv[k].y);
            d[k] = gv.x * lo.x + gv.y * lo.y + gv.z * hi.x + gv.w * hi.y;
          }
          float pgm = w[0] * d[0] + w[1] * d[1] + w[2] * d[2] + w[3] * d[3];
          float pgy = m * (fx * (d[3] - d[1]) + (1.f - fx) * (d[2] - d[0]));
          float pgx = m * (fy * (d[3] - d[2]) + (1.f - fy) * (d[1] - d[0]));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float wk = w[k] * m;
            if (wk != 0.f)
              red_v4(a.gi32 + DCN_BOUND(eo[k], 4, (long long)g.B * g.H * g.W * g.C, DBG_DG_SCATTER), wk * gv.x, wk * gv.y, wk * gv.z, wk * gv.w);
          }
          // the lane's partial sums replace the slab chunk it alone has read
          *reinterpret_cast<float4*>(ws->slab[rr] + ((j8 ^ (rr & 7)) << 2)) = make_float4(pgy, pgx, pgm, 0.f);
        }
        __syncwarp();
        // ---- row owner: sum the 8 lanes' partials of its row
        {
          const float* srow = ws->slab[lane];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float4 pv = *reinterpret_cast<const float4*>(srow + ((k ^ (lane & 7)) << 2));
            run_gy += pv.x;
            run_gx += pv.y;
            run_gm += pv.z;
          }
        }
        __syncwarp();
      }
      flush();
    }
  } else if (warp < D_EPI_WARPS) {
    // -------------------------------------------- epilogue: col2im + col2im_coord
    // Two phases per 16-channel slab of a gcol tile:
    //  (1) row owner (lane = TMEM row = pixel): reads its 16 gcol values from
    //      TMEM into the warp's slab buffer and, when the offset group changes,
    //      computes the sample's corners into the warp's table;
    //  (2) 4 lanes per pixel, 4 channels per lane: corner loads and
    //      red.global.add.v4.f32 scatters cover whole 32-byte sectors; the
    //      offset/mask partial sums are reduced across the lane pair and
    //      returned through the table to the row owner, which adds them to
    //      global memory once per (pixel, offset group, K chunk).
    const T* xh = static_cast<const T*>(a.xh);
    const T* off = static_cast<const T*>(a.off);
    const T* msk = static_cast<const T*>(a.msk);
    const int e = warp >> 2, q = warp & 3;
    DgWarpSmem* ws = reinterpret_cast<DgWarpSmem*>(smem + L.epi) + warp;
    const PixelCtx pc = pixel_ctx(g, (long long)tile * BM + q * 32 + lane);
    const int qq = lane & 3, seg = qq >> 1;
    bool ok = true;
    for (int i = e; i < nkc_cta; i += D_NBUF) {
      const bool ready = ok && mbar_wait(d_full(e), (i / D_NBUF) & 1, abort_flag, a.status, ST_D_EPI);
      ok = __all_sync(0xffffffffu, ready);
      if (!ok) break;
      tc_fence_after();
      KWalk kw;
      kw.start(g, kc_lo + i);
      const int cbase = grp * g.Cig + kw.cc * BK;
      int coord_o = -1, acc_o = -1;
      int tab_o[2] = {-1, -1};   // offset group currently in each table slot
      float run_gy = 0.f, run_gx = 0.f, run_gm = 0.f;
      // coordinates of the row owner's sample for offset group coord_o
      int cidx[4] = {0, 0, 0, 0};
      float cw[4] = {0.f, 0.f, 0.f, 0.f};
      float cfy = 0.f, cfx = 0.f, cm = 0.f;
      uint32_t cvb = 0;
      // (this variant reads stored mask values; the DCNv2 head layout, whose
      // mask holds logits, runs on the 32-channel variant only)
      auto flush = [&]() {
        if (acc_o >= 0 && pc.valid) {
          const long long ob =
              DCN_BOUND((long long)pc.b * g.off_bs + (long long)(acc_o * 2 * g.T + 2 * kw.t) * g.HWo + pc.p,
                        g.HWo + 1, g.B * g.off_bs, DBG_DG_COORD);
          atomicAdd(a.goff32 + ob, run_gy);
          atomicAdd(a.goff32 + ob + g.HWo, run_gx);
          if (g.use_mask)
            atomicAdd(a.gmsk32 + DCN_BOUND((long long)pc.b * g.msk_bs + (long long)(acc_o * g.T + kw.t) * g.HWo + pc.p,
                                           1, g.B * g.msk_bs, DBG_DG_COORD), run_gm);
        }
        run_gy = run_gx = run_gm = 0.f;
      };
#pragma unroll 1
      for (int sl = 0; sl < 4; ++sl) {
        // ---- phase 1: row owner
        uint32_t acc[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(e * 64 + sl * 16), acc);
        tmem_ld_wait();
        if (sl == 3) {  // last read of this TMEM buffer: let the MMA reuse it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(d_empty(e));
        }
        float* srow = ws->slab[lane];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          *reinterpret_cast<uint4*>(srow + slab_pos(lane, k)) =
              make_uint4(acc[4 * k], acc[4 * k + 1], acc[4 * k + 2], acc[4 * k + 3]);
        int slot_o[2];
#pragma unroll
        for (int sg = 0; sg < 2; ++sg) {
          const int o = (cbase + sl * 16 + sg * 8) / g.cpo;
          slot_o[sg] = o;
          // the table slot already holds this offset group's sample (same K chunk)
          if (sl > 0 && o == tab_o[sg]) continue;
          tab_o[sg] = o;
          if (o != coord_o) {
            coord_o = o;
            const RawSample<T> raw = load_raw(g, off, msk, pc, o, kw.t);
            const SamplePos sp =
                sample_pos(pc.y0 + kw.ti * g.dh, pc.x0 + kw.tj * g.dw, to_f(raw.dy), to_f(raw.dx));
            const Corners cs = corners_of(sp, g.H, g.W);
            const CoordCorners c4 = coord_corners_of(sp, g.H, g.W);
            cm = pc.valid ? to_f(raw.m) : 0.f;
            cfy = c4.fy;
            cfx = c4.fx;
            cvb = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const bool v = pc.valid && c4.v[k];
              cvb |= (v ? 1u : 0u) << k;
              cidx[k] = v ? (int)(pc.img + c4.idx[k]) : 0;
              cw[k] = pc.valid ? cs.w[k] : 0.f;
            }
          }
          uint32_t* trow = ws->tab[lane] + sg * 16;
          *reinterpret_cast<uint4*>(trow) = make_uint4(cidx[0], cidx[1], cidx[2], cidx[3]);
          *reinterpret_cast<uint4*>(trow + 4) = make_uint4(__float_as_uint(cw[0]), __float_as_uint(cw[1]),
                                                           __float_as_uint(cw[2]), __float_as_uint(cw[3]));
          *reinterpret_cast<uint4*>(trow + 8) = make_uint4(__float_as_uint(cfy), __float_as_uint(cfx),
                                                           __float_as_uint(cm), cvb);
        }
        __syncwarp();
        // ---- phase 2: 4 lanes per pixel
#pragma unroll 1
        for (int it = 0; it < 4; ++it) {
          const int rr = it * 8 + (lane >> 2);
          const uint32_t* tr = ws->tab[rr] + seg * 16;
          const uint4 tb = *reinterpret_cast<const uint4*>(tr);
          const uint4 tw = *reinterpret_cast<const uint4*>(tr + 4);
          const uint4 tx = *reinterpret_cast<const uint4*>(tr + 8);
          const float4 gv = *reinterpret_cast<const float4*>(ws->slab[rr] + slab_pos(rr, qq));
          const int c_abs = cbase + sl * 16 + qq * 4;
          const int ci[4] = {(int)tb.x, (int)tb.y, (int)tb.z, (int)tb.w};
          const float w[4] = {__uint_as_float(tw.x), __uint_as_float(tw.y), __uint_as_float(tw.z),
                              __uint_as_float(tw.w)};
          const float fy = __uint_as_float(tx.x), fx = __uint_as_float(tx.y), m = __uint_as_float(tx.z);
          const uint32_t cv = tx.w;
          uint2 xv[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            xv[k] = (cv >> k & 1u) ? __ldg(reinterpret_cast<const uint2*>(
                                         xh + DCN_BOUND((long long)ci[k] * g.C + c_abs, 4, (long long)g.B * g.H * g.W * g.C, DBG_DG_CORNER_X)))
                                   : make_uint2(0, 0);
          float d[4];  // per corner: sum over the lane's 4 channels of gcol * x
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 lo = Vec<T>::unpack(xv[k].x), hi = Vec<T>::unpack(xv[k].y);
            d[k] = gv.x * lo.x + gv.y * lo.y + gv.z * hi.x + gv.w * hi.y;
          }
          float pgm = w[0] * d[0] + w[1] * d[1] + w[2] * d[2] + w[3] * d[3];
          float pgy = fx * (d[3] - d[1]) + (1.f - fx) * (d[2] - d[0]);
          float pgx = fy * (d[3] - d[2]) + (1.f - fy) * (d[1] - d[0]);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float wk = w[k] * m;
            if (wk != 0.f)
              red_v4(a.gi32 + DCN_BOUND((long long)ci[k] * g.C + c_abs, 4, (long long)g.B * g.H * g.W * g.C, DBG_DG_SCATTER), wk * gv.x,
                     wk * gv.y, wk * gv.z, wk * gv.w);
          }
          pgy += __shfl_xor_sync(0xffffffffu, pgy, 1);
          pgx += __shfl_xor_sync(0xffffffffu, pgx, 1);
          pgm += __shfl_xor_sync(0xffffffffu, pgm, 1);
          if ((qq & 1) == 0) {
            uint32_t* tw2 = ws->tab[rr] + seg * 16 + 12;
            *reinterpret_cast<uint4*>(tw2) = make_uint4(__float_as_uint(m * pgy), __float_as_uint(m * pgx),
                                                        __float_as_uint(pgm), 0u);
          }
        }
        __syncwarp();
        // ---- row owner collects this slab's partial sums
#pragma unroll
        for (int sg = 0; sg < 2; ++sg) {
          if (slot_o[sg] != acc_o) {
            flush();
            acc_o = slot_o[sg];
          }
          const uint4 pa = *reinterpret_cast<const uint4*>(ws->tab[lane] + sg * 16 + 12);
          run_gy += __uint_as_float(pa.x);
          run_gx += __uint_as_float(pa.y);
          run_gm += __uint_as_float(pa.z);
        }
        __syncwarp();
      }
      flush();
    }
  } else if (warp == D_MMA_WARP) {
    // -------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = true;
      int committed = 0;
      for (int i = 0; i < nchunks && ok; ++i) {
        const int li = i % nkc_cta;
        if (li == 0) ok = mbar_wait(a_full, (i / nkc_cta) & 1, abort_flag, a.status, ST_D_MMA);  // the tile's gOt
        if (!ok) break;
        const int e = i % D_NBUF;
        ok = mbar_wait(d_empty(e), ((i / D_NBUF) & 1) ^ 1, abort_flag, a.status, ST_D_MMA);
        for (int kb = 0; kb < a.kb && ok; ++kb) {
          const int j = i * a.kb + kb, s = j % S;
          ok = mbar_wait(b_full(s), (j / S) & 1, abort_flag, a.status, ST_D_MMA);
          if (!ok) break;
          tc_fence_after();
          const uint32_t bbase = sbase + L.b + s * L.b_stage;
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const uint64_t ad = desc_kmajor_sw128(sbase + L.a + kb * A_STAGE_BYTES + k4 * 32);
            const uint64_t bd = desc_kmajor_sw128(bbase + k4 * 32);
            mma_f16(tmem + (uint32_t)(e * 64), ad, bd, a.idesc, (kb > 0 || k4 > 0) ? 1u : 0u);
          }
          mma_commit(b_empty(s));
          ++committed;
        }
        if (ok) {
          mma_commit(d_full(e));
          if (li == nkc_cta - 1) mma_commit(a_empty);  // the loader may replace the gOt tile
        }
      }
      if (!ok && committed > 0) {
        mma_commit(drain);
        mbar_wait(drain, 0, abort_flag, a.status, ST_D_DRAIN);
      }
    }
  } else {
    // -------------------------------------------- loader: gOt tile (TMA) + W^T tiles (bulk)
    if (lane == 0) {
      // K blocks of W^T in order (kc, kb): block j = kc*KB + kb, the same run for every tile
      const uint8_t* wbase = static_cast<const uint8_t*>(a.wdt) +
                             ((size_t)grp * a.nkc + kc_lo) * a.kb * L.b_stage;
      const int per_tile = nkc_cta * a.kb;
      int issued = 0, a_loads = 0;
      bool ok = true;
      for (int tl = 0; tl < ntile && ok; ++tl) {
        // the previous tile's MMAs have finished reading its gOt tile
        if (tl > 0 && !(ok = mbar_wait(a_empty, (tl - 1) & 1, abort_flag, a.status, ST_D_LOAD))) break;
        mbar_arrive_expect_tx(a_full, (uint32_t)a.kb * A_STAGE_BYTES);
        for (int cb = 0; cb < a.kb; ++cb)
          tma_load_2d(sbase + L.a + cb * A_STAGE_BYTES, &tmap_go, grp * g.Cog + cb * 64, tile_of(tl) * BM, a_full);
        ++a_loads;
        for (int jj = 0; jj < per_tile; ++jj) {
          const int j = tl * per_tile + jj, s = j % S;
          if (!(ok = mbar_wait(b_empty(s), ((j / S) & 1) ^ 1, abort_flag, a.status, ST_D_LOAD))) break;
          mbar_arrive_expect_tx(b_full(s), L.b_stage);
          bulk_g2s(sbase + L.b + s * L.b_stage, wbase + (size_t)jj * L.b_stage, L.b_stage, b_full(s));
          ++issued;
        }
      }
      // copies still in flight land before the CTA exits
      for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
        mbar_wait(b_full(i % S), (i / S) & 1, abort_flag, a.status, ST_D_LOAD);
      if (a_loads > 0) mbar_wait(a_full, (a_loads - 1) & 1, abort_flag, a.status, ST_D_LOAD);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == D_MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 64 * D_NBUF);
  }
}

// ================================================================ corner-quad sum
// gi32[b][y][x][8o..8o+7] = sum over the four roles of the fp32 corner-quad
// accumulator: corner 00 of record (y, x), 01 of (y, x-1), 10 of (y-1, x) and
// 11 of (y-1, x-1).  One thread per (image, pixel, offset group): four
// 32-byte reads (each record corner read once overall) and one 32-byte write.
__global__ void quad_sum_kernel(const float* __restrict__ gq, float* __restrict__ gi, int H, int W, int C,
                                long long n) {
  const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (t >= n) return;
  const int OG = C / 8;
  const int o = (int)(t % OG);
  const long long pix = t / OG;  // (b*H + y)*W + x
  const int x = (int)(pix % W);
  const long long by = pix / W;
  const int y = (int)(by % H);
  const int b = (int)(by / H);
  // record (y0, x0) -> index ((b*(H+1) + y0+1)*(W+1) + x0+1)*OG + o
  const long long r00 = (((long long)b * (H + 1) + y + 1) * (W + 1) + x + 1) * OG + o;
  const long long rows = (long long)(W + 1) * OG;
  const float4* p0 = reinterpret_cast<const float4*>(gq + r00 * 32);                     // corner 00 of (y, x)
  const float4* p1 = reinterpret_cast<const float4*>(gq + (r00 - OG) * 32 + 8);          // corner 01 of (y, x-1)
  const float4* p2 = reinterpret_cast<const float4*>(gq + (r00 - rows) * 32 + 16);       // corner 10 of (y-1, x)
  const float4* p3 = reinterpret_cast<const float4*>(gq + (r00 - rows - OG) * 32 + 24);  // corner 11 of (y-1, x-1)
  float4 lo = p0[0], hi = p0[1];
  const float4 a1 = p1[0], b1 = p1[1], a2 = p2[0], b2 = p2[1], a3 = p3[0], b3 = p3[1];
  lo.x += a1.x + a2.x + a3.x; lo.y += a1.y + a2.y + a3.y; lo.z += a1.z + a2.z + a3.z; lo.w += a1.w + a2.w + a3.w;
  hi.x += b1.x + b2.x + b3.x; hi.y += b1.y + b2.y + b3.y; hi.z += b1.z + b2.z + b3.z; hi.w += b1.w + b2.w + b3.w;
  float4* dst = reinterpret_cast<float4*>(gi + pix * C + o * 8);
  dst[0] = lo;
  dst[1] = hi;
}

// Reader for the NHWC -> NCHW pass that takes grad_input straight from the
// fp32 corner-quad accumulator: channels c..c+3 (one half of offset group
// c/8) of pixel (y, x) = corner 00 of record (y, x) + (corner 01 of (y, x-1)
// + corner 10 of (y-1, x) + corner 11 of (y-1, x-1)), summed in quad_sum's
// order, so the result is bitwise quad_sum's followed by the plain pass.
struct QuadSumReader {
  const float* gq;
  int H, W, C;
  __device__ __forceinline__ float4 operator()(int b, int hw, int c) const {
    const int OG = C / 8, o = c >> 3, h = (c & 7) >> 2;
    const int y = hw / W, x = hw - y * W;
    const long long r00 = (((long long)b * (H + 1) + y + 1) * (W + 1) + x + 1) * OG + o;
    const long long rows = (long long)(W + 1) * OG;
    const float4 p0 = *reinterpret_cast<const float4*>(gq + r00 * 32 + 4 * h);
    const float4 p1 = *reinterpret_cast<const float4*>(gq + (r00 - OG) * 32 + 8 + 4 * h);
    const float4 p2 = *reinterpret_cast<const float4*>(gq + (r00 - rows) * 32 + 16 + 4 * h);
    const float4 p3 = *reinterpret_cast<const float4*>(gq + (r00 - rows - OG) * 32 + 24 + 4 * h);
    return make_float4(p0.x + (p1.x + p2.x + p3.x), p0.y + (p1.y + p2.y + p3.y), p0.z + (p1.z + p2.z + p3.z),
                       p0.w + (p1.w + p2.w + p3.w));
  }
};

// ================================================================ prep / finalize
// grad_output NCHW [B][Co][HWo] -> gOt [B*HWo][Co]; gb32[co] += tile sums.
template <typename T>
__global__ void go_transpose_bias_kernel(const T* __restrict__ go, T* __restrict__ got,
                                         float* __restrict__ gb32, int Co, int HW) {
  __shared__ float tile[64][65];
  const int b = blockIdx.z, c0 = blockIdx.y * 64, hw0 = blockIdx.x * 64;
  const T* src = go + (long long)b * Co * HW;
  T* dst = got + (long long)b * HW * Co;
  for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
    const int cc = e / 64, hh = e % 64;
    const int c = c0 + cc, hw = hw0 + hh;
    tile[cc][hh] = (c < Co && hw < HW) ? to_f(src[(long long)c * HW + hw]) : 0.f;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
    const int hh = e / 64, cc = e % 64;
    const int c = c0 + cc, hw = hw0 + hh;
    if (c < Co && hw < HW) dst[(long long)hw * Co + c] = from_f<T>(tile[cc][hh]);
  }
  if (gb32 && threadIdx.x < 64 && c0 + threadIdx.x < Co) {
    float s = 0.f;
    for (int hh = 0; hh < 64; ++hh) s += tile[threadIdx.x][hh];
    atomicAdd(gb32 + c0 + threadIdx.x, s);
  }
}

// weight [Co][Cig][T] -> W^T tiles [G][NKC][KB][64 ch][64 co]: row = channel j
// of K chunk kc = (cc, t), 64 output channels per 128-byte row, chunk q
// (output channels 8q .. 8q+7 of the block) of row j stored at q ^ (j % 8);
// co >= Cog are zero.  blockIdx.x = grp * nkc + kc, blockIdx.y = kb; a thread
// gathers one 16-byte chunk and stores it whole.
template <typename T>
__global__ void weight_t_swizzle_kernel(const T* __restrict__ w, T* __restrict__ wdt, int Cog, int Cig,
                                        int T_, int nkc) {
  const int grp = blockIdx.x / nkc, kc = blockIdx.x - grp * nkc;
  const int t = kc % T_, cc = kc / T_;
  const int kb = blockIdx.y;
  T* blk = wdt + ((long long)blockIdx.x * gridDim.y + kb) * 4096;
  for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {
    const int j = i >> 3, q = i & 7;
    const int c = cc * BK + j;
    __align__(16) T buf[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int co = kb * 64 + q * 8 + k;
      buf[k] = co < Cog ? w[((long long)(grp * Cog + co) * Cig + c) * T_ + t] : from_f<T>(0.f);
    }
    *reinterpret_cast<uint4*>(blk + j * 64 + ((q ^ (j & 7)) << 3)) = *reinterpret_cast<const uint4*>(buf);
  }
}

}  // namespace

template <typename T>
void weight_t_images(const T* w, T* wdt, const Geom& g, cudaStream_t st) {
  const int nkc = (g.Cig / BK) * g.T, KB = (g.Cog + 63) / 64;
  weight_t_swizzle_kernel<T><<<dim3((unsigned)(g.G * nkc), (unsigned)KB), 256, 0, st>>>(w, wdt, g.Cog, g.Cig, g.T,
                                                                                        nkc);
}
template void weight_t_images<__half>(const __half*, __half*, const Geom&, cudaStream_t);
template void weight_t_images<__nv_bfloat16>(const __nv_bfloat16*, __nv_bfloat16*, const Geom&, cudaStream_t);

namespace {

// channels-last fp32 [B][HW][C] -> NCHW T [B][C][HW].
template <typename T>
__global__ void nhwc_f32_to_nchw_kernel(const float* __restrict__ src, T* __restrict__ dst, int C, int HW) {
  __shared__ float tile[64][65];
  const int b = blockIdx.z, c0 = blockIdx.y * 64, hw0 = blockIdx.x * 64;
  const float* s = src + (long long)b * HW * C;
  T* d = dst + (long long)b * C * HW;
  for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
    const int hh = e / 64, cc = e % 64;
    const int c = c0 + cc, hw = hw0 + hh;
    if (c < C && hw < HW) tile[cc][hh] = s[(long long)hw * C + c];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
    const int cc = e / 64, hh = e % 64;
    const int c = c0 + cc, hw = hw0 + hh;
    if (c < C && hw < HW) d[(long long)c * HW + hw] = from_f<T>(tile[cc][hh]);
  }
}

template <typename T>
__global__ void nchw_to_nhwc_bwd_kernel(const T* __restrict__ x, T* __restrict__ xh, int C, int HW) {
  __shared__ T tile[64][65];
  const int b = blockIdx.z, c0 = blockIdx.y * 64, hw0 = blockIdx.x * 64;
  const T* src = x + (long long)b * C * HW;
  T* dst = xh + (long long)b * C * HW;
  for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
    const int cc = e / 64, hh = e % 64;
    const int c = c0 + cc, hw = hw0 + hh;
    if (c < C && hw < HW) tile[cc][hh] = src[(long long)c * HW + hw];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
    const int hh = e / 64, cc = e % 64;
    const int c = c0 + cc, hw = hw0 + hh;
    if (c < C && hw < HW) dst[(long long)hw * C + c] = tile[cc][hh];
  }
}

// Up to 4 fp32 -> T conversions in one grid-stride launch.
struct ConvertJobs {
  const float* src[4];
  void* dst[4];
  long long count[4];
  int n;
};

template <typename T>
__global__ void convert_multi_kernel(const ConvertJobs jobs) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j >= jobs.n) break;
    const float* __restrict__ s = jobs.src[j];
    T* __restrict__ d = static_cast<T*>(jobs.dst[j]);
    const long long n = jobs.count[j];
    // 4 elements per step when both ends are aligned (workspace is; outputs from
    // the caching allocator are), scalar otherwise and for the tail
    const bool vec = ((reinterpret_cast<uintptr_t>(d) & 7) == 0) && ((reinterpret_cast<uintptr_t>(s) & 15) == 0);
    const long long n4 = vec ? n / 4 : 0;
    const float4* __restrict__ s4 = reinterpret_cast<const float4*>(s);
    uint2* __restrict__ d4 = reinterpret_cast<uint2*>(d);
    long long e = tid;
    for (; e + 3 * stride < n4; e += 4 * stride) {  // 4 independent loads in flight
      float4 v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = s4[e + k * stride];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        d4[e + k * stride] = make_uint2(Vec<T>::pack(v[k].x, v[k].y), Vec<T>::pack(v[k].z, v[k].w));
    }
    for (; e < n4; e += stride) {
      const float4 v = s4[e];
      d4[e] = make_uint2(Vec<T>::pack(v.x, v.y), Vec<T>::pack(v.z, v.w));
    }
    for (long long e = n4 * 4 + tid; e < n; e += stride) d[e] = from_f<T>(s[e]);
  }
}

// gW [Co][Cig][T] = sum over splits (in split order) of the partials
// [splits][Co][nkc][64] (kc in the producers' gather order t * (Cig/64) + cc),
// and gB = gb32 in T when gb is given.  One CTA per (output channel,
// 64-channel block cc): the 64 partials of each tap are contiguous, read as
// float4 and summed over the splits in registers; a padded shared-memory tile
// [t][j] turns them into the contiguous output run [j][t].  Dynamic shared
// memory: T * 65 floats.
constexpr int WR_THREADS = 128;
inline size_t wgrad_reduce_smem(int T_) { return sizeof(float) * (size_t)T_ * 65; }

template <typename T>
__global__ void __launch_bounds__(WR_THREADS)
wgrad_reduce_kernel(const float* __restrict__ gwp, T* __restrict__ gw, const float* __restrict__ gb32,
                    T* __restrict__ gb, int splits, int Co, int Cig, int T_) {
  extern __shared__ float wr_tile[];  // [T][65]
  if (gb && blockIdx.x == 0)  // the bias gradient rides along: fp32 sums -> T
    for (int i = threadIdx.x; i < Co; i += WR_THREADS) gb[i] = from_f<T>(gb32[i]);
  const int ncc = Cig / BK;
  const int co = blockIdx.x / ncc, cc = blockIdx.x - co * ncc;
  const int nkc = ncc * T_;
  const size_t split_stride4 = (size_t)Co * nkc * 16;
  const float4* src = reinterpret_cast<const float4*>(gwp + ((size_t)co * nkc + cc) * 64);
  for (int i = threadIdx.x; i < 16 * T_; i += WR_THREADS) {
    const size_t at = (size_t)(i >> 4) * ncc * 16 + (i & 15);  // tap i/16, float4 i%16
    float4 acc;
    if (splits < 16) {  // in split order
      acc = src[at];
      for (int sp = 1; sp < splits; ++sp) {
        const float4 v = src[(size_t)sp * split_stride4 + at];
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
    } else {
      // many splits (few K chunks, e.g. 64 channels): split s = 4j + u into
      // accumulator u, four loads in flight, then ((a0 + a1) + (a2 + a3))
      float4 a[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      int sp = 0;
      for (; sp + 4 <= splits; sp += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float4 v = src[(size_t)(sp + u) * split_stride4 + at];
          a[u].x += v.x; a[u].y += v.y; a[u].z += v.z; a[u].w += v.w;
        }
      }
#pragma unroll
      for (int u = 0; u < 3; ++u) {
        if (sp + u < splits) {
          const float4 v = src[(size_t)(sp + u) * split_stride4 + at];
          a[u].x += v.x; a[u].y += v.y; a[u].z += v.z; a[u].w += v.w;
        }
      }
      acc.x = (a[0].x + a[1].x) + (a[2].x + a[3].x);
      acc.y = (a[0].y + a[1].y) + (a[2].y + a[3].y);
      acc.z = (a[0].z + a[1].z) + (a[2].z + a[3].z);
      acc.w = (a[0].w + a[1].w) + (a[2].w + a[3].w);
    }
    float* row = wr_tile + (i >> 4) * 65 + (i & 15) * 4;
    row[0] = acc.x; row[1] = acc.y; row[2] = acc.z; row[3] = acc.w;
  }
  __syncthreads();
  T* dst = gw + ((size_t)co * Cig + (size_t)cc * BK) * T_;
  for (int e = threadIdx.x; e < BK * T_; e += WR_THREADS) {
    const int j = e / T_, t = e - j * T_;
    dst[e] = from_f<T>(wr_tile[t * 65 + j]);
  }
}

// gb32[co] += sum over pixels of go[p][co] for a channels-last grad_output
// [P][Co] (Co even, go 4-byte aligned).  A warp reads 64 channels (128 bytes)
// of one pixel row; 8 warps take 8 rows at a time; blockIdx.y strides the rows.
template <typename T>
__global__ void __launch_bounds__(256) bias_rows_kernel(const T* __restrict__ go, float* __restrict__ gb32,
                                                        long long P, int Co) {
  __shared__ float red[8][64];
  const int cp = threadIdx.x & 31, r0 = threadIdx.x >> 5;
  const int c = blockIdx.x * 64 + 2 * cp;
  float s0 = 0.f, s1 = 0.f;
  if (c < Co) {
    for (long long p = (long long)blockIdx.y * 8 + r0; p < P; p += (long long)gridDim.y * 8) {
      const float2 f = Vec<T>::unpack(*reinterpret_cast<const uint32_t*>(go + p * Co + c));
      s0 += f.x;
      s1 += f.y;
    }
  }
  red[r0][2 * cp] = s0;
  red[r0][2 * cp + 1] = s1;
  __syncthreads();
  const int cc = blockIdx.x * 64 + threadIdx.x;
  if (threadIdx.x < 64 && cc < Co) {
    float t = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r) t += red[r][threadIdx.x];
    atomicAdd(gb32 + cc, t);
  }
}

// ================================================================ host
// Work split of the weight-gradient GEMM: CTAs own nkg K chunks (TMEM holds
// mh * nkg * 64 fp32 columns <= 512) of one group and a contiguous range of
// pixel tiles; about one wave of CTAs (one CTA per SM), at least 4 tiles each.
struct WgradPlan {
  int mh, nkg, ncb, kgroups, splits, tiles_per_cta, n_tiles;
};
WgradPlan wgrad_plan(const Geom& g) {
  WgradPlan w;
  const int nkc = (g.Cig / BK) * g.T;
  w.n_tiles = (int)((g.P + BM - 1) / BM);
  w.mh = (g.Cog + BM - 1) / BM;
  const int nkg_max = 8 / w.mh;
  const int ngroups = (nkc + nkg_max - 1) / nkg_max;
  w.nkg = (nkc + ngroups - 1) / ngroups;
  w.ncb = (g.Cog + 63) / 64;
  w.kgroups = (nkc + w.nkg - 1) / w.nkg;
  int splits = 148 / (w.kgroups * g.G);
  if (splits > w.n_tiles / 4) splits = w.n_tiles / 4;
  if (splits < 1) splits = 1;
  w.tiles_per_cta = w.n_tiles > 0 ? (w.n_tiles + splits - 1) / splits : 1;
  w.splits = w.n_tiles > 0 ? (w.n_tiles + w.tiles_per_cta - 1) / w.tiles_per_cta : 1;
  return w;
}

// Epilogue slab width of dcn_dgrad_tc_kernel (see the kernel).
int dgrad_slab_width(const Geom& g) {
  const bool small_index = (long long)g.B * g.H * g.W * g.C < (1LL << 31);
  if (quad_ok(g)) return 8;  // corner-quad records (the forward keeps them in the training state)
  return (g.cpo % 64 == 0 && small_index) ? 64 : (g.cpo % 32 == 0 && small_index) ? 32 : 16;
}

struct BwdWs {
  size_t xh, got, wdt, xq, gi32, acc, gq32, goff32, gmsk32, gb32, acc_bytes, gwp, total;
};
BwdWs bwd_ws(const Geom& g, size_t es) {
  BwdWs L;
  const int KB = (g.Cog + 63) / 64;
  const int nkc = (g.Cig / BK) * g.T;
  const bool quad = dgrad_slab_width(g) == 8;
  size_t o = 0;
  L.xh = o;   o += ws_align(es * (size_t)g.B * g.H * g.W * g.C);
  L.got = o;  o += ws_align(es * (size_t)g.P * g.Co);
  L.wdt = o;  o += ws_align(es * (size_t)g.G * nkc * KB * 4096);
  // corner-quad epilogue: the input's corner-quad records, and grad_input as
  // the sum of the accumulator's four roles (written whole: not cleared)
  L.xq = o;   o += quad ? ws_align(es * (size_t)quad_elems(g)) : 0;  // when not kept by the forward
  L.gi32 = o; o += quad ? ws_align(4 * (size_t)g.B * g.H * g.W * g.C) : 0;
  L.acc = o;  // fp32 accumulators, contiguous so one memset clears them
  L.gq32 = o; o += quad ? ws_align(4 * (size_t)quad_elems(g)) : 0;
  if (!quad) { L.gi32 = o; o += ws_align(4 * (size_t)g.B * g.H * g.W * g.C); }
  // offset / mask gradient accumulators with the strides of the offset and
  // mask tensors; in the DCNv2 head layout one [B][3*OG*T][HWo] region holds
  // both (no larger than the two separate regions)
  // (the quad epilogue writes the offset and mask gradients directly)
  L.goff32 = o; o += quad ? 0 : ws_align(4 * (size_t)g.B * g.off_bs);
  L.gmsk32 = o; o += (quad || g.msk_logit) ? 0 : ws_align(4 * (size_t)g.B * g.msk_bs);
  L.gb32 = o;   o += ws_align(4 * (size_t)g.Co);
  L.acc_bytes = o - L.acc;
  L.gwp = o;  // written whole by the wgrad kernels: not cleared
  o += ws_align(4 * (size_t)wgrad_plan(g).splits * g.Co * g.Cig * g.T);
  L.total = o;
  return L;
}

uint32_t pow2_cols(int n) {
  uint32_t c = 32;
  while ((int)c < n) c <<= 1;
  return c;
}

template <typename T>
cudaError_t tc_backward_t(const Geom& g, const T* go, const T* x, const T* w, const T* off, const T* msk,
                          const void* saved, T* gin, T* gw, T* goff, T* gmsk, T* gb, void* workspace,
                          cudaStream_t st, dcn_params_ready_fn ready, void* user) {
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  const BwdWs L = bwd_ws(g, sizeof(T));
  char* ws = static_cast<char*>(workspace);
  const SavedLayout SV = saved_layout(g);
  // channels-last input: read in place; else the forward's copy or a new one
  T* xh = g.in_nhwc ? const_cast<T*>(x)
                    : saved ? reinterpret_cast<T*>(const_cast<char*>(static_cast<const char*>(saved)) + SV.xh)
                            : reinterpret_cast<T*>(ws + L.xh);
  const void* cols = saved ? static_cast<const char*>(saved) + SV.cols : nullptr;
  // channels-last grad_output is already the pixel-major [P][Co] operand (the
  // tensor map wants a 16-byte aligned base: otherwise it is copied once)
  const bool go_direct = g.out_nhwc && (reinterpret_cast<uintptr_t>(go) & 15) == 0;
  T* got = go_direct ? const_cast<T*>(go) : reinterpret_cast<T*>(ws + L.got);
  T* wdt = reinterpret_cast<T*>(ws + L.wdt);
  float* gi32 = reinterpret_cast<float*>(ws + L.gi32);
  float* goff32 = reinterpret_cast<float*>(ws + L.goff32);
  float* gmsk32 = g.msk_logit ? goff32 + (size_t)2 * g.OG * g.T * g.HWo : reinterpret_cast<float*>(ws + L.gmsk32);
  float* gwp = reinterpret_cast<float*>(ws + L.gwp);
  float* gb32 = reinterpret_cast<float*>(ws + L.gb32);
  int* status = nullptr;
  {
    const cudaError_t se = tc_status_ptr(&status);
    if (se != cudaSuccess) return se;
  }
  const bool need_d = gin || goff || gmsk;
  const int KB = (g.Cog + 63) / 64;
  const int nkc = (g.Cig / BK) * g.T;
  const int n_tiles = (int)((g.P + BM - 1) / BM);
  cudaError_t e;

  if ((e = cudaMemsetAsync(ws + L.acc, 0, L.acc_bytes, st)) != cudaSuccess) return e;
  if (g.out_nhwc) {
    if (!go_direct && (e = cudaMemcpyAsync(got, go, sizeof(T) * (size_t)g.P * g.Co, cudaMemcpyDeviceToDevice,
                                           st)) != cudaSuccess)
      return e;
    if (gb) {
      KernelScope ks("bias_rows", st);
      bias_rows_kernel<T><<<dim3((unsigned)((g.Co + 63) / 64), 296), 256, 0, st>>>(got, gb32, g.P, g.Co);
    }
  } else {
    KernelScope ks("go_transpose_bias", st);
    const dim3 grid = layout::tile_grid(g.Co, g.HWo, g.B);
    if (!layout::to_channels_last_vec_ok(go, got, g.Co, g.HWo))
      go_transpose_bias_kernel<T><<<grid, 256, 0, st>>>(go, got, gb ? gb32 : nullptr, g.Co, g.HWo);
    else if (gb)
      layout::to_channels_last16_kernel<T, true><<<grid, layout::LAYOUT_THREADS, 0, st>>>(go, got, gb32, g.Co, g.HWo);
    else
      layout::to_channels_last16_kernel<T, false><<<grid, layout::LAYOUT_THREADS, 0, st>>>(go, got, nullptr, g.Co, g.HWo);
  }
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (!saved && !g.in_nhwc) {  // channels-last input copy, unless the forward left one or the input is one
    KernelScope ks("nchw_to_nhwc", st);
    const dim3 grid = layout::tile_grid(g.C, (long long)g.H * g.W, g.B);
    if (layout::to_channels_last_vec_ok(x, xh, g.C, (long long)g.H * g.W))
      layout::to_channels_last16_kernel<T, false><<<grid, layout::LAYOUT_THREADS, 0, st>>>(
          x, xh, nullptr, g.C, g.H * g.W);
    else
      nchw_to_nhwc_bwd_kernel<T><<<grid, 256, 0, st>>>(x, xh, g.C, g.H * g.W);
  }
  if ((e = cudaGetLastError()) != cudaSuccess) return e;

  CUtensorMap tmap;
  if (!make_tmap_2d(&tmap, got, bf16, (uint64_t)g.P, (uint64_t)g.Co, BM, 64)) return cudaErrorInvalidValue;

  if (gw) {
    WgradArgs a;
    a.xh = xh; a.off = off; a.msk = g.use_mask ? msk : nullptr; a.gwp = gwp;
    a.status = status; a.g = g; a.nkc = nkc;
    const WgradPlan wp = wgrad_plan(g);
    a.mh = wp.mh;
    a.nkg = wp.nkg;
    a.ncb = wp.ncb;
    const int kgroups = wp.kgroups, splits = wp.splits;
    a.tiles_per_cta = wp.tiles_per_cta;
    a.n_tiles = n_tiles;
    a.b_stages = 4;
    a.a_stages = 2;
    while (wgrad_smem(a.mh, a.a_stages, a.b_stages).total + 1024 > 225 * 1024) {
      if (a.b_stages > 2) --a.b_stages;
      else if (a.a_stages > 1) --a.a_stages;
      else return cudaErrorInvalidConfiguration;
    }
    a.idesc = idesc_f16_major(BM, 64, bf16, true, true);
    a.tmem_cols = pow2_cols(a.mh * a.nkg * 64);
    const int smem = (int)wgrad_smem(a.mh, a.a_stages, a.b_stages).total + 1024;
    if (cols) {
      CUtensorMap tmap64;  // grad_output slices of 64 pixels
      if (!make_tmap_2d(&tmap64, got, bf16, (uint64_t)g.P, (uint64_t)g.Co, WC_SLICE, 64))
        return cudaErrorInvalidValue;
      WgradArgs c = a;
      c.idesc = bf16 ? 1u : 0u;  // operand type flag; the kernel builds N = 64*nk per CTA
      c.b_stages = 4;
      while (c.b_stages > 2 && wgrad_cols_smem(2 * c.mh, c.nkg, c.b_stages).total + 1024 > 225 * 1024) --c.b_stages;
      const int csmem = (int)wgrad_cols_smem(2 * c.mh, c.nkg, c.b_stages).total + 1024;
      if (csmem > 225 * 1024) return cudaErrorInvalidConfiguration;
      if ((e = cudaFuncSetAttribute(dcn_wgrad_cols_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    csmem)) != cudaSuccess)
        return e;
      KernelScope ks("dcn_wgrad_cols_tc", st);
      dcn_wgrad_cols_tc_kernel<T><<<dim3(kgroups, g.G, splits), WC_NTHREADS, csmem, st>>>(c, cols, tmap64);
    } else {
      auto wkern = g.msk_logit ? dcn_wgrad_tc_kernel<T, true> : dcn_wgrad_tc_kernel<T, false>;
      if ((e = cudaFuncSetAttribute(wkern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess)
        return e;
      KernelScope ks("dcn_wgrad_tc", st);
      wkern<<<dim3(kgroups, g.G, splits), W_NTHREADS, smem, st>>>(a, tmap);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    {
      KernelScope ks("wgrad_reduce", st);
      const size_t rsmem = wgrad_reduce_smem(g.T);
      if (rsmem > 48 * 1024 &&
          (e = cudaFuncSetAttribute(wgrad_reduce_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)rsmem)) != cudaSuccess)
        return e;
      wgrad_reduce_kernel<T><<<(unsigned)(g.Co * (g.Cig / BK)), WR_THREADS, rsmem, st>>>(
          gwp, gw, gb ? gb32 : nullptr, gb, splits, g.Co, g.Cig, g.T);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
  }
  if (gb && !gw) {  // bias gradient alone
    ConvertJobs jobs{};
    jobs.src[0] = gb32; jobs.dst[0] = gb; jobs.count[0] = g.Co; jobs.n = 1;
    KernelScope ks("f32_convert_multi", st);
    convert_multi_kernel<T><<<1, 256, 0, st>>>(jobs);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  const float* gq_fused = nullptr;  // corner-quad accumulator summed by the final NCHW pass
  if (need_d) {
    if (saved) {  // the forward built it with the training state
      wdt = reinterpret_cast<T*>(const_cast<char*>(static_cast<const char*>(saved)) + SV.wdt);
    } else {
      KernelScope ks("weight_images", st);
      if (!weight_images_launch<T>(w, nullptr, wdt, g, st)) weight_t_images(w, wdt, g, st);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    DgradArgs a;
    a.xh = xh; a.off = off; a.msk = g.use_mask ? msk : nullptr; a.wdt = wdt;
    a.gi32 = gi32; a.goff32 = goff32; a.gmsk32 = g.use_mask ? gmsk32 : nullptr;
    a.goff_t = a.gmsk_t = nullptr;
    a.status = status; a.g = g; a.nkc = nkc; a.kb = KB;
    a.b_stages = 4;
    // epilogue slab width (see the kernel); the 32-channel variant addresses
    // the input and grad_input with 32-bit element offsets
    const int sw = dgrad_slab_width(g);
    a.xq = nullptr;
    a.gq32 = nullptr;
    if (sw == 8) {  // corner-quad records of the input for the epilogue's corner reads
      T* xq;
      if (saved) {  // the forward's, kept with the training state
        xq = reinterpret_cast<T*>(const_cast<char*>(static_cast<const char*>(saved)) + SV.xq);
      } else {
        xq = reinterpret_cast<T*>(ws + L.xq);
        KernelScope ks("quad_records", st);
        quad_records_launch(xh, xq, g, st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
      }
      a.xq = xq;
      a.gq32 = gin ? reinterpret_cast<float*>(ws + L.gq32) : nullptr;
      a.gi32 = nullptr;
      a.goff_t = goff;
      a.gmsk_t = g.use_mask ? gmsk : nullptr;
      a.goff32 = a.gmsk32 = nullptr;
    }
    while (a.b_stages > 2 && dgrad_smem(KB, a.b_stages, sw).total + 1024 > 225 * 1024) --a.b_stages;
    if (dgrad_smem(KB, a.b_stages, sw).total + 1024 > 225 * 1024) return cudaErrorInvalidConfiguration;
    a.idesc = idesc_f16(BM, 64, bf16);
    const int smem = (int)dgrad_smem(KB, a.b_stages, sw).total + 1024;
    auto kern = sw == 64 ? dcn_dgrad_tc_kernel<T, 64>
              : sw == 32 ? dcn_dgrad_tc_kernel<T, 32>
              : sw == 8  ? dcn_dgrad_tc_kernel<T, 8>
                         : dcn_dgrad_tc_kernel<T, 16>;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess)
      return e;
    // split the K chunks of a tile over ksplit CTAs (>= 4 chunks each) when
    // that shortens the launch: one CTA per SM, so the launch takes
    // ceil(CTAs / 148) waves, and a CTA takes about one chunk time per chunk
    // of its busiest TMEM buffer group (the chunks go round-robin over the 4
    // buffers) plus about half of one for its prologue and last epilogue
    // (measured on the c5 layer at 8, 16 and 64 images per GPU)
    int ksplit = 1;
    long long best = -1;
    for (int k = 1; k <= 6 && nkc / k >= 4; ++k) {
      const long long waves = ((long long)n_tiles * g.G * k + 147) / 148;
      const int chunks = (nkc + k - 1) / k;
      const long long cost = waves * (2 * ((chunks + D_NBUF - 1) / D_NBUF) + 1);  // in half chunk times
      if (best < 0 || cost < best) { best = cost; ksplit = k; }
    }
    // corner-quad epilogue: 2 or 4 pixel tiles per CTA, back to back, while
    // that still leaves two waves of CTAs, so that the 4 TMEM buffers'
    // epilogue groups share a CTA's chunks evenly (9 chunks of one tile
    // would give one group 3 and the others 2)
    a.ntiles = n_tiles;
    a.tpc = 1;
    if (sw == 8 && ksplit == 1 && nkc % D_NBUF != 0)
      while (a.tpc < 4 && (long long)((n_tiles + 2 * a.tpc - 1) / (2 * a.tpc)) * g.G >= 2 * 148) a.tpc *= 2;
    {
      KernelScope ks("dcn_dgrad_tc", st);
      kern<<<dim3((n_tiles + a.tpc - 1) / a.tpc, g.G, ksplit), D_NTHREADS, smem, st>>>(a, tmap);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // grad_input = the accumulator's four roles: summed inside the final
    // NCHW pass below, or here (channels-last grad_input, unaligned pointers)
    if (a.gq32 && !g.in_nhwc && layout::from_channels_last_vec_ok(gi32, gin, g.C, (long long)g.H * g.W)) {
      gq_fused = a.gq32;
    } else if (a.gq32) {
      KernelScope ks("quad_sum", st);
      const long long n = (long long)g.B * g.H * g.W * (g.C / 8);
      quad_sum_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(a.gq32, gi32, g.H, g.W, g.C, n);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
  }
  // grad_weight and grad_bias are final once the work enqueued so far has run:
  // a caller can start their all-reduce on another stream now.  It then runs
  // alongside the final layout passes below, whose small CTAs leave room on
  // the SMs; beside the gradient GEMM kernels (one CTA per SM) the
  // collective's blocks would take SMs from them.
  if (ready) ready(user);
  // ---- finalize
  if (gin && !g.in_nhwc) {
    KernelScope ks("grad_input_to_nchw", st);
    const dim3 grid = layout::tile_grid(g.C, (long long)g.H * g.W, g.B);
    if (gq_fused)
      layout::from_channels_last_f32_16_kernel<T><<<grid, layout::LAYOUT_THREADS, 0, st>>>(
          QuadSumReader{gq_fused, g.H, g.W, g.C}, gin, g.C, g.H * g.W);
    else if (layout::from_channels_last_vec_ok(gi32, gin, g.C, (long long)g.H * g.W))
      layout::from_channels_last_f32_16_kernel<T><<<grid, layout::LAYOUT_THREADS, 0, st>>>(
          layout::NhwcF32Reader{gi32, g.C, g.H * g.W}, gin, g.C, g.H * g.W);
    else
      nhwc_f32_to_nchw_kernel<T><<<grid, 256, 0, st>>>(gi32, gin, g.C, g.H * g.W);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  {  // offset / mask (and channels-last input) gradients: fp32 -> T in one launch
     // (the quad epilogue wrote the offset and mask gradients already)
    const bool off_done = need_d && dgrad_slab_width(g) == 8;
    ConvertJobs jobs{};
    auto add = [&](const float* src, void* dst, long long n) {
      if (dst && n > 0) { jobs.src[jobs.n] = src; jobs.dst[jobs.n] = dst; jobs.count[jobs.n] = n; ++jobs.n; }
    };
    if (gin && g.in_nhwc) add(gi32, gin, (long long)g.B * g.H * g.W * g.C);  // channels-last: no transpose
    if (off_done) {
    } else if (g.msk_logit) {  // DCNv2 head layout: goff is the whole [B][3*OG*T][HWo] gradient
      add(goff32, goff, (long long)g.B * g.off_bs);
    } else {
      add(goff32, goff, (long long)g.B * g.OG * 2 * g.T * g.HWo);
      if (g.use_mask) add(gmsk32, gmsk, (long long)g.B * g.OG * g.T * g.HWo);
    }
    if (jobs.n > 0) {
      KernelScope ks("f32_convert_multi", st);
      convert_multi_kernel<T><<<148 * 16, 256, 0, st>>>(jobs);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
  }
  return cudaSuccess;
}

}  // namespace

bool tc_backward_supported(const dcn_conv_desc& d, const Geom& g) {
  // dgrad keeps the [128 px][C_out/group] grad_output tile resident next to
  // the epilogue scratch: C_out/group <= 256; corner indices are 32-bit; the
  // gW reduction stages T*65 floats in shared memory.
  return tc_forward_supported(d, g) && g.Cog <= 256 && (long long)g.B * g.H * g.W < (1LL << 31) &&
         wgrad_reduce_smem(g.T) <= 227 * 1024;
}

size_t tc_backward_workspace(const dcn_conv_desc& d, const Geom& g) {
  return bwd_ws(g, 2).total;
}

cudaError_t tc_backward(const dcn_conv_desc& d, const Geom& g, const void* grad_output, const void* input,
                        const void* weight, const void* offset, const void* mask, const void* saved,
                        void* grad_input, void* grad_weight, void* grad_offset, void* grad_mask,
                        void* grad_bias, void* workspace, cudaStream_t st, dcn_params_ready_fn ready,
                        void* user) {
  if (d.dtype == DCN_BFLOAT16) {
    using T = __nv_bfloat16;
    return tc_backward_t<T>(g, (const T*)grad_output, (const T*)input, (const T*)weight, (const T*)offset,
                            (const T*)mask, saved, (T*)grad_input, (T*)grad_weight, (T*)grad_offset,
                            (T*)grad_mask, (T*)grad_bias, workspace, st, ready, user);
  }
  using T = __half;
  return tc_backward_t<T>(g, (const T*)grad_output, (const T*)input, (const T*)weight, (const T*)offset,
                          (const T*)mask, saved, (T*)grad_input, (T*)grad_weight, (T*)grad_offset,
                          (T*)grad_mask, (T*)grad_bias, workspace, st, ready, user);
}

DCN_DEBUG_BOUNDS_TU(tc_bwd)

}  // namespace dcn
