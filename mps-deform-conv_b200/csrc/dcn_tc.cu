// dcn_tc.cu -- tensor-core (tcgen05 / TMEM) kernels for sm_100a.
//
// Forward (dcn_fwd_tc_kernel): an implicit GEMM
//     out[p][co] = sum_k A[p][k] * W[co][k] (+ bias[co])
// over M = 128 output pixels per CTA, N = C_out of one weight group, and
// K = (channel chunk of 64, tap) -- the reference's deformable_im2col
// (deform_conv2d_mps.mm:105-340) fused as the producer of the A operand and its
// at::mm / at::bmm (mm:765-782) as the tcgen05 MMA, so the column buffer never
// exists in memory.
//
// Warp roles (576 threads):
//   warps 0-15  gather producers (dcn_tc_common.cuh): gather_run_quad for
//               offset groups of 8 channels (each sample's four corners from
//               one 64-byte corner-quad record), gather_run_wide when offset
//               groups span whole 64-channel chunks (4 lanes per pixel row,
//               32 bytes of channels each, one sample per lane), else
//               gather_run (8 lanes per row, 16 bytes each, two rows per
//               lane);
//               they read the offset/mask of the (pixel, tap, offset group),
//               load the 4 bilinear corners from the channels-last input,
//               blend them with packed 16-bit FMAs and write the
//               128-byte-swizzled A rows to shared memory.  After the main
//               loop the same warps are the epilogue: TMEM -> registers ->
//               +bias -> NCHW (or channels-last) store.
//   warp 16     MMA issuer (one thread) and TMEM owner.
//   warp 17     lane 0: weight loader, one bulk copy (TMA engine) per K chunk
//               of the pre-swizzled weight image; lane 1 (training): stores
//               each full A stage to the saved column tiles with one bulk
//               copy.  No multicast.
// Every mbarrier wait is bounded (dcn_sm100.cuh): on expiry the kernel sets
// the device status word and unwinds.
#include <mutex>
#include <type_traits>

#include "dcn_layout.cuh"
#include "dcn_tc_common.cuh"

namespace dcn {

using namespace sm100;
using namespace tcc;

namespace sm100 {
// Device status word: set by a kernel whose bounded wait expired.
__device__ int g_dcn_status = 0;
}  // namespace sm100

namespace {

constexpr int NPROD_WARPS = GATHER_WARPS;
constexpr int NPROD = GATHER_THREADS;
constexpr int MMA_WARP = NPROD_WARPS;
constexpr int LOAD_WARP = NPROD_WARPS + 1;
constexpr int NTHREADS = (LOAD_WARP + 1) * 32;  // producers, MMA warp, loader warp

// status codes recorded on a wait that expired
constexpr int ST_PROD = 11, ST_MMA_A = 12, ST_MMA_B = 13, ST_LOAD = 14, ST_EPI = 15, ST_DRAIN = 16, ST_STORE = 17;

struct FwdSmem {  // offsets within the 1024-aligned dynamic shared memory
  uint32_t a, b, bar, total;
  int stages;
  uint32_t b_stage_bytes;
};

__host__ __device__ inline FwdSmem fwd_smem_layout(int Cog, int stages) {
  FwdSmem L;
  L.stages = stages;
  L.b_stage_bytes = (uint32_t)Cog * 128u;
  L.a = 0;
  L.b = L.a + stages * A_STAGE_BYTES;
  L.bar = L.b + stages * L.b_stage_bytes;
  // a_full[S], b_full[S], empty[S], acc_full, drain (8 B each) + tmem slot + abort flag
  L.total = L.bar + (3 * stages + 2) * 8 + 16;
  return L;
}

struct FwdArgs {
  const void* xh;     // input, channels-last [B][H][W][C]
  const void* off;    // offset NCHW
  const void* msk;    // mask NCHW or null
  const void* bias;   // [Co] or null
  void* out;          // [B][Co][Ho][Wo]
  const void* wsw;    // weights, pre-swizzled [G][NKC][Cog][64]
  const void* xq;     // corner-quad records (offset groups of 8 channels), or null
  void* cols;         // copy of every A tile [G][n_tiles][NKC][16 KB], or null
  int* status;
  Geom g;
  int nkc;            // K chunks per group = (Cig / 64) * T
  int stages;
  int n_mma;          // MMAs per K step along N (Cog / n_mma <= 256)
  uint32_t idesc;     // instruction descriptor for N = Cog / n_mma
  uint32_t tmem_cols;
};

// Gather producers (dcn_tc_common.cuh).
constexpr int PROD_GENERAL = 0;  // gather_run: any offset groups of a multiple of 8 channels
constexpr int PROD_WIDE = 1;     // gather_run_wide: offset groups span whole 64-channel chunks
constexpr int PROD_QUAD = 2;     // gather_run_quad: offset groups of 8 channels, corner-quad records

// LOGIT = a.g.msk_logit (mask logits of the DCNv2 head layout); PROD: the
// gather producer (above)
template <typename T, bool LOGIT, int PROD>
__global__ void __launch_bounds__(NTHREADS, 1) dcn_fwd_tc_kernel(const FwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Geom& g = a.g;
  const int S = a.stages;
  const FwdSmem L = fwd_smem_layout(g.Cog, S);
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bar_base = sbase + L.bar;
  auto a_full = [&](int s) { return bar_base + 8u * s; };
  auto b_full = [&](int s) { return bar_base + 8u * (S + s); };
  auto empty = [&](int s) { return bar_base + 8u * (2 * S + s); };
  const uint32_t acc_full = bar_base + 8u * (3 * S);
  const uint32_t drain = bar_base + 8u * (3 * S + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.bar + (3 * S + 2) * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.bar + (3 * S + 2) * 8 + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, grp = blockIdx.y;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(a_full(s), NPROD);
      mbar_init(b_full(s), 1);
      mbar_init(empty(s), a.cols ? 2 : 1);  // MMA commit (+ column-tile store done reading)
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
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

  if (warp < NPROD_WARPS) {
    // ------------------------------------------------ producers
    Ring ring{0, S, 0u};
    auto stage_of = [&](int s, uint8_t*& t, uint32_t& eb, uint32_t& fb) {
      t = smem + L.a + s * A_STAGE_BYTES;  // saved as a column tile by the store lane (training)
      eb = empty(s);
      fb = a_full(s);
    };
    bool ok;
    if (PROD == PROD_QUAD) {
      const int r0 = warp * 8 + (lane >> 3), q = lane & 7;
      const PixelCtx pc[2] = {pixel_ctx(g, (long long)tile * BM + r0), pixel_ctx(g, (long long)tile * BM + r0 + 4)};
      ok = gather_run_quad<T, LOGIT>(g, static_cast<const T*>(a.xq), off, msk, pc, r0, q, grp * g.Cig, 0, a.nkc,
                                     ring, abort_flag, a.status, ST_PROD, stage_of);
    } else if (PROD == PROD_WIDE) {
      const int r = warp * 8 + (lane >> 2);
      const PixelCtx pc = pixel_ctx(g, (long long)tile * BM + r);
      ok = gather_run_wide<T, LOGIT>(g, xh, off, msk, pc, r, lane & 3, grp * g.Cig, 0, a.nkc, ring, abort_flag,
                                     a.status, ST_PROD, stage_of);
    } else {
      const int r0 = warp * 8 + (lane >> 3), q = lane & 7;
      const PixelCtx pc[2] = {pixel_ctx(g, (long long)tile * BM + r0), pixel_ctx(g, (long long)tile * BM + r0 + 4)};
      ok = gather_run<T, LOGIT>(g, xh, off, msk, pc, r0, q, grp * g.Cig, 0, a.nkc, ring, abort_flag, a.status,
                                ST_PROD, stage_of);
    }
    // ------------------------------------------------ epilogue
    // (warp-uniform decision: tcgen05.ld is a .sync.aligned warp instruction)
    const bool acc_ready = ok && mbar_wait(acc_full, 0, abort_flag, a.status, ST_EPI);
    if (__all_sync(0xffffffffu, acc_ready)) {
      tc_fence_after();
      const int q = warp & 3, quarter = warp >> 2;
      const int row = q * 32 + lane;
      const long long opix = (long long)tile * BM + row;
      const bool ovalid = opix < g.P;
      const int ob = ovalid ? (int)(opix / g.HWo) : 0;
      const int op = ovalid ? (int)(opix - (long long)ob * g.HWo) : 0;
      T* out = static_cast<T*>(a.out);
      const T* bias = static_cast<const T*>(a.bias);
      for (int c0 = quarter * 16; c0 < g.Cog; c0 += 64) {
        uint32_t acc[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, acc);
        tmem_ld_wait();
        if (ovalid) {
          const int oc0 = grp * g.Cog + c0;
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(acc[j]) + (bias ? to_f(bias[oc0 + j]) : 0.f);
          if (g.out_nhwc) {  // channels-last output: the row's 16 channels are 32 contiguous bytes
            uint4* dst = reinterpret_cast<uint4*>(out + opix * g.Co + oc0);
            dst[0] = make_uint4(Vec<T>::pack(v[0], v[1]), Vec<T>::pack(v[2], v[3]), Vec<T>::pack(v[4], v[5]),
                                Vec<T>::pack(v[6], v[7]));
            dst[1] = make_uint4(Vec<T>::pack(v[8], v[9]), Vec<T>::pack(v[10], v[11]), Vec<T>::pack(v[12], v[13]),
                                Vec<T>::pack(v[14], v[15]));
          } else {
            T* dst = out + ((long long)ob * g.Co + oc0) * g.HWo + op;
#pragma unroll
            for (int j = 0; j < 16; ++j) dst[(long long)j * g.HWo] = from_f<T>(v[j]);
          }
        }
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const int nsub = g.Cog / a.n_mma;
      bool ok = true;
      int issued = 0;
      for (int i = 0; i < a.nkc && ok; ++i) {
        const int s = i % S;
        const uint32_t parity = (i / S) & 1;
        ok = mbar_wait(a_full(s), parity, abort_flag, a.status, ST_MMA_A) &&
             mbar_wait(b_full(s), parity, abort_flag, a.status, ST_MMA_B);
        if (!ok) break;
        tc_fence_after();
        const uint32_t as = sbase + L.a + s * A_STAGE_BYTES;
        const uint32_t bs = sbase + L.b + s * L.b_stage_bytes;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t ad = desc_kmajor_sw128(as + k * 32);
          for (int n = 0; n < a.n_mma; ++n) {
            const uint64_t bd = desc_kmajor_sw128(bs + n * nsub * 128 + k * 32);
            mma_f16(tmem + (uint32_t)(n * nsub), ad, bd, a.idesc, (i > 0 || k > 0) ? 1u : 0u);
          }
        }
        mma_commit(empty(s));
        ++issued;
      }
      if (ok) {
        mma_commit(acc_full);
      } else if (issued > 0) {
        // let the MMAs already issued finish before TMEM is released
        mma_commit(drain);
        mbar_wait(drain, 0, abort_flag, a.status, ST_DRAIN);
      }
    }
  } else {
    // ------------------------------------------------ weight loader
    if (lane == 0) {
      const uint8_t* wbase = static_cast<const uint8_t*>(a.wsw) +
                             (size_t)grp * a.nkc * L.b_stage_bytes;
      int issued = 0;
      for (int i = 0; i < a.nkc; ++i) {
        const int s = i % S;
        const uint32_t parity = ((i / S) & 1) ^ 1;
        if (!mbar_wait(empty(s), parity, abort_flag, a.status, ST_LOAD)) break;
        mbar_arrive_expect_tx(b_full(s), L.b_stage_bytes);
        bulk_g2s(sbase + L.b + s * L.b_stage_bytes, wbase + (size_t)i * L.b_stage_bytes,
                 L.b_stage_bytes, b_full(s));
        ++issued;
      }
      // copies still in flight must land before the CTA exits
      for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
        mbar_wait(b_full(i % S), (i / S) & 1, abort_flag, a.status, ST_LOAD);
    } else if (lane == 1 && a.cols) {
      // ---------------------------------------------- column-tile store (training)
      // Each full A stage is already the saved tile's image: one bulk copy
      // per chunk to `cols`, and the stage counts as empty once the copy has
      // read it (second arrival on `empty`, next to the MMA's commit).
      uint8_t* gbase = static_cast<uint8_t*>(a.cols) + ((size_t)grp * gridDim.x + tile) * a.nkc * (size_t)A_STAGE_BYTES;
      for (int i = 0; i < a.nkc; ++i) {
        const int s = i % S;
        if (!mbar_wait(a_full(s), (i / S) & 1, abort_flag, a.status, ST_STORE)) break;
        bulk_s2g(gbase + (size_t)i * A_STAGE_BYTES, sbase + L.a + s * A_STAGE_BYTES, A_STAGE_BYTES);
        bulk_commit();
        bulk_wait_read_all();
        mbar_arrive(empty(s));
      }
      bulk_wait_all();  // the tiles are in global memory before the CTA exits
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, a.tmem_cols);
  }
}

// ---------------------------------------------------------------- repacks
// input NCHW -> channels-last [B][H][W][C], 64x64 tiles through shared memory.
template <typename T>
__global__ void nchw_to_nhwc_kernel(const T* __restrict__ x, T* __restrict__ xh, int C, int HW) {
  __shared__ T tile[64][65];
  const int b = blockIdx.z;
  const int c0 = blockIdx.y * 64, hw0 = blockIdx.x * 64;
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

// weight [Co][Cig][T] -> [G][NKC][Cog][64] in the producers' gather order,
// K chunk kc = t * (Cig/64) + cc (channel chunk fastest), rows 128-byte
// swizzled (chunk q of row co at q ^ (co % 8)).
// blockIdx.x = grp * nkc + kc; a thread gathers the 8 channels of one 16-byte
// chunk and stores it whole.
template <typename T>
__global__ void weight_swizzle_kernel(const T* __restrict__ w, T* __restrict__ wsw, int Cog, int Cig,
                                      int T_, int nkc) {
  const int grp = blockIdx.x / nkc, kc = blockIdx.x - grp * nkc;
  const int ncc = Cig / BK;
  const int t = kc / ncc, cc = kc - t * ncc;
  const int i = blockIdx.y * blockDim.x + threadIdx.x;  // (co, chunk q)
  if (i >= Cog * 8) return;
  const int co = i >> 3, q = i & 7;
  const T* src = w + ((long long)(grp * Cog + co) * Cig + cc * BK + q * 8) * T_ + t;
  __align__(16) T buf[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) buf[k] = src[(long long)k * T_];
  T* dst = wsw + (long long)blockIdx.x * Cog * BK + co * BK + ((q ^ (co & 7)) << 3);
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(buf);
}

// Pipeline depth: as many stages (<= 4) as fit one CTA per SM (the kernel's
// register use keeps it at one CTA per SM).
int pick_stages(int Cog) {
  const int stage = A_STAGE_BYTES + Cog * 128;
  int s = (225 * 1024 - 2048) / stage;
  return s > 4 ? 4 : s;
}

uint32_t tmem_cols_for(int n) {
  uint32_t c = 32;
  while ((int)c < n) c <<= 1;
  return c;
}

}  // namespace

// ---------------------------------------------------------------- host side
bool tc_forward_supported(const dcn_conv_desc& d, const Geom& g) {
  if (d.dtype != DCN_BFLOAT16 && d.dtype != DCN_FLOAT16) return false;
  if (g.Cig % BK != 0) return false;                 // K chunks of 64 channels inside one group
  if (g.cpo % 8 != 0) return false;                  // 16-byte vectors inside one offset group
  if (g.Cog % 32 != 0 || g.Cog > 512) return false;  // N per MMA: Cog or Cog/2, multiple of 16
  if (pick_stages(g.Cog) < 2) return false;
  // the gather addresses the input and offset / mask tensors with 32-bit element offsets
  if ((long long)g.B * g.H * g.W * g.C >= (1LL << 31) || (long long)g.B * g.off_bs >= (1LL << 31) ||
      (long long)g.B * g.msk_bs >= (1LL << 31))
    return false;
  return true;
}

// Offset groups of 8 channels gather from corner-quad records (32-bit
// element offsets).
static bool use_quad(const Geom& g) { return quad_ok(g); }

struct FwdWs {
  size_t xh, wsw, xq, total;
};
static FwdWs fwd_ws(const Geom& g, size_t es) {
  FwdWs L;
  L.xh = 0;
  L.wsw = ws_align(es * (size_t)g.B * g.C * g.H * g.W);
  L.xq = L.wsw + ws_align(es * (size_t)g.Co * g.Cig * g.T);
  L.total = L.xq + (use_quad(g) ? ws_align(es * (size_t)quad_elems(g)) : 0);
  return L;
}

size_t tc_forward_workspace(const dcn_conv_desc& d, const Geom& g) {
  return fwd_ws(g, 2).total;
}

SavedLayout saved_layout(const Geom& g) {
  SavedLayout L;
  const size_t n_tiles = (size_t)((g.P + BM - 1) / BM);
  const size_t nkc = (size_t)(g.Cig / BK) * g.T;
  L.xh = 0;
  L.cols = ws_align(2 * (size_t)g.B * g.H * g.W * g.C);
  L.xq = L.cols + ws_align((size_t)g.G * n_tiles * nkc * A_STAGE_BYTES);
  L.wdt = L.xq + (use_quad(g) ? ws_align(2 * (size_t)quad_elems(g)) : 0);
  L.total = L.wdt + ws_align(2 * (size_t)g.G * nkc * ((g.Cog + 63) / 64) * 4096);
  return L;
}

// Current CUDA context of the calling thread (null when none is current or
// the driver entry point is missing).
static void* current_context() {
  typedef int (*CtxGetCurrentFn)(void**);  // CUresult cuCtxGetCurrent(CUcontext*)
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(f);
  });
  void* c = nullptr;
  if (fn && fn(&c) != 0) c = nullptr;
  return c;
}

cudaError_t device_symbol_address(DeviceSymbolCache& cache, const void* symbol, void** out) {
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= DeviceSymbolCache::kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(mu);
  void* ctx = current_context();
  if (cache.ptr[dev] && ctx && ctx == cache.ctx[dev]) {
    *out = cache.ptr[dev];
    return cudaSuccess;
  }
  void* p = nullptr;
  if ((e = cudaGetSymbolAddress(&p, symbol)) != cudaSuccess) return e;
  cache.ptr[dev] = p;
  cache.ctx[dev] = current_context();  // the lookup made the device's context current
  *out = p;
  return cudaSuccess;
}

cudaError_t tc_status_ptr(int** out) {
  static DeviceSymbolCache cache;  // one address per device
  void* p = nullptr;
  cudaError_t e = device_symbol_address(cache, &sm100::g_dcn_status, &p);
  *out = static_cast<int*>(p);
  return e;
}

bool make_tmap_2d(CUtensorMap* map, const void* base, bool bf16, uint64_t rows, uint64_t cols,
                  uint32_t box_rows, uint32_t box_cols) {
  typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                               const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                               CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                               CUtensorMapFloatOOBfill);
  static EncodeFn encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return false;
    encode = reinterpret_cast<EncodeFn>(fn);
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Forward weight image wsw of `w` (weight_images_kernel, or the per-image
// kernel when its staging does not fit).
template <typename T>
static void forward_weight_image(const T* w, T* wsw, T* wdt, const Geom& g, cudaStream_t st) {
  KernelScope ks("weight_images", st);
  if (!weight_images_launch<T>(w, wsw, wdt, g, st)) {
    const int nkc = (g.Cig / BK) * g.T;
    const dim3 grid((unsigned)(g.G * nkc), (unsigned)((g.Cog * 8 + 255) / 256));
    weight_swizzle_kernel<T><<<grid, 256, 0, st>>>(w, wsw, g.Cog, g.Cig, g.T, nkc);
    if (wdt) weight_t_images(w, wdt, g, st);
  }
}

// w_is_image: `w` is already the forward weight image (tc_weight_image), and
// nothing is saved.
template <typename T>
static cudaError_t tc_forward_t(const Geom& g, const T* x, const T* w, bool w_is_image, const T* off,
                                const T* msk, const T* bias, T* out, void* workspace, void* saved,
                                cudaStream_t st) {
  const FwdWs L = fwd_ws(g, sizeof(T));
  const SavedLayout SV = saved_layout(g);
  // channels-last input: the gather reads it directly; else a channels-last copy
  T* xh = g.in_nhwc ? const_cast<T*>(x)
                    : reinterpret_cast<T*>(saved ? static_cast<char*>(saved) + SV.xh
                                                 : static_cast<char*>(workspace) + L.xh);
  T* wsw = w_is_image ? const_cast<T*>(w) : reinterpret_cast<T*>(static_cast<char*>(workspace) + L.wsw);
  cudaError_t e;
  if (!g.in_nhwc) {
    KernelScope ks("nchw_to_nhwc", st);
    const dim3 grid = layout::tile_grid(g.C, (long long)g.H * g.W, g.B);
    if (layout::to_channels_last_vec_ok(x, xh, g.C, (long long)g.H * g.W))
      layout::to_channels_last16_kernel<T, false><<<grid, layout::LAYOUT_THREADS, 0, st>>>(
          x, xh, nullptr, g.C, g.H * g.W);
    else
      nchw_to_nhwc_kernel<T><<<grid, 256, 0, st>>>(x, xh, g.C, g.H * g.W);
  }
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (!w_is_image) {
    // both weight images in one pass; training keeps dgrad's with the saved state
    T* wdt = saved ? reinterpret_cast<T*>(static_cast<char*>(saved) + SV.wdt) : nullptr;
    forward_weight_image(w, wsw, wdt, g, st);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }

  const bool quad = use_quad(g) && (reinterpret_cast<uintptr_t>(xh) & 15) == 0;
  // training: the records stay with the saved state for the backward's corner reads
  T* xq = reinterpret_cast<T*>(saved ? static_cast<char*>(saved) + SV.xq : static_cast<char*>(workspace) + L.xq);
  if (quad) {
    KernelScope ks("quad_records", st);
    quad_records_launch(xh, xq, g, st);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }

  FwdArgs a;
  a.xh = xh; a.off = off; a.msk = g.use_mask ? msk : nullptr; a.bias = bias; a.out = out; a.wsw = wsw;
  a.xq = quad ? xq : nullptr;
  a.cols = saved ? static_cast<char*>(saved) + SV.cols : nullptr;
  if ((e = tc_status_ptr(&a.status)) != cudaSuccess) return e;
  a.g = g;
  a.nkc = (g.Cig / BK) * g.T;
  a.stages = pick_stages(g.Cog);
  a.n_mma = (g.Cog + 255) / 256;
  a.idesc = idesc_f16(BM, g.Cog / a.n_mma, std::is_same<T, __nv_bfloat16>::value);
  a.tmem_cols = tmem_cols_for(g.Cog);
  const FwdSmem SL = fwd_smem_layout(g.Cog, a.stages);
  const int smem = (int)SL.total + 1024;
  // producer: corner-quad records for offset groups of 8 channels, one
  // sample per lane when offset groups span whole 64-channel chunks, else
  // the general two-rows-per-lane gather
  const int prod = quad ? PROD_QUAD : g.cpo % BK == 0 ? PROD_WIDE : PROD_GENERAL;
  auto pick = [&](auto k0, auto k1, auto k2) { return prod == PROD_QUAD ? k2 : prod == PROD_WIDE ? k1 : k0; };
  auto kern = g.msk_logit ? pick(dcn_fwd_tc_kernel<T, true, PROD_GENERAL>, dcn_fwd_tc_kernel<T, true, PROD_WIDE>,
                                 dcn_fwd_tc_kernel<T, true, PROD_QUAD>)
                          : pick(dcn_fwd_tc_kernel<T, false, PROD_GENERAL>, dcn_fwd_tc_kernel<T, false, PROD_WIDE>,
                                 dcn_fwd_tc_kernel<T, false, PROD_QUAD>);
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess)
    return e;
  dim3 grid((unsigned)((g.P + BM - 1) / BM), (unsigned)g.G);
  {
    KernelScope ks("dcn_fwd_tc", st);
    kern<<<grid, NTHREADS, smem, st>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t tc_forward(const dcn_conv_desc& d, const Geom& g, const void* input, const void* weight,
                       bool weight_is_image, const void* offset, const void* mask, const void* bias,
                       void* output, void* workspace, void* saved, cudaStream_t st) {
  if (d.dtype == DCN_BFLOAT16)
    return tc_forward_t<__nv_bfloat16>(g, (const __nv_bfloat16*)input, (const __nv_bfloat16*)weight,
                                       weight_is_image, (const __nv_bfloat16*)offset, (const __nv_bfloat16*)mask,
                                       (const __nv_bfloat16*)bias, (__nv_bfloat16*)output, workspace, saved, st);
  return tc_forward_t<__half>(g, (const __half*)input, (const __half*)weight, weight_is_image,
                              (const __half*)offset, (const __half*)mask, (const __half*)bias, (__half*)output,
                              workspace, saved, st);
}

cudaError_t tc_weight_image(const dcn_conv_desc& d, const Geom& g, const void* weight, void* image,
                            cudaStream_t st) {
  if (d.dtype == DCN_BFLOAT16)
    forward_weight_image((const __nv_bfloat16*)weight, (__nv_bfloat16*)image, (__nv_bfloat16*)nullptr, g, st);
  else
    forward_weight_image((const __half*)weight, (__half*)image, (__half*)nullptr, g, st);
  return cudaGetLastError();
}


cudaError_t tc_read_and_clear_status(int* out, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, sm100::g_dcn_status, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return e;
  const int zero = 0;
  return cudaMemcpyToSymbol(sm100::g_dcn_status, &zero, sizeof(int));
}

DCN_DEBUG_BOUNDS_TU(tc)

}  // namespace dcn
