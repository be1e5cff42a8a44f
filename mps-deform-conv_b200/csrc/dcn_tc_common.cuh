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

// 32 bytes of read-only global memory in one 256-bit load (sm_100);
// p 32-byte aligned.
__device__ __forceinline__ void ldg256(const void* p, uint4& lo, uint4& hi) {
  asm("ld.global.nc.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(lo.x), "=r"(lo.y), "=r"(lo.z), "=r"(lo.w), "=r"(hi.x), "=r"(hi.y), "=r"(hi.z), "=r"(hi.w)
      : "l"(p));
}

// ---------------------------------------------------------------- gather
// A producer warp owns 8 consecutive pixel rows (8*warp .. 8*warp+7) of a
// 128-row operand tile [pixels][64 channels] (lane mapping: gather_run).
// The offset/mask values of the next K chunk are loaded while the current
// chunk's corners are in flight.
constexpr int GATHER_WARPS = 16;
constexpr int GATHER_THREADS = GATHER_WARPS * 32;

struct PixelCtx {
  bool valid;
  int b, p;
  int y0, x0;       // oy*stride - pad, ox*stride - pad
  long long img;    // b*H*W (pixel index of the image's first pixel)
};

__device__ __forceinline__ PixelCtx pixel_ctx(const Geom& g, long long pix) {
  PixelCtx c;
  c.valid = pix < g.P;
  c.b = c.valid ? (int)(pix / g.HWo) : 0;
  c.p = c.valid ? (int)(pix - (long long)c.b * g.HWo) : 0;
  const int oy = c.p / g.Wo, ox = c.p - oy * g.Wo;
  c.y0 = oy * g.sh - g.ph;
  c.x0 = ox * g.sw - g.pw;
  c.img = (long long)c.b * g.H * g.W;
  return c;
}

// Offset and mask values of one (pixel, offset group, tap), kept in the
// storage type so that the loads stay in flight until the values are used
// (the mask as stored: a logit in the DCNv2 head layout, see mask_of).
template <typename T>
struct RawSample {
  T dy, dx, m;
};

template <typename T>
__device__ __forceinline__ RawSample<T> load_raw(const Geom& g, const T* __restrict__ off,
                                                 const T* __restrict__ msk, const PixelCtx& pc, int o,
                                                 int t) {
  RawSample<T> r;
  const long long ob = DCN_BOUND((long long)pc.b * g.off_bs + (long long)(o * 2 * g.T + 2 * t) * g.HWo + pc.p,
                                 g.HWo + 1, g.B * g.off_bs, DBG_TC_GATHER_OFF);
  r.dy = off[ob];
  r.dx = off[ob + g.HWo];
  r.m = msk ? msk[DCN_BOUND((long long)pc.b * g.msk_bs + (long long)(o * g.T + t) * g.HWo + pc.p, 1,
                            g.B * g.msk_bs, DBG_TC_GATHER_MSK)]
            : from_f<T>(1.f);
  return r;
}

// sum_k w[k] * v[k] over 8 channels as a packed 16-bit FMA chain (two
// channels per instruction, no unpacking).  The chain rounds after each of
// its 4 steps; on bf16 data the resulting A-operand error stays within ~3e-3
// normwise of an fp32 blend, below the 1e-2 parity tolerance.
template <typename T> struct Packed;
template <> struct Packed<__nv_bfloat16> {
  using P2 = __nv_bfloat162;
  static __device__ __forceinline__ P2 splat(float w) { return __float2bfloat162_rn(w); }
};
template <> struct Packed<__half> {
  using P2 = __half2;
  static __device__ __forceinline__ P2 splat(float w) { return __float2half2_rn(w); }
};

template <typename T>
__device__ __forceinline__ uint4 blend8(const uint4 (&v)[4], const float (&w)[4]) {
  using P2 = typename Packed<T>::P2;
  const P2 w0 = Packed<T>::splat(w[0]), w1 = Packed<T>::splat(w[1]);
  const P2 w2 = Packed<T>::splat(w[2]), w3 = Packed<T>::splat(w[3]);
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t a0 = (&v[0].x)[e], a1 = (&v[1].x)[e], a2 = (&v[2].x)[e], a3 = (&v[3].x)[e];
    P2 acc = __hmul2(w0, *reinterpret_cast<const P2*>(&a0));
    acc = __hfma2(w1, *reinterpret_cast<const P2*>(&a1), acc);
    acc = __hfma2(w2, *reinterpret_cast<const P2*>(&a2), acc);
    acc = __hfma2(w3, *reinterpret_cast<const P2*>(&a3), acc);
    o[e] = *reinterpret_cast<uint32_t*>(&acc);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// K-chunk walker: kc = cc*T + t with t = ti*kw + tj, advanced without division.
struct KWalk {
  int t, cc, ti, tj;
  __device__ __forceinline__ void start(const Geom& g, int kc) {
    cc = kc / g.T;
    t = kc - cc * g.T;
    ti = t / g.kw;
    tj = t - ti * g.kw;
  }
  __device__ __forceinline__ void next(const Geom& g) {
    ++t;
    if (++tj == g.kw) { tj = 0; ++ti; }
    if (t == g.T) { t = 0; ti = 0; tj = 0; ++cc; }
  }
};

// Gather order of the producers' K chunks: kc = t * ncc + cc (ncc = Cig / 64
// channel chunks per tap), channel chunk fastest, so that consecutive chunks
// of one tap whose channels lie in the same offset group share the sampling
// point.  The forward's A/B operand tiles, its saved column tiles and the
// weight-gradient partials all follow this order (dgrad uses its own, KWalk).
struct GatherWalk {
  int t, cc, ti, tj;
  __device__ __forceinline__ void start(const Geom& g, int kc, int ncc) {
    t = kc / ncc;
    cc = kc - t * ncc;
    ti = t / g.kw;
    tj = t - ti * g.kw;
  }
  __device__ __forceinline__ void next(const Geom& g, int ncc) {
    if (++cc == ncc) {
      cc = 0;
      ++t;
      if (++tj == g.kw) { tj = 0; ++ti; }
    }
  }
};

// Offset group of a lane's 8-channel vector, tracked as the channel chunk
// advances by 64 channels (no division per chunk): og = c / cpo, rem = c % cpo.
struct OgTrack {
  int og, rem;
  __device__ __forceinline__ void set(int c, int cpo) {
    og = c / cpo;
    rem = c - og * cpo;
  }
  __device__ __forceinline__ void step64(int cpo) {
    rem += BK;
    while (rem >= cpo) { rem -= cpo; ++og; }
  }
};

// Ring position of a pipeline of S stages: stage s and the phase bit of its
// barriers (flips each time the ring wraps).
struct Ring {
  int s, S;
  uint32_t ph;
  __device__ __forceinline__ void next() {
    if (++s == S) { s = 0; ph ^= 1u; }
  }
};

// Corners of one sample as 32-bit element offsets of channel 0 within the
// image's channels-last plane (H*W*C < 2^31) and weights including the mask.
struct CornerSet32 {
  int off[4];
  float w[4];
};

// LOGIT: the mask holds logits (DCNv2 head layout, Geom::msk_logit); a
// compile-time choice, so the plain layout's producer carries no select.
template <typename T, bool LOGIT>
__device__ __forceinline__ CornerSet32 corner_set32(const Geom& g, const PixelCtx& pc, const RawSample<T>& r,
                                                    int ti, int tj) {
  CornerSet32 cs;
  const SamplePos sp = sample_pos(pc.y0 + ti * g.dh, pc.x0 + tj * g.dw, to_f(r.dy), to_f(r.dx));
  const Corners c = corners_of(sp, g.H, g.W);
  const float mv = to_f(r.m);
  const float m = pc.valid ? (LOGIT ? 1.f / (1.f + __expf(-mv)) : mv) : 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    cs.w[k] = c.w[k] * m;
    cs.off[k] = c.idx[k] * g.C;
  }
  return cs;
}

// One producer thread's share of a run of K chunks for one pixel tile (gather
// order above).  A producer warp owns 8 rows of the 128-row operand tile;
// lane l works on rows r0 = 8*warp + l/8 and r0 + 4 and on the 16-byte
// channel chunk q = l%8 of the K chunk, so one load instruction covers 4
// pixels x 128 contiguous bytes of a corner (whole cache lines).  Per chunk
// it waits for its stage to be free, gathers 16 bytes of the 4 corners of
// both pixels, blends, and writes its chunk of both rows into the swizzled
// tile.  The sampling points and the offset / mask loads are reused while
// consecutive chunks share the tap and the offset group.  `ring` is the
// stage ring position (advanced once per chunk);
// `stage_of(s, tile, empty_bar, full_bar)` gives the shared-memory tile of
// stage s and its barriers.  Returns false if a wait expired.  The input (B*H*W*C) and
// offset / mask tensors (B * per-sample stride) hold fewer than 2^31 elements.
template <typename T, bool LOGIT, class StageFn>
__device__ __forceinline__ bool gather_run(const Geom& g, const T* __restrict__ xh,
                                           const T* __restrict__ off, const T* __restrict__ msk,
                                           const PixelCtx (&pc)[2], int r0, int q, int cbase_grp, int kc0,
                                           int nk, Ring& ring, volatile int* abort_flag, int* status,
                                           int code, StageFn&& stage_of) {
  const int ncc = g.Cig / BK;
  // 32-bit element offsets of each pixel's image in the input and of its
  // (image, pixel) in the offset / mask tensors (whole tensors < 2^31 elements)
  int xo[2], oo[2], mo[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    xo[h] = (int)pc[h].img * g.C;
    oo[h] = pc[h].b * (int)g.off_bs + pc[h].p;
    mo[h] = pc[h].b * (int)g.msk_bs + pc[h].p;
  }
  auto load = [&](int h, int o, int t) {
    RawSample<T> rs;
    const int ob = DCN_BOUND(oo[h] + (o * 2 * g.T + 2 * t) * g.HWo, g.HWo + 1, g.B * g.off_bs, DBG_TC_GATHER_OFF);
    rs.dy = off[ob];
    rs.dx = off[ob + g.HWo];
    rs.m = msk ? msk[DCN_BOUND(mo[h] + (o * g.T + t) * g.HWo, 1, g.B * g.msk_bs, DBG_TC_GATHER_MSK)]
               : from_f<T>(1.f);
    return rs;
  };
  GatherWalk kw;
  kw.start(g, kc0, ncc);
  // offset group of the lane's 8-channel vector at chunk cc = 0 and now
  OgTrack a0, a;
  a0.set(cbase_grp + q * 8, g.cpo);
  a.set(cbase_grp + kw.cc * BK + q * 8, g.cpo);
  RawSample<T> raw[2] = {load(0, a.og, kw.t), load(1, a.og, kw.t)};
  CornerSet32 cs[2];
  bool reuse = false;  // cs already holds this chunk's corners
  const int r1 = r0 + 4;
  const int o0 = r0 * 128 + ((q ^ (r0 & 7)) << 4), o1 = r1 * 128 + ((q ^ (r1 & 7)) << 4);
  for (int i = 0; i < nk; ++i) {
    if (!reuse) {
      cs[0] = corner_set32<T, LOGIT>(g, pc[0], raw[0], kw.ti, kw.tj);
      cs[1] = corner_set32<T, LOGIT>(g, pc[1], raw[1], kw.ti, kw.tj);
    }
    const int c0 = cbase_grp + kw.cc * BK + q * 8;
    uint4 v[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int k = 0; k < 4; ++k)
        v[h][k] = (cs[h].w[k] != 0.f)
                      ? __ldg(reinterpret_cast<const uint4*>(
                            xh + DCN_BOUND((uint32_t)(xo[h] + cs[h].off[k] + c0), 8,
                                           (long long)g.B * g.H * g.W * g.C, DBG_TC_GATHER_X)))
                      : make_uint4(0, 0, 0, 0);
    // the next chunk: same sampling points, or prefetch their offsets and masks
    if (i + 1 < nk) {
      const int pt = kw.t, pa = a.og;
      kw.next(g, ncc);
      if (kw.cc == 0) a = a0;
      else a.step64(g.cpo);
      reuse = kw.t == pt && a.og == pa;
      if (!reuse) {
        raw[0] = load(0, a.og, kw.t);
        raw[1] = load(1, a.og, kw.t);
      }
    }
    uint8_t* tile;
    uint32_t empty_bar, full_bar;
    stage_of(ring.s, tile, empty_bar, full_bar);
    const uint4 b0 = blend8<T>(v[0], cs[0].w), b1 = blend8<T>(v[1], cs[1].w);
    if (!mbar_wait(empty_bar, ring.ph ^ 1u, abort_flag, status, code)) return false;
    *reinterpret_cast<uint4*>(tile + o0) = b0;
    *reinterpret_cast<uint4*>(tile + o1) = b1;
    fence_async_shared();
    mbar_arrive(full_bar);
    ring.next();
  }
  return true;
}

// Producer for problems whose offset groups span whole 64-channel chunks
// (channels per offset group a multiple of 64), where every row of a K chunk
// has one sample.  Lane l of a producer warp works on row r = 8*warp + l/4
// and on channels [8q, 8q+8) and [32+8q, 32+8q+8) of the chunk (q = l%4), so
// one load instruction covers 8 rows x 64 contiguous bytes of a corner and
// each lane computes one sampling point per new (tap, offset group) -- half
// the sample arithmetic of gather_run's two pixels per lane, for the same
// 8 corner loads in flight per lane.  The offsets and mask of the next new
// sample are loaded one chunk ahead.  Same stage protocol and return value as
// gather_run; the A tiles are bitwise those of gather_run.  (Issuing chunk
// i+1's corner loads before chunk i's blend needs about 140 registers per
// thread, above the 96 that 18 warps per CTA leave.)
template <typename T, bool LOGIT, class StageFn>
__device__ __forceinline__ bool gather_run_wide(const Geom& g, const T* __restrict__ xh,
                                                const T* __restrict__ off, const T* __restrict__ msk,
                                                const PixelCtx& pc, int r, int q, int cbase_grp, int kc0, int nk,
                                                Ring& ring, volatile int* abort_flag, int* status, int code,
                                                StageFn&& stage_of) {
  const int ncc = g.Cig / BK;
  const int cpc = g.cpo / BK;  // consecutive channel chunks per offset group
  const int xo = (int)pc.img * g.C;
  const int oo = pc.b * (int)g.off_bs + pc.p, mo = pc.b * (int)g.msk_bs + pc.p;
  const int og0 = cbase_grp / g.cpo;  // offset group of the weight group's first channel chunk
  auto load = [&](int o, int t) {
    RawSample<T> rs;
    const int ob = DCN_BOUND(oo + (o * 2 * g.T + 2 * t) * g.HWo, g.HWo + 1, g.B * g.off_bs, DBG_TC_GATHER_OFF);
    rs.dy = off[ob];
    rs.dx = off[ob + g.HWo];
    rs.m = msk ? msk[DCN_BOUND(mo + (o * g.T + t) * g.HWo, 1, g.B * g.msk_bs, DBG_TC_GATHER_MSK)]
               : from_f<T>(1.f);
    return rs;
  };
  // chunk position in gather order: tap t = (ti, tj), channel chunk cc, its
  // offset group o and the chunk's index within that offset group (oc)
  struct Pos {
    int t, ti, tj, cc, o, oc;
  };
  Pos p0;
  p0.t = kc0 / ncc;
  p0.cc = kc0 - p0.t * ncc;
  p0.ti = p0.t / g.kw;
  p0.tj = p0.t - p0.ti * g.kw;
  p0.o = og0 + p0.cc / cpc;
  p0.oc = p0.cc - (p0.cc / cpc) * cpc;
  auto advance = [&](Pos p) {
    if (++p.cc == ncc) {
      p.cc = 0;
      p.o = og0;
      p.oc = 0;
      ++p.t;
      if (++p.tj == g.kw) { p.tj = 0; ++p.ti; }
    } else if (++p.oc == cpc) {
      p.oc = 0;
      ++p.o;
    }
    return p;
  };
  // the lane's channels [8q, 8q+8) and [32+8q, 32+8q+8): two 128-bit loads
  // per corner (one 256-bit load of [16q, 16q+16) measured no faster)
  auto issue = [&](const CornerSet32& c, int cc, uint4 (&dst)[8]) {
    const int cb = cbase_grp + cc * BK + q * 8;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (c.w[k] != 0.f) {
        const uint4* src = reinterpret_cast<const uint4*>(
            xh + DCN_BOUND((uint32_t)(xo + c.off[k] + cb), 40, (long long)g.B * g.H * g.W * g.C, DBG_TC_GATHER_X));
        dst[2 * k] = __ldg(src);
        dst[2 * k + 1] = __ldg(src + 4);  // 32 channels further
      } else {
        dst[2 * k] = make_uint4(0, 0, 0, 0);
        dst[2 * k + 1] = make_uint4(0, 0, 0, 0);
      }
    }
  };
  CornerSet32 cs = corner_set32<T, LOGIT>(g, pc, load(p0.o, p0.t), p0.ti, p0.tj);
  uint4 v[8];
  issue(cs, p0.cc, v);
  Pos p1 = p0;
  RawSample<T> raw1{};
  if (nk > 1) {
    p1 = advance(p0);
    if (p1.t != p0.t || p1.o != p0.o) raw1 = load(p1.o, p1.t);
  }
  const int o_lo = r * 128 + ((q ^ (r & 7)) << 4), o_hi = r * 128 + (((q + 4) ^ (r & 7)) << 4);
  for (int i = 0; i < nk; ++i) {
    const uint4 c_lo[4] = {v[0], v[2], v[4], v[6]}, c_hi[4] = {v[1], v[3], v[5], v[7]};
    const uint4 b_lo = blend8<T>(c_lo, cs.w), b_hi = blend8<T>(c_hi, cs.w);
    uint8_t* tile;
    uint32_t empty_bar, full_bar;
    stage_of(ring.s, tile, empty_bar, full_bar);
    if (!mbar_wait(empty_bar, ring.ph ^ 1u, abort_flag, status, code)) return false;
    *reinterpret_cast<uint4*>(tile + o_lo) = b_lo;
    *reinterpret_cast<uint4*>(tile + o_hi) = b_hi;
    fence_async_shared();
    mbar_arrive(full_bar);
    ring.next();
    if (i + 1 < nk) {
      // chunk i+1: a new sampling point only when the tap or offset group
      // changes; then the offsets and mask of the chunk after it
      if (p1.t != p0.t || p1.o != p0.o) cs = corner_set32<T, LOGIT>(g, pc, raw1, p1.ti, p1.tj);
      issue(cs, p1.cc, v);
      p0 = p1;
      if (i + 2 < nk) {
        p1 = advance(p0);
        if (p1.t != p0.t || p1.o != p0.o) raw1 = load(p1.o, p1.t);
      }
    }
  }
  return true;
}

// Corner-quad records for offset groups of 8 channels.  Record (b, y0, x0, o)
// holds the 8 channels of offset group o at the four corners (y0, x0),
// (y0, x0+1), (y0+1, x0), (y0+1, x0+1) of image b, corner-major, 64 bytes;
// corners outside the image are zero.  y0 runs over [-1, H-1] and x0 over
// [-1, W-1], so every sample inside (-1, H) x (-1, W) has its record, and
// one record replaces the sample's four scattered 16-byte corner reads.
// Element offset of a record: ((b*(H+1) + y0+1)*(W+1) + x0+1)*C*4 + o*32.
__host__ __device__ inline long long quad_elems(const Geom& g) {
  return (long long)g.B * (g.H + 1) * (g.W + 1) * g.C * 4;
}
// The forward and the backward take the corner-quad path together: offset
// groups of 8 channels, 32-bit record offsets, one record row per grid row.
__host__ __device__ inline bool quad_ok(const Geom& g) {
  return g.cpo == 8 && quad_elems(g) < (1LL << 31) && (long long)g.B * (g.H + 1) <= 65535;
}

// channels-last input [B][H][W][C] -> corner-quad records (gather_run_quad):
// blockIdx.y = b*(H+1) + y0+1 is one row of records; its threads copy
// 16 bytes each (offset group o's 8 channels of one corner, zero outside the
// image), consecutive threads writing consecutive 16 bytes and reading whole
// 128-byte pixel rows.
template <typename T>
__global__ void quad_records_kernel(const T* __restrict__ xh, T* __restrict__ xq, int H, int W, int C) {
  const int yy = blockIdx.y % (H + 1), b = blockIdx.y / (H + 1);
  const int per_pix = C / 2;  // 16-byte pieces per record position: (C/8 groups) x 4 corners
  const int n = (W + 1) * per_pix;
  uint4* dst = reinterpret_cast<uint4*>(xq) + (size_t)blockIdx.y * n;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) {
    const int xx = e / per_pix, r = e - xx * per_pix;
    const int o = r >> 2, k = r & 3;
    const int y = yy - 1 + (k >> 1), x = xx - 1 + (k & 1);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (y >= 0 && y < H && x >= 0 && x < W)
      v = *reinterpret_cast<const uint4*>(xh + (((size_t)b * H + y) * W + x) * C + o * 8);
    dst[e] = v;
  }
}

template <typename T>
inline void quad_records_launch(const T* xh, T* xq, const Geom& g, cudaStream_t st) {
  const int n = (g.W + 1) * (g.C / 2);
  const dim3 grid((unsigned)((n + 255) / 256), (unsigned)(g.B * (g.H + 1)));
  quad_records_kernel<T><<<grid, 256, 0, st>>>(xh, xq, g.H, g.W, g.C);
}

// Producer for offset groups of exactly 8 channels (one group per lane's
// 16-byte channel vector): lanes and rows as gather_run, each sample read from
// its corner-quad record with two 256-bit loads.  Same stage protocol and
// return value as gather_run.
template <typename T, bool LOGIT, class StageFn>
__device__ __forceinline__ bool gather_run_quad(const Geom& g, const T* __restrict__ xq,
                                                const T* __restrict__ off, const T* __restrict__ msk,
                                                const PixelCtx (&pc)[2], int r0, int q, int cbase_grp, int kc0,
                                                int nk, Ring& ring, volatile int* abort_flag, int* status, int code,
                                                StageFn&& stage_of) {
  const int ncc = g.Cig / BK;
  int qb[2], oo[2], mo[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    qb[h] = pc[h].b * (g.H + 1);  // record row of (b, y0 = -1)
    oo[h] = pc[h].b * (int)g.off_bs + pc[h].p;
    mo[h] = pc[h].b * (int)g.msk_bs + pc[h].p;
  }
  auto load = [&](int h, int o, int t) {
    RawSample<T> rs;
    const int ob = DCN_BOUND(oo[h] + (o * 2 * g.T + 2 * t) * g.HWo, g.HWo + 1, g.B * g.off_bs, DBG_TC_GATHER_OFF);
    rs.dy = off[ob];
    rs.dx = off[ob + g.HWo];
    rs.m = msk ? msk[DCN_BOUND(mo[h] + (o * g.T + t) * g.HWo, 1, g.B * g.msk_bs, DBG_TC_GATHER_MSK)]
               : from_f<T>(1.f);
    return rs;
  };
  GatherWalk kw;
  kw.start(g, kc0, ncc);
  int o = (cbase_grp + kw.cc * BK) / 8 + q;  // the lane's offset group (8 channels each)
  RawSample<T> raw[2] = {load(0, o, kw.t), load(1, o, kw.t)};
  const int r1 = r0 + 4;
  const int o0 = r0 * 128 + ((q ^ (r0 & 7)) << 4), o1 = r1 * 128 + ((q ^ (r1 & 7)) << 4);
  for (int i = 0; i < nk; ++i) {
    uint4 v[2][4];
    float w[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const SamplePos sp = sample_pos(pc[h].y0 + kw.ti * g.dh, pc[h].x0 + kw.tj * g.dw, to_f(raw[h].dy),
                                      to_f(raw[h].dx));
      const Corners c = corners_of(sp, g.H, g.W);
      const float mv = to_f(raw[h].m);
      const float m = pc[h].valid ? (LOGIT ? 1.f / (1.f + __expf(-mv)) : mv) : 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) w[h][k] = c.w[k] * m;
      // a non-zero weight implies the sample lies inside (-1, H) x (-1, W)
      if (w[h][0] != 0.f || w[h][1] != 0.f || w[h][2] != 0.f || w[h][3] != 0.f) {
        const T* rec = xq + DCN_BOUND((uint32_t)(((qb[h] + sp.y0 + 1) * (g.W + 1) + sp.x0 + 1) * (g.C * 4) + o * 32),
                                      32, quad_elems(g), DBG_TC_GATHER_QUAD);
        ldg256(rec, v[h][0], v[h][1]);
        ldg256(rec + 16, v[h][2], v[h][3]);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) v[h][k] = make_uint4(0, 0, 0, 0);
      }
    }
    if (i + 1 < nk) {  // the next chunk's offsets and mask
      kw.next(g, ncc);
      o = (cbase_grp + kw.cc * BK) / 8 + q;
      raw[0] = load(0, o, kw.t);
      raw[1] = load(1, o, kw.t);
    }
    uint8_t* tile;
    uint32_t empty_bar, full_bar;
    stage_of(ring.s, tile, empty_bar, full_bar);
    const uint4 b0 = blend8<T>(v[0], w[0]), b1 = blend8<T>(v[1], w[1]);
    if (!mbar_wait(empty_bar, ring.ph ^ 1u, abort_flag, status, code)) return false;
    *reinterpret_cast<uint4*>(tile + o0) = b0;
    *reinterpret_cast<uint4*>(tile + o1) = b1;
    fence_async_shared();
    mbar_arrive(full_bar);
    ring.next();
  }
  return true;
}

// ---------------------------------------------------------------- weight images
// weight [Co][Cig][T] -> the two pre-swizzled tile images, in one pass: the
// forward's wsw [G][NKC][Cog][64] (K chunk kc = t*(Cig/64) + cc, chunk q of
// row co at q ^ (co % 8)) and dgrad's W^T tiles wdt [G][NKC][KB][64 ch][64 co]
// (kc = cc*T + t, chunk q of row j at q ^ (j % 8), co >= Cog zero); either
// output may be null.  blockIdx.x = 8 output channels (up to KB*64: the CTAs
// past Cog write wdt's zero chunks), blockIdx.y = group, blockIdx.z = the
// 64-channel block cc, whose T*64 weights of each output channel are
// contiguous: the 8 rows' blocks are staged in shared memory with coalesced
// loads, so every global access is a whole row run or a whole 16-byte chunk.
// Dynamic shared memory: weight_images_smem(T) bytes.
inline size_t weight_images_smem(int T_, size_t es) { return 8 * (size_t)BK * T_ * es; }

template <typename T>
__global__ void weight_images_kernel(const T* __restrict__ w, T* __restrict__ wsw, T* __restrict__ wdt, int Cog,
                                     int Cig, int T_) {
  extern __shared__ __align__(16) uint8_t wi_smem[];
  T* rows = reinterpret_cast<T*>(wi_smem);  // [8][64 * T]: channels cc*64 .. cc*64+63 of 8 output channels
  const int Kg = Cig * T_, ncc = Cig / BK, nkc = ncc * T_, KB = (Cog + 63) / 64, run = BK * T_;
  const int grp = blockIdx.y, co0 = blockIdx.x * 8, cc = blockIdx.z;
  const bool live = co0 < Cog;
  {  // a row's run is 128*T bytes at a 128-byte multiple of w: 16-byte loads
    const int run16 = run * (int)sizeof(T) / 16;
    uint4* rows16 = reinterpret_cast<uint4*>(rows);
    for (int i = threadIdx.x; i < 8 * run16; i += blockDim.x) {
      const int r = i / run16, e = i - r * run16;
      rows16[i] = live ? reinterpret_cast<const uint4*>(w + ((size_t)grp * Cog + co0 + r) * Kg +
                                                        (size_t)cc * run)[e]
                       : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  __syncthreads();
  if (wsw && live) {  // (row r, tap t, chunk q) -> 16 bytes of row co0 + r of K chunk t*ncc + cc
    for (int i = threadIdx.x; i < T_ * 64; i += blockDim.x) {
      const int q = i & 7, rt = i >> 3, t = rt % T_, r = rt / T_;
      const T* src = rows + r * run + (q * 8) * T_ + t;
      __align__(16) T v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = src[j * T_];
      const int co = co0 + r, kc = t * ncc + cc;
      *reinterpret_cast<uint4*>(wsw + (((size_t)grp * nkc + kc) * Cog + co) * BK + ((q ^ (co & 7)) << 3)) =
          *reinterpret_cast<const uint4*>(v);
    }
  }
  if (wdt) {  // (tap t, channel row j) -> the chunk of output channels co0 .. co0+7 of K chunk cc*T + t
    const int kb = co0 / 64, qq = (co0 % 64) / 8;
    for (int i = threadIdx.x; i < T_ * 64; i += blockDim.x) {
      const int j = i & 63, t = i >> 6;
      __align__(16) T v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = rows[k * run + j * T_ + t];
      const int kc = cc * T_ + t;
      *reinterpret_cast<uint4*>(wdt + ((((size_t)grp * nkc + kc) * KB + kb) * 64 + j) * 64 + ((qq ^ (j & 7)) << 3)) =
          *reinterpret_cast<const uint4*>(v);
    }
  }
}

// Launches weight_images_kernel; false when its staging does not fit (the
// caller then uses the per-image kernels).
template <typename T>
inline bool weight_images_launch(const T* w, T* wsw, T* wdt, const Geom& g, cudaStream_t st) {
  const size_t smem = weight_images_smem(g.T, sizeof(T));
  if (smem > 96 * 1024 || (reinterpret_cast<uintptr_t>(w) & 15)) return false;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(weight_images_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess)
    return false;
  const int KB = (g.Cog + 63) / 64;
  weight_images_kernel<T><<<dim3((unsigned)(KB * 8), (unsigned)g.G, (unsigned)(g.Cig / BK)), 256, smem, st>>>(
      w, wsw, wdt, g.Cog, g.Cig, g.T);
  return true;
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

// Host: device address of the status word on the current device.
cudaError_t tc_status_ptr(int** out);

}  // namespace dcn
