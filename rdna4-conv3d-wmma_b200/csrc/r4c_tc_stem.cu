// r4c_tc_stem.cu — tcgen05 forward conv for k=3 layers with 1..4 input
// channels (the network stem, e.g. the 1 -> 24 input conv of a 3D UNet).
//
// The general kernel (r4c_tc.cu) needs Cin padded to 8 channels and moves one
// 16-byte TMA row per brick position per stage; with Cin = 1 that is eight
// times the activation bytes, a TMA box of short rows (the slowest shape the
// TMA unit moves), and MMAs whose K is 7/8 zeros. Here instead:
//   * one TMA box per work unit brings the raw input brick
//     [P+2 planes][bh+2 rows][wb*Cin elements] — channels and width merged
//     into one dimension, so rows are hundreds of bytes long; the zero
//     padding of the conv comes from the TMA out-of-bounds fill;
//   * eight builder warps expand the brick into im2col rows in shared memory:
//     one 128-row A tile per 128 output positions, K = 27*Cin taps padded to
//     a multiple of 16, in the no-swizzle K-major core-matrix layout; the
//     tiles of a unit form one A buffer (two buffers alternate), handed to
//     the MMA thread with one barrier per unit — an mbarrier hand-off costs
//     a few hundred clocks, too much to pay per 128-row tile;
//   * one thread issues M=128 x N=Cout(16-padded) x K MMAs into TMEM (two
//     accumulator sets), the packed weight [N][K] staying resident in
//     shared memory;
//   * eight epilogue warps add the bias, round and store NDHWC rows.
// Warp roles: 0 TMA producer, 1 MMA issuer (TMEM owner), 2-9 epilogue,
// 10-17 builders. Every wait is bounded (1 s): on expiry the kernel raises the
// library's device error flag and all roles leave their loops.
//
// The arithmetic is the conv's definition (PyTorch Conv3d, cross-correlation):
//   y[n,z,y,x,co] = b[co] + sum_{c,kd,kh,kw} w[co,c,kd,kh,kw] *
//                   x[n, z+kd-pd, y+kh-ph, x+kw-pw, c]
// with fp32 accumulation of bf16/fp16 products and one rounding at the end,
// the contract of the reference's WMMA path (reference: rdna4_conv3d/
// conv3d_wmma.py, the implicit-GEMM forward with f32 accumulators).
#include <cuda.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "r4c_internal.h"
#include "r4c_sm100.cuh"

namespace r4c {
namespace stem {

using namespace sm100;

// warps: 0 TMA producer, 1 MMA issuer, 2..9 epilogue (two per TMEM lane
// quarter, alternate tiles), 10..17 builders (two per A row, alternate tiles).
// Each role is latency-bound per thread (shared loads feeding shifts feeding
// stores), so two warps of each per SM sub-partition hide each other's
// latency.
constexpr int kEpiWarps = 8;
constexpr int kBuildWarps = 8;
constexpr int kThreads = 64 + 32 * (kEpiWarps + kBuildWarps);
constexpr int kHeader = 4096;
constexpr int kMaxRaw = 16;   // raw brick stages (TMA latency under load is several us)
constexpr int kABufs = 2;     // A buffers (builders one unit ahead of the MMA)
constexpr int kMaxSets = 4;   // TMEM accumulator sets (MMA ahead of the epilogue)
constexpr int kSmemMax = 232448;

struct StemArgs {
  CUtensorMap xmap;  // (W*Cin, H, D, N, 1) elements, box (wb*Cin, bh+2, P+2, 1, 1)
  const uint8_t* wpack;
  const void* bias;
  void* y;
  int* err;
  int n, d, h, w, cin, cout;
  int od, oh, ow, pd, ph, pw;
  int bw, bh, P, wb, walign;
  int nwt, nht, nzb;
  int units;
  int nsets;
  int mtiles, npad, kpad, ksteps;
  int raw_bytes, raw_tx, a_bytes, w_bytes, w_region;
  int abuf_bytes;  // one A buffer: mtiles tiles of a_bytes
  int nraw;        // raw brick stages in the ring (<= kMaxRaw)
  int tmem_cols;
  uint32_t idesc;
};

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// 16 accumulator columns [cc, cc+16) of one output row: + bias, rounded,
// stored as 16-byte groups of 8 channels (vec_ok: cout % 8 == 0) or per
// element. bias4: the fp32 bias as float4 in shared memory.
template <typename T>
__device__ __forceinline__ void store_row(T* dst, const float* v, const float4* bias4, int cc, int cout,
                                          bool vec_ok) {
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const int c0 = cc + 8 * g;
    if (c0 >= cout) break;
    const float4 b0 = bias4[c0 / 4], b1 = bias4[c0 / 4 + 1];
    const float f[8] = {v[8 * g] + b0.x,     v[8 * g + 1] + b0.y, v[8 * g + 2] + b0.z, v[8 * g + 3] + b0.w,
                        v[8 * g + 4] + b1.x, v[8 * g + 5] + b1.y, v[8 * g + 6] + b1.z, v[8 * g + 7] + b1.w};
    if (vec_ok) {
      *reinterpret_cast<uint4*>(dst + c0) =
          make_uint4(pack2<T>(f[0], f[1]), pack2<T>(f[2], f[3]), pack2<T>(f[4], f[5]), pack2<T>(f[6], f[7]));
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (c0 + i < cout) dst[c0 + i] = Elem<T>::from_f(f[i]);
    }
  }
}

// K layout of the im2col rows: the 9 (kd, kh) brick rows are groups of
// 4*C elements, the 3*C taps (kw, c) of the group then C zeros. A group is
// then a whole number of 32-bit words starting on a word boundary, built from
// aligned shared loads with at most a funnel shift, instead of 27*C packed
// 16-bit taps (the padding taps get zero weights; K grows to 36*C).
template <int C> struct StemK {
  static constexpr int GW = 2 * C;                  // words per group
  static constexpr int KPAD = (36 * C + 15) / 16 * 16;
  static constexpr int WORDS = KPAD / 2;            // words per row
  static constexpr int KS = KPAD / 16;              // 16-wide K steps
};

// One im2col row (output position of the unit whose window starts at `raw`,
// in elements of the raw brick; `odd`: raw starts at an odd element — rows
// and planes of the brick have even lengths) written as KPAD/8 16-byte chunks
// of the core-matrix layout (chunk j of row m at (m/8)*KPAD*16 + j*128 +
// (m%8)*16).
template <int C>
__device__ __forceinline__ void build_row(uint8_t* slot, int m, const uint16_t* raw, int row_elems, int plane_elems,
                                          uint32_t odd, bool live, uint32_t one = 0u) {
  using K = StemK<C>;
  uint32_t wr[K::WORDS];
#pragma unroll
  for (int i = 0; i < K::WORDS; ++i) wr[i] = 0u;
  if (live) {
    const uint32_t sh = 16u * odd;
#pragma unroll
    for (int g = 0; g < 9; ++g) {
      const int kd = g / 3, kh = g % 3;
      const uint16_t* src = raw + kd * plane_elems + kh * row_elems;
      const uint32_t* w = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(src) & ~(uintptr_t)3);
      if constexpr (C % 2 == 0) {
        // even C: the run starts on a word; 3C/2 words, then C/2 zero words
#pragma unroll
        for (int j = 0; j < 3 * C / 2; ++j) wr[g * K::GW + j] = w[j];
      } else {
        // odd C: (3C+1)/2 words cover the run from either parity; pairs of
        // elements by funnel shift, the last element with a zero by byte
        // permute (high or low half of the last word)
        constexpr int NL = (3 * C + 1) / 2;
        uint32_t v[NL];
#pragma unroll
        for (int j = 0; j < NL; ++j) v[j] = w[j];
#pragma unroll
        for (int j = 0; j < (3 * C - 1) / 2; ++j) wr[g * K::GW + j] = __funnelshift_r(v[j], v[j + 1], sh);
        wr[g * K::GW + (3 * C - 1) / 2] = __byte_perm(v[NL - 1], 0u, odd ? 0x4432u : 0x4410u);
      }
    }
    // the weight gradient's db slot: element 3C (the first zero slot of
    // group 0) holds `one` (the 16-bit pattern of 1.0; 0 for the forward)
    wr[(3 * C) / 2] |= one << (16 * ((3 * C) & 1));
  }
  uint8_t* base = slot + (m >> 3) * (K::KPAD * 16) + (m & 7) * 16;
#pragma unroll
  for (int j = 0; j < K::KPAD / 8; ++j)
    *reinterpret_cast<uint4*>(base + j * 128) = make_uint4(wr[4 * j], wr[4 * j + 1], wr[4 * j + 2], wr[4 * j + 3]);
}

// This CTA's units u = blockIdx.x, + gridDim.x, ... as (nb, zb, hi, wi), wi
// fastest, advanced by carries (one add and compare per digit) rather than
// four divisions per unit in every role.
struct UnitWalk {
  int wi, hi, zb, nb, gw, gh, gz, gn;
  template <class Args> __device__ void init(const Args& a) {
    int u = blockIdx.x;
    wi = u % a.nwt; u /= a.nwt;
    hi = u % a.nht; u /= a.nht;
    zb = u % a.nzb; nb = u / a.nzb;
    int g = gridDim.x;
    gw = g % a.nwt; g /= a.nwt;
    gh = g % a.nht; g /= a.nht;
    gz = g % a.nzb; gn = g / a.nzb;
  }
  template <class Args> __device__ void next(const Args& a) {
    wi += gw;
    int c = wi >= a.nwt;
    if (c) wi -= a.nwt;
    hi += gh + c;
    c = hi >= a.nht;
    if (c) hi -= a.nht;
    zb += gz + c;
    c = zb >= a.nzb;
    if (c) zb -= a.nzb;
    nb += gn + c;
  }
};

template <typename T, int C>
__global__ void __launch_bounds__(kThreads, 1) stem_fwd_kernel(const __grid_constant__ StemArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* raw_empty = raw_full + kMaxRaw;
  uint64_t* a_full = raw_empty + kMaxRaw;
  uint64_t* a_empty = a_full + kABufs;
  uint64_t* tfull = a_empty + kABufs;
  uint64_t* tempty = tfull + kMaxSets;
  uint64_t* mdone = tempty + kMaxSets;
  uint64_t* wbar = mdone + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wbar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sbias = reinterpret_cast<float*>(smem + 1024);  // 256 floats (+8 of padding read as float4)
  uint8_t* wsm = smem + kHeader;
  uint8_t* raw0 = wsm + a.w_region;
  uint8_t* abuf0 = raw0 + a.nraw * a.raw_bytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if ((smem_u32(smem) & 1023u) != 0u || a.tmem_cols > 512) {
    if (threadIdx.x == 0) atomicExch(a.err, 2);
    return;
  }
  {
    const T* bias = static_cast<const T*>(a.bias);
    for (int i = threadIdx.x; i < a.npad + 8; i += kThreads)
      sbias[i] = (bias != nullptr && i < a.cout) ? Elem<T>::to_f(bias[i]) : 0.f;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kMaxRaw; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kBuildWarps);
    }
    for (int s = 0; s < kABufs; ++s) {
      mbar_init(&a_full[s], kBuildWarps);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < kMaxSets; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], kEpiWarps);
    }
    mbar_init(mdone, 1);
    mbar_init(wbar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, (uint32_t)a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const uint64_t kWaitNs = 1000000000ull;
  // Bounded wait; `nap` > 0 makes the polling thread sleep between polls so
  // that waiting roles leave issue slots to the working ones.
  auto wait = [&](uint64_t* bar, uint32_t par, uint32_t nap = 0) -> bool {
    uint64_t deadline = 0;  // the clock is read only once a wait has lasted a while
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, par)) {
      if (nap) __nanosleep(nap);
      if (((++spins) & 63u) == 0) {
        if (*abort_flag) return false;
        const uint64_t now = global_timer_ns();
        if (deadline == 0) {
          deadline = now + kWaitNs;
        } else if (now > deadline) {
          *abort_flag = 1;
          atomicExch(a.err, 1);
          return false;
        }
      }
    }
    return true;
  };
  UnitWalk uw;
  uw.init(a);
  const int set_cols = a.mtiles * a.npad;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&a.xmap);
      mbar_arrive_expect_tx(wbar, (uint32_t)a.w_bytes);
      bulk_load(wsm, a.wpack, (uint32_t)a.w_bytes, wbar);
      int rs = 0;
      uint32_t epar = 1;
      uint32_t pending = 0u, last_par = 0u;  // per stage bits
      for (int u = blockIdx.x; u < a.units; u += gridDim.x, uw.next(a)) {
        const int nb = uw.nb, z0 = uw.zb * a.P, y0 = uw.hi * a.bh, x0 = uw.wi * a.bw;
        if (!wait(&raw_empty[rs], epar, 64)) break;
        const int xs = x0 - a.pw;
        const int ws = xs & -a.walign;  // floor to a multiple of walign (a power of two)
        mbar_arrive_expect_tx(&raw_full[rs], (uint32_t)a.raw_tx);
        tma_load_5d(raw0 + (size_t)rs * a.raw_bytes, &a.xmap, &raw_full[rs], ws * a.cin, y0 - a.ph, z0 - a.pd, nb,
                    0);
        pending |= 1u << rs;
        last_par = (last_par & ~(1u << rs)) | ((epar ^ 1u) << rs);
        if (++rs == a.nraw) { rs = 0; epar ^= 1; }
      }
      // no copy may outlive the CTA (matters only after an abort: normally
      // the builders consumed every stage)
      const uint64_t deadline = global_timer_ns() + kWaitNs;
      for (int s = 0; s < a.nraw; ++s)
        if ((pending >> s) & 1u) mbar_wait_bounded(&raw_full[s], (last_par >> s) & 1u, deadline);
      mbar_wait_bounded(wbar, 0, deadline);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = wait(wbar, 0);
      uint32_t apar = 0u, tpar = (1u << kMaxSets) - 1u;  // per buffer / set phase bits
      int set = 0, ab = 0;
      constexpr int KS = StemK<C>::KS;  // 16-wide K steps
      const uint32_t a0 = smem_u32(abuf0);
      const uint32_t sbo = (uint32_t)a.kpad * 16u;
      const uint64_t bd0 = smem_desc(smem_u32(wsm), 128u, sbo);
      for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
        if (!wait(&tempty[set], (tpar >> set) & 1u)) { ok = false; break; }
        tpar ^= 1u << set;
        if (!wait(&a_full[ab], (apar >> ab) & 1u)) { ok = false; break; }
        apar ^= 1u << ab;
        tc_fence_after();
        // descriptors advance by start-address units (16 bytes): a K step is
        // two core-matrix columns (256 bytes), a tile a_bytes; K steps are
        // unrolled (an MMA per loop iteration costs a branch bubble)
        const uint64_t ad0 = smem_desc(a0 + (uint32_t)(ab * a.abuf_bytes), 128u, sbo);
#pragma unroll 2
        for (int t = 0; t < a.mtiles; ++t) {
          const uint32_t d = tmem + (uint32_t)(set * set_cols + t * a.npad);
          const uint64_t ad = ad0 + (uint64_t)((t * a.a_bytes) >> 4);
#pragma unroll
          for (int ks = 0; ks < KS; ++ks)
            mma_f16_ss(d, ad + (uint64_t)(ks * 16), bd0 + (uint64_t)(ks * 16), a.idesc, ks > 0 ? 1u : 0u);
        }
        mma_commit(&a_empty[ab]);
        mma_commit(&tfull[set]);
        if (++set == a.nsets) set = 0;
        ab ^= 1;
      }
      mma_commit(mdone);
      wait(mdone, 0);
    }
  } else if (warp < 2 + kEpiWarps) {
    // ---------------- epilogue (warps 2..9) ----------------
    const int q = warp & 3;             // TMEM lane quarter this warp may read
    const int t_first = (warp - 2) >> 2;  // tiles t_first, t_first + 2, ...
    const int row = q * 32 + lane;
    const float4* bias4 = reinterpret_cast<const float4*>(sbias);
    T* __restrict__ y = static_cast<T*>(a.y);
    const bool vec_ok = (a.cout % 8) == 0;
    uint32_t fpar = 0u;  // per set phase bits
    int set = 0;
    // this thread's rows of its (up to four) tiles, the same in every unit:
    // brick coordinates and position offset within the output
    const int per_plane = a.bh * a.bw;
    const int total = a.P * per_plane;
    int zo_[4], yo_[4], xo_[4], pos_[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int l = (t_first + 2 * i) * 128 + row;
      const int zo = l / per_plane, rem = l - zo * per_plane;
      yo_[i] = rem / a.bw;
      xo_[i] = rem - yo_[i] * a.bw;
      zo_[i] = l < total ? zo : (1 << 20);  // rows past the unit: never valid
      pos_[i] = (zo * a.oh + yo_[i]) * a.ow + xo_[i];
    }
    for (int u = blockIdx.x; u < a.units; u += gridDim.x, uw.next(a)) {
      const int nb = uw.nb, z0 = uw.zb * a.P, y0 = uw.hi * a.bh, x0 = uw.wi * a.bw;
      const long long ubase = (((long long)nb * a.od + z0) * a.oh + y0) * a.ow + x0;
      int got = 1;
      if (lane == 0) got = wait(&tfull[set], (fpar >> set) & 1u, 64) ? 1 : 0;
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      fpar ^= 1u << set;
      tc_fence_after();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = t_first + 2 * i;
        if (t >= a.mtiles) break;
        const bool valid = z0 + zo_[i] < a.od && y0 + yo_[i] < a.oh && x0 + xo_[i] < a.ow;
        T* dst = y + (ubase + pos_[i]) * a.cout;
        const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(set * set_cols + t * a.npad);
        int cc = 0;
        for (; cc + 32 <= a.npad; cc += 32) {
          float v[32];
          tmem_ld_32(tb + (uint32_t)cc, v);
          if (valid) {
            store_row<T>(dst, v, bias4, cc, a.cout, vec_ok);
            store_row<T>(dst, v + 16, bias4, cc + 16, a.cout, vec_ok);
          }
        }
        if (cc < a.npad) {
          float v[16];
          tmem_ld_16(tb + (uint32_t)cc, v);
          if (valid) store_row<T>(dst, v, bias4, cc, a.cout, vec_ok);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[set]);
      if (++set == a.nsets) set = 0;
    }
  } else {
    // ---------------- im2col builders (warps 10..17) ----------------
    const int bt = threadIdx.x - 32 * (2 + kEpiWarps);
    const int m = bt & 127;      // A row
    const int t_first = bt >> 7;  // tiles t_first, t_first + 2, ...
    const int per_plane = a.bh * a.bw;
    const int total = a.P * per_plane;
    const int row_elems = a.wb * C;
    const int plane_elems = (a.bh + 2) * row_elems;
    int rs = 0, ab = 0;
    uint32_t rpar = 0;
    uint32_t epar = (1u << kABufs) - 1u;  // per A buffer phase bits
    for (int u = blockIdx.x; u < a.units; u += gridDim.x, uw.next(a)) {
      const int nb = uw.nb, z0 = uw.zb * a.P, y0 = uw.hi * a.bh, x0 = uw.wi * a.bw;
      const int xs = x0 - a.pw;
      const int ws = xs & -a.walign;  // floor to a multiple of walign (a power of two)
      const int off = xs - ws;  // first needed column within the box
      int got = 1;
      if (lane == 0) got = (wait(&raw_full[rs], rpar, 32) && wait(&a_empty[ab], (epar >> ab) & 1u, 32)) ? 1 : 0;
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      epar ^= 1u << ab;
      const uint16_t* raw = reinterpret_cast<const uint16_t*>(raw0 + (size_t)rs * a.raw_bytes);
      uint8_t* abuf = abuf0 + (size_t)ab * a.abuf_bytes;
      for (int t = t_first; t < a.mtiles; t += 2) {
        const int l = t * 128 + m;
        const bool live = l < total;
        const int lc = live ? l : 0;
        const int zo = lc / per_plane;
        const int rem = lc - zo * per_plane;
        const int yo = rem / a.bw;
        const int xo = rem - yo * a.bw;
        const int e0 = zo * plane_elems + yo * row_elems + (off + xo) * C;  // rows and planes are even
        build_row<C>(abuf + (size_t)t * a.a_bytes, m, raw + e0, row_elems, plane_elems, (uint32_t)e0 & 1u, live);
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[ab]);
        mbar_arrive(&raw_empty[rs]);
      }
      ab ^= 1;
      if (++rs == a.nraw) { rs = 0; rpar ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)a.tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// Weight gradient of the stem conv (k=3, 1..4 input channels):
//   dW[co][c][kd][kh][kw] = sum_v dY[v][co] * x[v + (kd,kh,kw) - pad][c]
//   db[co]                = sum_v dY[v][co]
// as D[k][co] += A[k][v] * B[v][co] over the output positions v of each work
// unit (reference counterpart: the _wgrad_kernel GEMM with K = voxels and the
// separate db sum). A is the unit's im2col rows, built exactly as for the
// forward and read here as an MN-major operand (M = the StemK slots k, K =
// positions; slot 3C of group 0 holds ones, so D row 3C is db). B is the
// unit's dY brick: one TMA box of whole-channel rows (Cout*2 bytes, one TMA
// row per position) that the builders re-lay into 8-channel planes (MN-major,
// N = Cout). Each CTA accumulates all its units in one TMEM accumulator and
// writes it once as an fp32 partial; stem_dw_reduce sums the partials in CTA
// order (deterministic).
// Warps: 0 TMA producer, 1 MMA issuer, 2..9 builders (and, at the end, 2..5
// read the accumulator, one TMEM lane quarter each).
constexpr int kDwBuildWarps = 8;
constexpr int kDwThreads = 64 + 32 * kDwBuildWarps;
constexpr int kDwMaxStages = 16;
constexpr int kDwMaxBufs = 3;  // A+B buffer pairs: builders up to two units ahead of the MMA

struct StemDwArgs {
  CUtensorMap xmap;  // as StemArgs::xmap
  CUtensorMap gmap;  // dY: (Cout, OW, OH, OD, N), box (Cout, bw, bh, P, 1)
  float* part;       // [gridDim.x][kpad][npad] fp32
  int* err;
  int n, d, h, w, cin, cout;
  int od, oh, ow, pd, ph, pw;
  int bw, bh, P, wb, walign;
  int nwt, nht, nzb;
  int units;
  int mtiles, npad, kpad, mk;    // mk: 128-row M tiles over the kpad slots
  int raw_bytes, raw_tx, g_tx;   // stage = raw brick (raw_bytes) + dY brick
  int stage_bytes, nstages;
  int a_bytes, abuf_bytes;       // A tile (128 positions x kpad), A buffer (mtiles tiles)
  int plane_bytes, bbuf_bytes;   // B: npad/8 planes of mtiles*128 positions x 16 B
  int nbufs;                     // A+B buffer pairs (2 or 3)
  int tmem_cols;
  uint32_t idesc;
  uint32_t one;                  // 16-bit pattern of 1.0 in the element type
};

template <int C>
__global__ void __launch_bounds__(kDwThreads, 1) stem_dw_kernel(const __grid_constant__ StemDwArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* in_full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* in_empty = in_full + kDwMaxStages;
  uint64_t* b_full = in_empty + kDwMaxStages;  // A+B buffer pair ready
  uint64_t* b_empty = b_full + kDwMaxBufs;
  uint64_t* mdone = b_empty + kDwMaxBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* st0 = smem + kHeader;                         // input stages
  uint8_t* abuf0 = st0 + a.nstages * a.stage_bytes;      // nbufs A buffers
  uint8_t* bbuf0 = abuf0 + a.nbufs * a.abuf_bytes;       // nbufs B buffers (also take the M=128
                                                         // over-read of the last A buffer)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if ((smem_u32(smem) & 1023u) != 0u || a.tmem_cols > 512) {
    if (threadIdx.x == 0) atomicExch(a.err, 2);
    return;
  }
  // B planes for channels at or above Cout (npad padding) stay zero
  for (int bi = 0; bi < a.nbufs; ++bi)
    for (int pl = a.cout / 8; pl < a.npad / 8; ++pl)
      for (int i = threadIdx.x * 16; i < a.plane_bytes; i += kDwThreads * 16)
        *reinterpret_cast<uint4*>(bbuf0 + (size_t)bi * a.bbuf_bytes + (size_t)pl * a.plane_bytes + i) =
            make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kDwMaxStages; ++s) {
      mbar_init(&in_full[s], 1);
      mbar_init(&in_empty[s], kDwBuildWarps);
    }
    for (int s = 0; s < kDwMaxBufs; ++s) {
      mbar_init(&b_full[s], kDwBuildWarps);
      mbar_init(&b_empty[s], 1);
    }
    mbar_init(mdone, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, (uint32_t)a.tmem_cols);
    tmem_relinquish();
  }
  fence_proxy_async_smem();  // the zeroed B planes, for the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const uint64_t kWaitNs = 1000000000ull;
  auto wait = [&](uint64_t* bar, uint32_t par, uint32_t nap = 0) -> bool {
    uint64_t deadline = 0;  // the clock is read only once a wait has lasted a while
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, par)) {
      if (nap) __nanosleep(nap);
      if (((++spins) & 63u) == 0) {
        if (*abort_flag) return false;
        const uint64_t now = global_timer_ns();
        if (deadline == 0) {
          deadline = now + kWaitNs;
        } else if (now > deadline) {
          *abort_flag = 1;
          atomicExch(a.err, 1);
          return false;
        }
      }
    }
    return true;
  };
  UnitWalk uw;
  uw.init(a);

  if (warp == 0) {
    // ---------------- TMA producer: raw x brick + dY brick per unit ----------------
    if (lane == 0) {
      prefetch_tmap(&a.xmap);
      prefetch_tmap(&a.gmap);
      int s = 0;
      uint32_t epar = 1;
      uint32_t pending = 0u, last_par = 0u;  // per stage bits
      for (int u = blockIdx.x; u < a.units; u += gridDim.x, uw.next(a)) {
        const int nb = uw.nb, z0 = uw.zb * a.P, y0 = uw.hi * a.bh, x0 = uw.wi * a.bw;
        if (!wait(&in_empty[s], epar, 64)) break;
        const int ws = (x0 - a.pw) & -a.walign;  // floor to a multiple of walign (a power of two)
        uint8_t* sb = st0 + (size_t)s * a.stage_bytes;
        mbar_arrive_expect_tx(&in_full[s], (uint32_t)(a.raw_tx + a.g_tx));
        tma_load_5d(sb, &a.xmap, &in_full[s], ws * a.cin, y0 - a.ph, z0 - a.pd, nb, 0);
        tma_load_5d(sb + a.raw_bytes, &a.gmap, &in_full[s], 0, x0, y0, z0, nb);
        pending |= 1u << s;
        last_par = (last_par & ~(1u << s)) | ((epar ^ 1u) << s);
        if (++s == a.nstages) { s = 0; epar ^= 1; }
      }
      // no copy may outlive the CTA (matters only after an abort)
      const uint64_t deadline = global_timer_ns() + kWaitNs;
      for (int i = 0; i < a.nstages; ++i)
        if ((pending >> i) & 1u) mbar_wait_bounded(&in_full[i], (last_par >> i) & 1u, deadline);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: D[k][co] += A[k][v] B[v][co] ----------------
    if (lane == 0) {
      uint32_t fpar = 0u;  // b_full phase bits
      int ab = 0;
      uint32_t acc = 0u;   // the CTA's first K step starts the accumulator
      const int ksteps = a.mtiles * 8;  // 16 positions per K step
      for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
        if (!wait(&b_full[ab], (fpar >> ab) & 1u)) break;
        fpar ^= 1u << ab;
        tc_fence_after();
        // MN-major, no swizzle: A: LBO = 8-position group (kpad*16 B), SBO =
        // 8-slot group (128 B); B: LBO = 8-position group (128 B), SBO = plane
        const uint64_t ad0 = smem_desc(smem_u32(abuf0 + (size_t)ab * a.abuf_bytes), (uint32_t)a.kpad * 16u, 128u);
        const uint64_t bd0 = smem_desc(smem_u32(bbuf0 + (size_t)ab * a.bbuf_bytes), 128u, (uint32_t)a.plane_bytes);
        // K steps in blocks of 8 (ksteps = 8 * mtiles), unrolled: an MMA per
        // loop iteration would cost a branch bubble each
        constexpr int MK = (StemK<C>::KPAD + 127) / 128;  // 128-slot M tiles
        constexpr uint32_t KG = 2u * StemK<C>::KPAD;      // K step of A in 16-byte units
        for (int kb = 0; kb < ksteps; kb += 8) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint64_t ad = ad0 + (uint64_t)((kb + j) * KG);  // + ks * 2 groups * kpad*16 B
            const uint64_t bd = bd0 + (uint64_t)((kb + j) * 16);  // + ks * 256 B
#pragma unroll
            for (int mk = 0; mk < MK; ++mk)  // slots 128*mk..: + 16 groups of 128 B
              mma_f16_ss(tmem + (uint32_t)(mk * a.npad), ad + (uint64_t)(mk * 128), bd, a.idesc, acc);
            acc = 1u;
          }
        }
        mma_commit(&b_empty[ab]);
        if (++ab == a.nbufs) ab = 0;
      }
      mma_commit(mdone);
    }
  } else {
    // ---------------- builders (warps 2..9): A = im2col rows, B = dY planes ----------------
    const int bt = threadIdx.x - 64;
    const int m = bt & 127;       // A row / position within a tile
    const int t_first = bt >> 7;  // tiles t_first, t_first + 2, ...
    const int per_plane = a.bh * a.bw;
    const int total = a.P * per_plane;
    const int row_elems = a.wb * C;
    const int plane_elems = (a.bh + 2) * row_elems;
    const int nc8 = a.cout / 8;
    int s = 0, ab = 0;
    uint32_t rpar = 0u, epar = (1u << kDwMaxBufs) - 1u;  // in_full phase; b_empty phase bits
    for (int u = blockIdx.x; u < a.units; u += gridDim.x, uw.next(a)) {
      const int x0 = uw.wi * a.bw;
      const int xs = x0 - a.pw;
      const int off = xs - (xs & -a.walign);  // first needed column within the box
      int got = 1;
      if (lane == 0) got = (wait(&in_full[s], rpar, 32) && wait(&b_empty[ab], (epar >> ab) & 1u, 32)) ? 1 : 0;
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      epar ^= 1u << ab;
      const uint16_t* raw = reinterpret_cast<const uint16_t*>(st0 + (size_t)s * a.stage_bytes);
      const uint8_t* gsrc = st0 + (size_t)s * a.stage_bytes + a.raw_bytes;
      uint8_t* abuf = abuf0 + (size_t)ab * a.abuf_bytes;
      uint8_t* bbuf = bbuf0 + (size_t)ab * a.bbuf_bytes;
      for (int t = t_first; t < a.mtiles; t += 2) {
        const int l = t * 128 + m;
        const bool live = l < total;
        const int lc = live ? l : 0;
        const int zo = lc / per_plane;
        const int rem = lc - zo * per_plane;
        const int yo = rem / a.bw;
        const int xo = rem - yo * a.bw;
        const int e0 = zo * plane_elems + yo * row_elems + (off + xo) * C;  // rows and planes are even
        build_row<C>(abuf + (size_t)t * a.a_bytes, m, raw + e0, row_elems, plane_elems, (uint32_t)e0 & 1u, live,
                     a.one);
        // dY row of position l (Cout channels, dense) -> 8-channel planes
        const uint8_t* gr = gsrc + (size_t)lc * a.cout * 2;
        for (int c8 = 0; c8 < nc8; ++c8) {
          const uint4 v = live ? *reinterpret_cast<const uint4*>(gr + c8 * 16) : make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(bbuf + (size_t)c8 * a.plane_bytes + (size_t)l * 16) = v;
        }
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&b_full[ab]);
        mbar_arrive(&in_empty[s]);
      }
      if (++ab == a.nbufs) ab = 0;
      if (++s == a.nstages) { s = 0; rpar ^= 1u; }
    }
    // ---------------- accumulator -> fp32 partial (warps 2..5) ----------------
    if (warp < 6) {
      const int q = warp & 3;
      int got = 1;
      if (lane == 0) got = wait(mdone, 0, 64) ? 1 : 0;
      got = __shfl_sync(0xffffffffu, got, 0);
      if (got) {
        tc_fence_after();
        for (int mk = 0; mk < a.mk; ++mk) {
          const int k = mk * 128 + q * 32 + lane;  // slot row of D
          float* dst = a.part + ((size_t)blockIdx.x * a.kpad + k) * a.npad;
          for (int cc = 0; cc < a.npad; cc += 16) {
            float v[16];
            tmem_ld_16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(mk * a.npad + cc), v);
            if (k < a.kpad) {
#pragma unroll
              for (int i = 0; i < 16; i += 4)
                *reinterpret_cast<float4*>(dst + cc + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)a.tmem_cols);
  }
}

// Sum of the CTA partials: dW in OIDHW fp32 (slot k of tap (kd,kh,kw),
// channel c: k = (kd*3+kh)*4*cin + kw*cin + c) and db (slot 3*cin). A block
// covers 32 outputs with 8 lanes each (lane j sums partials j, j+8, ... in
// order; the lane sums are added in a fixed tree): a fixed association
// (bitwise-identical reruns) with 8 loads in flight per output.
__global__ void __launch_bounds__(256) stem_dw_reduce(const float* __restrict__ part, int nparts, int kpad, int npad,
                                                      int cin, int cout, float* __restrict__ dw,
                                                      float* __restrict__ db) {
  __shared__ float red[8][33];
  const int o = threadIdx.x & 31, lj = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + o;
  const int nw = cout * cin * 27;
  int k = -1, co = 0;
  if (i < nw) {
    co = i / (cin * 27);
    const int r = i - co * cin * 27;
    const int c = r / 27, tap = r - c * 27;
    k = (tap / 3) * 4 * cin + (tap % 3) * cin + c;
  } else if (db != nullptr && i < nw + cout) {
    co = i - nw;
    k = 3 * cin;
  }
  float s = 0.f;
  if (k >= 0)
    for (int b = lj; b < nparts; b += 8) s += part[((size_t)b * kpad + k) * npad + co];
  red[lj][o] = s;
  __syncthreads();
  if (lj == 0 && k >= 0) {
    const float t = ((red[0][o] + red[1][o]) + (red[2][o] + red[3][o])) +
                    ((red[4][o] + red[5][o]) + (red[6][o] + red[7][o]));
    if (i < nw) dw[i] = t;
    else db[co] = t;
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

static int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cached[dev] = v;
  }
  return cached[dev];
}

static int kpad_of(int cin) { return (36 * cin + 15) / 16 * 16; }  // StemK<cin>::KPAD
static int npad_of(int cout) { return (cout + 15) / 16 * 16; }
// Columns per box-start step: the box start, in elements of the merged
// W*Cin dimension, must be a multiple of 8 (16 bytes).
static int walign_of(int cin) {
  for (int a = 1; a <= 8; ++a)
    if ((a * cin) % 8 == 0) return a;
  return 8;
}

bool supported(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw) {
  if (ks != 3 || cin < 1 || cin > 4 || cout < 1 || cout > 256) return false;
  if (n < 1 || d < 1 || h < 1 || w < 1) return false;
  if (pd < 0 || pd > 2 || ph < 0 || ph > 2 || pw < 0 || pw > 2) return false;
  const int od = d + 2 * pd - 2, oh = h + 2 * ph - 2, ow = w + 2 * pw - 2;
  if (od < 1 || oh < 1 || ow < 1) return false;
  if (((long long)w * cin) % 8 != 0) return false;  // TMA row strides are multiples of 16 bytes
  return true;
}

size_t packed_bytes(int cin, int cout) { return (size_t)npad_of(cout) * kpad_of(cin) * 2; }

struct StemPlan {
  int bw, bh, P, wb, walign, mtiles, nsets, nraw, npad, kpad, raw_bytes, a_bytes, w_bytes, smem, tmem_cols;
  long long units;
};

// Tile choice: a brick row spans the whole output width when it fits the
// TMA box (<= 256 elements of W*Cin); a unit holds up to 8 M tiles (1024
// positions), rows of the brick first, then planes.
static bool make_plan(int n, int d, int h, int w, int cin, int cout, int pd, int ph, int pw, StemPlan* sp) {
  const int od = d + 2 * pd - 2, oh = h + 2 * ph - 2, ow = w + 2 * pw - 2;
  StemPlan p{};
  p.walign = walign_of(cin);
  p.npad = npad_of(cout);
  p.kpad = kpad_of(cin);
  p.a_bytes = 128 * p.kpad * 2;
  p.w_bytes = p.npad * p.kpad * 2;
  // widest brick row whose box (with halo and alignment slack) fits 256 elements
  int bw = ow;
  auto box_w = [&](int b) { return (b + 2 + p.walign - 1 + p.walign - 1) / p.walign * p.walign; };
  while (bw > 1 && box_w(bw) * cin > 256) bw = (bw + 1) / 2;
  if (box_w(bw) * cin > 256) return false;
  p.bw = bw;
  p.wb = box_w(bw);
  // Units of mt M tiles (rows first, then planes) in a ring of nsets TMEM
  // sets / A buffers: the most sets (deepest decoupling of builders, MMA and
  // epilogue), then the most tiles per unit, that fit TMEM (512 columns) and
  // shared memory (A buffers, three raw bricks, the weight).
  p.mtiles = 0;
  for (int ns = kMaxSets; ns >= 2 && p.mtiles == 0; --ns) {
    for (int mt = std::min(8, 512 / (ns * p.npad)); mt >= 1; --mt) {
      const int cap = mt * 128;
      const int bh = std::max(1, std::min(oh, cap / bw));
      const int P = std::max(1, std::min(od, cap / (bw * bh)));
      if (P + 2 > 256 || bh + 2 > 256) continue;
      const int mtiles = (P * bh * bw + 127) / 128;
      const int raw = ((P + 2) * (bh + 2) * p.wb * cin * 2 + 1023) / 1024 * 1024;
      const int fixed = kHeader + (p.w_bytes + 1023) / 1024 * 1024 + kABufs * mtiles * p.a_bytes;
      const int nraw = std::min(kMaxRaw, (kSmemMax - fixed) / raw);
      if (mtiles > mt || nraw < 3) continue;
      p.bh = bh;
      p.P = P;
      p.mtiles = mtiles;
      p.nsets = ns;
      p.raw_bytes = raw;
      p.nraw = nraw;
      p.smem = fixed + nraw * raw;
      break;
    }
  }
  if (p.mtiles < 1) return false;
  int cols = p.nsets * p.mtiles * p.npad, alloc = 32;
  while (alloc < cols) alloc *= 2;
  p.tmem_cols = alloc;
  p.units = (long long)n * ((od + p.P - 1) / p.P) * ((oh + p.bh - 1) / p.bh) * ((ow + bw - 1) / bw);
  if (p.units >= (1ll << 31)) return false;
  *sp = p;
  return true;
}

int describe(int n, int d, int h, int w, int cin, int cout, int pd, int ph, int pw, char* buf, size_t len) {
  StemPlan p;
  if (!make_plan(n, d, h, w, cin, cout, pd, ph, pw, &p)) return snprintf(buf, len, "stem: no plan");
  return snprintf(buf, len,
                  "tcgen05 stem conv (im2col in smem): cin=%d cout=%d(npad %d) K=%d brick=%dx%dx%d (box width %d) "
                  "mtiles=%d sets=%d raw=%dBx%d a_tile=%dB smem=%dB tmem=%d units=%lld",
                  cin, cout, p.npad, p.kpad, p.P, p.bh, p.bw, p.wb, p.mtiles, p.nsets, p.raw_bytes, p.nraw, p.a_bytes,
                  p.smem,
                  p.tmem_cols, p.units);
}

// OIDHW weight (fp32/bf16/fp16) -> [npad rows][kpad] core-matrix image in
// the StemK layout: k = (kd*3 + kh)*4*cin + kw*cin + c for kw < 3; the fourth
// slot of each group, rows >= cout and k >= 36*cin are zeros.
template <typename TO>
__global__ void pack_stem_kernel(const void* __restrict__ src, int sdt, TO* __restrict__ dst, int cin, int cout,
                                 int npad, int kpad) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= npad * kpad) return;
  const int nrow = i / kpad, k = i - nrow * kpad;
  float v = 0.f;
  const int g = k / (4 * cin), r = k - g * 4 * cin;
  if (nrow < cout && g < 9 && r < 3 * cin) {
    const int tap = g * 3 + r / cin, c = r % cin;
    const long long s = ((long long)nrow * cin + c) * 27 + tap;  // tap = (kd*3+kh)*3+kw
    if (sdt == R4C_F32) v = static_cast<const float*>(src)[s];
    else if (sdt == R4C_BF16) v = __bfloat162float(static_cast<const __nv_bfloat16*>(src)[s]);
    else v = __half2float(static_cast<const __half*>(src)[s]);
  }
  const size_t off = (size_t)(nrow >> 3) * (kpad * 16) + (size_t)(k >> 3) * 128 + (nrow & 7) * 16 + (k & 7) * 2;
  *reinterpret_cast<TO*>(reinterpret_cast<uint8_t*>(dst) + off) = Elem<TO>::from_f(v);
}

cudaError_t pack_weight(int cin, int cout, const void* w_src, int src_dtype, void* w_packed, int dtype,
                        cudaStream_t st) {
  const int npad = npad_of(cout), kpad = kpad_of(cin);
  const int total = npad * kpad;
  const int blocks = (total + 255) / 256;
  if (dtype == R4C_BF16)
    pack_stem_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(w_src, src_dtype, static_cast<__nv_bfloat16*>(w_packed),
                                                            cin, cout, npad, kpad);
  else
    pack_stem_kernel<__half><<<blocks, 256, 0, st>>>(w_src, src_dtype, static_cast<__half*>(w_packed), cin, cout,
                                                     npad, kpad);
  note_launches(1);
  return cudaGetLastError();
}

template <typename T, int C>
static cudaError_t launch_typed(const StemArgs& a, int grid, int smem, cudaStream_t st) {
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      e = cudaFuncSetAttribute(stem_fwd_kernel<T, C>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
      if (e != cudaSuccess) return e;
      done[dev] = true;
    }
  }
  stem_fwd_kernel<T, C><<<grid, kThreads, smem, st>>>(a);
  return cudaGetLastError();
}

int launch_fwd(int n, int d, int h, int w, int cin, int cout, int pd, int ph, int pw, const void* x,
               const void* w_packed, const void* bias, void* y, int dtype, cudaStream_t st) {
  if (!supported(n, d, h, w, cin, cout, 3, pd, ph, pw)) return R4C_ERR_UNSUPPORTED;
  if (((uintptr_t)x & 15) || ((uintptr_t)w_packed & 15)) return R4C_ERR_ALIGN;
  StemPlan p;
  if (!make_plan(n, d, h, w, cin, cout, pd, ph, pw, &p)) return R4C_ERR_UNSUPPORTED;
  StemArgs a;
  memset(&a, 0, sizeof(a));
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return R4C_ERR_CUDA;
  const cuuint64_t e = 2;
  cuuint64_t dims[5] = {(cuuint64_t)w * cin, (cuuint64_t)h, (cuuint64_t)d, (cuuint64_t)n, 1};
  cuuint64_t str[4] = {(cuuint64_t)w * cin * e, (cuuint64_t)h * w * cin * e, (cuuint64_t)d * h * w * cin * e,
                       (cuuint64_t)n * d * h * w * cin * e};
  cuuint32_t box[5] = {(cuuint32_t)(p.wb * cin), (cuuint32_t)(p.bh + 2), (cuuint32_t)(p.P + 2), 1, 1};
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  if (enc(&a.xmap, dtype == R4C_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
          const_cast<void*>(x), dims, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return R4C_ERR_INVALID;
  a.wpack = static_cast<const uint8_t*>(w_packed);
  a.bias = bias;
  a.y = y;
  a.err = tc::device_error_flag();
  if (!a.err) return R4C_ERR_CUDA;
  a.n = n; a.d = d; a.h = h; a.w = w; a.cin = cin; a.cout = cout;
  a.od = d + 2 * pd - 2; a.oh = h + 2 * ph - 2; a.ow = w + 2 * pw - 2;
  a.pd = pd; a.ph = ph; a.pw = pw;
  a.bw = p.bw; a.bh = p.bh; a.P = p.P; a.wb = p.wb; a.walign = p.walign;
  a.nwt = (a.ow + p.bw - 1) / p.bw;
  a.nht = (a.oh + p.bh - 1) / p.bh;
  a.nzb = (a.od + p.P - 1) / p.P;
  a.units = (int)p.units;
  a.nsets = p.nsets;
  a.mtiles = p.mtiles; a.npad = p.npad; a.kpad = p.kpad; a.ksteps = p.kpad / 16;
  a.raw_bytes = p.raw_bytes;
  a.raw_tx = (p.P + 2) * (p.bh + 2) * p.wb * cin * 2;
  a.a_bytes = p.a_bytes;
  a.w_bytes = p.w_bytes;
  a.w_region = (p.w_bytes + 1023) / 1024 * 1024;
  a.abuf_bytes = p.mtiles * p.a_bytes;
  a.nraw = p.nraw;
  a.tmem_cols = p.tmem_cols;
  a.idesc = instr_desc_f16(dtype == R4C_BF16, 128, p.npad, 0, 0);
  const int grid = (int)std::min<long long>(p.units, num_sms());
  // one CTA per SM: each allocates up to all 512 TMEM columns
  p.smem = std::max(p.smem, kSmemMax / 2 + 1024);
  cudaError_t ce;
  const bool bf = dtype == R4C_BF16;
  switch (cin) {
    case 1: ce = bf ? launch_typed<__nv_bfloat16, 1>(a, grid, p.smem, st) : launch_typed<__half, 1>(a, grid, p.smem, st); break;
    case 2: ce = bf ? launch_typed<__nv_bfloat16, 2>(a, grid, p.smem, st) : launch_typed<__half, 2>(a, grid, p.smem, st); break;
    case 3: ce = bf ? launch_typed<__nv_bfloat16, 3>(a, grid, p.smem, st) : launch_typed<__half, 3>(a, grid, p.smem, st); break;
    default: ce = bf ? launch_typed<__nv_bfloat16, 4>(a, grid, p.smem, st) : launch_typed<__half, 4>(a, grid, p.smem, st); break;
  }
  note_launches(1);
  return ce == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}


// ---------------------------------------------------------------------------
// Weight gradient host side.
// ---------------------------------------------------------------------------
struct StemDwPlan {
  int bw, bh, P, wb, walign, mtiles, npad, kpad, mk;
  int raw_bytes, g_bytes, stage_bytes, nstages, a_bytes, abuf_bytes, plane_bytes, bbuf_bytes, nbufs, smem, tmem_cols;
  long long units;
};

// Units of at most two M tiles (256 positions): two A and two B buffers stay
// small enough for at least 6 input stages (raw brick + dY brick) in flight.
static bool make_dw_plan(int n, int d, int h, int w, int cin, int cout, int pd, int ph, int pw, StemDwPlan* sp) {
  if (!supported(n, d, h, w, cin, cout, 3, pd, ph, pw) || cout % 8 != 0) return false;
  const int od = d + 2 * pd - 2, oh = h + 2 * ph - 2, ow = w + 2 * pw - 2;
  StemDwPlan p{};
  p.walign = walign_of(cin);
  p.npad = npad_of(cout);
  p.kpad = kpad_of(cin);
  p.mk = (p.kpad + 127) / 128;
  if (p.mk * p.npad > 512) return false;
  p.a_bytes = 128 * p.kpad * 2;
  int bw = ow;
  auto box_w = [&](int b) { return (b + 2 + p.walign - 1 + p.walign - 1) / p.walign * p.walign; };
  while (bw > 1 && (box_w(bw) * cin > 256 || bw > 256)) bw = (bw + 1) / 2;
  if (box_w(bw) * cin > 256) return false;
  p.bw = bw;
  p.wb = box_w(bw);
  p.mtiles = 0;
  for (int mt = 2; mt >= 1 && p.mtiles == 0; --mt) {
    const int cap = mt * 128;
    const int bh = std::max(1, std::min(oh, cap / bw));
    const int P = std::max(1, std::min(od, cap / (bw * bh)));
    if (P + 2 > 256 || bh + 2 > 256) continue;
    const int mtiles = (P * bh * bw + 127) / 128;
    if (mtiles > mt) continue;
    const int raw = ((P + 2) * (bh + 2) * p.wb * cin * 2 + 1023) / 1024 * 1024;
    const int gb = (P * bh * bw * cout * 2 + 1023) / 1024 * 1024;
    const int abuf = mtiles * p.a_bytes;
    const int plane = mtiles * 128 * 16;
    const int bbuf = (p.npad / 8) * plane;
    // three buffer pairs when at least four input stages still fit, else two
    int nb = kDwMaxBufs, nst = 0;
    for (; nb >= 2; --nb) {
      nst = std::min(kDwMaxStages, (kSmemMax - kHeader - nb * (abuf + bbuf)) / (raw + gb));
      if (nst >= (nb == 2 ? 3 : 4)) break;
    }
    if (nb < 2) continue;
    const int fixed = kHeader + nb * (abuf + bbuf);
    p.bh = bh; p.P = P; p.mtiles = mtiles;
    p.raw_bytes = raw; p.g_bytes = gb; p.stage_bytes = raw + gb; p.nstages = nst;
    p.abuf_bytes = abuf; p.plane_bytes = plane; p.bbuf_bytes = bbuf; p.nbufs = nb;
    p.smem = fixed + nst * (raw + gb);
  }
  if (p.mtiles < 1) return false;
  int alloc = 32;
  while (alloc < p.mk * p.npad) alloc *= 2;
  p.tmem_cols = alloc;
  p.units = (long long)n * ((od + p.P - 1) / p.P) * ((oh + p.bh - 1) / p.bh) * ((ow + bw - 1) / bw);
  if (p.units >= (1ll << 31)) return false;
  *sp = p;
  return true;
}

bool dw_supported(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw) {
  StemDwPlan p;
  return ks == 3 && make_dw_plan(n, d, h, w, cin, cout, pd, ph, pw, &p);
}

size_t dw_workspace(int n, int d, int h, int w, int cin, int cout, int pd, int ph, int pw) {
  StemDwPlan p;
  if (!make_dw_plan(n, d, h, w, cin, cout, pd, ph, pw, &p)) return 0;
  const long long grid = std::min<long long>(p.units, 1024);  // upper bound of the CTA count
  return (size_t)grid * p.kpad * p.npad * sizeof(float);
}

int dw_describe(int n, int d, int h, int w, int cin, int cout, int pd, int ph, int pw, char* buf, size_t len) {
  StemDwPlan p;
  if (!make_dw_plan(n, d, h, w, cin, cout, pd, ph, pw, &p)) return snprintf(buf, len, "stem dW: no plan");
  return snprintf(buf, len,
                  "tcgen05 stem dW (im2col in smem, dY planes re-laid in smem): cin=%d cout=%d(npad %d) K=%d "
                  "brick=%dx%dx%d mtiles=%d stages=%d (raw %dB + dY %dB) buffers=%d smem=%dB tmem=%d units=%lld",
                  cin, cout, p.npad, p.kpad, p.P, p.bh, p.bw, p.mtiles, p.nstages, p.raw_bytes, p.g_bytes, p.nbufs,
                  p.smem,
                  p.tmem_cols, p.units);
}

template <int C>
static cudaError_t launch_dw_typed(const StemDwArgs& a, int grid, int smem, cudaStream_t st) {
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      e = cudaFuncSetAttribute(stem_dw_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
      if (e != cudaSuccess) return e;
      done[dev] = true;
    }
  }
  stem_dw_kernel<C><<<grid, kDwThreads, smem, st>>>(a);
  return cudaGetLastError();
}

int launch_dw(int n, int d, int h, int w, int cin, int cout, int pd, int ph, int pw, const void* x, const void* go,
              float* dw, float* db, void* ws, size_t ws_bytes, int dtype, cudaStream_t st) {
  StemDwPlan p;
  if (!make_dw_plan(n, d, h, w, cin, cout, pd, ph, pw, &p)) return R4C_ERR_UNSUPPORTED;
  if (((uintptr_t)x & 15) || ((uintptr_t)go & 15) || ((uintptr_t)ws & 15)) return R4C_ERR_ALIGN;
  const int grid = (int)std::min<long long>(p.units, num_sms());
  if (!ws || ws_bytes < (size_t)grid * p.kpad * p.npad * sizeof(float)) return R4C_ERR_WORKSPACE;
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return R4C_ERR_CUDA;
  StemDwArgs a;
  memset(&a, 0, sizeof(a));
  const int od = d + 2 * pd - 2, oh = h + 2 * ph - 2, ow = w + 2 * pw - 2;
  const CUtensorMapDataType dt = dtype == R4C_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint64_t e = 2;
  {
    cuuint64_t dims[5] = {(cuuint64_t)w * cin, (cuuint64_t)h, (cuuint64_t)d, (cuuint64_t)n, 1};
    cuuint64_t str[4] = {(cuuint64_t)w * cin * e, (cuuint64_t)h * w * cin * e, (cuuint64_t)d * h * w * cin * e,
                         (cuuint64_t)n * d * h * w * cin * e};
    cuuint32_t box[5] = {(cuuint32_t)(p.wb * cin), (cuuint32_t)(p.bh + 2), (cuuint32_t)(p.P + 2), 1, 1};
    cuuint32_t es[5] = {1, 1, 1, 1, 1};
    if (enc(&a.xmap, dt, 5, const_cast<void*>(x), dims, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
      return R4C_ERR_INVALID;
  }
  {
    cuuint64_t dims[5] = {(cuuint64_t)cout, (cuuint64_t)ow, (cuuint64_t)oh, (cuuint64_t)od, (cuuint64_t)n};
    cuuint64_t str[4] = {(cuuint64_t)cout * e, (cuuint64_t)ow * cout * e, (cuuint64_t)oh * ow * cout * e,
                         (cuuint64_t)od * oh * ow * cout * e};
    cuuint32_t box[5] = {(cuuint32_t)cout, (cuuint32_t)p.bw, (cuuint32_t)p.bh, (cuuint32_t)p.P, 1};
    cuuint32_t es[5] = {1, 1, 1, 1, 1};
    if (enc(&a.gmap, dt, 5, const_cast<void*>(go), dims, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
      return R4C_ERR_INVALID;
  }
  a.part = static_cast<float*>(ws);
  a.err = tc::device_error_flag();
  if (!a.err) return R4C_ERR_CUDA;
  a.n = n; a.d = d; a.h = h; a.w = w; a.cin = cin; a.cout = cout;
  a.od = od; a.oh = oh; a.ow = ow; a.pd = pd; a.ph = ph; a.pw = pw;
  a.bw = p.bw; a.bh = p.bh; a.P = p.P; a.wb = p.wb; a.walign = p.walign;
  a.nwt = (ow + p.bw - 1) / p.bw;
  a.nht = (oh + p.bh - 1) / p.bh;
  a.nzb = (od + p.P - 1) / p.P;
  a.units = (int)p.units;
  a.mtiles = p.mtiles; a.npad = p.npad; a.kpad = p.kpad; a.mk = p.mk;
  a.raw_bytes = p.raw_bytes;
  a.raw_tx = (p.P + 2) * (p.bh + 2) * p.wb * cin * 2;
  a.g_tx = p.P * p.bh * p.bw * cout * 2;
  a.stage_bytes = p.stage_bytes; a.nstages = p.nstages;
  a.a_bytes = p.a_bytes; a.abuf_bytes = p.abuf_bytes;
  a.plane_bytes = p.plane_bytes; a.bbuf_bytes = p.bbuf_bytes; a.nbufs = p.nbufs;
  a.tmem_cols = p.tmem_cols;
  a.idesc = instr_desc_f16(dtype == R4C_BF16, 128, p.npad, 1, 1);
  a.one = dtype == R4C_BF16 ? 0x3F80u : 0x3C00u;
  const int smem = std::max(p.smem, kSmemMax / 2 + 1024);  // one CTA per SM (TMEM)
  cudaError_t ce;
  switch (cin) {
    case 1: ce = launch_dw_typed<1>(a, grid, smem, st); break;
    case 2: ce = launch_dw_typed<2>(a, grid, smem, st); break;
    case 3: ce = launch_dw_typed<3>(a, grid, smem, st); break;
    default: ce = launch_dw_typed<4>(a, grid, smem, st); break;
  }
  note_launches(1);
  if (ce != cudaSuccess) return R4C_ERR_CUDA;
  const int nout = cout * cin * 27 + cout;
  stem_dw_reduce<<<(nout + 31) / 32, 256, 0, st>>>(a.part, grid, p.kpad, p.npad, cin, cout, dw, db);
  note_launches(1);
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

}  // namespace stem
}  // namespace r4c
