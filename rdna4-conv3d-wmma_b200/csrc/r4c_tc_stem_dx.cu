// r4c_tc_stem_dx.cu — tcgen05 dX of k=3, pad 1, stride 1 convs with ONE
// input channel (the stem of a 3D UNet: dX of its 1 -> Cout input conv).
//
// Run as a conv, this dX has a single output channel: N = 1 against a K loop
// of 27 taps x Cout channels, so the tensor core spends its MMAs on one useful
// column. Here the channel contraction and the tap sum are separated:
//   Z[q][t] = sum_co dY[q][co] * w[co][0][t]          (t = (kd,kh,kw), 27 taps)
//   dX[z,y,x] = sum_{kd,kh,kw} Z[z+1-kd, y+1-kh, x+1-kw][kd,kh,kw]
// Z is a GEMM with M = positions, K = Cout and N = 27; the tap sum is a
// 27-point gather that never leaves the SM.
//
// Layout of the GEMM. dY (NDHWC, Cout <= 32 channels) is read as rows of two
// x-positions: the TMA map's innermost dimension is the 2*Cout channels of the
// position pair (2j, 2j+1), boxed to 64 elements with SWIZZLE_128B (the
// elements past 2*Cout are the out-of-bounds zero fill), so one 128-byte TMA
// row carries two positions — the TMA unit's cost is per row, not per byte.
// A stage is `rs` whole image rows of one plane (rs * W/2 <= 128 pairs: one
// M tile). Per stage one thread issues three MMAs per 16-channel K step whose
// A operands are the same rows shifted by -1, 0 and +1 pair (a K-major
// swizzled operand shifts by whole rows through its start address), against
// three weight blocks, so that TMEM lane j holds what pair j's two outputs
// need:
//   D-1 (N=16):  Z_odd(j-1)[kw=2]                          (9 columns used)
//   D0  (N=64):  Z_odd(j)[kw=0], Z_even(j)[kw=1]           (columns 0..17)
//                Z_odd(j)[kw=1], Z_even(j)[kw=2]           (columns 32..49)
//   D+1 (N=16):  Z_even(j+1)[kw=0]                         (9 columns used)
// so the x-sums of the three kw taps need no exchange between lanes; at the
// ends of an image row the neighbour terms are x = -1 / x = W, i.e. zero.
// Eight gather warps (two per TMEM lane quarter: even / odd outputs) write the
// 9 (kd,kh) x-sums of every position to a four-stage shared ring; after one
// named barrier each thread adds, for its output column, the three kh rows of
// each kd into three per-plane accumulators held in registers for the rows it
// owns. A work unit is (n, a slab of Pz output planes, a strip of R output
// rows, the full width): it walks dY planes z0-1 .. z0+Pz and, inside each, the
// R+2 rows of the strip in stages; an output plane is stored as soon as its
// last contributing dY plane is done. dY outside the volume is the TMA fill
// (zeros), so every edge of the conv's zero padding comes for free.
//
// Warps: 0 TMA producer, 1 MMA issuer (TMEM owner), 2..9 gather. Waits are
// bounded (1 s); on expiry the kernel raises the library's error flag and
// every role leaves its loop (the gather warps agree through a barrier
// reduction, so none is left waiting at a named barrier).
//
// The arithmetic is the transposed conv that PyTorch's conv3d backward takes
// for dX (reference: rdna4_conv3d/conv3d_wmma.py, the dgrad launch, which runs
// the same sum as a flipped-weight forward conv), fp32 accumulation of
// bf16/fp16 products and one rounding at the end.
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

namespace {

constexpr int kDxGatherWarps = 8;
constexpr int kDxThreads = 64 + 32 * kDxGatherWarps;
constexpr int kDxHeader = 1024;
constexpr int kDxWBytes = 96 * 128;        // weight image: 96 B rows x 64 K elements
// A stage is up to two M tiles (256 rows of 128 B = 32 KB): the TMA unit's
// throughput per SM is set by the bytes of each mbarrier transaction (~0.55 us
// per transaction up to ~32 KB, whatever the ring depth), so 16 KB stages
// deliver ~4.3 TB/s over 148 SMs and 32 KB stages reach HBM speed.
constexpr int kDxStageBytes = 256 * 128;
constexpr int kDxMaxStages = 6;
constexpr int kDxTSlots = 2;               // TMEM ring: 2 stages x 2 tiles x 96 columns
constexpr int kDxTCols = 96;               // columns per M tile: D-1 (16), D0 (64), D+1 (16)
constexpr int kDxSRing = 3;                // x-sum ring (stages); a stage's outputs read it and the one before
constexpr int kDxNStg = 8;                 // max stages per plane of a unit (accumulators per plane)
constexpr int kDxSmemMax = 232448;

struct StemDxArgs {
  CUtensorMap gmap;  // dY as (2*Cout, W/2, H, D, N), box (64, W/2, rs, 1, 1), SWIZZLE_128B
  const uint8_t* wpack;
  void* dx;
  int* err;
  int n, d, h, w;
  int pairs, rs, lanes;  // pairs per image row, rows per stage, rs * pairs (<= 256)
  int mt;                // M tiles per stage (lanes / 128 rounded up)
  int R, Pz, nyt, nzt, units;
  int ksteps;            // 16-channel K steps over 2*Cout (the kernel's KS)
  int nstages;
  int s_slot_floats;     // one x-sum ring slot: rs * 9 * W floats
  int ring_off;          // byte offset of the x-sum ring
  uint32_t idesc16, idesc64;
};

__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  // K-major, 128-byte swizzle: SBO = 8 rows x 128 B, layout code 2
  return smem_desc(addr, 16u, 1024u) | ((uint64_t)2u << 61);
}

// Barrier 1 over the 256 gather threads, returning the OR of `v` over them.
__device__ __forceinline__ int gather_bar_or(int v) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.s32 q, %1, 0;\n\t"
      "bar.red.or.pred p, 1, 256, q;\n\t"
      "selp.s32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(v)
      : "memory");
  return r;
}

// 16 + 16 + 2 TMEM columns (32 lanes each) behind one wait.
__device__ __forceinline__ void tmem_ld_34(uint32_t t0, uint32_t t1, uint32_t t2, float (&v)[34]) {
  uint32_t r[34];
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
      "%13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(t0));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
      "%13, %14, %15}, [%16];"
      : "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(t1));
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(r[32]), "=r"(r[33]) : "r"(t2));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                 "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
                 "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
                 "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]),
                 "+r"(r[32]), "+r"(r[33])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 34; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace

// KS: 16-channel K steps over the 2*Cout channels of a position pair.
template <typename T, int KS>
__global__ void __launch_bounds__(kDxThreads, 1) stem_dx_kernel(const __grid_constant__ StemDxArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kDxMaxStages;
  uint64_t* tfull = empty + kDxMaxStages;
  uint64_t* tempty = tfull + kDxTSlots;
  uint64_t* wbar = tempty + kDxTSlots;
  uint64_t* mdone = wbar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* wsm = smem + kDxHeader;     // weight image (1024-aligned)
  uint8_t* st0 = wsm + kDxWBytes;      // dY stages (1024-aligned); the MMA of the -1 shift reads the
                                       // 128 bytes before a tile, the +1 shift the 128 after it
  float* sring = reinterpret_cast<float*>(smem + a.ring_off);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if ((smem_u32(smem) & 1023u) != 0u) {
    if (threadIdx.x == 0) atomicExch(a.err, 2);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kDxMaxStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kDxTSlots; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], kDxGatherWarps);
    }
    mbar_init(wbar, 1);
    mbar_init(mdone, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512u);
    tmem_relinquish();
  }
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
  // work unit u -> (batch, first output plane, first output row, planes, rows)
  auto unit_of = [&](int u, int& nb, int& z0, int& y0, int& pz, int& re) {
    const int yt = u % a.nyt;
    const int t2 = u / a.nyt;
    const int zt = t2 % a.nzt;
    nb = t2 / a.nzt;
    z0 = zt * a.Pz;
    y0 = yt * a.R;
    pz = min(a.Pz, a.d - z0);
    re = min(a.R, a.h - y0);
  };

  if (warp == 0) {
    // ---------------- TMA producer: one stage = rs dY rows of one plane ----------------
    if (lane == 0) {
      prefetch_tmap(&a.gmap);
      mbar_arrive_expect_tx(wbar, (uint32_t)kDxWBytes);
      bulk_load(wsm, a.wpack, (uint32_t)kDxWBytes, wbar);
      const uint32_t tx = (uint32_t)a.lanes * 128u;
      int s = 0;
      uint32_t epar = 1u, pending = 0u, last_par = 0u;
      bool ok = true;
      for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
        int nb, z0, y0, pz, re;
        unit_of(u, nb, z0, y0, pz, re);
        const int ns = (re + 2 + a.rs - 1) / a.rs;
        for (int p = 0; p < pz + 2 && ok; ++p) {
          for (int k = 0; k < ns; ++k) {
            if (!wait(&empty[s], epar, 32)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[s], tx);
            tma_load_5d(st0 + (size_t)s * kDxStageBytes, &a.gmap, &full[s], 0, 0, y0 - 1 + a.rs * k, z0 - 1 + p,
                        nb);
            pending |= 1u << s;
            last_par = (last_par & ~(1u << s)) | ((epar ^ 1u) << s);
            if (++s == a.nstages) {
              s = 0;
              epar ^= 1u;
            }
          }
        }
      }
      // no copy may outlive the CTA (matters only after an abort)
      const uint64_t deadline = global_timer_ns() + kWaitNs;
      mbar_wait_bounded(wbar, 0u, deadline);
      for (int i = 0; i < a.nstages; ++i)
        if ((pending >> i) & 1u) mbar_wait_bounded(&full[i], (last_par >> i) & 1u, deadline);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: per M tile, three row shifts per K step ----------------
    // The whole warp runs the loop (descriptors stay warp-uniform) and the
    // elected lane issues: ~45 clk per MMA against ~70 from a lane-0 branch.
    {
      int ok0 = 1;
      if (lane == 0) ok0 = wait(wbar, 0u) ? 1 : 0;
      bool ok = __shfl_sync(0xffffffffu, ok0, 0) != 0;
      // descriptors: the weight blocks are fixed; a tile's A descriptor moves
      // by whole 128-byte rows (+-8 in 16-byte units) and 32-byte K steps
      const uint64_t wd = sw128_desc(smem_u32(wsm));
      uint64_t bd[3][KS];
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        bd[0][kk] = wd + (uint64_t)(2 * kk);
        bd[1][kk] = wd + (uint64_t)(2048 / 16 + 2 * kk);
        bd[2][kk] = wd + (uint64_t)(10240 / 16 + 2 * kk);
      }
      const uint32_t i16 = a.idesc16, i64 = a.idesc64;
      int s = 0, ts = 0;
      uint32_t fpar = 0u, tbits = (1u << kDxTSlots) - 1u;
      for (int u = blockIdx.x; u < a.units && ok; u += gridDim.x) {
        int nb, z0, y0, pz, re;
        unit_of(u, nb, z0, y0, pz, re);
        const int nst = (pz + 2) * ((re + 2 + a.rs - 1) / a.rs);
        for (int t = 0; t < nst; ++t) {
          int okk = 1;
          if (lane == 0) okk = (wait(&full[s], fpar) && wait(&tempty[ts], (tbits >> ts) & 1u)) ? 1 : 0;
          if (!__shfl_sync(0xffffffffu, okk, 0)) {
            ok = false;
            break;
          }
          tbits ^= 1u << ts;
          tc_fence_after();
          const uint64_t ad0 = sw128_desc(smem_u32(st0 + (size_t)s * kDxStageBytes));
          for (int mi = 0; mi < a.mt; ++mi) {
            const uint64_t ad = ad0 + (uint64_t)(mi * 1024);  // 128 rows of 128 B
            const uint32_t d0 = tmem + (uint32_t)((ts * 2 + mi) * kDxTCols);
#pragma unroll
            for (int kk = 0; kk < KS; ++kk) {
              const uint32_t acc = kk ? 1u : 0u;
              mma_f16_ss_warp(d0, ad - 8u + (uint64_t)(2 * kk), bd[0][kk], i16, acc);
              mma_f16_ss_warp(d0 + 16u, ad + (uint64_t)(2 * kk), bd[1][kk], i64, acc);
              mma_f16_ss_warp(d0 + 80u, ad + (uint64_t)(8 + 2 * kk), bd[2][kk], i16, acc);
            }
          }
          mma_commit_warp(&empty[s]);
          mma_commit_warp(&tfull[ts]);
          if (++s == a.nstages) {
            s = 0;
            fpar ^= 1u;
          }
          ts ^= 1;
        }
      }
      // every MMA of this CTA completes before TMEM is released
      mma_commit_warp(mdone);
      if (lane == 0) mbar_wait_bounded(mdone, 0u, global_timer_ns() + kWaitNs);
      __syncwarp();
    }
  } else {
    // ---------------- gather warps 2..9 ----------------
    const int gt = threadIdx.x - 64;
    const int q = warp & 3;            // TMEM lane quarter this warp may read
    const int hsel = (warp - 2) >> 2;  // 0: even outputs, 1: odd outputs
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t c0 = hsel == 0 ? 0u : 80u;   // D-1 / D+1
    const uint32_t c1 = hsel == 0 ? 16u : 48u;  // D0 columns 0..15 / 32..47
    const uint32_t c2 = hsel == 0 ? 32u : 64u;  // D0 columns 16..17 / 48..49
    const int istep = 2 * a.pairs;
    // x-sum role, per M tile of the stage: pair b of the stage (TMEM lane)
    bool va[2], nbr[2];
    int wa_idx[2];
#pragma unroll
    for (int mi = 0; mi < 2; ++mi) {
      const int b = mi * 128 + q * 32 + lane;
      va[mi] = b < a.lanes;
      const int ra = va[mi] ? b / a.pairs : 0;
      const int pja = va[mi] ? b - ra * a.pairs : 0;
      // the neighbour pair's term lies inside the image row (else x = -1 or W: zero)
      nbr[mi] = hsel == 0 ? (pja > 0) : (pja < a.pairs - 1);
      wa_idx[mi] = (ra * 18 + hsel) * a.pairs + pja;  // ring index of (row, i = 0, parity, pair)
    }
    // output role: outputs gt and gt + 256 of each stage, (row, parity, pair) with the pair fastest
    bool vb[2];
    int rbo[2], xb[2], soff[2][3], rowoff[2][3];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int o = gt + 256 * j;
      const int pjb = o % a.pairs;
      const int ub = o / a.pairs;
      const int parb = ub & 1;
      const int rb = ub >> 1;
      vb[j] = rb < a.rs;
      rbo[j] = rb;
      xb[j] = 2 * pjb + parb;
#pragma unroll
      for (int kh = 0; kh < 3; ++kh) {
        // dY row of tap kh: this stage (0) or the one before (-1; rs >= 2), and its row there
        const int dr = rb - kh;
        const int so = dr >= 0 ? 0 : -1;
        soff[j][kh] = so;
        rowoff[j][kh] = (((dr - so * a.rs) * 9 + kh) * 2 + parb) * a.pairs + pjb;
      }
    }
    const int kdstep = 3 * istep;
    T* dxp = static_cast<T*>(a.dx);

    float acc[3][kDxNStg][2];
    int ts = 0, cur = 0;  // TMEM stage slot, x-sum ring slot of the current stage
    uint32_t tbits = 0u;
    bool bad = false;
    for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
      int nb, z0, y0, pz, re;
      unit_of(u, nb, z0, y0, pz, re);
      const int ns = (re + 2 + a.rs - 1) / a.rs;
#pragma unroll
      for (int k = 0; k < kDxNStg; ++k)
#pragma unroll
        for (int j = 0; j < 2; ++j) acc[0][k][j] = acc[1][k][j] = acc[2][k][j] = 0.f;
      for (int p = 0; p < pz + 2; ++p) {
#pragma unroll
        for (int k = 0; k < kDxNStg; ++k) {
          if (k < ns) {
            // every lane polls; the vote keeps the warp's TMEM loads uniform
            const int got = __all_sync(0xffffffffu, wait(&tfull[ts], (tbits >> ts) & 1u)) ? 1 : 0;
            tbits ^= 1u << ts;
            if (got) {
              tc_fence_after();
              float* sl = sring + cur * a.s_slot_floats;
#pragma unroll
              for (int mi = 0; mi < 2; ++mi) {
                if (mi >= a.mt) break;
                float v[34];
                const uint32_t tb = lane_base + (uint32_t)((ts * 2 + mi) * kDxTCols);
                tmem_ld_34(tb + c0, tb + c1, tb + c2, v);
                if (va[mi]) {
                  float* sw = sl + wa_idx[mi];
#pragma unroll
                  for (int i = 0; i < 9; ++i) sw[i * istep] = v[16 + i] + v[25 + i] + (nbr[mi] ? v[i] : 0.f);
                }
              }
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&tempty[ts]);
            }
            if (gather_bar_or(!got)) {
              bad = true;
              break;
            }
            const int prev = cur == 0 ? kDxSRing - 1 : cur - 1;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int so_ = a.rs * k - 1 + rbo[j];  // output row of the strip (1..re) this stage completes
              if (vb[j] && so_ >= 1 && so_ <= re) {
#pragma unroll
                for (int kh = 0; kh < 3; ++kh) {
                  const float* sr = sring + (soff[j][kh] ? prev : cur) * a.s_slot_floats + rowoff[j][kh];
#pragma unroll
                  for (int kd = 0; kd < 3; ++kd) acc[kd][k][j] += sr[kd * kdstep];
                }
              }
            }
            cur = cur == kDxSRing - 1 ? 0 : cur + 1;
            ts ^= 1;
          }
        }
        if (bad) break;
        // output plane p-2 of the unit has had its last dY plane
        const int o = p - 2;
        if (o >= 0 && o < pz) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            if (!vb[j]) continue;
            const long long rowbase = ((long long)(nb * a.d + z0 + o) * a.h + (y0 - 1)) * a.w + xb[j];
#pragma unroll
            for (int k = 0; k < kDxNStg; ++k) {
              const int so_ = a.rs * k - 1 + rbo[j];
              if (k < ns && so_ >= 1 && so_ <= re)
                dxp[rowbase + (long long)so_ * a.w] = Elem<T>::from_f(acc[0][k][j]);
            }
          }
        }
#pragma unroll
        for (int k = 0; k < kDxNStg; ++k)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            acc[0][k][j] = acc[1][k][j];
            acc[1][k][j] = acc[2][k][j];
            acc[2][k][j] = 0.f;
          }
      }
      if (bad) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512u);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn dx_encode_fn() {
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

int dx_num_sms() {
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

struct DxPlan {
  int pairs, rs, lanes, mt, R, Pz, nyt, nzt, ns, nstages, slot_floats, ring_off, smem;
  long long units;
};

// Stage = rs whole image rows with rs * W/2 <= 256 pairs (up to two M tiles)
// and rs >= 2, so an output row's three dY rows lie in its stage and the one
// before. Strip height R (ns = ceil((R+2)/rs) <= kDxNStg stages per plane)
// and planes per unit Pz minimise the busiest CTA's stage count, then the
// total.
bool make_dx_plan(int n, int d, int h, int w, int sms, DxPlan* out) {
  DxPlan p{};
  p.pairs = w / 2;
  p.rs = std::min(256 / p.pairs, h + 2);
  if (p.rs < 2) return false;
  p.lanes = p.rs * p.pairs;
  p.mt = (p.lanes + 127) / 128;
  long long best = -1, best_total = 0;
  for (int ns = 1; ns <= kDxNStg; ++ns) {
    const int R = std::min(h, p.rs * ns - 2);
    if (R < 1 || (ns > 1 && R <= p.rs * (ns - 1) - 2)) continue;  // no taller strip than ns - 1 stages give
    const long long nyt = (h + R - 1) / R;
    for (int pz = 1; pz <= std::min(d, 64); ++pz) {
      const long long nzt = (d + pz - 1) / pz;
      const long long units = (long long)n * nzt * nyt;
      const long long grid = std::min<long long>(units, sms);
      const long long cost = (units + grid - 1) / grid * (long long)(pz + 2) * ns;
      const long long total = units * (pz + 2) * ns;
      if (best < 0 || cost < best || (cost == best && total < best_total)) {
        best = cost;
        best_total = total;
        p.R = R;
        p.Pz = pz;
        p.ns = ns;
      }
    }
  }
  if (best < 0) return false;
  p.nyt = (h + p.R - 1) / p.R;
  p.nzt = (d + p.Pz - 1) / p.Pz;
  p.units = (long long)n * p.nzt * p.nyt;
  if (p.units >= (1ll << 31)) return false;
  p.slot_floats = p.rs * 9 * w;
  const int ring_bytes = kDxSRing * p.slot_floats * 4;
  // + 1024: the +1 row shift of a stage's last tile reads 128 bytes past it
  const int fixed = kDxHeader + kDxWBytes + 1024 + ring_bytes;
  p.nstages = std::min(kDxMaxStages, (kDxSmemMax - fixed) / kDxStageBytes);
  if (p.nstages < 2) return false;
  p.ring_off = kDxHeader + kDxWBytes + p.nstages * kDxStageBytes + 1024;
  p.smem = p.ring_off + ring_bytes;
  *out = p;
  return true;
}

// OIDHW weight [cout][1][3][3][3] -> the three B blocks (96 rows x 64 K, K-major,
// 128-byte swizzle, as the kernel's shared image at a 1024-aligned address):
//   rows  0..15  (D-1): row i < 9 = odd-position taps (kd,kh) = i, kw = 2
//   rows 16..79  (D0):  m = row-16: m < 9 odd kw0; 9..17 even kw1; 32..40 odd kw1; 41..49 even kw2
//   rows 80..95  (D+1): row 80+i, i < 9 = even-position taps, kw = 0
// K index k < Cout is the pair's even position's channel k, Cout <= k < 2 Cout
// its odd position's channel k - Cout.
template <typename TO>
__global__ void pack_stem_dx_kernel(const void* __restrict__ src, int sdt, TO* __restrict__ dst, int cout) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 96 * 64) return;
  const int nrow = i / 64, k = i % 64;
  int par = -1, kw = 0, t9 = 0;
  if (nrow < 9) {
    par = 1; kw = 2; t9 = nrow;
  } else if (nrow >= 16 && nrow < 80) {
    const int m = nrow - 16;
    if (m < 9) { par = 1; kw = 0; t9 = m; }
    else if (m < 18) { par = 0; kw = 1; t9 = m - 9; }
    else if (m >= 32 && m < 41) { par = 1; kw = 1; t9 = m - 32; }
    else if (m >= 41 && m < 50) { par = 0; kw = 2; t9 = m - 41; }
  } else if (nrow >= 80 && nrow < 89) {
    par = 0; kw = 0; t9 = nrow - 80;
  }
  float v = 0.f;
  if (par >= 0 && k >= par * cout && k < (par + 1) * cout) {
    const long long s = (long long)(k - par * cout) * 27 + t9 * 3 + kw;  // tap = (kd*3 + kh)*3 + kw
    if (sdt == R4C_F32) v = static_cast<const float*>(src)[s];
    else if (sdt == R4C_BF16) v = __bfloat162float(static_cast<const __nv_bfloat16*>(src)[s]);
    else v = __half2float(static_cast<const __half*>(src)[s]);
  }
  const size_t off =
      (size_t)(nrow >> 3) * 1024 + (size_t)(nrow & 7) * 128 + (size_t)((((k >> 3) ^ (nrow & 7)) & 7) << 4) + (k & 7) * 2;
  *reinterpret_cast<TO*>(reinterpret_cast<uint8_t*>(dst) + off) = Elem<TO>::from_f(v);
}

template <typename T, int KS>
cudaError_t dx_launch_typed(const StemDxArgs& a, int grid, int smem, cudaStream_t st) {
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      e = cudaFuncSetAttribute(stem_dx_kernel<T, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDxSmemMax);
      if (e != cudaSuccess) return e;
      done[dev] = true;
    }
  }
  stem_dx_kernel<T, KS><<<grid, kDxThreads, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

bool dx_supported(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw) {
  if (ks != 3 || cin != 1 || pd != 1 || ph != 1 || pw != 1) return false;
  // the pair dimension's stride (4 * Cout bytes) must be a multiple of 16
  if (cout < 4 || cout > 32 || cout % 4 != 0) return false;
  if (n < 1 || d < 1 || h < 1 || w < 2 || w % 2 != 0 || w > 256) return false;
  DxPlan p;
  return make_dx_plan(n, d, h, w, 148, &p);
}

size_t dx_packed_bytes() { return (size_t)kDxWBytes; }

int dx_describe(int n, int d, int h, int w, int cout, char* buf, size_t len) {
  DxPlan p;
  if (!make_dx_plan(n, d, h, w, 148, &p)) return snprintf(buf, len, "stem dX: no plan");
  return snprintf(buf, len,
                  "tcgen05 stem dX (Z = dY.W^T per position pair, 27-point gather in smem): cout=%d pairs/row=%d "
                  "rows/stage=%d mtiles/stage=%d strip=%d planes/unit=%d stages/plane=%d ring=%d smem=%dB units=%lld",
                  cout, p.pairs, p.rs, p.mt, p.R, p.Pz, p.ns, p.nstages, p.smem, p.units);
}

cudaError_t dx_pack_weight(int cout, const void* w_src, int src_dtype, void* w_packed, int dtype, cudaStream_t st) {
  const int blocks = (96 * 64 + 255) / 256;
  if (dtype == R4C_BF16)
    pack_stem_dx_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(w_src, src_dtype,
                                                               static_cast<__nv_bfloat16*>(w_packed), cout);
  else
    pack_stem_dx_kernel<__half><<<blocks, 256, 0, st>>>(w_src, src_dtype, static_cast<__half*>(w_packed), cout);
  note_launches(1);
  return cudaGetLastError();
}

int launch_dx(int n, int d, int h, int w, int cout, const void* go, const void* w_packed, void* dx, int dtype,
              cudaStream_t st) {
  if (!dx_supported(n, d, h, w, 1, cout, 3, 1, 1, 1)) return R4C_ERR_UNSUPPORTED;
  if (((uintptr_t)go & 15) || ((uintptr_t)w_packed & 15)) return R4C_ERR_ALIGN;
  DxPlan p;
  if (!make_dx_plan(n, d, h, w, dx_num_sms(), &p)) return R4C_ERR_UNSUPPORTED;
  StemDxArgs a;
  memset(&a, 0, sizeof(a));
  EncodeTiledFn enc = dx_encode_fn();
  if (!enc) return R4C_ERR_CUDA;
  const cuuint64_t e = 2;
  cuuint64_t dims[5] = {(cuuint64_t)2 * cout, (cuuint64_t)w / 2, (cuuint64_t)h, (cuuint64_t)d, (cuuint64_t)n};
  cuuint64_t str[4] = {(cuuint64_t)2 * cout * e, (cuuint64_t)w * cout * e, (cuuint64_t)h * w * cout * e,
                       (cuuint64_t)d * h * w * cout * e};
  cuuint32_t box[5] = {64, (cuuint32_t)p.pairs, (cuuint32_t)p.rs, 1, 1};
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  if (enc(&a.gmap, dtype == R4C_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
          const_cast<void*>(go), dims, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return R4C_ERR_INVALID;
  a.wpack = static_cast<const uint8_t*>(w_packed);
  a.dx = dx;
  a.err = tc::device_error_flag();
  if (!a.err) return R4C_ERR_CUDA;
  a.n = n; a.d = d; a.h = h; a.w = w;
  a.pairs = p.pairs; a.rs = p.rs; a.lanes = p.lanes; a.mt = p.mt;
  a.R = p.R; a.Pz = p.Pz; a.nyt = p.nyt; a.nzt = p.nzt; a.units = (int)p.units;
  a.ksteps = (2 * cout + 15) / 16;
  a.nstages = p.nstages;
  a.s_slot_floats = p.slot_floats;
  a.ring_off = p.ring_off;
  a.idesc16 = instr_desc_f16(dtype == R4C_BF16, 128, 16, 0, 0);
  a.idesc64 = instr_desc_f16(dtype == R4C_BF16, 128, 64, 0, 0);
  const int grid = (int)std::min<long long>(p.units, dx_num_sms());
  const bool bf = dtype == R4C_BF16;
  cudaError_t ce;
  switch (a.ksteps) {
    case 1: ce = bf ? dx_launch_typed<__nv_bfloat16, 1>(a, grid, p.smem, st) : dx_launch_typed<__half, 1>(a, grid, p.smem, st); break;
    case 2: ce = bf ? dx_launch_typed<__nv_bfloat16, 2>(a, grid, p.smem, st) : dx_launch_typed<__half, 2>(a, grid, p.smem, st); break;
    case 3: ce = bf ? dx_launch_typed<__nv_bfloat16, 3>(a, grid, p.smem, st) : dx_launch_typed<__half, 3>(a, grid, p.smem, st); break;
    default: ce = bf ? dx_launch_typed<__nv_bfloat16, 4>(a, grid, p.smem, st) : dx_launch_typed<__half, 4>(a, grid, p.smem, st); break;
  }
  note_launches(1);
  return ce == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

}  // namespace stem
}  // namespace r4c
