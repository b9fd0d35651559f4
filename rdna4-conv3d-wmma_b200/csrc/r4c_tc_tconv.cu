// r4c_tc_tconv.cu — tcgen05 ConvTranspose3d k=2 s=2 p=0: forward and dX.
//
// With stride = kernel = 2 the eight taps never overlap, so both legs are
// plain GEMMs over the INPUT positions v = (n, z, y, x):
//   forward  Y8[v][(a,b,c,co)] = sum_ci X[v][ci] * W[ci][co][a][b][c] (+ b[co])
//            y[n, 2z+a, 2y+b, 2x+c, co] = Y8[v][(a,b,c,co)]
//   dX       dX[v][ci] = sum_{a,b,c,co} dY[n, 2z+a, 2y+b, 2x+c, co] * W[ci][co][a][b][c]
// (reference: rdna4_conv3d/conv3d_wmma.py, the k2s2 transpose kernels, which
// compute the same sums as one GEMM with a 2x2x2 scatter / gather.)
//
// An M tile is 128 input positions: R whole input rows of W <= 128 positions
// (R = 128 / W), or a 128-wide x segment of one row. Its A operand is a list
// of TMA boxes of 64 channels (128-byte rows, SWIZZLE_128B, K-major; channels
// past the tensor's extent are the out-of-bounds zero fill):
//   forward  x viewed as (Cin, W, H, D, N): one box per 64-channel group;
//   dX       dY viewed as (2*Cout, W, 2, H, 2D*N) — a dY row (2y+b) of plane
//            (2z+a) holds, for input column x, the 2*Cout elements (c, co) of
//            output columns 2x, 2x+1 — one box per (a, b) and 64-element
//            group of (c, co): the 2x2x2 gather is four box coordinates.
// K steps of 16 run over each box's real channels. B (the weights, K-major,
// the same swizzle) stays resident in shared memory for the CTA's task = a
// range of N columns small enough to fit; boxes of a tile are grouped into
// stages of up to ~64 KB (TMA moves one stage per mbarrier transaction, and
// its throughput per SM is set by the bytes per transaction).
// The forward epilogue adds the bias and writes each (a, b, c) block of Cout
// channels of a position as 16-byte stores at a linear offset from the output
// position (2z, 2y, 2x); the dX epilogue writes the Cin (task) channels of the
// position.
//
// Warps: 0 TMA producer, 1 MMA issuer (whole warp, elected lane; TMEM owner),
// 2..9 epilogue (two per TMEM lane quarter, halves of the columns). Two TMEM
// accumulator buffers. Waits are bounded (1 s): on expiry the kernel raises
// the library's error flag and every role leaves its loop.
#include <cuda.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "r4c_internal.h"
#include "r4c_sm100.cuh"

namespace r4c {
namespace tconv {

using namespace sm100;

namespace {

constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kHeader = 4096;           // barriers + column tables
constexpr int kMaxBoxes = 12;           // A boxes per tile (dX: 4 (a,b) x 3 groups)
constexpr int kMaxStages = 8;
constexpr int kBoxBytes = 128 * 128;    // 128 rows of 128 bytes
constexpr int kBMax = 100 * 1024;       // resident B per task
constexpr int kMaxCols = 256;           // MMA N per task
constexpr int kSmemMax = 232448;

struct TArgs {
  CUtensorMap amap;     // forward: x (Cin, W, H, D, N); dX: dY (2*Cout, W, 2, H, 2D*N)
  const uint8_t* bimg;  // per task, b_bytes each
  const void* bias;     // forward only, nullable
  void* out;
  int* err;
  int mode;             // 0 forward, 1 dX
  int n, d, h, w, cin, cout;
  int wt, R, nwt, nyb;  // tile: R rows x wt columns; x segments per row; row blocks
  long long tiles;      // per task
  int nbox, box_c0[kMaxBoxes], box_ab[kMaxBoxes], box_ks[kMaxBoxes];
  int bpst, spt;        // boxes per stage, stages per tile
  int nstages;
  int ntask, ncol;      // tasks; N columns per task (multiple of 16)
  int ncol_real;        // N columns in total (8*Cout or Cin)
  int b_bytes;
  int tmem_cols;
  uint32_t idesc;
  // forward TMA-store epilogue (stg_blk > 0): the output viewed as
  // (Cout, 2W, 2, H, 2D*N) with the voxel pitch ypitch; a tile's (a, b) block
  // of 2*Cout columns is staged as [positions][2*Cout] (stg_blk bytes per
  // block, two buffers) and written by one box (Cout, 2*wt, 1, R, 1)
  CUtensorMap ymap;
  int stg_blk;
  int ypitch;  // forward: elements between consecutive output voxels (>= cout)
};

// Barrier 1 over the 256 epilogue threads, returning the OR of `v` over them.
__device__ __forceinline__ int epi_bar_or(int v) {
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
__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  // K-major, 128-byte swizzle: SBO = 8 rows x 128 B, layout code 2
  return smem_desc(addr, 16u, 1024u) | ((uint64_t)2u << 61);
}

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) tconv_kernel(const __grid_constant__ TArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* wbar = tempty + 2;
  uint64_t* mdone = wbar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  long long* coloff = reinterpret_cast<long long*>(smem + 512);  // forward: per 8-column group
  float* bias_col = reinterpret_cast<float*>(smem + 1024);       // forward: per column
  uint8_t* bsm = smem + kHeader;
  uint8_t* st0 = bsm + ((a.b_bytes + 1023) / 1024) * 1024;
  const int stage_bytes = a.bpst * kBoxBytes;
  uint8_t* stg0 = st0 + (size_t)a.nstages * stage_bytes;  // forward store staging (two buffers)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if ((smem_u32(smem) & 1023u) != 0u || a.tmem_cols > 512) {
    if (threadIdx.x == 0) atomicExch(a.err, 2);
    return;
  }
  const int cpt = max(1, (int)gridDim.x / a.ntask);  // CTAs per task
  const int task = (int)blockIdx.x / cpt;
  const int sub = (int)blockIdx.x - task * cpt;
  if (task >= a.ntask) return;  // whole CTA: no barrier or TMEM touched yet

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMaxStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], kEpiWarps);
    }
    mbar_init(wbar, 1);
    mbar_init(mdone, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (a.mode == 0) {
    // column tables of this task: output offset of each 8-column group from
    // the position (2z, 2y, 2x), and the bias of each column
    const long long sa = 4ll * a.h * a.w * a.ypitch, sb = 2ll * a.w * a.ypitch;
    for (int i = threadIdx.x; i < a.ncol; i += kThreads) {
      const int gcol = task * a.ncol + i;
      float bv = 0.f;
      long long off = 0;
      if (gcol < a.ncol_real) {
        const int abc = gcol / a.cout, co = gcol - abc * a.cout;
        off = (abc >> 2) * sa + ((abc >> 1) & 1) * sb + (long long)(abc & 1) * a.ypitch + co;
        if (a.bias) bv = Elem<T>::to_f(static_cast<const T*>(a.bias)[co]);
      }
      bias_col[i] = bv;
      if ((i & 7) == 0) coloff[i >> 3] = off;
    }
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
  // tile t -> (batch, input plane, first row, first column)
  auto tile_of = [&](long long t, int& nb, int& z, int& y0, int& x0) {
    const int xs = (int)(t % a.nwt);
    long long r = t / a.nwt;
    const int yb = (int)(r % a.nyb);
    r /= a.nyb;
    z = (int)(r % a.d);
    nb = (int)(r / a.d);
    y0 = yb * a.R;
    x0 = xs * a.wt;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&a.amap);
      {
        // this task's weight image, in chunks of at most 32 KB
        mbar_arrive_expect_tx(wbar, (uint32_t)a.b_bytes);
        const uint8_t* src = a.bimg + (size_t)task * a.b_bytes;
        for (int off = 0; off < a.b_bytes; off += 32768)
          bulk_load(bsm + off, src + off, (uint32_t)min(32768, a.b_bytes - off), wbar);
      }
      const uint32_t box_tx = (uint32_t)(128 * a.R * a.wt);
      int s = 0;
      uint32_t epar = 1u, pending = 0u, last_par = 0u;
      bool ok = true;
      for (long long t = sub; t < a.tiles && ok; t += cpt) {
        int nb, z, y0, x0;
        tile_of(t, nb, z, y0, x0);
        for (int st = 0; st < a.spt; ++st) {
          const int j0 = st * a.bpst, j1 = min(a.nbox, j0 + a.bpst);
          if (!wait(&empty[s], epar, 32)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], box_tx * (uint32_t)(j1 - j0));
          uint8_t* dst = st0 + (size_t)s * stage_bytes;
          for (int j = j0; j < j1; ++j) {
            if (a.mode == 0) {
              tma_load_5d(dst + (size_t)(j - j0) * kBoxBytes, &a.amap, &full[s], a.box_c0[j], x0, y0, z, nb);
            } else {
              const int ab = a.box_ab[j];
              tma_load_5d(dst + (size_t)(j - j0) * kBoxBytes, &a.amap, &full[s], a.box_c0[j], x0, ab & 1, y0,
                          nb * 2 * a.d + 2 * z + (ab >> 1));
            }
          }
          pending |= 1u << s;
          last_par = (last_par & ~(1u << s)) | ((epar ^ 1u) << s);
          if (++s == a.nstages) {
            s = 0;
            epar ^= 1u;
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
    // ---------------- MMA issuer (whole warp; the elected lane issues) ----------------
    int ok0 = 1;
    if (lane == 0) ok0 = wait(wbar, 0u) ? 1 : 0;
    bool ok = __shfl_sync(0xffffffffu, ok0, 0) != 0;
    const uint32_t bbase = smem_u32(bsm);
    const uint32_t breg = (uint32_t)a.ncol * 128u;  // one box's B region
    int s = 0, buf = 0;
    uint32_t fpar = 0u, tbits = 3u;
    for (long long t = sub; t < a.tiles && ok; t += cpt) {
      int okk = 1;
      if (lane == 0) okk = wait(&tempty[buf], (tbits >> buf) & 1u) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, okk, 0)) break;
      tbits ^= 1u << buf;
      const uint32_t d0 = tmem + (uint32_t)(buf * a.ncol);
      uint32_t acc = 0u;
      for (int st = 0; st < a.spt; ++st) {
        const int j0 = st * a.bpst, j1 = min(a.nbox, j0 + a.bpst);
        if (lane == 0) okk = wait(&full[s], fpar) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, okk, 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(st0 + (size_t)s * stage_bytes);
        for (int j = j0; j < j1; ++j) {
          const uint64_t ad = sw128_desc(sa + (uint32_t)(j - j0) * kBoxBytes);
          const uint64_t bd = sw128_desc(bbase + (uint32_t)j * breg);
          const int ks = a.box_ks[j];
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            if (kk < ks) {
              mma_f16_ss_warp(d0, ad + (uint64_t)(2 * kk), bd + (uint64_t)(2 * kk), a.idesc, acc);
              acc = 1u;
            }
          }
        }
        mma_commit_warp(&empty[s]);
        if (++s == a.nstages) {
          s = 0;
          fpar ^= 1u;
        }
      }
      if (!ok) break;
      mma_commit_warp(&tfull[buf]);
      buf ^= 1;
    }
    // every MMA of this CTA completes before TMEM is released
    mma_commit_warp(mdone);
    if (lane == 0) mbar_wait_bounded(mdone, 0u, global_timer_ns() + kWaitNs);
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    if (a.stg_blk > 0) {
      // forward through staging tiles and TMA stores: each (a, b) block of the
      // tile is one contiguous [positions][2*Cout] box (full sectors written
      // once, instead of 16-byte stores strided by 2*Cout per position)
      const int q = warp & 3, half = (warp - 2) >> 2;
      const int l = q * 32 + lane;
      const int lanes = a.R * a.wt;
      const int c2 = 2 * a.cout;
      const int nblk = a.ncol / c2;
      const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
      const bool issuer = warp == 2 && lane == 0;
      const int ngrp = a.ncol / 16;
      int buf = 0, sb = 0;
      uint32_t tbits = 0u;
      for (long long t = sub; t < a.tiles; t += cpt) {
        int nb, z, y0, x0;
        tile_of(t, nb, z, y0, x0);
        int got = 1;
        if (lane == 0) got = wait(&tfull[buf], (tbits >> buf) & 1u, 64) ? 1 : 0;
        got = __shfl_sync(0xffffffffu, got, 0);
        // staging buffer sb was read by the stores of two tiles ago: at most
        // the previous tile's group may still be reading
        if (issuer) bulk_wait_read<1>();
        if (epi_bar_or(!got)) break;
        tbits ^= 1u << buf;
        tc_fence_after();
        uint8_t* stg = stg0 + (size_t)sb * nblk * a.stg_blk;
        for (int g = half; g < ngrp; g += 2) {
          float v[16];
          tmem_ld_16(lane_base + (uint32_t)(buf * a.ncol + g * 16), v);
          if (l >= lanes) continue;
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int col = g * 16 + e * 8;
            const int j = col / c2, eo = col - j * c2;
            const float* vv = v + 8 * e;
            const float* bc = bias_col + col;
            *reinterpret_cast<uint4*>(stg + (size_t)j * a.stg_blk + ((size_t)l * c2 + eo) * 2) =
                make_uint4(pack2<T>(vv[0] + bc[0], vv[1] + bc[1]), pack2<T>(vv[2] + bc[2], vv[3] + bc[3]),
                           pack2<T>(vv[4] + bc[4], vv[5] + bc[5]), pack2<T>(vv[6] + bc[6], vv[7] + bc[7]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
        fence_proxy_async_smem();  // staging writes -> visible to the TMA unit
        epi_bar_sync();
        if (issuer) {
          for (int j = 0; j < nblk; ++j) {
            const int ab = task * nblk + j;
            tma_store_5d(&a.ymap, stg + (size_t)j * a.stg_blk, 0, 2 * x0, ab & 1, y0,
                         nb * 2 * a.d + 2 * z + (ab >> 1));
          }
          bulk_commit_group();
        }
        buf ^= 1;
        sb ^= 1;
      }
      if (issuer) bulk_wait<0>();
    } else {
    const int q = warp & 3;             // TMEM lane quarter this warp may read
    const int half = (warp - 2) >> 2;   // 16-column groups half, half + 2, ...
    const int l = q * 32 + lane;        // tile row = position of the tile
    const int rr = l / a.wt, xx = l - rr * a.wt;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    T* out = static_cast<T*>(a.out);
    const int ngrp = a.ncol / 16;
    int buf = 0;
    uint32_t tbits = 0u;
    for (long long t = sub; t < a.tiles; t += cpt) {
      int nb, z, y0, x0;
      tile_of(t, nb, z, y0, x0);
      const int y = y0 + rr, x = x0 + xx;
      const bool valid = rr < a.R && y < a.h && x < a.w;
      int got = 1;
      if (lane == 0) got = wait(&tfull[buf], (tbits >> buf) & 1u, 64) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, got, 0)) break;
      tbits ^= 1u << buf;
      tc_fence_after();
      // output base of this position (elements)
      long long base;
      if (a.mode == 0)
        base = ((((long long)nb * 2 * a.d + 2 * z) * 2 * a.h + 2 * y) * 2 * a.w + 2 * x) * a.ypitch;
      else
        base = ((((long long)nb * a.d + z) * a.h + y) * a.w + x) * a.cin + (long long)task * a.ncol;
      for (int g = half; g < ngrp; g += 2) {
        float v[16];
        tmem_ld_16(lane_base + (uint32_t)(buf * a.ncol + g * 16), v);
        if (!valid) continue;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int col = g * 16 + e * 8;
          if (task * a.ncol + col >= a.ncol_real) continue;
          const float* vv = v + 8 * e;
          uint4 pk;
          if (a.mode == 0) {
            const float* bc = bias_col + col;
            pk = make_uint4(pack2<T>(vv[0] + bc[0], vv[1] + bc[1]), pack2<T>(vv[2] + bc[2], vv[3] + bc[3]),
                            pack2<T>(vv[4] + bc[4], vv[5] + bc[5]), pack2<T>(vv[6] + bc[6], vv[7] + bc[7]));
            *reinterpret_cast<uint4*>(out + base + coloff[col >> 3]) = pk;
          } else {
            pk = make_uint4(pack2<T>(vv[0], vv[1]), pack2<T>(vv[2], vv[3]), pack2<T>(vv[4], vv[5]),
                            pack2<T>(vv[6], vv[7]));
            *reinterpret_cast<uint4*>(out + base + col) = pk;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      buf ^= 1;
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

// ---------------------------------------------------------------------------
// dW: D[ci][(a,b,c,co)] += sum_v X[v][ci] * dY[n, 2z+a, 2y+b, 2x+c, co]
// over K = input positions, both operands MN-major from the same TMA boxes as
// above (64 positions per K tile: an x box gives 64 ci of each position, a dY
// box 64 elements (c, co) of one (a, b)): M = 128 ci (two x boxes; channels
// past Cin are the zero fill), N = the task's (a, b) pairs x 64-element
// groups. Split-K over positions, one fp32 partial per CTA, summed in split
// order by tconv_dw_reduce (deterministic).
// ---------------------------------------------------------------------------
namespace {

constexpr int kDwBox = 64 * 128;  // 64 positions x 128 bytes

struct DwTArgs {
  CUtensorMap xmap;  // x (Cin, W, H, D, N), box (64, wt, R, 1, 1)
  CUtensorMap gmap;  // dY (2*Cout, W, 2, H, 2D*N), box (64, wt, 1, R, 1)
  float* part;       // [task][S][128][ncol]
  int* err;
  int n, d, h, w, cin, cout;
  int wt, R, nwt, nyb;
  long long tiles;   // K tiles of 64 positions
  int S, ntask, nabg, nab, ngb, ncol, nmma, mma_n;
  int nbox;          // boxes per stage: 2 (x) + nab * ngb (dY)
  // db wanted and the last M tile (ones_mt) holds at most 64 channels: its
  // tasks do not load the second x box (channels 64..127 of the tile, all
  // zero fill); each stage holds instead a constant box whose channel 64 is
  // 1 at every position, so D row 64 of those tasks is the sum of dY (db)
  int ones, ones_mt;
  // db wanted and that tile holds 72..120 channels (a multiple of 8): the
  // MMA warp writes, once a stage's boxes have landed, a 1 into channel
  // ones_row of every position (the first chunk of the second x box's zero
  // fill), so D row ones_row of those tasks is the sum of dY (db)
  int ones_fill, ones_row;
  uint32_t one_bits;  // 1.0 in the element type
  int nstages;
  int tmem_cols;
  uint32_t idesc;
};

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) tconv_dw_kernel(const __grid_constant__ DwTArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  uint64_t* mdone = empty + kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* st0 = smem + kHeader;
  const int stage_bytes = a.nbox * kDwBox;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if ((smem_u32(smem) & 1023u) != 0u || a.tmem_cols > 512) {
    if (threadIdx.x == 0) atomicExch(a.err, 2);
    return;
  }
  const int task = (int)blockIdx.x / a.S;
  const int split = (int)blockIdx.x - task * a.S;
  const int mt = task / a.nabg, abg = task - mt * a.nabg;
  const long long t0 = a.tiles * split / a.S, t1 = a.tiles * (split + 1) / a.S;
  const bool ones = a.ones && mt == a.ones_mt;
  const bool fill = a.ones_fill && mt == a.ones_mt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMaxStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(mdone, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, (uint32_t)a.tmem_cols);
    tmem_relinquish();
  }
  if (ones) {
    // the constant ones box of every stage, in the 128-byte swizzled layout
    // of a TMA box: chunk 0 (channels 64..71) of row p sits at chunk p % 8
    for (int i = threadIdx.x; i < a.nstages * (kDwBox / 16); i += kThreads) {
      const int s = i / (kDwBox / 16), k = i - s * (kDwBox / 16);
      const int p = k >> 3, c = k & 7;
      *reinterpret_cast<uint4*>(st0 + (size_t)s * stage_bytes + kDwBox + (size_t)k * 16) =
          make_uint4(c == (p & 7) ? a.one_bits : 0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();  // generic writes -> visible to the tensor core
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

  if (warp == 0) {
    // ---------------- TMA producer: per K tile, 2 x boxes + the task's dY boxes ----------------
    if (lane == 0) {
      prefetch_tmap(&a.xmap);
      prefetch_tmap(&a.gmap);
      const uint32_t tx = (uint32_t)((a.nbox - (ones ? 1 : 0)) * 128 * a.R * a.wt);
      int s = 0;
      uint32_t epar = 1u, pending = 0u, last_par = 0u;
      for (long long t = t0; t < t1; ++t) {
        const int xs = (int)(t % a.nwt);
        long long r = t / a.nwt;
        const int yb = (int)(r % a.nyb);
        r /= a.nyb;
        const int z = (int)(r % a.d), nb = (int)(r / a.d);
        const int x0 = xs * a.wt, y0 = yb * a.R;
        if (!wait(&empty[s], epar, 32)) break;
        mbar_arrive_expect_tx(&full[s], tx);
        uint8_t* dst = st0 + (size_t)s * stage_bytes;
        tma_load_5d(dst, &a.xmap, &full[s], 128 * mt, x0, y0, z, nb);
        if (!ones) tma_load_5d(dst + kDwBox, &a.xmap, &full[s], 128 * mt + 64, x0, y0, z, nb);
        int j = 2;
        for (int ab = abg * a.nab; ab < (abg + 1) * a.nab; ++ab)
          for (int g = 0; g < a.ngb; ++g, ++j)
            tma_load_5d(dst + (size_t)j * kDwBox, &a.gmap, &full[s], 64 * g, x0, ab & 1, y0,
                        nb * 2 * a.d + 2 * z + (ab >> 1));
        pending |= 1u << s;
        last_par = (last_par & ~(1u << s)) | ((epar ^ 1u) << s);
        if (++s == a.nstages) {
          s = 0;
          epar ^= 1u;
        }
      }
      const uint64_t deadline = global_timer_ns() + kWaitNs;
      for (int i = 0; i < a.nstages; ++i)
        if ((pending >> i) & 1u) mbar_wait_bounded(&full[i], (last_par >> i) & 1u, deadline);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (whole warp; the elected lane issues) ----------------
    // MN-major, 128-byte swizzle: LBO = the next 64-element MN atom (the
    // next box), SBO = the next 8 positions (1024 B); a K step of 16
    // positions moves the start by 2048 B (128 units of 16 B)
    auto mn_desc = [](uint32_t addr) {
      return smem_desc(addr, (uint32_t)kDwBox, 1024u) | ((uint64_t)2u << 61);
    };
    int s = 0;
    uint32_t fpar = 0u, acc = 0u;
    for (long long t = t0; t < t1; ++t) {
      int okk = 1;
      if (lane == 0) okk = wait(&full[s], fpar) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, okk, 0)) break;
      tc_fence_after();
      if (fill) {
        // generic stores into the zero fill, made visible to the tensor core
        uint8_t* b2 = st0 + (size_t)s * stage_bytes + kDwBox;
        const int ch = (a.ones_row - 64) >> 3;
        for (int p = lane; p < 64; p += 32)
          *reinterpret_cast<uint4*>(b2 + p * 128 + ((ch ^ (p & 7)) << 4)) = make_uint4(a.one_bits, 0u, 0u, 0u);
        fence_proxy_async_smem();
        __syncwarp();
      }
      const uint32_t sa = smem_u32(st0 + (size_t)s * stage_bytes);
      const uint64_t ad = mn_desc(sa);
      const uint64_t bd = mn_desc(sa + 2u * kDwBox);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        for (int m = 0; m < a.nmma; ++m)
          mma_f16_ss_warp(tmem + (uint32_t)(m * a.mma_n), ad + (uint64_t)(128 * kk),
                          bd + (uint64_t)(128 * kk) + (uint64_t)(m * (a.mma_n / 64) * (kDwBox / 16)), a.idesc,
                          acc);
        acc = 1u;
      }
      mma_commit_warp(&empty[s]);
      if (++s == a.nstages) {
        s = 0;
        fpar ^= 1u;
      }
    }
    mma_commit_warp(mdone);
  } else {
    // ---------------- epilogue (warps 2..9): TMEM -> fp32 partial ----------------
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    int got = 1;
    if (lane == 0) got = wait(mdone, 0u, 256) ? 1 : 0;
    got = __shfl_sync(0xffffffffu, got, 0);
    if (got) {
      tc_fence_after();
      float* dst = a.part + (((size_t)task * a.S + split) * 128 + row) * a.ncol;
      const bool any = t1 > t0;  // an empty split writes zeros
      for (int g = half; g < a.ncol / 16; g += 2) {
        float v[16];
        tmem_ld_16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(g * 16), v);
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(dst + g * 16 + i) =
              any ? make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) mbar_wait_bounded(mdone, 0u, global_timer_ns() + kWaitNs);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)a.tmem_cols);
  }
}

// db[co] from the ones row of the partials of the M tile mt: a block
// covers 32 outputs with 8 lanes each; lane j adds, over (a, b, c) in order,
// splits j, j+8, ...; the lane sums are added in a fixed tree (deterministic).
__global__ void __launch_bounds__(256) tconv_db_reduce(const float* __restrict__ part, float* __restrict__ db,
                                                       int cout, int S, int mt, int row, int nabg, int nab,
                                                       int ngb, int ncol) {
  __shared__ float red[8][33];
  const int o = threadIdx.x & 31, lj = threadIdx.x >> 5;
  const int co = blockIdx.x * 32 + o;
  float acc = 0.f;
  if (co < cout) {
    for (int ab = 0; ab < 4; ++ab)
      for (int c = 0; c < 2; ++c) {
        const float* p = part + ((size_t)(mt * nabg + ab / nab) * S * 128 + row) * ncol + (ab % nab) * ngb * 64 + c * cout + co;
#pragma unroll 4
        for (int s = lj; s < S; s += 8) acc += p[(size_t)s * 128 * ncol];
      }
  }
  red[lj][o] = acc;
  __syncthreads();
  if (lj == 0 && co < cout)
    db[co] = ((red[0][o] + red[1][o]) + (red[2][o] + red[3][o])) + ((red[4][o] + red[5][o]) + (red[6][o] + red[7][o]));
}

// dw[ci][co][a][b][c] (fp32, PyTorch ConvTranspose3d layout) = sum over the
// splits, in split order, of the partials.
__global__ void tconv_dw_reduce(const float* __restrict__ part, float* __restrict__ dw, int cin, int cout, int S,
                                int nabg, int nab, int ngb, int ncol) {
  const long long total = (long long)cin * cout * 8;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int tap = (int)(i % 8);
  const long long r = i / 8;
  const int co = (int)(r % cout), ci = (int)(r / cout);
  const int ab = tap >> 1, c = tap & 1;
  const int task = (ci >> 7) * nabg + ab / nab;
  const int col = (ab % nab) * ngb * 64 + c * cout + co;
  const float* p = part + ((size_t)task * S * 128 + (ci & 127)) * ncol + col;
  float acc = 0.f;
  // in split order, eight loads in flight
#pragma unroll 8
  for (int s = 0; s < S; ++s) acc += p[(size_t)s * 128 * ncol];
  dw[i] = acc;
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

int sm_count() {
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

struct TPlan {
  int wt, R, nwt, nyb;
  long long tiles;
  int nbox, box_c0[kMaxBoxes], box_ab[kMaxBoxes], box_ks[kMaxBoxes];
  int bpst, spt, nstages, ntask, ncol, ncol_real, b_bytes, tmem_cols, smem;
  int stg_blk;  // forward TMA-store staging per (a, b) block (0: per-thread stores)
};

// mode 0: forward (A = x, N = 8*Cout), 1: dX (A = dY gathered per (a, b), N = Cin).
bool make_plan(int mode, int n, int d, int h, int w, int cin, int cout, TPlan* out) {
  if (n < 1 || d < 1 || h < 1 || w < 1) return false;
  // 16-byte TMA strides and 16-byte epilogue stores
  if (cin % 8 || cout % 8 || cin < 8 || cout < 8) return false;
  TPlan p{};
  const int ca = mode == 0 ? cin : 2 * cout;  // A channels per box set
  const int groups = (ca + 63) / 64;
  p.nbox = mode == 0 ? groups : 4 * groups;
  if (p.nbox > kMaxBoxes) return false;
  for (int j = 0; j < p.nbox; ++j) {
    const int g = j % groups;
    p.box_c0[j] = 64 * g;
    p.box_ab[j] = mode == 0 ? 0 : j / groups;
    p.box_ks[j] = (std::min(64, ca - 64 * g) + 15) / 16;
  }
  p.ncol_real = mode == 0 ? 8 * cout : cin;
  p.ntask = 0;
  for (int nt = 1; nt <= 64; ++nt) {
    const int nc = ((p.ncol_real + nt - 1) / nt + 15) / 16 * 16;
    if (nc <= kMaxCols && p.nbox * nc * 128 <= kBMax) {
      p.ntask = (p.ncol_real + nc - 1) / nc;
      p.ncol = nc;
      break;
    }
  }
  if (p.ntask == 0) return false;
  p.b_bytes = p.nbox * p.ncol * 128;
  if (w <= 128) {
    p.wt = w;
    p.R = std::max(1, 128 / w);
  } else {
    p.wt = 128;
    p.R = 1;
  }
  p.nwt = (w + p.wt - 1) / p.wt;
  p.nyb = (h + p.R - 1) / p.R;
  p.tiles = (long long)n * d * p.nyb * p.nwt;
  // forward: stage the output through two [blocks][positions][2*Cout] tiles
  // stored by TMA when the task's columns are whole (a, b) blocks and the
  // staging leaves room for two load stages (R4C_TCONV_STG=0 keeps
  // per-thread stores)
  const char* ev = getenv("R4C_TCONV_STG");
  const bool stg_ok = mode == 0 && p.ncol % (2 * cout) == 0 && (8 * cout) % p.ncol == 0 &&
                      2 * cout <= 256 && !(ev && ev[0] == '0');
  int stg_total = 0;
  p.nstages = 0;
  for (int stg = stg_ok ? 1 : 0; stg >= 0 && p.nstages == 0; --stg) {
    p.stg_blk = stg ? (p.R * p.wt * 2 * cout * 2 + 127) / 128 * 128 : 0;
    stg_total = p.stg_blk ? 2 * (p.ncol / (2 * cout)) * p.stg_blk : 0;
    // stages of up to 4 boxes (64 KB) balanced over the tile: the largest
    // that leaves three stages (else two) beside the resident weights
    const int avail = kSmemMax - kHeader - (p.b_bytes + 1023) / 1024 * 1024 - stg_total;
    for (int need = 3; need >= 2 && p.nstages == 0; --need) {
      for (int bp = std::min(4, p.nbox); bp >= 1; --bp) {
        const int spt = (p.nbox + bp - 1) / bp;
        const int bpst = (p.nbox + spt - 1) / spt;
        const int ns = std::min(kMaxStages, avail / (bpst * kBoxBytes));
        if (ns >= need) {
          p.spt = spt;
          p.bpst = bpst;
          p.nstages = ns;
          break;
        }
      }
    }
  }
  if (p.nstages < 2) return false;
  p.smem = kHeader + (p.b_bytes + 1023) / 1024 * 1024 + p.nstages * p.bpst * kBoxBytes + stg_total;
  int alloc = 32;
  while (alloc < 2 * p.ncol) alloc *= 2;
  if (alloc > 512) return false;
  p.tmem_cols = alloc;
  *out = p;
  return true;
}

// PyTorch ConvTranspose3d weight (Cin, Cout, 2, 2, 2) -> per task and box a
// [ncol rows][64 K] K-major image with the 128-byte swizzle (1024-aligned):
//   forward: row = output column (a,b,c,co) of the task, K = input channel c0_j + k
//   dX:      row = input channel of the task, K = element c0_j + k of (c, co) of box (a, b)
template <typename TO>
__global__ void pack_tconv_kernel(const void* __restrict__ src, int sdt, TO* __restrict__ dst, int mode, int cin,
                                  int cout, int ncol, int nbox, int groups, int total) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int k = i % 64;
  int r = i / 64;
  const int row = r % ncol;
  r /= ncol;
  const int j = r % nbox;
  const int task = r / nbox;
  const int g = j % groups;
  const int e = 64 * g + k;  // channel of the A box set
  float v = 0.f;
  int ci = -1, co = 0, tap = 0;
  if (mode == 0) {
    const int gcol = task * ncol + row;
    if (gcol < 8 * cout && e < cin) {
      ci = e;
      tap = gcol / cout;  // (a*2 + b)*2 + c
      co = gcol - tap * cout;
    }
  } else {
    const int cc = task * ncol + row;
    if (cc < cin && e < 2 * cout) {
      ci = cc;
      const int c = e / cout;
      co = e - c * cout;
      tap = (j / groups) * 2 + c;  // (a*2 + b)*2 + c
    }
  }
  if (ci >= 0) {
    const long long s = ((long long)ci * cout + co) * 8 + tap;
    if (sdt == R4C_F32) v = static_cast<const float*>(src)[s];
    else if (sdt == R4C_BF16) v = __bfloat162float(static_cast<const __nv_bfloat16*>(src)[s]);
    else v = __half2float(static_cast<const __half*>(src)[s]);
  }
  const size_t off = (size_t)(task * nbox + j) * ncol * 128 + (size_t)(row >> 3) * 1024 + (size_t)(row & 7) * 128 +
                     (size_t)((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2;
  *reinterpret_cast<TO*>(reinterpret_cast<uint8_t*>(dst) + off) = Elem<TO>::from_f(v);
}

template <typename T>
cudaError_t launch_typed(const TArgs& a, int grid, int smem, cudaStream_t st) {
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      e = cudaFuncSetAttribute(tconv_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
      if (e != cudaSuccess) return e;
      done[dev] = true;
    }
  }
  tconv_kernel<T><<<grid, kThreads, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

bool supported(int mode, int n, int d, int h, int w, int cin, int cout) {
  TPlan p;
  return make_plan(mode, n, d, h, w, cin, cout, &p);
}

size_t packed_bytes(int mode, int n, int d, int h, int w, int cin, int cout) {
  TPlan p;
  if (!make_plan(mode, n, d, h, w, cin, cout, &p)) return 0;
  return (size_t)p.ntask * p.b_bytes;
}

int describe(int mode, int n, int d, int h, int w, int cin, int cout, char* buf, size_t len) {
  TPlan p;
  if (!make_plan(mode, n, d, h, w, cin, cout, &p)) return snprintf(buf, len, "tcgen05 tconv: no plan");
  return snprintf(buf, len,
                  "tcgen05 tconv %s (k2s2 as one GEMM over input positions): tile=%dx%d boxes=%d (%d per stage) "
                  "stages=%d tasks=%d N/task=%d B/task=%dB smem=%dB tmem=%d tiles=%lld%s",
                  mode == 0 ? "fwd" : "dX", p.R, p.wt, p.nbox, p.bpst, p.nstages, p.ntask, p.ncol, p.b_bytes,
                  p.smem, p.tmem_cols, p.tiles, p.stg_blk ? " TMA-store epilogue" : "");
}

cudaError_t pack_weight(int mode, int n, int d, int h, int w, int cin, int cout, const void* w_src, int src_dtype,
                        void* w_packed, int dtype, cudaStream_t st) {
  TPlan p;
  if (!make_plan(mode, n, d, h, w, cin, cout, &p)) return cudaErrorInvalidValue;
  const int ca = mode == 0 ? cin : 2 * cout;
  const int groups = (ca + 63) / 64;
  const int total = p.ntask * p.nbox * p.ncol * 64;
  const int blocks = (total + 255) / 256;
  if (dtype == R4C_BF16)
    pack_tconv_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(w_src, src_dtype, static_cast<__nv_bfloat16*>(w_packed),
                                                             mode, cin, cout, p.ncol, p.nbox, groups, total);
  else
    pack_tconv_kernel<__half><<<blocks, 256, 0, st>>>(w_src, src_dtype, static_cast<__half*>(w_packed), mode, cin,
                                                      cout, p.ncol, p.nbox, groups, total);
  note_launches(1);
  return cudaGetLastError();
}

// x: forward input (NDHWC, Cin) or dY (NDHWC at 2x, Cout); out: y (2x, Cout) or dX (Cin).
int launch(int mode, int n, int d, int h, int w, int cin, int cout, const void* in, const void* w_packed,
           const void* bias, void* out, int dtype, cudaStream_t st, int ypitch) {
  if (ypitch == 0) ypitch = cout;
  if (mode != 0 && ypitch != cout) return R4C_ERR_UNSUPPORTED;
  if (ypitch < cout || ypitch % 8) return R4C_ERR_INVALID;
  TPlan p;
  if (!make_plan(mode, n, d, h, w, cin, cout, &p)) return R4C_ERR_UNSUPPORTED;
  if (((uintptr_t)in & 15) || ((uintptr_t)w_packed & 15) || ((uintptr_t)out & 15)) return R4C_ERR_ALIGN;
  TArgs a;
  memset(&a, 0, sizeof(a));
  EncodeTiledFn enc = encode_fn();
  if (!enc) return R4C_ERR_CUDA;
  const cuuint64_t e = 2;
  cuuint64_t dims[5], str[4];
  cuuint32_t box[5];
  if (mode == 0) {
    const cuuint64_t c = (cuuint64_t)cin;
    cuuint64_t dd[5] = {c, (cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)d, (cuuint64_t)n};
    cuuint64_t ss[4] = {c * e, c * w * e, c * w * h * e, c * w * h * d * e};
    cuuint32_t bb[5] = {64, (cuuint32_t)p.wt, (cuuint32_t)p.R, 1, 1};
    memcpy(dims, dd, sizeof(dd));
    memcpy(str, ss, sizeof(ss));
    memcpy(box, bb, sizeof(bb));
  } else {
    // dY (N, 2D, 2H, 2W, Cout) as (2*Cout, W, 2, H, 2D*N)
    const cuuint64_t c2 = 2ull * cout, row = 2ull * w * cout * e;
    cuuint64_t dd[5] = {c2, (cuuint64_t)w, 2, (cuuint64_t)h, 2ull * d * n};
    cuuint64_t ss[4] = {c2 * e, row, 2 * row, 2 * row * h};
    cuuint32_t bb[5] = {64, (cuuint32_t)p.wt, 1, (cuuint32_t)p.R, 1};
    memcpy(dims, dd, sizeof(dd));
    memcpy(str, ss, sizeof(ss));
    memcpy(box, bb, sizeof(bb));
  }
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  if (enc(&a.amap, dtype == R4C_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
          const_cast<void*>(in), dims, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return R4C_ERR_INVALID;
  a.bimg = static_cast<const uint8_t*>(w_packed);
  a.bias = mode == 0 ? bias : nullptr;
  a.out = out;
  a.err = tc::device_error_flag();
  if (!a.err) return R4C_ERR_CUDA;
  a.mode = mode;
  a.ypitch = ypitch;
  a.n = n; a.d = d; a.h = h; a.w = w; a.cin = cin; a.cout = cout;
  a.wt = p.wt; a.R = p.R; a.nwt = p.nwt; a.nyb = p.nyb; a.tiles = p.tiles;
  a.nbox = p.nbox;
  for (int j = 0; j < p.nbox; ++j) {
    a.box_c0[j] = p.box_c0[j];
    a.box_ab[j] = p.box_ab[j];
    a.box_ks[j] = p.box_ks[j];
  }
  a.bpst = p.bpst; a.spt = p.spt; a.nstages = p.nstages;
  a.ntask = p.ntask; a.ncol = p.ncol; a.ncol_real = p.ncol_real;
  a.b_bytes = p.b_bytes; a.tmem_cols = p.tmem_cols;
  a.idesc = instr_desc_f16(dtype == R4C_BF16, 128, p.ncol, 0, 0);
  if (p.stg_blk) {
    // output (N, 2D, 2H, 2W, ypitch) as (Cout, 2W, 2, H, 2D*N), box (Cout, 2*wt, 1, R, 1):
    // the staged [positions][2*Cout] block is [2*wt][Cout] per row
    const cuuint64_t yp = (cuuint64_t)ypitch, row = 2ull * w * yp * e;
    cuuint64_t dd[5] = {(cuuint64_t)cout, 2ull * w, 2, (cuuint64_t)h, 2ull * d * n};
    cuuint64_t ss[4] = {yp * e, row, 2 * row, 2 * row * h};
    cuuint32_t bb[5] = {(cuuint32_t)cout, 2u * (cuuint32_t)p.wt, 1, (cuuint32_t)p.R, 1};
    if (enc(&a.ymap, dtype == R4C_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, out,
            dd, ss, bb, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return R4C_ERR_INVALID;
    a.stg_blk = p.stg_blk;
  }
  // CTAs per task: the SMs shared out, at most one per tile
  const long long cpt = std::max<long long>(1, std::min<long long>(p.tiles, sm_count() / p.ntask));
  const int grid = (int)(cpt * p.ntask);
  const cudaError_t ce = dtype == R4C_BF16 ? launch_typed<__nv_bfloat16>(a, grid, p.smem, st)
                                           : launch_typed<__half>(a, grid, p.smem, st);
  note_launches(1);
  return ce == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}


// ---------------------------------------------------------------------------
// dW host side.
// ---------------------------------------------------------------------------
namespace {

struct DwTPlan {
  int wt, R, nwt, nyb;
  long long tiles;
  int S, ntask, nabg, nab, ngb, ncol, nmma, mma_n, nbox, nstages, tmem_cols, smem;
  size_t part_bytes;
};

bool make_dw_plan(int n, int d, int h, int w, int cin, int cout, int sms, DwTPlan* out) {
  if (n < 1 || d < 1 || h < 1 || w < 1) return false;
  if (cin % 8 || cout % 8 || cin < 8 || cout < 8 || cout > 256) return false;
  DwTPlan p{};
  p.ngb = (2 * cout + 63) / 64;
  p.nab = 4;
  while (p.nab > 1 && p.nab * p.ngb * 64 > 512) p.nab /= 2;
  p.ncol = p.nab * p.ngb * 64;
  if (p.ncol > 512) return false;
  p.mma_n = 64;
  for (int k = 4; k >= 1; --k)
    if (p.ncol % (64 * k) == 0) {
      p.mma_n = 64 * k;
      break;
    }
  p.nmma = p.ncol / p.mma_n;
  p.nabg = 4 / p.nab;
  p.ntask = ((cin + 127) / 128) * p.nabg;
  p.nbox = 2 + p.nab * p.ngb;
  p.nstages = std::min(kMaxStages, (kSmemMax - kHeader) / (p.nbox * kDwBox));
  if (p.nstages < 2) return false;
  p.smem = kHeader + p.nstages * p.nbox * kDwBox;
  // K tile: 64 positions = R rows x wt columns (wt a power of two >= W, up
  // to 64; columns past W and rows past H are the zero fill)
  p.wt = 1;
  while (p.wt < std::min(w, 64)) p.wt *= 2;
  p.R = 64 / p.wt;
  p.nwt = (w + p.wt - 1) / p.wt;
  p.nyb = (h + p.R - 1) / p.R;
  p.tiles = (long long)n * d * p.nyb * p.nwt;
  p.S = (int)std::max<long long>(1, std::min<long long>(p.tiles, sms / p.ntask));
  p.part_bytes = (size_t)p.ntask * p.S * 128 * p.ncol * sizeof(float);
  int alloc = 32;
  while (alloc < p.ncol) alloc *= 2;
  p.tmem_cols = alloc;
  *out = p;
  return true;
}

}  // namespace

bool dw_supported(int n, int d, int h, int w, int cin, int cout) {
  DwTPlan p;
  return make_dw_plan(n, d, h, w, cin, cout, 148, &p);
}

size_t dw_workspace(int n, int d, int h, int w, int cin, int cout) {
  DwTPlan p;
  if (!make_dw_plan(n, d, h, w, cin, cout, sm_count(), &p)) return 0;
  return (p.part_bytes + 255) / 256 * 256;
}

int dw_describe(int n, int d, int h, int w, int cin, int cout, char* buf, size_t len) {
  DwTPlan p;
  if (!make_dw_plan(n, d, h, w, cin, cout, 148, &p)) return snprintf(buf, len, "tcgen05 tconv dW: no plan");
  return snprintf(buf, len,
                  "tcgen05 tconv dW (MN-major x and dY boxes, split-K over positions): K tile=%dx%d tasks=%d "
                  "(a,b)/task=%d N/task=%d (%d MMAs of N=%d) boxes/stage=%d stages=%d splits=%d tiles=%lld",
                  p.R, p.wt, p.ntask, p.nab, p.ncol, p.nmma, p.mma_n, p.nbox, p.nstages, p.S, p.tiles);
}

// x (NDHWC, Cin), go (NDHWC at 2x, Cout) -> dw fp32 (Cin, Cout, 2, 2, 2); ws >= dw_workspace().
int launch_dw(int n, int d, int h, int w, int cin, int cout, const void* x, const void* go, float* dw, float* db,
              void* ws, size_t ws_bytes, int dtype, cudaStream_t st, bool* db_done) {
  if (db_done) *db_done = false;
  DwTPlan p;
  if (!make_dw_plan(n, d, h, w, cin, cout, sm_count(), &p)) return R4C_ERR_UNSUPPORTED;
  if (((uintptr_t)x & 15) || ((uintptr_t)go & 15)) return R4C_ERR_ALIGN;
  if (!ws || ws_bytes < p.part_bytes) return R4C_ERR_WORKSPACE;
  DwTArgs a;
  memset(&a, 0, sizeof(a));
  EncodeTiledFn enc = encode_fn();
  if (!enc) return R4C_ERR_CUDA;
  const CUtensorMapDataType dt = dtype == R4C_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint64_t e = 2;
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  {
    const cuuint64_t c = (cuuint64_t)cin;
    cuuint64_t dims[5] = {c, (cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)d, (cuuint64_t)n};
    cuuint64_t str[4] = {c * e, c * w * e, c * w * h * e, c * w * h * d * e};
    cuuint32_t box[5] = {64, (cuuint32_t)p.wt, (cuuint32_t)p.R, 1, 1};
    if (enc(&a.xmap, dt, 5, const_cast<void*>(x), dims, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return R4C_ERR_INVALID;
  }
  {
    const cuuint64_t c2 = 2ull * cout, row = 2ull * w * cout * e;
    cuuint64_t dims[5] = {c2, (cuuint64_t)w, 2, (cuuint64_t)h, 2ull * d * n};
    cuuint64_t str[4] = {c2 * e, row, 2 * row, 2 * row * h};
    cuuint32_t box[5] = {64, (cuuint32_t)p.wt, 1, (cuuint32_t)p.R, 1};
    if (enc(&a.gmap, dt, 5, const_cast<void*>(go), dims, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return R4C_ERR_INVALID;
  }
  a.part = static_cast<float*>(ws);
  a.err = tc::device_error_flag();
  if (!a.err) return R4C_ERR_CUDA;
  a.n = n; a.d = d; a.h = h; a.w = w; a.cin = cin; a.cout = cout;
  a.wt = p.wt; a.R = p.R; a.nwt = p.nwt; a.nyb = p.nyb; a.tiles = p.tiles;
  a.S = p.S; a.ntask = p.ntask; a.nabg = p.nabg; a.nab = p.nab; a.ngb = p.ngb;
  a.ncol = p.ncol; a.nmma = p.nmma; a.mma_n = p.mma_n; a.nbox = p.nbox; a.nstages = p.nstages;
  a.tmem_cols = p.tmem_cols;
  a.idesc = instr_desc_f16(dtype == R4C_BF16, 128, p.mma_n, 1, 1);
  a.ones_mt = (cin - 1) / 128;
  const int cin_last = cin - 128 * a.ones_mt;
  a.ones = (db != nullptr && cin_last <= 64) ? 1 : 0;
  // Opt-in (R4C_TCONV_DBFILL=1, read once): at 96->48 the db kernel path
  // measured 82 us for the dW leg, this fill path 91 us (the MMA warp's
  // stores + proxy fence stall each stage).
  static const bool fill_on = [] {
    const char* fe = getenv("R4C_TCONV_DBFILL");
    return fe && fe[0] == '1';
  }();
  a.ones_fill = (db != nullptr && cin_last > 64 && cin_last <= 120 && cin_last % 8 == 0 && fill_on) ? 1 : 0;
  a.ones_row = a.ones_fill ? cin_last : 64;
  a.one_bits = dtype == R4C_BF16 ? 0x3F80u : 0x3C00u;
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return R4C_ERR_CUDA;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 64 && !done[dev]) {
      if (cudaFuncSetAttribute(tconv_dw_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax) !=
          cudaSuccess)
        return R4C_ERR_CUDA;
      done[dev] = true;
    }
  }
  tconv_dw_kernel<<<p.ntask * p.S, kThreads, p.smem, st>>>(a);
  note_launches(1);
  if (cudaGetLastError() != cudaSuccess) return R4C_ERR_CUDA;
  const long long total = (long long)cin * cout * 8;
  tconv_dw_reduce<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(a.part, dw, cin, cout, p.S, p.nabg, p.nab, p.ngb,
                                                                   p.ncol);
  note_launches(1);
  if (a.ones || a.ones_fill) {
    tconv_db_reduce<<<(unsigned)((cout + 31) / 32), 256, 0, st>>>(a.part, db, cout, p.S, a.ones_mt, a.ones_row,
                                                                 p.nabg, p.nab, p.ngb, p.ncol);
    note_launches(1);
    if (db_done) *db_done = true;
  }
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

}  // namespace tconv
}  // namespace r4c
