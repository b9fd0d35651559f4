// r4c_tc.cu — tcgen05 + TMA implicit-GEMM Conv3d for sm_100a (k = 1 or 3,
// stride 1, Cin a multiple of 8, Cout <= 256). Runs the forward conv and, with
// the flipped/transposed weight and padding k-1-p, the input gradient.
//
// Reference counterpart: _fwd_k3_kernel / _fwd_k1_kernel and the k3 dX reuse
// in _launch_dgrad (src/rdna4_conv3d/conv3d_wmma.py:327-444, 1154-1162). The
// reference gathers a masked 27-tap im2col tile per K step; here the GEMM is
// laid out for the B200 memory system instead:
//
//  * Work unit = one output plane tile (n, z, ht rows x wt cols), persistent
//    CTAs (one per SM) walk the units.
//  * For each kd in 0..k-1 and each group of G 8-channel chunks, ONE TMA box
//    per chunk brings the (ht+k-1) x (wt+k-1) input halo of plane z+kd-pad into
//    shared memory as a "chunk plane": rows are brick positions, 16 bytes (8
//    channels) each. TMA's out-of-bounds zero fill is the conv padding.
//  * GEMM rows are brick positions p = hh*(wt+k-1) + ww ("padded grid"): a tap
//    (kh, kw) is then a constant shift of the A start address, so all k*k taps
//    read the same brick without any im2col copy. Rows with ww >= wt or
//    hh >= ht are junk and are simply not stored.
//  * tcgen05.mma kind::f16, M = 128, N = Cout padded to 16, K = 16 (two
//    8-channel core-matrix columns whose distance is the descriptor LBO). For
//    an odd number of chunks (Cin = 24) two taps share one K step: (kw, kw+1)
//    are 16 bytes apart, (kh, kh+1) one brick row apart.
//  * fp32 accumulators live in TMEM (double-buffered when they fit), the
//    epilogue warps read them with tcgen05.ld, add bias, round, and store.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer + TMEM
// owner, warps 2-5 epilogue (TMEM lane quarter = warp % 4).
#include <cuda.h>

#include <mutex>
#include <vector>

#include "r4c_internal.h"
#include "r4c_sm100.cuh"

namespace r4c {

__device__ int g_r4c_dev_error = 0;

namespace tc {

constexpr int kMaxSteps = 64;
constexpr int kMaxStages = 6;
constexpr int kThreads = 192;
constexpr int kSmemMax = 232448;  // 227 KB opt-in dynamic shared memory
constexpr int kHeader = 2048;     // barriers + bias

struct alignas(64) TcConvArgs {
  CUtensorMap tmap;
  const uint8_t* wpack;
  const void* bias;
  void* y;
  int n, od, oh, ow, cout, npad;
  int pd, ph, pw, ks;
  int ht, wt, nht, nwt;
  int pitch_w;
  int G, ngroups, nsteps;
  int mtiles, nsets;
  int cpb, a_bytes, b_bytes, stage_bytes, stages;
  int wres, wres_bytes;
  int tmem_cols;
  long long units;
  uint32_t idesc;
  uint32_t tx_bytes;
  int a_off[kMaxSteps];
  int lbo[kMaxSteps];
};

struct HalfRef {
  int kh, kw, c, zero;
};
struct Step {
  HalfRef h[2];
  int a_off;
  int lbo;
};

static int steps_per_stage(int ks, int G) {
  if (G % 2 == 0) return ks * ks * G / 2;
  return ks == 3 ? 4 * G + (G + 1) / 2 : (G + 1) / 2;
}

static void build_steps(int ks, int G, int pitch_w, int cpb, std::vector<Step>& st) {
  st.clear();
  auto off = [&](int kh, int kw, int c) { return c * cpb + (kh * pitch_w + kw) * 16; };
  auto ref = [](int kh, int kw, int c) { return HalfRef{kh, kw, c, 0}; };
  const HalfRef zero{0, 0, 0, 1};
  if (G % 2 == 0) {
    for (int kh = 0; kh < ks; ++kh)
      for (int kw = 0; kw < ks; ++kw)
        for (int j = 0; j < G / 2; ++j)
          st.push_back(Step{{ref(kh, kw, 2 * j), ref(kh, kw, 2 * j + 1)}, off(kh, kw, 2 * j), cpb});
    return;
  }
  if (ks == 3) {
    // (kw=0, kw=1) pairs: the second half is one brick position (16 B) later.
    for (int kh = 0; kh < 3; ++kh)
      for (int c = 0; c < G; ++c)
        st.push_back(Step{{ref(kh, 0, c), ref(kh, 1, c)}, off(kh, 0, c), 16});
    // kw=2: (kh=0, kh=1) pairs, one brick row apart.
    for (int c = 0; c < G; ++c)
      st.push_back(Step{{ref(0, 2, c), ref(1, 2, c)}, off(0, 2, c), pitch_w * 16});
    // (kh=2, kw=2): chunk pairs.
    for (int j = 0; j < (G - 1) / 2; ++j)
      st.push_back(Step{{ref(2, 2, 2 * j), ref(2, 2, 2 * j + 1)}, off(2, 2, 2 * j), cpb});
    // Last chunk: paired with a zero-weight half that reads the preceding row.
    st.push_back(Step{{zero, ref(2, 2, G - 1)}, off(2, 2, G - 1) - 16, 16});
  } else {
    for (int j = 0; j < (G - 1) / 2; ++j)
      st.push_back(Step{{ref(0, 0, 2 * j), ref(0, 0, 2 * j + 1)}, off(0, 0, 2 * j), cpb});
    st.push_back(Step{{zero, ref(0, 0, G - 1)}, off(0, 0, G - 1) - 16, 16});
  }
}

// ---------------------------------------------------------------------------
// Planner (host only).
// ---------------------------------------------------------------------------
static int round_up(int v, int a) { return (v + a - 1) / a * a; }

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

bool plan_conv(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw,
               ConvPlan* pl) {
  ConvPlan P{};
  P.ok = false;
  if (ks != 1 && ks != 3) return false;
  if (cin % 8 != 0 || cin <= 0 || cout <= 0 || cout > 256) return false;
  if (n <= 0 || d <= 0 || h <= 0 || w <= 0) return false;
  P.od = d + 2 * pd - (ks - 1);
  P.oh = h + 2 * ph - (ks - 1);
  P.ow = w + 2 * pw - (ks - 1);
  if (P.od <= 0 || P.oh <= 0 || P.ow <= 0) return false;
  // TMA coordinates are int32 and start at -pad: keep pads small.
  if (pd > 8 || ph > 8 || pw > 8 || pd < -8 || ph < -8 || pw < -8) return false;
  P.n = n; P.d = d; P.h = h; P.w = w;
  P.cin = cin; P.cout = cout; P.ks = ks; P.pd = pd; P.ph = ph; P.pw = pw;
  P.c8 = cin / 8;
  P.npad = round_up(cout, 16);

  std::vector<int> gs;
  if (P.c8 % 2 == 1) {
    if (P.c8 > 13) return false;
    gs.push_back(P.c8);
  } else {
    for (int g = std::min(P.c8, 14); g >= 2; g -= 2)
      if (P.c8 % g == 0) gs.push_back(g);
  }
  int wt_max = 256 - (ks - 1);
  int nw = (P.ow + wt_max - 1) / wt_max;
  int wt = (P.ow + nw - 1) / nw;
  const int sms = num_sms();

  // Cost model per work unit (SM clocks): tcgen05 issue (128xNx16 takes
  // about N/2 clocks, at least ~10 to issue), L2 -> SMEM copy traffic at
  // ~48 B/clk/SM, and the TMEM -> global epilogue (overlapped with the next
  // unit's MMAs when two accumulator sets fit in TMEM). Launch estimate =
  // waves * per-unit time; the plan with the smallest estimate wins.
  double best = 1e300;
  for (int G : gs) {
    int nsteps = steps_per_stage(ks, G);
    if (nsteps > kMaxSteps) continue;
    const int ngroups = P.c8 / G;
    const int b_bytes = nsteps * 2 * P.npad * 16;
    const int wbytes = ks * ngroups * b_bytes;
    for (int wres = 0; wres <= 1; ++wres) {
      if (wres && wbytes > 96 * 1024) continue;
      for (int ht = 1; ht <= P.oh && ht <= 256 - (ks - 1); ++ht) {
        int pitch_w = wt + ks - 1, pitch_h = ht + ks - 1;
        int span = (ht - 1) * pitch_w + wt;
        int mtiles = (span + 127) / 128;
        if (mtiles * P.npad > 512) break;
        int nsets = (2 * mtiles * P.npad <= 512) ? 2 : 1;
        int cpb = round_up(pitch_h * pitch_w * 16, 128);
        int maxrow = 128 * mtiles - 1 + (ks - 1) * (pitch_w + 1);
        int pad = round_up(std::max(0, (maxrow + 1) * 16 - cpb), 128);
        int a_bytes = 128 + G * cpb + pad;
        int stage = round_up(a_bytes + (wres ? 0 : b_bytes), 128);
        int avail = kSmemMax - kHeader - (wres ? round_up(wbytes, 128) : 0);
        int stages = std::min(kMaxStages, avail / stage);
        if (stages < 2) continue;
        int tiles_h = (P.oh + ht - 1) / ht;
        long long units = (long long)n * P.od * tiles_h * nw;
        double mma = (double)ks * ngroups * nsteps * mtiles * std::max(10.0, P.npad / 2.0);
        double load = (double)ks * ngroups * (G * pitch_h * pitch_w * 16.0 + (wres ? 0.0 : b_bytes)) / 48.0;
        double epi = (double)mtiles * (P.npad / 16.0) * 40.0;
        double t_unit = std::max(mma, load) + 200.0;
        t_unit = nsets == 2 ? std::max(t_unit, epi) : t_unit + epi;
        long long waves = (units + sms - 1) / sms;
        double est = (double)waves * t_unit + (wres ? wbytes / 48.0 : 0.0);
        if (est < best) {
          best = est;
          P.G = G; P.ngroups = ngroups; P.nsteps = nsteps;
          P.wt = wt; P.ht = ht; P.pitch_w = pitch_w; P.pitch_h = pitch_h;
          P.cpb = cpb; P.mtiles = mtiles; P.nsets = nsets;
          P.a_bytes = a_bytes; P.b_bytes = b_bytes; P.stage_bytes = stage; P.stages = stages;
          P.wres = wres; P.wres_bytes = wres ? round_up(wbytes, 128) : 0;
          P.smem_bytes = kHeader + P.wres_bytes + stages * stage;
          int cols = nsets * mtiles * P.npad;
          int alloc = 32;
          while (alloc < cols) alloc *= 2;
          P.tmem_cols = alloc;
          P.work_units = units;
          P.grid = (int)std::min<long long>(units, sms);
          P.est_cycles = est;
          P.ok = true;
        }
      }
    }
  }
  if (!P.ok) return false;
  if (pl) *pl = P;
  return true;
}


size_t packed_bytes(const ConvPlan& P) {
  return (size_t)P.ks * P.ngroups * P.b_bytes;
}

// ---------------------------------------------------------------------------
// Weight pack: PyTorch OIDHW -> per-stage K-step blocks [step][half][npad][8].
// ---------------------------------------------------------------------------
struct PackArgs {
  int ks, G, ngroups, nsteps, npad, cin, cout;  // cin/cout of the conv being run
  int cin_real;                                  // input channels present in the source (<= cin)
  int flip;                                      // dX: W'[o][i][t] = W[i][o][T-1-t]
  int src_cin;                                   // channel count of the OIDHW source's dim 1
  signed char kh[kMaxSteps][2], kw[kMaxSteps][2], c[kMaxSteps][2], zero[kMaxSteps][2];
};

template <typename TO>
__global__ void pack_tc_kernel(const void* __restrict__ src, int sdt, TO* __restrict__ dst, PackArgs a) {
  const long long total = (long long)a.ks * a.ngroups * a.nsteps * 2 * a.npad * 8;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  int e = (int)(i % 8);
  long long r = i / 8;
  int nrow = (int)(r % a.npad); r /= a.npad;
  int half = (int)(r % 2); r /= 2;
  int j = (int)(r % a.nsteps); r /= a.nsteps;
  int g = (int)(r % a.ngroups);
  int kd = (int)(r / a.ngroups);
  float v = 0.f;
  if (!a.zero[j][half] && nrow < a.cout) {
    int ci = (g * a.G + a.c[j][half]) * 8 + e;
    if (ci < a.cin_real) {
      int T = a.ks * a.ks * a.ks;
      int tap = (kd * a.ks + a.kh[j][half]) * a.ks + a.kw[j][half];
      long long s;
      if (!a.flip) {
        s = ((long long)nrow * a.src_cin + ci) * T + tap;  // W[co=nrow][ci][tap]
      } else {
        s = ((long long)ci * a.src_cin + nrow) * T + (T - 1 - tap);  // W[co=ci][ci'=nrow][T-1-tap]
      }
      if (sdt == R4C_F32) v = static_cast<const float*>(src)[s];
      else if (sdt == R4C_BF16) v = __bfloat162float(static_cast<const __nv_bfloat16*>(src)[s]);
      else v = __half2float(static_cast<const __half*>(src)[s]);
    }
  }
  dst[i] = Elem<TO>::from_f(v);
}

cudaError_t pack_weight(const ConvPlan& P, bool flip, int cin_real, const void* w_src, int src_dtype,
                        void* w_packed, int dtype, cudaStream_t st) {
  std::vector<Step> steps;
  build_steps(P.ks, P.G, P.pitch_w, P.cpb, steps);
  PackArgs a{};
  a.ks = P.ks; a.G = P.G; a.ngroups = P.ngroups; a.nsteps = (int)steps.size();
  a.npad = P.npad; a.cin = P.cin; a.cout = P.cout; a.flip = flip ? 1 : 0;
  a.cin_real = cin_real;
  // OIDHW source dim 1: the real Cin for the forward weight; for dX (flipped)
  // it is Cin of the layer, i.e. this conv's output channels.
  a.src_cin = flip ? P.cout : cin_real;
  for (int j = 0; j < a.nsteps; ++j)
    for (int hf = 0; hf < 2; ++hf) {
      a.kh[j][hf] = (signed char)steps[j].h[hf].kh;
      a.kw[j][hf] = (signed char)steps[j].h[hf].kw;
      a.c[j][hf] = (signed char)steps[j].h[hf].c;
      a.zero[j][hf] = (signed char)steps[j].h[hf].zero;
    }
  long long total = (long long)a.ks * a.ngroups * a.nsteps * 2 * a.npad * 8;
  unsigned blocks = (unsigned)((total + 255) / 256);
  if (dtype == R4C_BF16)
    pack_tc_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(w_src, src_dtype,
                                                          static_cast<__nv_bfloat16*>(w_packed), a);
  else
    pack_tc_kernel<__half><<<blocks, 256, 0, st>>>(w_src, src_dtype, static_cast<__half*>(w_packed), a);
  note_launches(1);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
using namespace r4c::sm100;

template <typename T>
__device__ __forceinline__ void store_row16(T* dst, const float (&v)[16], const float* bias, int cc, int cout,
                                            bool vec_ok) {
  if (vec_ok && cc + 16 <= cout) {
    uint32_t pk[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      T lo = Elem<T>::from_f(v[2 * i] + bias[cc + 2 * i]);
      T hi = Elem<T>::from_f(v[2 * i + 1] + bias[cc + 2 * i + 1]);
      pk[i] = (uint32_t)(*reinterpret_cast<uint16_t*>(&lo)) |
              ((uint32_t)(*reinterpret_cast<uint16_t*>(&hi)) << 16);
    }
    uint4* d4 = reinterpret_cast<uint4*>(dst + cc);
    d4[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    d4[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (cc + i < cout) dst[cc + i] = Elem<T>::from_f(v[i] + bias[cc + i]);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) tc_conv_kernel(const __grid_constant__ TcConvArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* mdone = tempty + 2;
  uint64_t* wbar = mdone + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wbar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sbias = reinterpret_cast<float*>(smem + 1024);
  uint8_t* wres_smem = smem + kHeader;
  uint8_t* stage0 = smem + kHeader + a.wres_bytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // TMA writes need 128-byte aligned destinations; every stage offset is a
  // multiple of 128 from the dynamic shared memory base, so check the base.
  if ((smem_u32(smem) & 127u) != 0u || a.tmem_cols > 512) {
    if (threadIdx.x == 0) atomicExch(&g_r4c_dev_error, 2);
    return;
  }

  // One-time set-up: zero the stage buffers (guard rows, inter-plane gaps and
  // the overrun pad are read by junk GEMM rows only, but keep them finite),
  // stage the bias as fp32, init barriers, allocate TMEM.
  {
    uint4 z = make_uint4(0, 0, 0, 0);
    const int total = a.stages * a.stage_bytes;
    for (int i = threadIdx.x * 16; i < total; i += kThreads * 16) *reinterpret_cast<uint4*>(stage0 + i) = z;
    const T* bias = static_cast<const T*>(a.bias);
    for (int i = threadIdx.x; i < a.npad; i += kThreads)
      sbias[i] = (bias != nullptr && i < a.cout) ? Elem<T>::to_f(bias[i]) : 0.f;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 4);
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
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int tiles_per_plane = a.nht * a.nwt;
  const long long units = a.units;
  const uint64_t kWaitNs = 1000000000ull;  // 1 s per wait

  auto wait = [&](uint64_t* bar, uint32_t par) -> bool {
    uint64_t deadline = global_timer_ns() + kWaitNs;
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, par)) {
      if (((++spins) & 255u) == 0) {
        if (*abort_flag) return false;
        if (global_timer_ns() > deadline) {
          *abort_flag = 1;
          atomicExch(&g_r4c_dev_error, 1);
          return false;
        }
      }
    }
    return true;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&a.tmap);
      if (a.wres) {
        mbar_arrive_expect_tx(wbar, (uint32_t)(a.ks * a.ngroups * a.b_bytes));
        bulk_load(wres_smem, a.wpack, (uint32_t)(a.ks * a.ngroups * a.b_bytes), wbar);
      }
      int stage = 0;
      uint32_t epar = 1;
      bool pending[kMaxStages];
      uint32_t last_par[kMaxStages];
      for (int s = 0; s < kMaxStages; ++s) { pending[s] = false; last_par[s] = 0; }
      bool ok = true;
      for (long long u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int wi = (int)(u % a.nwt);
        long long r = u / a.nwt;
        int hi = (int)(r % a.nht); r /= a.nht;
        int z = (int)(r % a.od);
        int nb = (int)(r / a.od);
        const int w0 = wi * a.wt - a.pw, h0 = hi * a.ht - a.ph;
        for (int kd = 0; kd < a.ks && ok; ++kd) {
          const int iz = z + kd - a.pd;
          for (int g = 0; g < a.ngroups; ++g) {
            if (!wait(&empty[stage], epar)) { ok = false; break; }
            uint8_t* sA = stage0 + (size_t)stage * a.stage_bytes;
            mbar_arrive_expect_tx(&full[stage], a.tx_bytes);
            for (int cl = 0; cl < a.G; ++cl)
              tma_load_5d(sA + 128 + cl * a.cpb, &a.tmap, &full[stage], (g * a.G + cl) * 8, w0, h0, iz, nb);
            if (!a.wres)
              bulk_load(sA + a.a_bytes, a.wpack + (size_t)(kd * a.ngroups + g) * a.b_bytes,
                        (uint32_t)a.b_bytes, &full[stage]);
            pending[stage] = true;
            last_par[stage] = epar ^ 1;
            if (++stage == a.stages) { stage = 0; epar ^= 1; }
          }
        }
      }
      // Wait (bounded) until every copy this thread issued has landed, so no
      // TMA write can outlive the CTA on the error path.
      if (a.wres) {
        uint64_t dl = global_timer_ns() + kWaitNs;
        while (!mbar_try_wait(wbar, 0) && global_timer_ns() < dl) {
        }
      }
      for (int s = 0; s < a.stages; ++s) {
        if (!pending[s]) continue;
        uint64_t dl = global_timer_ns() + kWaitNs;
        while (!mbar_try_wait(&full[s], last_par[s]) && global_timer_ns() < dl) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t fpar = 0;
      uint32_t tpar[2] = {1, 1};
      int acc = 0;
      const int nsets = a.nsets;
      bool ok = true;
      if (a.wres && !wait(wbar, 0)) ok = false;
      for (long long u = blockIdx.x; u < units && ok; u += gridDim.x) {
        if (!wait(&tempty[acc], tpar[acc])) { ok = false; break; }
        tpar[acc] ^= 1;
        tc_fence_after();
        const uint32_t dbase = tmem + (uint32_t)(acc * a.mtiles * a.npad);
        for (int kd = 0; kd < a.ks && ok; ++kd) {
          for (int g = 0; g < a.ngroups; ++g) {
            if (!wait(&full[stage], fpar)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sA = smem_u32(stage0 + (size_t)stage * a.stage_bytes) + 128;
            const uint32_t sB =
                a.wres ? smem_u32(wres_smem + (size_t)(kd * a.ngroups + g) * a.b_bytes)
                       : smem_u32(stage0 + (size_t)stage * a.stage_bytes + a.a_bytes);
            const bool first_stage = (kd == 0 && g == 0);
            // Descriptors: one build per K step, 64-bit adds for the M tiles
            // (2048 B = 128 descriptor units apart) and K steps of B.
            const uint64_t bdesc0 = smem_desc(sB, (uint32_t)(a.npad * 16), 128);
            const uint64_t bstep = (uint64_t)((2 * a.npad * 16) >> 4);
            for (int j = 0; j < a.nsteps; ++j) {
              const uint64_t bdesc = bdesc0 + (uint64_t)j * bstep;
              const uint64_t adesc = smem_desc((uint32_t)((int)sA + a.a_off[j]), (uint32_t)a.lbo[j], 128);
              const uint32_t accum = (first_stage && j == 0) ? 0u : 1u;
              uint32_t d = dbase;
              uint64_t ad = adesc;
              for (int t = 0; t < a.mtiles; ++t) {
                mma_f16_ss(d, ad, bdesc, a.idesc, accum);
                d += (uint32_t)a.npad;
                ad += 128;
              }
            }
            mma_commit(&empty[stage]);
            if (++stage == a.stages) { stage = 0; fpar ^= 1; }
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        if (nsets == 2) acc ^= 1;
      }
      // All MMAs issued by this thread complete before TMEM is released.
      mma_commit(mdone);
      wait(mdone, 0);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    T* __restrict__ y = static_cast<T*>(a.y);
    const bool vec_ok = (a.cout % 8) == 0;
    uint32_t fpar[2] = {0, 0};
    int acc = 0;
    for (long long u = blockIdx.x; u < units; u += gridDim.x) {
      int wi = (int)(u % a.nwt);
      long long r = u / a.nwt;
      int hi = (int)(r % a.nht); r /= a.nht;
      int z = (int)(r % a.od);
      int nb = (int)(r / a.od);
      const int h0 = hi * a.ht, w0 = wi * a.wt;
      if (!wait(&tfull[acc], fpar[acc])) break;
      fpar[acc] ^= 1;
      tc_fence_after();
      for (int t = 0; t < a.mtiles; ++t) {
        const int p = t * 128 + row;
        const int hh = p / a.pitch_w;
        const int ww = p - hh * a.pitch_w;
        const bool valid = hh < a.ht && ww < a.wt && (h0 + hh) < a.oh && (w0 + ww) < a.ow;
        T* dst = y + ((((long long)nb * a.od + z) * a.oh + (h0 + hh)) * a.ow + (w0 + ww)) * a.cout;
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * a.mtiles * a.npad + t * a.npad);
        for (int cc = 0; cc < a.npad; cc += 16) {
          float v[16];
          tmem_ld_16(tbase + (uint32_t)cc, v);
          if (valid) store_row16<T>(dst, v, sbias, cc, a.cout, vec_ok);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (a.nsets == 2) acc ^= 1;
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
// Host launch.
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

template <typename T>
static cudaError_t set_smem_attr() {
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && done[dev]) return cudaSuccess;
  e = cudaFuncSetAttribute(tc_conv_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  if (e == cudaSuccess && dev >= 0 && dev < 64) done[dev] = true;
  return e;
}

int launch_conv(const ConvPlan& P, const void* x, const void* w_packed, const void* bias, void* y, int dtype,
                cudaStream_t st) {
  if (((uintptr_t)x & 15) || ((uintptr_t)w_packed & 15)) return R4C_ERR_ALIGN;
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return R4C_ERR_CUDA;
  static_assert(sizeof(TcConvArgs) <= 4096, "kernel argument block too large");
  TcConvArgs a;
  memset(&a, 0, sizeof(a));
  const cuuint64_t esz = 2;
  cuuint64_t dims[5] = {(cuuint64_t)P.cin, (cuuint64_t)P.w, (cuuint64_t)P.h, (cuuint64_t)P.d, (cuuint64_t)P.n};
  cuuint64_t strides[4] = {P.cin * esz, (cuuint64_t)P.w * P.cin * esz, (cuuint64_t)P.h * P.w * P.cin * esz,
                           (cuuint64_t)P.d * P.h * P.w * P.cin * esz};
  cuuint32_t box[5] = {8, (cuuint32_t)P.pitch_w, (cuuint32_t)P.pitch_h, 1, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult cr = enc(&a.tmap, dtype == R4C_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                    5, const_cast<void*>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return R4C_ERR_INVALID;

  std::vector<Step> steps;
  const int G = P.G;
  const int cpb = P.cpb;
  build_steps(P.ks, G, P.pitch_w, cpb, steps);
  a.wpack = static_cast<const uint8_t*>(w_packed);
  a.bias = bias;
  a.y = y;
  a.n = P.n; a.od = P.od; a.oh = P.oh; a.ow = P.ow; a.cout = P.cout; a.npad = P.npad;
  a.pd = P.pd; a.ph = P.ph; a.pw = P.pw; a.ks = P.ks;
  a.ht = P.ht; a.wt = P.wt;
  a.nht = (P.oh + P.ht - 1) / P.ht;
  a.nwt = (P.ow + P.wt - 1) / P.wt;
  a.pitch_w = P.pitch_w;
  a.G = G; a.ngroups = P.ngroups; a.nsteps = (int)steps.size();
  a.mtiles = P.mtiles; a.nsets = P.nsets;
  a.cpb = cpb; a.a_bytes = P.a_bytes; a.b_bytes = P.b_bytes; a.stage_bytes = P.stage_bytes; a.stages = P.stages;
  a.wres = P.wres; a.wres_bytes = P.wres_bytes;
  a.tmem_cols = P.tmem_cols;
  a.units = P.work_units;
  a.idesc = sm100::instr_desc_f16(dtype == R4C_BF16, 128, P.npad, 0, 0);
  a.tx_bytes = (uint32_t)(G * P.pitch_h * P.pitch_w * 16 + (P.wres ? 0 : P.b_bytes));
  for (int j = 0; j < a.nsteps; ++j) {
    a.a_off[j] = steps[j].a_off;
    a.lbo[j] = steps[j].lbo;
  }
  cudaError_t e;
  if (dtype == R4C_BF16) {
    e = set_smem_attr<__nv_bfloat16>();
    if (e != cudaSuccess) return R4C_ERR_CUDA;
    tc_conv_kernel<__nv_bfloat16><<<P.grid, kThreads, P.smem_bytes, st>>>(a);
  } else {
    e = set_smem_attr<__half>();
    if (e != cudaSuccess) return R4C_ERR_CUDA;
    tc_conv_kernel<__half><<<P.grid, kThreads, P.smem_bytes, st>>>(a);
  }
  note_launches(1);
  e = cudaGetLastError();
  return e == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

}  // namespace tc
}  // namespace r4c

namespace r4c {
namespace tc {
// Device address of the error flag for the current device, for kernels in
// other translation units (device symbols are per translation unit without
// relocatable device code).
int* device_error_flag() {
  static int* ptrs[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_r4c_dev_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}
}  // namespace tc
}  // namespace r4c

extern "C" int r4c_device_error(r4c_stream_t stream, int clear) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return R4C_ERR_CUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, r4c::g_r4c_dev_error, sizeof(int)) != cudaSuccess) return R4C_ERR_CUDA;
  if (clear && v) {
    int z = 0;
    if (cudaMemcpyToSymbol(r4c::g_r4c_dev_error, &z, sizeof(int)) != cudaSuccess) return R4C_ERR_CUDA;
  }
  return v;
}

