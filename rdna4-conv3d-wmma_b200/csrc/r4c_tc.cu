// r4c_tc.cu — tcgen05 implicit-GEMM Conv3d for sm_100a (k = 1 or 3, stride 1,
// Cin a multiple of 8, Cout <= 256). Runs the forward conv and, with the
// flipped/transposed weight and padding k-1-p, the input gradient.
//
// Reference counterpart: _fwd_k3_kernel / _fwd_k1_kernel and the k3 dX reuse
// in _launch_dgrad (src/rdna4_conv3d/conv3d_wmma.py:327-444, 1154-1162). The
// reference gathers a masked 27-tap im2col tile per K step; here the GEMM is
// laid out for the B200 memory system instead:
//
//  * Work unit = a block of P consecutive output planes of one (ht x wt)
//    plane tile. Persistent CTAs (one per SM) walk the units.
//  * Each input plane of the block (P + k - 1 of them) is loaded ONCE, as
//    "chunk planes": for every 8-channel chunk, the (ht+k-1) x (wt+k-1) halo
//    brick with 16 bytes per position. Four producer warps gather it with
//    coalesced 16-byte cp.async copies (zero fill = the conv padding); TMA is
//    not used for activations because its rate is about one box row per
//    clock and the rows here are only 16 bytes wide.
//  * GEMM rows are brick positions p = hh*(wt+k-1) + ww ("padded grid"): a tap
//    (kh, kw) is a constant shift of the A start address, so the k*k taps of
//    a plane read the same brick. Rows with ww >= wt or hh >= ht are junk.
//  * kd is folded into N: input plane j feeds output planes j-kd (kd = 0..k-1)
//    of the block, so one tcgen05.mma (M = 128, N = slots * Cout_pad <= 256)
//    updates up to three output-plane accumulators. This matters because an
//    M=128 K=16 MMA costs ~45 SM clocks whatever N <= 48 is (shared-memory
//    operand fetch), so N=32 alone would cap the tensor pipe near 35%.
//  * K = 16 = two 8-channel core-matrix columns at distance LBO. Even chunk
//    counts pair (c, c+1); odd chunk counts (Cin = 24) pair taps instead:
//    (kw, kw+1) are 16 B apart, (kh, kh+1) one brick row apart; a final single
//    chunk pairs with a zero-weight half.
//  * fp32 accumulators live in TMEM ([set][tile][slot][Cout_pad] columns,
//    double-buffered when they fit); four epilogue warps read them with
//    tcgen05.ld, add bias, round and store NDHWC.
//
// Warp roles (416 threads): warps 0-7 producers, warp 8 MMA issuer + TMEM
// owner, warps 9-12 epilogue (TMEM lane quarter = warp % 4). Every wait is
// bounded (1 s); a timeout sets the device error flag and the kernel winds
// down (copies drained, TMEM released) instead of hanging.
#include <cuda.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "r4c_internal.h"
#include "r4c_sm100.cuh"

namespace r4c {

__device__ int g_r4c_dev_error = 0;

namespace tc {

constexpr int kMaxSteps = 64;
constexpr int kMaxStages = 8;
constexpr int kMaxMt = 8;  // M tiles per unit (the issue loop is unrolled over them)
constexpr int kMaxEntries = 8;  // 16-byte copies per producer thread per brick row
constexpr int kProducerWarps = 4;  // 8 warps copy faster alone (15.2 vs 11.4 B/clk/SM) but measured no faster in the kernel
constexpr int kProducerThreads = 32 * kProducerWarps;
constexpr int kMmaWarp = kProducerWarps;
constexpr int kThreads = kProducerThreads + 32 + 128;
constexpr int kSmemMax = 232448;  // 227 KB opt-in dynamic shared memory
constexpr int kHeader = 2048;     // barriers + bias

struct TcConvArgs {
  const void* x;
  const uint8_t* wpack;
  const void* bias;
  void* y;
  int n, d, h, w, cin;
  int od, oh, ow, cout;
  int pd, ph, pw, ks;
  int ht, wt, nht, nwt, nzb;
  int pitch_w, pitch_h;
  int slot_w, P, nin, fold;
  int G, ngroups, nsteps;
  int mtiles, nsets;
  int cpb, a_bytes, b_bytes, stage_bytes, stages;
  int wres, wres_bytes;
  int tmem_cols;
  long long units;
  uint32_t idesc[4];  // N = 1..3 slots
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

// K steps of one (input plane, chunk group) stage: which two 8-channel
// halves each K=16 step reads, the A offset of its first half and the
// distance (LBO) to its second half.
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
    for (int kh = 0; kh < 3; ++kh)
      for (int c = 0; c < G; ++c)
        st.push_back(Step{{ref(kh, 0, c), ref(kh, 1, c)}, off(kh, 0, c), 16});
    for (int c = 0; c < G; ++c)
      st.push_back(Step{{ref(0, 2, c), ref(1, 2, c)}, off(0, 2, c), pitch_w * 16});
    for (int j = 0; j < (G - 1) / 2; ++j)
      st.push_back(Step{{ref(2, 2, 2 * j), ref(2, 2, 2 * j + 1)}, off(2, 2, 2 * j), cpb});
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

// Clocks of one M=128 K=16 MMA with N columns when issued back to back
// (measured on B200: 45 for N <= 32, 56 for 96, 64 for 128, 128 for 256).
static double mma_clk(int n) { return std::max({n / 2.0, 40.0 + n / 6.0, 45.0}); }

// Tuning override: R4C_TC_PLAN="ht=4,nw=8,P=8,G=3,wres=1,stages=4" limits
// the search to candidates with the given values (any subset of the keys;
// stages caps the stage count). Unset keys are searched as usual.
struct PlanForce {
  int ht = 0, nw = 0, P = 0, G = 0, wres = -1, stages = 0;
};
static PlanForce plan_force() {
  PlanForce f;
  const char* e = getenv("R4C_TC_PLAN");
  if (!e) return f;
  char key[16];
  int val = 0, used = 0;
  while (*e && sscanf(e, " %15[a-zA-Z_] = %d%n", key, &val, &used) == 2) {
    if (!strcmp(key, "ht")) f.ht = val;
    else if (!strcmp(key, "nw")) f.nw = val;
    else if (!strcmp(key, "P")) f.P = val;
    else if (!strcmp(key, "G")) f.G = val;
    else if (!strcmp(key, "wres")) f.wres = val;
    else if (!strcmp(key, "stages")) f.stages = val;
    e += used;
    while (*e == ',' || *e == ' ') ++e;
  }
  return f;
}

// Every feasible plan of the conv, with its modelled cost in est_cycles, is
// passed to visit(). G_only > 0 restricts the chunk group size (the packed
// weight layout depends on G only).
template <typename F>
static void enumerate_plans(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw, int G_only,
                            const PlanForce& force, F&& visit) {
  ConvPlan P{};
  P.ok = false;
  if (ks != 1 && ks != 3) return;
  if (cin % 8 != 0 || cin <= 0 || cout <= 0 || cout > 256) return;
  if (n <= 0 || d <= 0 || h <= 0 || w <= 0) return;
  P.od = d + 2 * pd - (ks - 1);
  P.oh = h + 2 * ph - (ks - 1);
  P.ow = w + 2 * pw - (ks - 1);
  if (P.od <= 0 || P.oh <= 0 || P.ow <= 0) return;
  if (pd > 8 || ph > 8 || pw > 8 || pd < -8 || ph < -8 || pw < -8) return;
  P.n = n; P.d = d; P.h = h; P.w = w;
  P.cin = cin; P.cout = cout; P.ks = ks; P.pd = pd; P.ph = ph; P.pw = pw;
  P.c8 = cin / 8;
  P.npad = round_up(cout, 16);
  P.fold = std::max(1, std::min(ks, 256 / P.npad));

  std::vector<int> gs;
  if (P.c8 % 2 == 1) {
    if (P.c8 > 13) return;
    gs.push_back(P.c8);
  } else {
    for (int g = std::min(P.c8, 14); g >= 2; g -= 2)
      if (P.c8 % g == 0) gs.push_back(g);
  }
  const int wt_max = 254 - (ks - 1);
  const int nw_min = (P.ow + wt_max - 1) / wt_max;
  const int sms = num_sms();

  for (int G : gs) {
    if (force.G && G != force.G) continue;
    if (G_only > 0 && G != G_only) continue;
    const int nsteps = steps_per_stage(ks, G);
    if (nsteps > kMaxSteps) continue;
    const int ngroups = P.c8 / G;
    const int b_bytes = nsteps * 2 * ks * P.npad * 16;
    const int wbytes = ngroups * b_bytes;
    // a brick row (wt + k - 1 positions x G chunks) must fit the producers'
    // fixed per-thread copy slots
    const int wt_cap = kMaxEntries * kProducerThreads / G - (ks - 1);
    if (wt_cap < 1) continue;
    const int nw_lo = std::max(nw_min, (P.ow + wt_cap - 1) / wt_cap);
    const int nw_a = force.nw ? force.nw : nw_lo, nw_b = force.nw ? force.nw : nw_lo + 8;
    for (int nw = nw_a; nw <= nw_b && nw <= P.ow; ++nw) {
     const int wt = (P.ow + nw - 1) / nw;
     // the kernel decodes ceil(ow / wt) tiles per row; skip counts that differ
     if ((P.ow + wt - 1) / wt != nw) continue;
     const int entries = ((wt + ks - 1) * G + kProducerThreads - 1) / kProducerThreads;
     if (entries > kMaxEntries) continue;
     for (int wres = 1; wres >= 0; --wres) {
      if (force.wres >= 0 && wres != force.wres) continue;
      if (wres && wbytes > 96 * 1024) continue;
      for (int ht = 1; ht <= P.oh && ht <= 254 - (ks - 1); ++ht) {
        if (force.ht && ht != force.ht) continue;
        const int pitch_w = wt + ks - 1, pitch_h = ht + ks - 1;
        const int span = (ht - 1) * pitch_w + wt;
        const int mtiles = (span + 127) / 128;
        if (mtiles * P.npad > 512 || mtiles > kMaxMt) break;
        const int cpb = round_up(pitch_h * pitch_w * 16, 128);
        const int maxrow = 128 * mtiles - 1 + (ks - 1) * (pitch_w + 1);
        const int pad = round_up(std::max(0, (maxrow + 1) * 16 - cpb), 128);
        const int a_bytes = 128 + G * cpb + pad;
        const int avail = kSmemMax - kHeader - (wres ? round_up(wbytes, 128) : 0);
        const int tiles_h = (P.oh + ht - 1) / ht;
        for (int Pb = 1; Pb <= std::min(P.od, 16); ++Pb) {
          if (force.P && Pb != force.P) continue;
          // a stage holds the A brick and, unless resident, the weight slots
          // of the output planes its input plane feeds (at most min(ks, Pb))
          const int sb = std::min(ks, Pb) * nsteps * 2 * P.npad * 16;
          const int stage = round_up(a_bytes + (wres ? 0 : sb), 128);
          const int stages = std::min(force.stages ? force.stages : kMaxStages, std::min(kMaxStages, avail / stage));
          if (stages < 2) break;
          int nsets = 2;
          if (2 * Pb * P.npad * mtiles > 512) nsets = 1;
          if (Pb * P.npad * mtiles > 512) break;
          const int nin = Pb + ks - 1;
          // MMA clocks per unit: every input plane, every K step, every tile
          double mma = 0.0;
          for (int j = 0; j < nin; ++j) {
            const int lo = std::max(0, j - ks + 1), hi = std::min(Pb - 1, j);
            int ns = hi - lo + 1;
            double t = 0.0;
            while (ns > 0) {
              const int k = std::min(ns, P.fold);
              t += mma_clk(k * P.npad);
              ns -= k;
            }
            mma += t * nsteps * mtiles * ngroups;
          }
          // producer clocks per stage (measured on B200): the halo brick
          // arrives by 16-byte cp.async at ~3 B/clk per producer warp that
          // has copies in a brick row (11.4 B/clk per SM with four), plus
          // ~40 clk of addressing per row; the staged weight slots arrive by
          // bulk copies at ~30 B/clk, in parallel
          const int busy_warps = std::min(kProducerWarps, (pitch_w * G + 31) / 32);
          const double cp_rate = std::min(11.4, 3.0 * busy_warps);
          const double load =
              (double)nin * ngroups *
              (std::max(G * pitch_h * pitch_w * 16.0 / cp_rate + 40.0 * pitch_h, wres ? 0.0 : sb / 30.0) + 150.0);
          // epilogue clocks per unit: per (tile, plane) the TMEM reads (one
          // wait per 32 columns), 16-byte stores of 8 channels, addressing
          const double epi = (double)Pb * mtiles * (((P.npad + 31) / 32) * 100.0 + ((cout + 7) / 8) * 12.0 + 40.0);
          double t_unit = std::max(mma, load) + 100.0 * nin * ngroups;
          t_unit = nsets == 2 ? std::max(t_unit, epi) : t_unit + epi;
          const long long units = (long long)n * ((P.od + Pb - 1) / Pb) * tiles_h * nw;
          const long long waves = (units + sms - 1) / sms;
          const double est = (double)waves * t_unit;
          {
            P.G = G; P.ngroups = ngroups; P.nsteps = nsteps;
            P.wt = wt; P.ht = ht; P.pitch_w = pitch_w; P.pitch_h = pitch_h;
            P.cpb = cpb; P.mtiles = mtiles; P.nsets = nsets;
            P.P = Pb; P.nin = nin;
            P.a_bytes = a_bytes; P.b_bytes = b_bytes; P.stage_bytes = stage; P.stages = stages;
            P.wres = wres; P.wres_bytes = wres ? round_up(wbytes, 128) : 0;
            P.smem_bytes = kHeader + P.wres_bytes + stages * stage;
            const int cols = nsets * Pb * P.npad * mtiles;
            int alloc = 32;
            while (alloc < cols) alloc *= 2;
            P.tmem_cols = alloc;
            P.work_units = units;
            P.grid = (int)std::min<long long>(units, sms);
            P.est_cycles = est;
            P.ok = true;
            visit(static_cast<const ConvPlan&>(P));
          }
        }
      }
     }
    }
  }
}

struct PlanKey {
  int v[12];
  bool operator<(const PlanKey& o) const { return std::lexicographical_compare(v, v + 12, o.v, o.v + 12); }
};

// Best plan by the cost model; cached per shape and device (the search
// visits thousands of candidates) unless the tuning override is set.
bool plan_conv(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw, ConvPlan* pl) {
  static std::map<PlanKey, ConvPlan> cache;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  const PlanKey key{{n, d, h, w, cin, cout, ks, pd, ph, pw, dev, 0}};
  const PlanForce force = plan_force();
  const bool forced = getenv("R4C_TC_PLAN") != nullptr;
  if (!forced) {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      if (!it->second.ok) return false;
      if (pl) *pl = it->second;
      return true;
    }
  }
  ConvPlan best{};
  best.ok = false;
  enumerate_plans(n, d, h, w, cin, cout, ks, pd, ph, pw, 0, force, [&](const ConvPlan& c) {
    if (!best.ok || c.est_cycles < best.est_cycles) best = c;
  });
  if (!forced) {
    std::lock_guard<std::mutex> lk(mu);
    cache[key] = best;
  }
  if (!best.ok) return false;
  if (pl) *pl = best;
  return true;
}

// Candidates for on-device tuning: the plans with the model's chunk group
// size G (same packed weights, bit-identical results) ranked by modelled
// cost, top `k_top`, plus the cheapest of each brick-row count so that a
// model error in the halo/row trade-off cannot hide the fastest shape.
static std::vector<ConvPlan> plan_candidates(const ConvPlan& m, int k_top) {
  std::vector<ConvPlan> all;
  PlanForce none;
  enumerate_plans(m.n, m.d, m.h, m.w, m.cin, m.cout, m.ks, m.pd, m.ph, m.pw, m.G, none,
                  [&](const ConvPlan& c) { all.push_back(c); });
  std::sort(all.begin(), all.end(), [](const ConvPlan& a, const ConvPlan& b) { return a.est_cycles < b.est_cycles; });
  std::vector<ConvPlan> out;
  auto same = [](const ConvPlan& a, const ConvPlan& b) {
    return a.ht == b.ht && a.wt == b.wt && a.P == b.P && a.wres == b.wres && a.stages == b.stages;
  };
  auto add = [&](const ConvPlan& c) {
    for (const ConvPlan& o : out)
      if (same(o, c)) return;
    out.push_back(c);
  };
  for (size_t i = 0; i < all.size() && (int)out.size() < k_top; ++i) add(all[i]);
  for (int ht : {1, 2, 4, 8, 16}) {
    for (const ConvPlan& c : all)
      if (c.ht == ht) { add(c); break; }
  }
  return out;
}

size_t packed_bytes(const ConvPlan& P) { return (size_t)P.ngroups * P.b_bytes; }

// ---------------------------------------------------------------------------
// Weight pack: PyTorch OIDHW -> per chunk group, per K step:
// [half][slot b (kd = ks-1-b)][npad rows][8 elements]
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
  const long long total = (long long)a.ngroups * a.nsteps * 2 * a.ks * a.npad * 8;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int e = (int)(i % 8);
  long long r = i / 8;
  const int nrow = (int)(r % a.npad); r /= a.npad;
  const int b = (int)(r % a.ks); r /= a.ks;
  const int half = (int)(r % 2); r /= 2;
  const int j = (int)(r % a.nsteps);
  const int g = (int)(r / a.nsteps);
  const int kd = a.ks - 1 - b;
  float v = 0.f;
  if (!a.zero[j][half] && nrow < a.cout) {
    const int ci = (g * a.G + a.c[j][half]) * 8 + e;
    if (ci < a.cin_real) {
      const int T = a.ks * a.ks * a.ks;
      const int tap = (kd * a.ks + a.kh[j][half]) * a.ks + a.kw[j][half];
      long long s;
      if (!a.flip) s = ((long long)nrow * a.src_cin + ci) * T + tap;           // W[co=nrow][ci][tap]
      else s = ((long long)ci * a.src_cin + nrow) * T + (T - 1 - tap);         // W[co=ci][ci'=nrow][T-1-tap]
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
  const long long total = (long long)a.ngroups * a.nsteps * 2 * a.ks * a.npad * 8;
  const unsigned blocks = (unsigned)((total + 255) / 256);
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

// Store NV (16 or 32) accumulator columns starting at channel cc of one
// output row: bias added, rounded to T; every complete 8-channel group inside
// cout goes out as one 16-byte store when the row is 16-byte aligned.
template <typename T, int NV>
__device__ __forceinline__ void store_row(T* dst, const float (&v)[NV], const float* bias, int cc, int cout,
                                          bool vec_ok) {
#pragma unroll
  for (int g = 0; g < NV / 8; ++g) {
    const int c0 = cc + 8 * g;
    if (c0 >= cout) break;
    if (vec_ok && c0 + 8 <= cout) {
      uint32_t pk[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        T lo = Elem<T>::from_f(v[8 * g + 2 * i] + bias[c0 + 2 * i]);
        T hi = Elem<T>::from_f(v[8 * g + 2 * i + 1] + bias[c0 + 2 * i + 1]);
        pk[i] = (uint32_t)(*reinterpret_cast<uint16_t*>(&lo)) |
                ((uint32_t)(*reinterpret_cast<uint16_t*>(&hi)) << 16);
      }
      *reinterpret_cast<uint4*>(dst + c0) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (c0 + i < cout) dst[c0 + i] = Elem<T>::from_f(v[8 * g + i] + bias[c0 + i]);
    }
  }
}

// MMA issue for the nsteps K steps of one stage (one thread). MT tiles x NS slot segments per step are
// fully unrolled and four steps go per loop iteration: a loop iteration
// costs the issuing warp a ~40-clock bubble (branch resolution after an
// MMA), which straight-line MMAs hide, so one MMA per iteration runs at
// ~105 clocks instead of the tensor pipe's 56-64 (measured on B200).
//   adlo[s]  : low descriptor word of step s (A address field, biased by one
//              16-byte unit, and LBO), relative to the stage base sA4
//   bd0      : B descriptor of step 0; step s adds s * bstep
//   dk, bk, ik: TMEM column offset, B offset (16-byte units) and
//              instruction descriptor of slot segment k
// Every MMA accumulates: the epilogue zeroes the accumulators it drains.
template <int MT, int NS>
__device__ __forceinline__ void issue_steps(const uint32_t* __restrict__ adlo, int nsteps, uint32_t sA4,
                                            uint64_t bd0, uint64_t bstep, uint32_t dbase, uint32_t tile_cols,
                                            uint32_t d0, uint32_t d1, uint32_t d2, uint32_t b0, uint32_t b1,
                                            uint32_t b2, uint32_t i0, uint32_t i1, uint32_t i2) {
  constexpr uint64_t kAHi = (uint64_t)((128u >> 4) | (1u << 14)) << 32;  // SBO 128 B, version 1
  constexpr int U = (MT * NS >= 4) ? 1 : ((MT * NS >= 2) ? 2 : 4);
  const uint32_t dk[3] = {dbase + d0, dbase + d1, dbase + d2};
  const uint32_t bk[3] = {b0, b1, b2};
  const uint32_t ik[3] = {i0, i1, i2};
  int s = 0;
#pragma unroll 1
  for (; s + U <= nsteps; s += U) {
#pragma unroll
    for (int q = 0; q < U; ++q) {
      const uint64_t ad = kAHi | (uint64_t)(adlo[s + q] + sA4);
      const uint64_t bd = bd0 + (uint64_t)(s + q) * bstep;
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int k = 0; k < NS; ++k)
          mma_f16_ss(dk[k] + (uint32_t)t * tile_cols, ad + (uint64_t)(t * 128), bd + bk[k], ik[k], 1u);
    }
  }
#pragma unroll 1
  for (; s < nsteps; ++s) {
    const uint64_t ad = kAHi | (uint64_t)(adlo[s] + sA4);
    const uint64_t bd = bd0 + (uint64_t)s * bstep;
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int k = 0; k < NS; ++k)
        mma_f16_ss(dk[k] + (uint32_t)t * tile_cols, ad + (uint64_t)(t * 128), bd + bk[k], ik[k], 1u);
  }
}

#define R4C_ISSUE_ARGS adlo, nsteps, sA4, bd0, bstep, dbase, tile_cols, d0, d1, d2, b0, b1, b2, i0, i1, i2

template <int MT>
__device__ __forceinline__ void issue_ns(int ns, const uint32_t* adlo, int nsteps, uint32_t sA4, uint64_t bd0,
                                         uint64_t bstep, uint32_t dbase, uint32_t tile_cols, uint32_t d0,
                                         uint32_t d1, uint32_t d2, uint32_t b0, uint32_t b1, uint32_t b2,
                                         uint32_t i0, uint32_t i1, uint32_t i2) {
  switch (ns) {
    case 1: issue_steps<MT, 1>(R4C_ISSUE_ARGS); break;
    case 2: issue_steps<MT, 2>(R4C_ISSUE_ARGS); break;
    default: issue_steps<MT, 3>(R4C_ISSUE_ARGS); break;
  }
}

__device__ __forceinline__ void issue(int mt, int ns, const uint32_t* adlo, int nsteps, uint32_t sA4, uint64_t bd0,
                                      uint64_t bstep, uint32_t dbase, uint32_t tile_cols, uint32_t d0, uint32_t d1,
                                      uint32_t d2, uint32_t b0, uint32_t b1, uint32_t b2, uint32_t i0, uint32_t i1,
                                      uint32_t i2) {
  switch (mt) {
    case 1: issue_ns<1>(ns, R4C_ISSUE_ARGS); break;
    case 2: issue_ns<2>(ns, R4C_ISSUE_ARGS); break;
    case 3: issue_ns<3>(ns, R4C_ISSUE_ARGS); break;
    case 4: issue_ns<4>(ns, R4C_ISSUE_ARGS); break;
    case 5: issue_ns<5>(ns, R4C_ISSUE_ARGS); break;
    case 6: issue_ns<6>(ns, R4C_ISSUE_ARGS); break;
    case 7: issue_ns<7>(ns, R4C_ISSUE_ARGS); break;
    default: issue_ns<8>(ns, R4C_ISSUE_ARGS); break;
  }
}
#undef R4C_ISSUE_ARGS

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
  // low 32 bits of each K step's A descriptor relative to the stage base:
  // ((a_off + 16) >> 4) in the address field (offsets start at -16 B, so they
  // are biased by one 16-byte unit to stay non-negative) and the step's LBO
  uint32_t* s_adlo = reinterpret_cast<uint32_t*>(smem + 512);
  uint8_t* wres_smem = smem + kHeader;
  uint8_t* stage0 = smem + kHeader + a.wres_bytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Bulk copies need 16-byte aligned shared memory; keep the whole layout on
  // 128-byte boundaries from the base.
  if ((smem_u32(smem) & 127u) != 0u || a.tmem_cols > 512) {
    if (threadIdx.x == 0) atomicExch(&g_r4c_dev_error, 2);
    return;
  }

  // One-time set-up: zero the stage buffers (guard rows, inter-plane gaps and
  // the overrun pad are read by junk GEMM rows only, but keep them finite),
  // stage the bias as fp32, init barriers, allocate TMEM.
  {
    const uint4 z = make_uint4(0, 0, 0, 0);
    const int total = a.stages * a.stage_bytes;
    for (int i = threadIdx.x * 16; i < total; i += kThreads * 16) *reinterpret_cast<uint4*>(stage0 + i) = z;
    const T* bias = static_cast<const T*>(a.bias);
    for (int i = threadIdx.x; i < a.slot_w; i += kThreads)
      sbias[i] = (bias != nullptr && i < a.cout) ? Elem<T>::to_f(bias[i]) : 0.f;
    for (int i = threadIdx.x; i < a.nsteps; i += kThreads)
      s_adlo[i] = (uint32_t)(((a.a_off[i] + 16) >> 4) & 0x3FFF) | ((uint32_t)((a.lbo[i] >> 4) & 0x3FFF) << 16);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      // one (asynchronous) arrival per producer thread, plus the weight copy
      mbar_init(&full[s], kProducerThreads + (a.wres ? 0 : 1));
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
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, (uint32_t)a.tmem_cols);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const long long units = a.units;
  const uint64_t kWaitNs = 1000000000ull;  // 1 s per wait
  // Bounded wait. `nap` > 0 makes the polling thread sleep between polls so
  // that warps which only wait (producers, epilogue) leave issue slots to the
  // MMA warp; the MMA issuer polls without sleeping.
  auto wait = [&](uint64_t* bar, uint32_t par, uint32_t nap = 0) -> bool {
    const uint64_t deadline = global_timer_ns() + kWaitNs;
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, par)) {
      if (nap) __nanosleep(nap);
      if (((++spins) & 63u) == 0) {
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
  const int set_cols = a.P * a.slot_w * a.mtiles;

  if (warp < kProducerWarps) {
    // ---------------- producers: cp.async gather of the halo bricks ----------------
    const int pt = threadIdx.x;
    const T* __restrict__ x = static_cast<const T*>(a.x);
    // A brick row is pitch_w positions x G chunks = per_row 16-byte copies;
    // copy q goes to thread q % 128 as its entry q / 128 (at most kMaxEntries,
    // which the planner guarantees). Consecutive threads take consecutive
    // chunks of a position, so a warp reads 512 contiguous bytes. The
    // shared/global offsets of every entry are fixed for the whole kernel,
    // so a copy costs a handful of independent instructions.
    const int per_row = a.pitch_w * a.G;
    uint32_t soff[kMaxEntries];
    int goff[kMaxEntries], wpos[kMaxEntries];
    uint32_t qmask = 0;
#pragma unroll
    for (int e = 0; e < kMaxEntries; ++e) {
      const int q = pt + e * kProducerThreads;
      const int ww = q / a.G, c = q - (q / a.G) * a.G;
      soff[e] = (uint32_t)(c * a.cpb + ww * 16);
      goff[e] = ww * a.cin + c * 8;
      wpos[e] = ww;
      if (q < per_row) qmask |= 1u << e;
    }
    if (pt == 0 && a.wres) {
      const uint32_t wb = (uint32_t)(a.ngroups * a.b_bytes);
      mbar_arrive_expect_tx(wbar, wb);
      bulk_load(wres_smem, a.wpack, wb, wbar);
    }
    int stage = 0;
    uint32_t epar = 1;
    bool ok = true;
    for (long long u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const int wi = (int)(u % a.nwt);
      long long r = u / a.nwt;
      const int hi = (int)(r % a.nht); r /= a.nht;
      const int zb = (int)(r % a.nzb);
      const int nb = (int)(r / a.nzb);
      const int h0 = hi * a.ht - a.ph, w0 = wi * a.wt - a.pw;
      // entries whose input column lies inside the image for this unit
      uint32_t wmask = 0;
#pragma unroll
      for (int e = 0; e < kMaxEntries; ++e) {
        const int iw = w0 + wpos[e];
        if (((qmask >> e) & 1u) && iw >= 0 && iw < a.w) wmask |= 1u << e;
      }
      const long long wofs = (long long)w0 * a.cin;  // may be negative; only added to in-image offsets
      for (int j = 0; j < a.nin && ok; ++j) {
        const int iz = zb * a.P - a.pd + j;
        const bool z_ok = iz >= 0 && iz < a.d;
        for (int g = 0; g < a.ngroups; ++g) {
          int got = 1;
          if (lane == 0) got = wait(&empty[stage], epar, 64) ? 1 : 0;
          got = __shfl_sync(0xffffffffu, got, 0);
          if (!got) { ok = false; break; }
          uint8_t* sbase = stage0 + (size_t)stage * a.stage_bytes;
          const uint32_t sA = smem_u32(sbase) + 128u;
          for (int hh = 0; hh < a.pitch_h; ++hh) {
            const int ih = h0 + hh;
            const bool r_ok = z_ok && ih >= 0 && ih < a.h;
            const uint32_t m = r_ok ? wmask : 0u;
            const long long rbase =
                (((long long)nb * a.d + (r_ok ? iz : 0)) * a.h + (r_ok ? ih : 0)) * a.w * a.cin + wofs + g * a.G * 8;
            const uint32_t drow = sA + (uint32_t)(hh * a.pitch_w * 16);
#pragma unroll
            for (int e = 0; e < kMaxEntries; ++e) {
              if ((qmask >> e) & 1u) {
                const bool v = (m >> e) & 1u;
                const T* src = v ? x + (rbase + goff[e]) : x;
                cp_async_16(drow + soff[e], src, v ? 16u : 0u);
              }
            }
          }
          cp_async_commit();
          if (pt == 0 && !a.wres) {
            // weight rows of slots [lo, hi] for every K step and half:
            // global [g][step][half][ks slots][rows] -> smem [step][half][nsl slots][rows]
            const int lo = max(0, j - a.ks + 1), hi = min(a.P - 1, j);
            const int nsl = hi - lo + 1, b0 = (a.ks - 1) - (j - lo);
            const uint32_t slot_bytes = (uint32_t)(a.slot_w * 16);
            mbar_arrive_expect_tx(&full[stage], (uint32_t)(a.nsteps * 2 * nsl) * slot_bytes);
            const uint8_t* gsrc = a.wpack + (size_t)g * a.b_bytes + (size_t)b0 * slot_bytes;
            uint8_t* sdst = sbase + a.a_bytes;
            for (int sh = 0; sh < 2 * a.nsteps; ++sh)
              bulk_load(sdst + (size_t)sh * nsl * slot_bytes, gsrc + (size_t)sh * a.ks * slot_bytes,
                        (uint32_t)nsl * slot_bytes, &full[stage]);
          }
          // this thread's copies of the stage arrive on its full barrier when they land
          cp_async_arrive_noinc(&full[stage]);
          if (++stage == a.stages) { stage = 0; epar ^= 1; }
        }
      }
    }
    // no copy may outlive the CTA
    cp_async_wait<0>();
    if (pt == 0 && a.wres) {
      // no bulk copy may outlive the CTA: wait (bounded) for the weight copy
      const uint64_t dl = global_timer_ns() + kWaitNs;
      while (!mbar_try_wait(wbar, 0) && global_timer_ns() < dl) {
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer (lane 0) ----------------
    // One thread issues. A warp-wide issuer (elected lane, uniform
    // descriptors) issues each MMA slightly faster in isolation, but its 31
    // idle lanes wait in warp-synchronous instructions that take issue slots
    // from the producer warp sharing the sub-partition; measured slower.
    if (lane == 0) {
    int stage = 0;
    uint32_t fpar = 0;
    uint32_t tpar[2] = {0, 0};  // phase 0 of tempty = the epilogue's initial zeroing
    int set = 0;
    bool ok = true;
    if (a.wres && !wait(wbar, 0)) ok = false;
    const uint32_t bslot = (uint32_t)(a.slot_w * 16);  // bytes of one slot's B rows
    const int ks = a.ks, Pb = a.P, slot_w = a.slot_w, mtiles = a.mtiles, nsteps = a.nsteps;
    const int fold = a.fold, ngroups = a.ngroups, nin = a.nin;
    const uint32_t tile_cols = (uint32_t)(Pb * slot_w);
    for (long long u = blockIdx.x; u < units && ok; u += gridDim.x) {
      if (!wait(&tempty[set], tpar[set])) { ok = false; break; }
      tpar[set] ^= 1;
      tc_fence_after();
      const uint32_t dset = tmem + (uint32_t)(set * set_cols);
      for (int j = 0; j < nin && ok; ++j) {
        // input plane j feeds output slots lo..hi; one MMA per run of at
        // most `fold` slots (their B rows are adjacent: slot o uses the
        // weights of kd = j - o, stored in reverse kd order)
        const int lo = max(0, j - ks + 1), hi = min(Pb - 1, j);
        const int b0 = (ks - 1) - (j - lo);
        const int nsl = hi - lo + 1;
        uint32_t dd[3] = {0, 0, 0}, bb[3] = {0, 0, 0}, ii[3] = {0, 0, 0};
        int ns = 0;
        for (int o = lo; o <= hi && ns < 3; ++ns) {
          const int n = min(fold, hi - o + 1);
          dd[ns] = (uint32_t)(o * slot_w);
          bb[ns] = (uint32_t)(((o - lo) * bslot) >> 4);
          ii[ns] = a.idesc[n];
          o += n;
        }
        // resident weights keep all ks slots per (step, half); staged ones
        // only the nsl slots of this input plane
        const int bslots = a.wres ? ks : nsl;
        const uint64_t bstep = (uint64_t)((2 * bslots * bslot) >> 4);
        const uint32_t blbo = (uint32_t)(bslots * bslot);
        for (int g = 0; g < ngroups; ++g) {
          if (!wait(&full[stage], fpar)) { ok = false; break; }
          tc_fence_after();
          // stage A base in 16-byte units, minus the one-unit bias of s_adlo
          const uint32_t sA4 = ((smem_u32(stage0 + (size_t)stage * a.stage_bytes) + 128u) >> 4) - 1u;
          const uint32_t sB = a.wres ? smem_u32(wres_smem + (size_t)g * a.b_bytes) + (uint32_t)b0 * bslot
                                     : smem_u32(stage0 + (size_t)stage * a.stage_bytes + a.a_bytes);
          const uint64_t bdesc = smem_desc(sB, blbo, 128);
          issue(mtiles, ns, s_adlo, nsteps, sA4, bdesc, bstep, dset, tile_cols, dd[0], dd[1], dd[2], bb[0], bb[1],
                bb[2], ii[0], ii[1], ii[2]);
          mma_commit(&empty[stage]);
          if (++stage == a.stages) { stage = 0; fpar ^= 1; }
        }
      }
      if (!ok) break;
      mma_commit(&tfull[set]);
      if (a.nsets == 2) set ^= 1;
    }
    mma_commit(mdone);
    wait(mdone, 0);
    }
  } else {
    // ---------------- epilogue (warps 9..12) ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    T* __restrict__ y = static_cast<T*>(a.y);
    const bool vec_ok = (a.cout % 8) == 0;
    uint32_t fpar[2] = {0, 0};
    int set = 0;
    // Every MMA accumulates, so the accumulators start at zero: this warp
    // zeroes its lane quarter of every set now and of each set it drains,
    // and releases a set (tempty) only after those stores completed.
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    for (int c = 0; c < a.nsets * set_cols; c += 16) tmem_zero_16(tq + (uint32_t)c);
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&tempty[0]);
      mbar_arrive(&tempty[1]);
    }
    for (long long u = blockIdx.x; u < units; u += gridDim.x) {
      const int wi = (int)(u % a.nwt);
      long long r = u / a.nwt;
      const int hi = (int)(r % a.nht); r /= a.nht;
      const int zb = (int)(r % a.nzb);
      const int nb = (int)(r / a.nzb);
      const int h0 = hi * a.ht, w0 = wi * a.wt, z0 = zb * a.P;
      int got = 1;
      if (lane == 0) got = wait(&tfull[set], fpar[set], 128) ? 1 : 0;
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got) break;
      fpar[set] ^= 1;
      tc_fence_after();
      const long long plane = (long long)a.oh * a.ow * a.cout;  // elements per output plane
      T* const yu = y + ((((long long)nb * a.od + z0) * a.oh + h0) * a.ow + w0) * a.cout;
      const int nz = min(a.P, a.od - z0);
      for (int t = 0; t < a.mtiles; ++t) {
        const int p = t * 128 + row;
        const int hh = p / a.pitch_w;
        const int ww = p - hh * a.pitch_w;
        const bool pos_ok = hh < a.ht && ww < a.wt && (h0 + hh) < a.oh && (w0 + ww) < a.ow;
        T* dst = yu + ((long long)hh * a.ow + ww) * a.cout;
        for (int o = 0; o < a.P; ++o, dst += plane) {
          const bool valid = pos_ok && o < nz;
          const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) +
                              (uint32_t)(set * set_cols + t * a.P * a.slot_w + o * a.slot_w);
          int cc = 0;
          for (; cc + 32 <= a.slot_w; cc += 32) {
            float v[32];
            tmem_ld_32(tb + (uint32_t)cc, v);
            tmem_zero_16(tb + (uint32_t)cc);
            tmem_zero_16(tb + (uint32_t)cc + 16u);
            if (valid) store_row<T, 32>(dst, v, sbias, cc, a.cout, vec_ok);
          }
          if (cc < a.slot_w) {
            float v[16];
            tmem_ld_16(tb + (uint32_t)cc, v);
            tmem_zero_16(tb + (uint32_t)cc);
            if (valid) store_row<T, 16>(dst, v, sbias, cc, a.cout, vec_ok);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[set]);
      if (a.nsets == 2) set ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, (uint32_t)a.tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// Host launch.
// ---------------------------------------------------------------------------
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
  static_assert(sizeof(TcConvArgs) <= 4096, "kernel argument block too large");
  TcConvArgs a;
  memset(&a, 0, sizeof(a));
  std::vector<Step> steps;
  build_steps(P.ks, P.G, P.pitch_w, P.cpb, steps);
  a.x = x;
  a.wpack = static_cast<const uint8_t*>(w_packed);
  a.bias = bias;
  a.y = y;
  a.n = P.n; a.d = P.d; a.h = P.h; a.w = P.w; a.cin = P.cin;
  a.od = P.od; a.oh = P.oh; a.ow = P.ow; a.cout = P.cout;
  a.pd = P.pd; a.ph = P.ph; a.pw = P.pw; a.ks = P.ks;
  a.ht = P.ht; a.wt = P.wt;
  a.nht = (P.oh + P.ht - 1) / P.ht;
  a.nwt = (P.ow + P.wt - 1) / P.wt;
  a.nzb = (P.od + P.P - 1) / P.P;
  // the kernel's fixed-size per-thread tables and unrolled issue blocks
  if ((long long)P.n * a.nzb * a.nht * a.nwt != P.work_units) return R4C_ERR_INVALID;
  if ((P.pitch_w * P.G + kProducerThreads - 1) / kProducerThreads > kMaxEntries) return R4C_ERR_INVALID;
  if (P.mtiles < 1 || P.mtiles > kMaxMt) return R4C_ERR_INVALID;
  a.pitch_w = P.pitch_w; a.pitch_h = P.pitch_h;
  a.slot_w = P.npad; a.P = P.P; a.nin = P.nin; a.fold = P.fold;
  a.G = P.G; a.ngroups = P.ngroups; a.nsteps = (int)steps.size();
  a.mtiles = P.mtiles; a.nsets = P.nsets;
  a.cpb = P.cpb; a.a_bytes = P.a_bytes; a.b_bytes = P.b_bytes; a.stage_bytes = P.stage_bytes; a.stages = P.stages;
  a.wres = P.wres; a.wres_bytes = P.wres_bytes;
  a.tmem_cols = P.tmem_cols;
  a.units = P.work_units;
  for (int k = 1; k <= 3; ++k)
    a.idesc[k] = sm100::instr_desc_f16(dtype == R4C_BF16, 128, std::min(256, k * P.npad), 0, 0);
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

// Launch with the fastest plan measured on this device for this shape.
// The first call per (shape, dtype, device) times up to a dozen candidate
// plans that share the model plan's packed-weight layout (so results are
// bit-identical whichever wins) on the caller's buffers and stream, then
// caches the winner; the model's plan is used as is while the stream is
// being captured, when R4C_AUTOTUNE=0, or when R4C_TC_PLAN forces a plan.
static std::map<PlanKey, ConvPlan> g_tuned;
static std::mutex g_tuned_mu;

bool tuned_plan(const ConvPlan& model, int dtype, ConvPlan* out) {
  int dev = 0;
  cudaGetDevice(&dev);
  const PlanKey key{{model.n, model.d, model.h, model.w, model.cin, model.cout, model.ks, model.pd, model.ph,
                     model.pw, dev, dtype}};
  std::lock_guard<std::mutex> lk(g_tuned_mu);
  auto it = g_tuned.find(key);
  if (it == g_tuned.end()) return false;
  if (out) *out = it->second;
  return true;
}

int launch_conv_tuned(const ConvPlan& model, const void* x, const void* w_packed, const void* bias, void* y, int dtype,
                      cudaStream_t st) {
  std::map<PlanKey, ConvPlan>& tuned = g_tuned;
  std::mutex& mu = g_tuned_mu;
  int dev = 0;
  cudaGetDevice(&dev);
  const PlanKey key{{model.n, model.d, model.h, model.w, model.cin, model.cout, model.ks, model.pd, model.ph,
                     model.pw, dev, dtype}};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = tuned.find(key);
    if (it != tuned.end()) return launch_conv(it->second, x, w_packed, bias, y, dtype, st);
  }
  const char* at = getenv("R4C_AUTOTUNE");
  if (getenv("R4C_TC_PLAN") || (at && at[0] == '0')) return launch_conv(model, x, w_packed, bias, y, dtype, st);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
    return launch_conv(model, x, w_packed, bias, y, dtype, st);

  std::vector<ConvPlan> cands = plan_candidates(model, 8);
  if (cands.empty()) cands.push_back(model);
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) {
    if (e0) cudaEventDestroy(e0);
    return launch_conv(model, x, w_packed, bias, y, dtype, st);
  }
  ConvPlan best = model;
  float best_ms = 1e30f;
  int rc = R4C_OK;
  for (const ConvPlan& c : cands) {
    rc = launch_conv(c, x, w_packed, bias, y, dtype, st);  // warm-up (and module load)
    if (rc != R4C_OK) break;
    float ms = 1e30f;
    for (int rep = 0; rep < 2 && rc == R4C_OK; ++rep) {
      cudaEventRecord(e0, st);
      rc = launch_conv(c, x, w_packed, bias, y, dtype, st);
      cudaEventRecord(e1, st);
      if (cudaEventSynchronize(e1) != cudaSuccess) rc = R4C_ERR_CUDA;
      float t = 0.f;
      if (rc == R4C_OK && cudaEventElapsedTime(&t, e0, e1) == cudaSuccess) ms = std::min(ms, t);
    }
    if (rc != R4C_OK) break;
    if (ms < best_ms) {
      best_ms = ms;
      best = c;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc != R4C_OK) return rc;
  {
    std::lock_guard<std::mutex> lk(mu);
    tuned[key] = best;
  }
  return launch_conv(best, x, w_packed, bias, y, dtype, st);
}

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
