// r4c_tc_dw.cu — tcgen05 + TMA weight (and bias) gradient of a stride-1
// Conv3d (k = 1 or 3), split-K over output rows with a fixed-order reduce.
//
// Reference counterpart: _wgrad_kernel + _launch_wgrad + partial.sum(0) and
// the separate db reduction (src/rdna4_conv3d/conv3d_wmma.py:543-634,
// 1182-1214, 1318). The reference keeps taps in the GEMM's N dimension
// (M = Cout, N = k^3*Cin, K = voxels) with masked gathers; here:
//
//  * GEMM per kw: D[(c, kd, kh, ci8), co] += X[v + (kd, kh, kw)][c*8+ci8] *
//    dY[v][co] over the output positions v of one output row (K = 16
//    positions per MMA). Both operands are MN-major in shared memory.
//  * A (M rows): for one output row (n, z, y) and each 8-channel chunk c, ONE
//    TMA box (8 ch x pitch_w x k x k) loads the k x k input rows
//    (z+kd-pad, y+kh-pad) as a chunk plane [kd][kh][w]. The M groups
//    (c, kd, kh) are then k*k*C8 consecutive row blocks at a single stride
//    (pitch_w * 16 B): one descriptor covers 16 groups = one M tile. kw is a
//    16-byte shift of the start address.
//  * B (N columns): the dY row, one TMA box per 8-channel chunk.
//  * db: the group right after the last real one holds bf16 ones, so its
//    accumulator rows (junk rows otherwise) are sum_v dY[v][co].
//  * Each CTA owns one task (a range of M tiles, of N, of kw) for one split of
//    the output rows; fp32 partials go to the caller's workspace and a second
//    kernel sums them in split order into OIDHW dW and db (deterministic).
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer + TMEM
// owner, warps 2-5 epilogue (TMEM lane quarter = warp % 4). All waits are
// bounded (1 s), like r4c_tc.cu.
#include <cuda.h>

#include <stdio.h>
#include <string.h>
#include <stdlib.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "r4c_internal.h"
#include "r4c_sm100.cuh"

namespace r4c {
namespace tcdw {

using namespace r4c::sm100;

constexpr int kThreads = 192;
constexpr int kSmemMax = 232448;
constexpr int kHeader = 1024;
constexpr int kMaxStages = 6;

struct alignas(64) DwArgs {
  CUtensorMap tx;   // x:  dims (cin, w, h, d, n), box (8, pitch_w, k, k, 1)
  CUtensorMap tg;   // dy: dims (cout, ow, oh, od, n), box (8, kpad, 1, 1, 1)
  float* part;      // [S][cout][cin][k^3] fp32
  float* dbpart;    // [S][cout] fp32 (nullptr when db is not produced here)
  int* err;         // device error flag (r4c_device_error)
  int od, oh, ow, cin, cout, ks, pd, ph, pw;
  int c8, pitch_w, kpad, nwt, wt;
  int mt0, mtn, n0, nn, kw0, kwn;   // task ranges (M tiles, N columns, kw)
  int c_lo, c_hi;                    // chunks loaded for the task
  int ones_group;                    // absolute group index of the ones group (or -1)
  int a_bytes, g_bytes, stage_bytes, stages;
  int tmem_cols;
  long long rows;                    // output rows * w-tiles
  long long rows_per_split;
  int ntasks;
  uint32_t idesc;
  // wide mode: input channel groups of cw (16/32/64) in the swizzled MN-major
  // layout, one TMA box (cw, pitch_w, k, k) per group and row: an M tile is
  // apt = 128/cw consecutive (kd, kh) planes of one group (MN atoms, LBO =
  // plane), K groups of 8 positions at SBO = 16*cw bytes. dY boxes of cwb
  // channels, swizzled likewise (cwb = 8: the no-swizzle chunk layout).
  int wide;
  int cw, apt, plane_bytes, lay_a;
  int cwb, b_region, lay_b;
  int nbox, npad_w;                  // dY boxes per stage, MMA N
  int tail_bytes;                    // zeroed bytes past the last stage (M tile over-read)
  // chunk layout with kw folded into N: B holds the dY row three times,
  // shifted by kw = 0, 1, 2 positions (atoms kw * nn/8 + c), A the unshifted
  // input rows; one MMA of N = 3 nn per (M tile, K step)
  int fold;
  int row_bytes;  // one output row's slot in a stage (stage_bytes / rows per stage)
  // k = 1 wide layout with two atoms per M tile: the ones (db) atom is one
  // plane shared by every stage and row slot, at this byte offset from the
  // first stage (0: the per-row ones plane of the stage layout); each row's
  // A descriptor reaches it through its own LBO (shared plane - x plane)
  int ones_off;
};

struct Task {
  int mt0, mtn, n0, nn, kw0, kwn;
  int g;  // wide mode: input channel group (mt0 counts M tiles within it)
};

struct DwPlan {
  bool ok;
  bool wide;
  bool fold;
  int rpst;  // output rows per stage (wide layout: 2 or 4 when a row's boxes are under 32 KB)
  int ones_bytes;  // the shared ones plane (k = 1 wide layout), 0 when the stages hold it
  int cw, apt, tpg, ng, plane_bytes, region_bytes, cwb, nbox, npad_w, tail_bytes;
  int n, d, h, w, od, oh, ow, cin, cout, ks, pd, ph, pw;
  int c8, groups, mtiles, pitch_w, kpad, wt, nwt;
  int mtn, nn, kwn;  // task shape
  std::vector<Task> tasks;
  int S;
  long long rows, rows_per_split;
  int stages, stage_bytes, smem_bytes, tmem_cols;
  bool db_in_kernel;
  double est;
};

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

// Chunks [c_lo, c_hi] that the groups of M tiles [mt0, mt0+mtn) touch.
static void chunk_range(int mt0, int mtn, int k2, int c8, int* lo, int* hi) {
  int g0 = 16 * mt0, g1 = 16 * (mt0 + mtn) - 1;
  *lo = std::min(g0 / k2, c8 - 1);
  *hi = std::min(g1 / k2, c8 - 1);
}

// Clocks per M=128 x N x K=16 MMA with MN-major operands, issued back to back
// from the dW issue loop (measured on B200: ~70-80 for N <= 48; the A read
// bounds small N).
static double dw_mma_clk(int npad) { return std::max(72.0, 40.0 + npad / 2.0); }
// Load-to-use latency of a stage's TMA boxes under the kernel's own load
// (measured on B200 with per-row clock stamps: 2-3 us).
constexpr double kTmaLatencyClk = 5000.0;

static bool plan_dw(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw, DwPlan* out) {
  DwPlan P{};
  P.ok = false;
  if (ks != 1 && ks != 3) return false;
  if (cin % 8 || cout % 8 || cin <= 0 || cout <= 0) return false;
  if (n <= 0 || d <= 0 || h <= 0 || w <= 0) return false;
  if (pd < -8 || pd > 8 || ph < -8 || ph > 8 || pw < -8 || pw > 8) return false;
  P.n = n; P.d = d; P.h = h; P.w = w; P.cin = cin; P.cout = cout; P.ks = ks;
  P.pd = pd; P.ph = ph; P.pw = pw;
  P.od = d + 2 * pd - (ks - 1); P.oh = h + 2 * ph - (ks - 1); P.ow = w + 2 * pw - (ks - 1);
  if (P.od <= 0 || P.oh <= 0 || P.ow <= 0) return false;
  const int k2 = ks * ks;
  P.c8 = cin / 8;
  P.groups = k2 * P.c8;
  // ones group lives right after the real groups; it needs a spare row block
  // in the last M tile.
  P.db_in_kernel = (P.groups % 16) != 0;
  P.mtiles = (P.groups + (P.db_in_kernel ? 1 : 0) + 15) / 16;
  // W tiles: K positions per row must be a multiple of 16 except the last tile
  // (whose tail reads dY out of bounds = zeros), and the x box <= 256 wide.
  int wt = P.ow;
  while (round_up(wt, 16) + 8 > 256) wt = round_up((wt + 1) / 2, 16);
  P.wt = wt;
  P.nwt = (P.ow + wt - 1) / wt;
  P.kpad = round_up(wt, 16);
  P.pitch_w = round_up(P.kpad + ks - 1, 8);
  P.rows = (long long)n * P.od * P.oh * P.nwt;
  const int sms = num_sms();

  // R4C_DW_WIDE=0 / =1 restricts the search to the 8-channel chunk layout /
  // to the wide channel-group layout when the layer allows it.
  const char* wenv = getenv("R4C_DW_WIDE");
  const int wide_force = (wenv && wenv[0] == '0') ? 0 : (wenv && wenv[0] == '1') ? 1 : -1;
  const int cw_ok = cin % 64 == 0 ? 64 : cin % 32 == 0 ? 32 : cin % 16 == 0 ? 16 : 0;
  // Automatic choice of the wide layout. Measured on B200 (trunk layers,
  // batch 4): 192->192 k3 254 -> 210 us and 192->96 k1 83 -> 67 us with
  // 64-channel groups; with 32- and 16-channel groups the chunk layout first
  // won (96->96 206 vs 238 us, 48->48 248 vs 314 us: more M tiles per K step
  // outweigh the fewer TMA rows). R4C_DW_WIDE=1 enables the narrower groups,
  // =0 disables the wide layout.
  // k1 layers (a plain GEMM over positions, TMA-row-bound in the chunk
  // layout) take the wide layout with the channel groups padded up to 64 /
  // 32 / 16 (the TMA zero-fills channels past Cin): one TMA row per position
  // and group.
  const int cw_pad = cin >= 48 ? 64 : cin > 16 ? 32 : 16;
  // Re-measured with the wave-filling split counts: 96->96 k3 with 32-channel
  // groups 223 -> 165 us (chunk -> wide), 48->48 with 16-channel groups still
  // slower (260 vs 287 us); hence 32-channel groups from Cin = 96 up.
  const bool wide_auto = wide_force == -1 &&
                         ((cw_ok == 64 && cin >= 64) || (cw_ok == 32 && cin >= 96) || (ks == 1 && cin >= 16));
  const bool chunk_allowed = !((wide_force == 1 && cin >= 16) || wide_auto);

  // Splits of the output rows: one CTA per (task, split) at one CTA per SM,
  // so the cost is waves x rows per split; the split counts that fill whole
  // waves (1..4) are compared (rounding S up from 2 * SMs / tasks can add a
  // nearly empty third wave).
  auto pick_split = [&](long long rows, int ntasks, double per_row, int* S_out, long long* rps_out) {
    double bc = 1e300;
    for (int k = 1; k <= 4; ++k) {
      int S = (int)std::max<long long>(1, std::min<long long>(rows, (long long)k * sms / ntasks));
      const long long rps = (rows + S - 1) / S;
      S = (int)((rows + rps - 1) / rps);
      const long long waves = ((long long)ntasks * S + sms - 1) / sms;
      const double c = waves * (rps * per_row + 3000.0);
      if (c < bc) {
        bc = c;
        *S_out = S;
        *rps_out = rps;
      }
    }
    return bc;
  };
  // Task shape: largest N split and M-tile group that fits TMEM (512 cols)
  // with all kw in one task when possible.
  double best = 1e300;
  // W tile candidates: the widest, and its half (twice the stages in flight)
  for (int wtc : {wt}) {
    const int nwt_c = (P.ow + wtc - 1) / wtc;
    const int kpad_c = round_up(wtc, 16);
    const int pitch_c = round_up(kpad_c + ks - 1, 8);
    const long long rows_c = (long long)n * P.od * P.oh * nwt_c;
    for (int kwn : {ks, 1}) {
      if (!chunk_allowed) break;
      if (ks % kwn) continue;
      for (int nn = cout; nn >= 8; nn -= 8) {
        if (cout % nn) continue;
        int npad = round_up(nn, 16);
        if (npad > 256) continue;
        for (int mtn = std::min(P.mtiles, 8); mtn >= 1; --mtn) {
          int cols = kwn * mtn * npad;
          if (cols > 512) continue;
          int ntask_m = (P.mtiles + mtn - 1) / mtn;
          int ntasks = ntask_m * (cout / nn) * (ks / kwn);
          // stage bytes: chunks touched by an M group of mtn tiles
          int lo, hi;
          chunk_range(0, mtn, k2, P.c8, &lo, &hi);
          int nch = hi - lo + 2;  // +1 slack for a straddling group range
          if (nch > P.c8) nch = P.c8;
          int a_bytes = (nch * k2 + 1) * pitch_c * 16;
          a_bytes = round_up(a_bytes, 128);
          int g_bytes = (nn / 8) * kpad_c * 16;
          int stage = round_up(a_bytes + g_bytes, 128);
          int tail = 16 * mtn * pitch_c * 16 + 256;
          int stages = std::min(kMaxStages, (kSmemMax - kHeader - tail) / stage);
          if (stages < 2) continue;
          // cost per row per task
          double t_mma = std::max({npad / 2.0, (4096.0 + 32.0 * npad) / 128.0, 44.6});
          double mma = (double)(kpad_c / 16) * kwn * mtn * t_mma;
          double load = (double)(nch * k2 * pitch_c * 16 + g_bytes) / 48.0;
          double per_row = std::max(mma, load) + 60.0;
          int S = 1;
          long long rps = rows_c;
          const double est = pick_split(rows_c, ntasks, per_row, &S, &rps);
          if (est < best) {
            best = est;
            P.wide = false;
            P.fold = false;
            P.wt = wtc; P.nwt = nwt_c; P.kpad = kpad_c; P.pitch_w = pitch_c; P.rows = rows_c;
            P.mtn = mtn; P.nn = nn; P.kwn = kwn;
            P.S = S; P.rows_per_split = rps;
            P.stages = stages; P.stage_bytes = stage;
            P.smem_bytes = kHeader + stages * stage + tail;
            int alloc = 32;
            while (alloc < cols) alloc *= 2;
            P.tmem_cols = alloc;
            P.est = est;
            P.ok = true;
          }
        }
      }
    }
  }
  // kw folded into N (chunk layout, k = 3, one W tile per output row): the
  // stage's B holds three copies of the dY row shifted by kw = 0, 1, 2
  // positions (boxes of the same TMA transaction), A the unshifted input rows
  // over K = ow + 2 positions, so each (M tile, K step) takes one MMA of
  // N = 3 nn instead of three of N = nn. The MN-major A read bounds an MMA's
  // cost (~72 clk up to N ~ 64), so at 24->24 this is 18 instead of 48 MMAs
  // per output row.
  // Opt-in (R4C_DW_FOLD=1, taken whenever the layer allows it): measured on
  // B200 at 24->24 it ran 690 us against 546 for the chunk layout. The
  // 8-channel boxes move 16-byte TMA rows, whose cost is per row (~1 row per
  // clock), and the shifted copies add 28 % rows (5184 against 4056 per
  // output row) while the fewer MMAs no longer bound the row.
  const char* fenv = getenv("R4C_DW_FOLD");
  const int fold_force = (fenv && fenv[0] == '0') ? 0 : (fenv && fenv[0] == '1') ? 1 : -1;
  bool folded = false;
  if (fold_force == 1 && chunk_allowed && ks == 3 && round_up(P.ow + 2, 16) <= 256) {
    if (fold_force == 1) best = 1e300;
    const int kp = round_up(P.ow + 2, 16);
    const long long rows_f = (long long)n * P.od * P.oh;
    for (int nn = cout; nn >= 8; nn -= 8) {
      if (cout % nn) continue;
      const int npad = round_up(3 * nn, 16);
      if (npad > 256) continue;
      for (int mtn = std::min(P.mtiles, 8); mtn >= 1; --mtn) {
        const int cols = mtn * npad;
        if (cols > 512) continue;
        const int ntasks = ((P.mtiles + mtn - 1) / mtn) * (cout / nn);
        int lo, hi;
        chunk_range(0, mtn, k2, P.c8, &lo, &hi);
        int nch = hi - lo + 2;
        if (nch > P.c8) nch = P.c8;
        const int a_bytes = round_up((nch * k2 + 1) * kp * 16, 128);
        const int g_bytes = (npad / 8) * kp * 16;  // the shifted copies + the atoms the MMA's N reads past them
        const int stage = round_up(a_bytes + g_bytes, 128);
        // an M tile reads 16 row blocks from the task's first group, which
        // lies less than k^2 blocks past the A base: the reads past the last
        // stage stay within this zeroed tail
        const int tail = std::max(0, (k2 + 16 * mtn) * kp * 16 - stage) + 256;
        const int stages = std::min(kMaxStages, (kSmemMax - kHeader - tail) / stage);
        if (stages < 2) continue;
        // the chunk layout's MMA model, so that the two compare on one scale
        const double t_mma = std::max({npad / 2.0, (4096.0 + 32.0 * npad) / 128.0, 44.6});
        const double mma = (double)(kp / 16) * mtn * t_mma;
        const double load = (double)(nch * k2 * kp * 16 + 3 * (nn / 8) * kp * 16) / 48.0;
        const double per_row = std::max(mma, load) + 60.0;
        int S = 1;
        long long rps = rows_f;
        const double est = pick_split(rows_f, ntasks, per_row, &S, &rps);
        if (est < best) {
          best = est;
          P.wide = false;
          P.fold = true;
          P.wt = P.ow; P.nwt = 1; P.kpad = kp; P.pitch_w = kp; P.rows = rows_f;
          P.mtn = mtn; P.nn = nn; P.kwn = 3;
          P.S = S; P.rows_per_split = rps;
          P.stages = stages; P.stage_bytes = stage;
          P.smem_bytes = kHeader + stages * stage + tail;
          P.tail_bytes = tail;
          int alloc = 32;
          while (alloc < cols) alloc *= 2;
          P.tmem_cols = alloc;
          P.est = est;
          P.ok = true;
          folded = true;
        }
      }
    }
  }
  // Wide mode (Cin a multiple of 16, at least 32): one swizzled box per
  // channel group and row instead of one 16-byte-row box per 8 channels.
  const int cw = (wide_force == 1 || ks == 1) ? cw_pad : cw_ok;
  if (cin >= 16 && (wide_force == 1 || wide_auto) && !(fold_force == 1 && folded)) {
    const int apt = 128 / cw, atoms = k2 + 1;  // + the ones (group 0) / zero plane
    const int tpg = (atoms + apt - 1) / apt, ng = (cin + cw - 1) / cw;
    // W tile: the chunk layout's, halved until two stages fit
    int wt_w = P.wt;
    auto plane_of = [&](int t) { return round_up(round_up(t, 16) + ks - 1, 8) * cw * 2; };
    while (wt_w > 16 && kHeader + 2 * (round_up(atoms * plane_of(wt_w), 1024) +
                                       round_up(cout * round_up(wt_w, 16) * 2, 1024)) +
                            (tpg * apt - atoms) * plane_of(wt_w) + 1024 > kSmemMax)
      wt_w = round_up((wt_w + 1) / 2, 16);
    const int nwt_w = (P.ow + wt_w - 1) / wt_w;
    const int kpad_w = round_up(wt_w, 16);
    const int pitch_ww = round_up(kpad_w + ks - 1, 8);
    const long long rows_w = (long long)n * P.od * P.oh * nwt_w;
    const int plane = pitch_ww * cw * 2;
    // k = 1, two atoms per tile: the x plane alone per row, one ones plane
    // for the whole ring (its own LBO per row slot)
    const bool shared = ks == 1 && apt == 2;
    const int ones_b = shared ? round_up(plane, 1024) : 0;
    const int region = round_up((shared ? 1 : atoms) * plane, 1024);
    const int tail = (tpg * apt - atoms) * plane + 1024;
    for (int kwn : {1}) {  // one kw per task: keeps the wide issue code (runtime steps) small
      for (int nn = cout; nn >= 8; nn -= 8) {
        if (cout % nn) continue;
        // dY boxes of cwb channels, the last padded (channels past nn are
        // computed and dropped, past Cout zero-filled); MMA N = the boxes
        const int cwb0 = nn % 64 == 0 ? 64 : nn % 32 == 0 ? 32 : nn % 16 == 0 ? 16 : nn <= 16 ? 16 : nn <= 32 ? 32 : 64;
        // k = 1: 64-channel boxes first when they mean fewer boxes (fewer,
        // longer TMA rows, so they win ties: a TMA box row costs ~5 clk
        // whatever its length up to 128 B, measured on the k1 dW rows of
        // 32-96 bytes)
       const bool fewer = ks == 1 && (nn + 63) / 64 < (nn + cwb0 - 1) / cwb0;  // 64-channel boxes save boxes
       for (int cwb : {fewer ? 64 : cwb0, fewer ? cwb0 : 0}) {
        if (cwb == 0) continue;
        const int nbox = (nn + cwb - 1) / cwb;
        const int npad = round_up(nbox * cwb, 16);
        if (npad > 256) continue;
        // the last stage's over-reads past its end stay inside the zeroed
        // tail: A tiles past the group's planes, B chunks past the boxes
        const int tail_nn = std::max(tail, (npad - nbox * cwb) / 8 * kpad_w * 16 + 1024);
        for (int mtn = std::min(tpg, 5); mtn >= 1; --mtn) {
          const int cols = kwn * mtn * npad;
          if (cols > 512) continue;
          const int ntasks = ng * ((tpg + mtn - 1) / mtn) * (cout / nn) * (ks / kwn);
          if (ntasks > 128) continue;
          const int stage = region + round_up(nbox * cwb * kpad_w * 2, 1024);
          const int stages = std::min(kMaxStages, (kSmemMax - kHeader - round_up(tail_nn, 1024) - ones_b) / stage);
          if (stages < 2) continue;
          const double t_mma = dw_mma_clk(npad);
          const double mma = (double)(kpad_w / 16) * kwn * mtn * t_mma;
          const double rows = (double)k2 * pitch_ww + (double)nbox * kpad_w;
          const double bytes = (double)k2 * plane + (double)nbox * cwb * kpad_w * 2;
          const double load = std::max(bytes / 48.0, rows * 2.2);
          const double per_row = std::max(std::max(mma, load) + 60.0, (kTmaLatencyClk + mma) / stages);
          int S = 1;
          long long rps = rows_w;
          const double est = pick_split(rows_w, ntasks, per_row, &S, &rps);
          if (est < best) {
            best = est;
            P.wide = true;
            P.fold = false;
            P.wt = wt_w; P.nwt = nwt_w; P.kpad = kpad_w; P.pitch_w = pitch_ww; P.rows = rows_w;
            P.cw = cw; P.apt = apt; P.tpg = tpg; P.ng = ng; P.plane_bytes = plane; P.region_bytes = region;
            P.cwb = cwb; P.nbox = nbox; P.npad_w = npad; P.tail_bytes = tail_nn;
            P.mtn = mtn; P.nn = nn; P.kwn = kwn;
            P.S = S; P.rows_per_split = rps;
            P.stages = stages; P.stage_bytes = stage;
            P.ones_bytes = ones_b;
            P.smem_bytes = kHeader + stages * stage + round_up(tail_nn, 1024) + ones_b;
            int alloc = 32;
            while (alloc < cols) alloc *= 2;
            P.tmem_cols = alloc;
            P.est = est;
            P.db_in_kernel = true;
            P.ok = true;
          }
        }
       }
      }
    }
  }
  if (!P.ok) return false;
  // Two or four output rows per stage in the wide layout when a row's boxes
  // move less than 32 KB: the TMA's throughput per SM is set by the bytes of
  // each mbarrier transaction (~0.55 us per transaction below ~32 KB). k1
  // layers (10-24 KB per row) are the ones this reaches: four rows while a
  // stage stays within 64 KB and three stages fit. R4C_DW_ROWS=1 keeps one.
  P.rpst = 1;
  if (!P.wide) P.ones_bytes = 0;
  {
    const char* re = getenv("R4C_DW_ROWS");
    if (P.wide && P.stage_bytes < 32768 && !(re && re[0] == '1')) {
      const int row = P.stage_bytes;
      const int fixed = kHeader + round_up(P.tail_bytes, 1024) + P.ones_bytes;
      for (int r : {4, 2}) {
        if (r == 4 && (4 * row > 65536 || (re && re[0] == '2'))) continue;
        const int st = std::min(kMaxStages, (kSmemMax - fixed) / (r * row));
        if (st >= 3) {
          P.rpst = r;
          P.stage_bytes = r * row;
          P.stages = st;
          P.smem_bytes = fixed + st * r * row;
          break;
        }
      }
    }
  }
  P.tasks.clear();
  if (P.wide) {
    for (int g = 0; g < P.ng; ++g)
      for (int mt0 = 0; mt0 < P.tpg; mt0 += P.mtn)
        for (int n0 = 0; n0 < cout; n0 += P.nn)
          for (int kw0 = 0; kw0 < ks; kw0 += P.kwn)
            P.tasks.push_back(Task{mt0, std::min(P.mtn, P.tpg - mt0), n0, P.nn, kw0, P.kwn, g});
  } else {
    for (int mt0 = 0; mt0 < P.mtiles; mt0 += P.mtn)
      for (int n0 = 0; n0 < cout; n0 += P.nn)
        for (int kw0 = 0; kw0 < ks; kw0 += P.kwn)
          P.tasks.push_back(Task{mt0, std::min(P.mtn, P.mtiles - mt0), n0, P.nn, kw0, P.kwn, 0});
  }
  if (out) *out = P;
  return true;
}

// ---------------------------------------------------------------------------
// Kernel
// ---------------------------------------------------------------------------
template <typename T> struct OneBits;
template <> struct OneBits<__nv_bfloat16> { static constexpr uint32_t v = 0x3F803F80u; };  // bf16 1.0 x2
template <> struct OneBits<__half> { static constexpr uint32_t v = 0x3C003C00u; };         // fp16 1.0 x2

struct TaskTable {
  int mt0[128], mtn[128], n0[128], kw0[128], g[128];
};

__device__ __forceinline__ uint64_t desc_layout(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  return smem_desc(addr, lbo, sbo) | ((uint64_t)(layout & 7u) << 61);
}

// MMA issue for one output row (ksteps K steps of 16 positions): every
// (kw, M tile) accumulator takes one MMA per K step. The (kw, tile) block is
// fully unrolled and K steps are unrolled so that a loop iteration carries
// at least four MMAs: the issuing thread's per-iteration bubble (~40 clk)
// otherwise dominates (one MMA per iteration ran at ~210 clk per MMA).
// Descriptor start-address steps (16-byte units) of one operand layout: a K
// step of 16 positions for A and B, a kw shift of A (one position), an M tile.
struct DwSteps {
  uint32_t ks_a, kw_a, tile_a, ks_b;
};

// WIDE = false: the chunk layout's steps are compile-time constants (256 B
// per K step, 16 B per kw), which keeps the issue loop short.
template <int MTN, int KWN, bool WIDE>
__device__ __forceinline__ void dw_step(int ks, uint64_t a0, uint64_t b0, uint32_t tmem, uint32_t npad,
                                        const DwSteps& st, uint32_t idesc, uint32_t acc) {
  const uint32_t ks_a = WIDE ? st.ks_a : 16u, kw_a = WIDE ? st.kw_a : 1u, ks_b = WIDE ? st.ks_b : 16u;
  const uint64_t b = b0 + (uint64_t)(ks * ks_b);
#pragma unroll
  for (int kw = 0; kw < KWN; ++kw)
#pragma unroll
    for (int t = 0; t < MTN; ++t)
      mma_f16_ss(tmem + (uint32_t)(kw * MTN + t) * npad,
                 a0 + (uint64_t)(ks * ks_a + kw * kw_a) + (uint64_t)t * st.tile_a, b, idesc, acc);
}

template <int MTN, int KWN, bool WIDE>
__device__ __forceinline__ void dw_issue_row(uint64_t a0, uint64_t b0, uint32_t tmem, uint32_t npad,
                                             const DwSteps& a_tile, int ksteps, uint32_t idesc, bool first) {
  constexpr int U = (MTN * KWN >= 4) ? 1 : ((MTN * KWN >= 2) ? 2 : 4);
  int ks = 0;
  if (first && ksteps > 0) {  // the task's first K step initialises every accumulator
    dw_step<MTN, KWN, WIDE>(0, a0, b0, tmem, npad, a_tile, idesc, 0u);
    ks = 1;
  }
#pragma unroll 1
  for (; ks + U <= ksteps; ks += U) {
#pragma unroll
    for (int u = 0; u < U; ++u) dw_step<MTN, KWN, WIDE>(ks + u, a0, b0, tmem, npad, a_tile, idesc, 1u);
  }
#pragma unroll 1
  for (; ks < ksteps; ++ks) dw_step<MTN, KWN, WIDE>(ks, a0, b0, tmem, npad, a_tile, idesc, 1u);
}

template <int KWN, bool WIDE>
__device__ __forceinline__ void dw_issue_mt(int mtn, uint64_t a0, uint64_t b0, uint32_t tmem, uint32_t npad,
                                            const DwSteps& a_tile, int ksteps, uint32_t idesc, bool first) {
  switch (mtn) {
    case 1: dw_issue_row<1, KWN, WIDE>(a0, b0, tmem, npad, a_tile, ksteps, idesc, first); break;
    case 2: dw_issue_row<2, KWN, WIDE>(a0, b0, tmem, npad, a_tile, ksteps, idesc, first); break;
    case 3: dw_issue_row<3, KWN, WIDE>(a0, b0, tmem, npad, a_tile, ksteps, idesc, first); break;
    case 4: dw_issue_row<4, KWN, WIDE>(a0, b0, tmem, npad, a_tile, ksteps, idesc, first); break;
    case 5: dw_issue_row<5, KWN, WIDE>(a0, b0, tmem, npad, a_tile, ksteps, idesc, first); break;
    case 6: dw_issue_row<6, KWN, WIDE>(a0, b0, tmem, npad, a_tile, ksteps, idesc, first); break;
    case 7: dw_issue_row<7, KWN, WIDE>(a0, b0, tmem, npad, a_tile, ksteps, idesc, first); break;
    default: dw_issue_row<8, KWN, WIDE>(a0, b0, tmem, npad, a_tile, ksteps, idesc, first); break;
  }
}

// FOLD: the kw-folded chunk layout (DwArgs::fold); RPS: output rows per stage
// (2 only in the wide layout). Separate instantiations, so that the chunk
// layout's issue loop keeps its register allocation.
template <typename T, bool FOLD, int RPS>
__global__ void __launch_bounds__(kThreads, 1)
    tc_dw_kernel(const __grid_constant__ DwArgs a, const __grid_constant__ TaskTable tt) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  uint64_t* done = empty + kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* stage0 = smem + kHeader;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if ((smem_u32(smem) & (a.wide ? 1023u : 127u)) != 0u) {  // swizzled boxes need 1024-byte alignment
    if (threadIdx.x == 0) atomicExch(a.err, 2);
    return;
  }
  const int task = blockIdx.x % a.ntasks;
  const int split = blockIdx.x / a.ntasks;
  const int mt0 = tt.mt0[task], mtn = tt.mtn[task], n0 = tt.n0[task], kw0 = tt.kw0[task];
  const int grp = tt.g[task];
  const int k2 = a.ks * a.ks;
  int c_lo = min((16 * mt0) / k2, a.c8 - 1);
  int c_hi = min((16 * (mt0 + mtn) - 1) / k2, a.c8 - 1);
  const int nch = c_hi - c_lo + 1;
  const int sbo_a = a.pitch_w * 16;
  // group g (absolute) lives at row block (g - c_lo*k2) of the stage's A region
  // wide mode: plane k2 of group 0 holds ones (its D rows are db)
  const bool has_ones = a.wide ? (grp == 0 && kw0 == 0 && a.dbpart != nullptr && k2 >= mt0 * a.apt &&
                                  k2 < (mt0 + mtn) * a.apt)
                               : (a.ones_group >= 16 * mt0 && a.ones_group < 16 * (mt0 + mtn) && kw0 == 0 &&
                                  a.dbpart != nullptr);
  // MMA N. Kept as arithmetic on the task width: loading it as a plain
  // argument changes the issue loop's register allocation (96 registers, no
  // descriptor reuse) and measured 9 % slower at 24->24.
  const int npad = ((a.wide ? a.nbox * a.cwb : a.nn * (FOLD ? 3 : 1)) + 15) / 16 * 16;
  const uint32_t tx_bytes = a.wide ? (uint32_t)(k2 * a.plane_bytes + a.nbox * a.cwb * a.kpad * 2)
                                   : (uint32_t)(nch * k2 * sbo_a + (FOLD ? 3 : 1) * (a.nn / 8) * a.kpad * 16);

  // zero the whole dynamic region (finite junk rows), then the ones rows
  {
    const int total = a.ones_off ? a.ones_off + a.plane_bytes
                                 : a.stages * a.stage_bytes + ((a.wide || FOLD) ? a.tail_bytes : 16 * mtn * sbo_a + 256);
    uint4 z = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x * 16; i < total; i += kThreads * 16) *reinterpret_cast<uint4*>(stage0 + i) = z;
    __syncthreads();
    if (a.wide) {
      if (grp == 0 && a.dbpart != nullptr && a.ones_off) {
        uint32_t* o = reinterpret_cast<uint32_t*>(stage0 + a.ones_off);
        for (int i = threadIdx.x; i < a.plane_bytes / 4; i += kThreads) o[i] = OneBits<T>::v;
      } else if (grp == 0 && a.dbpart != nullptr)
        for (int s = 0; s < a.stages * RPS; ++s) {
          uint32_t* o = reinterpret_cast<uint32_t*>(stage0 + (size_t)(s / RPS) * a.stage_bytes +
                                                    (size_t)(s % RPS) * a.row_bytes + (size_t)k2 * a.plane_bytes);
          for (int i = threadIdx.x; i < a.plane_bytes / 4; i += kThreads) o[i] = OneBits<T>::v;
        }
    } else if (a.ones_group >= 0) {
      const int rel = a.ones_group - c_lo * k2;
      if (rel >= 0 && (rel + 1) * sbo_a <= a.a_bytes) {
        for (int s = 0; s < a.stages; ++s) {
          uint32_t* o = reinterpret_cast<uint32_t*>(stage0 + (size_t)s * a.stage_bytes + (size_t)rel * sbo_a);
          for (int i = threadIdx.x; i < sbo_a / 4; i += kThreads) o[i] = OneBits<T>::v;
        }
      }
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
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

  const long long r_beg = (long long)split * a.rows_per_split;
  const long long r_end = min(r_beg + a.rows_per_split, a.rows);
  const uint64_t kWaitNs = 1000000000ull;
  // Bounded wait; `nap` > 0 sleeps between polls (waiting warps leave issue
  // slots to the producer and MMA threads on their sub-partitions).
  auto wait = [&](uint64_t* bar, uint32_t par, uint32_t nap = 0) -> bool {
    uint64_t deadline = 0;  // the clock is read only once a wait has lasted a while
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, par)) {
      if (nap) __nanosleep(nap);
      if (((++spins) & (nap ? 15u : 255u)) == 0) {
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
    if (lane == 0) {
      prefetch_tmap(&a.tx);
      prefetch_tmap(&a.tg);
      int stage = 0;
      uint32_t epar = 1;
      bool pending[kMaxStages];
      uint32_t last_par[kMaxStages];
      for (int s = 0; s < kMaxStages; ++s) { pending[s] = false; last_par[s] = 0; }
      for (long long r = r_beg; r < r_end; ++r) {
        const int wi = (int)(r % a.nwt);
        long long q = r / a.nwt;
        const int y = (int)(q % a.oh); q /= a.oh;
        const int z = (int)(q % a.od);
        const int nb = (int)(q / a.od);
        const int w0 = wi * a.wt;
        const int slot = RPS == 1 ? 0 : (int)((r - r_beg) % RPS);  // row slot in the stage
        if (slot == 0) {
          if (!wait(&empty[stage], epar)) break;
          const uint32_t nrow = RPS == 1 ? 1u : (uint32_t)min((long long)RPS, r_end - r);
          mbar_arrive_expect_tx(&full[stage], tx_bytes * nrow);
        }
        uint8_t* sA = stage0 + (size_t)stage * a.stage_bytes + (size_t)slot * a.row_bytes;
        if (a.wide) {
          // the k x k input rows of the group: planes [kd][kh] of pitch_w positions
          tma_load_5d(sA, &a.tx, &full[stage], grp * a.cw, w0 - a.pw, y - a.ph, z - a.pd, nb);
          for (int c = 0; c < a.nbox; ++c)
            tma_load_5d(sA + a.a_bytes + (size_t)c * a.b_region, &a.tg, &full[stage], n0 + c * a.cwb, w0, y, z, nb);
        } else {
          for (int c = 0; c < nch; ++c)
            tma_load_5d(sA + (size_t)c * k2 * sbo_a, &a.tx, &full[stage], (c_lo + c) * 8, w0 - a.pw, y - a.ph,
                        z - a.pd, nb);
          // fold: copy kw starts kw positions early (position p of the K range
          // holds dY[w0 + p - kw]; the TMA fills the out-of-range ones with zeros)
          const int nkw = FOLD ? 3 : 1;
          for (int kw = 0; kw < nkw; ++kw)
            for (int c = 0; c < a.nn / 8; ++c)
              tma_load_5d(sA + a.a_bytes + (size_t)(kw * (a.nn / 8) + c) * a.kpad * 16, &a.tg, &full[stage],
                          n0 + c * 8, w0 - kw, y, z, nb);
        }
        pending[stage] = true;
        last_par[stage] = epar ^ 1;
        if (slot == RPS - 1 || r + 1 == r_end) {
          if (++stage == a.stages) { stage = 0; epar ^= 1; }
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
    if (lane == 0) {
      int stage = 0;
      uint32_t fpar = 0;
      bool first = true;
      const int rel0 = 16 * mt0 - c_lo * k2;                     // first group of the task (chunk mode)
      // descriptor steps (16-byte units): K step, kw shift, M tile, B K step
      const DwSteps stp = a.wide ? DwSteps{(uint32_t)(2 * a.cw), (uint32_t)(a.cw / 8),
                                           (uint32_t)(a.apt * a.plane_bytes / 16), (uint32_t)(2 * a.cwb)}
                                 : DwSteps{16u, 1u, (uint32_t)(16 * sbo_a) >> 4, 16u};
      for (long long r = r_beg; r < r_end; ++r) {
        const int slot = RPS == 1 ? 0 : (int)((r - r_beg) % RPS);
        if (slot == 0) {
          if (!wait(&full[stage], fpar)) break;
          tc_fence_after();
        }
        const uint32_t sA = smem_u32(stage0 + (size_t)stage * a.stage_bytes + (size_t)slot * a.row_bytes);
        uint64_t a0, b0;
        if (a.wide) {
          // swizzled MN-major: LBO = MN atom stride, SBO = 8-position K group
          const uint32_t xa = sA + (uint32_t)(mt0 * a.apt * a.plane_bytes) + (uint32_t)(kw0 * a.cw * 2);
          const uint32_t lbo = a.ones_off ? smem_u32(stage0) + (uint32_t)a.ones_off - xa : (uint32_t)a.plane_bytes;
          a0 = desc_layout(xa, lbo, (uint32_t)(16 * a.cw), (uint32_t)a.lay_a);
          b0 = a.cwb > 8 ? desc_layout(sA + (uint32_t)a.a_bytes, (uint32_t)a.b_region, (uint32_t)(16 * a.cwb),
                                       (uint32_t)a.lay_b)
                         : smem_desc(sA + (uint32_t)a.a_bytes, 128, (uint32_t)(a.kpad * 16));
        } else {
          // no swizzle MN-major: LBO = K group (128 B), SBO = MN group
          a0 = smem_desc(sA + (uint32_t)(rel0 * sbo_a) + (uint32_t)(kw0 * 16), 128, (uint32_t)sbo_a);
          b0 = smem_desc(sA + (uint32_t)a.a_bytes, 128, (uint32_t)(a.kpad * 16));
        }
        const int ksteps = a.kpad / 16;
        if (a.wide) {  // wide tasks: one kw, at most 5 M tiles (10 planes / 2 per tile)
          switch (mtn) {
            case 1: dw_issue_row<1, 1, true>(a0, b0, tmem, (uint32_t)npad, stp, ksteps, a.idesc, first); break;
            case 2: dw_issue_row<2, 1, true>(a0, b0, tmem, (uint32_t)npad, stp, ksteps, a.idesc, first); break;
            case 3: dw_issue_row<3, 1, true>(a0, b0, tmem, (uint32_t)npad, stp, ksteps, a.idesc, first); break;
            case 4: dw_issue_row<4, 1, true>(a0, b0, tmem, (uint32_t)npad, stp, ksteps, a.idesc, first); break;
            default: dw_issue_row<5, 1, true>(a0, b0, tmem, (uint32_t)npad, stp, ksteps, a.idesc, first); break;
          }
        } else {
          if (FOLD)
            dw_issue_mt<1, false>(mtn, a0, b0, tmem, (uint32_t)npad, stp, ksteps, a.idesc, first);
          else if (a.kwn == 3)
            dw_issue_mt<3, false>(mtn, a0, b0, tmem, (uint32_t)npad, stp, ksteps, a.idesc, first);
          else
            dw_issue_mt<1, false>(mtn, a0, b0, tmem, (uint32_t)npad, stp, ksteps, a.idesc, first);
        }
        first = false;
        if (slot == RPS - 1 || r + 1 == r_end) {
          mma_commit(&empty[stage]);
          if (++stage == a.stages) { stage = 0; fpar ^= 1; }
        }
      }
      mma_commit(done);
    }
  } else {
    // epilogue: wait (lane 0, sleeping between polls) for every MMA, then
    // write the fp32 partials of this task
    int got = 1;
    if (lane == 0) got = wait(done, 0, 256) ? 1 : 0;
    got = __shfl_sync(0xffffffffu, got, 0);
    if (got) {
      tc_fence_after();
      const int q = warp & 3;
      const int row = q * 32 + lane;
      for (int kw = 0; kw < (FOLD ? 1 : a.kwn); ++kw) {
        for (int t = 0; t < mtn; ++t) {
          // chunk mode: absolute 8-channel group (c, kd, kh) and channel in it;
          // wide mode: (kd, kh) plane (atom) of group grp and channel in it
          const int g = a.wide ? (mt0 + t) * a.apt + row / a.cw : 16 * (mt0 + t) + row / 8;
          const int ci8 = a.wide ? row % a.cw : row % 8;
          const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((kw * mtn + t) * npad);
          for (int cc = 0; cc < npad; cc += 16) {
            float v[16];
            tmem_ld_16(tb + (uint32_t)cc, v);
            const bool real_ci = !a.wide || grp * a.cw + ci8 < a.cin;  // padded group channels
            if ((a.wide ? g < k2 : g < k2 * a.c8) && real_ci) {
              const int c = a.wide ? grp : g / k2, rem = a.wide ? g : g % k2;
              const int kd = rem / a.ks, kh = rem % a.ks;
              const int ci = c * (a.wide ? a.cw : 8) + ci8;
              const int tap = (kd * a.ks + kh) * a.ks + (kw0 + kw);
              const int ntap = k2 * a.ks;
              float* dst = a.part + (size_t)split * a.cout * a.cin * ntap;
              if (FOLD) {
                // column j = kw * nn + channel
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const int j = cc + i, kwi = j / a.nn, co = n0 + j - kwi * a.nn;
                  if (kwi < 3) dst[((size_t)co * a.cin + ci) * ntap + tap + kwi] = v[i];
                }
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const int co = n0 + cc + i;
                  if (cc + i < a.nn) dst[((size_t)co * a.cin + ci) * ntap + tap] = v[i];
                }
              }
            } else if (has_ones && g == (a.wide ? k2 : a.ones_group) && ci8 == 0 && kw == 0) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (cc + i < a.nn) a.dbpart[(size_t)split * a.cout + n0 + cc + i] = v[i];
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

// dw[co][ci][tap] (ci < cin_real) = sum over splits of the partials laid out
// with cin_pad input channels. A block covers 32 outputs with LANES lanes
// each: lane j sums splits j, j+LANES, ... in order, then the lane sums are
// added in a fixed tree — a fixed association, so reruns are bitwise
// identical. LANES = 8 keeps 8x the loads in flight when S is large (one
// thread per output was latency-bound at S ~ 100-300 splits); LANES = 1 for
// few splits over many outputs.
template <int LANES>
__global__ void __launch_bounds__(256) dw_reduce_kernel(const float* __restrict__ part, int S, int cout,
                                                               int cin_pad, int cin_real, int ntap,
                                                               float* __restrict__ dw,
                                                               const float* __restrict__ dbpart,
                                                               float* __restrict__ db) {
  __shared__ float red[8][33];
  const long long total_pad = (long long)cout * cin_pad * ntap;
  const long long total = (long long)cout * cin_real * ntap;
  constexpr int OPB = 256 / LANES;  // outputs per block
  const int o = threadIdx.x % OPB, lj = threadIdx.x / OPB;
  const long long i = (long long)blockIdx.x * OPB + o;
  // outputs [0, total) are dW; [total, total + cout) are db (when requested)
  const bool is_dw = i < total;
  const bool is_db = !is_dw && db != nullptr && dbpart != nullptr && i < total + cout;
  float s = 0.f;
  if (is_dw) {
    const int tap = (int)(i % ntap);
    const long long r = i / ntap;
    const int ci = (int)(r % cin_real);
    const int co = (int)(r / cin_real);
    const long long j = ((long long)co * cin_pad + ci) * ntap + tap;
    for (int k = lj; k < S; k += LANES) s += part[(size_t)k * total_pad + j];
  } else if (is_db) {
    const long long c = i - total;
    for (int k = lj; k < S; k += LANES) s += dbpart[(size_t)k * cout + c];
  }
  float t = s;
  if (LANES > 1) {
    red[lj][o] = s;
    __syncthreads();
    t = ((red[0][o] + red[1][o]) + (red[2][o] + red[3][o])) + ((red[4][o] + red[5][o]) + (red[6][o] + red[7][o]));
  }
  if (lj == 0 && (is_dw || is_db)) {
    if (is_dw) dw[i] = t;
    else db[i - total] = t;
  }
}

// ---------------------------------------------------------------------------
// Host side
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

// NDHWC map, box (bc channels, bx, by, bz, 1), swizzled by the box row width
// (bc*2 = 32/64/128 bytes; 16 bytes: no swizzle).
static bool encode_ndhwc(CUtensorMap* m, const void* base, int dtype, int c, int w, int h, int d, int n,
                         int bx, int by, int bz, int bc = 8) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const cuuint64_t e = 2;
  cuuint64_t dims[5] = {(cuuint64_t)c, (cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)d, (cuuint64_t)n};
  cuuint64_t str[4] = {c * e, (cuuint64_t)w * c * e, (cuuint64_t)h * w * c * e, (cuuint64_t)d * h * w * c * e};
  cuuint32_t box[5] = {(cuuint32_t)bc, (cuuint32_t)bx, (cuuint32_t)by, (cuuint32_t)bz, 1};
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  const CUtensorMapSwizzle sw = bc == 64   ? CU_TENSOR_MAP_SWIZZLE_128B
                                : bc == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                : bc == 16 ? CU_TENSOR_MAP_SWIZZLE_32B
                                           : CU_TENSOR_MAP_SWIZZLE_NONE;
  return enc(m, dtype == R4C_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
             const_cast<void*>(base), dims, str, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, bool FOLD, int RPS>
static cudaError_t set_attr() {
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && done[dev]) return cudaSuccess;
  e = cudaFuncSetAttribute(tc_dw_kernel<T, FOLD, RPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  if (e == cudaSuccess && dev >= 0 && dev < 64) done[dev] = true;
  return e;
}

// ---------------------------------------------------------------------------
// Row-stage layout (k = 3, padding 1): one pipeline stage per INPUT row.
//
// For output plane z and input row yi the products that row takes part in
// are, for each kw,
//   D[(kd, ci), (kh, co)] += sum_x X[z+kd-1][yi][x+kw-1][ci] * dY[z][yi+1-kh][x][co]
// so a stage holds two TMA boxes: the input row yi of the three planes
// z-1..z+1 (M atoms kd, cw channels each, swizzled MN-major: LBO = one plane
// slot) and the three dY rows yi-1..yi+1 of plane z (N atoms kh' = 2 - kh,
// cwb channels each: LBO = one dY row slot). kw is a start-address shift of
// A by kw positions, as in the wide layout. Per 16 positions: one MMA per
// (kw, M tile) with N = 3 * cwb — 24 MMAs of N = 96 per row at 24 -> 24
// against 48 of N = 32 in the chunk layout, and ~50 KB of boxes per row
// against ~65 KB. Summing over every (z, yi) covers each (output row, tap)
// pair exactly once: dY rows outside the volume are TMA zero fill.
// Plane slot 3 holds bf16 ones, so its D rows (junk otherwise) are
// sum_x dY: taken from kh' = 1 (dY row yi) and kw = 0, each dY row once: db.
// Tasks: (input channel group g of cw, dY channel chunk n0 of cwb, kw range).
// ---------------------------------------------------------------------------
struct alignas(64) DwsArgs {
  CUtensorMap tx;   // x:  box (cw, pitch, 1, 3, 1)
  CUtensorMap tg;   // dy: box (cwb, kpad, 3, 1, 1)
  float* part;      // [S][cout][cin][27]
  float* dbpart;    // [S][cout] or nullptr
  int* err;
  int d, h, w, cin, cout;
  int cw, cwb, apt, mtiles, nslots, kwn;
  int pitch, kpad, wt, nwt;
  int bz;                            // planes walked innermost at each input row (a divisor of d)
  int plane_bytes, brow_bytes, a_bytes, stage_bytes, stages;
  int tmem_cols, npad;
  long long rows, rows_per_split;
  int ntasks;
  uint32_t idesc;
  int lay_a, lay_b;
};

struct DwsTasks {
  int g[128], n0[128], kw0[128];
};

template <int MT, int KWN>
__device__ __forceinline__ void dws_issue(uint64_t a0, uint64_t b0, uint32_t tmem, uint32_t npad, uint32_t tile_a,
                                          uint32_t row_a, uint32_t ks_a, uint32_t ks_b, int ksteps, uint32_t idesc,
                                          bool first) {
#pragma unroll 1
  for (int ks = 0; ks < ksteps; ++ks) {
    const uint32_t acc = (first && ks == 0) ? 0u : 1u;
    const uint64_t b = b0 + (uint64_t)(ks * ks_b);
#pragma unroll
    for (int kw = 0; kw < KWN; ++kw)
#pragma unroll
      for (int t = 0; t < MT; ++t)
        mma_f16_ss(tmem + (uint32_t)(kw * MT + t) * npad,
                   a0 + (uint64_t)(ks * ks_a + kw * row_a) + (uint64_t)t * tile_a, b, idesc, acc);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    tc_dws_kernel(const __grid_constant__ DwsArgs a, const __grid_constant__ DwsTasks tt) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  uint64_t* done = empty + kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* stage0 = smem + kHeader;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if ((smem_u32(smem) & 1023u) != 0u) {
    if (threadIdx.x == 0) atomicExch(a.err, 2);
    return;
  }
  const int task = blockIdx.x % a.ntasks;
  const int split = blockIdx.x / a.ntasks;
  const int grp = tt.g[task], n0 = tt.n0[task], kw0 = tt.kw0[task];

  // zero every stage and tail (junk atoms read finite data), then fill plane
  // slot 3 of every stage with ones (never written by TMA)
  {
    const int total = a.stages * a.stage_bytes;
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x * 16; i < total; i += kThreads * 16) *reinterpret_cast<uint4*>(stage0 + i) = z;
    __syncthreads();
    for (int s = 0; s < a.stages; ++s) {
      uint32_t* o = reinterpret_cast<uint32_t*>(stage0 + (size_t)s * a.stage_bytes + (size_t)3 * a.plane_bytes);
      for (int i = threadIdx.x; i < a.plane_bytes / 4; i += kThreads) o[i] = OneBits<T>::v;
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
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

  const long long r_beg = (long long)split * a.rows_per_split;
  const long long r_end = min(r_beg + a.rows_per_split, a.rows);
  const uint64_t kWaitNs = 1000000000ull;
  auto wait = [&](uint64_t* bar, uint32_t par, uint32_t nap = 0) -> bool {
    return bounded_wait(bar, par, kWaitNs, abort_flag, a.err, 1, nap);
  };
  const uint32_t tx_bytes = (uint32_t)(3 * a.plane_bytes + 3 * a.brow_bytes);

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&a.tx);
      prefetch_tmap(&a.tg);
      int stage = 0;
      uint32_t epar = 1;
      bool pending[kMaxStages];
      uint32_t last_par[kMaxStages];
      for (int s = 0; s < kMaxStages; ++s) { pending[s] = false; last_par[s] = 0; }
      for (long long r = r_beg; r < r_end; ++r) {
        // row order (n, z block, yi, z in block, w tile): an input row is
        // reused by the next planes of its block and a dY row by the next
        // rows while both are still in L2
        const int wi = (int)(r % a.nwt);
        long long q = r / a.nwt;
        const int zi = (int)(q % a.bz); q /= a.bz;
        const int yi = (int)(q % a.h); q /= a.h;
        const int nzb = a.d / a.bz;
        const int z = (int)(q % nzb) * a.bz + zi;
        const int nb = (int)(q / nzb);
        const int x0 = wi * a.wt;
        if (!wait(&empty[stage], epar)) break;
        mbar_arrive_expect_tx(&full[stage], tx_bytes);
        uint8_t* sA = stage0 + (size_t)stage * a.stage_bytes;
        // input row yi of planes z-1, z, z+1 (positions x0-1 ..), then dY rows yi-1..yi+1 of plane z
        tma_load_5d(sA, &a.tx, &full[stage], grp * a.cw, x0 - 1, yi, z - 1, nb);
        tma_load_5d(sA + a.a_bytes, &a.tg, &full[stage], n0, x0, yi - 1, z, nb);
        pending[stage] = true;
        last_par[stage] = epar ^ 1;
        if (++stage == a.stages) { stage = 0; epar ^= 1; }
      }
      for (int s = 0; s < a.stages; ++s) {
        if (!pending[s]) continue;
        uint64_t dl = global_timer_ns() + kWaitNs;
        while (!mbar_try_wait(&full[s], last_par[s]) && global_timer_ns() < dl) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t fpar = 0;
      bool first = true;
      const int ksteps = a.kpad / 16;
      // descriptor steps in 16-byte units: A row (one position), 16 rows (K
      // step), M tile (apt plane slots); B 16 rows
      const uint32_t row_a = (uint32_t)(a.cw / 8), ks_a = (uint32_t)(2 * a.cw);
      const uint32_t tile_a = (uint32_t)(a.apt * a.plane_bytes / 16), ks_b = (uint32_t)(2 * a.cwb);
      for (long long r = r_beg; r < r_end; ++r) {
        if (!wait(&full[stage], fpar)) break;
        tc_fence_after();
        const uint32_t sA = smem_u32(stage0 + (size_t)stage * a.stage_bytes);
        const uint64_t a0 = desc_layout(sA + (uint32_t)(kw0 * a.cw * 2), (uint32_t)a.plane_bytes,
                                        (uint32_t)(16 * a.cw), (uint32_t)a.lay_a);
        const uint64_t b0 = desc_layout(sA + (uint32_t)a.a_bytes, (uint32_t)a.brow_bytes, (uint32_t)(16 * a.cwb),
                                        (uint32_t)a.lay_b);
        const uint32_t np = (uint32_t)a.npad;
        if (a.kwn == 3) {
          if (a.mtiles == 1) dws_issue<1, 3>(a0, b0, tmem, np, tile_a, row_a, ks_a, ks_b, ksteps, a.idesc, first);
          else dws_issue<2, 3>(a0, b0, tmem, np, tile_a, row_a, ks_a, ks_b, ksteps, a.idesc, first);
        } else {
          if (a.mtiles == 1) dws_issue<1, 1>(a0, b0, tmem, np, tile_a, row_a, ks_a, ks_b, ksteps, a.idesc, first);
          else dws_issue<2, 1>(a0, b0, tmem, np, tile_a, row_a, ks_a, ks_b, ksteps, a.idesc, first);
        }
        first = false;
        mma_commit(&empty[stage]);
        if (++stage == a.stages) { stage = 0; fpar ^= 1; }
      }
      mma_commit(done);
    }
  } else {
    // epilogue: the task's fp32 partials (and db from the ones atom)
    int got = 1;
    if (lane == 0) got = wait(done, 0, 256) ? 1 : 0;
    got = __shfl_sync(0xffffffffu, got, 0);
    if (got && r_beg < r_end) {
      tc_fence_after();
      const int q = warp & 3;
      const int row = q * 32 + lane;
      float* dst = a.part + (size_t)split * a.cout * a.cin * 27;
      for (int kw = 0; kw < a.kwn; ++kw)
        for (int t = 0; t < a.mtiles; ++t) {
          const int atom = t * a.apt + row / a.cw;
          const int ci = grp * a.cw + row % a.cw;
          const bool real = atom < 3 && ci < a.cin;
          const bool dbrow = atom == 3 && grp == 0 && row % a.cw == 0 && kw0 + kw == 0 && a.dbpart != nullptr;
          const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((kw * a.mtiles + t) * a.npad);
          for (int cc = 0; cc < a.npad; cc += 16) {
            float v[16];
            tmem_ld_16(tb + (uint32_t)cc, v);
            if (real) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int col = cc + i, khp = col / a.cwb, co = n0 + col % a.cwb;
                if (khp < 3 && co < a.cout)
                  dst[((size_t)co * a.cin + ci) * 27 + (atom * 3 + (2 - khp)) * 3 + kw0 + kw] = v[i];
              }
            } else if (dbrow) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int col = cc + i, khp = col / a.cwb, co = n0 + col % a.cwb;
                if (khp == 1 && co < a.cout) a.dbpart[(size_t)split * a.cout + co] = v[i];
              }
            }
          }
        }
    } else if (got) {
      // an empty split: its partials are zero
      const int q = warp & 3;
      const int row = q * 32 + lane;
      float* dst = a.part + (size_t)split * a.cout * a.cin * 27;
      for (int t = 0; t < a.mtiles; ++t) {
        const int atom = t * a.apt + row / a.cw, ci = grp * a.cw + row % a.cw;
        if (atom < 3 && ci < a.cin)
          for (int kw = 0; kw < a.kwn; ++kw)
            for (int col = 0; col < 3 * a.cwb; ++col) {
              const int khp = col / a.cwb, co = n0 + col % a.cwb;
              if (co < a.cout) dst[((size_t)co * a.cin + ci) * 27 + (atom * 3 + (2 - khp)) * 3 + kw0 + kw] = 0.f;
            }
        if (atom == 3 && grp == 0 && row % a.cw == 0 && kw0 == 0 && a.dbpart != nullptr)
          for (int c = 0; c < a.cwb; ++c)
            if (n0 + c < a.cout) a.dbpart[(size_t)split * a.cout + n0 + c] = 0.f;
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

struct DwsPlan {
  bool ok;
  int cw, cwb, ng, nco, apt, mtiles, nslots, kwn;
  int pitch, kpad, wt, nwt, bz;
  int plane_bytes, brow_bytes, a_bytes, stage_bytes, stages, smem_bytes, tmem_cols, npad;
  long long rows, rows_per_split;
  int S;
  std::vector<Task> tasks;  // g, n0, kw0 used
  double est;
};

// Row-stage plan: k = 3, padding (1, 1, 1), Cin and Cout multiples of 8.
// R4C_DW_STRIP=0 disables it (the chunk / wide layouts then run).
static bool plan_dws(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw, DwsPlan* out) {
  // automatic for input and output channel counts up to 64 (the layers whose
  // chunk-layout dW moves the most bytes per FLOP); R4C_DW_STRIP=1 takes it
  // for any eligible layer, =0 never
  const char* env = getenv("R4C_DW_STRIP");
  if (env && env[0] == '0') return false;
  if (!(env && env[0] == '1') && (cin > 64 || cout > 64)) return false;
  if (ks != 3 || pd != 1 || ph != 1 || pw != 1) return false;
  if (cin % 8 || cout % 8 || cin <= 0 || cout <= 0 || n <= 0 || d <= 0 || h <= 0 || w <= 0) return false;
  DwsPlan P{};
  P.cw = cin <= 16 ? 16 : cin <= 32 ? 32 : 64;
  P.ng = (cin + P.cw - 1) / P.cw;
  P.cwb = cout <= 16 ? 16 : cout <= 32 ? 32 : 64;
  P.nco = (cout + P.cwb - 1) / P.cwb;
  P.apt = 128 / P.cw;
  P.mtiles = (4 + P.apt - 1) / P.apt;          // atoms kd = 0..2 and the ones atom
  P.nslots = P.mtiles * P.apt;                 // plane slots an M tile may read
  P.npad = 3 * P.cwb;
  // W tiles: multiples of 16 except the last (whose tail reads dY zero fill)
  int wt = w;
  while (wt > 16 && (round_up(wt, 16) + 8 > 256)) wt = round_up((wt + 1) / 2, 16);
  auto stage_of = [&](int t) {
    const int kpad = round_up(t, 16), pitch = round_up(kpad + 2, 8);
    return round_up(P.nslots * pitch * P.cw * 2, 1024) + round_up(3 * kpad * P.cwb * 2, 1024);
  };
  while (wt > 16 && kHeader + 3 * stage_of(wt) > kSmemMax) wt = round_up((wt + 1) / 2, 16);
  P.wt = wt;
  P.nwt = (w + wt - 1) / wt;
  P.kpad = round_up(wt, 16);
  P.pitch = round_up(P.kpad + 2, 8);
  if (P.pitch > 256 || P.kpad > 256) return false;
  P.plane_bytes = P.pitch * P.cw * 2;
  P.brow_bytes = P.kpad * P.cwb * 2;
  P.a_bytes = round_up(P.nslots * P.plane_bytes, 1024);
  P.stage_bytes = P.a_bytes + round_up(3 * P.brow_bytes, 1024);
  P.stages = std::min(kMaxStages, (kSmemMax - kHeader) / P.stage_bytes);
  if (P.stages < 2) return false;
  P.smem_bytes = kHeader + P.stages * P.stage_bytes;
  P.kwn = 3 * P.mtiles * P.npad <= 512 ? 3 : 1;
  const int cols = P.kwn * P.mtiles * P.npad;
  if (cols > 512) return false;
  int alloc = 32;
  while (alloc < cols) alloc *= 2;
  P.tmem_cols = alloc;
  for (int g = 0; g < P.ng; ++g)
    for (int c = 0; c < P.nco; ++c)
      for (int kw0 = 0; kw0 < 3; kw0 += P.kwn) P.tasks.push_back(Task{0, P.mtiles, c * P.cwb, P.cwb, kw0, P.kwn, g});
  if ((int)P.tasks.size() > 128) return false;
  P.rows = (long long)n * d * h * P.nwt;
  P.bz = d % 4 == 0 ? 4 : d % 2 == 0 ? 2 : 1;
  {
    const char* bze = getenv("R4C_DW_BZ");   // tuning: planes per block (must divide d)
    if (bze && atoi(bze) > 0 && d % atoi(bze) == 0) P.bz = atoi(bze);
  }
  // cost per row: the MMAs (measured ~45 clk at N <= 32, N/2 above) or the
  // boxes' bytes (~30 B/clk per SM), plus the stage hand-off
  const double t_mma = std::max(45.0, P.npad / 2.0 + 8.0) * (P.kpad / 16) * P.kwn * P.mtiles;
  const double t_load = (3.0 * P.plane_bytes + 3.0 * P.brow_bytes) / 30.0;
  const double per_row = std::max(t_mma, t_load) + 80.0;
  const int sms = num_sms();
  const int ntasks = (int)P.tasks.size();
  double best = 1e300;
  for (int k = 1; k <= 4; ++k) {
    int S = (int)std::max<long long>(1, std::min<long long>(P.rows, (long long)k * sms / ntasks));
    const long long rps = (P.rows + S - 1) / S;
    S = (int)((P.rows + rps - 1) / rps);
    const long long waves = ((long long)ntasks * S + sms - 1) / sms;
    const double c = waves * (rps * per_row + 3000.0);
    if (c < best) {
      best = c;
      P.S = S;
      P.rows_per_split = rps;
    }
  }
  P.est = best;
  P.ok = true;
  if (out) *out = P;
  return true;
}

template <typename T>
static cudaError_t set_attr_dws() {
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && done[dev]) return cudaSuccess;
  e = cudaFuncSetAttribute(tc_dws_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  if (e == cudaSuccess && dev >= 0 && dev < 64) done[dev] = true;
  return e;
}

}  // namespace tcdw

namespace tc {

bool dw_supported(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw) {
  if (tcdw::plan_dws(n, d, h, w, cin, cout, ks, pd, ph, pw, nullptr)) return true;
  tcdw::DwPlan P;
  return tcdw::plan_dw(n, d, h, w, cin, cout, ks, pd, ph, pw, &P) && (int)P.tasks.size() <= 128;
}

size_t dw_workspace(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw) {
  tcdw::DwsPlan R;
  if (tcdw::plan_dws(n, d, h, w, cin, cout, ks, pd, ph, pw, &R)) {
    size_t part = (size_t)R.S * cout * cin * 27 * sizeof(float);
    part = (part + 255) / 256 * 256;
    return part + ((size_t)R.S * cout * sizeof(float) + 255) / 256 * 256;
  }
  tcdw::DwPlan P;
  if (!tcdw::plan_dw(n, d, h, w, cin, cout, ks, pd, ph, pw, &P)) return 0;
  size_t T = (size_t)ks * ks * ks;
  size_t part = (size_t)P.S * cout * cin * T * sizeof(float);
  part = (part + 255) / 256 * 256;
  size_t dbp = (size_t)P.S * cout * sizeof(float);
  return part + (dbp + 255) / 256 * 256;
}

int dw_describe(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw, char* buf,
                size_t len) {
  tcdw::DwsPlan R;
  if (tcdw::plan_dws(n, d, h, w, cin, cout, ks, pd, ph, pw, &R)) {
    snprintf(buf, len,
             "tcgen05 dW (row stages: input row x 3 planes as A, 3 dY rows as B): cw=%d cwb=%d groups=%d "
             "co_chunks=%d M tiles=%d kw/task=%d N=%d tasks=%d splits=%d rows/split=%lld wt=%d kpad=%d pitch=%d "
             "stages=%d stage=%dB smem=%dB tmem=%d est=%.0fus",
             R.cw, R.cwb, R.ng, R.nco, R.mtiles, R.kwn, R.npad, (int)R.tasks.size(), R.S, R.rows_per_split, R.wt,
             R.kpad, R.pitch, R.stages, R.stage_bytes, R.smem_bytes, R.tmem_cols, R.est / 1.9e3);
    return 1;
  }
  tcdw::DwPlan P;
  if (!tcdw::plan_dw(n, d, h, w, cin, cout, ks, pd, ph, pw, &P)) return 0;
  if (P.wide)
    snprintf(buf, len,
             "tcgen05 dW (wide: %d-channel swizzled groups x%d, M tiles/group=%d, dY boxes of %d): "
             "task(mt=%d n=%d kw=%d) tasks=%d splits=%d rows/split=%lld wt=%d kpad=%d pitch=%d stages=%d "
             "stage=%dB smem=%dB tmem=%d est=%.0fus",
             P.cw, P.ng, P.tpg, P.cwb, P.mtn, P.nn, P.kwn, (int)P.tasks.size(), P.S, P.rows_per_split, P.wt,
             P.kpad, P.pitch_w, P.stages, P.stage_bytes, P.smem_bytes, P.tmem_cols, P.est / 1.9e3);
  else
    snprintf(buf, len,
             "tcgen05 dW%s: groups=%d mtiles=%d task(mt=%d n=%d kw=%d) tasks=%d splits=%d rows/split=%lld "
             "wt=%d kpad=%d pitch=%d stages=%d stage=%dB smem=%dB tmem=%d db_in_kernel=%d est=%.0fus",
             P.fold ? " (kw folded into N)" : "", P.groups, P.mtiles, P.mtn, P.nn, P.kwn, (int)P.tasks.size(), P.S,
             P.rows_per_split, P.wt, P.kpad,
             P.pitch_w, P.stages, P.stage_bytes, P.smem_bytes, P.tmem_cols, (int)P.db_in_kernel, P.est / 1.9e3);
  return 1;
}

int launch_dw(int n, int d, int h, int w, int cin, int cin_real, int cout, int ks, int pd, int ph, int pw,
              const void* x, const void* go, float* dw, float* db, void* ws, size_t ws_bytes, int dtype,
              cudaStream_t st, bool* db_done) {
  using namespace tcdw;
  {
    DwsPlan R;
    if (plan_dws(n, d, h, w, cin, cout, ks, pd, ph, pw, &R)) {
      if (((uintptr_t)x & 15) || ((uintptr_t)go & 15)) return R4C_ERR_ALIGN;
      const size_t part_bytes = ((size_t)R.S * cout * cin * 27 * sizeof(float) + 255) / 256 * 256;
      const size_t need = part_bytes + ((size_t)R.S * cout * sizeof(float) + 255) / 256 * 256;
      if (ws_bytes < need || ws == nullptr) return R4C_ERR_WORKSPACE;
      DwsArgs a;
      memset(&a, 0, sizeof(a));
      if (!encode_ndhwc(&a.tx, x, dtype, cin, w, h, d, n, R.pitch, 1, 3, R.cw)) return R4C_ERR_INVALID;
      if (!encode_ndhwc(&a.tg, go, dtype, cout, w, h, d, n, R.kpad, 3, 1, R.cwb)) return R4C_ERR_INVALID;
      a.part = static_cast<float*>(ws);
      a.dbpart = db ? reinterpret_cast<float*>(static_cast<char*>(ws) + part_bytes) : nullptr;
      a.err = device_error_flag();
      if (!a.err) return R4C_ERR_CUDA;
      a.d = d; a.h = h; a.w = w; a.cin = cin; a.cout = cout;
      a.cw = R.cw; a.cwb = R.cwb; a.apt = R.apt; a.mtiles = R.mtiles; a.nslots = R.nslots; a.kwn = R.kwn;
      a.pitch = R.pitch; a.kpad = R.kpad; a.wt = R.wt; a.nwt = R.nwt; a.bz = R.bz;
      a.plane_bytes = R.plane_bytes; a.brow_bytes = R.brow_bytes; a.a_bytes = R.a_bytes;
      a.stage_bytes = R.stage_bytes; a.stages = R.stages; a.tmem_cols = R.tmem_cols; a.npad = R.npad;
      a.rows = R.rows; a.rows_per_split = R.rows_per_split; a.ntasks = (int)R.tasks.size();
      a.idesc = sm100::instr_desc_f16(dtype == R4C_BF16, 128, R.npad, 1, 1);
      auto lay = [](int c) { return c == 64 ? 2 : c == 32 ? 4 : c == 16 ? 6 : 0; };
      a.lay_a = lay(R.cw);
      a.lay_b = lay(R.cwb);
      DwsTasks tt;
      memset(&tt, 0, sizeof(tt));
      for (size_t i = 0; i < R.tasks.size(); ++i) {
        tt.g[i] = R.tasks[i].g; tt.n0[i] = R.tasks[i].n0; tt.kw0[i] = R.tasks[i].kw0;
      }
      const unsigned grid = (unsigned)(R.tasks.size() * R.S);
      const bool bf = dtype == R4C_BF16;
      cudaError_t e = bf ? set_attr_dws<__nv_bfloat16>() : set_attr_dws<__half>();
      if (e != cudaSuccess) return R4C_ERR_CUDA;
      if (bf) tc_dws_kernel<__nv_bfloat16><<<grid, kThreads, R.smem_bytes, st>>>(a, tt);
      else tc_dws_kernel<__half><<<grid, kThreads, R.smem_bytes, st>>>(a, tt);
      if (cudaGetLastError() != cudaSuccess) return R4C_ERR_CUDA;
      const long long total = (long long)cout * cin_real * 27;
      const long long nout = total + (a.dbpart ? cout : 0);
      if (R.S >= 48)
        dw_reduce_kernel<8><<<(unsigned)((nout + 31) / 32), 256, 0, st>>>(a.part, R.S, cout, cin, cin_real, 27, dw,
                                                                          a.dbpart, a.dbpart ? db : nullptr);
      else
        dw_reduce_kernel<1><<<(unsigned)((nout + 255) / 256), 256, 0, st>>>(a.part, R.S, cout, cin, cin_real, 27,
                                                                            dw, a.dbpart, a.dbpart ? db : nullptr);
      note_launches(2);
      if (cudaGetLastError() != cudaSuccess) return R4C_ERR_CUDA;
      if (db_done) *db_done = (a.dbpart != nullptr);
      return R4C_OK;
    }
  }
  DwPlan P;
  if (!plan_dw(n, d, h, w, cin, cout, ks, pd, ph, pw, &P)) return R4C_ERR_UNSUPPORTED;
  if ((int)P.tasks.size() > 128) return R4C_ERR_UNSUPPORTED;
  if (((uintptr_t)x & 15) || ((uintptr_t)go & 15)) return R4C_ERR_ALIGN;
  const size_t T = (size_t)ks * ks * ks;
  size_t part_bytes = ((size_t)P.S * cout * cin * T * sizeof(float) + 255) / 256 * 256;
  size_t need = part_bytes + ((size_t)P.S * cout * sizeof(float) + 255) / 256 * 256;
  if (ws_bytes < need || ws == nullptr) return R4C_ERR_WORKSPACE;
  DwArgs a;
  memset(&a, 0, sizeof(a));
  if (!encode_ndhwc(&a.tx, x, dtype, cin, w, h, d, n, P.pitch_w, ks, ks, P.wide ? P.cw : 8)) return R4C_ERR_INVALID;
  if (!encode_ndhwc(&a.tg, go, dtype, cout, P.ow, P.oh, P.od, n, P.kpad, 1, 1, P.wide ? P.cwb : 8))
    return R4C_ERR_INVALID;
  a.part = static_cast<float*>(ws);
  a.err = device_error_flag();
  if (!a.err) return R4C_ERR_CUDA;
  a.dbpart = (db != nullptr && P.db_in_kernel) ? reinterpret_cast<float*>(static_cast<char*>(ws) + part_bytes)
                                               : nullptr;
  a.od = P.od; a.oh = P.oh; a.ow = P.ow; a.cin = cin; a.cout = cout; a.ks = ks;
  a.pd = pd; a.ph = ph; a.pw = pw;
  a.c8 = P.c8; a.pitch_w = P.pitch_w; a.kpad = P.kpad; a.nwt = P.nwt; a.wt = P.wt;
  a.mtn = P.mtn; a.nn = P.nn; a.kwn = P.kwn;
  a.ones_group = P.db_in_kernel ? P.groups : -1;
  a.stages = P.stages; a.stage_bytes = P.stage_bytes;
  a.row_bytes = P.stage_bytes / P.rpst;
  {
    int lo, hi;
    chunk_range(0, P.mtn, ks * ks, P.c8, &lo, &hi);
    int nch = std::min(hi - lo + 2, P.c8);
    a.a_bytes = round_up((nch * ks * ks + 1) * P.pitch_w * 16, 128);
  }
  a.g_bytes = (P.nn / 8) * P.kpad * 16;
  a.fold = P.fold ? 1 : 0;
  if (P.fold) a.tail_bytes = P.tail_bytes;
  if (P.wide) {
    auto lay = [](int c) { return c == 64 ? 2 : c == 32 ? 4 : c == 16 ? 6 : 0; };
    a.wide = 1;
    a.cw = P.cw; a.apt = P.apt; a.plane_bytes = P.plane_bytes; a.lay_a = lay(P.cw);
    a.cwb = P.cwb; a.b_region = P.kpad * P.cwb * 2; a.lay_b = lay(P.cwb);
    a.nbox = P.nbox; a.npad_w = P.npad_w;
    a.a_bytes = P.region_bytes;
    a.tail_bytes = P.tail_bytes;
    a.ones_off = P.ones_bytes ? P.stages * P.stage_bytes + round_up(P.tail_bytes, 1024) : 0;
    a.ones_group = -1;
  }
  a.tmem_cols = P.tmem_cols;
  a.rows = P.rows;
  a.rows_per_split = P.rows_per_split;
  a.ntasks = (int)P.tasks.size();
  a.idesc = sm100::instr_desc_f16(dtype == R4C_BF16, 128, P.wide ? P.npad_w : round_up(P.nn * (P.fold ? 3 : 1), 16),
                                  1, 1);
  TaskTable tt;
  memset(&tt, 0, sizeof(tt));
  for (size_t i = 0; i < P.tasks.size(); ++i) {
    tt.mt0[i] = P.tasks[i].mt0; tt.mtn[i] = P.tasks[i].mtn; tt.n0[i] = P.tasks[i].n0; tt.kw0[i] = P.tasks[i].kw0;
    tt.g[i] = P.tasks[i].g;
  }
  const unsigned grid = (unsigned)(P.tasks.size() * P.S);
  cudaError_t e;
  // instantiations: chunk / wide (one row per stage), fold, wide with two or four rows per stage
  const bool bf = dtype == R4C_BF16;
  if (P.fold) {
    e = bf ? set_attr<__nv_bfloat16, true, 1>() : set_attr<__half, true, 1>();
    if (e != cudaSuccess) return R4C_ERR_CUDA;
    if (bf) tc_dw_kernel<__nv_bfloat16, true, 1><<<grid, kThreads, P.smem_bytes, st>>>(a, tt);
    else tc_dw_kernel<__half, true, 1><<<grid, kThreads, P.smem_bytes, st>>>(a, tt);
  } else if (P.rpst == 4) {
    e = bf ? set_attr<__nv_bfloat16, false, 4>() : set_attr<__half, false, 4>();
    if (e != cudaSuccess) return R4C_ERR_CUDA;
    if (bf) tc_dw_kernel<__nv_bfloat16, false, 4><<<grid, kThreads, P.smem_bytes, st>>>(a, tt);
    else tc_dw_kernel<__half, false, 4><<<grid, kThreads, P.smem_bytes, st>>>(a, tt);
  } else if (P.rpst == 2) {
    e = bf ? set_attr<__nv_bfloat16, false, 2>() : set_attr<__half, false, 2>();
    if (e != cudaSuccess) return R4C_ERR_CUDA;
    if (bf) tc_dw_kernel<__nv_bfloat16, false, 2><<<grid, kThreads, P.smem_bytes, st>>>(a, tt);
    else tc_dw_kernel<__half, false, 2><<<grid, kThreads, P.smem_bytes, st>>>(a, tt);
  } else {
    e = bf ? set_attr<__nv_bfloat16, false, 1>() : set_attr<__half, false, 1>();
    if (e != cudaSuccess) return R4C_ERR_CUDA;
    if (bf) tc_dw_kernel<__nv_bfloat16, false, 1><<<grid, kThreads, P.smem_bytes, st>>>(a, tt);
    else tc_dw_kernel<__half, false, 1><<<grid, kThreads, P.smem_bytes, st>>>(a, tt);
  }
  if (cudaGetLastError() != cudaSuccess) return R4C_ERR_CUDA;
  const long long total = (long long)cout * cin_real * T;
  const long long nout = total + (a.dbpart ? cout : 0);
  if (P.S >= 48)
    dw_reduce_kernel<8><<<(unsigned)((nout + 31) / 32), 256, 0, st>>>(a.part, P.S, cout, cin, cin_real, (int)T, dw,
                                                                      a.dbpart, a.dbpart ? db : nullptr);
  else
    dw_reduce_kernel<1><<<(unsigned)((nout + 255) / 256), 256, 0, st>>>(a.part, P.S, cout, cin, cin_real, (int)T, dw,
                                                                    a.dbpart, a.dbpart ? db : nullptr);
  note_launches(2);
  if (cudaGetLastError() != cudaSuccess) return R4C_ERR_CUDA;
  if (db_done) *db_done = (a.dbpart != nullptr);
  return R4C_OK;
}

}  // namespace tc
}  // namespace r4c
