// r4c_api.cu — the extern "C" entry points declared in include/r4c_conv3d.h.
//
// Dispatch: every leg first asks the tcgen05 planner (r4c_tc.cu) whether its
// kernel covers the descriptor; otherwise the SIMT kernels in r4c_generic.cu
// run. Both paths are CUDA; there is no host fallback in this library.
#include <stdio.h>
#include <string.h>

#include <atomic>

#include "r4c_internal.h"

namespace r4c {
static std::atomic<uint64_t> g_launches{0};
void note_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }
}  // namespace r4c

using namespace r4c;

namespace {

constexpr int kVersion = 1;

bool valid_dtype(int dt) { return dt == R4C_BF16 || dt == R4C_F16; }

// Validates the descriptor for `leg` and fills `g`.
int check_desc(const r4c_conv_desc* ds, int leg, Geom* g) {
  if (!ds || !make_geom(ds, g)) return R4C_ERR_INVALID;
  if (!valid_dtype(ds->dtype)) return R4C_ERR_INVALID;
  if (g->n < 0 || g->d < 0 || g->h < 0 || g->w < 0) return R4C_ERR_INVALID;
  if (g->cin <= 0 || g->cout <= 0) return R4C_ERR_INVALID;
  const bool tconv = leg == R4C_LEG_TFWD || leg == R4C_LEG_TDX || leg == R4C_LEG_TDW;
  if (tconv) {
    if (g->k != 2) return R4C_ERR_UNSUPPORTED;
    if (g->pd || g->ph || g->pw) return R4C_ERR_UNSUPPORTED;
  } else {
    if (g->k != 1 && g->k != 3) return R4C_ERR_UNSUPPORTED;
    if (g->pd < 0 || g->ph < 0 || g->pw < 0) return R4C_ERR_INVALID;
    if (g->od <= 0 || g->oh <= 0 || g->ow <= 0) return R4C_ERR_INVALID;
  }
  // Element offsets are 64-bit, but a single GEMM row index must fit the
  // kernels' 32-bit channel arithmetic.
  if ((int64_t)g->cin * g->k * g->k * g->k > (1 << 24)) return R4C_ERR_UNSUPPORTED;
  if ((int64_t)g->cout * 8 > (1 << 24)) return R4C_ERR_UNSUPPORTED;
  return R4C_OK;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? R4C_OK : R4C_ERR_CUDA; }

// --- weight packing kernels (generic layouts) ------------------------------
template <typename TO>
__device__ __forceinline__ TO cvt_from(const void* src, int64_t i, int sdt) {
  float v;
  if (sdt == R4C_F32) v = static_cast<const float*>(src)[i];
  else if (sdt == R4C_BF16) v = __bfloat162float(static_cast<const __nv_bfloat16*>(src)[i]);
  else v = __half2float(static_cast<const __half*>(src)[i]);
  return Elem<TO>::from_f(v);
}

// leg FWD: dst[(tap*Cin + ci)*Cout + co] = W[co][ci][tap]
// leg DX : dst[(tap*Cout + co)*Cin + ci] = W[co][ci][T-1-tap]
// leg TFWD: dst[ci*8Cout + tap*Cout + co] = Wt[ci][co][tap]
// leg TDX : dst[(tap*Cout + co)*Cin + ci] = Wt[ci][co][tap]
template <typename TO>
__global__ void pack_generic_kernel(const void* __restrict__ src, int sdt, TO* __restrict__ dst,
                                    int leg, int cin, int cout, int taps) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t total = (int64_t)cin * cout * taps;
  if (i >= total) return;
  int64_t s;
  if (leg == R4C_LEG_FWD) {
    int co = (int)(i % cout); int64_t r = i / cout;
    int ci = (int)(r % cin); int tap = (int)(r / cin);
    s = ((int64_t)co * cin + ci) * taps + tap;
  } else if (leg == R4C_LEG_DX) {
    int ci = (int)(i % cin); int64_t r = i / cin;
    int co = (int)(r % cout); int tap = (int)(r / cout);
    s = ((int64_t)co * cin + ci) * taps + (taps - 1 - tap);
  } else if (leg == R4C_LEG_TFWD) {
    int j = (int)(i % (8 * cout)); int ci = (int)(i / (8 * cout));
    int tap = j / cout, co = j - tap * cout;
    s = ((int64_t)ci * cout + co) * 8 + tap;
  } else {
    int ci = (int)(i % cin); int64_t r = i / cin;
    int co = (int)(r % cout); int tap = (int)(r / cout);
    s = ((int64_t)ci * cout + co) * 8 + tap;
  }
  dst[i] = cvt_from<TO>(src, s, sdt);
}

struct WgradLayout {
  int S; int chunk; size_t part_bytes;
  int Sdb; int64_t dbchunk; size_t db_bytes;
};

WgradLayout wgrad_layout(const Geom& g, bool tconv) {
  WgradLayout L{};
  int P = tconv ? g.cin : g.k * g.k * g.k * g.cin;
  int N = tconv ? 8 * g.cout : g.cout;
  int64_t M = tconv ? g.in_vox() : g.out_vox();
  generic::wgrad_split(M, P, N, &L.S, &L.chunk);
  L.part_bytes = align_up((size_t)L.S * P * N * sizeof(float), 256);
  int64_t V = tconv ? 8 * g.in_vox() : g.out_vox();
  generic::db_split(V, &L.Sdb, &L.dbchunk);
  L.db_bytes = align_up((size_t)L.Sdb * g.cout * sizeof(float), 256);
  return L;
}

// Channel padding: TMA needs the innermost stride (Cin * 2 bytes) to be a
// multiple of 16, so forward and dW with Cin not a multiple of 8 first copy
// the activation into caller workspace with Cin rounded up to 8 (zeros in the
// extra channels; their weights are packed as zeros).
int cin_eff(const Geom& g) { return g.cin % 8 ? (g.cin + 7) / 8 * 8 : g.cin; }
bool needs_cpad(const Geom& g) { return g.cin % 8 != 0; }
size_t cpad_bytes(const Geom& g) {
  return needs_cpad(g) ? align_up((size_t)g.in_vox() * cin_eff(g) * 2, 256) : 0;
}

template <typename T>
__global__ void cpad_kernel(const T* __restrict__ x, T* __restrict__ xp, int64_t vox, int cin, int cinp) {
  const int chunks = cinp / 8;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= vox * chunks) return;
  const int64_t v = i / chunks;
  const int c0 = (int)(i - v * chunks) * 8;
  __align__(16) T tmp[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) tmp[j] = (c0 + j < cin) ? x[v * cin + c0 + j] : Elem<T>::from_f(0.f);
  *reinterpret_cast<uint4*>(xp + v * cinp + c0) = *reinterpret_cast<const uint4*>(tmp);
}

cudaError_t launch_cpad_n(const void* x, void* xp, int64_t vox, int c, int cp, int dtype, cudaStream_t st) {
  const int64_t n = vox * (cp / 8);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (n == 0) return cudaSuccess;
  if (dtype == R4C_BF16)
    cpad_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x),
                                                       static_cast<__nv_bfloat16*>(xp), vox, c, cp);
  else
    cpad_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(x), static_cast<__half*>(xp), vox, c, cp);
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_cpad(const void* x, void* xp, const Geom& g, int dtype, cudaStream_t st) {
  return launch_cpad_n(x, xp, g.in_vox(), g.cin, cin_eff(g), dtype, st);
}

// The same for dY when Cout is not a multiple of 8 (dX and dW legs: dY is the
// source the TMA reads): dY copied with Cout rounded up to 8, zeros past
// Cout; the dX weights of the padded channels are packed as zeros and the dW
// rows of the padded channels (zero) are dropped.
int cout_eff(const Geom& g) { return g.cout % 8 ? (g.cout + 7) / 8 * 8 : g.cout; }
bool needs_gpad(const Geom& g) { return g.cout % 8 != 0; }
size_t gpad_bytes(const Geom& g) {
  return needs_gpad(g) ? align_up((size_t)g.out_vox() * cout_eff(g) * 2, 256) : 0;
}
// dW / db of the padded Cout, of which the first Cout rows are the result
// (OIDHW: a prefix), when dY is padded.
size_t gpad_dw_bytes(const Geom& g) {
  if (!needs_gpad(g)) return 0;
  return align_up((size_t)cout_eff(g) * g.cin * g.k * g.k * g.k * sizeof(float), 256) +
         align_up((size_t)cout_eff(g) * sizeof(float), 256);
}

// Forward of a k=3 layer with 1..4 input channels: the stem kernel.
bool use_stem(const r4c_conv_desc* ds, int leg, const Geom& g) {
  if (ds->force_kernel == R4C_KERNEL_GENERIC || leg != R4C_LEG_FWD) return false;
  return stem::supported(g.n, g.d, g.h, g.w, g.cin, g.cout, g.k, g.pd, g.ph, g.pw);
}

// Weight gradient of the same layers (Cout a multiple of 8): the stem dW kernel.
bool use_stem_dw(const r4c_conv_desc* ds, int leg, const Geom& g) {
  if (ds->force_kernel == R4C_KERNEL_GENERIC || leg != R4C_LEG_DW) return false;
  return stem::dw_supported(g.n, g.d, g.h, g.w, g.cin, g.cout, g.k, g.pd, g.ph, g.pw);
}

// Data gradient of the one-input-channel k=3 layers: the stem dX kernel.
bool use_stem_dx(const r4c_conv_desc* ds, int leg, const Geom& g) {
  if (ds->force_kernel == R4C_KERNEL_GENERIC || leg != R4C_LEG_DX) return false;
  return stem::dx_supported(g.n, g.d, g.h, g.w, g.cin, g.cout, g.k, g.pd, g.ph, g.pw);
}

// ConvTranspose3d k2s2 forward / dX: the tcgen05 transpose-conv kernel.
bool use_tc_tconv(const r4c_conv_desc* ds, int leg, const Geom& g) {
  if (ds->force_kernel == R4C_KERNEL_GENERIC || (leg != R4C_LEG_TFWD && leg != R4C_LEG_TDX)) return false;
  return tconv::supported(leg == R4C_LEG_TFWD ? 0 : 1, g.n, g.d, g.h, g.w, g.cin, g.cout);
}

// ConvTranspose3d k2s2 weight gradient: the tcgen05 transpose-conv dW kernel.
bool use_tc_tconv_dw(const r4c_conv_desc* ds, int leg, const Geom& g) {
  if (ds->force_kernel == R4C_KERNEL_GENERIC || leg != R4C_LEG_TDW) return false;
  return tconv::dw_supported(g.n, g.d, g.h, g.w, g.cin, g.cout);
}

bool use_tc(const r4c_conv_desc* ds, int leg, const Geom& g, tc::ConvPlan* pl) {
  if (ds->force_kernel == R4C_KERNEL_GENERIC) return false;
  if (leg == R4C_LEG_FWD)
    return tc::plan_conv(g.n, g.d, g.h, g.w, cin_eff(g), g.cout, g.k, g.pd, g.ph, g.pw, pl);
  if (leg == R4C_LEG_DX)
    return tc::plan_conv(g.n, g.od, g.oh, g.ow, cout_eff(g), g.cin, g.k, g.k - 1 - g.pd,
                         g.k - 1 - g.ph, g.k - 1 - g.pw, pl);
  if (leg == R4C_LEG_DW)
    return tc::dw_supported(g.n, g.d, g.h, g.w, cin_eff(g), cout_eff(g), g.k, g.pd, g.ph, g.pw);
  return false;
}

// Workspace of the tcgen05 dW: its split partials plus the generic db
// partials (used when the kernel cannot fold db into its spare rows).
size_t tc_dw_ws(const Geom& g, size_t* part_bytes) {
  size_t a = align_up(tc::dw_workspace(g.n, g.d, g.h, g.w, cin_eff(g), cout_eff(g), g.k, g.pd, g.ph, g.pw), 256);
  int Sdb; int64_t ch;
  generic::db_split(g.out_vox(), &Sdb, &ch);
  if (part_bytes) *part_bytes = a;
  return a + align_up((size_t)Sdb * g.cout * sizeof(float), 256);
}

}  // namespace

extern "C" {

const char* r4c_strerror(int status) {
  switch (status) {
    case R4C_OK: return "ok";
    case R4C_ERR_INVALID: return "invalid argument (pointer, size or descriptor field)";
    case R4C_ERR_UNSUPPORTED: return "geometry outside the supported scope";
    case R4C_ERR_WORKSPACE: return "workspace smaller than r4c_workspace_size()";
    case R4C_ERR_CUDA: return "CUDA call failed";
    case R4C_ERR_ALIGN: return "pointer misaligned for the selected kernel";
    case R4C_ERR_NO_DEVICE: return "no sm_100 device is current";
    case R4C_ERR_TOO_LARGE: return "size above the entry point's fixed maximum";
    default: return "unknown status";
  }
}

int r4c_version(void) { return kVersion; }

uint64_t r4c_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int r4c_plan_kernel(const r4c_conv_desc* desc, int leg) {
  Geom g;
  int st = check_desc(desc, leg, &g);
  if (st != R4C_OK) return st;
  tc::ConvPlan pl;
  if (use_stem(desc, leg, g) || use_stem_dw(desc, leg, g) || use_stem_dx(desc, leg, g) ||
      use_tc_tconv(desc, leg, g) || use_tc_tconv_dw(desc, leg, g) || use_tc(desc, leg, g, &pl))
    return R4C_KERNEL_TC;
  return R4C_KERNEL_GENERIC;
}

int r4c_describe_plan(const r4c_conv_desc* desc, int leg, char* buf, size_t len) {
  Geom g;
  int st = check_desc(desc, leg, &g);
  char tmp[512];
  if (st != R4C_OK) {
    snprintf(tmp, sizeof(tmp), "invalid: %s", r4c_strerror(st));
  } else {
    tc::ConvPlan pl;
    if (use_stem(desc, leg, g)) {
      stem::describe(g.n, g.d, g.h, g.w, g.cin, g.cout, g.pd, g.ph, g.pw, tmp, sizeof(tmp));
      st = R4C_KERNEL_TC;
    } else if (use_stem_dw(desc, leg, g)) {
      stem::dw_describe(g.n, g.d, g.h, g.w, g.cin, g.cout, g.pd, g.ph, g.pw, tmp, sizeof(tmp));
      st = R4C_KERNEL_TC;
    } else if (use_stem_dx(desc, leg, g)) {
      stem::dx_describe(g.n, g.d, g.h, g.w, g.cout, tmp, sizeof(tmp));
      st = R4C_KERNEL_TC;
    } else if (use_tc_tconv(desc, leg, g)) {
      tconv::describe(leg == R4C_LEG_TFWD ? 0 : 1, g.n, g.d, g.h, g.w, g.cin, g.cout, tmp, sizeof(tmp));
      st = R4C_KERNEL_TC;
    } else if (use_tc_tconv_dw(desc, leg, g)) {
      tconv::dw_describe(g.n, g.d, g.h, g.w, g.cin, g.cout, tmp, sizeof(tmp));
      st = R4C_KERNEL_TC;
    } else if (leg == R4C_LEG_DW && use_tc(desc, leg, g, &pl)) {
      tc::dw_describe(g.n, g.d, g.h, g.w, cin_eff(g), cout_eff(g), g.k, g.pd, g.ph, g.pw, tmp, sizeof(tmp));
      if (needs_cpad(g)) strncat(tmp, " (input channels padded to a multiple of 8)", sizeof(tmp) - strlen(tmp) - 1);
      st = R4C_KERNEL_TC;
    } else if (use_tc(desc, leg, g, &pl)) {
      snprintf(tmp, sizeof(tmp),
               "tcgen05 conv: cin=%d cout=%d(npad %d) k=%d planes/unit=%d fold=%d tile=%dx%d pitch=%dx%d G=%d groups=%d "
               "padg=%d steps=%d mtiles=%d sets=%d stages=%d stage=%dB wres=%d stg=%d smem=%dB tmem=%d units=%lld "
               "grid=%d est=%.0fus wi=%d pps=%d",
               pl.cin, pl.cout, pl.npad, pl.ks, pl.P, pl.fold, pl.ht, pl.wt, pl.pitch_h, pl.pitch_w, pl.G, pl.ngroups,
               pl.padg, pl.nsteps, pl.mtiles, pl.nsets, pl.stages, pl.stage_bytes, pl.wres_bytes, pl.stg_bytes,
               pl.smem_bytes,
               pl.tmem_cols, (long long)pl.work_units, pl.grid, pl.est_cycles / 1.9e3, pl.warp_issue, pl.pps);
      tc::ConvPlan tp;
      if (tc::tuned_plan(pl, desc->dtype, &tp)) {
        char t2[160];
        snprintf(t2, sizeof(t2),
                 " | tuned on device: planes/unit=%d tile=%dx%d mtiles=%d sets=%d stages=%d wres=%d stg=%d wi=%d pps=%d",
                 tp.P, tp.ht, tp.wt, tp.mtiles, tp.nsets, tp.stages, tp.wres_bytes, tp.stg_bytes, tp.warp_issue, tp.pps);
        strncat(tmp, t2, sizeof(tmp) - strlen(tmp) - 1);
      }
      st = R4C_KERNEL_TC;
    } else {
      snprintf(tmp, sizeof(tmp), "simt generic");
      st = R4C_KERNEL_GENERIC;
    }
  }
  if (buf && len) {
    strncpy(buf, tmp, len - 1);
    buf[len - 1] = 0;
  }
  return st;
}

size_t r4c_packed_weight_bytes(const r4c_conv_desc* desc, int leg) {
  Geom g;
  if (check_desc(desc, leg, &g) != R4C_OK) return 0;
  if (use_stem(desc, leg, g)) return stem::packed_bytes(g.cin, g.cout);
  if (use_stem_dx(desc, leg, g)) return stem::dx_packed_bytes();
  if (use_tc_tconv(desc, leg, g))
    return tconv::packed_bytes(leg == R4C_LEG_TFWD ? 0 : 1, g.n, g.d, g.h, g.w, g.cin, g.cout);
  tc::ConvPlan pl;
  if (use_tc(desc, leg, g, &pl)) return tc::packed_bytes(pl);
  int taps = (leg == R4C_LEG_TFWD || leg == R4C_LEG_TDX) ? 8 : g.k * g.k * g.k;
  return (size_t)g.cin * g.cout * taps * 2;
}

size_t r4c_workspace_size(const r4c_conv_desc* desc, int leg) {
  Geom g;
  if (check_desc(desc, leg, &g) != R4C_OK) return 0;
  if (leg == R4C_LEG_DW) {
    if (use_stem_dw(desc, leg, g)) return stem::dw_workspace(g.n, g.d, g.h, g.w, g.cin, g.cout, g.pd, g.ph, g.pw);
    tc::ConvPlan pl;
    if (use_tc(desc, leg, g, &pl)) return cpad_bytes(g) + gpad_bytes(g) + gpad_dw_bytes(g) + tc_dw_ws(g, nullptr);
  }
  if (leg == R4C_LEG_DX) {
    tc::ConvPlan pl;
    if (!use_stem_dx(desc, leg, g) && use_tc(desc, leg, g, &pl)) return gpad_bytes(g);
  }
  if (leg == R4C_LEG_FWD) {
    if (use_stem(desc, leg, g)) return 0;
    tc::ConvPlan pl;
    if (use_tc(desc, leg, g, &pl)) return cpad_bytes(g);
  }
  if (leg == R4C_LEG_TDW && use_tc_tconv_dw(desc, leg, g)) {
    WgradLayout L = wgrad_layout(g, true);
    return tconv::dw_workspace(g.n, g.d, g.h, g.w, g.cin, g.cout) + L.db_bytes;
  }
  if (leg == R4C_LEG_DW || leg == R4C_LEG_TDW) {
    WgradLayout L = wgrad_layout(g, leg == R4C_LEG_TDW);
    return L.part_bytes + L.db_bytes;
  }
  return 0;
}

int r4c_pack_weight(const r4c_conv_desc* desc, int leg, const void* w_src, int src_dtype,
                    void* w_packed, r4c_stream_t stream) {
  Geom g;
  int st = check_desc(desc, leg, &g);
  if (st != R4C_OK) return st;
  if (leg != R4C_LEG_FWD && leg != R4C_LEG_DX && leg != R4C_LEG_TFWD && leg != R4C_LEG_TDX)
    return R4C_ERR_INVALID;
  if (src_dtype != R4C_F32 && src_dtype != R4C_BF16 && src_dtype != R4C_F16) return R4C_ERR_INVALID;
  if (!w_src || !w_packed) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (use_stem(desc, leg, g)) {
    if ((reinterpret_cast<uintptr_t>(w_packed) & 15) != 0) return R4C_ERR_ALIGN;
    return cuda_status(stem::pack_weight(g.cin, g.cout, w_src, src_dtype, w_packed, desc->dtype, s));
  }
  if (use_stem_dx(desc, leg, g)) {
    if ((reinterpret_cast<uintptr_t>(w_packed) & 15) != 0) return R4C_ERR_ALIGN;
    return cuda_status(stem::dx_pack_weight(g.cout, w_src, src_dtype, w_packed, desc->dtype, s));
  }
  if (use_tc_tconv(desc, leg, g)) {
    if ((reinterpret_cast<uintptr_t>(w_packed) & 15) != 0) return R4C_ERR_ALIGN;
    return cuda_status(tconv::pack_weight(leg == R4C_LEG_TFWD ? 0 : 1, g.n, g.d, g.h, g.w, g.cin, g.cout, w_src,
                                          src_dtype, w_packed, desc->dtype, s));
  }
  tc::ConvPlan pl;
  if (use_tc(desc, leg, g, &pl)) {
    if ((reinterpret_cast<uintptr_t>(w_packed) & 15) != 0) return R4C_ERR_ALIGN;
    // dX: the conv runs over dY's channels (padded to a multiple of 8); the
    // padded channels get zero weights
    return cuda_status(tc::pack_weight(pl, leg == R4C_LEG_DX, leg == R4C_LEG_DX ? g.cout : g.cin, w_src,
                                       src_dtype, w_packed, desc->dtype, s));
  }
  int taps = (leg == R4C_LEG_TFWD || leg == R4C_LEG_TDX) ? 8 : g.k * g.k * g.k;
  int64_t total = (int64_t)g.cin * g.cout * taps;
  unsigned blocks = (unsigned)cdiv(total, 256);
  if (desc->dtype == R4C_BF16)
    pack_generic_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
        w_src, src_dtype, static_cast<__nv_bfloat16*>(w_packed), leg, g.cin, g.cout, taps);
  else
    pack_generic_kernel<__half><<<blocks, 256, 0, s>>>(
        w_src, src_dtype, static_cast<__half*>(w_packed), leg, g.cin, g.cout, taps);
  note_launches(1);
  return cuda_status(cudaGetLastError());
}

int r4c_conv3d_fwd(const r4c_conv_desc* desc, const void* x, const void* w_packed,
                   const void* bias, void* y, void* workspace, size_t ws_bytes,
                   r4c_stream_t stream) {
  Geom g;
  int st = check_desc(desc, R4C_LEG_FWD, &g);
  if (st != R4C_OK) return st;
  if (g.out_vox() == 0) return R4C_OK;
  if (!x || !w_packed || !y) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (use_stem(desc, R4C_LEG_FWD, g))
    return stem::launch_fwd(g.n, g.d, g.h, g.w, g.cin, g.cout, g.pd, g.ph, g.pw, x, w_packed, bias, y,
                            desc->dtype, s);
  tc::ConvPlan pl;
  if (use_tc(desc, R4C_LEG_FWD, g, &pl)) {
    const void* xin = x;
    if (needs_cpad(g)) {
      if (!workspace || ws_bytes < cpad_bytes(g)) return R4C_ERR_WORKSPACE;
      if (launch_cpad(x, workspace, g, desc->dtype, s) != cudaSuccess) return R4C_ERR_CUDA;
      xin = workspace;
    }
    return tc::launch_conv_tuned(pl, xin, w_packed, bias, y, desc->dtype, s);
  }
  generic::FwdParams p{};
  p.a = x; p.b = w_packed; p.bias = bias; p.out = y;
  p.M = g.out_vox(); p.N = g.cout; p.K = g.k * g.k * g.k * g.cin;
  p.sd = g.d; p.sh = g.h; p.sw = g.w; p.sc = g.cin;
  p.md = g.od; p.mh = g.oh; p.mw = g.ow;
  p.ks = g.k; p.pd = g.pd; p.ph = g.ph; p.pw = g.pw;
  return cuda_status(generic::launch_fwd(p, MODE_CONV, desc->dtype, s));
}

int r4c_conv3d_dx(const r4c_conv_desc* desc, const void* go, const void* w_packed, void* dx,
                  void* workspace, size_t ws_bytes, r4c_stream_t stream) {
  Geom g;
  int st = check_desc(desc, R4C_LEG_DX, &g);
  if (st != R4C_OK) return st;
  if (g.in_vox() == 0) return R4C_OK;
  if (!go || !w_packed || !dx) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (use_stem_dx(desc, R4C_LEG_DX, g))
    return stem::launch_dx(g.n, g.d, g.h, g.w, g.cout, go, w_packed, dx, desc->dtype, s);
  tc::ConvPlan pl;
  if (use_tc(desc, R4C_LEG_DX, g, &pl)) {
    const void* src = go;
    if (needs_gpad(g)) {
      if (!workspace || ws_bytes < gpad_bytes(g)) return R4C_ERR_WORKSPACE;
      if (launch_cpad_n(go, workspace, g.out_vox(), g.cout, cout_eff(g), desc->dtype, s) != cudaSuccess)
        return R4C_ERR_CUDA;
      src = workspace;
    }
    return tc::launch_conv_tuned(pl, src, w_packed, nullptr, dx, desc->dtype, s);
  }
  // dX of a stride-1 conv is a conv of dY with the flipped, transposed kernel
  // and padding k-1-p (negative padding crops).
  generic::FwdParams p{};
  p.a = go; p.b = w_packed; p.bias = nullptr; p.out = dx;
  p.M = g.in_vox(); p.N = g.cin; p.K = g.k * g.k * g.k * g.cout;
  p.sd = g.od; p.sh = g.oh; p.sw = g.ow; p.sc = g.cout;
  p.md = g.d; p.mh = g.h; p.mw = g.w;
  p.ks = g.k; p.pd = g.k - 1 - g.pd; p.ph = g.k - 1 - g.ph; p.pw = g.k - 1 - g.pw;
  return cuda_status(generic::launch_fwd(p, MODE_CONV, desc->dtype, s));
}

int r4c_conv3d_dw(const r4c_conv_desc* desc, const void* x, const void* go, float* dw,
                  float* db, void* workspace, size_t ws_bytes, r4c_stream_t stream) {
  Geom g;
  int st = check_desc(desc, R4C_LEG_DW, &g);
  if (st != R4C_OK) return st;
  if (!dw) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int taps = g.k * g.k * g.k;
  if (g.out_vox() > 0 && use_stem_dw(desc, R4C_LEG_DW, g)) {
    if (!x || !go) return R4C_ERR_INVALID;
    return stem::launch_dw(g.n, g.d, g.h, g.w, g.cin, g.cout, g.pd, g.ph, g.pw, x, go, dw, db, workspace, ws_bytes,
                           desc->dtype, s);
  }
  tc::ConvPlan tcp;
  if (g.out_vox() > 0 && use_tc(desc, R4C_LEG_DW, g, &tcp)) {
    size_t part_bytes = 0;
    const size_t xpad = cpad_bytes(g), gpad = gpad_bytes(g), dwtmp = gpad_dw_bytes(g);
    const size_t need = xpad + gpad + dwtmp + tc_dw_ws(g, &part_bytes);
    if (ws_bytes < need || !workspace) return R4C_ERR_WORKSPACE;
    if (!x || !go) return R4C_ERR_INVALID;
    const void* xin = x;
    const void* gin = go;
    char* wsb = static_cast<char*>(workspace);
    if (xpad) {
      if (launch_cpad(x, wsb, g, desc->dtype, s) != cudaSuccess) return R4C_ERR_CUDA;
      xin = wsb;
      wsb += xpad;
    }
    float* dw_k = dw;
    float* db_k = db;
    if (gpad) {
      if (launch_cpad_n(go, wsb, g.out_vox(), g.cout, cout_eff(g), desc->dtype, s) != cudaSuccess)
        return R4C_ERR_CUDA;
      gin = wsb;
      wsb += gpad;
      dw_k = reinterpret_cast<float*>(wsb);
      db_k = db ? reinterpret_cast<float*>(wsb + align_up((size_t)cout_eff(g) * g.cin * taps * sizeof(float), 256))
                : nullptr;
      wsb += dwtmp;
    }
    bool db_done = false;
    int rc = tc::launch_dw(g.n, g.d, g.h, g.w, cin_eff(g), g.cin, cout_eff(g), g.k, g.pd, g.ph, g.pw, xin, gin, dw_k,
                           db_k, wsb, part_bytes, desc->dtype, s, &db_done);
    if (rc != R4C_OK) return rc;
    if (gpad) {  // OIDHW: the real Cout rows are a prefix of the padded result
      cudaError_t e = cudaMemcpyAsync(dw, dw_k, sizeof(float) * g.cout * g.cin * taps, cudaMemcpyDeviceToDevice, s);
      if (e == cudaSuccess && db && db_done)
        e = cudaMemcpyAsync(db, db_k, sizeof(float) * g.cout, cudaMemcpyDeviceToDevice, s);
      if (e != cudaSuccess) return R4C_ERR_CUDA;
    }
    if (db && !db_done) {
      float* part = reinterpret_cast<float*>(wsb + part_bytes);
      return cuda_status(generic::launch_db(go, g.out_vox(), g.cout, desc->dtype, part, db, s));
    }
    return R4C_OK;
  }
  WgradLayout L = wgrad_layout(g, false);
  if (ws_bytes < L.part_bytes + L.db_bytes || (!workspace && L.part_bytes + L.db_bytes))
    return R4C_ERR_WORKSPACE;
  if (g.out_vox() == 0) {
    cudaError_t e = cudaMemsetAsync(dw, 0, sizeof(float) * g.cout * g.cin * taps, s);
    if (e == cudaSuccess && db) e = cudaMemsetAsync(db, 0, sizeof(float) * g.cout, s);
    return cuda_status(e);
  }
  if (!x || !go) return R4C_ERR_INVALID;
  generic::WgradParams p{};
  p.x = x; p.go = go; p.partial = static_cast<float*>(workspace);
  p.P = taps * g.cin; p.N = g.cout; p.M = g.out_vox(); p.chunk = L.chunk;
  p.d = g.d; p.h = g.h; p.w = g.w; p.cin = g.cin;
  p.md = g.od; p.mh = g.oh; p.mw = g.ow; p.cout = g.cout;
  p.ks = g.k; p.pd = g.pd; p.ph = g.ph; p.pw = g.pw;
  cudaError_t e = generic::launch_wgrad(p, MODE_CONV, desc->dtype, L.S, dw, taps, s);
  if (e != cudaSuccess) return R4C_ERR_CUDA;
  if (db) {
    float* part = reinterpret_cast<float*>(static_cast<char*>(workspace) + L.part_bytes);
    e = generic::launch_db(go, g.out_vox(), g.cout, desc->dtype, part, db, s);
  }
  return cuda_status(e);
}

int r4c_tconv_fwd(const r4c_conv_desc* desc, const void* x, const void* w_packed,
                  const void* bias, void* y, void* workspace, size_t ws_bytes,
                  r4c_stream_t stream) {
  (void)workspace; (void)ws_bytes;
  Geom g;
  int st = check_desc(desc, R4C_LEG_TFWD, &g);
  if (st != R4C_OK) return st;
  if (g.in_vox() == 0) return R4C_OK;
  if (!x || !w_packed || !y) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (use_tc_tconv(desc, R4C_LEG_TFWD, g))
    return tconv::launch(0, g.n, g.d, g.h, g.w, g.cin, g.cout, x, w_packed, bias, y, desc->dtype, s);
  generic::FwdParams p{};
  p.a = x; p.b = w_packed; p.bias = bias; p.out = y;
  p.M = g.in_vox(); p.N = 8 * g.cout; p.K = g.cin;
  p.sd = g.d; p.sh = g.h; p.sw = g.w; p.sc = g.cin;
  p.md = g.d; p.mh = g.h; p.mw = g.w; p.oc = g.cout;
  p.ks = 2;
  return cuda_status(generic::launch_fwd(p, MODE_TFWD, desc->dtype, s));
}

int r4c_tconv_fwd_pitched(const r4c_conv_desc* desc, const void* x, const void* w_packed, const void* bias,
                          void* y, int y_pitch, void* workspace, size_t ws_bytes, r4c_stream_t stream) {
  Geom g;
  int st = check_desc(desc, R4C_LEG_TFWD, &g);
  if (st != R4C_OK) return st;
  if (y_pitch == g.cout) return r4c_tconv_fwd(desc, x, w_packed, bias, y, workspace, ws_bytes, stream);
  if (y_pitch < g.cout || y_pitch % 8) return R4C_ERR_INVALID;
  if (g.in_vox() == 0) return R4C_OK;
  if (!x || !w_packed || !y) return R4C_ERR_INVALID;
  if (!use_tc_tconv(desc, R4C_LEG_TFWD, g)) return R4C_ERR_UNSUPPORTED;
  return tconv::launch(0, g.n, g.d, g.h, g.w, g.cin, g.cout, x, w_packed, bias, y, desc->dtype,
                       reinterpret_cast<cudaStream_t>(stream), y_pitch);
}

int r4c_tconv_dx(const r4c_conv_desc* desc, const void* go, const void* w_packed, void* dx,
                 void* workspace, size_t ws_bytes, r4c_stream_t stream) {
  (void)workspace; (void)ws_bytes;
  Geom g;
  int st = check_desc(desc, R4C_LEG_TDX, &g);
  if (st != R4C_OK) return st;
  if (g.in_vox() == 0) return R4C_OK;
  if (!go || !w_packed || !dx) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (use_tc_tconv(desc, R4C_LEG_TDX, g))
    return tconv::launch(1, g.n, g.d, g.h, g.w, g.cin, g.cout, go, w_packed, nullptr, dx, desc->dtype, s);
  generic::FwdParams p{};
  p.a = go; p.b = w_packed; p.bias = nullptr; p.out = dx;
  p.M = g.in_vox(); p.N = g.cin; p.K = 8 * g.cout;
  p.sd = 2 * g.d; p.sh = 2 * g.h; p.sw = 2 * g.w; p.sc = g.cout;
  p.md = g.d; p.mh = g.h; p.mw = g.w;
  p.ks = 2;
  return cuda_status(generic::launch_fwd(p, MODE_TDX, desc->dtype, s));
}

int r4c_tconv_dw(const r4c_conv_desc* desc, const void* x, const void* go, float* dw,
                 float* db, void* workspace, size_t ws_bytes, r4c_stream_t stream) {
  Geom g;
  int st = check_desc(desc, R4C_LEG_TDW, &g);
  if (st != R4C_OK) return st;
  if (!dw) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  WgradLayout L = wgrad_layout(g, true);
  if (g.in_vox() > 0 && use_tc_tconv_dw(desc, R4C_LEG_TDW, g)) {
    const size_t pb = tconv::dw_workspace(g.n, g.d, g.h, g.w, g.cin, g.cout);
    if (!workspace || ws_bytes < pb + L.db_bytes) return R4C_ERR_WORKSPACE;
    if (!x || !go) return R4C_ERR_INVALID;
    bool db_done = false;
    int rc = tconv::launch_dw(g.n, g.d, g.h, g.w, g.cin, g.cout, x, go, dw, db, workspace, pb, desc->dtype, s,
                              &db_done);
    if (rc != R4C_OK || !db || db_done) return rc;
    float* part = reinterpret_cast<float*>(static_cast<char*>(workspace) + pb);
    return cuda_status(generic::launch_db(go, 8 * g.in_vox(), g.cout, desc->dtype, part, db, s));
  }
  if (ws_bytes < L.part_bytes + L.db_bytes || (!workspace && L.part_bytes + L.db_bytes))
    return R4C_ERR_WORKSPACE;
  if (g.in_vox() == 0) {
    cudaError_t e = cudaMemsetAsync(dw, 0, sizeof(float) * g.cout * g.cin * 8, s);
    if (e == cudaSuccess && db) e = cudaMemsetAsync(db, 0, sizeof(float) * g.cout, s);
    return cuda_status(e);
  }
  if (!x || !go) return R4C_ERR_INVALID;
  generic::WgradParams p{};
  p.x = x; p.go = go; p.partial = static_cast<float*>(workspace);
  p.P = g.cin; p.N = 8 * g.cout; p.M = g.in_vox(); p.chunk = L.chunk;
  p.d = g.d; p.h = g.h; p.w = g.w; p.cin = g.cin;
  p.md = g.d; p.mh = g.h; p.mw = g.w; p.cout = g.cout;
  p.ks = 2;
  cudaError_t e = generic::launch_wgrad(p, MODE_TDW, desc->dtype, L.S, dw, 8, s);
  if (e != cudaSuccess) return R4C_ERR_CUDA;
  if (db) {
    float* part = reinterpret_cast<float*>(static_cast<char*>(workspace) + L.part_bytes);
    e = generic::launch_db(go, 8 * g.in_vox(), g.cout, desc->dtype, part, db, s);
  }
  return cuda_status(e);
}

}  // extern "C"
