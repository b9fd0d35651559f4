// r4c_general.cu — Conv3d of any geometry: per-axis kernel size, stride,
// zero padding, dilation and groups (forward, dX, dW + db).
//
// The reference's kernels cover k in {1,3}, stride 1, dilation 1, groups 1
// (conv3d_wmma.py:89-95) and send every other geometry to the vendor library
// (conv3d_wmma.py:1241-1242); its generic Triton kernels (_fwd_kernel /
// _dgrad_kernel, conv3d_wmma.py:246-541) carry the general index arithmetic.
// Here:
//
//  * k = 2, stride 2, pad 0, dilation 1, groups 1 with even input extents —
//    the downsampling conv of encoder-decoder nets — is the transpose of the
//    k2s2 ConvTranspose3d, so it runs on the tcgen05 transpose-conv kernels
//    with the roles swapped: forward = the transpose conv's dX kernel (x in
//    place of dY), dX = its forward kernel (dY in place of x, no bias), dW =
//    its weight-gradient kernel with x and dY swapped (the transpose conv's
//    weight layout (Cin_t, Cout_t, 2, 2, 2) is the conv's (Cout, Cin, 2, 2, 2)).
//    db is summed from dY separately.
//  * everything else runs SIMT implicit GEMMs (64 x 64 tiles, fp32
//    accumulation) whose gathers apply stride, dilation and padding per axis
//    and whose tiles stay inside one group:
//      fwd  y[m, g*Cog + j]  = sum_{(tap, c)} x[in(m, tap), g*Cig + c] * w[g*Cog + j][c][tap]
//      dX   dx[m, g*Cig + j] = sum_{(tap, o)} dy[out(m, tap), g*Cog + o] * w[g*Cog + o][j][tap]
//           where out(m, tap) = (i + p - t*dil) / s when that divides exactly
//      dW   dw[g*Cog + j][c][tap] = sum_m dy[m, g*Cog + j] * x[in(m, tap), g*Cig + c],
//           split over m, partials summed in split order (deterministic)
//    Weights are read in PyTorch's own layout (Cout, Cin/groups, kd, kh, kw).
#include <algorithm>

#include "r4c_internal.h"

namespace r4c {
namespace general {

constexpr int BM = 64, BN = 64, BK = 16, NT = 256;

struct Geo {
  int n, d, h, w, od, oh, ow;
  int cin, cout, groups, cig, cog;
  int kd, kh, kw, taps;
  int sd, sh, sw, pd, ph, pw, dd, dh, dw;
  __host__ __device__ int64_t in_vox() const { return (int64_t)n * d * h * w; }
  __host__ __device__ int64_t out_vox() const { return (int64_t)n * od * oh * ow; }
};

static int out_extent(int i, int k, int s, int p, int dl) { return (i + 2 * p - dl * (k - 1) - 1) / s + 1; }

static int make_geo(const r4c_convex_desc* ds, Geo* g) {
  if (!ds) return R4C_ERR_INVALID;
  if (ds->dtype != R4C_BF16 && ds->dtype != R4C_F16 && ds->dtype != R4C_F32) return R4C_ERR_INVALID;
  if (ds->n < 0 || ds->d <= 0 || ds->h <= 0 || ds->w <= 0) return R4C_ERR_INVALID;
  if (ds->groups <= 0 || ds->cin <= 0 || ds->cout <= 0) return R4C_ERR_INVALID;
  if (ds->cin % ds->groups || ds->cout % ds->groups) return R4C_ERR_INVALID;
  const int ks[3] = {ds->kd, ds->kh, ds->kw}, st[3] = {ds->sd, ds->sh, ds->sw};
  const int pa[3] = {ds->pd, ds->ph, ds->pw}, dl[3] = {ds->dd, ds->dh, ds->dw};
  for (int i = 0; i < 3; ++i)
    if (ks[i] <= 0 || ks[i] > 64 || st[i] <= 0 || st[i] > 64 || pa[i] < 0 || pa[i] > 256 || dl[i] <= 0 || dl[i] > 64)
      return R4C_ERR_UNSUPPORTED;
  g->n = ds->n; g->d = ds->d; g->h = ds->h; g->w = ds->w;
  g->cin = ds->cin; g->cout = ds->cout; g->groups = ds->groups;
  g->cig = ds->cin / ds->groups; g->cog = ds->cout / ds->groups;
  g->kd = ds->kd; g->kh = ds->kh; g->kw = ds->kw; g->taps = ds->kd * ds->kh * ds->kw;
  g->sd = ds->sd; g->sh = ds->sh; g->sw = ds->sw;
  g->pd = ds->pd; g->ph = ds->ph; g->pw = ds->pw;
  g->dd = ds->dd; g->dh = ds->dh; g->dw = ds->dw;
  g->od = out_extent(g->d, g->kd, g->sd, g->pd, g->dd);
  g->oh = out_extent(g->h, g->kh, g->sh, g->ph, g->dh);
  g->ow = out_extent(g->w, g->kw, g->sw, g->pw, g->dw);
  if (g->od <= 0 || g->oh <= 0 || g->ow <= 0) return R4C_ERR_UNSUPPORTED;
  return R4C_OK;
}

// k2 s2 p0 d1 g1, even extents, channels the transpose-conv kernels take.
static bool k2s2_fast(const r4c_convex_desc* ds, const Geo& g) {
  if (ds->dtype == R4C_F32) return false;
  if (g.kd != 2 || g.kh != 2 || g.kw != 2 || g.sd != 2 || g.sh != 2 || g.sw != 2) return false;
  if (g.pd || g.ph || g.pw || g.dd != 1 || g.dh != 1 || g.dw != 1 || g.groups != 1) return false;
  if ((g.d | g.h | g.w) & 1) return false;
  return g.cin % 8 == 0 && g.cout % 8 == 0;
}

// The transpose conv whose legs are this conv's: its input is the conv's
// output grid with Cout channels, its output the conv's input grid.
static r4c_conv_desc tdesc_of(const Geo& g, int dtype) {
  r4c_conv_desc t{};
  t.n = g.n; t.d = g.od; t.h = g.oh; t.w = g.ow;
  t.cin = g.cout; t.cout = g.cin; t.k = 2;
  t.dtype = dtype;
  return t;
}

// ---------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------
struct KParams {
  const void* a;     // fwd: x; dx: dy
  const void* w;     // PyTorch layout weight
  const void* bias;  // fwd only, may be null
  void* out;
  Geo g;
};

// MODE 0: forward (rows = output voxels, cols = Cout of one group)
// MODE 1: dX      (rows = input voxels,  cols = Cin of one group)
template <typename T, int MODE>
__global__ void __launch_bounds__(NT) gemm_kernel(const KParams p) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const Geo& g = p.g;
  const T* __restrict__ src = static_cast<const T*>(p.a);
  const T* __restrict__ wt = static_cast<const T*>(p.w);
  const int tid = threadIdx.x;
  const int64_t M = MODE == 0 ? g.out_vox() : g.in_vox();
  const int ncol = MODE == 0 ? g.cog : g.cig;   // output channels of one group
  const int kred = MODE == 0 ? g.cig : g.cog;   // reduced channels of one group
  const int K = g.taps * kred;
  const int ntile = (ncol + BN - 1) / BN;
  const int grp = blockIdx.y / ntile;
  const int n0 = (blockIdx.y % ntile) * BN;
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  // row grid: the output grid (fwd) or the input grid (dX)
  const int gd = MODE == 0 ? g.od : g.d, gh = MODE == 0 ? g.oh : g.h, gw = MODE == 0 ? g.ow : g.w;
  // source grid and channels
  const int sd = MODE == 0 ? g.d : g.od, sh = MODE == 0 ? g.h : g.oh, sw = MODE == 0 ? g.w : g.ow;
  const int sc = MODE == 0 ? g.cin : g.cout;

  const int ak = tid & 15, am = tid >> 4;
  int rn[4], rz[4], ry[4], rx[4];
  bool rv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + am + 16 * i;
    rv[i] = m < M;
    int64_t t = rv[i] ? m : 0;
    rx[i] = (int)(t % gw); t /= gw;
    ry[i] = (int)(t % gh); t /= gh;
    rz[i] = (int)(t % gd);
    rn[i] = (int)(t / gd);
  }
  const int bk = tid >> 4, bn = (tid & 15) * 4;
  const int ty = tid >> 4, tx = tid & 15;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < K; k0 += BK) {
    // A: k = tap * kred + c (c fastest: consecutive channels of one position)
    {
      const int k = k0 + ak;
      int c = 0, td = 0, th = 0, tw = 0;
      if (k < K) {
        const int tap = k / kred;
        c = k - tap * kred;
        tw = tap % g.kw;
        th = (tap / g.kw) % g.kh;
        td = tap / (g.kw * g.kh);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float v = 0.f;
        if (rv[i] && k < K) {
          int iz, iy, ix;
          bool ok;
          if (MODE == 0) {
            iz = rz[i] * g.sd + td * g.dd - g.pd;
            iy = ry[i] * g.sh + th * g.dh - g.ph;
            ix = rx[i] * g.sw + tw * g.dw - g.pw;
            ok = true;
          } else {  // the output position this input position meets through tap (td, th, tw)
            const int nz = rz[i] + g.pd - td * g.dd, ny = ry[i] + g.ph - th * g.dh, nx = rx[i] + g.pw - tw * g.dw;
            ok = nz >= 0 && ny >= 0 && nx >= 0 && nz % g.sd == 0 && ny % g.sh == 0 && nx % g.sw == 0;
            iz = nz / g.sd; iy = ny / g.sh; ix = nx / g.sw;
          }
          if (ok && iz >= 0 && iz < sd && iy >= 0 && iy < sh && ix >= 0 && ix < sw)
            v = Elem<T>::to_f(src[((((int64_t)rn[i] * sd + iz) * sh + iy) * sw + ix) * sc + grp * kred + c]);
        }
        As[ak][am + 16 * i] = v;
      }
    }
    // B[k][j]: fwd w[grp*Cog + j][c][tap]; dX w[grp*Cog + o][j][tap] (k = (tap, o))
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = k0 + bk, col = n0 + bn + j;
      float v = 0.f;
      if (k < K && col < ncol) {
        const int tap = k / kred, c = k - tap * kred;
        const int64_t widx = MODE == 0 ? ((int64_t)(grp * g.cog + col) * g.cig + c) * g.taps + tap
                                       : ((int64_t)(grp * g.cog + c) * g.cig + col) * g.taps + tap;
        v = Elem<T>::to_f(wt[widx]);
      }
      Bs[bk][bn + j] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  T* __restrict__ out = static_cast<T*>(p.out);
  const T* __restrict__ bias = static_cast<const T*>(p.bias);
  const int oc = MODE == 0 ? g.cout : g.cin;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = n0 + tx * 4 + j;
      if (col >= ncol) continue;
      const int ch = grp * ncol + col;
      float v = acc[i][j];
      if (MODE == 0 && bias) v += Elem<T>::to_f(bias[ch]);
      out[m * oc + ch] = Elem<T>::from_f(v);
    }
  }
}

// dW partials: part[s][co][c * taps + tap] over the output voxels of split s.
template <typename T>
__global__ void __launch_bounds__(NT) wgrad_kernel(const void* xv, const void* gov, float* part, Geo g, int64_t chunk) {
  __shared__ float As[BK][BM + 4];  // [m][p]   p = tap * Cig + c
  __shared__ float Bs[BK][BN + 4];  // [m][j]
  const T* __restrict__ x = static_cast<const T*>(xv);
  const T* __restrict__ go = static_cast<const T*>(gov);
  const int tid = threadIdx.x;
  const int P = g.taps * g.cig;
  const int ntile = (g.cog + BN - 1) / BN;
  const int grp = blockIdx.y / ntile;
  const int n0 = (blockIdx.y % ntile) * BN;
  const int p0 = blockIdx.x * BM;
  const int s = blockIdx.z;
  const int64_t M = g.out_vox();
  const int64_t mbeg = (int64_t)s * chunk, mend = min(mbeg + chunk, M);
  const int lc = tid & 63, lr = tid >> 6;
  const int pp = p0 + lc;
  const bool a_ok = pp < P;
  int a_c = 0, a_d = 0, a_h = 0, a_w = 0;
  if (a_ok) {
    const int tap = pp / g.cig;
    a_c = pp - tap * g.cig;
    a_w = tap % g.kw;
    a_h = (tap / g.kw) % g.kh;
    a_d = tap / (g.kw * g.kh);
  }
  const int col = n0 + lc;
  const bool b_ok = col < g.cog;
  const int ty = tid >> 4, tx = tid & 15;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int64_t mb = mbeg; mb < mend; mb += BK) {
#pragma unroll
    for (int r = 0; r < BK / 4; ++r) {
      const int ml = lr + 4 * r;
      const int64_t m = mb + ml;
      float av = 0.f, bv = 0.f;
      if (m < mend) {
        int64_t t = m;
        const int ox = (int)(t % g.ow); t /= g.ow;
        const int oy = (int)(t % g.oh); t /= g.oh;
        const int oz = (int)(t % g.od);
        const int on = (int)(t / g.od);
        if (a_ok) {
          const int iz = oz * g.sd + a_d * g.dd - g.pd, iy = oy * g.sh + a_h * g.dh - g.ph,
                    ix = ox * g.sw + a_w * g.dw - g.pw;
          if (iz >= 0 && iz < g.d && iy >= 0 && iy < g.h && ix >= 0 && ix < g.w)
            av = Elem<T>::to_f(x[((((int64_t)on * g.d + iz) * g.h + iy) * g.w + ix) * g.cin + grp * g.cig + a_c]);
        }
        if (b_ok) bv = Elem<T>::to_f(go[m * g.cout + grp * g.cog + col]);
      }
      As[ml][lc] = av;
      Bs[ml][lc] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  // part layout [s][co_abs][c * taps + tap] = PyTorch's per-co order
  float* dst = part + (int64_t)s * g.cout * P;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int pr = p0 + ty * 4 + i;
    if (pr >= P) continue;
    const int tap = pr / g.cig, c = pr - tap * g.cig;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int cj = n0 + tx * 4 + j;
      if (cj >= g.cog) continue;
      dst[(int64_t)(grp * g.cog + cj) * P + (int64_t)c * g.taps + tap] = acc[i][j];
    }
  }
}

// Fixed-order sum of the split partials (deterministic).
__global__ void reduce_kernel(const float* __restrict__ part, int S, int64_t n, float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v = 0.f;
  for (int s = 0; s < S; ++s) v += part[(int64_t)s * n + i];
  out[i] = v;
}

// y[m][c] += bias[c] over a dense NDHWC tensor of n elements.
template <typename T>
__global__ void bias_kernel(void* yv, const void* bv, int64_t n, int C) {
  T* __restrict__ y = static_cast<T*>(yv);
  const T* __restrict__ b = static_cast<const T*>(bv);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = Elem<T>::from_f(Elem<T>::to_f(y[i]) + Elem<T>::to_f(b[i % C]));
}

// db partials: part[s][c] = sum over the voxels of split s (fixed order).
template <typename T>
__global__ void db_kernel(const void* gov, int64_t V, int C, int64_t chunk, float* part) {
  const T* __restrict__ go = static_cast<const T*>(gov);
  const int s = blockIdx.x;
  const int64_t b = (int64_t)s * chunk, e = min(b + chunk, V);
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float v = 0.f;
    for (int64_t m = b; m < e; ++m) v += Elem<T>::to_f(go[m * C + c]);
    part[(int64_t)s * C + c] = v;
  }
}

// ---------------------------------------------------------------------------
// Host
// ---------------------------------------------------------------------------
struct WgradSplit {
  int S;
  int64_t chunk;
  int Sdb;
  int64_t dbchunk;
  size_t part_bytes, db_bytes;
};

static WgradSplit wgrad_split(const Geo& g) {
  WgradSplit w{};
  const int P = g.taps * g.cig;
  const int tiles = cdiv(P, BM) * cdiv(g.cog, BN) * g.groups;
  const int64_t M = std::max<int64_t>(g.out_vox(), 1);
  int s = std::max(1, std::min(64, cdiv(2 * 148, tiles)));
  int64_t c = (M + s - 1) / s;
  c = std::max<int64_t>(BK, (c + BK - 1) / BK * BK);
  w.chunk = c;
  w.S = (int)((M + c - 1) / c);
  w.part_bytes = align_up((size_t)w.S * g.cout * P * sizeof(float), 256);
  const int64_t V = g.out_vox();
  w.dbchunk = std::max<int64_t>(256, (V + 295) / 296);
  w.Sdb = (int)std::max<int64_t>(1, (V + w.dbchunk - 1) / w.dbchunk);
  w.db_bytes = align_up((size_t)w.Sdb * g.cout * sizeof(float), 256);
  return w;
}

static int status(cudaError_t e) { return e == cudaSuccess ? R4C_OK : R4C_ERR_CUDA; }

template <typename T>
static cudaError_t launch_gemm(int mode, const KParams& p, cudaStream_t st) {
  const Geo& g = p.g;
  const int64_t M = mode == 0 ? g.out_vox() : g.in_vox();
  const int ncol = mode == 0 ? g.cog : g.cig;
  dim3 grid((unsigned)cdiv(M, BM), (unsigned)(cdiv(ncol, BN) * g.groups));
  if (mode == 0) gemm_kernel<T, 0><<<grid, NT, 0, st>>>(p);
  else gemm_kernel<T, 1><<<grid, NT, 0, st>>>(p);
  note_launches(1);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_wgrad(const Geo& g, const WgradSplit& sp, const void* x, const void* go, float* dw,
                                float* db, char* ws, cudaStream_t st) {
  float* part = reinterpret_cast<float*>(ws);
  const int P = g.taps * g.cig;
  dim3 grid((unsigned)cdiv(P, BM), (unsigned)(cdiv(g.cog, BN) * g.groups), (unsigned)sp.S);
  wgrad_kernel<T><<<grid, NT, 0, st>>>(x, go, part, g, sp.chunk);
  const int64_t n = (int64_t)g.cout * P;
  reduce_kernel<<<(unsigned)cdiv(n, 256), 256, 0, st>>>(part, sp.S, n, dw);
  note_launches(2);
  if (db) {
    float* dpart = reinterpret_cast<float*>(ws + sp.part_bytes);
    db_kernel<T><<<sp.Sdb, 256, 0, st>>>(go, g.out_vox(), g.cout, sp.dbchunk, dpart);
    reduce_kernel<<<(unsigned)cdiv(g.cout, 256), 256, 0, st>>>(dpart, sp.Sdb, g.cout, db);
    note_launches(2);
  }
  return cudaGetLastError();
}

}  // namespace general
}  // namespace r4c

using r4c::general::Geo;

extern "C" {

int r4c_convex_plan(const r4c_convex_desc* desc) {
  Geo g;
  const int st = r4c::general::make_geo(desc, &g);
  if (st != R4C_OK) return st;
  return r4c::general::k2s2_fast(desc, g) ? R4C_KERNEL_TC : R4C_KERNEL_GENERIC;
}

size_t r4c_convex_workspace_size(const r4c_convex_desc* desc, int leg) {
  Geo g;
  if (r4c::general::make_geo(desc, &g) != R4C_OK) return 0;
  if (r4c::general::k2s2_fast(desc, g)) {
    const r4c_conv_desc t = r4c::general::tdesc_of(g, desc->dtype);
    if (leg == R4C_LEG_FWD) return r4c::align_up(r4c_packed_weight_bytes(&t, R4C_LEG_TDX), 256) +
                                   r4c_workspace_size(&t, R4C_LEG_TDX);
    if (leg == R4C_LEG_DX) return r4c::align_up(r4c_packed_weight_bytes(&t, R4C_LEG_TFWD), 256) +
                                  r4c_workspace_size(&t, R4C_LEG_TFWD);
    if (leg == R4C_LEG_DW) return r4c_workspace_size(&t, R4C_LEG_TDW) + r4c::general::wgrad_split(g).db_bytes;
    return 0;
  }
  if (leg != R4C_LEG_DW) return 0;
  const auto sp = r4c::general::wgrad_split(g);
  return sp.part_bytes + sp.db_bytes;
}

int r4c_convex_fwd(const r4c_convex_desc* desc, const void* x, const void* w, const void* bias, void* y,
                   void* workspace, size_t ws_bytes, r4c_stream_t stream) {
  Geo g;
  const int st = r4c::general::make_geo(desc, &g);
  if (st != R4C_OK) return st;
  if (g.out_vox() == 0) return R4C_OK;
  if (!x || !w || !y) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (r4c::general::k2s2_fast(desc, g)) {
    // forward = the transpose conv's dX: the conv's x plays its dY
    const r4c_conv_desc t = r4c::general::tdesc_of(g, desc->dtype);
    const size_t pb = r4c::align_up(r4c_packed_weight_bytes(&t, R4C_LEG_TDX), 256);
    const size_t tw = r4c_workspace_size(&t, R4C_LEG_TDX);
    if (!workspace || ws_bytes < pb + tw) return R4C_ERR_WORKSPACE;
    int rc = r4c_pack_weight(&t, R4C_LEG_TDX, w, desc->dtype, workspace, stream);
    if (rc != R4C_OK) return rc;
    rc = r4c_tconv_dx(&t, x, workspace, y, static_cast<char*>(workspace) + pb, tw, stream);
    if (rc != R4C_OK || !bias) return rc;
    // the bias is not part of the transpose conv's dX: added in place
    cudaError_t e;
    const int64_t n = g.out_vox() * g.cout;
    if (desc->dtype == R4C_BF16)
      r4c::general::bias_kernel<__nv_bfloat16><<<(unsigned)r4c::cdiv(n, 256), 256, 0, s>>>(y, bias, n, g.cout);
    else
      r4c::general::bias_kernel<__half><<<(unsigned)r4c::cdiv(n, 256), 256, 0, s>>>(y, bias, n, g.cout);
    r4c::note_launches(1);
    e = cudaGetLastError();
    return r4c::general::status(e);
  }
  r4c::general::KParams p{x, w, bias, y, g};
  cudaError_t e;
  if (desc->dtype == R4C_BF16) e = r4c::general::launch_gemm<__nv_bfloat16>(0, p, s);
  else if (desc->dtype == R4C_F16) e = r4c::general::launch_gemm<__half>(0, p, s);
  else e = r4c::general::launch_gemm<float>(0, p, s);
  return r4c::general::status(e);
}

int r4c_convex_dx(const r4c_convex_desc* desc, const void* go, const void* w, void* dx, void* workspace,
                  size_t ws_bytes, r4c_stream_t stream) {
  Geo g;
  const int st = r4c::general::make_geo(desc, &g);
  if (st != R4C_OK) return st;
  if (g.in_vox() == 0) return R4C_OK;
  if (!go || !w || !dx) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (r4c::general::k2s2_fast(desc, g)) {
    // dX = the transpose conv's forward of dY (no bias)
    const r4c_conv_desc t = r4c::general::tdesc_of(g, desc->dtype);
    const size_t pb = r4c::align_up(r4c_packed_weight_bytes(&t, R4C_LEG_TFWD), 256);
    const size_t tw = r4c_workspace_size(&t, R4C_LEG_TFWD);
    if (!workspace || ws_bytes < pb + tw) return R4C_ERR_WORKSPACE;
    int rc = r4c_pack_weight(&t, R4C_LEG_TFWD, w, desc->dtype, workspace, stream);
    if (rc != R4C_OK) return rc;
    return r4c_tconv_fwd(&t, go, workspace, nullptr, dx, static_cast<char*>(workspace) + pb, tw, stream);
  }
  r4c::general::KParams p{go, w, nullptr, dx, g};
  cudaError_t e;
  if (desc->dtype == R4C_BF16) e = r4c::general::launch_gemm<__nv_bfloat16>(1, p, s);
  else if (desc->dtype == R4C_F16) e = r4c::general::launch_gemm<__half>(1, p, s);
  else e = r4c::general::launch_gemm<float>(1, p, s);
  return r4c::general::status(e);
}

int r4c_convex_dw(const r4c_convex_desc* desc, const void* x, const void* go, float* dw, float* db, void* workspace,
                  size_t ws_bytes, r4c_stream_t stream) {
  Geo g;
  const int st = r4c::general::make_geo(desc, &g);
  if (st != R4C_OK) return st;
  if (!dw) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t need = r4c_convex_workspace_size(desc, R4C_LEG_DW);
  if (ws_bytes < need || (need && !workspace)) return R4C_ERR_WORKSPACE;
  if (g.out_vox() == 0) {
    cudaError_t e = cudaMemsetAsync(dw, 0, sizeof(float) * g.cout * g.cig * g.taps, s);
    if (e == cudaSuccess && db) e = cudaMemsetAsync(db, 0, sizeof(float) * g.cout, s);
    return r4c::general::status(e);
  }
  if (!x || !go) return R4C_ERR_INVALID;
  const auto sp = r4c::general::wgrad_split(g);
  if (r4c::general::k2s2_fast(desc, g)) {
    // dW = the transpose conv's dW with x and dY swapped; db from dY here
    const r4c_conv_desc t = r4c::general::tdesc_of(g, desc->dtype);
    const size_t tw = r4c_workspace_size(&t, R4C_LEG_TDW);
    int rc = r4c_tconv_dw(&t, go, x, dw, nullptr, workspace, tw, stream);
    if (rc != R4C_OK || !db) return rc;
    float* dpart = reinterpret_cast<float*>(static_cast<char*>(workspace) + tw);
    cudaError_t e;
    if (desc->dtype == R4C_BF16)
      r4c::general::db_kernel<__nv_bfloat16><<<sp.Sdb, 256, 0, s>>>(go, g.out_vox(), g.cout, sp.dbchunk, dpart);
    else
      r4c::general::db_kernel<__half><<<sp.Sdb, 256, 0, s>>>(go, g.out_vox(), g.cout, sp.dbchunk, dpart);
    r4c::general::reduce_kernel<<<(unsigned)r4c::cdiv(g.cout, 256), 256, 0, s>>>(dpart, sp.Sdb, g.cout, db);
    r4c::note_launches(2);
    e = cudaGetLastError();
    return r4c::general::status(e);
  }
  char* ws = static_cast<char*>(workspace);
  cudaError_t e;
  if (desc->dtype == R4C_BF16) e = r4c::general::launch_wgrad<__nv_bfloat16>(g, sp, x, go, dw, db, ws, s);
  else if (desc->dtype == R4C_F16) e = r4c::general::launch_wgrad<__half>(g, sp, x, go, dw, db, ws, s);
  else e = r4c::general::launch_wgrad<float>(g, sp, x, go, dw, db, ws, s);
  return r4c::general::status(e);
}

}  // extern "C"
