// r4c_generic.cu — SIMT implicit-GEMM kernels for every leg and channel count.
//
// These are the always-available CUDA path: any Cin/Cout, k in {1,3} with any
// zero padding, and the k2s2 transpose conv. The tcgen05 kernels in r4c_tc.cu
// take the shapes they support (channels a multiple of 8); everything else
// lands here. GEMM views follow the reference's Triton kernels:
//   fwd   Y[m, co]  = sum_{k=(tap,ci)} X[shift_tap(m), ci] * Wp[k, co]
//         (_fwd_k3_kernel / _fwd_kernel, conv3d_wmma.py:246-444)
//   dW    dW[(tap,ci), co] = sum_m X[shift_tap(m), ci] * dY[m, co], split over m
//         (_wgrad_kernel, conv3d_wmma.py:543-634)
//   tfwd  Y8[m, (tap,co)] = X[m, :] @ Wt[:, (tap,co)], scattered 2x2x2
//         (_tr_k2s2_fwd_kernel, conv3d_wmma.py:792-860)
//   tdx   dX[m, ci] = sum_{(tap,co)} dY[2m+tap, co] * Wt[ci, (tap,co)]
//         (_tr_k2s2_dx_kernel, conv3d_wmma.py:862-931)
//   tdw   dW[ci, (tap,co)] = sum_m X[m, ci] * dY[2m+tap, co]
//         (_tr_k2s2_dw_kernel, conv3d_wmma.py:933-1012)
// All accumulate in fp32; split-K partials are summed in a fixed order.
#include "r4c_internal.h"

namespace r4c {
namespace generic {

constexpr int BM = 64, BN = 64, BK = 16, NT = 256;

// ---------------------------------------------------------------------------
// Forward-shaped GEMM: conv fwd / conv dX (as a conv of dY) / tconv fwd / tconv dX
// ---------------------------------------------------------------------------
template <typename T, int MODE>
__global__ void __launch_bounds__(NT) fwd_gemm_kernel(FwdParams p) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const T* __restrict__ src = static_cast<const T*>(p.a);
  const T* __restrict__ wk = static_cast<const T*>(p.b);
  const int tid = threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;

  // A loader: k_local = tid % 16, rows am + 16*i.
  const int ak = tid & 15;
  const int am = tid >> 4;
  int rn[4], rz[4], ry[4], rx[4];
  bool rv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t m = m0 + am + 16 * i;
    rv[i] = m < p.M;
    int64_t t = rv[i] ? m : 0;
    rx[i] = (int)(t % p.mw); t /= p.mw;
    ry[i] = (int)(t % p.mh); t /= p.mh;
    rz[i] = (int)(t % p.md); t /= p.md;
    rn[i] = (int)t;
  }
  // B loader: k_local = tid / 16, four consecutive n.
  const int bk = tid >> 4;
  const int bn = (tid & 15) * 4;
  // Compute mapping.
  const int ty = tid >> 4, tx = tid & 15;

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < p.K; k0 += BK) {
    const int k = k0 + ak;
    // decode k
    int c = 0, kd = 0, kh = 0, kw = 0;
    if (k < p.K) {
      if (MODE == MODE_CONV) {
        int tap = k / p.sc;
        c = k - tap * p.sc;
        kw = tap % p.ks; int t2 = tap / p.ks;
        kh = t2 % p.ks; kd = t2 / p.ks;
      } else if (MODE == MODE_TDX) {
        int tap = k / p.sc;
        c = k - tap * p.sc;
        kd = tap >> 2; kh = (tap >> 1) & 1; kw = tap & 1;
      } else {
        c = k;
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float v = 0.f;
      if (rv[i] && k < p.K) {
        int64_t off = -1;
        if (MODE == MODE_CONV) {
          int iz = rz[i] + kd - p.pd, iy = ry[i] + kh - p.ph, ix = rx[i] + kw - p.pw;
          if (iz >= 0 && iz < p.sd && iy >= 0 && iy < p.sh && ix >= 0 && ix < p.sw)
            off = ((((int64_t)rn[i] * p.sd + iz) * p.sh + iy) * p.sw + ix) * p.sc + c;
        } else if (MODE == MODE_TDX) {
          int iz = 2 * rz[i] + kd, iy = 2 * ry[i] + kh, ix = 2 * rx[i] + kw;
          off = ((((int64_t)rn[i] * p.sd + iz) * p.sh + iy) * p.sw + ix) * p.sc + c;
        } else {
          off = (m0 + am + 16 * i) * (int64_t)p.sc + c;
        }
        if (off >= 0) v = Elem<T>::to_f(src[off]);
      }
      As[ak][am + 16 * i] = v;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int kk = k0 + bk, nn = n0 + bn + j;
      Bs[bk][bn + j] = (kk < p.K && nn < p.N) ? Elem<T>::to_f(wk[(int64_t)kk * p.N + nn]) : 0.f;
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

  // Epilogue.
  T* __restrict__ out = static_cast<T*>(p.out);
  const T* __restrict__ bias = static_cast<const T*>(p.bias);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t m = m0 + ty * 4 + i;
    if (m >= p.M) continue;
    int64_t oidx_base = 0;
    int ox = 0, oy = 0, oz = 0, on = 0;
    if (MODE == MODE_TFWD) {
      int64_t t = m;
      ox = (int)(t % p.mw); t /= p.mw;
      oy = (int)(t % p.mh); t /= p.mh;
      oz = (int)(t % p.md); on = (int)(t / p.md);
    } else {
      oidx_base = m * (int64_t)p.N;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int nn = n0 + tx * 4 + j;
      if (nn >= p.N) continue;
      float v = acc[i][j];
      if (MODE == MODE_TFWD) {
        int tap = nn / p.oc, co = nn - tap * p.oc;
        if (bias) v += Elem<T>::to_f(bias[co]);
        int kd = tap >> 2, kh = (tap >> 1) & 1, kw = tap & 1;
        int64_t yi = ((((int64_t)on * (2 * p.md) + 2 * oz + kd) * (2 * p.mh) + 2 * oy + kh) *
                          (2 * p.mw) + 2 * ox + kw) * p.oc + co;
        out[yi] = Elem<T>::from_f(v);
      } else {
        if (bias) v += Elem<T>::to_f(bias[nn]);
        out[oidx_base + nn] = Elem<T>::from_f(v);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Weight-gradient GEMM with split-K over voxels: partial[s][p][n].
// ---------------------------------------------------------------------------
template <typename T, int MODE>
__global__ void __launch_bounds__(NT) wgrad_gemm_kernel(WgradParams p) {
  __shared__ float As[BK][BM + 4];  // [m_local][p_local]
  __shared__ float Bs[BK][BN + 4];  // [m_local][n_local]
  const T* __restrict__ x = static_cast<const T*>(p.x);
  const T* __restrict__ go = static_cast<const T*>(p.go);
  const int tid = threadIdx.x;
  const int p0 = blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;
  const int s = blockIdx.z;
  const int64_t mbeg = (int64_t)s * p.chunk;
  const int64_t mend = min(mbeg + (int64_t)p.chunk, p.M);

  // Loader mapping: column = tid % 64, rows tid/64 + 4*i.
  const int lc = tid & 63;
  const int lr = tid >> 6;
  // Row (p) decode for the A loader (fixed for the CTA).
  const int pp = p0 + lc;
  int a_ci = 0, a_kd = 0, a_kh = 0, a_kw = 0;
  const bool a_ok = pp < p.P;
  if (MODE == MODE_CONV) {
    int tap = pp / p.cin;
    a_ci = pp - tap * p.cin;
    a_kw = tap % p.ks; int t2 = tap / p.ks;
    a_kh = t2 % p.ks; a_kd = t2 / p.ks;
  } else {
    a_ci = pp;
  }
  // Column (n) decode for the B loader.
  const int nn = n0 + lc;
  const bool b_ok = nn < p.N;
  int b_co = nn, b_kd = 0, b_kh = 0, b_kw = 0;
  if (MODE == MODE_TDW) {
    int tap = nn / p.cout;
    b_co = nn - tap * p.cout;
    b_kd = tap >> 2; b_kh = (tap >> 1) & 1; b_kw = tap & 1;
  }
  const int ty = tid >> 4, tx = tid & 15;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int64_t mk = mbeg; mk < mend; mk += BK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int ml = lr + 4 * i;
      const int64_t m = mk + ml;
      float av = 0.f, bv = 0.f;
      if (m < mend) {
        // decode m over the reduction grid (md, mh, mw)
        int64_t t = m;
        int x0 = (int)(t % p.mw); t /= p.mw;
        int y0 = (int)(t % p.mh); t /= p.mh;
        int z0 = (int)(t % p.md); int n_ = (int)(t / p.md);
        if (a_ok) {
          if (MODE == MODE_CONV) {
            int iz = z0 + a_kd - p.pd, iy = y0 + a_kh - p.ph, ix = x0 + a_kw - p.pw;
            if (iz >= 0 && iz < p.d && iy >= 0 && iy < p.h && ix >= 0 && ix < p.w)
              av = Elem<T>::to_f(x[((((int64_t)n_ * p.d + iz) * p.h + iy) * p.w + ix) * p.cin + a_ci]);
          } else {
            av = Elem<T>::to_f(x[m * p.cin + a_ci]);
          }
        }
        if (b_ok) {
          if (MODE == MODE_CONV) {
            bv = Elem<T>::to_f(go[m * p.cout + b_co]);
          } else {
            int gz = 2 * z0 + b_kd, gy = 2 * y0 + b_kh, gx = 2 * x0 + b_kw;
            bv = Elem<T>::to_f(go[((((int64_t)n_ * (2 * p.md) + gz) * (2 * p.mh) + gy) * (2 * p.mw) + gx) *
                                      p.cout + b_co]);
          }
        }
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
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int prow = p0 + ty * 4 + i;
    if (prow >= p.P) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int col = n0 + tx * 4 + j;
      if (col >= p.N) continue;
      p.partial[((int64_t)s * p.P + prow) * p.N + col] = acc[i][j];
    }
  }
}

// Fixed-order sum of the split partials, written in PyTorch's weight layout.
__global__ void wgrad_reduce_kernel(const float* __restrict__ partial, int S, int P, int N,
                                    float* __restrict__ dw, int mode, int cin, int cout, int taps) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)P * N) return;
  int prow = (int)(idx / N), col = (int)(idx % N);
  float sum = 0.f;
  for (int s = 0; s < S; ++s) sum += partial[((int64_t)s * P + prow) * N + col];
  if (mode == MODE_CONV) {
    int tap = prow / cin, ci = prow - tap * cin;
    dw[((int64_t)col * cin + ci) * taps + tap] = sum;
  } else {
    int tap = col / cout, co = col - tap * cout;
    dw[((int64_t)prow * cout + co) * 8 + tap] = sum;
  }
}

// ---------------------------------------------------------------------------
// Bias gradient: per-block channel sums over a voxel range, then a fixed-order
// sum of the block partials.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NT) db_partial_kernel(const T* __restrict__ go, int64_t V, int C,
                                                         int64_t chunk, float* __restrict__ part) {
  __shared__ float red[NT];
  const int s = blockIdx.x;
  const int64_t vbeg = (int64_t)s * chunk;
  const int64_t vend = min(vbeg + chunk, V);
  for (int c0 = 0; c0 < C; c0 += NT) {
    const int cw = min(NT, C - c0);
    const int rows = NT / cw;
    const int tid = threadIdx.x;
    const int r = tid / cw, c = tid - r * cw;
    float acc = 0.f;
    if (r < rows) {
      for (int64_t v = vbeg + r; v < vend; v += rows) acc += Elem<T>::to_f(go[v * C + c0 + c]);
    }
    red[tid] = acc;
    __syncthreads();
    if (tid < cw) {
      float sum = 0.f;
      for (int rr = 0; rr < rows; ++rr) sum += red[rr * cw + tid];
      part[(int64_t)s * C + c0 + tid] = sum;
    }
    __syncthreads();
  }
}

// C a multiple of 8: thread (r, g) of a block sums 8-channel group g of the
// positions vbeg + r, vbeg + r + rows, ... with 16-byte loads (consecutive
// threads read consecutive 16-byte groups of a position, then the next
// position), four loads in flight; the block then adds its rows in a fixed
// order. The scalar kernel above keeps ~10 two-byte loads in flight per
// block and ran at ~0.3 TB/s.
template <typename T>
__global__ void __launch_bounds__(256) db_partial_vec_kernel(const T* __restrict__ go, int64_t V, int C,
                                                             int64_t chunk, float* __restrict__ part) {
  __shared__ float red[256 * 8];
  const int G = C / 8;
  const int rows = 256 / G;
  const int tid = threadIdx.x;
  const int r = tid / G, g = tid - r * G;
  const int64_t vbeg = (int64_t)blockIdx.x * chunk;
  const int64_t vend = min(vbeg + chunk, V);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (r < rows) {
    const T* base = go + 8 * g;
    int64_t v = vbeg + r;
    for (; v + 3 * rows < vend; v += 4 * rows) {
      uint4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = *reinterpret_cast<const uint4*>(base + (v + u * rows) * C);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const T* e = reinterpret_cast<const T*>(&q[u]);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += Elem<T>::to_f(e[i]);
      }
    }
    for (; v < vend; v += rows) {
      const uint4 q = *reinterpret_cast<const uint4*>(base + v * C);
      const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += Elem<T>::to_f(e[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[tid * 8 + i] = acc[i];
  __syncthreads();
  // thread (g, i) adds row r's value of channel 8g + i, rows in order
  if (tid < C) {
    const int gg = tid / 8, i = tid - gg * 8;
    float sum = 0.f;
    for (int rr = 0; rr < rows; ++rr) sum += red[(rr * G + gg) * 8 + i];
    part[(int64_t)blockIdx.x * C + tid] = sum;
  }
}

// A block covers 32 channels with 8 lanes each: lane j adds splits j, j+8,
// ... in order and the eight lane sums meet in a fixed tree (deterministic).
// One thread per channel walking all splits was a chain of ~40 dependent L2
// round trips even with eight loads in flight.
__global__ void __launch_bounds__(256) db_reduce_kernel(const float* __restrict__ part, int S, int C,
                                                        float* __restrict__ db) {
  __shared__ float red[8][33];
  const int o = threadIdx.x & 31, lj = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + o;
  float sum = 0.f;
  if (c < C) {
#pragma unroll 4
    for (int s = lj; s < S; s += 8) sum += part[(int64_t)s * C + c];
  }
  red[lj][o] = sum;
  __syncthreads();
  if (lj == 0 && c < C)
    db[c] = ((red[0][o] + red[1][o]) + (red[2][o] + red[3][o])) + ((red[4][o] + red[5][o]) + (red[6][o] + red[7][o]));
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
template <typename T>
static cudaError_t launch_fwd_t(const FwdParams& p, int mode, cudaStream_t st) {
  dim3 grid((unsigned)cdiv(p.M, BM), (unsigned)cdiv(p.N, BN));
  if (mode == MODE_CONV) fwd_gemm_kernel<T, MODE_CONV><<<grid, NT, 0, st>>>(p);
  else if (mode == MODE_TFWD) fwd_gemm_kernel<T, MODE_TFWD><<<grid, NT, 0, st>>>(p);
  else fwd_gemm_kernel<T, MODE_TDX><<<grid, NT, 0, st>>>(p);
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_fwd(const FwdParams& p, int mode, int dtype, cudaStream_t st) {
  if (p.M <= 0 || p.N <= 0) return cudaSuccess;
  if (dtype == R4C_BF16) return launch_fwd_t<__nv_bfloat16>(p, mode, st);
  return launch_fwd_t<__half>(p, mode, st);
}

void wgrad_split(int64_t M, int P, int N, int* S, int* chunk) {
  int tiles = cdiv(P, BM) * cdiv(N, BN);
  int s = cdiv(2 * 148, tiles);
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  int64_t c = (M + s - 1) / s;
  c = (c + BK - 1) / BK * BK;
  if (c < BK) c = BK;
  *chunk = (int)c;
  *S = (int)((M + c - 1) / c);
  if (*S < 1) *S = 1;
}

void db_split(int64_t V, int* S, int64_t* chunk) {
  int s = 2 * 148;
  int64_t c = (V + s - 1) / s;
  if (c < 256) c = 256;
  *chunk = c;
  *S = (int)((V + c - 1) / c);
  if (*S < 1) *S = 1;
}

template <typename T>
static cudaError_t launch_wgrad_t(const WgradParams& p, int mode, int S, float* dw, int taps,
                                  cudaStream_t st) {
  dim3 grid((unsigned)cdiv(p.P, BM), (unsigned)cdiv(p.N, BN), (unsigned)S);
  if (mode == MODE_CONV) wgrad_gemm_kernel<T, MODE_CONV><<<grid, NT, 0, st>>>(p);
  else wgrad_gemm_kernel<T, MODE_TDW><<<grid, NT, 0, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int64_t tot = (int64_t)p.P * p.N;
  wgrad_reduce_kernel<<<(unsigned)cdiv(tot, 256), 256, 0, st>>>(p.partial, S, p.P, p.N, dw, mode,
                                                                 p.cin, p.cout, taps);
  note_launches(2);
  return cudaGetLastError();
}

cudaError_t launch_wgrad(const WgradParams& p, int mode, int dtype, int S, float* dw, int taps,
                         cudaStream_t st) {
  if (p.P <= 0 || p.N <= 0) return cudaSuccess;
  if (dtype == R4C_BF16) return launch_wgrad_t<__nv_bfloat16>(p, mode, S, dw, taps, st);
  return launch_wgrad_t<__half>(p, mode, S, dw, taps, st);
}

cudaError_t launch_db(const void* go, int64_t V, int C, int dtype, float* part, float* db,
                      cudaStream_t st) {
  if (C <= 0) return cudaSuccess;
  int S; int64_t chunk;
  db_split(V, &S, &chunk);
  if (V <= 0) {
    cudaError_t e = cudaMemsetAsync(db, 0, sizeof(float) * C, st);
    return e;
  }
  const bool vec = C % 8 == 0 && C <= 256 && (reinterpret_cast<uintptr_t>(go) & 15) == 0;
  if (vec && dtype == R4C_BF16)
    db_partial_vec_kernel<__nv_bfloat16><<<S, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(go), V, C, chunk,
                                                             part);
  else if (vec)
    db_partial_vec_kernel<__half><<<S, 256, 0, st>>>(static_cast<const __half*>(go), V, C, chunk, part);
  else if (dtype == R4C_BF16)
    db_partial_kernel<__nv_bfloat16><<<S, NT, 0, st>>>(static_cast<const __nv_bfloat16*>(go), V, C, chunk, part);
  else
    db_partial_kernel<__half><<<S, NT, 0, st>>>(static_cast<const __half*>(go), V, C, chunk, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  db_reduce_kernel<<<cdiv(C, 32), 256, 0, st>>>(part, S, C, db);
  note_launches(2);
  return cudaGetLastError();
}

}  // namespace generic
}  // namespace r4c
