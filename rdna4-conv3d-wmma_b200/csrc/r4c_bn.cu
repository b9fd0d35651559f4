// r4c_bn.cu — BatchNorm3d (training statistics) fused with ReLU, NDHWC.
//
// The reference's model blocks are Conv3d -> BatchNorm3d -> ReLU
// (benches/unet_e2e.py:13-20 of the reference), and its design notes put
// BatchNorm at ~11 ms of its step (the reference's docs/DESIGN.md:66). Stock PyTorch runs BN
// and ReLU as separate kernels: statistics, normalise, ReLU forward; ReLU
// backward, BN reduction, BN dX — about 13 full passes over the activation.
// Here the pair takes 5 + 3:
//   forward   stats (read x)  ->  finalize (C threads)  ->  y = relu(w*(x-mean)*invstd + b) (read x, write y)
//   backward  sums of g and g*(x-mean), g = dy * [pre-activation > 0] (read dy, x)
//             -> finalize -> dx = (g - mean(g) - (x-mean)*invstd^2*mean(g*(x-mean))) * w*invstd
//                           (read dy, x, write dx)
// These are the normalisation and gradient expressions of PyTorch's own
// BatchNorm kernels, so the fused pair rounds like the stock one. The ReLU
// mask is recomputed from x with the forward's own expression, so it is
// bit-identical to the forward's.
//
// Reductions are deterministic: each block owns a fixed voxel range and sums
// it in a fixed thread order, block partials are summed in block order in
// double. Elements: bf16 / fp16 storage, fp32 arithmetic; C a multiple of 8
// (16-byte vectors of 8 channels of one voxel).
#include <algorithm>

#include "r4c_internal.h"

namespace r4c {
namespace bn {

constexpr int kMaxThreads = 256;

// Threads per block for C channels: (C/8) vector lanes x R voxel rows.
static int rows_for(int C) { return std::max(1, kMaxThreads / (C / 8)); }

template <typename T>
struct Vec8 {
  uint4 raw;
  __device__ __forceinline__ void to_f(float* f) const {
    const T* p = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = Elem<T>::to_f(p[i]);
  }
  __device__ __forceinline__ void from_f(const float* f) {
    T* p = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) p[i] = Elem<T>::from_f(f[i]);
  }
};

// MODE 0: part[b] = (sum u, sum u^2) per channel over the block's voxels,
//         u = x - pivot (pivot = the first voxel's value: sums of deviations
//         from a value inside the distribution keep E[u^2] - E[u]^2 free of
//         the cancellation that E[x^2] - E[x]^2 suffers when |mean| >> std).
// MODE 1: part[b] = (sum g, sum g*(x - mean)), g = dy * [pre-activation > 0]
//         (g = dy when relu is 0).
// Layout: part[b][0..C) first sum, part[b][C..2C) second.
// Pre-activation of the normalisation, in PyTorch's order of operations.
__device__ __forceinline__ float bn_pre(float x, float mean, float invstd, float w, float b) {
  return w * (x - mean) * invstd + b;
}
template <typename T, int MODE>
__global__ void __launch_bounds__(kMaxThreads) sums_kernel(const T* __restrict__ x, const T* __restrict__ dy,
                                                           const float* __restrict__ af, const float* __restrict__ mi,
                                                           int64_t vox, int C, int64_t chunk, int relu,
                                                           float* __restrict__ part) {
  extern __shared__ float red[];  // [R][2*C]
  const int nv = C / 8;
  const int lane = threadIdx.x % nv, row = threadIdx.x / nv;
  const int R = blockDim.x / nv;
  const int c0 = lane * 8;
  float s1[8], s2[8], sc[8], sh[8], mu[8], is[8];
  {
    float pv[8];
    if (MODE == 0) {
      if (mi) {  // the caller's pivot
#pragma unroll
        for (int i = 0; i < 8; ++i) pv[i] = mi[c0 + i];
      } else {   // voxel 0
        Vec8<T> p0;
        p0.raw = *reinterpret_cast<const uint4*>(x + c0);
        p0.to_f(pv);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s1[i] = 0.f;
      s2[i] = 0.f;
      sc[i] = MODE == 1 ? af[c0 + i] : 0.f;       // gamma
      sh[i] = MODE == 1 ? af[C + c0 + i] : 0.f;   // beta
      mu[i] = MODE == 1 ? mi[c0 + i] : pv[i];
      is[i] = MODE == 1 ? mi[C + c0 + i] : 1.f;
    }
  }
  const int64_t v0 = (int64_t)blockIdx.x * chunk, v1 = min(v0 + chunk, vox);
  if (row < R) {
    // four voxels per iteration, loads first (four 16-byte loads in flight)
    for (int64_t vb = v0 + row; vb < v1; vb += 4 * (int64_t)R) {
      Vec8<T> a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t v = vb + (int64_t)u * R;
        if (v < v1) {
          a[u].raw = *reinterpret_cast<const uint4*>(x + v * C + c0);
          if (MODE == 1) b[u].raw = *reinterpret_cast<const uint4*>(dy + v * C + c0);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t v = vb + (int64_t)u * R;
        if (v >= v1) break;
        float xf[8];
        a[u].to_f(xf);
        if (MODE == 0) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float u = xf[i] - mu[i];
            s1[i] += u;
            s2[i] = fmaf(u, u, s2[i]);
          }
        } else {
          float gf[8];
          b[u].to_f(gf);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float g = (!relu || bn_pre(xf[i], mu[i], is[i], sc[i], sh[i]) > 0.f) ? gf[i] : 0.f;
            s1[i] += g;
            s2[i] = fmaf(g, xf[i] - mu[i], s2[i]);
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      red[row * 2 * C + c0 + i] = s1[i];
      red[row * 2 * C + C + c0 + i] = s2[i];
    }
  }
  __syncthreads();
  // fixed-order sum over the rows, one thread per output
  for (int o = threadIdx.x; o < 2 * C; o += blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < R; ++r) acc += red[r * 2 * C + o];
    part[(int64_t)blockIdx.x * 2 * C + o] = acc;
  }
}

// Forward finalize: mean, invstd, and the affine pair (gamma, beta; 1 and 0
// when absent); running statistics updated with the unbiased variance.
__global__ void fwd_finalize_kernel(const float* __restrict__ sums_in, int C, double count,
                                    const float* __restrict__ gamma, const float* __restrict__ beta, float eps,
                                    float momentum, float* running_mean, float* running_var, float* mean_invstd,
                                    float* affine) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const double s1 = sums_in[c], s2 = sums_in[C + c];
  const double pivot = sums_in[2 * C + c];             // the stats pass's pivot
  const double du = s1 / count;                       // mean of x - pivot
  const double mean = pivot + du;
  double var = s2 / count - du * du;
  if (var < 0.0) var = 0.0;
  const float invstd = (float)(1.0 / sqrt(var + (double)eps));
  const float g = gamma ? gamma[c] : 1.f, b = beta ? beta[c] : 0.f;
  mean_invstd[c] = (float)mean;
  mean_invstd[C + c] = invstd;
  affine[c] = g;
  affine[C + c] = b;
  if (running_mean) {
    const double unbiased = count > 1.0 ? var * count / (count - 1.0) : var;
    running_mean[c] = (1.f - momentum) * running_mean[c] + momentum * (float)mean;
    running_var[c] = (1.f - momentum) * running_var[c] + momentum * (float)unbiased;
  }
}

// Sum of the block partials (fixed order, double) into sums[2C]; with
// `pivots`, also the pivot the statistics pass used into sums[2C:3C) (the
// caller's, or voxel 0 of x).
template <typename T>
__global__ void sum_parts_kernel(const float* __restrict__ part, int S, int C, float* __restrict__ sums, int pivots,
                                 const float* __restrict__ pivot, const T* __restrict__ x) {
  // one warp per output: lane l sums partials l, l+32, ... in order, then a
  // fixed butterfly over the lanes (same result on every run). Four loads
  // are issued before their adds (the adds keep their order): one load at a
  // time left each of these small launches waiting on ~19 L2 round trips.
  const int o = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (o < 2 * C) {
    double a = 0.0;
    const int64_t st = 2 * (int64_t)C;
    int s = lane;
    for (; s + 96 < S; s += 128) {
      const float v0 = part[(int64_t)s * st + o], v1 = part[(int64_t)(s + 32) * st + o];
      const float v2 = part[(int64_t)(s + 64) * st + o], v3 = part[(int64_t)(s + 96) * st + o];
      a += v0;
      a += v1;
      a += v2;
      a += v3;
    }
    for (; s < S; s += 32) a += part[(int64_t)s * st + o];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
    if (lane == 0) sums[o] = (float)a;
  }
  if (pivots && lane == 0 && o < C) sums[2 * C + o] = pivot ? pivot[o] : Elem<T>::to_f(x[o]);
}

// Backward finalize from (sum g, sum g*(x - mean)): dgamma = sum g*(x-mean) *
// invstd, dbeta = sum g, and the dX coefficients (mean(g), invstd^2 *
// mean(g*(x-mean)), gamma * invstd).
__global__ void bwd_finalize_kernel(const float* __restrict__ sums, const float* __restrict__ mean_invstd,
                                    const float* __restrict__ affine, int C, double count, float* dgamma,
                                    float* dbeta, float* coef) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const float sg = sums[c], sgx = sums[C + c];
  const float invstd = mean_invstd[C + c];
  if (dgamma) dgamma[c] = sgx * invstd;
  if (dbeta) dbeta[c] = sg;
  const float norm = (float)(1.0 / count);
  coef[c] = sg * norm;
  coef[C + c] = invstd * invstd * (sgx * norm);
  coef[2 * C + c] = affine[c] * invstd;
}

// Elementwise passes: each thread takes U = 4 vectors of 8 channels per
// iteration (all loads issued before any use, so four 16-byte loads per
// thread are in flight), then grid-strides.
constexpr int kU = 4;

// y = relu(w*(x-mean)*invstd + b) (relu optional).
template <typename T>
__global__ void __launch_bounds__(256) apply_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                    const float* __restrict__ mi, const float* __restrict__ af,
                                                    int64_t nvec, int C, int relu) {
  // blockDim is a multiple of C/8 (vec_threads), so every vector a thread
  // touches holds the same 8 channels: their parameters stay in registers
  const int nv = C / 8;
  const int c0 = (int)(threadIdx.x % nv) * 8;
  float pm[8], pi[8], pw[8], pb[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    pm[k] = __ldg(mi + c0 + k);
    pi[k] = __ldg(mi + C + c0 + k);
    pw[k] = __ldg(af + c0 + k);
    pb[k] = __ldg(af + C + c0 + k);
  }
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < nvec; base += stride * kU) {
    Vec8<T> a[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * stride;
      if (i < nvec) a[u].raw = __ldcs(reinterpret_cast<const uint4*>(x) + i);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * stride;
      if (i >= nvec) break;
      float f[8];
      a[u].to_f(f);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float v = bn_pre(f[k], pm[k], pi[k], pw[k], pb[k]);
        f[k] = relu ? (v > 0.f ? v : 0.f) : v;
      }
      a[u].from_f(f);
      reinterpret_cast<uint4*>(y)[i] = a[u].raw;
    }
  }
}

// dx = (g - mean(g) - (x-mean) * f1) * f2, g = dy * [pre-activation > 0] (relu) or dy.
template <typename T>
__global__ void __launch_bounds__(256) dx_kernel(const T* __restrict__ dy, const T* __restrict__ x, T* __restrict__ dx,
                                                 const float* __restrict__ mi, const float* __restrict__ af,
                                                 const float* __restrict__ coef, int64_t nvec, int C, int relu) {
  // blockDim is a multiple of C/8: fixed channels per thread, parameters in registers
  const int nv = C / 8;
  const int c0 = (int)(threadIdx.x % nv) * 8;
  float pm[8], pi[8], pw[8], pb[8], q0[8], q1[8], q2[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    pm[k] = __ldg(mi + c0 + k);
    pi[k] = __ldg(mi + C + c0 + k);
    pw[k] = __ldg(af + c0 + k);
    pb[k] = __ldg(af + C + c0 + k);
    q0[k] = __ldg(coef + c0 + k);
    q1[k] = __ldg(coef + C + c0 + k);
    q2[k] = __ldg(coef + 2 * C + c0 + k);
  }
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < nvec; base += stride * kU) {
    Vec8<T> a[kU], b[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * stride;
      if (i < nvec) {
        a[u].raw = __ldcs(reinterpret_cast<const uint4*>(x) + i);
        b[u].raw = __ldcs(reinterpret_cast<const uint4*>(dy) + i);
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * stride;
      if (i >= nvec) break;
      float xf[8], gf[8];
      a[u].to_f(xf);
      b[u].to_f(gf);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float g = gf[k];
        if (relu && !(bn_pre(xf[k], pm[k], pi[k], pw[k], pb[k]) > 0.f)) g = 0.f;
        xf[k] = (g - q0[k] - (xf[k] - pm[k]) * q1[k]) * q2[k];
      }
      a[u].from_f(xf);
      reinterpret_cast<uint4*>(dx)[i] = a[u].raw;
    }
  }
}

// ---------------------------------------------------------------------------
// BatchNorm + ReLU + MaxPool3d(2), NDHWC, even extents. One thread per
// (pooled voxel, 4-channel group): it normalises the 2x2x2 window, writes
// the eight outputs y (with a channel pitch, so y can be a channel slice of a
// wider buffer: the decoder's concatenation) and their maximum p. Backward
// recomputes the window's outputs from x, takes the argmax the way PyTorch's
// max_pool3d does (scan in (d, h, w) order, first maximum; a NaN wins), and
// routes dP there: g = [pre > 0] * (dY + [argmax] * dP).
// Four channels (8-byte vectors) per thread rather than eight: the backward
// holds the window's x and dY as raw vectors plus the parameters, and at
// eight channels that took ~250 registers (two blocks per SM, issue-bound);
// at four the kernels fit in 128 registers, four blocks per SM.
// ---------------------------------------------------------------------------
struct PoolGeo {
  int n, d, h, w, C;
  int ypitch;          // channels between consecutive voxels of y / dY
  int64_t pvox;        // pooled voxels n * d/2 * h/2 * w/2 (< 2^32: a pooled voxel is >= 128 bytes of x)
};

template <typename T>
struct Vec4 {
  uint2 raw;
  __device__ __forceinline__ void to_f(float* f) const {
    const T* p = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = Elem<T>::to_f(p[i]);
  }
  __device__ __forceinline__ void from_f(const float* f) {
    T* p = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = Elem<T>::from_f(f[i]);
  }
};

// Voxel index of the (0, 0, 0) corner of pooled voxel pv's window, and the
// offset of window voxel k = (a, b, c) from it (32-bit decomposition of pv).
__device__ __forceinline__ int64_t window_base(const PoolGeo& g, uint32_t pv) {
  const uint32_t pw = (uint32_t)g.w >> 1, ph = (uint32_t)g.h >> 1, pd = (uint32_t)g.d >> 1;
  uint32_t t = pv;
  const uint32_t px = t % pw; t /= pw;
  const uint32_t py = t % ph; t /= ph;
  const uint32_t pz = t % pd;
  const uint32_t nb = t / pd;
  return (((int64_t)nb * g.d + 2 * pz) * g.h + 2 * py) * g.w + 2 * px;
}
__device__ __forceinline__ int64_t window_off(const PoolGeo& g, int k) {
  return (int64_t)(k >> 2) * g.h * g.w + ((k >> 1) & 1) * g.w + (k & 1);
}

template <typename T>
__device__ __forceinline__ float round_to(float v) { return Elem<T>::to_f(Elem<T>::from_f(v)); }

// The normalisation parameters of the 4 channels c0..c0+3.
struct BnPar4 {
  float m[4], is[4], w[4], b[4];
};
__device__ __forceinline__ void load_par4(BnPar4& P, const float* mi, const float* af, int C, int c0) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    P.m[j] = __ldg(mi + c0 + j);
    P.is[j] = __ldg(mi + C + c0 + j);
    P.w[j] = __ldg(af + c0 + j);
    P.b[j] = __ldg(af + C + c0 + j);
  }
}

// 8 window voxels x 4 channels of a pitched NDHWC tensor, as raw vectors.
template <typename T>
__device__ __forceinline__ void window_load(const T* __restrict__ src, const PoolGeo& g, int64_t base, int pitch,
                                            int c0, uint2 (&r)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) r[k] = *reinterpret_cast<const uint2*>(src + (base + window_off(g, k)) * pitch + c0);
}

// Per channel j the maximum of the window's rounded outputs (mx) and its
// voxel (3 bits at 3j of the result), the way PyTorch's max_pool3d scans:
// (d, h, w) order, first maximum, a NaN wins.
template <typename T>
__device__ __forceinline__ uint32_t window_argmax(const uint2 (&xr)[8], const BnPar4& P, float (&mx)[4]) {
  uint32_t am = 0u;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    Vec4<T> a;
    a.raw = xr[k];
    float xf[4];
    a.to_f(xf);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float pre = bn_pre(xf[i], P.m[i], P.is[i], P.w[i], P.b[i]);
      const float y = round_to<T>(pre > 0.f ? pre : 0.f);
      if (k == 0 || y > mx[i] || isnan(y)) {
        mx[i] = y;
        am = (am & ~(7u << (3 * i))) | ((uint32_t)k << (3 * i));
      }
    }
  }
  return am;
}

// g = [pre > 0] * (dY + [argmax] * dP) of window voxel k; xf = x there.
template <typename T>
__device__ __forceinline__ void window_grad_k(int k, const uint2& xr, const uint2& gyr, const float (&gpf)[4],
                                              uint32_t am, const BnPar4& P, float (&xf)[4], float (&gf)[4]) {
  Vec4<T> a, b;
  a.raw = xr;
  b.raw = gyr;
  a.to_f(xf);
  b.to_f(gf);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float pre = bn_pre(xf[j], P.m[j], P.is[j], P.w[j], P.b[j]);
    const float v = gf[j] + (((am >> (3 * j)) & 7u) == (uint32_t)k ? gpf[j] : 0.f);
    gf[j] = pre > 0.f ? v : 0.f;
  }
}

// zlead > 0: the zlead channels before y's of each voxel (the lead part of
// the concatenation buffer that y is a slice of) are written with zeros in
// the same pass, so that every line of the buffer is written whole. A
// slice written alone leaves partial 32-byte sectors, and on this HBM a
// partial sector costs a read-modify-write: at the UNet's level 0 the
// pitched forward measured 222 us against 97 us for the same bytes dense.
template <typename T>
__global__ void __launch_bounds__(128, 4) pool_fwd_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                          T* __restrict__ p, const float* __restrict__ mi,
                                                          const float* __restrict__ af, PoolGeo g, int zlead,
                                                          uint16_t* __restrict__ amo) {
  const uint32_t nv = (uint32_t)g.C / 4;
  const uint64_t total = (uint64_t)g.pvox * nv;
  BnPar4 P;
  int pc0 = -1;  // channel group whose parameters P holds (fixed when blockDim % nv == 0)
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t pv = (uint32_t)i / nv;  // i < total < 2^32
    const int c0 = (int)((uint32_t)i - pv * nv) * 4;
    if (c0 != pc0) {
      load_par4(P, mi, af, g.C, c0);
      pc0 = c0;
    }
    const int64_t base = window_base(g, pv);
    uint2 xr[8];
    window_load<T>(x, g, base, g.C, c0, xr);
    float mx[4];
    const uint32_t am = window_argmax<T>(xr, P, mx);
    if (amo) amo[i] = (uint16_t)am;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      Vec4<T> a;
      a.raw = xr[k];
      float f[4];
      a.to_f(f);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float pre = bn_pre(f[j], P.m[j], P.is[j], P.w[j], P.b[j]);
        f[j] = pre > 0.f ? pre : 0.f;
      }
      Vec4<T> o;
      o.from_f(f);
      T* yv = y + (base + window_off(g, k)) * g.ypitch;
      for (int c = c0; c < zlead; c += g.C) *reinterpret_cast<uint2*>(yv - zlead + c) = make_uint2(0u, 0u);
      *reinterpret_cast<uint2*>(yv + c0) = o.raw;
    }
    Vec4<T> o;
    o.from_f(mx);
    reinterpret_cast<uint2*>(p)[i] = o.raw;
  }
}

// part[b] = (sum g, sum g*(x - mean)) over the block's pooled voxels; a
// block is R rows of C/4 lanes (R = 1 and several groups per lane when
// C/4 > blockDim).
template <typename T>
__global__ void __launch_bounds__(512) pool_sums_kernel(const T* __restrict__ x, const T* __restrict__ gy,
                                                        const T* __restrict__ gp, const float* __restrict__ mi,
                                                        const float* __restrict__ af, PoolGeo g, int64_t chunk,
                                                        const uint16_t* __restrict__ ami, float* __restrict__ part) {
  extern __shared__ float red[];  // [R][2*C]
  const int nv = g.C / 4;
  const int lane = threadIdx.x % nv, row = threadIdx.x / nv;
  const int R = blockDim.x / nv;
  const int c0 = lane * 4;
  BnPar4 P;
  load_par4(P, mi, af, g.C, c0);
  float s1[4], s2[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) { s1[j] = 0.f; s2[j] = 0.f; }
  const int64_t v0 = (int64_t)blockIdx.x * chunk, v1 = min(v0 + chunk, g.pvox);
  if (row < R) {
    for (int64_t pv = v0 + row; pv < v1; pv += R) {
      const int64_t base = window_base(g, (uint32_t)pv);
      uint2 xr[8], gyr[8];
      window_load<T>(x, g, base, g.C, c0, xr);
      window_load<T>(gy, g, base, g.ypitch, c0, gyr);
      Vec4<T> pb;
      pb.raw = reinterpret_cast<const uint2*>(gp)[pv * nv + lane];
      float gpf[4], mx[4];
      pb.to_f(gpf);
      const uint32_t am = ami ? (uint32_t)ami[pv * nv + lane] : window_argmax<T>(xr, P, mx);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float xf[4], gf[4];
        window_grad_k<T>(k, xr[k], gyr[k], gpf, am, P, xf, gf);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s1[j] += gf[j];
          s2[j] = fmaf(gf[j], xf[j] - P.m[j], s2[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      red[row * 2 * g.C + c0 + j] = s1[j];
      red[row * 2 * g.C + g.C + c0 + j] = s2[j];
    }
  }
  __syncthreads();
  for (int o = threadIdx.x; o < 2 * g.C; o += blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < R; ++r) acc += red[r * 2 * g.C + o];
    part[(int64_t)blockIdx.x * 2 * g.C + o] = acc;
  }
}

template <typename T>
__global__ void __launch_bounds__(128, 3) pool_dx_kernel(const T* __restrict__ x, const T* __restrict__ gy,
                                                         const T* __restrict__ gp, T* __restrict__ dx,
                                                         const float* __restrict__ mi, const float* __restrict__ af,
                                                         const float* __restrict__ coef, PoolGeo g,
                                                         const uint16_t* __restrict__ ami) {
  const uint32_t nv = (uint32_t)g.C / 4;
  const uint64_t total = (uint64_t)g.pvox * nv;
  BnPar4 P;
  float q0[4], q1[4], q2[4];
  int pc0 = -1;  // channel group whose parameters are held (fixed when blockDim % nv == 0)
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t pv = (uint32_t)i / nv;  // i < total < 2^32
    const int c0 = (int)((uint32_t)i - pv * nv) * 4;
    if (c0 != pc0) {
      load_par4(P, mi, af, g.C, c0);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        q0[j] = __ldg(coef + c0 + j);
        q1[j] = __ldg(coef + g.C + c0 + j);
        q2[j] = __ldg(coef + 2 * g.C + c0 + j);
      }
      pc0 = c0;
    }
    const int64_t base = window_base(g, pv);
    uint2 xr[8], gyr[8];
    window_load<T>(x, g, base, g.C, c0, xr);
    window_load<T>(gy, g, base, g.ypitch, c0, gyr);
    Vec4<T> pb;
    pb.raw = reinterpret_cast<const uint2*>(gp)[i];
    float gpf[4], mx[4];
    pb.to_f(gpf);
    const uint32_t am = ami ? (uint32_t)ami[i] : window_argmax<T>(xr, P, mx);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float xf[4], gf[4], f[4];
      window_grad_k<T>(k, xr[k], gyr[k], gpf, am, P, xf, gf);
#pragma unroll
      for (int j = 0; j < 4; ++j) f[j] = (gf[j] - q0[j] - (xf[j] - P.m[j]) * q1[j]) * q2[j];
      Vec4<T> o;
      o.from_f(f);
      *reinterpret_cast<uint2*>(dx + (base + window_off(g, k)) * g.C + c0) = o.raw;
    }
  }
}

struct Split {
  int S;
  int64_t chunk;
};

static Split split_for(int64_t vox, int64_t min_chunk = 64) {
  // about four blocks per SM (small levels of a UNet need the blocks: each
  // thread's voxel loop is a chain of dependent loads), at least min_chunk
  // voxels each
  Split s;
  s.chunk = std::max<int64_t>(min_chunk, (vox + 591) / 592);
  s.S = (int)std::max<int64_t>(1, (vox + s.chunk - 1) / s.chunk);
  return s;
}

static int grid_for(int64_t nvec) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((nvec + 255) / 256, 148 * 4));
}
// Threads per block of the element-wise kernels: a multiple of C/8 (the 16-byte
// vectors of one voxel), so each thread keeps the same 8 channels.
static int vec_threads(int C) { return (256 / (C / 8)) * (C / 8); }
// Pool kernels (128 threads, 4 channels each): likewise a multiple of C/4
// when C/4 <= 128.
static int pool_threads(int C) { return C / 4 <= 128 ? (128 / (C / 4)) * (C / 4) : 128; }

static bool ok_args(const void* p, int64_t vox, int C, int dtype) {
  return p && vox >= 0 && C > 0 && C % 8 == 0 && C <= 2048 && (dtype == R4C_BF16 || dtype == R4C_F16) &&
         (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

// Dense copy of a channel slice: dst[v][0..C) = src[v * pitch + 0..C), in
// 16-byte vectors (nvec = C/8 per voxel, pitch16 = pitch/8). A slice of a
// wider NDHWC buffer read this way touches only its own bytes; PyTorch's
// strided copy of the same view runs a scalar element loop (~1.8 TB/s at
// UNet sizes). Four independent vectors per thread and step keep enough
// loads in flight.
template <typename I>
__global__ void __launch_bounds__(256) slice_copy_kernel(const uint4* __restrict__ src, int64_t pitch16,
                                                         uint4* __restrict__ dst, I nvec, I total) {
  const I stride = (I)gridDim.x * blockDim.x;
  for (I i = (I)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += 4 * stride) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const I e = i + u * stride;
      if (e < total) {
        const I vx = e / nvec;
        v[u] = src[(int64_t)vx * pitch16 + (e - vx * nvec)];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const I e = i + u * stride;
      if (e < total) dst[e] = v[u];
    }
  }
}

}  // namespace bn
}  // namespace r4c

using namespace r4c::bn;

extern "C" {

size_t r4c_bn_workspace_size(int64_t vox, int C) {
  if (C <= 0) return 0;
  const Split s = split_for(vox);
  return r4c::align_up((size_t)s.S * 2 * C * sizeof(float), 256);
}

static int launch_sums(int mode, const void* x, const void* dy, const float* ss, const float* mi, int64_t vox, int C,
                       int dtype, int relu, float* sums, void* ws, size_t ws_bytes, cudaStream_t s) {
  const Split sp = split_for(vox);
  if (!ws || ws_bytes < r4c_bn_workspace_size(vox, C)) return R4C_ERR_WORKSPACE;
  float* part = static_cast<float*>(ws);
  const int R = rows_for(C);
  const int threads = R * (C / 8);
  const size_t smem = (size_t)R * 2 * C * sizeof(float);
  if (smem > 48 * 1024) return R4C_ERR_UNSUPPORTED;
  if (dtype == R4C_BF16) {
    const auto* xb = static_cast<const __nv_bfloat16*>(x);
    const auto* gb = static_cast<const __nv_bfloat16*>(dy);
    if (mode == 0) sums_kernel<__nv_bfloat16, 0><<<sp.S, threads, smem, s>>>(xb, gb, ss, mi, vox, C, sp.chunk, relu, part);
    else sums_kernel<__nv_bfloat16, 1><<<sp.S, threads, smem, s>>>(xb, gb, ss, mi, vox, C, sp.chunk, relu, part);
  } else {
    const auto* xh = static_cast<const __half*>(x);
    const auto* gh = static_cast<const __half*>(dy);
    if (mode == 0) sums_kernel<__half, 0><<<sp.S, threads, smem, s>>>(xh, gh, ss, mi, vox, C, sp.chunk, relu, part);
    else sums_kernel<__half, 1><<<sp.S, threads, smem, s>>>(xh, gh, ss, mi, vox, C, sp.chunk, relu, part);
  }
  if (dtype == R4C_BF16)
    sum_parts_kernel<__nv_bfloat16><<<(2 * C + 7) / 8, 256, 0, s>>>(part, sp.S, C, sums, mode == 0, mi,
                                                                     static_cast<const __nv_bfloat16*>(x));
  else
    sum_parts_kernel<__half><<<(2 * C + 7) / 8, 256, 0, s>>>(part, sp.S, C, sums, mode == 0, mi,
                                                              static_cast<const __half*>(x));
  r4c::note_launches(2);
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

int r4c_bn_stats(const void* x, int64_t vox, int C, int dtype, const float* pivot, float* sums, void* ws,
                 size_t ws_bytes, r4c_stream_t stream) {
  if (!ok_args(x, vox, C, dtype) || !sums) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (vox == 0) {
    if (cudaMemsetAsync(sums, 0, 2 * C * sizeof(float), s) != cudaSuccess) return R4C_ERR_CUDA;
    if (pivot) return cudaMemcpyAsync(sums + 2 * C, pivot, C * sizeof(float), cudaMemcpyDeviceToDevice, s) ==
                              cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
    return cudaMemsetAsync(sums + 2 * C, 0, C * sizeof(float), s) == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
  }
  return launch_sums(0, x, nullptr, nullptr, pivot, vox, C, dtype, 0, sums, ws, ws_bytes, s);
}

int r4c_bn_finalize(const float* sums, double count, int C, const float* gamma, const float* beta, float eps,
                    float momentum, float* running_mean, float* running_var, float* mean_invstd,
                    float* affine, r4c_stream_t stream) {
  if (!sums || !mean_invstd || !affine || C <= 0 || count <= 0.0) return R4C_ERR_INVALID;
  if ((running_mean == nullptr) != (running_var == nullptr)) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  fwd_finalize_kernel<<<(C + 127) / 128, 128, 0, s>>>(sums, C, count, gamma, beta, eps, momentum, running_mean,
                                                       running_var, mean_invstd, affine);
  r4c::note_launches(1);
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

int r4c_bn_relu_fwd(const void* x, void* y, const float* mean_invstd, const float* affine, int64_t vox, int C,
                    int dtype, int relu, r4c_stream_t stream) {
  if (!ok_args(x, vox, C, dtype) || !ok_args(y, vox, C, dtype) || !mean_invstd || !affine) return R4C_ERR_INVALID;
  if (vox == 0) return R4C_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t nvec = vox * (C / 8);
  if (dtype == R4C_BF16)
    apply_kernel<__nv_bfloat16><<<grid_for(nvec), vec_threads(C), 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                               static_cast<__nv_bfloat16*>(y), mean_invstd, affine, nvec,
                                                               C, relu);
  else
    apply_kernel<__half><<<grid_for(nvec), vec_threads(C), 0, s>>>(static_cast<const __half*>(x), static_cast<__half*>(y),
                                                        mean_invstd, affine, nvec, C, relu);
  r4c::note_launches(1);
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

int r4c_bn_relu_bwd_sums(const void* dy, const void* x, const float* mean_invstd, const float* affine,
                         int64_t vox, int C, int dtype, int relu, float* sums, void* ws, size_t ws_bytes,
                         r4c_stream_t stream) {
  if (!ok_args(x, vox, C, dtype) || !ok_args(dy, vox, C, dtype) || !affine || !mean_invstd || !sums)
    return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (vox == 0) return cudaMemsetAsync(sums, 0, 2 * C * sizeof(float), s) == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
  return launch_sums(1, x, dy, affine, mean_invstd, vox, C, dtype, relu, sums, ws, ws_bytes, s);
}

int r4c_bn_relu_bwd_dx(const void* dy, const void* x, void* dx, const float* mean_invstd, const float* affine,
                       const float* sums, double count, int64_t vox, int C, int dtype, int relu, float* dgamma,
                       float* dbeta, float* coef, r4c_stream_t stream) {
  if (!ok_args(x, vox, C, dtype) || !ok_args(dy, vox, C, dtype) || !affine || !mean_invstd || !sums || !coef)
    return R4C_ERR_INVALID;
  if (dx && !ok_args(dx, vox, C, dtype)) return R4C_ERR_INVALID;
  if (count <= 0.0) return R4C_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  bwd_finalize_kernel<<<(C + 127) / 128, 128, 0, s>>>(sums, mean_invstd, affine, C, count, dgamma, dbeta, coef);
  r4c::note_launches(1);
  if (dx && vox > 0) {
    const int64_t nvec = vox * (C / 8);
    if (dtype == R4C_BF16)
      dx_kernel<__nv_bfloat16><<<grid_for(nvec), vec_threads(C), 0, s>>>(
          static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(dx),
          mean_invstd, affine, coef, nvec, C, relu);
    else
      dx_kernel<__half><<<grid_for(nvec), vec_threads(C), 0, s>>>(static_cast<const __half*>(dy), static_cast<const __half*>(x),
                                                       static_cast<__half*>(dx), mean_invstd, affine, coef, nvec, C,
                                                       relu);
    r4c::note_launches(1);
  }
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

static bool pool_args(const void* x, int n, int d, int h, int w, int C, int pitch, int dtype) {
  return x && n >= 0 && d > 0 && h > 0 && w > 0 && !(d & 1) && !(h & 1) && !(w & 1) && C > 0 && C % 8 == 0 &&
         C <= 2048 && pitch >= C && pitch % 8 == 0 && (dtype == R4C_BF16 || dtype == R4C_F16) &&
         (reinterpret_cast<uintptr_t>(x) & 15) == 0;
}

static PoolGeo pool_geo(int n, int d, int h, int w, int C, int pitch) {
  PoolGeo g;
  g.n = n; g.d = d; g.h = h; g.w = w; g.C = C; g.ypitch = pitch;
  g.pvox = (int64_t)n * (d / 2) * (h / 2) * (w / 2);
  return g;
}

int r4c_channel_slice_copy(const void* src, int src_pitch, void* dst, int64_t vox, int C, int dtype,
                           r4c_stream_t stream) {
  if (!src || !dst || vox < 0 || C <= 0 || C % 8 || src_pitch < C || src_pitch % 8 ||
      (dtype != R4C_BF16 && dtype != R4C_F16) || (reinterpret_cast<uintptr_t>(src) & 15) ||
      (reinterpret_cast<uintptr_t>(dst) & 15))
    return R4C_ERR_INVALID;
  const int64_t nvec = C / 8;
  const int64_t total = vox * nvec;
  if (total == 0) return R4C_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 1023) / 1024, 148 * 8));
  if (total < (int64_t)0xFFFFFFFF - 4ll * grid * 256)
    slice_copy_kernel<uint32_t><<<grid, 256, 0, s>>>(static_cast<const uint4*>(src), src_pitch / 8,
                                                     static_cast<uint4*>(dst), (uint32_t)nvec, (uint32_t)total);
  else
    slice_copy_kernel<int64_t><<<grid, 256, 0, s>>>(static_cast<const uint4*>(src), src_pitch / 8,
                                                    static_cast<uint4*>(dst), nvec, total);
  r4c::note_launches(1);
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

static int pool_fwd_launch(const void* x, void* y, int y_pitch, int zlead, void* p, void* argmax,
                           const float* mean_invstd, const float* affine, int n, int d, int h, int w, int C,
                           int dtype, r4c_stream_t stream) {
  const PoolGeo g = pool_geo(n, d, h, w, C, y_pitch);
  if (g.pvox == 0) return R4C_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t total = g.pvox * (C / 4);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 127) / 128, 148 * 8));
  if (dtype == R4C_BF16)
    pool_fwd_kernel<__nv_bfloat16><<<grid, pool_threads(g.C), 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                        static_cast<__nv_bfloat16*>(y), static_cast<__nv_bfloat16*>(p),
                                                        mean_invstd, affine, g, zlead,
                                                        static_cast<uint16_t*>(argmax));
  else
    pool_fwd_kernel<__half><<<grid, pool_threads(g.C), 0, s>>>(static_cast<const __half*>(x), static_cast<__half*>(y),
                                                 static_cast<__half*>(p), mean_invstd, affine, g, zlead,
                                                 static_cast<uint16_t*>(argmax));
  r4c::note_launches(1);
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

int r4c_bn_relu_pool_fwd(const void* x, void* y, int y_pitch, void* p, const float* mean_invstd, const float* affine,
                         int n, int d, int h, int w, int C, int dtype, r4c_stream_t stream) {
  if (!pool_args(x, n, d, h, w, C, C, dtype) || !pool_args(y, n, d, h, w, C, y_pitch, dtype) ||
      !pool_args(p, n, d, h, w, C, C, dtype) || !mean_invstd || !affine)
    return R4C_ERR_INVALID;
  return pool_fwd_launch(x, y, y_pitch, 0, p, nullptr, mean_invstd, affine, n, d, h, w, C, dtype, stream);
}

int r4c_bn_relu_pool_fwd_cat(const void* x, void* buf, int lead, void* p, void* argmax, const float* mean_invstd,
                             const float* affine, int n, int d, int h, int w, int C, int dtype, r4c_stream_t stream) {
  if (argmax && (reinterpret_cast<uintptr_t>(argmax) & 1)) return R4C_ERR_INVALID;
  if (lead < 0 || lead % 8 || !buf || (reinterpret_cast<uintptr_t>(buf) & 15)) return R4C_ERR_INVALID;
  void* y = static_cast<uint8_t*>(buf) + (size_t)lead * 2;
  if (!pool_args(x, n, d, h, w, C, C, dtype) || !pool_args(y, n, d, h, w, C, lead + C, dtype) ||
      !pool_args(p, n, d, h, w, C, C, dtype) || !mean_invstd || !affine)
    return R4C_ERR_INVALID;
  return pool_fwd_launch(x, y, lead + C, lead, p, argmax, mean_invstd, affine, n, d, h, w, C, dtype, stream);
}

size_t r4c_bn_pool_workspace_size(int n, int d, int h, int w, int C) {
  if (C <= 0 || n < 0) return 0;
  const Split s = split_for((int64_t)n * (d / 2) * (h / 2) * (w / 2), 8);
  return r4c::align_up((size_t)s.S * 2 * C * sizeof(float), 256);
}

int r4c_bn_relu_pool_bwd_sums(const void* gy, int gy_pitch, const void* gp, const void* argmax, const void* x,
                              const float* mean_invstd, const float* affine, int n, int d, int h, int w, int C,
                              int dtype, float* sums, void* ws, size_t ws_bytes, r4c_stream_t stream) {
  if (argmax && (reinterpret_cast<uintptr_t>(argmax) & 1)) return R4C_ERR_INVALID;
  if (!pool_args(x, n, d, h, w, C, C, dtype) || !pool_args(gy, n, d, h, w, C, gy_pitch, dtype) ||
      !pool_args(gp, n, d, h, w, C, C, dtype) || !mean_invstd || !affine || !sums)
    return R4C_ERR_INVALID;
  const PoolGeo g = pool_geo(n, d, h, w, C, gy_pitch);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (g.pvox == 0) return cudaMemsetAsync(sums, 0, 2 * C * sizeof(float), s) == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
  const Split sp = split_for(g.pvox, 8);   // a pooled voxel is 8 voxels of work
  if (!ws || ws_bytes < r4c_bn_pool_workspace_size(n, d, h, w, C)) return R4C_ERR_WORKSPACE;
  float* part = static_cast<float*>(ws);
  const int R = std::max(1, 128 / (C / 4));
  const int threads = R * (C / 4);  // <= 512: C <= 2048
  const size_t smem = (size_t)R * 2 * C * sizeof(float);
  if (smem > 48 * 1024) return R4C_ERR_UNSUPPORTED;
  if (dtype == R4C_BF16)
    pool_sums_kernel<__nv_bfloat16><<<sp.S, threads, smem, s>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(gy),
        static_cast<const __nv_bfloat16*>(gp), mean_invstd, affine, g, sp.chunk,
        static_cast<const uint16_t*>(argmax), part);
  else
    pool_sums_kernel<__half><<<sp.S, threads, smem, s>>>(static_cast<const __half*>(x), static_cast<const __half*>(gy),
                                                         static_cast<const __half*>(gp), mean_invstd, affine, g,
                                                         sp.chunk, static_cast<const uint16_t*>(argmax), part);
  if (dtype == R4C_BF16)
    sum_parts_kernel<__nv_bfloat16><<<(2 * C + 7) / 8, 256, 0, s>>>(part, sp.S, C, sums, 0, nullptr, nullptr);
  else
    sum_parts_kernel<__half><<<(2 * C + 7) / 8, 256, 0, s>>>(part, sp.S, C, sums, 0, nullptr, nullptr);
  r4c::note_launches(2);
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

int r4c_bn_relu_pool_bwd_dx(const void* gy, int gy_pitch, const void* gp, const void* argmax, const void* x, void* dx,
                            const float* mean_invstd, const float* affine, const float* sums, double count, int n,
                            int d, int h, int w, int C, int dtype, float* dgamma, float* dbeta, float* coef,
                            r4c_stream_t stream) {
  if (argmax && (reinterpret_cast<uintptr_t>(argmax) & 1)) return R4C_ERR_INVALID;
  if (!pool_args(x, n, d, h, w, C, C, dtype) || !pool_args(gy, n, d, h, w, C, gy_pitch, dtype) ||
      !pool_args(gp, n, d, h, w, C, C, dtype) || !mean_invstd || !affine || !sums || !coef || count <= 0.0)
    return R4C_ERR_INVALID;
  if (dx && !pool_args(dx, n, d, h, w, C, C, dtype)) return R4C_ERR_INVALID;
  const PoolGeo g = pool_geo(n, d, h, w, C, gy_pitch);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  bwd_finalize_kernel<<<(C + 127) / 128, 128, 0, s>>>(sums, mean_invstd, affine, C, count, dgamma, dbeta, coef);
  r4c::note_launches(1);
  if (dx && g.pvox > 0) {
    const int64_t total = g.pvox * (C / 4);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 127) / 128, 148 * 8));
    if (dtype == R4C_BF16)
      pool_dx_kernel<__nv_bfloat16><<<grid, pool_threads(g.C), 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(gy),
          static_cast<const __nv_bfloat16*>(gp), static_cast<__nv_bfloat16*>(dx), mean_invstd, affine, coef, g,
          static_cast<const uint16_t*>(argmax));
    else
      pool_dx_kernel<__half><<<grid, pool_threads(g.C), 0, s>>>(static_cast<const __half*>(x), static_cast<const __half*>(gy),
                                                  static_cast<const __half*>(gp), static_cast<__half*>(dx), mean_invstd,
                                                  affine, coef, g, static_cast<const uint16_t*>(argmax));
    r4c::note_launches(1);
  }
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

}  // extern "C"
