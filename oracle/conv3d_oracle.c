/*
 * conv3d_oracle.c — CPU restatement of the reference's implicit-GEMM Conv3d
 * algorithm, for tests only.
 *
 * TEST INFRASTRUCTURE: this file is the parity checker. Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it. The
 * product path (rdna4_conv3d + libr4c_conv3d.so) never calls it.
 *
 * Every function restates one piece of src/rdna4_conv3d/conv3d_wmma.py
 * (path:line cited per function) in fp32 with fp32 accumulation, on NDHWC
 * activations and the reference's packed weight layouts:
 *   conv weight  Wp[(tap*Cin + ci) * Cout + co], tap = (kd*K + kh)*K + kw
 *   tconv weight Wt[ci * 8*Cout + tap*Cout + co], tap = kd*4 + kh*2 + kw
 * Pinned against golden vectors produced by the reference's own Triton
 * kernels (tests/golden/make_golden.py).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define IDX5(n, d, h, w, c, D, H, W, C) \
  ((((((int64_t)(n) * (D) + (d)) * (H) + (h)) * (W) + (w)) * (C)) + (c))

static int out_size(int i, int k, int p) { return i + 2 * p - (k - 1); }

/* _pack_weight (conv3d_wmma.py:1023-1026): OIDHW -> (K^3*Cin, Cout). */
void oracle_pack_weight(const float* w, int cout, int cin, int k, float* packed) {
  const int T = k * k * k;
  for (int co = 0; co < cout; ++co)
    for (int ci = 0; ci < cin; ++ci)
      for (int t = 0; t < T; ++t)
        packed[((int64_t)t * cin + ci) * cout + co] = w[((int64_t)co * cin + ci) * T + t];
}

/* _unpack_weight (conv3d_wmma.py:1029-1030): (K^3*Cin, Cout) -> OIDHW. */
void oracle_unpack_weight(const float* packed, int cout, int cin, int k, float* w) {
  const int T = k * k * k;
  for (int co = 0; co < cout; ++co)
    for (int ci = 0; ci < cin; ++ci)
      for (int t = 0; t < T; ++t)
        w[((int64_t)co * cin + ci) * T + t] = packed[((int64_t)t * cin + ci) * cout + co];
}

/*
 * Forward implicit GEMM, stride 1 / dilation 1 (_fwd_kernel / _fwd_k3_kernel,
 * conv3d_wmma.py:246-325, 371-444): Y[m, co] = sum_{tap, ci} X[shift(m,tap), ci]
 * * Wp[tap*Cin+ci, co] (+ bias), zero outside the input (the masked load).
 */
void oracle_conv_fwd(const float* x, int n, int d, int h, int w, int cin, const float* packed, int cout,
                     int k, int pd, int ph, int pw, const float* bias, float* y) {
  const int od = out_size(d, k, pd), oh = out_size(h, k, ph), ow = out_size(w, k, pw);
  float* acc = (float*)malloc(sizeof(float) * (size_t)cout);
  for (int b = 0; b < n; ++b)
    for (int z = 0; z < od; ++z)
      for (int yy = 0; yy < oh; ++yy)
        for (int xx = 0; xx < ow; ++xx) {
          for (int co = 0; co < cout; ++co) acc[co] = 0.f;
          for (int kd = 0; kd < k; ++kd)
            for (int kh = 0; kh < k; ++kh)
              for (int kw = 0; kw < k; ++kw) {
                const int iz = z + kd - pd, iy = yy + kh - ph, ix = xx + kw - pw;
                if (iz < 0 || iz >= d || iy < 0 || iy >= h || ix < 0 || ix >= w) continue;
                const int tap = (kd * k + kh) * k + kw;
                const float* xr = x + IDX5(b, iz, iy, ix, 0, d, h, w, cin);
                for (int ci = 0; ci < cin; ++ci) {
                  const float xv = xr[ci];
                  const float* wr = packed + ((int64_t)tap * cin + ci) * cout;
                  for (int co = 0; co < cout; ++co) acc[co] += xv * wr[co];
                }
              }
          float* yr = y + IDX5(b, z, yy, xx, 0, od, oh, ow, cout);
          for (int co = 0; co < cout; ++co) yr[co] = acc[co] + (bias ? bias[co] : 0.f);
        }
  free(acc);
}

/*
 * Input gradient by output-side gather (_dgrad_kernel, conv3d_wmma.py:446-541):
 * dX[m, ci] = sum_{tap, co} dY[m + pad - k_off(tap), co] * Wp[tap*Cin+ci, co],
 * over the taps whose output position lies inside dY. Correct for every pad.
 */
void oracle_conv_dgrad(const float* go, int n, int d, int h, int w, int cin, const float* packed, int cout,
                       int k, int pd, int ph, int pw, float* dx) {
  const int od = out_size(d, k, pd), oh = out_size(h, k, ph), ow = out_size(w, k, pw);
  for (int b = 0; b < n; ++b)
    for (int z = 0; z < d; ++z)
      for (int yy = 0; yy < h; ++yy)
        for (int xx = 0; xx < w; ++xx) {
          float* dr = dx + IDX5(b, z, yy, xx, 0, d, h, w, cin);
          for (int ci = 0; ci < cin; ++ci) dr[ci] = 0.f;
          for (int kd = 0; kd < k; ++kd)
            for (int kh = 0; kh < k; ++kh)
              for (int kw = 0; kw < k; ++kw) {
                const int oz = z + pd - kd, oy = yy + ph - kh, ox = xx + pw - kw;
                if (oz < 0 || oz >= od || oy < 0 || oy >= oh || ox < 0 || ox >= ow) continue;
                const int tap = (kd * k + kh) * k + kw;
                const float* gr = go + IDX5(b, oz, oy, ox, 0, od, oh, ow, cout);
                for (int ci = 0; ci < cin; ++ci) {
                  const float* wr = packed + ((int64_t)tap * cin + ci) * cout;
                  float s = 0.f;
                  for (int co = 0; co < cout; ++co) s += gr[co] * wr[co];
                  dr[ci] += s;
                }
              }
        }
}

/*
 * Weight gradient with split-K (_wgrad_kernel + _launch_wgrad,
 * conv3d_wmma.py:543-634, 1182-1214): K = N*OD*OH*OW output voxels split
 * into `split` chunks of cdiv(K, split); each chunk accumulates a private
 * fp32 partial dWp[tap*Cin+ci, co]; the partials are then summed in split
 * order (partial.sum(0)). Writes the packed (K^3*Cin, Cout) layout.
 */
void oracle_conv_wgrad(const float* x, const float* go, int n, int d, int h, int w, int cin, int cout, int k,
                       int pd, int ph, int pw, int split, float* dwp) {
  const int od = out_size(d, k, pd), oh = out_size(h, k, ph), ow = out_size(w, k, pw);
  const int T = k * k * k;
  const int64_t K = (int64_t)n * od * oh * ow;
  const int64_t P = (int64_t)T * cin * cout;
  if (split < 1) split = 1;
  const int64_t chunk = (K + split - 1) / split;
  float* part = (float*)calloc((size_t)P, sizeof(float));
  memset(dwp, 0, sizeof(float) * (size_t)P);
  for (int s = 0; s < split; ++s) {
    memset(part, 0, sizeof(float) * (size_t)P);
    const int64_t kb = (int64_t)s * chunk;
    const int64_t ke = kb + chunk < K ? kb + chunk : K;
    for (int64_t m = kb; m < ke; ++m) {
      int64_t t = m;
      const int xx = (int)(t % ow); t /= ow;
      const int yy = (int)(t % oh); t /= oh;
      const int z = (int)(t % od);
      const int b = (int)(t / od);
      const float* gr = go + m * cout;
      for (int kd = 0; kd < k; ++kd)
        for (int kh = 0; kh < k; ++kh)
          for (int kw = 0; kw < k; ++kw) {
            const int iz = z + kd - pd, iy = yy + kh - ph, ix = xx + kw - pw;
            if (iz < 0 || iz >= d || iy < 0 || iy >= h || ix < 0 || ix >= w) continue;
            const int tap = (kd * k + kh) * k + kw;
            const float* xr = x + IDX5(b, iz, iy, ix, 0, d, h, w, cin);
            for (int ci = 0; ci < cin; ++ci) {
              float* pr = part + ((int64_t)tap * cin + ci) * cout;
              const float xv = xr[ci];
              for (int co = 0; co < cout; ++co) pr[co] += xv * gr[co];
            }
          }
    }
    for (int64_t i = 0; i < P; ++i) dwp[i] += part[i];
  }
  free(part);
}

/* db = dY.sum(dim=(0,2,3,4)) (conv3d_wmma.py:1318), fp32, voxel order. */
void oracle_bias_grad(const float* go, int64_t vox, int cout, float* db) {
  for (int co = 0; co < cout; ++co) db[co] = 0.f;
  for (int64_t v = 0; v < vox; ++v)
    for (int co = 0; co < cout; ++co) db[co] += go[v * cout + co];
}

/* _tr_pack_w (conv3d_wmma.py:1453-1455): (Cin, Cout, 2,2,2) -> (Cin, 8*Cout). */
void oracle_tr_pack_w(const float* w, int cin, int cout, float* packed) {
  for (int ci = 0; ci < cin; ++ci)
    for (int co = 0; co < cout; ++co)
      for (int t = 0; t < 8; ++t)
        packed[(int64_t)ci * 8 * cout + t * cout + co] = w[((int64_t)ci * cout + co) * 8 + t];
}

/* _tr_unpack_w (conv3d_wmma.py:1458-1459). */
void oracle_tr_unpack_w(const float* packed, int cin, int cout, float* w) {
  for (int ci = 0; ci < cin; ++ci)
    for (int co = 0; co < cout; ++co)
      for (int t = 0; t < 8; ++t)
        w[((int64_t)ci * cout + co) * 8 + t] = packed[(int64_t)ci * 8 * cout + t * cout + co];
}

/*
 * ConvTranspose3d k2s2 forward (_tr_k2s2_fwd_kernel, conv3d_wmma.py:792-860):
 * Y8[m, tap*Cout+co] = X[m, :] . Wt[:, tap*Cout+co] (+ bias[co]) stored at
 * output (2*id+kd, 2*ih+kh, 2*iw+kw).
 */
void oracle_tconv_fwd(const float* x, int n, int d, int h, int w, int cin, const float* packed, int cout,
                      const float* bias, float* y) {
  const int N8 = 8 * cout;
  float* acc = (float*)malloc(sizeof(float) * (size_t)N8);
  for (int b = 0; b < n; ++b)
    for (int z = 0; z < d; ++z)
      for (int yy = 0; yy < h; ++yy)
        for (int xx = 0; xx < w; ++xx) {
          const float* xr = x + IDX5(b, z, yy, xx, 0, d, h, w, cin);
          for (int j = 0; j < N8; ++j) acc[j] = 0.f;
          for (int ci = 0; ci < cin; ++ci) {
            const float* wr = packed + (int64_t)ci * N8;
            for (int j = 0; j < N8; ++j) acc[j] += xr[ci] * wr[j];
          }
          for (int t = 0; t < 8; ++t) {
            const int kd = t >> 2, kh = (t >> 1) & 1, kw = t & 1;
            float* yr = y + IDX5(b, 2 * z + kd, 2 * yy + kh, 2 * xx + kw, 0, 2 * d, 2 * h, 2 * w, cout);
            for (int co = 0; co < cout; ++co) yr[co] = acc[t * cout + co] + (bias ? bias[co] : 0.f);
          }
        }
  free(acc);
}

/* ConvTranspose3d k2s2 dX (_tr_k2s2_dx_kernel, conv3d_wmma.py:862-931):
 * dX[m, ci] = sum_{tap, co} dY[2m+tap, co] * Wt[ci, tap*Cout+co]. */
void oracle_tconv_dx(const float* go, int n, int d, int h, int w, int cin, const float* packed, int cout,
                     float* dx) {
  for (int b = 0; b < n; ++b)
    for (int z = 0; z < d; ++z)
      for (int yy = 0; yy < h; ++yy)
        for (int xx = 0; xx < w; ++xx) {
          float* dr = dx + IDX5(b, z, yy, xx, 0, d, h, w, cin);
          for (int ci = 0; ci < cin; ++ci) {
            float s = 0.f;
            for (int t = 0; t < 8; ++t) {
              const int kd = t >> 2, kh = (t >> 1) & 1, kw = t & 1;
              const float* gr = go + IDX5(b, 2 * z + kd, 2 * yy + kh, 2 * xx + kw, 0, 2 * d, 2 * h, 2 * w, cout);
              const float* wr = packed + (int64_t)ci * 8 * cout + t * cout;
              for (int co = 0; co < cout; ++co) s += gr[co] * wr[co];
            }
            dr[ci] = s;
          }
        }
}

/* ConvTranspose3d k2s2 dW with split-K over input voxels
 * (_tr_k2s2_dw_kernel + transpose_k2s2_dw, conv3d_wmma.py:933-1012,
 * 1517-1542): packed dWt[ci, tap*Cout+co], partials summed in split order. */
void oracle_tconv_dw(const float* x, const float* go, int n, int d, int h, int w, int cin, int cout, int split,
                     float* dwp) {
  const int64_t K = (int64_t)n * d * h * w;
  const int64_t P = (int64_t)cin * 8 * cout;
  if (split < 1) split = 1;
  const int64_t chunk = (K + split - 1) / split;
  float* part = (float*)calloc((size_t)P, sizeof(float));
  memset(dwp, 0, sizeof(float) * (size_t)P);
  for (int s = 0; s < split; ++s) {
    memset(part, 0, sizeof(float) * (size_t)P);
    const int64_t kb = (int64_t)s * chunk;
    const int64_t ke = kb + chunk < K ? kb + chunk : K;
    for (int64_t m = kb; m < ke; ++m) {
      int64_t t = m;
      const int xx = (int)(t % w); t /= w;
      const int yy = (int)(t % h); t /= h;
      const int z = (int)(t % d);
      const int b = (int)(t / d);
      const float* xr = x + m * cin;
      for (int tp = 0; tp < 8; ++tp) {
        const int kd = tp >> 2, kh = (tp >> 1) & 1, kw = tp & 1;
        const float* gr = go + IDX5(b, 2 * z + kd, 2 * yy + kh, 2 * xx + kw, 0, 2 * d, 2 * h, 2 * w, cout);
        for (int ci = 0; ci < cin; ++ci) {
          float* pr = part + (int64_t)ci * 8 * cout + tp * cout;
          for (int co = 0; co < cout; ++co) pr[co] += xr[ci] * gr[co];
        }
      }
    }
    for (int64_t i = 0; i < P; ++i) dwp[i] += part[i];
  }
  free(part);
}
