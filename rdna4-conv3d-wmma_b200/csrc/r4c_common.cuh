// r4c_common.cuh — shared device/host helpers of the B200 conv3d library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "r4c_conv3d.h"

namespace r4c {

// ---------------------------------------------------------------------------
// Element traits: 16-bit storage, fp32 arithmetic.
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};

// ---------------------------------------------------------------------------
// Geometry derived from a descriptor.
// ---------------------------------------------------------------------------
struct Geom {
  int n, d, h, w;      // input spatial
  int od, oh, ow;      // output spatial
  int cin, cout, k;
  int pd, ph, pw;
  int64_t in_vox() const { return (int64_t)n * d * h * w; }
  int64_t out_vox() const { return (int64_t)n * od * oh * ow; }
};

inline int out_size(int i, int k, int p) { return i + 2 * p - (k - 1); }

inline bool make_geom(const r4c_conv_desc* ds, Geom* g) {
  if (!ds) return false;
  g->n = ds->n; g->d = ds->d; g->h = ds->h; g->w = ds->w;
  g->cin = ds->cin; g->cout = ds->cout; g->k = ds->k;
  g->pd = ds->pad_d; g->ph = ds->pad_h; g->pw = ds->pad_w;
  if (g->k == 2) {
    g->od = 2 * g->d; g->oh = 2 * g->h; g->ow = 2 * g->w;
  } else {
    g->od = out_size(g->d, g->k, g->pd);
    g->oh = out_size(g->h, g->k, g->ph);
    g->ow = out_size(g->w, g->k, g->pw);
  }
  return true;
}

// Counts kernel launches made by the library (r4c_launch_count()).
void note_launches(int n);

inline size_t dtype_bytes(int dt) { return dt == R4C_F32 ? 4 : 2; }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline int cdiv(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

}  // namespace r4c
