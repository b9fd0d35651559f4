// r4c_ce.cu — cross-entropy over the channel dimension of NDHWC logits.
//
// The UNet training step ends in F.cross_entropy over (N, C, D, H, W) logits
// with integer labels (mean over voxels). On channels_last_3d bf16 logits the
// stock path casts them to fp32 (autocast), makes them dense NCDHW for its
// softmax and NLL kernels and runs four of those, forward and backward. Here
// the forward is one pass over the logits and labels (per-voxel log-sum-exp
// in fp32, deterministic block partials summed in a fixed order in double)
// and the backward one pass that writes d(loss)/d(logits) in the logits'
// own dtype and layout:
//   loss = (1/n) * sum_v [lse(z_v) - z_v[t_v]],  n = voxels whose label is not ignore_index
//   dz_v[c] = g * (softmax(z_v)[c] - [c == t_v]) / n   (0 for ignored voxels)
// with g the upstream gradient of the loss, read from device memory.
#include <algorithm>
#include <cmath>

#include "r4c_internal.h"

namespace r4c {
namespace ce {

constexpr int kThreads = 256;
constexpr int kMaxBlocks = 1184;  // 8 per SM; fixed per problem size (deterministic sums)

static int blocks_for(int64_t vox) {
  const int64_t b = (vox + kThreads * 8 - 1) / (kThreads * 8);
  return (int)std::max<int64_t>(1, std::min<int64_t>(b, kMaxBlocks));
}

// Label of voxel v, or -1 when it takes no part (ignore_index); labels
// outside [0, C) are treated as ignored and reported through the error flag.
__device__ __forceinline__ int label_of(const int64_t* tgt, int64_t v, int C, int64_t ignore, int* err) {
  const int64_t t = tgt[v];
  if (t == ignore) return -1;
  if (t < 0 || t >= C) {
    atomicExch(err, 6);
    return -1;
  }
  return (int)t;
}

// part[b] = (sum of per-voxel losses, number of counted voxels) over block
// b's contiguous voxel range; fixed thread order, tree in shared memory.
template <typename T>
__global__ void __launch_bounds__(kThreads) fwd_kernel(const T* __restrict__ z, const int64_t* __restrict__ tgt,
                                                       int64_t vox, int C, int64_t ignore, double* __restrict__ part,
                                                       int* err) {
  const int64_t per = (vox + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = (int64_t)blockIdx.x * per, v1 = min(vox, v0 + per);
  double s = 0.0, n = 0.0;
  for (int64_t v = v0 + threadIdx.x; v < v1; v += kThreads) {
    const int t = label_of(tgt, v, C, ignore, err);
    if (t < 0) continue;
    const T* zv = z + v * C;
    float m = -INFINITY;
    for (int c = 0; c < C; ++c) m = fmaxf(m, Elem<T>::to_f(zv[c]));
    float e = 0.f;
    for (int c = 0; c < C; ++c) e += expf(Elem<T>::to_f(zv[c]) - m);
    s += (double)(m + logf(e) - Elem<T>::to_f(zv[t]));
    n += 1.0;
  }
  __shared__ double sh[2][kThreads];
  sh[0][threadIdx.x] = s;
  sh[1][threadIdx.x] = n;
  __syncthreads();
  for (int off = kThreads / 2; off > 0; off >>= 1) {
    if ((int)threadIdx.x < off) {
      sh[0][threadIdx.x] += sh[0][threadIdx.x + off];
      sh[1][threadIdx.x] += sh[1][threadIdx.x + off];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    part[2 * blockIdx.x] = sh[0][0];
    part[2 * blockIdx.x + 1] = sh[1][0];
  }
}

// loss_count = (mean loss, count): one block, partials in block order.
__global__ void __launch_bounds__(kThreads) finalize_kernel(const double* __restrict__ part, int nblk,
                                                            float* __restrict__ loss_count) {
  __shared__ double sh[2][kThreads];
  double s = 0.0, n = 0.0;
  for (int b = threadIdx.x; b < nblk; b += kThreads) {
    s += part[2 * b];
    n += part[2 * b + 1];
  }
  sh[0][threadIdx.x] = s;
  sh[1][threadIdx.x] = n;
  __syncthreads();
  for (int off = kThreads / 2; off > 0; off >>= 1) {
    if ((int)threadIdx.x < off) {
      sh[0][threadIdx.x] += sh[0][threadIdx.x + off];
      sh[1][threadIdx.x] += sh[1][threadIdx.x + off];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const double cnt = sh[1][0];
    loss_count[0] = cnt > 0.0 ? (float)(sh[0][0] / cnt) : NAN;  // mean over no voxels: NaN, as PyTorch
    loss_count[1] = (float)cnt;
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) bwd_kernel(const T* __restrict__ z, const int64_t* __restrict__ tgt,
                                                       int64_t vox, int C, int64_t ignore,
                                                       const float* __restrict__ loss_count,
                                                       const float* __restrict__ grad, T* __restrict__ dz, int* err) {
  const float scale = grad[0] / loss_count[1];
  for (int64_t v = (int64_t)blockIdx.x * kThreads + threadIdx.x; v < vox; v += (int64_t)gridDim.x * kThreads) {
    const int t = label_of(tgt, v, C, ignore, err);
    const T* zv = z + v * C;
    T* dv = dz + v * C;
    if (t < 0) {
      for (int c = 0; c < C; ++c) dv[c] = Elem<T>::from_f(0.f);
      continue;
    }
    float m = -INFINITY;
    for (int c = 0; c < C; ++c) m = fmaxf(m, Elem<T>::to_f(zv[c]));
    float e = 0.f;
    for (int c = 0; c < C; ++c) e += expf(Elem<T>::to_f(zv[c]) - m);
    const float inv = 1.f / e;
    for (int c = 0; c < C; ++c) {
      const float p = expf(Elem<T>::to_f(zv[c]) - m) * inv;
      dv[c] = Elem<T>::from_f(scale * (p - (c == t ? 1.f : 0.f)));
    }
  }
}

}  // namespace ce
}  // namespace r4c

using namespace r4c;

extern "C" size_t r4c_ce_workspace_size(int64_t vox) {
  return vox < 0 ? 0 : (size_t)ce::blocks_for(vox) * 2 * sizeof(double);
}

extern "C" int r4c_ce_fwd(const void* logits, const int64_t* target, int64_t vox, int C, int dtype,
                          int64_t ignore_index, float* loss_count, void* ws, size_t ws_bytes, r4c_stream_t stream) {
  if (vox < 0 || C <= 0 || !loss_count || (vox > 0 && (!logits || !target))) return R4C_ERR_INVALID;
  if (dtype != R4C_BF16 && dtype != R4C_F16) return R4C_ERR_UNSUPPORTED;
  const int nblk = ce::blocks_for(vox);
  if (!ws || ws_bytes < r4c_ce_workspace_size(vox)) return R4C_ERR_WORKSPACE;
  int* err = tc::device_error_flag();
  if (!err) return R4C_ERR_CUDA;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  double* part = static_cast<double*>(ws);
  if (dtype == R4C_BF16)
    ce::fwd_kernel<__nv_bfloat16><<<nblk, ce::kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(logits), target,
                                                                vox, C, ignore_index, part, err);
  else
    ce::fwd_kernel<__half><<<nblk, ce::kThreads, 0, s>>>(static_cast<const __half*>(logits), target, vox, C,
                                                         ignore_index, part, err);
  ce::finalize_kernel<<<1, ce::kThreads, 0, s>>>(part, nblk, loss_count);
  note_launches(2);
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}

extern "C" int r4c_ce_bwd(const void* logits, const int64_t* target, int64_t vox, int C, int dtype,
                          int64_t ignore_index, const float* loss_count, const float* grad_loss, void* dlogits,
                          r4c_stream_t stream) {
  if (vox < 0 || C <= 0 || !loss_count || !grad_loss || (vox > 0 && (!logits || !target || !dlogits)))
    return R4C_ERR_INVALID;
  if (dtype != R4C_BF16 && dtype != R4C_F16) return R4C_ERR_UNSUPPORTED;
  if (vox == 0) return R4C_OK;
  int* err = tc::device_error_flag();
  if (!err) return R4C_ERR_CUDA;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int nblk = (int)std::min<int64_t>((vox + ce::kThreads - 1) / ce::kThreads, 148 * 16);
  if (dtype == R4C_BF16)
    ce::bwd_kernel<__nv_bfloat16><<<nblk, ce::kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(logits), target,
                                                                vox, C, ignore_index, loss_count, grad_loss,
                                                                static_cast<__nv_bfloat16*>(dlogits), err);
  else
    ce::bwd_kernel<__half><<<nblk, ce::kThreads, 0, s>>>(static_cast<const __half*>(logits), target, vox, C,
                                                         ignore_index, loss_count, grad_loss,
                                                         static_cast<__half*>(dlogits), err);
  note_launches(1);
  return cudaGetLastError() == cudaSuccess ? R4C_OK : R4C_ERR_CUDA;
}
