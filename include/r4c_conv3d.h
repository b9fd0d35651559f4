/*
 * r4c_conv3d.h — C ABI of the B200 (sm_100a) Conv3d / ConvTranspose3d hot path.
 *
 * This library replaces the device half of the rdna4_conv3d package: the Triton
 * launchers in src/rdna4_conv3d/conv3d_wmma.py and the optional HIP fprop
 * (src/rdna4_conv3d/conv3d_wmma_hip.hip:148-195). Each entry point below names
 * the reference function it stands in for.
 *
 * Conventions
 *   - Activations are NDHWC (channels_last_3d), bf16 or fp16, densely packed:
 *     element (n, d, h, w, c) lives at ((((n*D + d)*H + h)*W + w)*C + c).
 *   - Weights are handed over pre-packed by r4c_pack_weight(); the packed
 *     layout is private to the kernel that the descriptor selects, so a packed
 *     buffer must come from r4c_pack_weight() with the same descriptor and leg.
 *   - Weight and bias gradients are written in fp32, in PyTorch's own layout
 *     (OIDHW for Conv3d, (Cin, Cout, 2, 2, 2) for ConvTranspose3d).
 *   - Every buffer, including the workspace, is owned by the caller. Nothing is
 *     allocated inside the library and no state is kept between calls apart
 *     from a per-device cache of kernel attributes.
 *   - Work is enqueued on the given stream and ordered only by it; calls may
 *     come from any host thread. One exception: the first r4c_conv3d_fwd /
 *     r4c_conv3d_dx call for a new (shape, dtype, device) times a few plan
 *     candidates on the caller's buffers and synchronizes the stream once to
 *     read the timings (skipped while the stream is being captured, and with
 *     the environment variable R4C_AUTOTUNE=0, which takes the modelled plan).
 *     Results never depend on the plan chosen. Make one call per shape before
 *     timing or capturing if that synchronization matters.
 *   - Errors are returned as negative status codes; nothing is thrown across
 *     the ABI. r4c_strerror() turns a code into text.
 */
#ifndef R4C_CONV3D_H_
#define R4C_CONV3D_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st* r4c_stream_t;

/* Status codes. */
enum {
  R4C_OK = 0,
  R4C_ERR_INVALID = -1,      /* bad pointer, size or descriptor field            */
  R4C_ERR_UNSUPPORTED = -2,  /* geometry outside k in {1,3} / tconv k2s2 scope   */
  R4C_ERR_WORKSPACE = -3,    /* workspace smaller than r4c_workspace_size()      */
  R4C_ERR_CUDA = -4,         /* a CUDA runtime/driver call failed                */
  R4C_ERR_ALIGN = -5,        /* pointer not aligned as the kernel requires       */
  R4C_ERR_NO_DEVICE = -6,    /* no sm_100 device current                         */
  R4C_ERR_TOO_LARGE = -7     /* size above a fixed maximum of the entry point    */
};

/* Element types of activations / packed weights. */
enum { R4C_BF16 = 0, R4C_F16 = 1, R4C_F32 = 2 };

/* Legs, for r4c_pack_weight / r4c_workspace_size. */
enum {
  R4C_LEG_FWD = 0,   /* Conv3d forward                          */
  R4C_LEG_DX = 1,    /* Conv3d input gradient                   */
  R4C_LEG_DW = 2,    /* Conv3d weight (+bias) gradient          */
  R4C_LEG_TFWD = 3,  /* ConvTranspose3d k2s2 forward            */
  R4C_LEG_TDX = 4,   /* ConvTranspose3d k2s2 input gradient     */
  R4C_LEG_TDW = 5    /* ConvTranspose3d k2s2 weight gradient    */
};

/* Kernel families the dispatcher can pick (r4c_plan_kernel). */
enum {
  R4C_KERNEL_NONE = 0,
  R4C_KERNEL_GENERIC = 1,   /* SIMT implicit GEMM, any channel count         */
  R4C_KERNEL_TC = 2         /* tcgen05 + TMA implicit GEMM (sm_100a)          */
};

/*
 * Problem descriptor. For Conv3d (k = 1 or 3, stride 1, dilation 1, groups 1)
 * n/d/h/w are the INPUT sizes; the output is
 *   o = i + 2*pad - (k - 1)    per spatial axis.
 * For ConvTranspose3d (k = 2, stride 2, pad 0) n/d/h/w are the input sizes and
 * the output is 2x in every spatial axis; pad_* must be 0.
 */
typedef struct r4c_conv_desc {
  int32_t n, d, h, w;
  int32_t cin, cout;
  int32_t k;                 /* 1 or 3 (Conv3d), 2 (ConvTranspose3d) */
  int32_t pad_d, pad_h, pad_w;
  int32_t dtype;             /* R4C_BF16 or R4C_F16 */
  int32_t force_kernel;      /* 0 = automatic, else an R4C_KERNEL_* value */
} r4c_conv_desc;

/* Library / error text. */
const char* r4c_strerror(int status);
int r4c_version(void);

/*
 * Device-side error flag of the current device. Every wait inside a kernel is
 * bounded (about one second); a wait that runs out makes the kernel record a
 * non-zero code here and return early instead of hanging the GPU. The call
 * synchronizes `stream`, returns the flag (0 = none) and clears it when
 * `clear` is non-zero. No reference counterpart (the Triton kernels have no
 * device-side waits).
 */
int r4c_device_error(r4c_stream_t stream, int clear);

/*
 * Self-test of those bounded waits: launches one block that waits, through
 * the kernels' own bounded-wait routine, on a barrier nothing arrives at, for
 * `limit_ns` nanoseconds (at most 2 s). The wait runs out, the block records
 * code 3 in the device error flag and returns; read it with
 * r4c_device_error(). No reference counterpart.
 */
int r4c_watchdog_selftest(uint64_t limit_ns, r4c_stream_t stream);

/* Total number of CUDA kernels this library has launched in this process
 * (all devices, all threads). Lets a caller count the kernels behind a timed
 * region. No reference counterpart. */
uint64_t r4c_launch_count(void);

/* Which kernel family runs `leg` for `desc` (an R4C_KERNEL_* value, or a
 * negative status when the geometry is out of scope). Pure host logic. */
int r4c_plan_kernel(const r4c_conv_desc* desc, int leg);

/* Human-readable description of the kernel plan for `leg` (family, tiles,
 * stages, shared memory) written into buf (NUL-terminated, truncated to
 * len). Returns the same value as r4c_plan_kernel. Pure host logic. */
int r4c_describe_plan(const r4c_conv_desc* desc, int leg, char* buf, size_t len);

/* Bytes of the packed weight buffer for `leg` (FWD, DX, TFWD or TDX). */
size_t r4c_packed_weight_bytes(const r4c_conv_desc* desc, int leg);

/* Bytes of caller-owned workspace that `leg` needs (0 when none). */
size_t r4c_workspace_size(const r4c_conv_desc* desc, int leg);

/*
 * Pack a PyTorch-layout weight for one leg.
 *   Conv3d:          w_src is OIDHW (Cout, Cin, k, k, k).
 *   ConvTranspose3d: w_src is (Cin, Cout, 2, 2, 2).
 * src_dtype is R4C_F32, R4C_BF16 or R4C_F16; the packed buffer is desc->dtype.
 * Replaces _pack_weight / _tr_pack_w and the flip/transpose/repack that k3 dX
 * does per call (src/rdna4_conv3d/conv3d_wmma.py:1023-1026,1154-1162,1453-1459).
 */
int r4c_pack_weight(const r4c_conv_desc* desc, int leg, const void* w_src,
                    int src_dtype, void* w_packed, r4c_stream_t stream);

/*
 * Conv3d forward: y = conv3d(x, w) + bias.
 * x NDHWC [n,d,h,w,cin]; y NDHWC [n,od,oh,ow,cout]; bias (cout) in desc->dtype
 * or NULL. Replaces _launch_fwd (conv3d_wmma.py:1048-1105) and the HIP
 * fwd_k3 (conv3d_wmma_hip.hip:148-195).
 */
int r4c_conv3d_fwd(const r4c_conv_desc* desc, const void* x, const void* w_packed,
                   const void* bias, void* y, void* workspace, size_t ws_bytes,
                   r4c_stream_t stream);

/*
 * Conv3d input gradient: dx = conv3d_input(go, w).
 * go NDHWC [n,od,oh,ow,cout]; dx NDHWC [n,d,h,w,cin]; w_packed from
 * r4c_pack_weight(..., R4C_LEG_DX, ...). Replaces _launch_dgrad
 * (conv3d_wmma.py:1108-1179); the k3 case uses pad' = 2 - pad, so every pad in
 * {0,1,2} is exact (the reference reuses pad, correct only for pad 1).
 */
int r4c_conv3d_dx(const r4c_conv_desc* desc, const void* go, const void* w_packed,
                  void* dx, void* workspace, size_t ws_bytes, r4c_stream_t stream);

/*
 * Conv3d weight and bias gradient, fp32, deterministic.
 * x NDHWC, go NDHWC; dw OIDHW fp32 [cout,cin,k,k,k]; db fp32 [cout] or NULL.
 * Split-K partials over N*D*H*W go to the workspace and are summed in a fixed
 * order. Replaces _launch_wgrad + partial.sum(0) (conv3d_wmma.py:1182-1214)
 * and the separate db reduction (conv3d_wmma.py:1318).
 */
int r4c_conv3d_dw(const r4c_conv_desc* desc, const void* x, const void* go,
                  float* dw, float* db, void* workspace, size_t ws_bytes,
                  r4c_stream_t stream);

/*
 * ConvTranspose3d k2 s2 p0 forward. x NDHWC [n,d,h,w,cin]; y NDHWC
 * [n,2d,2h,2w,cout]; bias (cout) or NULL. Replaces transpose_k2s2_fwd
 * (conv3d_wmma.py:1462-1488).
 */
int r4c_tconv_fwd(const r4c_conv_desc* desc, const void* x, const void* w_packed,
                  const void* bias, void* y, void* workspace, size_t ws_bytes,
                  r4c_stream_t stream);

/* r4c_tconv_fwd into a channel slice of a wider NDHWC buffer: consecutive
 * output voxels are y_pitch elements apart (y_pitch >= Cout, a multiple of 8,
 * y 16-byte aligned), so the up-convolution of a UNet decoder writes its
 * output straight into the first channels of the skip concatenation
 * (torch.cat([up, skip], 1) of the reference's UNet, benches/unet_e2e.py:38)
 * instead of into a tensor that is then copied there. y_pitch == Cout is
 * r4c_tconv_fwd; other pitches need the tcgen05 path (R4C_ERR_UNSUPPORTED
 * otherwise). */
int r4c_tconv_fwd_pitched(const r4c_conv_desc* desc, const void* x, const void* w_packed,
                          const void* bias, void* y, int y_pitch, void* workspace, size_t ws_bytes,
                          r4c_stream_t stream);

/* ConvTranspose3d k2s2 input gradient. Replaces transpose_k2s2_dx
 * (conv3d_wmma.py:1491-1514). */
int r4c_tconv_dx(const r4c_conv_desc* desc, const void* go, const void* w_packed,
                 void* dx, void* workspace, size_t ws_bytes, r4c_stream_t stream);

/* ConvTranspose3d k2s2 weight/bias gradient, fp32 (Cin,Cout,2,2,2) and
 * (Cout). Replaces transpose_k2s2_dw (conv3d_wmma.py:1517-1542). */
int r4c_tconv_dw(const r4c_conv_desc* desc, const void* x, const void* go,
                 float* dw, float* db, void* workspace, size_t ws_bytes,
                 r4c_stream_t stream);

/*
 * Conv3d of any geometry: per-axis kernel size, stride, zero padding,
 * dilation and groups. The reference runs these geometries on the vendor
 * library (src/rdna4_conv3d/conv3d_wmma.py:1241-1242; its generic Triton
 * kernels, conv3d_wmma.py:246-541, hold the same index arithmetic).
 *   - k = 2, stride 2, pad 0, dilation 1, groups 1 with even input extents,
 *     bf16/fp16, channels multiples of 8 (the downsampling conv) runs on the
 *     tcgen05 ConvTranspose3d kernels with the roles swapped (its forward is
 *     the transpose conv's dX, its dX the transpose conv's forward);
 *   - everything else on SIMT implicit GEMMs with fp32 accumulation
 *     (bf16, fp16 or fp32 tensors).
 * n/d/h/w are the input sizes; output o = (i + 2p - dil*(k-1) - 1) / s + 1
 * per axis. Weights are in PyTorch's layout (Cout, Cin/groups, kd, kh, kw)
 * and desc->dtype, unpacked; bias (Cout) in desc->dtype or NULL; dW / db
 * fp32. Workspace: r4c_convex_workspace_size(desc, leg) bytes (leg =
 * R4C_LEG_FWD / R4C_LEG_DX / R4C_LEG_DW), caller-owned.
 */
typedef struct r4c_convex_desc {
  int32_t n, d, h, w;
  int32_t cin, cout, groups;
  int32_t kd, kh, kw;
  int32_t sd, sh, sw;        /* stride */
  int32_t pd, ph, pw;        /* zero padding */
  int32_t dd, dh, dw;        /* dilation */
  int32_t dtype;             /* R4C_BF16, R4C_F16 or R4C_F32 */
} r4c_convex_desc;

/* R4C_KERNEL_TC (k2s2 on the transpose-conv kernels), R4C_KERNEL_GENERIC, or
 * a negative status for an invalid descriptor. Pure host logic. */
int r4c_convex_plan(const r4c_convex_desc* desc);
size_t r4c_convex_workspace_size(const r4c_convex_desc* desc, int leg);
int r4c_convex_fwd(const r4c_convex_desc* desc, const void* x, const void* w, const void* bias, void* y,
                   void* workspace, size_t ws_bytes, r4c_stream_t stream);
int r4c_convex_dx(const r4c_convex_desc* desc, const void* go, const void* w, void* dx, void* workspace,
                  size_t ws_bytes, r4c_stream_t stream);
int r4c_convex_dw(const r4c_convex_desc* desc, const void* x, const void* go, float* dw, float* db,
                  void* workspace, size_t ws_bytes, r4c_stream_t stream);

/*
 * BatchNorm3d with batch statistics, fused with ReLU, on NDHWC activations
 * of `vox` voxels x C channels (bf16 / fp16, C a multiple of 8, 16-byte
 * aligned). No reference kernel: the reference's model blocks are Conv3d ->
 * BatchNorm3d -> ReLU on the vendor library (benches/unet_e2e.py:13-20).
 * Training forward:  r4c_bn_stats -> r4c_bn_finalize -> r4c_bn_relu_fwd.
 * Backward:          r4c_bn_relu_bwd_sums -> r4c_bn_relu_bwd_dx.
 * Every reduction is deterministic (fixed block ranges and orders). All
 * per-channel arrays are fp32; `ws` is r4c_bn_workspace_size(vox, C) bytes.
 * A caller that shards one volume across processes all-reduces `sums`
 * (element-wise sum) between the first and second call of each direction.
 */
size_t r4c_bn_workspace_size(int64_t vox, int C);
/* sums (3*C floats): [0:C) = sum (x - p), [C:2C) = sum (x - p)^2, [2C:3C) =
 * the pivot p used: `pivot` (C floats) when given, else the first voxel of x.
 * Deviations from a value inside the distribution keep the variance free of
 * the cancellation E[x^2] - E[x]^2 suffers when |mean| >> std. Shards of one
 * volume whose sums are all-reduced must pass the same pivot. */
int r4c_bn_stats(const void* x, int64_t vox, int C, int dtype, const float* pivot, float* sums, void* ws,
                 size_t ws_bytes, r4c_stream_t stream);
/* From sums over `count` voxels: mean_invstd = (mean, 1/sqrt(var + eps)),
 * affine = (gamma, beta), 1 and 0 where gamma / beta are NULL. Running
 * statistics (both or neither) get the momentum update with the unbiased
 * variance, as torch.nn.BatchNorm3d does. */
int r4c_bn_finalize(const float* sums, double count, int C, const float* gamma, const float* beta, float eps,
                    float momentum, float* running_mean, float* running_var, float* mean_invstd,
                    float* affine, r4c_stream_t stream);
/* y = relu(gamma * (x - mean) * invstd + beta) (no ReLU when relu == 0), the
 * expression and order of PyTorch's BatchNorm kernels; y may alias x. */
int r4c_bn_relu_fwd(const void* x, void* y, const float* mean_invstd, const float* affine, int64_t vox, int C,
                    int dtype, int relu, r4c_stream_t stream);
/* sums[0:C) = sum g, sums[C:2C) = sum g*(x - mean) with g = dy masked by the
 * forward's ReLU (recomputed from x with the forward's expression). */
int r4c_bn_relu_bwd_sums(const void* dy, const void* x, const float* mean_invstd, const float* affine,
                         int64_t vox, int C, int dtype, int relu, float* sums, void* ws, size_t ws_bytes,
                         r4c_stream_t stream);
/* dgamma, dbeta (nullable) and dx (nullable) from the backward sums over
 * `count` voxels; coef is 3*C floats of scratch. */
int r4c_bn_relu_bwd_dx(const void* dy, const void* x, void* dx, const float* mean_invstd, const float* affine,
                       const float* sums, double count, int64_t vox, int C, int dtype, int relu, float* dgamma,
                       float* dbeta, float* coef, r4c_stream_t stream);

/*
 * BatchNorm + ReLU + MaxPool3d(2) in one pass, NDHWC, even D/H/W (n/d/h/w are
 * the unpooled sizes). Forward writes y = relu(bn(x)) with a channel pitch
 * `y_pitch` >= C (y may be a channel slice of a wider NDHWC buffer, e.g. the
 * decoder's concatenation) and p = maxpool(y) dense. Backward routes dP to
 * each window's argmax, recomputed from x with PyTorch's max_pool3d rule
 * (scan in (d, h, w) order, first maximum, a NaN wins), adds dY (read with
 * pitch `gy_pitch`) and runs the fused BN backward: r4c_bn_relu_pool_bwd_sums
 * then r4c_bn_relu_pool_bwd_dx, workspace r4c_bn_pool_workspace_size().
 * Statistics come from r4c_bn_stats / r4c_bn_finalize over x as above.
 */
/*
 * Dense NDHWC copy of a channel slice: dst[v][0..C) = src[v * src_pitch +
 * 0..C) for vox voxels (src points at the slice's first channel). The
 * up-conv backward's dY is such a slice of the decoder concatenation's
 * gradient (torch.cat in the reference's UNet, benches/unet_e2e.py:38).
 * C and src_pitch multiples of 8, 16-bit dtypes, 16-byte aligned pointers.
 */
int r4c_channel_slice_copy(const void* src, int src_pitch, void* dst, int64_t vox, int C, int dtype,
                           r4c_stream_t stream);
int r4c_bn_relu_pool_fwd(const void* x, void* y, int y_pitch, void* p, const float* mean_invstd, const float* affine,
                         int n, int d, int h, int w, int C, int dtype, r4c_stream_t stream);
/* The same forward into a whole concatenation buffer buf (n, d, h, w,
 * lead + C): channels [lead, lead + C) get relu(bn(x)) and channels
 * [0, lead) zeros (the caller's up-conv output overwrites them), so that
 * every line of buf is written whole in one pass: writing only the slice
 * leaves partial sectors, which HBM3e merges by read-modify-write (2.3x the
 * time at the UNet's level 0). lead a multiple of 8. argmax (nullable):
 * n*(d/2)*(h/2)*(w/2)*(C/4) uint16, per (pooled voxel, 4-channel group) the
 * window position of each channel's maximum in 3-bit fields; the backward
 * entries take it instead of recomputing it from x. */
int r4c_bn_relu_pool_fwd_cat(const void* x, void* buf, int lead, void* p, void* argmax, const float* mean_invstd,
                             const float* affine, int n, int d, int h, int w, int C, int dtype, r4c_stream_t stream);
size_t r4c_bn_pool_workspace_size(int n, int d, int h, int w, int C);
/* argmax (nullable): as written by r4c_bn_relu_pool_fwd_cat for the same x
 * and statistics; null recomputes it from x. */
int r4c_bn_relu_pool_bwd_sums(const void* gy, int gy_pitch, const void* gp, const void* argmax, const void* x,
                              const float* mean_invstd,
                              const float* affine, int n, int d, int h, int w, int C, int dtype, float* sums, void* ws,
                              size_t ws_bytes, r4c_stream_t stream);
int r4c_bn_relu_pool_bwd_dx(const void* gy, int gy_pitch, const void* gp, const void* argmax, const void* x, void* dx,
                            const float* mean_invstd, const float* affine, const float* sums, double count, int n,
                            int d, int h, int w, int C, int dtype, float* dgamma, float* dbeta, float* coef,
                            r4c_stream_t stream);

/*
 * Cross-entropy over the channel dimension of NDHWC (channels-last) logits,
 * mean over the voxels whose label is not `ignore_index` — F.cross_entropy
 * with reduction='mean' and no class weights, the loss of the UNet training
 * step measured here (four classes). No reference kernel: the reference's
 * training step computes its loss with stock PyTorch (benches/unet_e2e.py:
 * 41-52). Logits bf16 or
 * fp16 (fp32 arithmetic), `vox` voxels x C classes, int64 labels.
 * r4c_ce_fwd writes loss_count[0] = mean loss, loss_count[1] = the number of
 * counted voxels (device memory, 2 floats); `ws` holds
 * r4c_ce_workspace_size(vox) bytes; the sum is deterministic (fixed blocks,
 * fixed order). r4c_ce_bwd writes dlogits = grad_loss[0] * (softmax - onehot)
 * / count (zero for ignored voxels) in the logits' dtype and layout,
 * grad_loss a device scalar. A label outside [0, C) that is not ignore_index
 * is skipped and sets code 6 in the device error flag.
 */
size_t r4c_ce_workspace_size(int64_t vox);
int r4c_ce_fwd(const void* logits, const int64_t* target, int64_t vox, int C, int dtype, int64_t ignore_index,
               float* loss_count, void* ws, size_t ws_bytes, r4c_stream_t stream);
int r4c_ce_bwd(const void* logits, const int64_t* target, int64_t vox, int C, int dtype, int64_t ignore_index,
               const float* loss_count, const float* grad_loss, void* dlogits, r4c_stream_t stream);

/*
 * Conv3d weight and bias gradient without any allocation. No counterpart in
 * the reference: it exists for callers that cannot allocate device memory,
 * e.g. a plugin or custom op running inside another framework that owns the
 * whole device memory pool (its guests may not call cudaMalloc, which would
 * bypass the pool and can synchronize the device), or code on a latency path
 * that must make no allocation call at all.
 *
 * Same inputs, outputs and results as r4c_conv3d_dw(), but the split-K
 * scratch lives in a fixed device array inside this library
 * (R4C_NOALLOC_SCRATCH_BYTES, present on every GPU that loads the library
 * until the process exits) instead of a caller workspace. Descriptors whose
 * r4c_workspace_size(desc, R4C_LEG_DW) exceeds that size are rejected with
 * R4C_ERR_TOO_LARGE. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current; make that first
 * call before any stream capture. The address is kept per device and looked
 * up again when the device's current context has changed (after a
 * cudaDeviceReset the library's module is loaded anew and the array may
 * move); the first call after such a change should likewise come before any
 * stream capture. All calls share the one array: calls whose
 * work overlaps on the GPU (different streams, or different host threads)
 * race on it and must be serialized by the caller. The kernels write every
 * scratch element they read, so stale contents from a previous call are
 * never used.
 */
#define R4C_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)
int r4c_conv3d_dw_noalloc(const r4c_conv_desc* desc, const void* x, const void* go,
                          float* dw, float* db, r4c_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* R4C_CONV3D_H_ */
