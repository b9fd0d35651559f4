// r4c_internal.h — declarations shared by the library's translation units.
#pragma once

#include "r4c_common.cuh"

namespace r4c {

enum { MODE_CONV = 0, MODE_TFWD = 1, MODE_TDX = 2, MODE_TDW = 3 };

namespace generic {

// Forward-shaped implicit GEMM: out[M, N] = A[M, K] * B[K, N] (+ bias).
struct FwdParams {
  const void* a;      // activation source, NDHWC
  const void* b;      // packed weight, row-major [K][N]
  const void* bias;   // [N] (MODE_CONV) or [oc] (MODE_TFWD), may be null
  void* out;          // NDHWC
  int64_t M;
  int N, K;
  int sd, sh, sw, sc; // source tensor spatial dims and channels
  int md, mh, mw;     // grid the GEMM row index m walks (n is the outer index)
  int ks, pd, ph, pw; // conv kernel size and zero padding (MODE_CONV)
  int oc;             // channels of y (MODE_TFWD)
};

// Weight-gradient GEMM: partial[s][P][N] = sum over m in split s.
struct WgradParams {
  const void* x;
  const void* go;
  float* partial;
  int P, N;
  int64_t M;
  int chunk;
  int d, h, w, cin;   // x dims
  int md, mh, mw;     // reduction grid (go dims for conv, x dims for tconv)
  int cout;
  int ks, pd, ph, pw;
};

cudaError_t launch_fwd(const FwdParams& p, int mode, int dtype, cudaStream_t st);
void wgrad_split(int64_t M, int P, int N, int* S, int* chunk);
void db_split(int64_t V, int* S, int64_t* chunk);
cudaError_t launch_wgrad(const WgradParams& p, int mode, int dtype, int S, float* dw, int taps,
                         cudaStream_t st);
cudaError_t launch_db(const void* go, int64_t V, int C, int dtype, float* part, float* db,
                      cudaStream_t st);

}  // namespace generic

namespace tc {

// Host-side plan of the tcgen05 conv kernel (k in {1,3}; fwd, or dX run as a
// conv of dY with the flipped weight and padding k-1-p).
struct ConvPlan {
  bool ok;
  int n, d, h, w;        // source (input) dims of the conv actually run
  int od, oh, ow;        // its output dims
  int cin, cout;         // its channels (dX: cin = Cout of the layer)
  int ks, pd, ph, pw;
  int c8;                // 8-channel chunks of cin
  int npad;              // cout rounded up to the MMA N granule (16): one TMEM "slot"
  int P;                 // output planes per work unit (plane block)
  int nin;               // input planes per unit: P + ks - 1
  int fold;              // output-plane slots one MMA may cover (kd folded into N)
  int G, ngroups;        // chunks per pipeline stage, stages per kd plane
  int padg;              // 1: the last channel group is padded up to a swizzle width (TMA zero fill past Cin)
  int nsteps;            // 16-wide K steps per stage
  int wt, ht;            // output tile (cols, rows) of one plane
  int pitch_w, pitch_h;  // brick pitches: wt + ks - 1, ht + ks - 1
  int cpb;               // bytes of one chunk plane (128-aligned)
  int mtiles, nsets;     // 128-row M tiles per unit; TMEM accumulator sets
  int a_bytes, b_bytes, stage_bytes, stages, smem_bytes;
  int wres;              // 1: the whole packed weight stays resident in smem
  int wres_bytes;        // its size (ks * ngroups * b_bytes) when resident
  int warp_issue;        // 1: the whole MMA warp runs the issue loop (elect.sync); 0: lane 0 alone
  int tmem_cols;
  int stg_bytes;         // output staging buffer (one of two) for TMA stores; 0: per-thread stores
  int pps;               // input planes per pipeline stage (1, or 2 with resident weights)
  double est_cycles;     // planner's cost-model estimate for the whole launch
  int64_t work_units;    // n * ceil(od / P) * tiles_h * tiles_w
  int grid;
};

bool plan_conv(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw,
               ConvPlan* pl);
size_t packed_bytes(const ConvPlan& pl);
// Packs the PyTorch-layout weight into the K-step blocks of the plan; input
// channels at or above cin_real (channel padding) get zero weights.
cudaError_t pack_weight(const ConvPlan& pl, bool flip_for_dx, int cin_real, const void* w_src,
                        int src_dtype, void* w_packed, int dtype, cudaStream_t st);
int launch_conv(const ConvPlan& pl, const void* x, const void* w_packed, const void* bias,
                void* y, int dtype, cudaStream_t st);
// launch_conv with the plan found fastest on this device for this shape
// (timed on the first call, then cached); same packed weights as `pl`.
int launch_conv_tuned(const ConvPlan& pl, const void* x, const void* w_packed, const void* bias,
                      void* y, int dtype, cudaStream_t st);
// The plan launch_conv_tuned settled on for this shape, if it ran already.
bool tuned_plan(const ConvPlan& pl, int dtype, ConvPlan* out);

// Device address of the kernels' bounded-wait error flag (current device).
int* device_error_flag();

// tcgen05 weight gradient (r4c_tc_dw.cu). Geometry is the layer's: input
// dims, Cin, Cout, k and pads. db is produced in-kernel when *db_done is set.
bool dw_supported(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw);
size_t dw_workspace(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw);
int dw_describe(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw, char* buf,
                size_t len);
int launch_dw(int n, int d, int h, int w, int cin, int cin_real, int cout, int ks, int pd, int ph, int pw,
              const void* x, const void* go, float* dw, float* db, void* ws, size_t ws_bytes, int dtype,
              cudaStream_t st, bool* db_done);

}  // namespace tc

// tcgen05 forward conv for k=3 layers with 1..4 input channels (r4c_tc_stem.cu):
// raw input brick by TMA, im2col rows built in shared memory, K = 27*Cin.
namespace stem {
bool supported(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw);
size_t packed_bytes(int cin, int cout);
cudaError_t pack_weight(int cin, int cout, const void* w_src, int src_dtype, void* w_packed, int dtype,
                        cudaStream_t st);
int launch_fwd(int n, int d, int h, int w, int cin, int cout, int pd, int ph, int pw, const void* x,
               const void* w_packed, const void* bias, void* y, int dtype, cudaStream_t st);
int describe(int n, int d, int h, int w, int cin, int cout, int pd, int ph, int pw, char* buf, size_t len);
// Weight gradient (dW fp32 OIDHW, db fp32 when non-null) of the same layers,
// Cout a multiple of 8; `ws` holds one fp32 partial per CTA.
bool dw_supported(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw);
size_t dw_workspace(int n, int d, int h, int w, int cin, int cout, int pd, int ph, int pw);
int dw_describe(int n, int d, int h, int w, int cin, int cout, int pd, int ph, int pw, char* buf, size_t len);
int launch_dw(int n, int d, int h, int w, int cin, int cout, int pd, int ph, int pw, const void* x, const void* go,
              float* dw, float* db, void* ws, size_t ws_bytes, int dtype, cudaStream_t st);
// dX of k=3, pad 1 layers with one input channel and Cout a multiple of 4 up
// to 32 (W even, <= 256); dY and dX NDHWC, packed weight dx_packed_bytes().
bool dx_supported(int n, int d, int h, int w, int cin, int cout, int ks, int pd, int ph, int pw);
size_t dx_packed_bytes();
cudaError_t dx_pack_weight(int cout, const void* w_src, int src_dtype, void* w_packed, int dtype, cudaStream_t st);
int dx_describe(int n, int d, int h, int w, int cout, char* buf, size_t len);
int launch_dx(int n, int d, int h, int w, int cout, const void* go, const void* w_packed, void* dx, int dtype,
              cudaStream_t st);
}  // namespace stem

// ConvTranspose3d k=2 s=2 p=0 forward (mode 0) and dX (mode 1) on tcgen05;
// activations NDHWC, Cin and Cout multiples of 8. The packed weight is the
// per-task shared-memory image of packed_bytes().
namespace tconv {
bool supported(int mode, int n, int d, int h, int w, int cin, int cout);
size_t packed_bytes(int mode, int n, int d, int h, int w, int cin, int cout);
int describe(int mode, int n, int d, int h, int w, int cin, int cout, char* buf, size_t len);
cudaError_t pack_weight(int mode, int n, int d, int h, int w, int cin, int cout, const void* w_src, int src_dtype,
                        void* w_packed, int dtype, cudaStream_t st);
// ypitch (forward only): elements between consecutive output voxels, >= cout
// and a multiple of 8 (0: cout) — the output may be a channel slice of a
// wider NDHWC buffer.
int launch(int mode, int n, int d, int h, int w, int cin, int cout, const void* in, const void* w_packed,
           const void* bias, void* out, int dtype, cudaStream_t st, int ypitch = 0);
// dW (fp32, PyTorch ConvTranspose3d layout) from x and dY; `ws` holds the
// split partials (dw_workspace() bytes).
bool dw_supported(int n, int d, int h, int w, int cin, int cout);
size_t dw_workspace(int n, int d, int h, int w, int cin, int cout);
int dw_describe(int n, int d, int h, int w, int cin, int cout, char* buf, size_t len);
// db (nullable) is produced here when Cin <= 64 (*db_done set).
int launch_dw(int n, int d, int h, int w, int cin, int cout, const void* x, const void* go, float* dw, float* db,
              void* ws, size_t ws_bytes, int dtype, cudaStream_t st, bool* db_done);
}  // namespace tconv

}  // namespace r4c
