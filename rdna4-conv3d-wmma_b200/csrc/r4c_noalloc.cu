// r4c_noalloc.cu — the allocation-free weight-gradient entry point.
//
// For callers that cannot allocate device memory (a guest inside another
// framework's memory pool, or a path that must not call cudaMalloc): the
// split-K scratch of r4c_conv3d_dw() comes from a fixed array in this
// library instead of a caller workspace. Everything else is the regular dW
// path, unchanged.
#include <cuda.h>

#include <mutex>

#include "r4c_internal.h"

namespace {

// Fixed scratch, one copy per device context that loads the library.
static __device__ __align__(256) unsigned char g_r4c_noalloc_scratch[R4C_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
struct ScratchAddr {
  void* ctx;  // the context the address belongs to
  void* ptr;
};
ScratchAddr g_scratch[kMaxDevices] = {};
std::mutex g_scratch_mu;

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// The current context, through the driver entry point (the library links only
// the runtime); null when it cannot be queried.
void* current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  CUcontext c = nullptr;
  if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

// Device address of the scratch array for the current device. In host code
// the symbol itself is only a host-side stand-in, so the address must come
// from cudaGetSymbolAddress, with the device current. It is looked up once
// per device and again whenever the device's context has changed (after a
// cudaDeviceReset the module is loaded anew and the array may move).
int scratch_for_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return R4C_ERR_NO_DEVICE;
  if (dev >= kMaxDevices) return R4C_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  void* ctx = current_context();
  ScratchAddr& c = g_scratch[dev];
  if (c.ptr == nullptr || ctx == nullptr || c.ctx != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_r4c_noalloc_scratch) != cudaSuccess || p == nullptr) return R4C_ERR_CUDA;
    c.ptr = p;
    c.ctx = current_context();  // queried after the lookup, which makes the primary context current if needed
  }
  *out = c.ptr;
  return R4C_OK;
}

}  // namespace

extern "C" int r4c_conv3d_dw_noalloc(const r4c_conv_desc* desc, const void* x, const void* go, float* dw,
                                     float* db, r4c_stream_t stream) {
  const int plan = r4c_plan_kernel(desc, R4C_LEG_DW);
  if (plan < 0) return plan;
  const size_t need = r4c_workspace_size(desc, R4C_LEG_DW);
  if (need > R4C_NOALLOC_SCRATCH_BYTES) return R4C_ERR_TOO_LARGE;
  void* scratch = nullptr;
  const int st = scratch_for_current_device(&scratch);
  if (st != R4C_OK) return st;
  return r4c_conv3d_dw(desc, x, go, dw, db, need ? scratch : nullptr, need, stream);
}
