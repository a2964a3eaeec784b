// ctmr_conv3d_noalloc: the convolution of ctmr_conv3d for callers that cannot
// allocate device memory.
//
// Some hosts of this library may not call cudaMalloc at all: a plugin that
// runs inside another framework's memory pool or allocator-instrumented
// process, or a real-time or safety-constrained caller whose allocations are
// all made before it starts and that may not allocate afterwards. ctmr_conv3d needs a scratch
// buffer for the prepared operand (the group-norm / SiLU / pooled /
// upsampled / bf16- or split-fp16-cast input the tensor cores read), which such
// callers cannot provide. This entry point instead uses one file-scope
// `static __device__` array of CTMR_CONV3D_NOALLOC_SCRATCH_BYTES (32 MiB). Every GPU that
// loads the library holds that array until the process exits.
//
// Contract:
//   * The caller still passes every input and output (desc as for ctmr_conv3d).
//   * A convolution whose prepared operand needs more than the 32 MiB
//     is rejected with CTMR_ERR_WORKSPACE before anything is launched.
//   * The first call on a device looks up the array's device address with
//     cudaGetSymbolAddress while that device is current (once per device, then
//     cached). Make that first call before any stream capture. The cache
//     remembers the CUDA context the address belongs to (its process-unique
//     id): after cudaDeviceReset the next call on that device, in the new
//     context, looks the address up again instead of using the stale one.
//   * Every call on a device shares the same array, which keeps the last
//     call's contents. Nothing in it has to start at zero: the preparation pass
//     writes every byte the GEMM then reads. Calls whose kernels overlap on the
//     GPU (different streams without ordering between them) race on the array
//     and must not be issued.
//   * Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "ctmr_b200.h"

namespace ctmr {
int set_last_error(int status, const char* message);  // capi.cu
}  // namespace ctmr

namespace {

constexpr size_t kNoAllocScratchBytes = CTMR_CONV3D_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// The scratch the no-allocation entry point uses instead of a caller workspace.
// In host code this name is only a stand-in for the symbol, never a device
// address: the address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};  // id of the context each address belongs to

template <typename Fn>
Fn driver_entry(const char* name, int version) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPointByVersion(name, &p, version, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}

// Process-unique id of the current device's CUDA context (cuCtxGetId), 0 if unavailable.
unsigned long long current_context_id() {
  static const PFN_cuCtxGetCurrent_v4000 get_current = driver_entry<PFN_cuCtxGetCurrent_v4000>("cuCtxGetCurrent", 4000);
  static const PFN_cuCtxGetId_v12000 get_id = driver_entry<PFN_cuCtxGetId_v12000>("cuCtxGetId", 12000);
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of the scratch array on the current device: looked up once per device and
// context. Before the runtime's first call on a device there is no current context yet (id 0);
// cudaGetSymbolAddress creates it, and its id is read afterwards.
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return ctmr::set_last_error(CTMR_ERR_CUDA, "conv3d_noalloc: no usable current CUDA device");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  unsigned long long ctx = current_context_id();
  if (g_scratch_ptr[dev] == nullptr || ctx == 0 || ctx != g_scratch_ctx[dev]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return ctmr::set_last_error(CTMR_ERR_CUDA, "conv3d_noalloc: cudaGetSymbolAddress of the static scratch failed");
    g_scratch_ptr[dev] = ptr;
    g_scratch_ctx[dev] = ctx != 0 ? ctx : current_context_id();
  }
  *out = g_scratch_ptr[dev];
  return CTMR_OK;
}

}  // namespace

extern "C" {

int ctmr_conv3d_noalloc(const ctmr_conv3d_desc* desc, void* stream) {
  if (desc == nullptr) return ctmr::set_last_error(CTMR_ERR_INVALID, "conv3d_noalloc: null descriptor");
  // Size check first (host only): a rejected call launches nothing and touches no device state.
  const size_t need = ctmr_conv3d_workspace_size(desc);
  if (need > kNoAllocScratchBytes)
    return ctmr::set_last_error(CTMR_ERR_WORKSPACE,
                                "conv3d_noalloc: this convolution's prepared operand exceeds the 32 MiB static "
                                "scratch (CTMR_CONV3D_NOALLOC_SCRATCH_BYTES); call ctmr_conv3d with a workspace");
  void* scratch = nullptr;
  if (need > 0) {
    const int st = scratch_for_current_device(&scratch);
    if (st != CTMR_OK) return st;
  }
  return ctmr_conv3d(desc, scratch, need > 0 ? kNoAllocScratchBytes : 0, stream);
}

}  // extern "C"
