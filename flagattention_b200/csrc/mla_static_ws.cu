// mla_static_ws.cu -- MLA decode without any device allocation by the caller.
//
// fa_mla_decode needs a split workspace (partial outputs and log-sum-exps of
// sequences that several SM parts share).  Some callers cannot provide one:
// serving engines that reserve nearly all device memory for their KV-cache
// pool at start-up (a later cudaMalloc fails, and also synchronises the
// device in the middle of a decode step), and plugin or FFI hosts whose
// interface hands the plugin device pointers but no allocator.  For them,
// fa_mla_decode_static_workspace runs the same decode and combine kernels
// with the workspace taken from a fixed array in device memory that this
// library defines at file scope.
//
// Properties of that array (kMaxBytes = FA_MLA_STATIC_WORKSPACE_BYTES):
//   * every GPU that loads the library holds it until the process exits;
//   * all calls on a device share it and it keeps the last call's contents,
//     so two calls whose kernels overlap on the GPU (different streams
//     without ordering) race -- serialise them on one stream;
//   * nothing in it has to start at zero: every partial the combine reads is
//     written by the same call's decode kernel first.
// The first call in a CUDA context (per device, and again after
// cudaDeviceReset) looks up the array's device address (cudaGetSymbolAddress
// with that device current); make that first call before capturing work into
// a stream.  No cudaMalloc / cudaFree or
// allocating library routine is ever called here.
#include <mutex>

#include <cstdio>

#include "common.cuh"
#include "flagattn_b200.h"

namespace fa {
int record_error(int status, const char *msg);
}  // namespace fa

namespace {

constexpr size_t kMaxBytes = FA_MLA_STATIC_WORKSPACE_BYTES;
constexpr int kMaxContexts = 256;

// The workspace itself.  In host code this name is only a stand-in for the
// symbol, never a device address: it is resolved per device below.
static __device__ __align__(256) unsigned char g_mla_workspace[kMaxBytes];

// Resolved addresses, keyed by the CUDA context they were looked up in (its
// process-unique id): a context created after cudaDeviceReset loads the
// module again, possibly at another address, and gets its own entry.
struct Resolved {
  unsigned long long ctx_id;
  void *addr;
};
std::mutex g_lock;
Resolved g_addr[kMaxContexts] = {};
int g_count = 0;

size_t round_up_256(size_t x) { return (x + 255) / 256 * 256; }

// Driver entry points looked up through the runtime, so the library does
// not link against libcuda (it loads where no driver is installed, e.g. for
// the host-only functions).
using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);
template <typename Fn>
Fn driver_fn(const char *name) {
  void *ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return reinterpret_cast<Fn>(ptr);
}

}  // namespace

extern "C" int fa_mla_decode_static_workspace(const fa_mla_args *args, void *stream) {
  if (!args) return fa::record_error(FA_ERR_INVALID_ARGUMENT, "null args");
  size_t po = 0, pl = 0;
  int st = fa_mla_workspace_size(args->batch, args->s_q, args->h_q, args->d_v,
                                 args->num_sm_parts, &po, &pl);
  if (st != FA_OK) return st;
  const size_t need = round_up_256(po) + pl;
  if (need > kMaxBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "static workspace too small: this call needs %zu bytes of split scratch "
             "((batch + num_sm_parts) * s_q * h_q * (d_v + 1) * 4), the fixed array holds %zu; "
             "use fewer sm parts or a smaller batch, or fa_mla_decode with your own workspace",
             need, kMaxBytes);
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, msg);
  }

  // The context the kernels will run in: the calling thread's current one
  // (a runtime call makes the current device's primary context current when
  // the thread has none yet).
  static const CtxGetCurrentFn ctx_get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static const CtxGetIdFn ctx_get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  if (!ctx_get_current || !ctx_get_id)
    return fa::record_error(FA_ERR_NO_DEVICE, "CUDA driver entry points unavailable");
  CUcontext ctx = nullptr;
  if (ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
    void *probe = nullptr;
    if (cudaGetSymbolAddress(&probe, g_mla_workspace) != cudaSuccess) {
      cudaGetLastError();
      return fa::record_error(FA_ERR_NO_DEVICE, "no usable CUDA device");
    }
    if (ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr)
      return fa::record_error(FA_ERR_NO_DEVICE, "no current CUDA context");
  }
  unsigned long long ctx_id = 0;
  if (ctx_get_id(ctx, &ctx_id) != CUDA_SUCCESS)
    return fa::record_error(FA_ERR_CUDA, "cuCtxGetId failed");
  void *base = nullptr;
  {
    std::lock_guard<std::mutex> guard(g_lock);
    for (int i = 0; i < g_count; ++i)
      if (g_addr[i].ctx_id == ctx_id) base = g_addr[i].addr;
    if (base == nullptr) {
      void *p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_mla_workspace);
      if (e != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        return fa::record_error(FA_ERR_CUDA, "cudaGetSymbolAddress of the static workspace failed");
      }
      if (g_count == kMaxContexts)
        return fa::record_error(FA_ERR_CUDA, "static workspace: too many CUDA contexts");
      g_addr[g_count++] = Resolved{ctx_id, p};
      base = p;
    }
  }
  fa_mla_args a = *args;
  a.part_o = static_cast<float *>(base);
  a.part_lse = reinterpret_cast<float *>(static_cast<unsigned char *>(base) + round_up_256(po));
  return fa_mla_decode(&a, stream);
}
