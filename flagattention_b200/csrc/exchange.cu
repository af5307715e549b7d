// exchange.cu -- KV-page-sharded decode across GPUs without a collective
// library call on the data path.
//
// Every rank decodes its range of the sequences' KV pages; its partial result
// (per query row: O normalised by its own row sum, f32, and the LSE) must
// reach every rank, which then merges the ranks' partials by log-sum-exp (the
// algebra of split_kv.py:198-228; the reference itself is single-GPU).
// Instead of a separate all-gather, the kernel that produces a rank's partial
// rows writes each finished row straight into the gather buffer of every
// rank (peer stores over NVLink through CUDA IPC mappings) and then adds the
// number of rows it delivered to a per-source counter on every rank.  The
// merge kernel on each rank waits -- with a time limit -- until every source's
// counter shows its rows, and merges from its local gather buffer.
//
// Gather buffer of a rank (f32): part r of rank r at parts + r * part_stride,
// part_stride = rows * (d_v + 1): O rows [rows][d_v] in (batch, token, head)
// order, then the rows' LSEs [rows].  Counters: uint64 [world], counter r =
// rows of rank r delivered so far.  Counters only grow: after the k-th
// exchange every counter holds k * rows, so nothing is reset between calls.
// No multicast object or multicast load is used: plain peer stores and local
// loads only.
#include <algorithm>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "flagattn_b200.h"
#include "merge.cuh"

namespace fa {

struct PeerTargets {
  float *parts[FA_EXCHANGE_MAX_RANKS];
  unsigned long long *counters[FA_EXCHANGE_MAX_RANKS];
};

__device__ __forceinline__ void red_release_sys_add(unsigned long long *p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long load_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Rows a task covers: four (narrow form, one warp per row) or two (wide form,
// four warps per row, see mla_row_state).
template <bool kWide>
constexpr int rows_per_task() {
  return kWide ? 2 : 4;
}

// One task of the combine-and-push step: rows task_x * rows_per_task .. of
// sequence b of the rank's decode.  A sequence split over several parts is
// merged from the split workspace; a sequence decoded by one part is read
// from the decode's f32 output.  Each row goes to slot `rank` of every
// rank's gather buffer.  Returns the rows covered (0 .. rows_per_task).
// Every thread of the block calls it (the wide form synchronises the block).
template <bool kWide>
__device__ __forceinline__ int push_rows(const float *__restrict__ part_o,
                                         const float *__restrict__ part_lse,
                                         const int32_t *__restrict__ num_splits,
                                         const float *__restrict__ out, int64_t o_sb, int64_t o_ss,
                                         int64_t o_sh, const float *__restrict__ lse_in, int batch,
                                         int s_q, int h_q, int d_v, const PeerTargets &peers,
                                         int world, int rank, int task_x, int b,
                                         MergeState (*states)[32]) {
  const int first = num_splits[b];
  const int n = num_splits[b + 1] - first;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = s_q * h_q;
  const int64_t rows_all = static_cast<int64_t>(batch) * rows;
  const int64_t part_stride = rows_all * (d_v + 1);
  const int flat = task_x * rows_per_task<kWide>() + (kWide ? (warp >> 2) : warp);
  const int j = kWide ? (warp & 3) : 0;
  float4 v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  float l = -INFINITY;
  if (n >= 2) {
    MergeState st;
    mla_row_state<kWide>(st, part_o, part_lse, first, n, rows, flat, d_v, lane, j, warp, states);
    l = (st.z > 0.f) ? st.m + __logf(st.z) : -INFINITY;
    const float inv = (st.z > 0.f) ? 1.f / st.z : 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      v[k] = make_float4(st.acc[k].x * inv, st.acc[k].y * inv, st.acc[k].z * inv,
                         st.acc[k].w * inv);
  } else if (flat < rows && j == 0) {
    const int s = flat / h_q, h = flat % h_q;
    const float *src = out + b * o_sb + s * o_ss + h * o_sh;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int d = lane * 4 + k * 128;
      v[k] = d < d_v ? __ldcg(reinterpret_cast<const float4 *>(src + d))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    l = __ldcg(lse_in + (static_cast<int64_t>(b) * h_q + h) * s_q + s);
  }
  if (flat < rows && j == 0) {
    const int64_t grow = static_cast<int64_t>(b) * rows + flat;
#pragma unroll
    for (int r = 0; r < FA_EXCHANGE_MAX_RANKS; ++r) {  // unrolled: the pointers stay in registers
      if (r >= world) break;
      float *dst = peers.parts[r] + rank * part_stride;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int d = lane * 4 + k * 128;
        if (d < d_v) *reinterpret_cast<float4 *>(dst + grow * d_v + d) = v[k];
      }
      if (lane == 0) dst[rows_all * d_v + grow] = l;
    }
  }
  return max(0, min(rows_per_task<kWide>(), rows - task_x * rows_per_task<kWide>()));
}

// Thread 0 of the block: count `done` rows of this rank on every receiver,
// with a release add at system scope (the caller's barrier orders the
// block's peer stores before it; release makes them visible to whoever
// acquires the counter).
__device__ __forceinline__ void count_rows(const PeerTargets &peers, int world, int rank,
                                           unsigned long long done) {
  if (done == 0) return;
#pragma unroll
  for (int r = 0; r < FA_EXCHANGE_MAX_RANKS; ++r)
    if (r < world) red_release_sys_add(peers.counters[r] + rank, done);
}

// Thread 0 of the block: wait until every rank's counter holds `target` rows,
// at most timeout_ns of the global timer (a block that finds the exchange
// timeout already recorded does not wait again).
__device__ __forceinline__ bool wait_rows(const unsigned long long *counters, int world,
                                          unsigned long long target, int *status,
                                          long long timeout_ns) {
  if (status != nullptr && *reinterpret_cast<volatile int *>(status) == kDevTimeoutExchange)
    return false;
  const uint64_t t0 = global_ns();
  for (int r = 0; r < world; ++r) {
    while (load_acquire_sys(counters + r) < target) {
      if (static_cast<long long>(global_ns() - t0) > timeout_ns) {
        if (status) atomicExch(status, kDevTimeoutExchange);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// The calling warp merges the `world` parts of row `row` of the local gather
// buffer into out / lse.
template <typename T>
__device__ __forceinline__ void merge_gathered_row(const float *__restrict__ parts, int world,
                                                   int64_t rows_all, int d_v, int64_t row,
                                                   T *__restrict__ out, float *__restrict__ lse,
                                                   int lane) {
  const int64_t part_stride = rows_all * (d_v + 1);
  MergeState st;
  st.init();
  fold_parts<true, 4>(st, parts, parts + rows_all * d_v, 0, 0, 1, world, part_stride, part_stride,
                      row * d_v, row, d_v, lane);
  const float l = finish_row<T>(st, d_v, out + row * d_v, lane);
  if (lane == 0) lse[row] = l;
}

struct PushArgs {
  const float *part_o, *part_lse;
  const int32_t *num_splits;
  const float *out;
  int64_t o_sb, o_ss, o_sh;
  const float *lse_in;
  int batch, s_q, h_q, d_v;
};

// Combine and push (grid: row tasks x sequences).  Launched as a
// programmatic dependent of the decode kernel.
template <bool kWide>
__global__ void __launch_bounds__(kWide ? 256 : 128, kWide ? 2 : 4)
    mla_combine_push_kernel(const PushArgs a, PeerTargets peers, int world, int rank) {
  __shared__ MergeState states[kWide ? 8 : 1][32];
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the decode's outputs are complete
  const int done = push_rows<kWide>(a.part_o, a.part_lse, a.num_splits, a.out, a.o_sb, a.o_ss,
                                    a.o_sh, a.lse_in, a.batch, a.s_q, a.h_q, a.d_v, peers, world,
                                    rank, blockIdx.x, blockIdx.y, states);
  __syncthreads();
  if (threadIdx.x == 0) count_rows(peers, world, rank, done);
}

// Wait for every rank's rows, then merge (four rows per block).  On a
// timeout the block writes nothing and the status word says so.
template <typename T>
__global__ void __launch_bounds__(128, 4)
    lse_merge_wait_kernel(const float *__restrict__ parts, int world, int64_t rows_all, int d_v,
                          const unsigned long long *__restrict__ counters,
                          unsigned long long target, T *__restrict__ out, float *__restrict__ lse,
                          int *status, long long timeout_ns) {
  __shared__ int arrived;
  if (threadIdx.x == 0) arrived = wait_rows(counters, world, target, status, timeout_ns);
  __syncthreads();
  if (!arrived) return;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  if (row < rows_all)
    merge_gathered_row<T>(parts, world, rows_all, d_v, row, out, lse, threadIdx.x & 31);
}

// Both steps in one cooperative (all blocks resident) persistent grid of
// 256-thread blocks (the wide form: four warps per row): every block first
// combines and pushes its share of row tasks and counts its rows on every
// rank, and only then waits for all ranks' rows and merges its share of the
// gathered rows.  No block waits before its own pushes are done and all
// blocks run at once, so every rank's rows arrive unless a rank fails (then
// the bounded wait ends with the status set and nothing merged).
template <typename T>
__global__ void __launch_bounds__(256, 2)
    mla_exchange_kernel(const PushArgs a, PeerTargets peers, int world, int rank,
                        const float *__restrict__ parts, const unsigned long long *counters,
                        unsigned long long target, T *__restrict__ out, float *__restrict__ lse,
                        int *status, long long timeout_ns) {
  __shared__ MergeState states[8][32];
  __shared__ int arrived;
  const int rows = a.s_q * a.h_q;
  const int tasks_x = (rows + rows_per_task<true>() - 1) / rows_per_task<true>();
  const int tasks = tasks_x * a.batch;
  unsigned long long done = 0;
  for (int t = blockIdx.x; t < tasks; t += gridDim.x) {
    done += push_rows<true>(a.part_o, a.part_lse, a.num_splits, a.out, a.o_sb, a.o_ss, a.o_sh,
                            a.lse_in, a.batch, a.s_q, a.h_q, a.d_v, peers, world, rank,
                            t % tasks_x, t / tasks_x, states);
    // the folding warps have read every warp's state before the next task's
    // states overwrite `states`
    __syncthreads();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    count_rows(peers, world, rank, done);
    arrived = wait_rows(counters, world, target, status, timeout_ns);
  }
  __syncthreads();
  if (!arrived) return;
  const int64_t rows_all = static_cast<int64_t>(a.batch) * rows;
  const int warp = threadIdx.x >> 5;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp; row < rows_all;
       row += static_cast<int64_t>(gridDim.x) * 8)
    merge_gathered_row<T>(parts, world, rows_all, a.d_v, row, out, lse, threadIdx.x & 31);
}

int record_error(int status, const char *msg);

namespace {

using MemGetAddressRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

MemGetAddressRangeFn address_range_fn() {
  static MemGetAddressRangeFn fn = [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return static_cast<MemGetAddressRangeFn>(nullptr);
    }
    return reinterpret_cast<MemGetAddressRangeFn>(ptr);
  }();
  return fn;
}

}  // namespace
}  // namespace fa

extern "C" {

int fa_ipc_export(const void *ptr, void *handle, uint64_t *offset) {
  if (!ptr || !handle || !offset) return fa::record_error(FA_ERR_INVALID_ARGUMENT, "ipc export: null");
  auto range = fa::address_range_fn();
  if (!range) return fa::record_error(FA_ERR_CUDA, "ipc export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "ipc export: not a device allocation");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fa::record_error(FA_ERR_CUDA,
                            "ipc export: cudaIpcGetMemHandle failed (memory from cudaMalloc is "
                            "needed; a virtual-memory-managed pool cannot be exported this way)");
  }
  static_assert(sizeof(h) == FA_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
  return FA_OK;
}

int fa_ipc_open(const void *handle, void **base) {
  if (!handle || !base) return fa::record_error(FA_ERR_INVALID_ARGUMENT, "ipc open: null");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fa::record_error(FA_ERR_CUDA, "ipc open: cudaIpcOpenMemHandle failed");
  }
  return FA_OK;
}

int fa_ipc_close(void *base) {
  if (!base) return fa::record_error(FA_ERR_INVALID_ARGUMENT, "ipc close: null");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fa::record_error(FA_ERR_CUDA, "ipc close: cudaIpcCloseMemHandle failed");
  }
  return FA_OK;
}

namespace {

// Shared argument checks of the exchange entry points; fills the push
// arguments and the peer targets.
int exchange_setup(const fa_mla_args *a, float *const *dst_parts,
                   unsigned long long *const *dst_counters, int world, int rank,
                   fa::PushArgs *pa, fa::PeerTargets *t) {
  if (!a || !dst_parts || !dst_counters)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "exchange: null argument");
  if (world < 1 || world > FA_EXCHANGE_MAX_RANKS || rank < 0 || rank >= world)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "exchange: world / rank");
  if (a->out_dtype != FA_DTYPE_F32 || !a->out || !a->lse || !a->part_o || !a->part_lse ||
      !a->num_splits || a->d_v != 512 || a->batch < 0 || a->s_q <= 0 || a->h_q <= 0)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT,
                            "exchange: needs the decode's f32 output, LSE and workspace");
  if ((reinterpret_cast<uintptr_t>(a->out) & 15u) ||
      ((a->o_stride_b | a->o_stride_s | a->o_stride_h) & 3))
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "exchange: output rows not 16-byte aligned");
  *t = fa::PeerTargets{};
  for (int r = 0; r < world; ++r) {
    if (!dst_parts[r] || !dst_counters[r] || (reinterpret_cast<uintptr_t>(dst_parts[r]) & 15u))
      return fa::record_error(FA_ERR_INVALID_ARGUMENT,
                              "exchange: every rank's gather buffer (16-byte aligned) and "
                              "counters are needed");
    t->parts[r] = dst_parts[r];
    t->counters[r] = dst_counters[r];
  }
  *pa = fa::PushArgs{a->part_o, a->part_lse, a->num_splits, static_cast<const float *>(a->out),
                     a->o_stride_b, a->o_stride_s, a->o_stride_h,
                     static_cast<const float *>(a->lse), a->batch, a->s_q, a->h_q, a->d_v};
  return FA_OK;
}

int cuda_error(cudaError_t e, const char *what) {
  cudaGetLastError();
  char msg[200];
  snprintf(msg, sizeof(msg), "%s: %s", what, cudaGetErrorString(e));
  return fa::record_error(FA_ERR_CUDA, msg);
}

}  // namespace

int fa_mla_combine_push(const fa_mla_args *a, float *const *dst_parts,
                        unsigned long long *const *dst_counters, int world, int rank,
                        void *stream) {
  fa::PushArgs pa;
  fa::PeerTargets t;
  int st = exchange_setup(a, dst_parts, dst_counters, world, rank, &pa, &t);
  if (st != FA_OK || a->batch == 0) return st;
  const int rows = a->s_q * a->h_q;
  // few sequences over many parts: a row's partials spread over four warps
  const bool wide = static_cast<int64_t>(a->batch) * 4 <= a->num_sm_parts;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = wide ? dim3((rows + 1) / 2, a->batch) : dim3((rows + 3) / 4, a->batch);
  cfg.blockDim = dim3(wide ? 256 : 128);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto kern = wide ? fa::mla_combine_push_kernel<true> : fa::mla_combine_push_kernel<false>;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, pa, t, world, rank);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? FA_OK : cuda_error(e, "combine push launch");
}

int fa_lse_merge_wait(const float *parts, int world, int64_t rows, int d_v,
                      const unsigned long long *counters, unsigned long long target, void *out,
                      int dtype, float *lse, int32_t *status, int64_t timeout_ns, void *stream) {
  if (!parts || !counters || !out || !lse || world < 1 || world > FA_EXCHANGE_MAX_RANKS ||
      rows < 0 || d_v != 512 || timeout_ns <= 0)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "merge wait: bad arguments");
  if (reinterpret_cast<uintptr_t>(parts) & 15u)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "merge wait: parts must be 16-byte aligned");
  if (dtype != FA_DTYPE_BF16 && dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_F32)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "merge wait: dtype");
  if (rows == 0) return FA_OK;
  const dim3 grid(static_cast<unsigned>((rows + 3) / 4));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == FA_DTYPE_BF16)
    fa::lse_merge_wait_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(
        parts, world, rows, d_v, counters, target, static_cast<__nv_bfloat16 *>(out), lse, status,
        timeout_ns);
  else if (dtype == FA_DTYPE_F16)
    fa::lse_merge_wait_kernel<__half><<<grid, 128, 0, s>>>(
        parts, world, rows, d_v, counters, target, static_cast<__half *>(out), lse, status,
        timeout_ns);
  else
    fa::lse_merge_wait_kernel<float><<<grid, 128, 0, s>>>(
        parts, world, rows, d_v, counters, target, static_cast<float *>(out), lse, status,
        timeout_ns);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FA_OK : cuda_error(e, "merge wait launch");
}

int fa_mla_combine_exchange(const fa_mla_args *a, float *const *dst_parts,
                            unsigned long long *const *dst_counters, int world, int rank,
                            unsigned long long target, void *out, int dtype, float *lse,
                            int32_t *status, int64_t timeout_ns, void *stream) {
  fa::PushArgs pa;
  fa::PeerTargets t;
  int st = exchange_setup(a, dst_parts, dst_counters, world, rank, &pa, &t);
  if (st != FA_OK) return st;
  if (!out || !lse || timeout_ns <= 0 ||
      (dtype != FA_DTYPE_BF16 && dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_F32))
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "exchange: out / lse / dtype / timeout");
  if (a->batch == 0) return FA_OK;
  const int tasks = (a->s_q * a->h_q + 1) / 2 * a->batch;
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  void *kern = dtype == FA_DTYPE_BF16   ? reinterpret_cast<void *>(fa::mla_exchange_kernel<__nv_bfloat16>)
               : dtype == FA_DTYPE_F16 ? reinterpret_cast<void *>(fa::mla_exchange_kernel<__half>)
                                       : reinterpret_cast<void *>(fa::mla_exchange_kernel<float>);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0);
  if (e != cudaSuccess) return cuda_error(e, "exchange occupancy query");
  const int grid = std::max(1, std::min(tasks, sms * per_sm));
  const float *parts = dst_parts[rank];
  const unsigned long long *counters = dst_counters[rank];
  long long tns = timeout_ns;
  void *params[] = {&pa, &t, &world, &rank, &parts, &counters, &target, &out, &lse, &status, &tns};
  e = cudaLaunchCooperativeKernel(kern, dim3(grid), dim3(256), params, 0,
                                  static_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? FA_OK : cuda_error(e, "exchange launch");
}

}  // extern "C"
