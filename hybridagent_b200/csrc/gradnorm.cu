// Multi-tensor sum of squared gradients for the global norm (sm_100a).
//
// Replaces the per-tensor `grad.float().square().sum()` loop of
// hybrid_rl/optimizer.py:149-151 (three eager kernels and ~18 bytes of traffic per
// element) with one read of each gradient (2 bytes per bf16 element).
//
// Accuracy and determinism: squares of bf16/fp16 values are exact in fp32; each thread
// sums one 16-byte vector's squares pairwise in fp32, widens that to fp64 and
// accumulates in fp64; warps and the CTA combine in fixed trees; every chunk writes its
// own fp64 partial and one CTA adds the partials in a fixed order.  The result therefore
// depends only on the data and HA_SUMSQ_CHUNK, not on scheduling, and is far closer to
// the exact sum than the reference's fp32 accumulation.  NaN and Inf propagate, so a
// non-finite gradient anywhere makes the sum non-finite (the caller's skip decision).
#include <cuda.h>

#include <mutex>

#include "ha_common.cuh"

namespace ha {
namespace {

constexpr int64_t kChunk = HA_SUMSQ_CHUNK;

template <int DT>
struct Vec;  // elements per 16-byte load
template <>
struct Vec<HA_F32> {
  static constexpr int n = 4;
};
template <>
struct Vec<HA_BF16> {
  static constexpr int n = 8;
};
template <>
struct Vec<HA_F16> {
  static constexpr int n = 8;
};

template <int DT>
__device__ __forceinline__ float sq(float x) {
  return __fmul_rn(x, x);  // exact for 16-bit inputs; fp32 inputs round like torch's square()
}

// Pairwise fp32 sum of the squares of one 16-byte vector.
template <int DT>
__device__ __forceinline__ float vec_sumsq(uint4 w) {
  if constexpr (DT == HA_F32) {
    const float a = sq<DT>(__uint_as_float(w.x)), b = sq<DT>(__uint_as_float(w.y));
    const float c = sq<DT>(__uint_as_float(w.z)), d = sq<DT>(__uint_as_float(w.w));
    return __fadd_rn(__fadd_rn(a, b), __fadd_rn(c, d));
  } else {
    float q[8];
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q[2 * i] = sq<DT>(Elem<DT>::widen(uint16_t(words[i] & 0xffffu)));
      q[2 * i + 1] = sq<DT>(Elem<DT>::widen(uint16_t(words[i] >> 16)));
    }
    return __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[1]), __fadd_rn(q[2], q[3])),
                     __fadd_rn(__fadd_rn(q[4], q[5]), __fadd_rn(q[6], q[7])));
  }
}

__device__ __forceinline__ double block_sum(double x, double* smem) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem[warp] = x;
  __syncthreads();
  const int nwarps = blockDim.x >> 5;
  if (warp == 0) {
    x = lane < nwarps ? smem[lane] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  }
  return x;  // valid in thread 0
}

// One CTA per chunk, or fewer CTAs each taking chunks blockIdx.x, blockIdx.x + gridDim.x, ...
// (a capped grid leaves SMs to kernels running beside it).  Either way every chunk writes its
// own partial, computed the same way, so the result does not depend on the grid.
template <int DT>
__global__ void __launch_bounds__(kThreads) sumsq_kernel(const ha_tensor* __restrict__ tensors,
                                                         const ha_chunk* __restrict__ chunks, int64_t n_chunks,
                                                         double* __restrict__ partials) {
  __shared__ StagedChunk sc;
  __shared__ double red[kThreads / 32];
  for (int64_t ci = blockIdx.x; ci < n_chunks; ci += gridDim.x) {
    if (threadIdx.x < 4) {
      const ha_chunk c = chunks[ci];
      reinterpret_cast<uint4*>(&sc.t)[threadIdx.x] = reinterpret_cast<const uint4*>(tensors + c.tensor)[threadIdx.x];
      if (threadIdx.x == 0) sc.index = c.index;
    }
    __syncthreads();
    double acc = 0.0;
    if (sc.t.grad != 0) {
      constexpr int V = Vec<DT>::n;
      using raw = typename Elem<DT>::raw;
      const raw* grad = reinterpret_cast<const raw*>(sc.t.grad);
      const int64_t begin = int64_t(sc.index) * kChunk;
      const int64_t end = min(begin + kChunk, sc.t.numel);
      if ((sc.t.grad & 15) == 0) {
        constexpr int kPerPass = kThreads * V;       // elements per CTA pass
        constexpr int kUnroll = 4;                   // loads in flight per thread
        int64_t e = begin + int64_t(threadIdx.x) * V;
        for (; e + int64_t(kUnroll - 1) * kPerPass + V <= end; e += int64_t(kUnroll) * kPerPass) {
          uint4 w[kUnroll];
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) w[u] = __ldcs(reinterpret_cast<const uint4*>(grad + e + u * kPerPass));
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) acc += double(vec_sumsq<DT>(w[u]));
        }
        for (; e + V <= end; e += kPerPass) acc += double(vec_sumsq<DT>(__ldcs(reinterpret_cast<const uint4*>(grad + e))));
        if (e < end) {  // ragged tail of the tensor: at most V-1 elements, one thread
          float s = 0.0f;
          for (int64_t k = e; k < end; ++k) s = __fadd_rn(s, sq<DT>(Elem<DT>::widen(grad[k])));
          acc += double(s);
        }
      } else {
        for (int64_t k = begin + threadIdx.x; k < end; k += kThreads) acc += double(sq<DT>(Elem<DT>::widen(grad[k])));
      }
    }
    acc = block_sum(acc, red);
    if (threadIdx.x == 0) partials[ci] = acc;
    __syncthreads();  // sc and red are rewritten for the next chunk
  }
}

// One CTA adds the per-chunk partials: thread i takes partials i, i+1024, ... in order
// (four interleaved accumulators), then a fixed tree.
constexpr int kFinalThreads = 1024;
__global__ void __launch_bounds__(kFinalThreads) finalize_kernel(const double* __restrict__ partials, int64_t n,
                                                                  double* __restrict__ out) {
  __shared__ double red[kFinalThreads / 32];
  double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
  int64_t i = threadIdx.x;
  for (; i + 3 * kFinalThreads < n; i += 4 * kFinalThreads) {
    a0 += partials[i];
    a1 += partials[i + kFinalThreads];
    a2 += partials[i + 2 * kFinalThreads];
    a3 += partials[i + 3 * kFinalThreads];
  }
  for (; i < n; i += kFinalThreads) a0 += partials[i];
  double x = block_sum((a0 + a1) + (a2 + a3), red);
  if (threadIdx.x == 0) out[0] = x;
}

}  // namespace
}  // namespace ha

extern "C" int ha_grad_sumsq(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks,
                             int64_t chunk_elems, int grad_dtype, double* d_partials, double* d_out, void* stream) {
  return ha_grad_sumsq_ctas(d_tensors, d_chunks, n_chunks, chunk_elems, grad_dtype, d_partials, d_out, 0, stream);
}

extern "C" int ha_grad_sumsq_ctas(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks,
                                  int64_t chunk_elems, int grad_dtype, double* d_partials, double* d_out,
                                  int max_ctas, void* stream) {
  HA_NVTX_RANGE();
  using namespace ha;
  if (chunk_elems != HA_SUMSQ_CHUNK) return fail(HA_ERR_INVALID, "ha_grad_sumsq: chunk_elems must be %d", HA_SUMSQ_CHUNK);
  if (max_ctas < 0) return fail(HA_ERR_INVALID, "ha_grad_sumsq_ctas: max_ctas %d", max_ctas);
  if (!valid_float_dtype(grad_dtype)) return fail(HA_ERR_UNSUPPORTED, "ha_grad_sumsq: grad dtype %d", grad_dtype);
  if (n_chunks < 0 || n_chunks > 0x7fffffffLL) return fail(HA_ERR_INVALID, "ha_grad_sumsq: n_chunks %lld", (long long)n_chunks);
  if (d_out == nullptr) return fail(HA_ERR_INVALID, "ha_grad_sumsq: NULL output");
  if (n_chunks > 0 && (d_tensors == nullptr || d_chunks == nullptr || d_partials == nullptr))
    return fail(HA_ERR_INVALID, "ha_grad_sumsq: NULL table or partials");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_chunks > 0) {
    const dim3 grid(static_cast<unsigned>(max_ctas > 0 && max_ctas < n_chunks ? max_ctas : n_chunks));
    switch (grad_dtype) {
      case HA_F32: sumsq_kernel<HA_F32><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, n_chunks, d_partials); break;
      case HA_BF16: sumsq_kernel<HA_BF16><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, n_chunks, d_partials); break;
      default: sumsq_kernel<HA_F16><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, n_chunks, d_partials); break;
    }
    const int rc = check_launch("sumsq_kernel");
    if (rc != HA_OK) return rc;
  }
  finalize_kernel<<<1, kFinalThreads, 0, st>>>(d_partials, n_chunks, d_out);
  return check_launch("sumsq_finalize_kernel");
}

// ---------------------------------------------------------------------------------------
// Allocation-free variant of ha_grad_sumsq.
//
// Some callers cannot hand us a scratch buffer: an engine that has already reserved
// nearly all of HBM for its own pools (a cudaMalloc of a few MB then fails or forces its
// allocator to release cached blocks), a latency-critical loop that must not make the
// implicitly synchronizing cudaMalloc / cudaFree calls, or a host binding with no device
// allocator of its own.  For them the per-chunk fp64 partials live in the fixed array
// below, reserved once in every GPU that loads this library and held until the process
// exits: HA_NOALLOC_SUMSQ_MAX_CHUNKS doubles (2 MiB), enough for 8.59e9 elements per call.
//
// The host-side name of a __device__ array is not a device address, so the address is
// looked up with cudaGetSymbolAddress the first time the entry point runs on each device
// (with that device current) and cached together with the unique ID of the CUDA context it
// belongs to.  A later call on a different context of that device (the primary context was
// reset with cudaDeviceReset and re-created) looks the address up again, so the cached
// pointer never outlives its context.  Every call shares the one array: two calls
// whose kernels overlap on the GPU (different streams, or different host threads) race on
// it.  Each call writes every partial before reading it, so stale contents left by an
// earlier call never reach a result and nothing needs clearing first.
static __device__ __align__(256) double ha_noalloc_sumsq_partials[HA_NOALLOC_SUMSQ_MAX_CHUNKS];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
double* g_noalloc_ptr[kMaxDevices] = {};
unsigned long long g_noalloc_ctx[kMaxDevices] = {};

// Unique ID of the calling thread's current CUDA context (cuCtxGetCurrent + cuCtxGetId,
// reached through the runtime's driver entry points), or 0 where the driver cannot say.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(f);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of the partials array on the current device: looked up once per device
// and context (cudaGetSymbolAddress with the device current), then reused.
int noalloc_partials(double** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return ha::fail(HA_ERR_CUDA, "ha_grad_sumsq_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return ha::fail(HA_ERR_UNSUPPORTED, "ha_grad_sumsq_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  const unsigned long long ctx = g_noalloc_ptr[dev] != nullptr ? current_context_id() : 0;
  if (g_noalloc_ptr[dev] == nullptr || (ctx != 0 && ctx != g_noalloc_ctx[dev])) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, ha_noalloc_sumsq_partials);
    if (e != cudaSuccess || p == nullptr)
      return ha::fail(HA_ERR_CUDA, "ha_grad_sumsq_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<double*>(p);
    g_noalloc_ctx[dev] = current_context_id();  // the lookup made the device's context current
  }
  *out = g_noalloc_ptr[dev];
  return HA_OK;
}
}  // namespace

extern "C" int ha_grad_sumsq_noalloc(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks,
                                     int64_t chunk_elems, int grad_dtype, double* d_out, void* stream) {
  HA_NVTX_RANGE();
  using namespace ha;
  if (chunk_elems != HA_SUMSQ_CHUNK)
    return fail(HA_ERR_INVALID, "ha_grad_sumsq_noalloc: chunk_elems must be %d", HA_SUMSQ_CHUNK);
  if (!valid_float_dtype(grad_dtype)) return fail(HA_ERR_UNSUPPORTED, "ha_grad_sumsq_noalloc: grad dtype %d", grad_dtype);
  if (n_chunks < 0 || n_chunks > HA_NOALLOC_SUMSQ_MAX_CHUNKS)
    return fail(HA_ERR_INVALID,
                "ha_grad_sumsq_noalloc: %lld chunks exceed the fixed scratch of %d chunks (%lld elements); "
                "use ha_grad_sumsq with a caller-allocated partials buffer",
                (long long)n_chunks, HA_NOALLOC_SUMSQ_MAX_CHUNKS,
                (long long)HA_NOALLOC_SUMSQ_MAX_CHUNKS * HA_SUMSQ_CHUNK);
  if (d_out == nullptr) return fail(HA_ERR_INVALID, "ha_grad_sumsq_noalloc: NULL output");
  if (n_chunks > 0 && (d_tensors == nullptr || d_chunks == nullptr))
    return fail(HA_ERR_INVALID, "ha_grad_sumsq_noalloc: NULL table");
  double* partials = nullptr;
  if (int rc = noalloc_partials(&partials)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_chunks > 0) {
    const dim3 grid(static_cast<unsigned>(n_chunks));
    switch (grad_dtype) {
      case HA_F32: sumsq_kernel<HA_F32><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, n_chunks, partials); break;
      case HA_BF16: sumsq_kernel<HA_BF16><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, n_chunks, partials); break;
      default: sumsq_kernel<HA_F16><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, n_chunks, partials); break;
    }
    const int rc = check_launch("sumsq_kernel (noalloc)");
    if (rc != HA_OK) return rc;
  }
  finalize_kernel<<<1, kFinalThreads, 0, st>>>(partials, n_chunks, d_out);
  return check_launch("sumsq_finalize_kernel (noalloc)");
}
