// Peer-to-peer (NVLink / NVSwitch) pieces of the multi-GPU ZeRO-1 step (sm_100a).
//
// The reference moves gradients with one dist.reduce per owner bucket and parameters with
// one dist.broadcast per tensor (hybrid_rl/optimizer.py:136, :194).  Here every rank maps
// its peers' receive and parameter buffers (CUDA IPC) and moves data with plain loads and
// stores from its own kernels:
//   * push: each rank stores its gradient of every tensor into region <rank> of the
//     owner's receive buffer (ha_gather with peer destinations) -- the pack and the
//     transfer in one pass over the local gradients;
//   * ha_sum_regions (this file): the owner adds the W regions in fp32 in rank order,
//     rounds once to the gradient dtype, writes the sum into its own gradient buffer and
//     emits the sum of squares of the result (the global norm's partials) in the same pass;
//   * ha_adamw_step_peers (adamw.cu): the update also stores each new parameter value
//     into every peer's parameter buffer (the all-gather fused into the update).
// Ordering between ranks comes from the caller's NCCL collectives between these launches
// (no kernel here waits on another GPU).  No TMA and no multicast: plain 8/16-byte peer
// accesses only.
#include <cuda_runtime.h>

#include <cstring>

#include "ha_common.cuh"

namespace ha {
namespace {

constexpr int64_t kChunk = HA_SUM_REGIONS_CHUNK;
constexpr int kGroups = 4;  // 4-element groups per thread per pass
constexpr int kMaxWorld = HA_MAX_PEERS + 1;

__device__ __forceinline__ double block_sum(double x, double* smem) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem[warp] = x;
  __syncthreads();
  if (warp == 0) {
    x = lane < (int)(blockDim.x >> 5) ? smem[lane] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  }
  return x;
}

template <int DT>
__device__ __forceinline__ float round_to(float x) {
  if constexpr (DT == HA_F32) {
    return x;
  } else {
    return Elem<DT>::widen(Elem<DT>::narrow(x));
  }
}

template <int DT>
__device__ __forceinline__ void store4_as(void* base, int64_t e, float4 x) {
  if constexpr (DT == HA_F32) {
    store4_f32(static_cast<float*>(base), e, x);
  } else {
    store4_narrow<DT>(base, e, x);
  }
}

// regions: W consecutive regions of region_elems elements; the sum of elements [0, count)
// of every region lands in `out` (which may be one of the regions).
template <int DT>
__global__ void __launch_bounds__(kThreads) sum_regions_kernel(const void* regions, int world, int64_t region_elems,
                                                               int64_t count, void* out,
                                                               double* __restrict__ partials) {
  __shared__ double red[kThreads / 32];
  using raw = typename Elem<DT>::raw;
  const raw* base = static_cast<const raw*>(regions);
  raw* own = static_cast<raw*>(out);
  const int64_t begin = int64_t(blockIdx.x) * kChunk;
  const int64_t end = min(begin + kChunk, count);
  double acc = 0.0;
  for (int64_t pass = begin; pass < end; pass += int64_t(kThreads) * kGroups * 4) {
    float4 s[kGroups];
    int64_t e[kGroups];
#pragma unroll
    for (int u = 0; u < kGroups; ++u) {
      e[u] = pass + 4 * (int64_t(threadIdx.x) + int64_t(u) * kThreads);
      if (e[u] + 4 <= end) s[u] = load4<DT>(base, e[u]);
    }
    for (int r = 1; r < world; ++r) {
      const raw* reg = base + int64_t(r) * region_elems;
#pragma unroll
      for (int u = 0; u < kGroups; ++u) {
        if (e[u] + 4 <= end) {
          const float4 x = load4<DT>(reg, e[u]);
          s[u].x = __fadd_rn(s[u].x, x.x);
          s[u].y = __fadd_rn(s[u].y, x.y);
          s[u].z = __fadd_rn(s[u].z, x.z);
          s[u].w = __fadd_rn(s[u].w, x.w);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kGroups; ++u) {
      if (e[u] + 4 <= end) {
        const float4 o = make_float4(round_to<DT>(s[u].x), round_to<DT>(s[u].y), round_to<DT>(s[u].z),
                                     round_to<DT>(s[u].w));
        store4_as<DT>(own, e[u], o);
        acc += double(__fadd_rn(__fadd_rn(__fmul_rn(o.x, o.x), __fmul_rn(o.y, o.y)),
                                __fadd_rn(__fmul_rn(o.z, o.z), __fmul_rn(o.w, o.w))));
      } else {
        for (int64_t k = e[u]; k < end; ++k) {  // ragged end of the region (one thread)
          float t = Elem<DT>::widen(base[k]);
          for (int r = 1; r < world; ++r) t = __fadd_rn(t, Elem<DT>::widen(base[int64_t(r) * region_elems + k]));
          t = round_to<DT>(t);
          if constexpr (DT == HA_F32) {
            own[k] = t;
          } else {
            own[k] = Elem<DT>::narrow(t);
          }
          acc += double(__fmul_rn(t, t));
        }
      }
    }
  }
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) partials[blockIdx.x] = acc;
}

constexpr int kFinalThreads = 1024;
__global__ void __launch_bounds__(kFinalThreads) finalize_regions_kernel(const double* __restrict__ partials,
                                                                          int64_t n, double* __restrict__ out) {
  __shared__ double red[kFinalThreads / 32];
  double a0 = 0.0, a1 = 0.0;
  int64_t i = threadIdx.x;
  for (; i + kFinalThreads < n; i += 2 * kFinalThreads) {
    a0 += partials[i];
    a1 += partials[i + kFinalThreads];
  }
  for (; i < n; i += kFinalThreads) a0 += partials[i];
  const double x = block_sum(a0 + a1, red);
  if (threadIdx.x == 0) out[0] = x;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return HA_OK;
  return fail(HA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace
}  // namespace ha

extern "C" int ha_malloc(size_t bytes, void** out) {
  if (out == nullptr || bytes == 0) return ha::fail(HA_ERR_INVALID, "ha_malloc: bad arguments");
  *out = nullptr;
  return ha::cuda_status(cudaMalloc(out, bytes), "cudaMalloc");
}

extern "C" int ha_free(void* ptr) {
  if (ptr == nullptr) return HA_OK;
  return ha::cuda_status(cudaFree(ptr), "cudaFree");
}

extern "C" int ha_memset(void* ptr, int value, size_t bytes, void* stream) {
  HA_NVTX_RANGE();
  if (ptr == nullptr && bytes > 0) return ha::fail(HA_ERR_INVALID, "ha_memset: NULL");
  return ha::cuda_status(cudaMemsetAsync(ptr, value, bytes, static_cast<cudaStream_t>(stream)), "cudaMemsetAsync");
}

extern "C" int ha_ipc_get_handle(const void* ptr, uint8_t out[HA_IPC_HANDLE_BYTES]) {
  static_assert(sizeof(cudaIpcMemHandle_t) == HA_IPC_HANDLE_BYTES, "IPC handle size");
  if (ptr == nullptr || out == nullptr) return ha::fail(HA_ERR_INVALID, "ha_ipc_get_handle: NULL");
  cudaIpcMemHandle_t h;
  if (int rc = ha::cuda_status(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "cudaIpcGetMemHandle")) return rc;
  memcpy(out, &h, sizeof h);
  return HA_OK;
}

extern "C" int ha_ipc_open(const uint8_t handle[HA_IPC_HANDLE_BYTES], void** out) {
  if (handle == nullptr || out == nullptr) return ha::fail(HA_ERR_INVALID, "ha_ipc_open: NULL");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  *out = nullptr;
  return ha::cuda_status(cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

extern "C" int ha_ipc_close(void* ptr) {
  if (ptr == nullptr) return HA_OK;
  return ha::cuda_status(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
}

extern "C" int ha_sum_regions(const void* d_regions, int32_t world, int64_t region_elems, int64_t count,
                              void* d_sum, int dtype, double* d_partials, double* d_out, void* stream) {
  HA_NVTX_RANGE();
  using namespace ha;
  if (!valid_float_dtype(dtype)) return fail(HA_ERR_UNSUPPORTED, "ha_sum_regions: dtype %d", dtype);
  if (world < 1 || world > kMaxWorld)
    return fail(HA_ERR_INVALID, "ha_sum_regions: world %d (at most %d ranks)", world, kMaxWorld);
  if (count < 0 || count > region_elems || region_elems % 64 != 0)
    return fail(HA_ERR_INVALID, "ha_sum_regions: count %lld, region %lld (multiple of 64 elements)",
                (long long)count, (long long)region_elems);
  if (d_out == nullptr || (count > 0 && (d_regions == nullptr || d_partials == nullptr || d_sum == nullptr)))
    return fail(HA_ERR_INVALID, "ha_sum_regions: NULL buffer");
  if (((reinterpret_cast<uintptr_t>(d_regions) | reinterpret_cast<uintptr_t>(d_sum)) & 15) != 0)
    return fail(HA_ERR_INVALID, "ha_sum_regions: regions and sum must be 16-byte aligned");
  const int64_t n_chunks = (count + kChunk - 1) / kChunk;
  if (n_chunks > 0x7fffffffLL) return fail(HA_ERR_INVALID, "ha_sum_regions: too many chunks");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_chunks > 0) {
    const dim3 grid(static_cast<unsigned>(n_chunks));
    switch (dtype) {
      case HA_F32:
        sum_regions_kernel<HA_F32><<<grid, kThreads, 0, st>>>(d_regions, world, region_elems, count, d_sum, d_partials);
        break;
      case HA_BF16:
        sum_regions_kernel<HA_BF16><<<grid, kThreads, 0, st>>>(d_regions, world, region_elems, count, d_sum, d_partials);
        break;
      default:
        sum_regions_kernel<HA_F16><<<grid, kThreads, 0, st>>>(d_regions, world, region_elems, count, d_sum, d_partials);
        break;
    }
    if (int rc = check_launch("sum_regions_kernel")) return rc;
  }
  finalize_regions_kernel<<<1, kFinalThreads, 0, st>>>(d_partials, n_chunks, d_out);
  return check_launch("finalize_regions_kernel");
}
