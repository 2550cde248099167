// Multi-tensor copy / zero-fill (sm_100a).
//
// Moves every rank's gradients in one launch, replacing the per-tensor
// `flat[offset:offset+n].copy_(grad)` / `.zero_()` bucket packing of
// hybrid_rl/optimizer.py:126-135: into the local owner-major pack (nccl mode) or, with
// peer-mapped destinations, straight into the owners' receive windows (p2p mode).  Stream
// order makes the stores visible to the collective enqueued after the launch.  One CTA copies one chunk of one table
// entry with 16-byte loads and stores when both ends are 16-byte aligned.
//
// ha_gather_capped runs the same copies on at most max_ctas CTAs, each walking the chunk
// list with the grid's stride and keeping 4 vectors per thread in flight: the early
// gradient pushes that run beside backward use it so that they occupy a few SMs' thread
// slots instead of all of them.  ha_copy_async issues the copies to the copy engines
// (one cudaMemcpyAsync / cudaMemsetAsync per entry) and uses no SM at all.
#include <algorithm>
#include <type_traits>

#include "ha_common.cuh"

namespace ha {
namespace {

// Copies (or zero-fills, src == 0) elements [index*chunk_elems, +chunk_elems) of one table
// entry; the CTA's threads stride through it with U 16-byte vectors per thread in flight.
// Each thread's vector starts are begin + tid*V + j*kThreads*V, so exactly one thread meets
// the final partial vector and writes its tail elements.
template <typename T, int U>
__device__ __forceinline__ void copy_chunk(const ha_copy& c, uint32_t index, int64_t chunk_elems) {
  const int64_t begin = int64_t(index) * chunk_elems;
  const int64_t end = min(begin + chunk_elems, c.numel);
  T* dst = reinterpret_cast<T*>(c.dst);
  const T* src = reinterpret_cast<const T*>(c.src);
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
  constexpr int64_t step = int64_t(kThreads) * V;
  const bool vec = ((c.dst | c.src) & 15) == 0;  // chunk starts are multiples of V elements
  if (vec) {
    int64_t e = begin + int64_t(threadIdx.x) * V;
    if constexpr (U > 1) {
      for (; e + (U - 1) * step + V <= end; e += U * step) {
        uint4 w[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          w[u] = src ? __ldcs(reinterpret_cast<const uint4*>(src + e + u * step)) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < U; ++u) __stcs(reinterpret_cast<uint4*>(dst + e + u * step), w[u]);
      }
    }
    for (; e + V <= end; e += step) {
      const uint4 w = src ? __ldcs(reinterpret_cast<const uint4*>(src + e)) : make_uint4(0, 0, 0, 0);
      __stcs(reinterpret_cast<uint4*>(dst + e), w);
    }
    for (int64_t k = e; k < end && k < e + V; ++k) dst[k] = src ? src[k] : T(0);
  } else {
    for (int64_t k = begin + threadIdx.x; k < end; k += kThreads) dst[k] = src ? src[k] : T(0);
  }
}

// Stages chunk q's copy descriptor and index in shared memory (16-byte shared stores).
__device__ __forceinline__ void stage_copy(const ha_copy* __restrict__ copies, const ha_chunk* __restrict__ chunks,
                                           int64_t q, ha_copy* c, uint32_t* index) {
  if (threadIdx.x < 2) {
    const ha_chunk ch = chunks[q];
    reinterpret_cast<uint4*>(c)[threadIdx.x] = reinterpret_cast<const uint4*>(copies + ch.tensor)[threadIdx.x];
    if (threadIdx.x == 0) *index = ch.index;
  }
  __syncthreads();
}

template <int BYTES>
__global__ void __launch_bounds__(kThreads) gather_kernel(const ha_copy* __restrict__ copies,
                                                          const ha_chunk* __restrict__ chunks, int64_t chunk_elems) {
  using T = typename std::conditional<BYTES == 2, uint16_t, uint32_t>::type;
  __shared__ __align__(16) ha_copy c;
  __shared__ uint32_t index;
  stage_copy(copies, chunks, blockIdx.x, &c, &index);
  if (c.src == c.dst) return;  // the data already sits in its slot
  copy_chunk<T, 1>(c, index, chunk_elems);
}

// One CTA per SM slot it is given: walks chunks blockIdx.x, blockIdx.x + gridDim.x, ...
template <int BYTES>
__global__ void __launch_bounds__(kThreads) gather_capped_kernel(const ha_copy* __restrict__ copies,
                                                                 const ha_chunk* __restrict__ chunks, int64_t n_chunks,
                                                                 int64_t chunk_elems) {
  using T = typename std::conditional<BYTES == 2, uint16_t, uint32_t>::type;
  __shared__ __align__(16) ha_copy c;
  __shared__ uint32_t index;
  for (int64_t q = blockIdx.x; q < n_chunks; q += gridDim.x) {
    stage_copy(copies, chunks, q, &c, &index);
    if (c.src != c.dst) copy_chunk<T, 4>(c, index, chunk_elems);
    __syncthreads();  // every thread is done with this descriptor before the next is staged
  }
}

int launch_gather(const ha_copy* d_copies, const ha_chunk* d_chunks, int64_t n_chunks, int64_t chunk_elems,
                  int elem_bytes, int32_t max_ctas, void* stream, const char* what) {
  if (elem_bytes != 2 && elem_bytes != 4) return fail(HA_ERR_UNSUPPORTED, "%s: elem_bytes %d", what, elem_bytes);
  if (chunk_elems <= 0 || chunk_elems % 8 != 0) return fail(HA_ERR_INVALID, "%s: chunk_elems %lld", what, (long long)chunk_elems);
  if (n_chunks < 0 || n_chunks > 0x7fffffffLL) return fail(HA_ERR_INVALID, "%s: n_chunks %lld", what, (long long)n_chunks);
  if (max_ctas < 0) return fail(HA_ERR_INVALID, "%s: max_ctas %d", what, max_ctas);
  if (n_chunks == 0) return HA_OK;
  if (d_copies == nullptr || d_chunks == nullptr) return fail(HA_ERR_INVALID, "%s: NULL table", what);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (max_ctas == 0) {  // one CTA per chunk
    const dim3 grid(static_cast<unsigned>(n_chunks));
    if (elem_bytes == 2) {
      gather_kernel<2><<<grid, kThreads, 0, st>>>(d_copies, d_chunks, chunk_elems);
    } else {
      gather_kernel<4><<<grid, kThreads, 0, st>>>(d_copies, d_chunks, chunk_elems);
    }
  } else {
    const dim3 grid(static_cast<unsigned>(std::min<int64_t>(n_chunks, max_ctas)));
    if (elem_bytes == 2) {
      gather_capped_kernel<2><<<grid, kThreads, 0, st>>>(d_copies, d_chunks, n_chunks, chunk_elems);
    } else {
      gather_capped_kernel<4><<<grid, kThreads, 0, st>>>(d_copies, d_chunks, n_chunks, chunk_elems);
    }
  }
  return check_launch(what);
}

}  // namespace
}  // namespace ha

extern "C" int ha_gather(const ha_copy* d_copies, const ha_chunk* d_chunks, int64_t n_chunks, int64_t chunk_elems,
                         int elem_bytes, void* stream) {
  HA_NVTX_RANGE();
  return ha::launch_gather(d_copies, d_chunks, n_chunks, chunk_elems, elem_bytes, 0, stream, "ha_gather");
}

extern "C" int ha_gather_capped(const ha_copy* d_copies, const ha_chunk* d_chunks, int64_t n_chunks,
                                int64_t chunk_elems, int elem_bytes, int32_t max_ctas, void* stream) {
  HA_NVTX_RANGE();
  if (max_ctas <= 0) return ha::fail(HA_ERR_INVALID, "ha_gather_capped: max_ctas %d", max_ctas);
  return ha::launch_gather(d_copies, d_chunks, n_chunks, chunk_elems, elem_bytes, max_ctas, stream,
                           "ha_gather_capped");
}

extern "C" int ha_copy_async(const ha_copy* h_copies, int64_t n, int elem_bytes, void* stream) {
  HA_NVTX_RANGE();
  if (elem_bytes != 2 && elem_bytes != 4) return ha::fail(HA_ERR_UNSUPPORTED, "ha_copy_async: elem_bytes %d", elem_bytes);
  if (n < 0 || (n > 0 && h_copies == nullptr)) return ha::fail(HA_ERR_INVALID, "ha_copy_async: %lld entries", (long long)n);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int64_t k = 0; k < n; ++k) {
    const ha_copy& c = h_copies[k];
    if (c.numel < 0 || c.dst == 0) return ha::fail(HA_ERR_INVALID, "ha_copy_async: entry %lld", (long long)k);
    if (c.numel == 0 || c.src == c.dst) continue;
    const size_t bytes = static_cast<size_t>(c.numel) * static_cast<size_t>(elem_bytes);
    const cudaError_t e = c.src == 0 ? cudaMemsetAsync(reinterpret_cast<void*>(c.dst), 0, bytes, st)
                                     : cudaMemcpyAsync(reinterpret_cast<void*>(c.dst), reinterpret_cast<const void*>(c.src),
                                                       bytes, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return ha::fail(HA_ERR_CUDA, "ha_copy_async: entry %lld: %s", (long long)k, cudaGetErrorString(e));
  }
  return HA_OK;
}
