// Multi-tensor copy / zero-fill (sm_100a).
//
// Moves every rank's gradients in one launch, replacing the per-tensor
// `flat[offset:offset+n].copy_(grad)` / `.zero_()` bucket packing of
// hybrid_rl/optimizer.py:126-135: into the local owner-major pack (nccl mode) or, with
// peer-mapped destinations, straight into the owners' receive windows (p2p mode).  Stream
// order makes the stores visible to the collective enqueued after the launch.  One CTA copies one chunk of one table
// entry with 16-byte loads and stores when both ends are 16-byte aligned.
#include <type_traits>

#include "ha_common.cuh"

namespace ha {
namespace {

template <int BYTES>
__global__ void __launch_bounds__(kThreads) gather_kernel(const ha_copy* __restrict__ copies,
                                                          const ha_chunk* __restrict__ chunks, int64_t chunk_elems) {
  using T = typename std::conditional<BYTES == 2, uint16_t, uint32_t>::type;
  __shared__ __align__(16) ha_copy c;  // written with 16-byte shared stores
  __shared__ uint32_t index;
  if (threadIdx.x < 2) {
    const ha_chunk ch = chunks[blockIdx.x];
    reinterpret_cast<uint4*>(&c)[threadIdx.x] = reinterpret_cast<const uint4*>(copies + ch.tensor)[threadIdx.x];
    if (threadIdx.x == 0) index = ch.index;
  }
  __syncthreads();
  if (c.src == c.dst) return;  // the data already sits in its slot
  const int64_t begin = int64_t(index) * chunk_elems;
  const int64_t end = min(begin + chunk_elems, c.numel);
  T* dst = reinterpret_cast<T*>(c.dst);
  const T* src = reinterpret_cast<const T*>(c.src);
  constexpr int V = 16 / BYTES;  // elements per 16-byte vector
  const bool vec = ((c.dst | c.src) & 15) == 0;  // chunk starts are multiples of V elements
  if (vec) {
    int64_t e = begin + int64_t(threadIdx.x) * V;
    for (; e + V <= end; e += int64_t(kThreads) * V) {
      const uint4 w = src ? __ldcs(reinterpret_cast<const uint4*>(src + e)) : make_uint4(0, 0, 0, 0);
      __stcs(reinterpret_cast<uint4*>(dst + e), w);
    }
    for (int64_t k = e; k < end && k < e + V; ++k) dst[k] = src ? src[k] : T(0);
  } else {
    for (int64_t k = begin + threadIdx.x; k < end; k += kThreads) dst[k] = src ? src[k] : T(0);
  }
}

int launch_gather(const ha_copy* d_copies, const ha_chunk* d_chunks, int64_t n_chunks, int64_t chunk_elems,
                  int elem_bytes, void* stream, const char* what) {
  if (elem_bytes != 2 && elem_bytes != 4) return fail(HA_ERR_UNSUPPORTED, "%s: elem_bytes %d", what, elem_bytes);
  if (chunk_elems <= 0 || chunk_elems % 8 != 0) return fail(HA_ERR_INVALID, "%s: chunk_elems %lld", what, (long long)chunk_elems);
  if (n_chunks < 0 || n_chunks > 0x7fffffffLL) return fail(HA_ERR_INVALID, "%s: n_chunks %lld", what, (long long)n_chunks);
  if (n_chunks == 0) return HA_OK;
  if (d_copies == nullptr || d_chunks == nullptr) return fail(HA_ERR_INVALID, "%s: NULL table", what);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(n_chunks));
  if (elem_bytes == 2) {
    gather_kernel<2><<<grid, kThreads, 0, st>>>(d_copies, d_chunks, chunk_elems);
  } else {
    gather_kernel<4><<<grid, kThreads, 0, st>>>(d_copies, d_chunks, chunk_elems);
  }
  return check_launch(what);
}

}  // namespace
}  // namespace ha

extern "C" int ha_gather(const ha_copy* d_copies, const ha_chunk* d_chunks, int64_t n_chunks, int64_t chunk_elems,
                         int elem_bytes, void* stream) {
  return ha::launch_gather(d_copies, d_chunks, n_chunks, chunk_elems, elem_bytes, stream, "ha_gather");
}
