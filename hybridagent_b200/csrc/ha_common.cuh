// Shared device helpers of the ZeRO-1 AdamW kernels (sm_100a).
//
// Every floating-point operation of the update goes through an explicitly rounded
// intrinsic (__fmul_rn, __fmaf_rn, __fdiv_rn, __fsqrt_rn, ...) so that each torch op of
// the reference (hybrid_rl/optimizer.py:176-191) is reproduced with exactly the
// rounding torch's CUDA kernel gives it; the library is also built with -fmad=false so
// no other contraction can appear.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "hybridagent_b200.h"
#include "ha_nvtx.h"

namespace ha {

constexpr int kThreads = 256;  // threads per CTA of every multi-tensor kernel

// Sets the thread-local error message; returns `code`.
int fail(int code, const char* fmt, ...);
// HA_ERR_CUDA with cudaGetErrorString when the last launch failed.
int check_launch(const char* what);

template <int DT>
struct Elem;
template <>
struct Elem<HA_F32> {
  using raw = float;
  static __device__ __forceinline__ float widen(float x) { return x; }
  static __device__ __forceinline__ float narrow(float x) { return x; }  // value already fp32
};
template <>
struct Elem<HA_BF16> {
  using raw = uint16_t;
  static __device__ __forceinline__ float widen(uint16_t x) { return __uint_as_float(uint32_t(x) << 16); }
  static __device__ __forceinline__ uint16_t narrow(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
  }
};
template <>
struct Elem<HA_F16> {
  using raw = uint16_t;
  static __device__ __forceinline__ float widen(uint16_t x) { return __half2float(__ushort_as_half(x)); }
  static __device__ __forceinline__ uint16_t narrow(float x) { return __half_as_ushort(__float2half_rn(x)); }
};

// torch's `grad.mul_(scale)` of a DT gradient: float(g) * (float)scale, rounded to DT
// (optimizer.py:159), widened again for the update's `.float()` (optimizer.py:176).
template <int DT>
__device__ __forceinline__ float clip_round(float g, float mult) {
  const float p = __fmul_rn(g, mult);
  if constexpr (DT == HA_F32) {
    return p;
  } else {
    return Elem<DT>::widen(Elem<DT>::narrow(p));
  }
}

// Four consecutive elements of a DT array as fp32 (fp32: one 16-byte load; 16-bit types:
// one 8-byte load).  Streaming loads: every byte is touched once per step.
template <int DT>
__device__ __forceinline__ float4 load4(const void* base, int64_t e) {
  if constexpr (DT == HA_F32) {
    return __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(base) + e));
  } else {
    const uint2 w = __ldcs(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(base) + e));
    return make_float4(Elem<DT>::widen(uint16_t(w.x & 0xffffu)), Elem<DT>::widen(uint16_t(w.x >> 16)),
                       Elem<DT>::widen(uint16_t(w.y & 0xffffu)), Elem<DT>::widen(uint16_t(w.y >> 16)));
  }
}

template <int DT>
__device__ __forceinline__ float load1(const void* base, int64_t e) {
  return Elem<DT>::widen(static_cast<const typename Elem<DT>::raw*>(base)[e]);
}

__device__ __forceinline__ float4 load4_f32(const float* base, int64_t e) {
  return __ldcs(reinterpret_cast<const float4*>(base + e));
}
__device__ __forceinline__ void store4_f32(float* base, int64_t e, float4 x) {
  __stcs(reinterpret_cast<float4*>(base + e), x);
}

// Rounds four fp32 values to a 16-bit DT and stores them with one 8-byte store.
template <int DT>
__device__ __forceinline__ void store4_narrow(void* base, int64_t e, float4 x) {
  const uint32_t lo = uint32_t(Elem<DT>::narrow(x.x)) | (uint32_t(Elem<DT>::narrow(x.y)) << 16);
  const uint32_t hi = uint32_t(Elem<DT>::narrow(x.z)) | (uint32_t(Elem<DT>::narrow(x.w)) << 16);
  __stcs(reinterpret_cast<uint2*>(static_cast<uint16_t*>(base) + e), make_uint2(lo, hi));
}

// The 64-byte tensor descriptor and the chunk index of this CTA, staged in shared memory
// by four threads (one 16-byte load each).
struct __align__(16) StagedChunk {  // written with 16-byte shared stores
  ha_tensor t;
  uint32_t index;
};

__device__ __forceinline__ void stage_chunk(const ha_tensor* __restrict__ tensors,
                                            const ha_chunk* __restrict__ chunks, StagedChunk* s) {
  static_assert(sizeof(ha_tensor) == 64, "ha_tensor must stay 64 bytes");
  if (threadIdx.x < 4) {
    const ha_chunk c = chunks[blockIdx.x];
    reinterpret_cast<uint4*>(&s->t)[threadIdx.x] = reinterpret_cast<const uint4*>(tensors + c.tensor)[threadIdx.x];
    if (threadIdx.x == 0) s->index = c.index;
  }
  __syncthreads();
}

inline bool valid_float_dtype(int dt) { return dt == HA_F32 || dt == HA_BF16 || dt == HA_F16; }

}  // namespace ha
