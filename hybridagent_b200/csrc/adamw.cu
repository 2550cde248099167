// Fused multi-tensor AdamW step and in-place gradient scaling (sm_100a).
//
// Replaces the per-tensor loop of hybrid_rl/optimizer.py:173-191 (about thirteen torch
// eager kernels per tensor, ~116 bytes of HBM traffic per parameter) with one launch
// that streams each element once: read grad + master + exp_avg + exp_avg_sq, write
// master + exp_avg + exp_avg_sq + the low-precision parameter copy.
//
// Work split: one CTA per chunk of HA_ADAMW_CHUNK = 16384 elements of one tensor
// (ha_chunk table), in four passes of 256 threads x 4 groups x 4 elements.  Within a
// pass the 4 groups' loads (224 bytes per thread for bf16) are all issued before any
// math, so a CTA keeps ~56 KB of reads in flight.  Consecutive lanes own consecutive
// 4-element groups, so every warp-wide load or store is one contiguous 512-byte (fp32) or
// 256-byte (16-bit) segment.  Tensors whose pointers are not 16-byte aligned (possible
// for caller-owned gradients) take a scalar path with identical arithmetic.
#include "ha_common.cuh"

namespace ha {
namespace {

constexpr int kGroups = 4;                                  // 4-element groups per thread per pass
constexpr int64_t kPass = int64_t(kThreads) * kGroups * 4;   // elements per CTA pass
constexpr int64_t kChunk = HA_ADAMW_CHUNK;
static_assert(kChunk % kPass == 0, "chunk geometry");

struct Scalars {
  float b1, a1, b2, a2, eps;
  int use_decay;
  int clip;
  float clip_mult;
};

// One element, torch CUDA rounding op by op (optimizer.py:184-189):
//   master.mul_(1 - lr*wd)                          -> master * decay
//   mean.mul_(b1).add_(g, alpha=1-b1)               -> fma(a1, g, m*b1)
//   variance.mul_(b2).addcmul_(g, g, value=1-b2)    -> fma(a2, g*g, v*b2)
//   (variance / c2).sqrt().add_(eps)                -> sqrt(v * rc2) + eps, rc2 = (float)(1.0 / c2)
//   master.addcdiv_(mean / c1, denom, value=-lr)    -> fma(-lr, (m * rc1) / denom, master)
// (torch divides by a Python float by multiplying with its double reciprocal rounded to fp32)
__device__ __forceinline__ void adamw_elem(const Scalars& s, float decay, float neg_lr, float rc1, float rc2,
                                           float g, float& ms, float& m, float& v) {
  if (s.use_decay) ms = __fmul_rn(ms, decay);
  m = __fmaf_rn(s.a1, g, __fmul_rn(m, s.b1));
  v = __fmaf_rn(s.a2, __fmul_rn(g, g), __fmul_rn(v, s.b2));
  const float den = __fadd_rn(__fsqrt_rn(__fmul_rn(v, rc2)), s.eps);
  ms = __fmaf_rn(neg_lr, __fdiv_rn(__fmul_rn(m, rc1), den), ms);
}

template <int DT>
__device__ __forceinline__ float grad_in(const Scalars& s, float g) {
  return s.clip ? clip_round<DT>(g, s.clip_mult) : g;
}

struct Peers {
  int n;
  int64_t delta[HA_MAX_PEERS];
};

// Four values rounded to a 16-bit DT, packed as one 8-byte word.
template <int DT>
__device__ __forceinline__ uint2 pack4(float4 x) {
  return make_uint2(uint32_t(Elem<DT>::narrow(x.x)) | (uint32_t(Elem<DT>::narrow(x.y)) << 16),
                    uint32_t(Elem<DT>::narrow(x.z)) | (uint32_t(Elem<DT>::narrow(x.w)) << 16));
}

// The same 8 bytes at `local` + e in every peer's copy of the packed parameter buffer.
__device__ __forceinline__ void push_raw4(const Peers& p, uint64_t local, int64_t e, uint2 w) {
#pragma unroll
  for (int q = 0; q < HA_MAX_PEERS; ++q) {  // constant indices keep delta[] in the parameter bank
    if (q >= p.n) break;
    __stcs(reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(local + p.delta[q]) + e), w);
  }
}

__device__ __forceinline__ void push_f32x4(const Peers& p, uint64_t local, int64_t e, float4 x) {
#pragma unroll
  for (int q = 0; q < HA_MAX_PEERS; ++q) {
    if (q >= p.n) break;
    store4_f32(reinterpret_cast<float*>(local + p.delta[q]), e, x);
  }
}

template <int DT>
__device__ __forceinline__ void push1(const Peers& p, uint64_t local, int64_t k, float x) {
#pragma unroll
  for (int q = 0; q < HA_MAX_PEERS; ++q) {
    if (q >= p.n) break;
    if constexpr (DT == HA_F32) {
      reinterpret_cast<float*>(local + p.delta[q])[k] = x;
    } else {
      reinterpret_cast<uint16_t*>(local + p.delta[q])[k] = Elem<DT>::narrow(x);
    }
  }
}

// DT is the gradient and parameter dtype.  For HA_F32 the master is the parameter
// (optimizer.py:71-73) and no separate copy is written.  PEERS: the parameter all-gather is
// fused in -- every new parameter value also goes to the same place in every peer's copy of
// the packed parameter buffer (the per-tensor dist.broadcast of optimizer.py:192-194).
//
// DELTA (16-bit parameters): a 4-element group of the parameter copy is stored -- locally and,
// with PEERS, to every peer -- only if its rounded value changed, i.e. if RNE(new master)
// differs from RNE(old master).  The caller guarantees that every copy of the parameter holds
// RNE(old master) on entry (the optimizer falls back to the dense kernel for a step after
// anything else wrote a parameter or a master); every copy then ends with exactly the bits a
// full write would leave.  With the small learning rates of RL fine-tuning few bf16 values move
// in a step, so this saves the 2 B/param parameter write in HBM and nearly all of the
// all-gather's NVLink bytes.
//
// `changed` (DELTA, may be null): the number of stored groups (scalar-path elements count as
// groups; on the vector path a changed group stores the three others of its 32-byte sector too)
// is added to it, one atomic per CTA, so the caller can tell how much moved.
template <int DT, bool PEERS, bool DELTA>
__global__ void __launch_bounds__(kThreads) adamw_kernel(const ha_tensor* __restrict__ tensors,
                                                         const ha_chunk* __restrict__ chunks, Scalars s, Peers peers,
                                                         unsigned long long* changed) {
  static_assert(!(DELTA && DT == HA_F32), "fp32 parameters are their own masters: always written");
  __shared__ StagedChunk sc;
  __shared__ uint32_t stored_in_cta;
  stage_chunk(tensors, chunks, &sc);
  const ha_tensor& t = sc.t;
  if (t.grad == 0) return;  // no gradient: skipped entirely (optimizer.py:174)
  const int64_t begin = int64_t(sc.index) * kChunk;
  const int64_t end = min(begin + kChunk, t.numel);
  const void* grad = reinterpret_cast<const void*>(t.grad);
  float* master = reinterpret_cast<float*>(t.master);
  float* exp_avg = reinterpret_cast<float*>(t.exp_avg);
  float* exp_avg_sq = reinterpret_cast<float*>(t.exp_avg_sq);
  void* param = reinterpret_cast<void*>(t.param);
  const float decay = t.decay, neg_lr = t.neg_lr, rc1 = t.rc1, rc2 = t.rc2;
  const uint64_t pushed = DT == HA_F32 ? t.master : t.param;  // the parameter's local address

  constexpr uint64_t kNarrowAlign = DT == HA_F32 ? 15 : 7;
  const bool vec = ((t.master | t.exp_avg | t.exp_avg_sq) & 15) == 0 && (t.grad & kNarrowAlign) == 0 &&
                   (DT == HA_F32 || (t.param & kNarrowAlign) == 0);
  uint32_t stored = 0;  // DELTA: groups this thread stored
  if (DELTA && threadIdx.x == 0) stored_in_cta = 0;
  // one element on the scalar paths (ragged tails, unaligned tensors)
  auto one = [&](int64_t k) {
    float a = master[k], b = exp_avg[k], c = exp_avg_sq[k];
    const float before = a;
    adamw_elem(s, decay, neg_lr, rc1, rc2, grad_in<DT>(s, load1<DT>(grad, k)), a, b, c);
    master[k] = a;
    exp_avg[k] = b;
    exp_avg_sq[k] = c;
    if constexpr (DT != HA_F32) {
      const uint16_t w = Elem<DT>::narrow(a);
      if (!DELTA || w != Elem<DT>::narrow(before)) {
        static_cast<uint16_t*>(param)[k] = w;
        if constexpr (PEERS) push1<DT>(peers, pushed, k, a);
        stored += DELTA;
      }
    } else if constexpr (PEERS) {
      push1<DT>(peers, pushed, k, a);
    }
  };
  if (vec) {
    for (int64_t base = begin; base < end; base += kPass) {
      float4 g[kGroups], ms[kGroups], m[kGroups], v[kGroups];
      int64_t e[kGroups];
#pragma unroll
      for (int u = 0; u < kGroups; ++u) {
        e[u] = base + 4 * (int64_t(threadIdx.x) + int64_t(u) * kThreads);
        if (e[u] + 4 <= end) {
          g[u] = load4<DT>(grad, e[u]);
          ms[u] = load4_f32(master, e[u]);
          m[u] = load4_f32(exp_avg, e[u]);
          v[u] = load4_f32(exp_avg_sq, e[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < kGroups; ++u) {
        const bool full = e[u] + 4 <= end;
        uint2 w = make_uint2(0, 0);
        bool changed = false;
        if (full) {
          uint2 before = make_uint2(0, 0);
          if constexpr (DELTA) before = pack4<DT>(ms[u]);
          adamw_elem(s, decay, neg_lr, rc1, rc2, grad_in<DT>(s, g[u].x), ms[u].x, m[u].x, v[u].x);
          adamw_elem(s, decay, neg_lr, rc1, rc2, grad_in<DT>(s, g[u].y), ms[u].y, m[u].y, v[u].y);
          adamw_elem(s, decay, neg_lr, rc1, rc2, grad_in<DT>(s, g[u].z), ms[u].z, m[u].z, v[u].z);
          adamw_elem(s, decay, neg_lr, rc1, rc2, grad_in<DT>(s, g[u].w), ms[u].w, m[u].w, v[u].w);
          store4_f32(master, e[u], ms[u]);
          store4_f32(exp_avg, e[u], m[u]);
          store4_f32(exp_avg_sq, e[u], v[u]);
          if constexpr (DT != HA_F32) {
            w = pack4<DT>(ms[u]);
            changed = w.x != before.x || w.y != before.y;
          } else if constexpr (PEERS) {
            push_f32x4(peers, pushed, e[u], ms[u]);
          }
        }
        if constexpr (DT != HA_F32) {
          // DELTA: the four lanes whose groups share a 32-byte sector store together when any of
          // them changed (a whole sector, which the memory system writes without fetching it; the
          // other groups' values are unchanged, so every copy still ends with the same bits).
          // Every lane of the warp reaches the shuffles: the pass loop is uniform across the CTA.
          bool store = full;
          if constexpr (DELTA) {
            uint32_t any = changed ? 1u : 0u;
            any |= __shfl_xor_sync(0xffffffffu, any, 1);
            any |= __shfl_xor_sync(0xffffffffu, any, 2);
            store = full && any;
          }
          if (store) {
            __stcs(reinterpret_cast<uint2*>(static_cast<uint16_t*>(param) + e[u]), w);
            if constexpr (PEERS) push_raw4(peers, pushed, e[u], w);
            stored += DELTA;
          }
        }
        if (!full) {
          for (int64_t k = e[u]; k < end; ++k) one(k);  // ragged tail of the tensor (one thread)
        }
      }
    }
  } else {
    for (int64_t k = begin + threadIdx.x; k < end; k += kThreads) one(k);
  }
  if constexpr (DELTA) {
    if (changed != nullptr) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) stored += __shfl_xor_sync(0xffffffffu, stored, o);
      __syncthreads();  // stored_in_cta was cleared before any thread adds to it
      if ((threadIdx.x & 31) == 0 && stored) atomicAdd(&stored_in_cta, stored);
      __syncthreads();
      if (threadIdx.x == 0 && stored_in_cta) atomicAdd(changed, static_cast<unsigned long long>(stored_in_cta));
    }
  }
}

// grad.mul_(scale) in the gradient's dtype, in place (optimizer.py:157-159).
template <int DT>
__global__ void __launch_bounds__(kThreads) scale_kernel(const ha_tensor* __restrict__ tensors,
                                                         const ha_chunk* __restrict__ chunks, float mult) {
  __shared__ StagedChunk sc;
  stage_chunk(tensors, chunks, &sc);
  if (sc.t.grad == 0) return;
  using raw = typename Elem<DT>::raw;
  raw* grad = reinterpret_cast<raw*>(sc.t.grad);
  const int64_t begin = int64_t(sc.index) * kChunk;
  const int64_t end = min(begin + kChunk, sc.t.numel);
  for (int64_t k = begin + threadIdx.x; k < end; k += kThreads) {
    const float p = __fmul_rn(Elem<DT>::widen(grad[k]), mult);
    if constexpr (DT == HA_F32) {
      grad[k] = p;
    } else {
      grad[k] = Elem<DT>::narrow(p);
    }
  }
}

}  // namespace
}  // namespace ha

extern "C" int ha_adamw_step(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks,
                             int64_t chunk_elems, int grad_dtype, int param_dtype, const ha_adamw_scalars* sc,
                             void* stream) {
  HA_NVTX_RANGE();
  using namespace ha;
  if (chunk_elems != HA_ADAMW_CHUNK) return fail(HA_ERR_INVALID, "ha_adamw_step: chunk_elems must be %d", HA_ADAMW_CHUNK);
  if (!valid_float_dtype(grad_dtype)) return fail(HA_ERR_UNSUPPORTED, "ha_adamw_step: grad dtype %d", grad_dtype);
  if (grad_dtype != HA_F32 && param_dtype != grad_dtype)
    return fail(HA_ERR_UNSUPPORTED, "ha_adamw_step: param dtype %d with grad dtype %d", param_dtype, grad_dtype);
  if (n_chunks < 0 || n_chunks > 0x7fffffffLL) return fail(HA_ERR_INVALID, "ha_adamw_step: n_chunks %lld", (long long)n_chunks);
  if (sc == nullptr) return fail(HA_ERR_INVALID, "ha_adamw_step: scalars is NULL");
  if (n_chunks == 0) return HA_OK;
  if (d_tensors == nullptr || d_chunks == nullptr) return fail(HA_ERR_INVALID, "ha_adamw_step: NULL table");
  const Scalars s{sc->b1, sc->a1, sc->b2, sc->a2, sc->eps, sc->use_decay, sc->clip, sc->clip_mult};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(n_chunks));
  const Peers none{};
  switch (grad_dtype) {
    case HA_F32: adamw_kernel<HA_F32, false, false><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, s, none, nullptr); break;
    case HA_BF16: adamw_kernel<HA_BF16, false, false><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, s, none, nullptr); break;
    default: adamw_kernel<HA_F16, false, false><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, s, none, nullptr); break;
  }
  return check_launch("adamw_kernel");
}

extern "C" int ha_adamw_step_peers(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks,
                                   int64_t chunk_elems, int grad_dtype, int param_dtype, const ha_adamw_scalars* sc,
                                   const ha_peers* peers, void* stream) {
  HA_NVTX_RANGE();
  using namespace ha;
  if (chunk_elems != HA_ADAMW_CHUNK)
    return fail(HA_ERR_INVALID, "ha_adamw_step_peers: chunk_elems must be %d", HA_ADAMW_CHUNK);
  if (!valid_float_dtype(grad_dtype)) return fail(HA_ERR_UNSUPPORTED, "ha_adamw_step_peers: grad dtype %d", grad_dtype);
  if (grad_dtype != HA_F32 && param_dtype != grad_dtype)
    return fail(HA_ERR_UNSUPPORTED, "ha_adamw_step_peers: param dtype %d with grad dtype %d", param_dtype, grad_dtype);
  if (n_chunks < 0 || n_chunks > 0x7fffffffLL)
    return fail(HA_ERR_INVALID, "ha_adamw_step_peers: n_chunks %lld", (long long)n_chunks);
  if (sc == nullptr || peers == nullptr) return fail(HA_ERR_INVALID, "ha_adamw_step_peers: NULL scalars or peers");
  if (peers->n < 0 || peers->n > HA_MAX_PEERS) return fail(HA_ERR_INVALID, "ha_adamw_step_peers: %d peers", peers->n);
  for (int q = 0; q < peers->n; ++q)
    if ((peers->delta[q] & 15) != 0) return fail(HA_ERR_INVALID, "ha_adamw_step_peers: peer %d offset not 16-byte aligned", q);
  if (n_chunks == 0) return HA_OK;
  if (d_tensors == nullptr || d_chunks == nullptr) return fail(HA_ERR_INVALID, "ha_adamw_step_peers: NULL table");
  const Scalars s{sc->b1, sc->a1, sc->b2, sc->a2, sc->eps, sc->use_decay, sc->clip, sc->clip_mult};
  Peers p{};
  p.n = peers->n;
  for (int q = 0; q < peers->n; ++q) p.delta[q] = peers->delta[q];
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(n_chunks));
  switch (grad_dtype) {
    case HA_F32: adamw_kernel<HA_F32, true, false><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, s, p, nullptr); break;
    case HA_BF16: adamw_kernel<HA_BF16, true, false><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, s, p, nullptr); break;
    default: adamw_kernel<HA_F16, true, false><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, s, p, nullptr); break;
  }
  return check_launch("adamw_kernel (peers)");
}

extern "C" int ha_adamw_step_delta(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks,
                                   int64_t chunk_elems, int param_dtype, const ha_adamw_scalars* sc,
                                   const ha_peers* peers, unsigned long long* d_changed_groups, void* stream) {
  HA_NVTX_RANGE();
  using namespace ha;
  if (chunk_elems != HA_ADAMW_CHUNK)
    return fail(HA_ERR_INVALID, "ha_adamw_step_delta: chunk_elems must be %d", HA_ADAMW_CHUNK);
  if (param_dtype != HA_BF16 && param_dtype != HA_F16)
    return fail(HA_ERR_UNSUPPORTED, "ha_adamw_step_delta: param dtype %d (16-bit parameters only)", param_dtype);
  if (n_chunks < 0 || n_chunks > 0x7fffffffLL)
    return fail(HA_ERR_INVALID, "ha_adamw_step_delta: n_chunks %lld", (long long)n_chunks);
  if (sc == nullptr) return fail(HA_ERR_INVALID, "ha_adamw_step_delta: NULL scalars");
  if (peers != nullptr) {
    if (peers->n < 0 || peers->n > HA_MAX_PEERS) return fail(HA_ERR_INVALID, "ha_adamw_step_delta: %d peers", peers->n);
    for (int q = 0; q < peers->n; ++q)
      if ((peers->delta[q] & 15) != 0)
        return fail(HA_ERR_INVALID, "ha_adamw_step_delta: peer %d offset not 16-byte aligned", q);
  }
  if (n_chunks == 0) return HA_OK;
  if (d_tensors == nullptr || d_chunks == nullptr) return fail(HA_ERR_INVALID, "ha_adamw_step_delta: NULL table");
  const Scalars s{sc->b1, sc->a1, sc->b2, sc->a2, sc->eps, sc->use_decay, sc->clip, sc->clip_mult};
  Peers p{};
  if (peers != nullptr) {
    p.n = peers->n;
    for (int q = 0; q < peers->n; ++q) p.delta[q] = peers->delta[q];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(n_chunks));
  const bool with_peers = peers != nullptr && p.n > 0;
  unsigned long long* cnt = d_changed_groups;
  if (param_dtype == HA_BF16) {
    if (with_peers) adamw_kernel<HA_BF16, true, true><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, s, p, cnt);
    else adamw_kernel<HA_BF16, false, true><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, s, p, cnt);
  } else {
    if (with_peers) adamw_kernel<HA_F16, true, true><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, s, p, cnt);
    else adamw_kernel<HA_F16, false, true><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, s, p, cnt);
  }
  return check_launch("adamw_kernel (delta)");
}

extern "C" int ha_scale_grads(const ha_tensor* d_tensors, const ha_chunk* d_chunks, int64_t n_chunks,
                              int64_t chunk_elems, int grad_dtype, float mult, void* stream) {
  HA_NVTX_RANGE();
  using namespace ha;
  if (chunk_elems != HA_ADAMW_CHUNK) return fail(HA_ERR_INVALID, "ha_scale_grads: chunk_elems must be %d", HA_ADAMW_CHUNK);
  if (!valid_float_dtype(grad_dtype)) return fail(HA_ERR_UNSUPPORTED, "ha_scale_grads: grad dtype %d", grad_dtype);
  if (n_chunks < 0 || n_chunks > 0x7fffffffLL) return fail(HA_ERR_INVALID, "ha_scale_grads: n_chunks %lld", (long long)n_chunks);
  if (n_chunks == 0) return HA_OK;
  if (d_tensors == nullptr || d_chunks == nullptr) return fail(HA_ERR_INVALID, "ha_scale_grads: NULL table");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(n_chunks));
  switch (grad_dtype) {
    case HA_F32: scale_kernel<HA_F32><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, mult); break;
    case HA_BF16: scale_kernel<HA_BF16><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, mult); break;
    default: scale_kernel<HA_F16><<<grid, kThreads, 0, st>>>(d_tensors, d_chunks, mult); break;
  }
  return check_launch("scale_kernel");
}
