// Host-side half of the C ABI: error reporting, ownership, chunk planning and the fp32
// scalars of each step.  Needs no GPU; built with -ffp-contract=off so the double
// arithmetic matches CPython's (hybrid_rl/optimizer.py computes these in Python floats).
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <functional>
#include <numeric>
#include <queue>
#include <string>
#include <utility>
#include <vector>

#include <cuda_runtime.h>

#include "hybridagent_b200.h"

namespace ha {

namespace {
thread_local std::string g_error;
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(HA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return HA_OK;
}

}  // namespace ha

extern "C" const char* ha_last_error(void) { return ha::g_error.c_str(); }

extern "C" int ha_abi_version(void) { return 1; }

extern "C" int ha_greedy_owners(int64_t n, const int64_t* numels, int32_t world, int32_t* owner_out) {
  using ha::fail;
  if (n < 0 || world < 1) return fail(HA_ERR_INVALID, "ha_greedy_owners: n=%lld world=%d", (long long)n, world);
  if (n > 0 && (numels == nullptr || owner_out == nullptr)) return fail(HA_ERR_INVALID, "ha_greedy_owners: NULL");
  std::vector<int64_t> order(static_cast<size_t>(n));
  std::iota(order.begin(), order.end(), 0);
  // largest first; equal sizes keep list order (Python's sorted is stable)
  std::stable_sort(order.begin(), order.end(), [&](int64_t a, int64_t b) { return numels[a] > numels[b]; });
  // least-loaded rank, ties to the lowest rank: a min-heap on (load, rank)
  using Slot = std::pair<int64_t, int32_t>;
  std::priority_queue<Slot, std::vector<Slot>, std::greater<Slot>> heap;
  for (int32_t r = 0; r < world; ++r) heap.push({0, r});
  for (const int64_t i : order) {
    Slot s = heap.top();
    heap.pop();
    owner_out[i] = s.second;
    s.first += numels[i];
    heap.push(s);
  }
  return HA_OK;
}

extern "C" int ha_plan_chunks(int64_t n_tensors, const int64_t* numels, const uint8_t* include, int64_t chunk_elems,
                              ha_chunk* out, int64_t cap, int64_t* n_out) {
  using ha::fail;
  if (n_tensors < 0 || chunk_elems <= 0 || n_out == nullptr || (n_tensors > 0 && numels == nullptr) ||
      n_tensors > 0xffffffffLL)
    return fail(HA_ERR_INVALID, "ha_plan_chunks: bad arguments");
  int64_t k = 0;
  for (int64_t i = 0; i < n_tensors; ++i) {
    if (include != nullptr && include[i] == 0) continue;
    if (numels[i] < 0) return fail(HA_ERR_INVALID, "ha_plan_chunks: numel[%lld] < 0", (long long)i);
    const int64_t nc = (numels[i] + chunk_elems - 1) / chunk_elems;
    if (nc > 0xffffffffLL) return fail(HA_ERR_INVALID, "ha_plan_chunks: tensor %lld too large", (long long)i);
    for (int64_t c = 0; c < nc; ++c, ++k) {
      if (out != nullptr && k < cap) out[k] = ha_chunk{static_cast<uint32_t>(i), static_cast<uint32_t>(c)};
    }
  }
  *n_out = k;
  return HA_OK;
}

extern "C" int ha_check_chunks(int64_t n_tensors, const int64_t* numels, const ha_chunk* chunks, int64_t n_chunks,
                               int64_t chunk_elems) {
  using ha::fail;
  if (n_chunks < 0 || chunk_elems <= 0 || (n_chunks > 0 && chunks == nullptr) || (n_tensors > 0 && numels == nullptr))
    return fail(HA_ERR_INVALID, "ha_check_chunks: bad arguments");
  for (int64_t k = 0; k < n_chunks; ++k) {
    const ha_chunk c = chunks[k];
    if (static_cast<int64_t>(c.tensor) >= n_tensors)
      return fail(HA_ERR_INVALID, "chunk %lld: tensor %u out of range (%lld tensors)", (long long)k, c.tensor,
                  (long long)n_tensors);
    if (static_cast<int64_t>(c.index) * chunk_elems >= numels[c.tensor])
      return fail(HA_ERR_INVALID, "chunk %lld: start %lld beyond numel %lld of tensor %u", (long long)k,
                  (long long)(static_cast<int64_t>(c.index) * chunk_elems), (long long)numels[c.tensor], c.tensor);
  }
  return HA_OK;
}

extern "C" int ha_fill_step_scalars(int64_t n, const double* lrs, const int64_t* steps, double beta1, double beta2,
                                    double weight_decay, ha_tensor* table) {
  using ha::fail;
  if (n < 0 || (n > 0 && (lrs == nullptr || steps == nullptr || table == nullptr)))
    return fail(HA_ERR_INVALID, "ha_fill_step_scalars: bad arguments");
  for (int64_t i = 0; i < n; ++i) {
    const double lr = lrs[i];
    // optimizer.py:182-183: correction = 1.0 - beta ** param_steps (CPython float ** int -> pow)
    const double c1 = 1.0 - std::pow(beta1, static_cast<double>(steps[i]));
    const double c2 = 1.0 - std::pow(beta2, static_cast<double>(steps[i]));
    table[i].decay = static_cast<float>(1.0 - lr * weight_decay);  // optimizer.py:185
    table[i].neg_lr = static_cast<float>(-lr);                     // optimizer.py:189 value=-lr
    // torch's CUDA `tensor / python_float` multiplies by the divisor's reciprocal taken
    // in double and rounded to fp32 once (measured on B200 for every step count)
    table[i].rc1 = static_cast<float>(1.0 / c1);
    table[i].rc2 = static_cast<float>(1.0 / c2);
  }
  return HA_OK;
}

extern "C" int ha_make_scalars(double beta1, double beta2, double eps, double weight_decay, int grad_dtype, int clip,
                               double clip_scale, ha_adamw_scalars* out) {
  using ha::fail;
  if (out == nullptr) return fail(HA_ERR_INVALID, "ha_make_scalars: NULL output");
  if (grad_dtype != HA_F32 && grad_dtype != HA_BF16 && grad_dtype != HA_F16)
    return fail(HA_ERR_UNSUPPORTED, "ha_make_scalars: grad dtype %d", grad_dtype);
  out->b1 = static_cast<float>(beta1);
  out->a1 = static_cast<float>(1.0 - beta1);
  out->b2 = static_cast<float>(beta2);
  out->a2 = static_cast<float>(1.0 - beta2);
  out->eps = static_cast<float>(eps);
  out->use_decay = weight_decay != 0.0 ? 1 : 0;
  out->clip = clip ? 1 : 0;
  out->clip_mult = clip ? static_cast<float>(clip_scale) : 1.0f;
  return HA_OK;
}
