// NCCL collectives of the ZeRO-1 step over NVLink 5 / NVSwitch.
//
// Replaces the reference's collectives (hybrid_rl/optimizer.py:105 used-mask MAX,
// :136 per-owner bucketed reduce, :153 norm SUM, :194 per-tensor broadcast) with one
// reduce-scatter and one all-gather over owner-major packed buffers plus two small
// all-reduces.  libnccl.so.2 is opened on first use, so the library loads (and its host
// helpers run) on machines without NCCL or a GPU; when torch has already loaded its
// NCCL, dlopen returns that same copy.
#include <dlfcn.h>

#include <cstring>
#include <mutex>
#include <string>

#include <cuda_runtime.h>
#include <nccl.h>

#include "hybridagent_b200.h"
#include "ha_nvtx.h"

namespace ha {
int fail(int code, const char* fmt, ...);
}

namespace {

// Entry points resolved from libnccl.so.2 with dlsym; the types come from nccl.h.
struct Nccl {
  decltype(&ncclGetUniqueId) GetUniqueId;
  decltype(&ncclCommInitRank) CommInitRank;
  decltype(&ncclCommDestroy) CommDestroy;
  decltype(&ncclCommAbort) CommAbort;
  decltype(&ncclReduceScatter) ReduceScatter;
  decltype(&ncclAllGather) AllGather;
  decltype(&ncclAllReduce) AllReduce;
  decltype(&ncclGetErrorString) GetErrorString;
  bool ok = false;
};

Nccl g_nccl;
std::once_flag g_nccl_once;
std::string g_nccl_error;

template <class F>
bool bind(void* h, const char* name, F* fn) {
  *fn = reinterpret_cast<F>(dlsym(h, name));
  return *fn != nullptr;
}

void load_nccl() {
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (h == nullptr) {
    const char* e = dlerror();
    g_nccl_error = e ? e : "dlopen(libnccl.so.2) failed";
    return;
  }
  bool ok = bind(h, "ncclGetUniqueId", &g_nccl.GetUniqueId) && bind(h, "ncclCommInitRank", &g_nccl.CommInitRank) &&
            bind(h, "ncclCommDestroy", &g_nccl.CommDestroy) && bind(h, "ncclCommAbort", &g_nccl.CommAbort) &&
            bind(h, "ncclReduceScatter", &g_nccl.ReduceScatter) &&
            bind(h, "ncclAllGather", &g_nccl.AllGather) && bind(h, "ncclAllReduce", &g_nccl.AllReduce) &&
            bind(h, "ncclGetErrorString", &g_nccl.GetErrorString);
  if (!ok) g_nccl_error = "libnccl.so.2 lacks an expected symbol";
  g_nccl.ok = ok;
}

int need_nccl() {
  std::call_once(g_nccl_once, load_nccl);
  if (!g_nccl.ok) return ha::fail(HA_ERR_NCCL, "NCCL unavailable: %s", g_nccl_error.c_str());
  return HA_OK;
}

int nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return HA_OK;
  return ha::fail(HA_ERR_NCCL, "%s: %s", what, g_nccl.GetErrorString(r));
}

bool nccl_type(int dtype, ncclDataType_t* out) {
  switch (dtype) {
    case HA_F32: *out = ncclFloat32; return true;
    case HA_BF16: *out = ncclBfloat16; return true;
    case HA_F16: *out = ncclFloat16; return true;
    case HA_F64: *out = ncclFloat64; return true;
    case HA_I32: *out = ncclInt32; return true;
    case HA_U8: *out = ncclUint8; return true;
    default: return false;
  }
}

}  // namespace

struct ha_comm {
  ncclComm_t comm;
  int world;
  int rank;
  bool aborted;
};

extern "C" int ha_comm_unique_id(uint8_t out[128]) {
  if (out == nullptr) return ha::fail(HA_ERR_INVALID, "ha_comm_unique_id: NULL");
  if (int rc = need_nccl()) return rc;
  ncclUniqueId id;
  if (int rc = nccl_status(g_nccl.GetUniqueId(&id), "ncclGetUniqueId")) return rc;
  std::memcpy(out, id.internal, 128);
  return HA_OK;
}

extern "C" int ha_comm_init(const uint8_t id[128], int32_t world, int32_t rank, ha_comm** out) {
  if (id == nullptr || out == nullptr || world < 1 || rank < 0 || rank >= world)
    return ha::fail(HA_ERR_INVALID, "ha_comm_init: bad arguments (world=%d rank=%d)", world, rank);
  if (int rc = need_nccl()) return rc;
  ncclUniqueId uid;
  std::memcpy(uid.internal, id, 128);
  ncclComm_t c = nullptr;
  if (int rc = nccl_status(g_nccl.CommInitRank(&c, world, uid, rank), "ncclCommInitRank")) return rc;
  *out = new ha_comm{c, world, rank, false};
  return HA_OK;
}

extern "C" int ha_comm_destroy(ha_comm* comm) {
  if (comm == nullptr) return HA_OK;
  int rc = HA_OK;
  if (g_nccl.ok && comm->comm != nullptr && !comm->aborted)
    rc = nccl_status(g_nccl.CommDestroy(comm->comm), "ncclCommDestroy");
  delete comm;
  return rc;
}

extern "C" int ha_comm_abort(ha_comm* comm) {
  if (comm == nullptr) return ha::fail(HA_ERR_INVALID, "ha_comm_abort: NULL");
  if (comm->aborted || comm->comm == nullptr || !g_nccl.ok) return HA_OK;
  comm->aborted = true;
  return nccl_status(g_nccl.CommAbort(comm->comm), "ncclCommAbort");
}

namespace {
int usable(ha_comm* comm, const char* what) {
  if (comm == nullptr) return ha::fail(HA_ERR_INVALID, "%s: NULL communicator", what);
  if (comm->aborted) return ha::fail(HA_ERR_NCCL, "%s: communicator was aborted", what);
  return HA_OK;
}
}  // namespace

extern "C" int ha_reduce_scatter(ha_comm* comm, const void* send, void* recv, size_t count, int dtype, void* stream) {
  HA_NVTX_RANGE();
  ncclDataType_t t;
  if (int rc = usable(comm, "ha_reduce_scatter")) return rc;
  if (!nccl_type(dtype, &t)) return ha::fail(HA_ERR_INVALID, "ha_reduce_scatter: bad arguments");
  return nccl_status(g_nccl.ReduceScatter(send, recv, count, t, ncclSum, comm->comm, static_cast<cudaStream_t>(stream)),
                     "ncclReduceScatter");
}

extern "C" int ha_all_gather(ha_comm* comm, const void* send, void* recv, size_t count, int dtype, void* stream) {
  HA_NVTX_RANGE();
  ncclDataType_t t;
  if (int rc = usable(comm, "ha_all_gather")) return rc;
  if (!nccl_type(dtype, &t)) return ha::fail(HA_ERR_INVALID, "ha_all_gather: bad arguments");
  return nccl_status(g_nccl.AllGather(send, recv, count, t, comm->comm, static_cast<cudaStream_t>(stream)),
                     "ncclAllGather");
}

extern "C" int ha_all_reduce_sum(ha_comm* comm, void* buf, size_t count, int dtype, void* stream) {
  HA_NVTX_RANGE();
  ncclDataType_t t;
  if (int rc = usable(comm, "ha_all_reduce_sum")) return rc;
  if (!nccl_type(dtype, &t)) return ha::fail(HA_ERR_INVALID, "ha_all_reduce_sum: bad arguments");
  return nccl_status(g_nccl.AllReduce(buf, buf, count, t, ncclSum, comm->comm, static_cast<cudaStream_t>(stream)),
                     "ncclAllReduce(sum)");
}

extern "C" int ha_all_reduce_max(ha_comm* comm, void* buf, size_t count, int dtype, void* stream) {
  HA_NVTX_RANGE();
  ncclDataType_t t;
  if (int rc = usable(comm, "ha_all_reduce_max")) return rc;
  if (!nccl_type(dtype, &t)) return ha::fail(HA_ERR_INVALID, "ha_all_reduce_max: bad arguments");
  return nccl_status(g_nccl.AllReduce(buf, buf, count, t, ncclMax, comm->comm, static_cast<cudaStream_t>(stream)),
                     "ncclAllReduce(max)");
}
