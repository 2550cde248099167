// NVTX ranges over the library's entry points: every call that launches work shows up by
// name (ha_adamw_step, ha_gather, ...) on the CPU timeline of Nsight Systems and as the
// enclosing range of its kernels in Nsight Compute.  NVTX v3 is header-only; without an
// attached tool each push / pop is a check of one function pointer.
#pragma once

#include <nvtx3/nvToolsExt.h>

namespace ha {

class NvtxRange {
 public:
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

}  // namespace ha

// One range named after the enclosing entry point, for the rest of its scope.
#define HA_NVTX_RANGE() ::ha::NvtxRange ha_nvtx_range_(__func__)
