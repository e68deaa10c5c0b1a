// Host-side helpers shared by the translation units of libsmm: error
// reporting (thread-local last-error text + status codes), launch counting,
// and the per-device status word the kernels write on a bounded-wait expiry.
#pragma once
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include "../../include/smm.h"

namespace smm {

// Records the failure text for smm_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
// Clears the last-error text (entry points call it on success paths).
void clear_error();
// Converts a CUDA error into SMM_ERR_CUDA with context.
int cuda_fail(cudaError_t e, const char* what);
// Counts one kernel launch issued by the library.
void count_launch(unsigned n = 1);
// Device address of this device's status word (sticky kernel error bits).
uint32_t* device_status_word();
// Wait limit handed to the pipelined kernels (ns); SMM_WAIT_LIMIT_MS overrides.
unsigned long long wait_limit_ns();

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Names one library call on profiler timelines (an NVTX range, header-only
// NVTX v3: a no-op unless a profiling tool is attached).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};
#define SMM_RANGE(name) ::smm::NvtxRange smm_nvtx_range_(name)

#define SMM_CUDA_TRY(expr, what)                  \
  do {                                            \
    cudaError_t _e = (expr);                      \
    if (_e != cudaSuccess) return ::smm::cuda_fail(_e, what); \
  } while (0)

}  // namespace smm
