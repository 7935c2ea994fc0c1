// Host-side helpers shared by the C-ABI translation units: error reporting, SM count,
// and TMA descriptor encoding through the driver entry point (no link-time libcuda
// dependency, so the library also loads on machines without a GPU driver).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <string>
#include <utility>

#include "../../include/b200fp8.h"

namespace b2f {

void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);
int sm_count();
// Identifies the CUDA context current on this thread (0 when unknown).  Per-device caches
// of device addresses or function attributes compare it so that they are rebuilt after a
// cudaDeviceReset or a primary-context reset instead of handing out stale values.
unsigned long long context_token();

// Encode a 2-D (or 3-D) tiled tensor map for an 8- or 16-bit row-major tensor.
// dims/strides are innermost first; strides are in bytes for dims 1..rank-1.
bool encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                 const unsigned long long* dims, const unsigned long long* strides_bytes,
                 const unsigned int* box, CUtensorMapSwizzle swizzle, std::string* err);

// Launch with programmatic stream serialisation: the kernel may begin (its prologue up to
// pdl_wait()) while the previous kernel on the stream finishes, which hides the launch
// gap between the short kernels of a block.  Every kernel launched this way calls
// pdl_wait() before its first global-memory access.  B2F_NO_PDL=1 in the environment
// launches them plainly.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

#define B2F_CUDA_TRY(expr)                                   \
  do {                                                       \
    cudaError_t _e = (expr);                                 \
    if (_e != cudaSuccess) return ::b2f::cuda_fail(_e, #expr); \
  } while (0)

}  // namespace b2f
