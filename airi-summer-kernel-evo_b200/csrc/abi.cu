// C-ABI plumbing: version, thread-local error messages, the device status word, the op
// registry and TMA descriptor encoding.
#include <mutex>
#include <string>
#include <vector>
#include <cstring>
#include <cstdlib>

#include "common.cuh"
#include "host_common.h"

namespace b2f {

__device__ unsigned int g_b2f_status = 0;

namespace {
thread_local std::string t_last_error;
std::mutex g_mu;
std::vector<int> g_sm_cache;  // per-device SM count, -1 = unknown

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn g_ctx_get = nullptr;
}  // namespace

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("B2F_NO_PDL");
    return !(e != nullptr && e[0] != '\0' && e[0] != '0');
  }();
  return on;
}

unsigned long long context_token() {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_ctx_get == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 12000, cudaEnableDefault,
                                           &q) != cudaSuccess ||
          fn == nullptr || q != cudaDriverEntryPointSuccess)
        return 0;
      g_ctx_get = reinterpret_cast<CtxGetCurrentFn>(fn);
    }
  }
  CUcontext c = nullptr;
  if (g_ctx_get(&c) != CUDA_SUCCESS) return 0;
  return reinterpret_cast<unsigned long long>(c);
}

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  set_error(std::string(what) + ": " + cudaGetErrorString(e));
  return B2F_ERR_CUDA;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  std::lock_guard<std::mutex> lk(g_mu);
  if ((int)g_sm_cache.size() <= dev) g_sm_cache.resize(dev + 1, -1);
  if (g_sm_cache[dev] < 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    g_sm_cache[dev] = n;
  }
  return g_sm_cache[dev];
}

bool encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                 const unsigned long long* dims, const unsigned long long* strides_bytes,
                 const unsigned int* box, CUtensorMapSwizzle swizzle, std::string* err) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_encode == nullptr) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e =
          cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
      if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess) {
        *err = "cuTensorMapEncodeTiled entry point unavailable";
        return false;
      }
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
  }
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) s[i] = strides_bytes[i];
  CUresult r = g_encode(map, dtype, rank, const_cast<void*>(base), d, s, b, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r);
    return false;
  }
  return true;
}

// Waits on a barrier nothing arrives on, with a caller-given limit; exercises the
// bounded-wait / status-word path without faulting the GPU.
__global__ void debug_bounded_wait_kernel(unsigned long long wait_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer();
    while (!mbar_test(&bar, 0)) {
      if (globaltimer() - t0 > wait_ns) {
        record_error(kDevTimeoutEpilogue);
        break;
      }
    }
  }
}

}  // namespace b2f


namespace {
const b2f_op g_ops[] = {
    {"gemm_fp8", B2F_ABI_VERSION, (void*)&b2f_gemm_fp8, "b2f_gemm_args"},
    {"norm_quant", B2F_ABI_VERSION, (void*)&b2f_norm_quant, "b2f_norm_args"},
    {"attention_fp8", B2F_ABI_VERSION, (void*)&b2f_attention_fp8, "b2f_attn_args"},
    {"head_norm_rope", B2F_ABI_VERSION, (void*)&b2f_head_norm_rope, "b2f_rope_args"},
    {"swiglu_fp8", B2F_ABI_VERSION, (void*)&b2f_swiglu_fp8, "(gate, gate_ld, up, up_ld, out, out_ld, rows, cols, in_scale, out_scale)"},
    {"fp8_to_bf16", B2F_ABI_VERSION, (void*)&b2f_fp8_to_bf16, "(in, in_ld, out, out_ld, rows, cols, scale)"},
    {"fp8_to_f16", B2F_ABI_VERSION, (void*)&b2f_fp8_to_f16, "(in, in_ld, out, out_ld, rows, cols, scale)"},
    {"gpt2_block", B2F_ABI_VERSION, (void*)&b2f_gpt2_block, "b2f_gpt2_block_args"},
    {"qwen_block", B2F_ABI_VERSION, (void*)&b2f_qwen_block, "b2f_qwen_block_args"},
    {"quantize_fp8", B2F_ABI_VERSION, (void*)&b2f_quantize_fp8, "b2f_quant_args"},
    {"layer_norm_rows", B2F_ABI_VERSION, (void*)&b2f_layer_norm_rows, "b2f_lnrows_args"},
};
}

extern "C" {

int b2f_version(void) { return B2F_ABI_VERSION; }

const char* b2f_last_error(void) { return b2f::t_last_error.c_str(); }

int b2f_num_sms(void) { return b2f::sm_count(); }

int b2f_status_read(int reset) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, b2f::g_b2f_status, sizeof(v)) != cudaSuccess) return -1;
  if (reset) {
    unsigned int z = 0;
    if (cudaMemcpyToSymbol(b2f::g_b2f_status, &z, sizeof(z)) != cudaSuccess) return -1;
  }
  return (int)v;
}

int b2f_debug_bounded_wait(unsigned long long wait_ns, b2f_stream_t stream) {
  b2f::debug_bounded_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(wait_ns);
  B2F_CUDA_TRY(cudaGetLastError());
  return B2F_OK;
}

const b2f_op* b2f_registry_lookup(const char* name) {
  if (name == nullptr) return nullptr;
  for (const b2f_op& op : g_ops)
    if (std::strcmp(op.name, name) == 0) return &op;
  return nullptr;
}

int b2f_registry_size(void) { return (int)(sizeof(g_ops) / sizeof(g_ops[0])); }

const b2f_op* b2f_registry_at(int index) {
  if (index < 0 || index >= b2f_registry_size()) return nullptr;
  return &g_ops[index];
}

}  // extern "C"
