// Per-tensor e4m3 quantisation of an activation (C ABI: b2f_quantize_fp8).
//
//   s = amax(|x|) / 448 (dynamic; 1 when x is all zero) or the caller's static scale
//   q = e4m3(x / s)   (IEEE division, round-to-nearest-even, saturating at +-448)
// This is the quantisation the reference applies to every FP8 operand it builds
// (e.g. `(source / scale).to(torch.float8_e4m3fn)` in
// tasks/level1_01_square_matrix_multiplication_fp8/starter.py:61-99 and the per-tensor amax
// scales of BASELINE's configs), done on the device so an FP8 GEMM can take f32 / bf16
// activations straight from the caller.
//
// Dynamic scale: pass 1 (grid-stride, 16-byte loads, block max, one atomic per CTA) reduces
// amax into a caller buffer; pass 2 re-reads x, divides by s and stores q.  With
// `scale_mul`, pass 2 also writes s * (*scale_mul) to `scale_prod_out`: the product of two
// operands' scales that a GEMM takes as its device-side alpha.
#include <algorithm>
#include <string>

#include "common.cuh"
#include "host_common.h"

namespace b2f {
namespace {

struct QuantParams {
  const void* x;
  int x_dtype;
  long long x_ld;
  uint8_t* q;
  long long q_ld;
  int rows, cols;
  float scale;  // static scale (amax == nullptr in pass 2)
  float* amax;
  float* scale_out;
  const float* scale_mul;
  float* scale_prod_out;
};

__device__ __forceinline__ void load8x(const void* base, int dt, long long off, float (&v)[8]) {
  if (dt == kBF16) {
    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + off);
    const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z),
                 d = unpack_bf16x2(u.w);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
  } else {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + off);
    const float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

template <int DT>
__global__ void __launch_bounds__(256) quant_amax_kernel(const QuantParams p) {
  __shared__ float red[8];
  const int vpr = p.cols / 8;
  const long long total = (long long)p.rows * vpr;
  float m = 0.f;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += (long long)gridDim.x * 256) {
    const long long r = i / vpr, v = i - r * vpr;
    float x[8];
    load8x(p.x, DT, r * p.x_ld + v * 8, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(x[j]));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = 0.f;
    for (int w = 0; w < 8; ++w) b = fmaxf(b, red[w]);
    atomic_max_nonneg(p.amax, b);
  }
}

template <int DT>
__global__ void __launch_bounds__(256) quant_apply_kernel(const QuantParams p) {
  float s = p.scale;
  if (p.amax != nullptr) {
    const float a = *p.amax;
    s = a > 0.f ? a / 448.0f : 1.0f;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (p.scale_out != nullptr) *p.scale_out = s;
    if (p.scale_prod_out != nullptr) *p.scale_prod_out = s * *p.scale_mul;
  }
  const int vpr = p.cols / 8;
  const long long total = (long long)p.rows * vpr;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += (long long)gridDim.x * 256) {
    const long long r = i / vpr, v = i - r * vpr;
    float x[8];
    load8x(p.x, DT, r * p.x_ld + v * 8, x);
    uint2 o;
    o.x = uint32_t(f32x2_to_e4m3x2(__fdiv_rn(x[0], s), __fdiv_rn(x[1], s))) |
          (uint32_t(f32x2_to_e4m3x2(__fdiv_rn(x[2], s), __fdiv_rn(x[3], s))) << 16);
    o.y = uint32_t(f32x2_to_e4m3x2(__fdiv_rn(x[4], s), __fdiv_rn(x[5], s))) |
          (uint32_t(f32x2_to_e4m3x2(__fdiv_rn(x[6], s), __fdiv_rn(x[7], s))) << 16);
    *reinterpret_cast<uint2*>(p.q + r * p.q_ld + v * 8) = o;
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace b2f

extern "C" {

void b2f_quant_args_init(b2f_quant_args* a) {
  if (a == nullptr) return;
  *a = b2f_quant_args{};
  a->x_dtype = B2F_DTYPE_F32;
  a->scale = 1.0f;
}

int b2f_quantize_fp8(const b2f_quant_args* a, b2f_stream_t stream) {
  using namespace b2f;
  if (a == nullptr) return fail(B2F_ERR_ARG, "quantize_fp8: null args");
  if (a->rows <= 0 || a->cols <= 0) return fail(B2F_ERR_ARG, "quantize_fp8: empty shape");
  if (a->cols % 8) return fail(B2F_ERR_ARG, "quantize_fp8: cols must be a multiple of 8");
  if (a->x == nullptr || a->q == nullptr) return fail(B2F_ERR_ARG, "quantize_fp8: null tensor");
  if (a->x_dtype != B2F_DTYPE_F32 && a->x_dtype != B2F_DTYPE_BF16)
    return fail(B2F_ERR_ARG, "quantize_fp8: x must be f32 or bf16");
  const int xs = a->x_dtype == B2F_DTYPE_F32 ? 4 : 2;
  if (!al16(a->x) || a->x_ld < a->cols || (a->x_ld * xs) % 16)
    return fail(B2F_ERR_ARG, "quantize_fp8: x layout (16-byte aligned rows)");
  if ((reinterpret_cast<uintptr_t>(a->q) & 7) || a->q_ld < a->cols || a->q_ld % 8)
    return fail(B2F_ERR_ARG, "quantize_fp8: q layout (8-byte aligned rows)");
  if (a->dynamic && (a->amax == nullptr || a->scale_out == nullptr))
    return fail(B2F_ERR_ARG, "quantize_fp8: dynamic scale needs amax and scale_out buffers");
  if (!a->dynamic && !(a->scale > 0.0f)) return fail(B2F_ERR_ARG, "quantize_fp8: scale must be > 0");
  if ((a->scale_mul == nullptr) != (a->scale_prod_out == nullptr))
    return fail(B2F_ERR_ARG, "quantize_fp8: scale_mul and scale_prod_out go together");
  QuantParams p;
  p.x = a->x; p.x_dtype = a->x_dtype; p.x_ld = a->x_ld;
  p.q = reinterpret_cast<uint8_t*>(a->q); p.q_ld = a->q_ld;
  p.rows = a->rows; p.cols = a->cols;
  p.scale = a->scale;
  p.amax = a->dynamic ? a->amax : nullptr;
  p.scale_out = a->scale_out;
  p.scale_mul = a->scale_mul; p.scale_prod_out = a->scale_prod_out;
  cudaStream_t s = (cudaStream_t)stream;
  const long long vecs = (long long)a->rows * (a->cols / 8);
  const int grid = (int)std::min<long long>((vecs + 255) / 256, (long long)sm_count() * 8);
  if (a->dynamic) {
    B2F_CUDA_TRY(cudaMemsetAsync(a->amax, 0, sizeof(float), s));
    if (a->x_dtype == B2F_DTYPE_F32) quant_amax_kernel<kF32><<<grid, 256, 0, s>>>(p);
    else quant_amax_kernel<kBF16><<<grid, 256, 0, s>>>(p);
    B2F_CUDA_TRY(cudaGetLastError());
  }
  if (a->x_dtype == B2F_DTYPE_F32) quant_apply_kernel<kF32><<<grid, 256, 0, s>>>(p);
  else quant_apply_kernel<kBF16><<<grid, 256, 0, s>>>(p);
  B2F_CUDA_TRY(cudaGetLastError());
  return B2F_OK;
}

}  // extern "C"
