// Residual-add + RMSNorm / LayerNorm + e4m3 quantisation (C ABI: b2f_norm_quant).
//
// A group of up to 256 threads owns one row (4 vectors of 8 elements per thread, coalesced
// 16-byte-per-lane sweeps), keeps the whole row in registers, reduces with warp shuffles
// (plus shared memory across the warps of a row) and writes every output in one pass:
//   h   = x * x_scale + residual                (updated residual stream, optional store)
//   y   = RMSNorm(h) * (w + w_offset)           (w_offset = 1 for Qwen's (1 + w))
//       | LayerNorm(h) * w + b
//   q   = e4m3(y / s)
// Static scale s (the block tasks' fixed NORM_SCALE) is one HBM pass.  Dynamic
// per-tensor scale s = amax(|y|)/448 needs the global max before
// quantising: pass 1 writes h and reduces amax, pass 2 re-reads h (rows in reverse
// order, so the most recently written rows still sit in L2), recomputes y and quantises.
// No scratch memory: the statistics are recomputed from h in pass 2.
//
// Reference math: residual RMSNorm cute_kernels/fused_residual_rmsnorm_fp8/submission.py:139-145,
// Qwen RMSNorm tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:167-171,
// GPT-2 LayerNorm tasks/model_gpt2_small_transformer_block_fp8/starter.py:407-416,461-470.
#include <string>

#include "common.cuh"
#include "host_common.h"

namespace b2f {

namespace {

constexpr int kMaxCols = 8192;  // 256 threads x 4 vectors x 8 elements

struct NormParams {
  const void* x;
  int x_dtype;
  float x_scale;
  long long x_ld;
  const void* residual;
  int res_dtype;
  long long res_ld;
  const void* weight;
  const void* bias;
  int w_dtype;
  float w_offset;
  int kind;  // 0 RMS, 1 LayerNorm
  float eps;
  void* h_out;
  int h_dtype;
  long long h_ld;
  void* y_out;  // optional bf16 normalised output
  long long y_ld;
  uint8_t* q_out;
  long long q_ld;
  float q_scale;  // static scale (dynamic == 0)
  int dynamic;
  float* amax;       // dynamic: amax accumulator (zeroed by the launcher)
  float* scale_out;  // dynamic: s = amax/448 written by pass 2
  int rows, cols;
};

__device__ __forceinline__ void load8(const void* base, int dtype, long long off, float scale,
                                      float (&v)[8]) {
  if (dtype == kBF16) {
    uint4 q = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + off);
    float2 a = unpack_bf16x2(q.x), b = unpack_bf16x2(q.y), c = unpack_bf16x2(q.z),
           d = unpack_bf16x2(q.w);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
  } else if (dtype == kF32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + off);
    float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    uint2 q = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(base) + off);
    float2 a = e4m3x2_to_f32x2(q.x & 0xFFFF), b = e4m3x2_to_f32x2(q.x >> 16),
           c = e4m3x2_to_f32x2(q.y & 0xFFFF), d = e4m3x2_to_f32x2(q.y >> 16);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
  }
  if (scale != 1.0f) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] *= scale;
  }
}

__device__ __forceinline__ void store8(void* base, int dtype, long long off, const float (&v)[8]) {
  if (dtype == kBF16) {
    uint4 q;
    q.x = pack_bf16x2(v[0], v[1]); q.y = pack_bf16x2(v[2], v[3]);
    q.z = pack_bf16x2(v[4], v[5]); q.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + off) = q;
  } else {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + off);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

__device__ __forceinline__ void round_bf16(float (&v)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(v[j]));
}

__device__ __forceinline__ uint2 quant8(const float (&y)[8], float inv) {
  uint2 r;
  r.x = uint32_t(f32x2_to_e4m3x2(y[0] * inv, y[1] * inv)) |
        (uint32_t(f32x2_to_e4m3x2(y[2] * inv, y[3] * inv)) << 16);
  r.y = uint32_t(f32x2_to_e4m3x2(y[4] * inv, y[5] * inv)) |
        (uint32_t(f32x2_to_e4m3x2(y[6] * inv, y[7] * inv)) << 16);
  return r;
}

// ---------------------------------------------------------------------------------------
// Row layout: a group of TPR threads (a multiple of 32) owns one row; thread t of the group
// holds vectors vi = t + TPR * i (i < 4) of 8 elements, so each i is one coalesced
// 16-byte-per-lane sweep.  All loads of a row are issued before any store (the stored
// residual stream may alias nothing the kernel still has to read), and the dtype switch
// sits outside the load loop so the loads issue back to back.
constexpr int VPT = 4;  // vectors of 8 elements per thread

template <int DT>
__device__ __forceinline__ void load4(const void* __restrict__ base, long long row_off, int t,
                                      int tpr, int nvec, float scale, float (&v)[VPT][8]) {
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = t + tpr * i;
    if (vi < nvec) {
      load8(base, DT, row_off + (long long)vi * 8, scale, v[i]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
    }
  }
}

__device__ __forceinline__ void load_any(const void* base, int dt, long long row_off, int t,
                                         int tpr, int nvec, float scale, float (&v)[VPT][8]) {
  switch (dt) {
    case kBF16: load4<kBF16>(base, row_off, t, tpr, nvec, scale, v); break;
    case kF32: load4<kF32>(base, row_off, t, tpr, nvec, scale, v); break;
    default: load4<kE4M3>(base, row_off, t, tpr, nvec, scale, v); break;
  }
}

// Sum over the TPR threads of a row group (every thread of the CTA must call it).
__device__ __forceinline__ float group_sum(float v, float* red, int tpr) {
  v = warp_sum(v);
  const int wpr = tpr >> 5;
  if (wpr == 1) return v;
  const int warp = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  const int g0 = (warp / wpr) * wpr;
  float s = 0.f;
  for (int w = 0; w < wpr; ++w) s += red[g0 + w];
  return s;
}

// h = x * x_scale + residual (rounded to the stored residual dtype), optional store of h,
// then the row statistics.
__device__ __forceinline__ void row_stats(const NormParams& p, const void* x, int xdt, float xs,
                                          long long xld, const void* res, bool store_h,
                                          int row, bool row_ok, int t, int tpr, int nvec,
                                          float* red, float (&h)[VPT][8], float& mean,
                                          float& inv) {
  const long long r = row_ok ? row : 0;
  load_any(x, xdt, r * xld, t, tpr, nvec, xs, h);
  if (res != nullptr) {
    float rv[VPT][8];
    load_any(res, p.res_dtype, r * p.res_ld, t, tpr, nvec, 1.0f, rv);
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) h[i][j] += rv[i][j];
  }
  if (p.h_out != nullptr && p.h_dtype == kBF16) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) round_bf16(h[i]);
  }
  if (store_h && row_ok && p.h_out != nullptr) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = t + tpr * i;
      if (vi < nvec) store8(p.h_out, p.h_dtype, r * p.h_ld + (long long)vi * 8, h[i]);
    }
  }
  const float n = float(p.cols);
  float s1 = 0.f, s2 = 0.f;
  if (p.kind == 1) {
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) s1 += h[i][j];
    mean = group_sum(s1, red, tpr) / n;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      if (t + tpr * i < nvec) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float d = h[i][j] - mean;
          s2 += d * d;
        }
      }
    }
  } else {
    mean = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) s2 += h[i][j] * h[i][j];
  }
  inv = rsqrtf(group_sum(s2, red, tpr) / n + p.eps);
}

__device__ __forceinline__ void norm8(const NormParams& p, int col, float mean, float inv,
                                      const float (&h)[8], float (&y)[8]) {
  float w[8];
  load8(p.weight, p.w_dtype, col, 1.0f, w);
  if (p.kind == 1) {
    float b[8];
    if (p.bias != nullptr) {
      load8(p.bias, p.w_dtype, col, 1.0f, b);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = (h[j] - mean) * inv * w[j] + b[j];
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = h[j] * inv * (w[j] + p.w_offset);
  }
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
  return m;
}

// Static scale (one pass), or pass 1 of the dynamic schedule (no q store; amax reduce).
__global__ void __launch_bounds__(256) norm_pass1_kernel(const NormParams p, int tpr) {
  __shared__ float red[8];
  const int rpc = blockDim.x / tpr;
  const int t = threadIdx.x % tpr;
  const int row = blockIdx.x * rpc + threadIdx.x / tpr;
  const bool row_ok = row < p.rows;
  const int nvec = p.cols / 8;
  float h[VPT][8];
  float mean, inv;
  row_stats(p, p.x, p.x_dtype, p.x_scale, p.x_ld, p.residual, true, row, row_ok, t, tpr, nvec,
            red, h, mean, inv);
  const float qinv = 1.0f / p.q_scale;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = t + tpr * i;
    if (row_ok && vi < nvec) {
      float y[8];
      norm8(p, vi * 8, mean, inv, h[i], y);
      if (p.dynamic) {
        round_bf16(y);
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(y[j]));
      } else {
        // Quantise the f32 value (as the reference's `(y / scale).to(e4m3)`); the
        // optional bf16 copy is rounded separately.
        *reinterpret_cast<uint2*>(p.q_out + (long long)row * p.q_ld + vi * 8) = quant8(y, qinv);
        if (p.y_out != nullptr) {
          round_bf16(y);
          store8(p.y_out, kBF16, (long long)row * p.y_ld + vi * 8, y);
        }
      }
    }
  }
  if (p.dynamic) {
    const float m = block_max(amax, red);
    if (threadIdx.x == 0) atomic_max_nonneg(p.amax, m);
  }
}

// Pass 2 of the dynamic schedule: row blocks in reverse order (the most recently written
// h rows are still in L2), h re-read, statistics recomputed, quantised with amax / 448.
__global__ void __launch_bounds__(256) norm_pass2_kernel(const NormParams p, int tpr) {
  __shared__ float red[8];
  const int rpc = blockDim.x / tpr;
  const int t = threadIdx.x % tpr;
  const int row = (gridDim.x - 1 - blockIdx.x) * rpc + threadIdx.x / tpr;
  const bool row_ok = row < p.rows;
  const float amax = *p.amax;
  const float s = amax > 0.f ? amax / 448.0f : 1.0f;
  if (blockIdx.x == 0 && threadIdx.x == 0) *p.scale_out = s;
  const int nvec = p.cols / 8;
  float h[VPT][8];
  float mean, inv;
  NormParams q = p;
  q.h_out = nullptr;
  if (p.h_out != nullptr)
    row_stats(q, p.h_out, p.h_dtype, 1.0f, p.h_ld, nullptr, false, row, row_ok, t, tpr, nvec,
              red, h, mean, inv);
  else
    row_stats(q, p.x, p.x_dtype, p.x_scale, p.x_ld, p.residual, false, row, row_ok, t, tpr,
              nvec, red, h, mean, inv);
  const float qinv = 1.0f / s;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = t + tpr * i;
    if (row_ok && vi < nvec) {
      float y[8];
      norm8(p, vi * 8, mean, inv, h[i], y);
      round_bf16(y);
      if (p.y_out != nullptr) store8(p.y_out, kBF16, (long long)row * p.y_ld + vi * 8, y);
      *reinterpret_cast<uint2*>(p.q_out + (long long)row * p.q_ld + vi * 8) = quant8(y, qinv);
    }
  }
}

int launch_norm(const NormParams& p, cudaStream_t s) {
  const int nvec = p.cols / 8;
  int tpr = ((nvec + VPT - 1) / VPT + 31) / 32 * 32;  // threads per row
  const int rpc = 256 / tpr;                            // rows per CTA
  const int threads = rpc * tpr;
  const int grid = (p.rows + rpc - 1) / rpc;
  if (p.dynamic) {
    B2F_CUDA_TRY(cudaMemsetAsync(p.amax, 0, sizeof(float), s));
    norm_pass1_kernel<<<grid, threads, 0, s>>>(p, tpr);
    B2F_CUDA_TRY(cudaGetLastError());
    norm_pass2_kernel<<<grid, threads, 0, s>>>(p, tpr);
  } else {
    norm_pass1_kernel<<<grid, threads, 0, s>>>(p, tpr);
  }
  B2F_CUDA_TRY(cudaGetLastError());
  return B2F_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace b2f

extern "C" {

void b2f_norm_args_init(b2f_norm_args* a) {
  if (a == nullptr) return;
  *a = b2f_norm_args{};
  a->x_dtype = B2F_DTYPE_BF16;
  a->x_scale = 1.0f;
  a->residual_dtype = B2F_DTYPE_BF16;
  a->weight_dtype = B2F_DTYPE_BF16;
  a->kind = B2F_NORM_RMS;
  a->eps = 1e-6f;
  a->h_dtype = B2F_DTYPE_BF16;
  a->q_scale = 1.0f;
}

int b2f_norm_quant(const b2f_norm_args* a, b2f_stream_t stream) {
  using namespace b2f;
  if (a == nullptr) return fail(B2F_ERR_ARG, "norm_quant: null args");
  if (a->rows <= 0 || a->cols <= 0) return fail(B2F_ERR_ARG, "norm_quant: empty shape");
  if (a->cols % 8 != 0) return fail(B2F_ERR_ARG, "norm_quant: cols must be a multiple of 8");
  if (a->cols > kMaxCols)
    return fail(B2F_ERR_UNSUPPORTED, "norm_quant: cols > 8192 not supported");
  if (a->x == nullptr || a->weight == nullptr || a->q_out == nullptr)
    return fail(B2F_ERR_ARG, "norm_quant: null tensor");
  if (a->kind != B2F_NORM_RMS && a->kind != B2F_NORM_LAYER)
    return fail(B2F_ERR_ARG, "norm_quant: bad kind");
  if (a->x_dtype < 0 || a->x_dtype > 2 || a->residual_dtype < 0 || a->residual_dtype > 1 ||
      a->weight_dtype < 0 || a->weight_dtype > 1 || a->h_dtype < 0 || a->h_dtype > 1)
    return fail(B2F_ERR_ARG, "norm_quant: bad dtype");
  if (a->dynamic_scale && (a->amax == nullptr || a->scale_out == nullptr))
    return fail(B2F_ERR_ARG, "norm_quant: dynamic scale needs amax and scale_out buffers");
  if (!a->dynamic_scale && !(a->q_scale > 0.0f))
    return fail(B2F_ERR_ARG, "norm_quant: q_scale must be > 0");
  const int xs = a->x_dtype == B2F_DTYPE_F32 ? 4 : (a->x_dtype == B2F_DTYPE_BF16 ? 2 : 1);
  if (!al16(a->x) || (a->x_ld * xs) % 16 || a->x_ld < a->cols) return fail(B2F_ERR_ARG, "norm_quant: x layout");
  if (a->residual && (!al16(a->residual) || a->residual_ld < a->cols || (a->residual_ld * 2) % 16))
    return fail(B2F_ERR_ARG, "norm_quant: residual layout");
  if (a->h_out && (!al16(a->h_out) || a->h_ld < a->cols || (a->h_ld * 2) % 16))
    return fail(B2F_ERR_ARG, "norm_quant: h_out layout");
  if (a->y_out && (!al16(a->y_out) || a->y_ld < a->cols || (a->y_ld * 2) % 16))
    return fail(B2F_ERR_ARG, "norm_quant: y_out layout");
  if ((((uintptr_t)a->q_out) & 7) || a->q_ld < a->cols || a->q_ld % 8) return fail(B2F_ERR_ARG, "norm_quant: q_out layout");
  if (!al16(a->weight) || (a->bias && !al16(a->bias))) return fail(B2F_ERR_ARG, "norm_quant: weight alignment");
  NormParams p;
  p.x = a->x; p.x_dtype = a->x_dtype; p.x_scale = a->x_scale; p.x_ld = a->x_ld;
  p.residual = a->residual; p.res_dtype = a->residual_dtype; p.res_ld = a->residual_ld;
  p.weight = a->weight; p.bias = a->bias; p.w_dtype = a->weight_dtype; p.w_offset = a->weight_offset;
  p.kind = a->kind; p.eps = a->eps;
  p.h_out = a->h_out; p.h_dtype = a->h_dtype; p.h_ld = a->h_ld;
  p.y_out = a->y_out; p.y_ld = a->y_ld;
  p.q_out = reinterpret_cast<uint8_t*>(a->q_out); p.q_ld = a->q_ld;
  p.q_scale = a->q_scale; p.dynamic = a->dynamic_scale;
  p.amax = a->amax; p.scale_out = a->scale_out;
  p.rows = a->rows; p.cols = a->cols;
  cudaStream_t s = (cudaStream_t)stream;
  return launch_norm(p, s);
}

}  // extern "C"
