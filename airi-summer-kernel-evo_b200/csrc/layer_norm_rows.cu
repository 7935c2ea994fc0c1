// LayerNorm of a few very long rows, split over many CTAs (C ABI: b2f_layer_norm_rows).
//
//   y[r, :] = (x[r, :] * x_scale - mean_r) * rsqrt(var_r + eps) [* w + b]
//
// The reference task level1_40 normalises 16 rows of 4,194,304 e4m3 values each
// (tasks/level1_40_layer_norm_fp8/starter.py:84-166: x = stored / 448, F.layer_norm over the
// whole row, eps 1e-5, f32 output); its CuTe submission gives each row to one CTA
// (cute_kernels/level1_40_layer_norm_fp8/submission.py:71-134), which occupies 16 of the
// 148 SMs.  Here every row is cut into chunks so the whole GPU streams it:
//   pass 1  one CTA per (row, chunk): f32 sum and sum of squares of the chunk from 16-byte
//           vector loads, one f64 pair per chunk to the caller's workspace;
//   pass 2  one CTA per (row, chunk): the row's chunk pairs are combined in f64 (mean, var),
//           then the chunk is re-read (an e4m3 row block of 64 KB is still in L2) and
//           written normalised with 16-byte stores.
// HBM-bound: compulsory bytes = rows * cols * (in_esize + out_esize).
#include <cstdint>
#include <string>

#include "common.cuh"
#include "host_common.h"

namespace b2f {
namespace {

constexpr int kLnThreads = 256;
constexpr int kLnVec = 16;                       // elements per thread per step
constexpr int kLnChunk = kLnThreads * kLnVec * 16;  // 65536 elements per CTA

// 16 consecutive elements as f32 (x_scale applied).
template <int XT>
__device__ __forceinline__ void ln_load16(const uint8_t* p, float x_scale, float (&v)[16]) {
  if constexpr (XT == B2F_DTYPE_E4M3) {
    const uint4 q = __ldcs(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 a = e4m3x2_to_f32x2(uint16_t(w[i] & 0xFFFF));
      const float2 b = e4m3x2_to_f32x2(uint16_t(w[i] >> 16));
      v[4 * i] = a.x * x_scale; v[4 * i + 1] = a.y * x_scale;
      v[4 * i + 2] = b.x * x_scale; v[4 * i + 3] = b.y * x_scale;
    }
  } else if constexpr (XT == B2F_DTYPE_BF16) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 q = __ldcs(reinterpret_cast<const uint4*>(p) + h);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = unpack_bf16x2(w[i]);
        v[8 * h + 2 * i] = a.x * x_scale;
        v[8 * h + 2 * i + 1] = a.y * x_scale;
      }
    }
  } else {
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float4 q = __ldcs(reinterpret_cast<const float4*>(p) + h);
      v[4 * h] = q.x * x_scale; v[4 * h + 1] = q.y * x_scale;
      v[4 * h + 2] = q.z * x_scale; v[4 * h + 3] = q.w * x_scale;
    }
  }
}

template <int XT>
__device__ __forceinline__ float ln_load1(const uint8_t* row, long long c, float x_scale) {
  if constexpr (XT == B2F_DTYPE_E4M3) return e4m3_to_f32(row[c]) * x_scale;
  else if constexpr (XT == B2F_DTYPE_BF16)
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[c]) * x_scale;
  else return reinterpret_cast<const float*>(row)[c] * x_scale;
}

constexpr int esize(int dt) { return dt == B2F_DTYPE_F32 ? 4 : (dt == B2F_DTYPE_BF16 ? 2 : 1); }

struct LnRowsParams {
  const uint8_t* x;
  long long x_ld;  // elements
  float x_scale;
  int rows;
  long long cols;
  int chunks;      // CTAs per row
  const float* w;
  const float* b;
  float eps;
  void* out;
  long long out_ld;
  double* partial;  // [rows][chunks][2]: sum, sum of squares
};

__device__ __forceinline__ double block_sum_f64(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x < 32) {
    t = lane < (kLnThreads / 32) ? red[lane] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  return t;  // valid in thread 0
}

template <int XT, bool VEC>
__global__ void __launch_bounds__(kLnThreads)
    ln_rows_stats_kernel(const LnRowsParams p) {
  __shared__ double red[2][kLnThreads / 32];
  const int r = blockIdx.y;
  const long long c0 = (long long)blockIdx.x * kLnChunk;
  const long long c1 = c0 + kLnChunk < p.cols ? c0 + kLnChunk : p.cols;
  const uint8_t* row = p.x + (long long)r * p.x_ld * esize(XT);
  float s = 0.f, s2 = 0.f;
  if (VEC) {
    for (long long c = c0 + (long long)threadIdx.x * kLnVec; c < c1; c += kLnThreads * kLnVec) {
      if (c + kLnVec <= c1) {
        float v[16];
        ln_load16<XT>(row + c * esize(XT), p.x_scale, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) { s += v[i]; s2 = fmaf(v[i], v[i], s2); }
      } else {
        for (long long e = c; e < c1; ++e) {
          const float v = ln_load1<XT>(row, e, p.x_scale);
          s += v; s2 = fmaf(v, v, s2);
        }
      }
    }
  } else {
    for (long long e = c0 + threadIdx.x; e < c1; e += kLnThreads) {
      const float v = ln_load1<XT>(row, e, p.x_scale);
      s += v; s2 = fmaf(v, v, s2);
    }
  }
  const double ts = block_sum_f64((double)s, red[0]);
  const double ts2 = block_sum_f64((double)s2, red[1]);
  if (threadIdx.x == 0) {
    double* dst = p.partial + ((long long)r * p.chunks + blockIdx.x) * 2;
    dst[0] = ts;
    dst[1] = ts2;
  }
}

template <int XT, int OT, bool VEC>
__global__ void __launch_bounds__(kLnThreads)
    ln_rows_apply_kernel(const LnRowsParams p) {
  __shared__ float stat[2];
  const int r = blockIdx.y;
  if (threadIdx.x < 32) {
    // Combine the row's chunk sums in f64 (chunks is small: cols / 65536).
    double s = 0.0, s2 = 0.0;
    const double* src = p.partial + (long long)r * p.chunks * 2;
    for (int i = threadIdx.x; i < p.chunks; i += 32) { s += src[2 * i]; s2 += src[2 * i + 1]; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s += __shfl_xor_sync(0xffffffffu, s, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (threadIdx.x == 0) {
      const double n = (double)p.cols;
      const double mean = s / n;
      double var = s2 / n - mean * mean;
      if (var < 0.0) var = 0.0;
      stat[0] = (float)mean;
      stat[1] = (float)(1.0 / sqrt(var + (double)p.eps));
    }
  }
  __syncthreads();
  const float mean = stat[0], rstd = stat[1];
  const long long c0 = (long long)blockIdx.x * kLnChunk;
  const long long c1 = c0 + kLnChunk < p.cols ? c0 + kLnChunk : p.cols;
  const uint8_t* row = p.x + (long long)r * p.x_ld * esize(XT);
  uint8_t* orow = reinterpret_cast<uint8_t*>(p.out) + (long long)r * p.out_ld * esize(OT);
  auto norm = [&](float v, long long c) {
    float y = (v - mean) * rstd;
    if (p.w != nullptr) y *= __ldg(p.w + c);
    if (p.b != nullptr) y += __ldg(p.b + c);
    return y;
  };
  auto store1 = [&](long long c, float y) {
    if constexpr (OT == B2F_DTYPE_F32) reinterpret_cast<float*>(orow)[c] = y;
    else reinterpret_cast<__nv_bfloat16*>(orow)[c] = __float2bfloat16_rn(y);
  };
  if (VEC) {
    for (long long c = c0 + (long long)threadIdx.x * kLnVec; c < c1; c += kLnThreads * kLnVec) {
      if (c + kLnVec <= c1) {
        float v[16];
        ln_load16<XT>(row + c * esize(XT), p.x_scale, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = norm(v[i], c + i);
        if constexpr (OT == B2F_DTYPE_F32) {
          float4* o = reinterpret_cast<float4*>(orow + c * 4);
#pragma unroll
          for (int h = 0; h < 4; ++h)
            __stcs(o + h, make_float4(v[4 * h], v[4 * h + 1], v[4 * h + 2], v[4 * h + 3]));
        } else {
          uint4* o = reinterpret_cast<uint4*>(orow + c * 2);
#pragma unroll
          for (int h = 0; h < 2; ++h)
            __stcs(o + h, make_uint4(pack_bf16x2(v[8 * h], v[8 * h + 1]),
                                     pack_bf16x2(v[8 * h + 2], v[8 * h + 3]),
                                     pack_bf16x2(v[8 * h + 4], v[8 * h + 5]),
                                     pack_bf16x2(v[8 * h + 6], v[8 * h + 7])));
        }
      } else {
        for (long long e = c; e < c1; ++e) store1(e, norm(ln_load1<XT>(row, e, p.x_scale), e));
      }
    }
  } else {
    for (long long e = c0 + threadIdx.x; e < c1; e += kLnThreads)
      store1(e, norm(ln_load1<XT>(row, e, p.x_scale), e));
  }
}

template <int XT, int OT>
int launch_ln_rows(const LnRowsParams& p, bool vec, cudaStream_t s) {
  const dim3 grid(p.chunks, p.rows);
  if (vec) {
    ln_rows_stats_kernel<XT, true><<<grid, kLnThreads, 0, s>>>(p);
    ln_rows_apply_kernel<XT, OT, true><<<grid, kLnThreads, 0, s>>>(p);
  } else {
    ln_rows_stats_kernel<XT, false><<<grid, kLnThreads, 0, s>>>(p);
    ln_rows_apply_kernel<XT, OT, false><<<grid, kLnThreads, 0, s>>>(p);
  }
  B2F_CUDA_TRY(cudaGetLastError());
  return B2F_OK;
}

}  // namespace
}  // namespace b2f

extern "C" {

long long b2f_layer_norm_rows_workspace_bytes(int rows, long long cols) {
  if (rows <= 0 || cols <= 0) return 0;
  const long long chunks = (cols + b2f::kLnChunk - 1) / b2f::kLnChunk;
  return (long long)rows * chunks * 2 * (long long)sizeof(double);
}

int b2f_layer_norm_rows(const b2f_lnrows_args* a, b2f_stream_t stream) {
  using namespace b2f;
  if (a == nullptr) return fail(B2F_ERR_ARG, "layer_norm_rows: null args");
  if (a->rows <= 0 || a->cols <= 0) return fail(B2F_ERR_ARG, "layer_norm_rows: empty shape");
  if (a->rows > 65535) return fail(B2F_ERR_UNSUPPORTED, "layer_norm_rows: at most 65535 rows");
  if (a->x == nullptr || a->out == nullptr || a->workspace == nullptr)
    return fail(B2F_ERR_ARG, "layer_norm_rows: null tensor or workspace");
  if (a->x_ld < a->cols || a->out_ld < a->cols)
    return fail(B2F_ERR_ARG, "layer_norm_rows: leading dimension < cols");
  if (a->x_dtype != B2F_DTYPE_E4M3 && a->x_dtype != B2F_DTYPE_BF16 && a->x_dtype != B2F_DTYPE_F32)
    return fail(B2F_ERR_ARG, "layer_norm_rows: x must be e4m3, bf16 or f32");
  if (a->out_dtype != B2F_DTYPE_F32 && a->out_dtype != B2F_DTYPE_BF16)
    return fail(B2F_ERR_ARG, "layer_norm_rows: out must be f32 or bf16");
  if (a->workspace_bytes < b2f_layer_norm_rows_workspace_bytes(a->rows, a->cols) ||
      (reinterpret_cast<uintptr_t>(a->workspace) & 7))
    return fail(B2F_ERR_ARG, "layer_norm_rows: workspace must hold "
                             "b2f_layer_norm_rows_workspace_bytes(rows, cols), 8-byte aligned");
  LnRowsParams p;
  p.x = reinterpret_cast<const uint8_t*>(a->x);
  p.x_ld = a->x_ld;
  p.x_scale = a->x_scale;
  p.rows = a->rows;
  p.cols = a->cols;
  p.chunks = (int)((a->cols + kLnChunk - 1) / kLnChunk);
  p.w = a->weight;
  p.b = a->bias;
  p.eps = a->eps;
  p.out = a->out;
  p.out_ld = a->out_ld;
  p.partial = reinterpret_cast<double*>(a->workspace);
  const int xe = esize(a->x_dtype), oe = esize(a->out_dtype);
  // 16-element vector steps need every row start 16-byte aligned for both tensors.
  const bool vec = (reinterpret_cast<uintptr_t>(a->x) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(a->out) % 16 == 0) &&
                   ((a->x_ld * xe) % 16 == 0) && ((a->out_ld * oe) % 16 == 0);
  cudaStream_t s = (cudaStream_t)stream;
  const int key = a->x_dtype * 4 + a->out_dtype;
  switch (key) {
    case B2F_DTYPE_E4M3 * 4 + B2F_DTYPE_F32: return launch_ln_rows<B2F_DTYPE_E4M3, B2F_DTYPE_F32>(p, vec, s);
    case B2F_DTYPE_E4M3 * 4 + B2F_DTYPE_BF16: return launch_ln_rows<B2F_DTYPE_E4M3, B2F_DTYPE_BF16>(p, vec, s);
    case B2F_DTYPE_BF16 * 4 + B2F_DTYPE_F32: return launch_ln_rows<B2F_DTYPE_BF16, B2F_DTYPE_F32>(p, vec, s);
    case B2F_DTYPE_BF16 * 4 + B2F_DTYPE_BF16: return launch_ln_rows<B2F_DTYPE_BF16, B2F_DTYPE_BF16>(p, vec, s);
    case B2F_DTYPE_F32 * 4 + B2F_DTYPE_F32: return launch_ln_rows<B2F_DTYPE_F32, B2F_DTYPE_F32>(p, vec, s);
    default: return launch_ln_rows<B2F_DTYPE_F32, B2F_DTYPE_BF16>(p, vec, s);
  }
}

void b2f_lnrows_args_init(b2f_lnrows_args* a) {
  if (a == nullptr) return;
  *a = b2f_lnrows_args{};
  a->x_dtype = B2F_DTYPE_E4M3;
  a->x_scale = 1.0f;
  a->eps = 1e-5f;
  a->out_dtype = B2F_DTYPE_F32;
}

}  // extern "C"
