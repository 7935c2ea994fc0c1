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
#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

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
  int schedule;       // B2F_NORM_SCHEDULE_*
  float* row_stats;   // optional [rows] x (mean, rstd) handed from pass 1 to pass 2
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

// Round to bf16 (RN) in place, two values per conversion.
__device__ __forceinline__ void round_bf16(float (&v)[8]) {
#pragma unroll
  for (int j = 0; j < 8; j += 2) {
    const float2 f = unpack_bf16x2(pack_bf16x2(v[j], v[j + 1]));
    v[j] = f.x;
    v[j + 1] = f.y;
  }
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
  pdl_wait();
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
  pdl_wait();
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


// ---------------------------------------------------------------------------------------
// Streaming schedule (the default whenever rows are 16-byte multiples): a persistent CTA of
// TPR threads owns one row at a time and keeps STAGES rows in flight in a shared-memory
// ring, each row fetched by one or two untiled bulk copies (cp.async.bulk, completion on
// the slot's mbarrier) issued by thread 0 as soon as the slot is free.  Per-row arithmetic
// and the thread->vector mapping are those of the row-group kernels above (registers hold
// the row between the statistics and the outputs).  Gamma (and the LayerNorm bias) are
// staged once per CTA in shared memory.
//   PASS2 == false: static scale (one pass) or pass 1 of the dynamic schedule.
//   PASS2 == true : pass 2 of the dynamic schedule, rows walked in reverse order.
constexpr int kStreamMaxStages = 8;

struct StreamCfg {
  const void* src0;  // x (pass 1) or h (pass 2)
  int dt0;
  float scale0;
  long long ld0;
  const void* src1;  // residual or nullptr
  int dt1;
  long long ld1;
  uint32_t bytes0, bytes1;  // row bytes of each source (16-byte multiples)
  uint32_t slot_bytes;      // bytes0 + bytes1
  uint32_t wbytes;          // staged gamma bytes, 16-byte rounded
  uint32_t bbytes;          // staged bias bytes (0 without a LayerNorm bias)
  int stages;
  int tpr;
  bool round_h;  // round h to bf16 before the statistics (pass 1 writing a bf16 h)
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Compile-time specialisation of the streaming kernel.  kDyn selects the runtime value
// (the generic instance); kNone (residual only) means no residual.  FULL: every thread owns
// exactly VPT vectors (cols == 8 * VPT * TPR), so no per-vector bounds checks.
constexpr int kDyn = -1;
constexpr int kNone = -2;

__device__ __forceinline__ void st16_hint(void* ptr, uint4 v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(ptr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "l"(pol)
               : "memory");
}

template <int DT>
__device__ __forceinline__ void ld8(const uint8_t* base, int rt, long long off, float (&v)[8]) {
  load8(base, DT == kDyn ? rt : DT, off, 1.0f, v);
}

template <bool PASS2, int KIND, int DT0, int DT1, int WDT, bool FULL>
__global__ void __launch_bounds__(256, 3) norm_stream_kernel(const NormParams p, const StreamCfg c) {
  pdl_wait();
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kStreamMaxStages];
  __shared__ float red[8];
  const int tpr = c.tpr;
  const int t = threadIdx.x;
  const int nvec = p.cols / 8;
  const int G = gridDim.x;
  const int kind = KIND == kDyn ? p.kind : KIND;
  const int dt0 = DT0 == kDyn ? c.dt0 : DT0;
  const bool has_res = DT1 == kNone ? false : (DT1 == kDyn ? c.src1 != nullptr : true);
  const int dt1 = DT1 >= 0 ? DT1 : c.dt1;
  const int wdt = WDT == kDyn ? p.w_dtype : WDT;
  uint8_t* sw = smem;
  uint8_t* sb = smem + c.wbytes;
  uint8_t* ring = smem + c.wbytes + c.bbytes;
  const int nrows = blockIdx.x < p.rows ? (p.rows - 1 - blockIdx.x) / G + 1 : 0;
  auto row_of = [&](int k) -> long long {
    const int r = blockIdx.x + k * G;
    return PASS2 ? p.rows - 1 - r : r;
  };
  const uint64_t pol = policy_evict_first();
  const uint64_t pol_keep = policy_evict_last();
  const int e0 = dt0 == kF32 ? 4 : (dt0 == kBF16 ? 2 : 1);
  const int e1 = dt1 == kF32 ? 4 : 2;
  auto issue = [&](int k) {
    const int slot = k % c.stages;
    const long long r = row_of(k);
    uint8_t* dst = ring + (size_t)slot * c.slot_bytes;
    mbar_arrive_expect_tx(&full[slot], c.slot_bytes);
    bulk_load(dst, static_cast<const uint8_t*>(c.src0) + r * c.ld0 * e0, c.bytes0, &full[slot],
              pol);
    if (has_res)
      bulk_load(dst + c.bytes0, static_cast<const uint8_t*>(c.src1) + r * c.ld1 * e1, c.bytes1,
                &full[slot], pol);
  };
  if (t == 0) {
    for (int i = 0; i < c.stages; ++i) mbar_init(&full[i], 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  int issued = 0;
  if (t == 0)
    for (; issued < c.stages && issued < nrows; ++issued) issue(issued);
  const bool has_b = kind == 1 && p.bias != nullptr;
  {
    // Gamma (plus the RMSNorm weight offset, the same f32 addition the formula makes) and
    // the LayerNorm bias, staged as f32: no per-element conversion or offset add later.
    const float woff = kind == 1 ? 0.0f : p.w_offset;
    for (int i = t; i < nvec; i += blockDim.x) {
      float v[8];
      load8(p.weight, wdt, (long long)i * 8, 1.0f, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += woff;
      reinterpret_cast<float4*>(sw)[2 * i] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(sw)[2 * i + 1] = make_float4(v[4], v[5], v[6], v[7]);
      if (has_b) {
        load8(p.bias, wdt, (long long)i * 8, 1.0f, v);
        reinterpret_cast<float4*>(sb)[2 * i] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(sb)[2 * i + 1] = make_float4(v[4], v[5], v[6], v[7]);
      }
    }
  }
  // (the first row-wait's barrier below publishes the staged gamma / bias)

  float s = p.q_scale;
  if (PASS2) {
    const float amax = *p.amax;
    s = amax > 0.f ? amax / 448.0f : 1.0f;
    if (blockIdx.x == 0 && t == 0) *p.scale_out = s;
  }
  const float qinv = 1.0f / s;
  const bool dyn1 = !PASS2 && p.dynamic;
  const bool store_h = !PASS2 && p.h_out != nullptr;
  const bool scale0 = c.scale0 != 1.0f;
  const float n = float(p.cols);
  const float w_off = p.w_offset;
  float amax = 0.f;
  int k = 0;
  bool aborted = false;
  for (; k < nrows; ++k) {
    const int slot = k % c.stages;
    const bool ok = mbar_wait(&full[slot], (k / c.stages) & 1, kDevTimeoutProducer, nullptr);
    if (__syncthreads_or(!ok)) {
      aborted = true;
      break;
    }
    const uint8_t* src = ring + (size_t)slot * c.slot_bytes;
    float h[VPT][8];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = t + tpr * i;
      if (FULL || vi < nvec) {
        ld8<DT0>(src, dt0, (long long)vi * 8, h[i]);
        if (scale0) {
#pragma unroll
          for (int j = 0; j < 8; ++j) h[i][j] *= c.scale0;
        }
        if (has_res) {
          float r[8];
          ld8<DT1 >= 0 ? DT1 : kDyn>(src + c.bytes0, dt1, (long long)vi * 8, r);
#pragma unroll
          for (int j = 0; j < 8; ++j) h[i][j] += r[j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) h[i][j] = 0.f;
      }
    }
    __syncthreads();  // every thread has its row in registers: the slot can be refilled
    if (t == 0 && issued < nrows) {
      fence_proxy_async_smem();
      issue(issued);
    }
    if (issued < nrows) ++issued;
    const long long row = row_of(k);
    if (c.round_h) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) round_bf16(h[i]);
    }
    if (store_h) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = t + tpr * i;
        if (FULL || vi < nvec) {
          const long long off = row * p.h_ld + (long long)vi * 8;
          if (dyn1 && p.h_dtype == kBF16) {
            // Pass 2 re-reads h (newest rows first): ask L2 to keep it.
            uint4 q;
            q.x = pack_bf16x2(h[i][0], h[i][1]); q.y = pack_bf16x2(h[i][2], h[i][3]);
            q.z = pack_bf16x2(h[i][4], h[i][5]); q.w = pack_bf16x2(h[i][6], h[i][7]);
            st16_hint(reinterpret_cast<__nv_bfloat16*>(p.h_out) + off, q, pol_keep);
          } else {
            store8(p.h_out, p.h_dtype, off, h[i]);
          }
        }
      }
    }
    float mean = 0.f, inv;
    if (PASS2 && p.row_stats != nullptr) {
      // (mean, rstd) left by pass 1: bit-identical to recomputing them from h
      const float2 st = reinterpret_cast<const float2*>(p.row_stats)[row];
      mean = st.x;
      inv = st.y;
    } else {
      float s1 = 0.f, s2 = 0.f;
      if (kind == 1) {
#pragma unroll
        for (int i = 0; i < VPT; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) s1 += h[i][j];
        mean = group_sum(s1, red, tpr) / n;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
          if (FULL || t + tpr * i < nvec) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float d = h[i][j] - mean;
              s2 += d * d;
            }
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < VPT; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) s2 += h[i][j] * h[i][j];
      }
      inv = rsqrtf(group_sum(s2, red, tpr) / n + p.eps);
      if (!PASS2 && dyn1 && p.row_stats != nullptr && t == 0)
        reinterpret_cast<float2*>(p.row_stats)[row] = make_float2(mean, inv);
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = t + tpr * i;
      if (FULL || vi < nvec) {
        float w[8], y[8];
        ld8<kF32>(sw, kF32, (long long)vi * 8, w);
        if (kind == 1) {
          float b[8];
          if (has_b) {
            ld8<kF32>(sb, kF32, (long long)vi * 8, b);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) b[j] = 0.f;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) y[j] = (h[i][j] - mean) * inv * w[j] + b[j];
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) y[j] = h[i][j] * inv * w[j];  // w: gamma + offset
        }
        if (dyn1) {
          round_bf16(y);
#pragma unroll
          for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(y[j]));
        } else if (PASS2) {
          round_bf16(y);
          if (p.y_out != nullptr) store8(p.y_out, kBF16, row * p.y_ld + (long long)vi * 8, y);
          *reinterpret_cast<uint2*>(p.q_out + row * p.q_ld + vi * 8) = quant8(y, qinv);
        } else {
          *reinterpret_cast<uint2*>(p.q_out + row * p.q_ld + vi * 8) = quant8(y, qinv);
          if (p.y_out != nullptr) {
            round_bf16(y);
            store8(p.y_out, kBF16, row * p.y_ld + (long long)vi * 8, y);
          }
        }
      }
    }
  }
  if (aborted) {
    // Let the copies still in flight land before the CTA's shared memory is released.
    if (t == 0)
      for (int j = k; j < issued; ++j)
        mbar_wait(&full[j % c.stages], (j / c.stages) & 1, kDevTimeoutDrain, nullptr);
    return;
  }
  if (dyn1) {
    const float m = block_max(amax, red);
    if (t == 0) atomic_max_nonneg(p.amax, m);
  }
}

using StreamFn = void (*)(const NormParams, const StreamCfg);

// The specialised instances: (KIND, DT0, DT1, WDT) of the library's callers (BASELINE
// config 3 passes 1 and 2, the GPT-2 / vision LayerNorms, the Qwen RMSNorms); anything
// else runs the generic instance.
template <bool PASS2, bool FULL>
StreamFn pick_stream(int kind, int dt0, int dt1, int wdt) {
#define B2F_STREAM(K, D0, D1, W)                                   \
  if (kind == K && dt0 == D0 && dt1 == D1 && wdt == W)             \
    return norm_stream_kernel<PASS2, K, D0, D1, W, FULL>;
  B2F_STREAM(0, kBF16, kBF16, kBF16)
  B2F_STREAM(0, kBF16, kNone, kBF16)
  B2F_STREAM(0, kBF16, kNone, kF32)
  B2F_STREAM(0, kF32, kNone, kF32)
  B2F_STREAM(0, kE4M3, kNone, kF32)
  B2F_STREAM(1, kBF16, kNone, kF32)
  B2F_STREAM(1, kF32, kNone, kF32)
  B2F_STREAM(1, kE4M3, kNone, kF32)
  B2F_STREAM(1, kBF16, kBF16, kF32)
#undef B2F_STREAM
  return norm_stream_kernel<PASS2, kDyn, kDyn, kDyn, kDyn, false>;
}

// ---------------------------------------------------------------------------------------
// Short rows (the blocks' LayerNorms / input RMSNorms: <= 32 * 8 * kWarpMaxNV columns, bf16
// x, bf16 or f32 weights, static scale, no residual / h / y outputs): one warp per row.
// Lane l owns vectors l + 32 i, the order of the row-group kernels with 32 threads per row.
constexpr int kWarpMaxNV = 12;

// Warp per row without staging: the row's 16-byte vectors go straight into registers,
// gamma / bias come through the L1 cache, and each warp takes one row (grid = rows / 8), so
// a kernel of this size runs like a plain elementwise pass.  Measured in a CUDA graph on
// [8192 x 768] LayerNorm: 7.0 us, where a shared-memory ring filled by one bulk copy per
// row and a persistent kernel prefetching the next row into registers (weights staged per
// CTA) took 9.5-10.8 us and a plain 25 MB copy 4.2 us.  Statistics in the row-group
// kernels' order; outputs in packed f32x2 arithmetic, the same operations per element.
template <int NV, bool WF32>
__global__ void __launch_bounds__(256, NV <= 6 ? 4 : 3) norm_warp_direct_kernel(const NormParams p) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int nvec = p.cols / 8;
  const bool ln = p.kind == 1;
  const bool has_b = ln && p.bias != nullptr;
  const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.x) + row * p.x_ld);
  uint4 raw[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int vi = lane + 32 * i;
    raw[i] = vi < nvec ? __ldcs(src + vi) : make_uint4(0u, 0u, 0u, 0u);
  }
  // The row stays packed between passes: the fence keeps the compiler from carrying the
  // unpacked f32 values (8 per vector) across the warp reductions, which spills.
  auto fence = [&]() {
#pragma unroll
    for (int i = 0; i < NV; ++i)
      asm volatile("" : "+r"(raw[i].x), "+r"(raw[i].y), "+r"(raw[i].z), "+r"(raw[i].w));
  };
  auto unpack = [&](const uint4& q, float (&v)[8]) {
    const float2 a = unpack_bf16x2(q.x), b = unpack_bf16x2(q.y), c = unpack_bf16x2(q.z),
                 d = unpack_bf16x2(q.w);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x;
    v[7] = d.y;
    if (p.x_scale != 1.0f) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] *= p.x_scale;
    }
  };
  auto load_w = [&](const void* base, int vi, float2 (&o)[4]) {
    if constexpr (WF32) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(base) + 2 * vi);
      const float4 b = __ldg(reinterpret_cast<const float4*>(base) + 2 * vi + 1);
      o[0] = make_float2(a.x, a.y); o[1] = make_float2(a.z, a.w);
      o[2] = make_float2(b.x, b.y); o[3] = make_float2(b.z, b.w);
    } else {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(base) + vi);
      o[0] = unpack_bf16x2(q.x); o[1] = unpack_bf16x2(q.y);
      o[2] = unpack_bf16x2(q.z); o[3] = unpack_bf16x2(q.w);
    }
  };
  const float n = float(p.cols);
  float mean = 0.f, s2 = 0.f;
  if (ln) {
    float s1 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float v[8];
      unpack(raw[i], v);
#pragma unroll
      for (int j = 0; j < 8; ++j) s1 += v[j];
    }
    mean = warp_sum(s1) / n;
    fence();
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (lane + 32 * i < nvec) {
        float v[8];
        unpack(raw[i], v);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float d = v[j] - mean;
          s2 += d * d;
        }
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float v[8];
      unpack(raw[i], v);
#pragma unroll
      for (int j = 0; j < 8; ++j) s2 += v[j] * v[j];
    }
  }
  const float inv = rsqrtf(warp_sum(s2) / n + p.eps);
  fence();
  const float qinv = 1.0f / p.q_scale;
  const float2 inv2 = make_float2(inv, inv), nmean2 = make_float2(-mean, -mean);
  const float2 qinv2 = make_float2(qinv, qinv), off2 = make_float2(p.w_offset, p.w_offset);
  uint8_t* qrow = p.q_out + row * p.q_ld;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      float h[8];
      unpack(raw[i], h);
      float2 w2[4], b2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                             make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      load_w(p.weight, vi, w2);
      if (has_b) load_w(p.bias, vi, b2);
      uint32_t o16[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float2 x = make_float2(h[2 * t], h[2 * t + 1]);
        float2 y;
        if (ln) {
          x = fmul2(fadd2(x, nmean2), inv2);
          y = ffma2(x, w2[t], b2[t]);
        } else {
          y = fmul2(fmul2(x, inv2), fadd2(w2[t], off2));
        }
        y = fmul2(y, qinv2);
        o16[t] = f32x2_to_e4m3x2(y.x, y.y);
      }
      __stcs(reinterpret_cast<uint2*>(qrow + vi * 8),
             make_uint2(o16[0] | (o16[1] << 16), o16[2] | (o16[3] << 16)));
    }
  }
}

using WarpDirectFn = void (*)(const NormParams);

template <bool WF32>
WarpDirectFn pick_warp_direct(int nv) {
  switch (nv) {
    case 1: return norm_warp_direct_kernel<1, WF32>;
    case 2: return norm_warp_direct_kernel<2, WF32>;
    case 3: return norm_warp_direct_kernel<3, WF32>;
    case 4: return norm_warp_direct_kernel<4, WF32>;
    case 5: return norm_warp_direct_kernel<5, WF32>;
    case 6: return norm_warp_direct_kernel<6, WF32>;
    case 7: return norm_warp_direct_kernel<7, WF32>;
    case 8: return norm_warp_direct_kernel<8, WF32>;
    case 9: return norm_warp_direct_kernel<9, WF32>;
    case 10: return norm_warp_direct_kernel<10, WF32>;
    case 11: return norm_warp_direct_kernel<11, WF32>;
    default: return norm_warp_direct_kernel<12, WF32>;
  }
}

// The warp-per-row schedule applies to: static scale, bf16 x, bf16 or f32 weights, no
// residual / h / y outputs, 16-byte aligned rows and 8-byte aligned q rows.
bool plan_warp(const NormParams& p) {
  const int nvec = p.cols / 8;
  if (p.dynamic != B2F_SCALE_STATIC || p.residual != nullptr || p.h_out != nullptr ||
      p.y_out != nullptr)
    return false;
  if (p.x_dtype != kBF16 || (p.w_dtype != kBF16 && p.w_dtype != kF32) ||
      nvec > 32 * kWarpMaxNV)
    return false;
  if ((reinterpret_cast<uintptr_t>(p.x) & 15) || (p.x_ld * 2) % 16) return false;
  if ((reinterpret_cast<uintptr_t>(p.weight) & 15) ||
      (p.bias != nullptr && (reinterpret_cast<uintptr_t>(p.bias) & 15)))
    return false;
  if ((reinterpret_cast<uintptr_t>(p.q_out) & 7) || p.q_ld % 8) return false;
  return true;
}

int launch_warp(const NormParams& p, cudaStream_t s) {
  const int nvec = p.cols / 8;
  const WarpDirectFn fn = p.w_dtype == kF32 ? pick_warp_direct<true>((nvec + 31) / 32)
                                            : pick_warp_direct<false>((nvec + 31) / 32);
  B2F_CUDA_TRY(launch_pdl(fn, dim3((p.rows + 7) / 8), dim3(256), 0, s, p));
  return B2F_OK;
}

// Host-side choice between the streaming schedule and the one-row-per-group kernels.
struct StreamLaunch {
  StreamCfg cfg;
  StreamFn fn;
  int grid;
  size_t smem;
};

int stream_occupancy(const void* fn, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, int, size_t>, int> cache;
  static std::map<std::pair<int, const void*>, bool> opted;
  std::lock_guard<std::mutex> g(mu);
  int dev = 0;
  cudaGetDevice(&dev);
  auto key = std::make_tuple(dev, fn, threads, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  // Opt the kernel in once to the device's whole per-block shared memory (a per-function
  // attribute: lowering it for one launch size would break launches of larger ones).
  if (!opted[{dev, fn}]) {
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - 1024) !=
        cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    opted[{dev, fn}] = true;
  }
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    blocks = 0;
  }
  cache[key] = blocks;
  return blocks;
}

bool plan_stream(const NormParams& p, bool pass2, StreamLaunch& L) {
  StreamCfg& c = L.cfg;
  const int nvec = p.cols / 8;
  c.tpr = ((nvec + VPT - 1) / VPT + 31) / 32 * 32;
  auto esz = [](int dt) { return dt == kF32 ? 4 : (dt == kBF16 ? 2 : 1); };
  if (pass2 && p.h_out != nullptr) {
    c.src0 = p.h_out; c.dt0 = p.h_dtype; c.scale0 = 1.0f; c.ld0 = p.h_ld;
    c.src1 = nullptr; c.dt1 = kBF16; c.ld1 = 0;
    c.round_h = false;
  } else {
    c.src0 = p.x; c.dt0 = p.x_dtype; c.scale0 = p.x_scale; c.ld0 = p.x_ld;
    c.src1 = p.residual; c.dt1 = p.res_dtype; c.ld1 = p.res_ld;
    c.round_h = !pass2 && p.h_out != nullptr && p.h_dtype == kBF16;
  }
  c.bytes0 = (uint32_t)(p.cols * esz(c.dt0));
  c.bytes1 = c.src1 != nullptr ? (uint32_t)(p.cols * esz(c.dt1)) : 0u;
  if (c.bytes0 % 16 || c.bytes1 % 16) return false;
  if ((reinterpret_cast<uintptr_t>(c.src0) & 15) || (c.ld0 * esz(c.dt0)) % 16) return false;
  if (c.src1 != nullptr &&
      ((reinterpret_cast<uintptr_t>(c.src1) & 15) || (c.ld1 * esz(c.dt1)) % 16))
    return false;
  c.slot_bytes = c.bytes0 + c.bytes1;
  c.wbytes = (uint32_t)((p.cols * 4 + 15) / 16 * 16);  // f32 staging
  c.bbytes = (p.kind == 1 && p.bias != nullptr) ? c.wbytes : 0u;
  // About 32 KiB of rows in flight per CTA (at least two), several CTAs per SM.
  c.stages = (int)std::max<uint32_t>(
      2u, std::min<uint32_t>((uint32_t)kStreamMaxStages, (32u * 1024u) / c.slot_bytes));
  L.smem = (size_t)c.wbytes + c.bbytes + (size_t)c.stages * c.slot_bytes;
  const bool full = c.tpr * VPT == nvec;
  const int d1 = c.src1 != nullptr ? c.dt1 : kNone;
  L.fn = pass2 ? (full ? pick_stream<true, true>(p.kind, c.dt0, d1, p.w_dtype)
                       : pick_stream<true, false>(p.kind, c.dt0, d1, p.w_dtype))
               : (full ? pick_stream<false, true>(p.kind, c.dt0, d1, p.w_dtype)
                       : pick_stream<false, false>(p.kind, c.dt0, d1, p.w_dtype));
  const int per_sm = stream_occupancy((const void*)L.fn, c.tpr, L.smem);
  if (per_sm <= 0) return false;
  L.grid = std::min(p.rows, sm_count() * per_sm);
  return true;
}

int launch_stream(const NormParams& p, const StreamLaunch& L, cudaStream_t s) {
  B2F_CUDA_TRY(launch_pdl(L.fn, dim3(L.grid), dim3(L.cfg.tpr), L.smem, s, p, L.cfg));
  B2F_CUDA_TRY(cudaGetLastError());
  return B2F_OK;
}

int launch_norm(const NormParams& p, cudaStream_t s) {
  const int nvec = p.cols / 8;
  int tpr = ((nvec + VPT - 1) / VPT + 31) / 32 * 32;  // threads per row
  const int rpc = 256 / tpr;                            // rows per CTA
  const int threads = rpc * tpr;
  const int grid = (p.rows + rpc - 1) / rpc;
  const bool run1 = p.dynamic != B2F_SCALE_DYNAMIC_APPLY;
  const bool run2 = p.dynamic == B2F_SCALE_DYNAMIC || p.dynamic == B2F_SCALE_DYNAMIC_APPLY;
  if (run1 && p.dynamic) B2F_CUDA_TRY(cudaMemsetAsync(p.amax, 0, sizeof(float), s));
  StreamLaunch L;
  if (p.schedule == B2F_NORM_SCHEDULE_AUTO && plan_warp(p)) return launch_warp(p, s);
  if (run1) {
    if (p.schedule == B2F_NORM_SCHEDULE_AUTO && plan_stream(p, false, L)) {
      if (int rc = launch_stream(p, L, s)) return rc;
    } else {
      B2F_CUDA_TRY(launch_pdl(norm_pass1_kernel, dim3(grid), dim3(threads), 0, s, p, tpr));
      B2F_CUDA_TRY(cudaGetLastError());
    }
  }
  if (run2) {
    if (p.schedule == B2F_NORM_SCHEDULE_AUTO && plan_stream(p, true, L)) {
      if (int rc = launch_stream(p, L, s)) return rc;
    } else {
      B2F_CUDA_TRY(launch_pdl(norm_pass2_kernel, dim3(grid), dim3(threads), 0, s, p, tpr));
      B2F_CUDA_TRY(cudaGetLastError());
    }
  }
  return B2F_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Validates the C-ABI arguments and fills the kernel parameters.
int build_params(const b2f_norm_args* a, NormParams& p) {
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
  if (a->dynamic_scale < B2F_SCALE_STATIC || a->dynamic_scale > B2F_SCALE_DYNAMIC_APPLY)
    return fail(B2F_ERR_ARG, "norm_quant: bad dynamic_scale mode");
  if (a->schedule != B2F_NORM_SCHEDULE_AUTO && a->schedule != B2F_NORM_SCHEDULE_ROWGROUP)
    return fail(B2F_ERR_ARG, "norm_quant: bad schedule");
  if (a->dynamic_scale == B2F_SCALE_DYNAMIC_STATS && a->amax == nullptr)
    return fail(B2F_ERR_ARG, "norm_quant: the stats pass needs an amax buffer");
  if ((a->dynamic_scale == B2F_SCALE_DYNAMIC || a->dynamic_scale == B2F_SCALE_DYNAMIC_APPLY) &&
      (a->amax == nullptr || a->scale_out == nullptr))
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
  p.schedule = a->schedule;
  p.row_stats = a->row_stats;
  if (a->row_stats != nullptr && (reinterpret_cast<uintptr_t>(a->row_stats) & 7))
    return fail(B2F_ERR_ARG, "norm_quant: row_stats must be 8-byte aligned");
  return B2F_OK;
}

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
  NormParams p;
  if (int rc = build_params(a, p)) return rc;
  return launch_norm(p, (cudaStream_t)stream);
}

int b2f_norm_plan(const b2f_norm_args* a) {
  using namespace b2f;
  NormParams p;
  if (int rc = build_params(a, p)) return -rc;
  if (p.schedule != B2F_NORM_SCHEDULE_AUTO) return B2F_NORM_SCHEDULE_ROWGROUP;
  if (plan_warp(p)) return 2;  // warp-per-row schedule
  StreamLaunch L;
  const bool pass1 = p.dynamic != B2F_SCALE_DYNAMIC_APPLY;
  return plan_stream(p, !pass1, L) ? B2F_NORM_SCHEDULE_AUTO : B2F_NORM_SCHEDULE_ROWGROUP;
}


}  // extern "C"
