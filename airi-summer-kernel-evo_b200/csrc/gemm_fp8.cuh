// Persistent warp-specialised e4m3 x e4m3 -> f32 GEMM on 5th-generation tensor cores.
//
//   C[M,N] = epilogue( (A[M,K] . B[N,K]^T) * alpha )
//
// A and B are K-major (row-major [rows, K] bytes), exactly the `matrix_a` / `matrix_b_nk`
// operands of the reference's square-GEMM and GEMM+epilogue tasks
// (tasks/level1_01_square_matrix_multiplication_fp8/starter.py:125-138,
//  tasks/level2_76_gemm_add_relu_fp8/starter.py:148-169).
//
// Roles (320 threads, one CTA per SM, grid = min(#tiles, #SMs)):
//   warp 0   TMA producer: streams 128-byte K blocks of A (128 rows) and B (BN rows) into
//            a STAGES-deep ring of 128B-swizzled shared-memory slots.
//   warp 1   allocates TMEM (2 accumulators x BN f32 columns), then one thread issues
//            tcgen05.mma.kind::f8f6f4 (M=128, N=BN, K=32) four times per K block and
//            releases each slot with tcgen05.commit.
//   warps 2-9 epilogue: two warps per TMEM lane quadrant, each draining half the tile's
//            columns with tcgen05.ld; the fused epilogue runs in registers and leaves
//            through shared memory with TMA stores.  Double-buffered accumulators let the
//            epilogue of tile i overlap the main loop of tile i+1.
#pragma once
#include "common.cuh"

namespace b2f {

enum : int { kOutF32 = 0, kOutBF16 = 1, kOutE4M3 = 2 };
enum : int { kActNone = 0, kActRelu = 1, kActGeluTanh = 2, kActLeakyRelu = 3, kActSilu = 4 };
enum : int { kModeStore = 0, kModeRowSum = 1 };

// Attention-operand preparation fused into a q / gate / k / v projection's epilogue (CTA
// pair kernel, 256-column tiles: each epilogue warp's 128-column half of a tile is one head
// or one plain block of columns).  Half-tiles that are a q or k head are rounded to e4m3 at
// the projection's scale (the values a separate GEMM would have stored), RMS-normalised
// over the head, rotated (RoPE over the whole head) and stored as e4m3 in q_out / k_out;
// half-tiles that are a v head are rounded the same way and stored as 16-bit codes in
// v_out; every other column (the attention gate) takes the ordinary epilogue into `out`.
struct HeadPrepParams {
  int on;
  int q_off, q_hstride, q_heads;  // q head h at columns q_off + h * q_hstride, 128 wide
  int k_off, k_heads;             // k head h at k_off + 128 h
  int v_off, v_heads;             // v head h at v_off + 128 h
  int v_f16;                      // v_out holds f16 (else bf16) codes
  uint8_t* q_out;
  long long q_ld;
  uint8_t* k_out;
  long long k_ld;
  uint16_t* v_out;
  long long v_ld;
  const float* q_w;  // [128] RMSNorm weight (+ w_offset), or null: no norm
  const float* k_w;
  float w_offset, eps;
  const float* cos;  // [seq][128] rotary tables (sign of rotate_half not folded), or null
  const float* sin;
  int seq;               // rotary position = row % seq
  float x_scale;         // one e4m3 code of the projection = x_scale (its out_scale)
  float out_inv_scale;   // q / k codes = e4m3(y * out_inv_scale)
};

struct EpilogueParams {
  float alpha;             // scale_a * scale_b
  const float* alpha_ptr;  // optional device scalar multiplied into alpha (may be null)
  const float* col_scale;  // optional [N] f32 per-column scale (may be null)
  const float* bias;       // [N] f32, may be null
  float pre_mul, pre_add;  // v = (alpha*acc + bias)*pre_mul + pre_add
  int act;                 // activation applied after the affine step
  float act_param;         // LeakyReLU negative slope
  float post_mul;          // v *= post_mul after the activation
  const void* gate;        // optional f32 / bf16 [M, gate_ld]: v *= gate after post_mul
  int gate_dtype;
  long long gate_ld;
  int gate_vec;            // gate base and row pitch 16-byte aligned: vector loads
  const void* residual;    // optional [M, res_ld] tensor added after the gate
  int res_dtype;           // kOutF32 / kOutBF16 / kOutE4M3
  long long res_ld;
  float res_scale;         // residual value = stored * res_scale
  void* out;               // output [M, out_ld]  (RowSum mode: f32 [M])
  int out_dtype;
  long long out_ld;
  float out_inv_scale;     // stored = v * out_inv_scale (quantised outputs)
  float* amax;             // optional: atomic max of |v| over the whole output
  int mode;                // kModeStore / kModeRowSum
  int out_vec;             // out base and row pitch 16-byte aligned: vector stores
  int res_vec;             // residual base and row pitch 16-byte aligned: vector loads
  int chunk_bytes;         // TMA store box width: 128 (SW128) or 64 (SW64) bytes
  float* ws;               // split-K: f32 partial tiles [splits][rows_pad][ws_ld]
  long long ws_ld;
  long long ws_slice;      // elements per split slice (rows_pad * ws_ld)
  unsigned int* counters;  // split-K: per output tile, (epoch << 8) | arrival state
  unsigned int epoch;      // split-K: this call's 24-bit tag (a counter whose tag differs
                           // is stale, left by an aborted call, and reads as zero)
  HeadPrepParams hp;       // fused attention-operand preparation (pair kernel only)
};

// Split-K tile counter update: adds `add` to the tile's arrival state for this call and
// returns the state before the update.  A counter whose epoch tag is not this call's
// (a call that timed out or aborted left it mid-protocol) counts as zero, so one failed
// call cannot mislead the next one that shares the workspace.
__device__ __forceinline__ unsigned splitk_arrive(unsigned int* c, unsigned epoch, unsigned add) {
  unsigned old = atomicAdd(c, 0u);  // L2-coherent read
  while (true) {
    const unsigned state = (old >> 8) == epoch ? (old & 0xFFu) : 0u;
    const unsigned prev = atomicCAS(c, old, (epoch << 8) | (state + add));
    if (prev == old) return state;
    old = prev;
  }
}

// Reads the tile's arrival state for this call (zero when the tag is stale).
__device__ __forceinline__ unsigned splitk_state(unsigned int* c, unsigned epoch) {
  const unsigned v = atomicAdd(c, 0u);
  return (v >> 8) == epoch ? (v & 0xFFu) : 0u;
}

struct GemmShape {
  int M, N, K;
  int splits;   // K slices per output tile (split-K, 1-CTA kernel only); 1 = off
  int group_m;  // row blocks per raster group (tile_coords)
};

// Hardware tanh (MUFU, max relative error ~2^-11); every GELU output is requantised to
// e4m3 (relative step 2^-3), so the approximation is far below the output resolution.
__device__ __forceinline__ float tanh_hw(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float gelu_tanh(float x) {
  // 0.5 x (1 + tanh( sqrt(2/pi) (x + 0.044715 x^3) )), as torch's approximate="tanh".
  const float k0 = 0.7978845608028654f;
  const float k1 = 0.044715f;
  const float u = k0 * fmaf(k1 * x, x * x, x);
  return 0.5f * x * (1.0f + tanh_hw(u));
}

// Activation of a pair of values, selected at compile time (a runtime switch inside the
// element loop gets if-converted into evaluating every activation for every element).
// GELU-tanh: 0.5 x (1 + tanh(x (k0 + k0 k1 x^2))) with packed pair arithmetic and the
// hardware tanh per element.
template <int ACT>
__device__ __forceinline__ float2 act_pair(float2 v, float p) {
  if constexpr (ACT == kActRelu) {
    return make_float2(fmaxf(v.x, 0.0f), fmaxf(v.y, 0.0f));
  } else if constexpr (ACT == kActGeluTanh) {
    const float k0 = 0.7978845608028654f;
    const float k0k1 = 0.7978845608028654f * 0.044715f;
    const float2 x2 = fmul2(v, v);
    const float2 u = fmul2(ffma2(x2, make_float2(k0k1, k0k1), make_float2(k0, k0)), v);
    const float2 h = fmul2(v, make_float2(0.5f, 0.5f));
    return ffma2(h, make_float2(tanh_hw(u.x), tanh_hw(u.y)), h);
  } else if constexpr (ACT == kActLeakyRelu) {
    return make_float2(v.x >= 0.0f ? v.x : v.x * p, v.y >= 0.0f ? v.y : v.y * p);
  } else if constexpr (ACT == kActSilu) {
    return make_float2(v.x / (1.0f + expf(-v.x)), v.y / (1.0f + expf(-v.y)));
  } else {
    return v;
  }
}

// acc * m + a per column (m, a broadcast from the lanes that hold column j's values when
// LANES, else uniform), then the activation, then post_mul: 16 pairs.  ACT is a compile-time
// activation (none / ReLU / GELU); kActDyn selects the rarely used ones at run time.
// Few instances on purpose: with one per (activation, bias, column scale) combination the
// epilogue outgrew the instruction cache (instruction-fetch stalls in the short-K GEMMs).
constexpr int kActDyn = -1;

__device__ __forceinline__ float act_dyn(float v, int act, float p) {
  switch (act) {
    case kActRelu: return fmaxf(v, 0.0f);
    case kActGeluTanh: return gelu_tanh(v);
    case kActLeakyRelu: return v >= 0.0f ? v : v * p;
    case kActSilu: return v / (1.0f + expf(-v));
    default: return v;
  }
}

template <int ACT, bool LANES>
__device__ __forceinline__ void affine_act32(const uint32_t (&acc)[32], float (&v)[32],
                                             float m, float a, float lane_mul, float lane_add,
                                             int act, float p, float post_mul) {
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float2 m2 = LANES ? make_float2(__shfl_sync(0xffffffffu, lane_mul, j),
                                          __shfl_sync(0xffffffffu, lane_mul, j + 1))
                            : make_float2(m, m);
    const float2 a2 = LANES ? make_float2(__shfl_sync(0xffffffffu, lane_add, j),
                                          __shfl_sync(0xffffffffu, lane_add, j + 1))
                            : make_float2(a, a);
    float2 x = ffma2(make_float2(__uint_as_float(acc[j]), __uint_as_float(acc[j + 1])), m2, a2);
    if constexpr (ACT == kActDyn) x = make_float2(act_dyn(x.x, act, p), act_dyn(x.y, act, p));
    else x = act_pair<ACT>(x, p);
    if (post_mul != 1.0f) x = fmul2(x, make_float2(post_mul, post_mul));
    v[j] = x.x;
    v[j + 1] = x.y;
  }
}

template <int ACT>
__device__ __forceinline__ void affine_act32_sel(const EpilogueParams& ep, const uint32_t (&acc)[32],
                                                 float (&v)[32], float m, float a,
                                                 float lane_mul, float lane_add) {
  // (lane_mul / lane_add hold alpha * pre_mul / pre_add in every lane when there is no
  // column scale / bias, so either one alone takes the lane path)
  if (ep.col_scale != nullptr || ep.bias != nullptr)
    affine_act32<ACT, true>(acc, v, m, a, lane_mul, lane_add, ep.act, ep.act_param, ep.post_mul);
  else
    affine_act32<ACT, false>(acc, v, m, a, lane_mul, lane_add, ep.act, ep.act_param, ep.post_mul);
}

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 128;  // bytes of K per stage = one 128B swizzle row
  static constexpr int STAGES = (BN == 256) ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators
  static constexpr int SMEM_BYTES =
      STAGES * STAGE_BYTES + 4 * 8192 /*epilogue staging*/ + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int THREADS = 320;  // producer, MMA, 8 epilogue warps
};

// Tile order: groups of GROUP_M row-blocks sweep all column blocks, so the CTAs that run
// concurrently share A rows and B columns in L2 (GROUP_M chosen on the host: group_rows).
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int GROUP_M, int& mb,
                                            int& nb) {
  const int per_group = GROUP_M * num_n;
  const int g = t / per_group;
  const int first_m = g * GROUP_M;
  const int gsize = min(num_m - first_m, GROUP_M);
  const int r = t - g * per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

// Epilogue math for 32 consecutive columns of one row:
//   v = act(acc * m_c + a_c) * post_mul  [* gate]  [+ residual * res_scale]
// with m_c = alpha * col_scale[c] * pre_mul and a_c = bias[c] * pre_mul + pre_add (the
// affine step of (alpha acc col_scale + bias) pre_mul + pre_add folded per column; lane j
// of the warp holds column col0 + j's m_c / a_c, broadcast by shuffle); tracks |v| (amax)
// and the row sum.  Returns the f32 values before the store.
__device__ __forceinline__ void epi_values(const EpilogueParams& ep, float alpha, int row,
                                           int col0, int M, int N, const uint32_t (&acc)[32],
                                           float (&v)[32], float& rowsum, float& amax_local,
                                           float lane_add, float lane_mul) {
  const bool row_ok = row < M;
  const float m = alpha * ep.pre_mul;  // uniform multiplier (no column scale)
  const float a = ep.pre_add;          // uniform addend (no bias)
  switch (ep.act) {  // uniform branch, once per 32 columns
    case kActNone: affine_act32_sel<kActNone>(ep, acc, v, m, a, lane_mul, lane_add); break;
    case kActRelu: affine_act32_sel<kActRelu>(ep, acc, v, m, a, lane_mul, lane_add); break;
    case kActGeluTanh: affine_act32_sel<kActGeluTanh>(ep, acc, v, m, a, lane_mul, lane_add); break;
    default: affine_act32<kActDyn, true>(acc, v, m, a, lane_mul, lane_add, ep.act, ep.act_param,
                                         ep.post_mul);
  }
  const bool in_n = row_ok && (col0 + 32 <= N);
  if (ep.gate != nullptr && row_ok) {
    const bool full = in_n && ep.gate_vec;
    if (ep.gate_dtype == kOutF32) {
      const float* gp = reinterpret_cast<const float*>(ep.gate) + (long long)row * ep.gate_ld + col0;
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 q = __ldcs(reinterpret_cast<const float4*>(gp + j));
          v[j] *= q.x; v[j + 1] *= q.y; v[j + 2] *= q.z; v[j + 3] *= q.w;
        }
      } else {
        for (int j = 0; j < 32; ++j)
          if (col0 + j < N) v[j] *= gp[j];
      }
    } else {
      const __nv_bfloat16* gp =
          reinterpret_cast<const __nv_bfloat16*>(ep.gate) + (long long)row * ep.gate_ld + col0;
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          const uint4 q = __ldcs(reinterpret_cast<const uint4*>(gp + j));
          const float2 a = unpack_bf16x2(q.x), b = unpack_bf16x2(q.y), c = unpack_bf16x2(q.z),
                       d = unpack_bf16x2(q.w);
          v[j] *= a.x; v[j + 1] *= a.y; v[j + 2] *= b.x; v[j + 3] *= b.y;
          v[j + 4] *= c.x; v[j + 5] *= c.y; v[j + 6] *= d.x; v[j + 7] *= d.y;
        }
      } else {
        for (int j = 0; j < 32; ++j)
          if (col0 + j < N) v[j] *= __bfloat162float(gp[j]);
      }
    }
  }
  if (ep.residual != nullptr && row_ok) {
    const bool full = in_n && ep.res_vec;
    const float2 rs2 = make_float2(ep.res_scale, ep.res_scale);
    if (ep.res_dtype == kOutBF16) {
      const __nv_bfloat16* rp =
          reinterpret_cast<const __nv_bfloat16*>(ep.residual) + (long long)row * ep.res_ld + col0;
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 q = *reinterpret_cast<const uint4*>(rp + j);
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float2 r = ffma2(unpack_bf16x2(w[t]), rs2,
                                   make_float2(v[j + 2 * t], v[j + 2 * t + 1]));
            v[j + 2 * t] = r.x;
            v[j + 2 * t + 1] = r.y;
          }
        }
      } else {
        for (int j = 0; j < 32; ++j)
          if (col0 + j < N) v[j] += __bfloat162float(rp[j]) * ep.res_scale;
      }
    } else if (ep.res_dtype == kOutF32) {
      const float* rp = reinterpret_cast<const float*>(ep.residual) + (long long)row * ep.res_ld + col0;
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 q = *reinterpret_cast<const float4*>(rp + j);
          const float2 r0 = ffma2(make_float2(q.x, q.y), rs2, make_float2(v[j], v[j + 1]));
          const float2 r1 = ffma2(make_float2(q.z, q.w), rs2, make_float2(v[j + 2], v[j + 3]));
          v[j] = r0.x; v[j + 1] = r0.y; v[j + 2] = r1.x; v[j + 3] = r1.y;
        }
      } else {
        for (int j = 0; j < 32; ++j)
          if (col0 + j < N) v[j] += rp[j] * ep.res_scale;
      }
    } else {
      const uint8_t* rp = reinterpret_cast<const uint8_t*>(ep.residual) + (long long)row * ep.res_ld + col0;
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) v[j] += e4m3_to_f32(rp[j]) * ep.res_scale;
    }
  }
  if (ep.amax != nullptr && row_ok) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < N) amax_local = fmaxf(amax_local, fabsf(v[j]));
  }
  if (ep.mode == kModeRowSum && row_ok) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < N) rowsum += v[j];
  }
}

// Packs 32 f32 values into the output type: 16 (f32: 32, e4m3: 8) 32-bit words.
__device__ __forceinline__ void epi_pack(const EpilogueParams& ep, const float (&v)[32],
                                         uint32_t (&w)[32]) {
  const float s = ep.out_inv_scale;
  if (ep.out_dtype == kOutBF16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) w[j] = pack_bf16x2(v[2 * j] * s, v[2 * j + 1] * s);
  } else if (ep.out_dtype == kOutF32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(v[j] * s);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      w[j] = uint32_t(f32x2_to_e4m3x2(v[4 * j] * s, v[4 * j + 1] * s)) |
             (uint32_t(f32x2_to_e4m3x2(v[4 * j + 2] * s, v[4 * j + 3] * s)) << 16);
  }
}

// Fallback store for outputs whose base or row pitch is not 16-byte aligned.
__device__ __forceinline__ void epi_store_direct(const EpilogueParams& ep, int row, int col0,
                                                 int N, const float (&v)[32]) {
  const float s = ep.out_inv_scale;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (col0 + j >= N) continue;
    const long long o = (long long)row * ep.out_ld + col0 + j;
    if (ep.out_dtype == kOutBF16)
      reinterpret_cast<__nv_bfloat16*>(ep.out)[o] = __float2bfloat16_rn(v[j] * s);
    else if (ep.out_dtype == kOutF32)
      reinterpret_cast<float*>(ep.out)[o] = v[j] * s;
    else
      reinterpret_cast<uint8_t*>(ep.out)[o] =
          static_cast<uint8_t>(f32x2_to_e4m3x2(v[j] * s, 0.0f) & 0xFF);
  }
}

// Bytes per output element and columns per 128-byte staging row.
__device__ __forceinline__ int out_esize(int dt) { return dt == kOutF32 ? 4 : (dt == kOutBF16 ? 2 : 1); }

// Drains one 128 x BN accumulator (this warp: 32 TMEM lanes = 32 rows) through the fused
// epilogue.  Output goes through a per-warp, double-buffered 32 x 128-byte shared-memory
// staging tile in the 128B-swizzle layout and leaves with TMA bulk-tensor stores (full
// 128-byte lines, clipped at the M/N edges by the TMA unit).  `stage` points at this
// warp's 2 x 4 KB staging area (1024-byte aligned).
// Split-K workspace layout: each 32-row x 32-column block of a slice is 1024 contiguous
// floats ordered [column / 4][row % 32][column % 4], so a warp (32 rows) moving one float4
// column group touches 512 contiguous bytes.  Offset of the block holding (row0, col0),
// row0 and col0 multiples of 32, within a slice:
__device__ __forceinline__ long long splitk_block(const EpilogueParams& ep, int row0, int col0) {
  return (long long)row0 * ep.ws_ld + (long long)col0 * 32;
}

// Split-K drain of this warp's 32 rows x HALF columns: the f32 partial tile of K slice
// `sk` goes to its own workspace slice (plain 16-byte stores; no atomics, so the final sum
// has a fixed order and results are bitwise reproducible).
template <int HALF>
__device__ __forceinline__ void splitk_store(const EpilogueParams& ep, uint32_t t_row, int row0,
                                             int col_base, int sk) {
  const int lane = threadIdx.x & 31;
  float* w = ep.ws + (long long)sk * ep.ws_slice;
#pragma unroll 1
  for (int c = 0; c < HALF; c += 32) {
    uint32_t r[32];
    tmem_ld32(t_row + c, r);
    float* blk = w + splitk_block(ep, row0, col_base + c) + lane * 4;
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      __stcg(reinterpret_cast<float4*>(blk + j * 32),
             make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                         __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3])));
  }
}

// Two-slice split-K, second slice: adds the other slice's partial tile (workspace slice
// `sk`) into this warp's 32 rows x HALF columns of the tensor-memory accumulator, which then
// drains through the normal epilogue (two addends: the same bits in either order).
template <int HALF>
__device__ __forceinline__ void splitk_accumulate(const EpilogueParams& ep, uint32_t t_row,
                                                  int row0, int col_base, int sk) {
  const int lane = threadIdx.x & 31;
  const float* w = ep.ws + (long long)sk * ep.ws_slice;
#pragma unroll 1
  for (int c = 0; c < HALF; c += 32) {
    uint32_t r[32];
    tmem_ld32_async(t_row + c, r);
    const float* blk = w + splitk_block(ep, row0, col_base + c) + lane * 4;
    float4 pv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) pv[j] = __ldcg(reinterpret_cast<const float4*>(blk + j * 128));
    tmem_ld_wait_regs(r);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      r[4 * j] = __float_as_uint(__uint_as_float(r[4 * j]) + pv[j].x);
      r[4 * j + 1] = __float_as_uint(__uint_as_float(r[4 * j + 1]) + pv[j].y);
      r[4 * j + 2] = __float_as_uint(__uint_as_float(r[4 * j + 2]) + pv[j].z);
      r[4 * j + 3] = __float_as_uint(__uint_as_float(r[4 * j + 3]) + pv[j].w);
    }
    tmem_st16p(t_row + c, r);
    tmem_st16p(t_row + c + 16, r + 16);
  }
  tmem_st_wait();
}

// Pulls this lane's residual row segment [col_base, col_base + HALF) into L2 while the
// accumulator is still being computed, so the epilogue's residual loads hit L2.
template <int HALF>
__device__ __forceinline__ void epi_prefetch_residual(const EpilogueParams& ep, int row,
                                                      int col_base, int M, int N) {
  if (row >= M || col_base >= N) return;
  const int cols = min(HALF, N - col_base);
  if (ep.residual != nullptr) {
    const int esz = ep.res_dtype == kOutF32 ? 4 : (ep.res_dtype == kOutBF16 ? 2 : 1);
    const uint8_t* p = reinterpret_cast<const uint8_t*>(ep.residual) +
                       ((long long)row * ep.res_ld + col_base) * esz;
    for (int off = 0; off < cols * esz; off += 32)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p + off));
  }
  if (ep.gate != nullptr) {
    const int esz = ep.gate_dtype == kOutF32 ? 4 : 2;
    const uint8_t* p = reinterpret_cast<const uint8_t*>(ep.gate) +
                       ((long long)row * ep.gate_ld + col_base) * esz;
    for (int off = 0; off < cols * esz; off += 32)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p + off));
  }
}

// Per-lane epilogue vectors for the 32 columns starting at col0 (one coalesced load each),
// folded with the affine step: lane_add = bias[c] * pre_mul + pre_add and lane_mul =
// alpha * col_scale[c] * pre_mul for this lane's column c.
__device__ __forceinline__ void epi_lane_vectors(const EpilogueParams& ep, float alpha, int col0,
                                                 int N, float& lane_add, float& lane_mul) {
  const int c = col0 + (threadIdx.x & 31);
  const float bias = (ep.bias != nullptr && c < N) ? __ldg(ep.bias + c) : 0.f;
  const float cs = (ep.col_scale != nullptr && c < N) ? __ldg(ep.col_scale + c) : 1.f;
  lane_add = fmaf(bias, ep.pre_mul, ep.pre_add);
  lane_mul = alpha * cs * ep.pre_mul;
}

// Drains one 128 x BN accumulator (this warp: 32 TMEM lanes = 32 rows) through the fused
// epilogue.  TMEM loads are software-pipelined (the load of columns u+1 is in flight while
// columns u are processed).  Output goes through a per-warp, double-buffered 32 x 128-byte
// shared-memory staging tile in the 128B-swizzle layout and leaves with TMA bulk-tensor
// stores (full 128-byte lines, clipped at the M/N edges by the TMA unit).  `stage` points
// at this warp's 4 KB staging area (1024-byte aligned).
//
// SRC selects where the accumulator chunks come from: 0 = tensor memory; 1 = the workspace,
// K slices 0..slice_arg-1 summed in order (the last slice of a split-K tile).
template <int BN, int SRC = 0>
__device__ __forceinline__ void epilogue_tile(const EpilogueParams& ep, const CUtensorMap* tmap_out,
                                              float alpha, uint32_t t_row, int row, int row0,
                                              int col_base, int M, int N, uint8_t* stage,
                                              int& buf, float& rowsum, float& amax_local,
                                              const float (&lbv)[BN / 32],
                                              const float (&lcv)[BN / 32], int slice_arg = 0) {
  const int lane = threadIdx.x & 31;
  const bool tma = ep.out_vec && ep.mode == kModeStore;
  const int esz = out_esize(ep.out_dtype);
  const int cb = ep.chunk_bytes;                 // staging row / TMA box width in bytes
  const int subs = tma ? (cb / esz) / 32 : 1;    // 32-column units per staging row
  const int g = 2 * esz;                         // 16-byte granules per unit
  int units = BN / 32;
  const int n_left = N - col_base;
  if (n_left < BN) units = (n_left + 31) / 32;   // columns past N are skipped (uniform)
  // One 32-column TMEM load in flight at a time: a second buffer (prefetching the next
  // chunk) pushed the 168-register budget into spills, which cost more than the exposed
  // load latency (measured on the K = 768 GEMMs of the GPT-2 block).
  uint32_t cur[32];
#pragma unroll 1
  for (int uu = 0; uu < units; ++uu) {
    {
      const int col0 = col_base + uu * 32;
      // this chunk's bias / column scale (loaded before the accumulator was ready)
      float lb = lbv[0], lc = lcv[0];
#pragma unroll
      for (int x = 1; x < BN / 32; ++x)
        if (uu == x) { lb = lbv[x]; lc = lcv[x]; }
      if constexpr (SRC == 1) {
        float sum[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) sum[j] = 0.f;
        const float* blk = ep.ws + splitk_block(ep, row0, col0) + lane * 4;
#pragma unroll 1
        for (int sk = 0; sk < slice_arg; ++sk) {
          const float* bs = blk + (long long)sk * ep.ws_slice;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(bs + j * 32));
            sum[j] += v.x; sum[j + 1] += v.y; sum[j + 2] += v.z; sum[j + 3] += v.w;
          }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) cur[j] = __float_as_uint(sum[j]);
      } else {
        tmem_ld32_async(t_row + uu * 32, cur);
        tmem_ld_wait_regs(cur);
      }
      float v[32];
      epi_values(ep, alpha, row, col0, M, N, cur, v, rowsum, amax_local, lb, lc);
      if (ep.mode == kModeRowSum) continue;
      if (!tma) {
        if (row < M) epi_store_direct(ep, row, col0, N, v);
        continue;
      }
      const int sub = uu % subs;
      uint8_t* sbuf = stage;
      if (sub == 0) {
        // The previous chunk's TMA store must have finished reading the staging buffer.
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
      }
      uint32_t w[32];
      epi_pack(ep, v, w);
      // swizzled staging row: 128B pattern (granule ^ row%8) or 64B (granule ^ (row/2)%4)
      uint8_t* rowp = sbuf + lane * cb;
      const int sw = (cb == 128) ? (lane & 7) : ((lane >> 1) & 3);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (q < g) {
          const int gi = sub * g + q;
          *reinterpret_cast<uint4*>(rowp + ((gi ^ sw) << 4)) =
              make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
        }
      }
      if (sub == subs - 1 || uu == units - 1) {
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tmap_out, sbuf, (col_base + (uu - sub) * 32) * esz, row0);
          bulk_commit();
        }
        buf ^= 1;
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// Fused attention-operand preparation (HeadPrepParams) for one 128-column half-tile.

// Kernel feature bits: each launch runs the instance with only the code it needs (the
// split-K protocol and the head preparation would otherwise sit in every GEMM's instruction
// stream; the short-K GEMMs measured instruction-fetch stalls as their largest stall).
enum : int { kFeatSplitK = 1, kFeatHeadPrep = 2 };

// Which head (if any) the half-tile starting at column c0 is: 1 = q, 2 = k, 3 = v, 0 = none.
__device__ __forceinline__ int head_prep_kind(const HeadPrepParams& h, int c0, int& head) {
  if (!h.on) return 0;
  if (c0 >= h.q_off && c0 < h.q_off + h.q_heads * h.q_hstride &&
      (c0 - h.q_off) % h.q_hstride == 0) {
    head = (c0 - h.q_off) / h.q_hstride;
    return 1;
  }
  if (c0 >= h.k_off && c0 < h.k_off + h.k_heads * 128 && (c0 - h.k_off) % 128 == 0) {
    head = (c0 - h.k_off) / 128;
    return 2;
  }
  if (c0 >= h.v_off && c0 < h.v_off + h.v_heads * 128 && (c0 - h.v_off) % 128 == 0) {
    head = (c0 - h.v_off) / 128;
    return 3;
  }
  return 0;
}

// Columns [e0, e0 + 16) of this lane's row as the projection's e4m3 codes (as f32): acc *
// (alpha * col_scale) + bias (the multiplier / addend of column e0 + j in lane (e0 + j) % 32
// of `lane_mul` / `lane_add`), rounded to e4m3 at the projection's scale exactly as the
// ordinary epilogue stores it.
__device__ __forceinline__ void head_prep_codes16(uint32_t taddr, float lane_mul,
                                                  float lane_add, bool add, int lo,
                                                  float inv_scale, float (&code)[16]) {
  uint32_t r[16];
  tmem_ld16(taddr, r);
#pragma unroll
  for (int j = 0; j < 16; j += 2) {
    const float2 m2 = make_float2(__shfl_sync(0xffffffffu, lane_mul, lo + j),
                                  __shfl_sync(0xffffffffu, lane_mul, lo + j + 1));
    const float2 a2 = add ? make_float2(__shfl_sync(0xffffffffu, lane_add, lo + j),
                                        __shfl_sync(0xffffffffu, lane_add, lo + j + 1))
                          : make_float2(0.f, 0.f);
    const float2 v = ffma2(make_float2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])), m2,
                           a2);
    const float2 c = e4m3x2_to_f32x2(f32x2_to_e4m3x2(v.x * inv_scale, v.y * inv_scale));
    code[j] = c.x;
    code[j + 1] = c.y;
  }
}

// q / k half-tile: RMSNorm over the head (f32 sum of squares in the order of the standalone
// head-norm kernel: eight 16-column partial sums combined pairwise), weight, RoPE
// (rotate_half: column e pairs with e + 64), e4m3 store.  `lm` / `la` hold the lane multipliers /
// addends of the half-tile's four 32-column chunks.
__device__ __forceinline__ void head_prep_qk(const HeadPrepParams& h, uint32_t t_row, int row,
                                             int M, const float* w, uint8_t* dst,
                                             const float (&lm)[4], const float (&la)[4],
                                             bool add, float inv_scale) {
  float inv = 1.0f;
  if (w != nullptr) {
    float part[8];
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      float code[16];
      head_prep_codes16(t_row + s * 16, lm[s >> 1], la[s >> 1], add, (s & 1) * 16, inv_scale,
                        code);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float x = code[e] * h.x_scale;
        ss = fmaf(x, x, ss);
      }
      part[s] = ss;
    }
    const float ss = ((part[0] + part[1]) + (part[2] + part[3])) +
                     ((part[4] + part[5]) + (part[6] + part[7]));
    inv = rsqrtf(ss / 128.0f + h.eps);
  }
  const bool rope = h.cos != nullptr;
  const long long pos = rope ? (long long)(row % h.seq) * 128 : 0;
#pragma unroll 1
  for (int s = 0; s < 4; ++s) {  // columns [16 s, 16 s + 16) and their partners + 64
    float a[16], b[16];
    head_prep_codes16(t_row + s * 16, lm[s >> 1], la[s >> 1], add, (s & 1) * 16, inv_scale,
                      a);
    head_prep_codes16(t_row + 64 + s * 16, lm[2 + (s >> 1)], la[2 + (s >> 1)], add,
                      (s & 1) * 16, inv_scale, b);
    uint32_t oa[4], ob[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int e = s * 16 + g * 4;
      float4 wa = make_float4(1.f, 1.f, 1.f, 1.f), wb = wa;
      if (w != nullptr) {
        wa = __ldg(reinterpret_cast<const float4*>(w + e));
        wb = __ldg(reinterpret_cast<const float4*>(w + e + 64));
        wa.x += h.w_offset; wa.y += h.w_offset; wa.z += h.w_offset; wa.w += h.w_offset;
        wb.x += h.w_offset; wb.y += h.w_offset; wb.z += h.w_offset; wb.w += h.w_offset;
      }
      const float wav[4] = {wa.x, wa.y, wa.z, wa.w}, wbv[4] = {wb.x, wb.y, wb.z, wb.w};
      float ya[4], yb[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        ya[t] = a[g * 4 + t] * h.x_scale;
        yb[t] = b[g * 4 + t] * h.x_scale;
        if (w != nullptr) {
          ya[t] = ya[t] * inv * wav[t];
          yb[t] = yb[t] * inv * wbv[t];
        }
      }
      if (rope) {
        // (each lane reads its own row's tables: these loads do not coalesce, which makes
        // RoPE in this epilogue slower than in a separate launch)
        const float4 ca = __ldg(reinterpret_cast<const float4*>(h.cos + pos + e));
        const float4 sa = __ldg(reinterpret_cast<const float4*>(h.sin + pos + e));
        const float4 cb = __ldg(reinterpret_cast<const float4*>(h.cos + pos + e + 64));
        const float4 sb = __ldg(reinterpret_cast<const float4*>(h.sin + pos + e + 64));
        const float cav[4] = {ca.x, ca.y, ca.z, ca.w}, sav[4] = {sa.x, sa.y, sa.z, sa.w};
        const float cbv[4] = {cb.x, cb.y, cb.z, cb.w}, sbv[4] = {sb.x, sb.y, sb.z, sb.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float xa = ya[t], xb = yb[t];
          ya[t] = xa * cav[t] + xb * (-1.0f * sav[t]);
          yb[t] = xb * cbv[t] + xa * (1.0f * sbv[t]);
        }
      }
      oa[g] = uint32_t(f32x2_to_e4m3x2(ya[0] * h.out_inv_scale, ya[1] * h.out_inv_scale)) |
              (uint32_t(f32x2_to_e4m3x2(ya[2] * h.out_inv_scale, ya[3] * h.out_inv_scale)) << 16);
      ob[g] = uint32_t(f32x2_to_e4m3x2(yb[0] * h.out_inv_scale, yb[1] * h.out_inv_scale)) |
              (uint32_t(f32x2_to_e4m3x2(yb[2] * h.out_inv_scale, yb[3] * h.out_inv_scale)) << 16);
    }
    if (row < M) {
      *reinterpret_cast<uint4*>(dst + s * 16) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
      *reinterpret_cast<uint4*>(dst + 64 + s * 16) = make_uint4(ob[0], ob[1], ob[2], ob[3]);
    }
  }
}

// v half-tile: the e4m3 codes as 16-bit floats (exact), 128 columns of this lane's row.
__device__ __forceinline__ void head_prep_v(const HeadPrepParams& h, uint32_t t_row, int row,
                                            int M, uint16_t* dst, const float (&lm)[4],
                                            const float (&la)[4], bool add, float inv_scale) {
#pragma unroll 1
  for (int s = 0; s < 8; ++s) {
    float code[16];
    head_prep_codes16(t_row + s * 16, lm[s >> 1], la[s >> 1], add, (s & 1) * 16, inv_scale,
                        code);
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      o[j] = h.v_f16 ? pack_f16x2(code[2 * j], code[2 * j + 1])
                     : pack_bf16x2(code[2 * j], code[2 * j + 1]);
    if (row < M) {
      *reinterpret_cast<uint4*>(dst + s * 16) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(dst + s * 16 + 8) = make_uint4(o[4], o[5], o[6], o[7]);
    }
  }
}

// One 128- or HALF-column half-tile of the accumulator to its destination: a q / k / v head
// of a fused preparation (HeadPrepParams, 128-column halves only), else the ordinary
// epilogue.
template <int HALF, bool HP>
__device__ __forceinline__ void drain_half(const EpilogueParams& ep, const CUtensorMap* tmap_out,
                                           float alpha, uint32_t t_row, int row, int row0,
                                           int col_base, int M, int N, uint8_t* stage, int& buf,
                                           float& rowsum, float& amax_local,
                                           const float (&lbv)[HALF / 32],
                                           const float (&lcv)[HALF / 32]) {
  if constexpr (HP && HALF == 128) {
    int head = 0;
    const int kind = head_prep_kind(ep.hp, col_base, head);
    if (kind != 0) {
      const HeadPrepParams& hp = ep.hp;
      const bool add = ep.bias != nullptr;
      if (kind == 3) {
        head_prep_v(hp, t_row, row, M, hp.v_out + (long long)row * hp.v_ld + head * 128, lcv,
                    lbv, add, ep.out_inv_scale);
      } else {
        const bool isq = kind == 1;
        uint8_t* dst = isq ? hp.q_out + (long long)row * hp.q_ld + head * 128
                           : hp.k_out + (long long)row * hp.k_ld + head * 128;
        head_prep_qk(hp, t_row, row, M, isq ? hp.q_w : hp.k_w, dst, lcv, lbv, add,
                     ep.out_inv_scale);
      }
      return;
    }
  }
  epilogue_tile<HALF>(ep, tmap_out, alpha, t_row, row, row0, col_base, M, N, stage, buf, rowsum,
                      amax_local, lbv, lcv);
}

template <int BN, int FEAT>
__global__ void __launch_bounds__(320, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b,
                    const __grid_constant__ CUtensorMap tmap_out, const GemmShape shape,
                    const EpilogueParams ep) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * Cfg::A_BYTES;
  uint8_t* smem_stage = smem + STAGES * Cfg::STAGE_BYTES;  // 8 warps x 4 KB
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem_stage + 4 * 8192);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2]
  uint64_t* drain_bar = tempty_bar + 2;       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = shape.M, N = shape.N, K = shape.K;
  const int num_m = (M + Cfg::BM - 1) / Cfg::BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + Cfg::BK - 1) / Cfg::BK;
  const int splits = (FEAT & kFeatSplitK) ? shape.splits : 1;
  const int num_units = num_tiles * splits;  // unit u: tile u / splits, K slice u % splits
  uint64_t* split_done = drain_bar + 8;       // 8 epilogue warps finished their partials
  uint64_t* split_flag_bar = split_done + 1;  // "is this the tile's last slice" published
  uint64_t* split_ready = split_flag_bar + 1; // two slices: the other slice's partial is in
  volatile int* split_last = abort_flag + 1;
  volatile int* split_ok = abort_flag + 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 8);
    }
    mbar_init(split_done, 8);
    mbar_init(split_flag_bar, 1);
    mbar_init(split_ready, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if (ep.out_vec && ep.mode == kModeStore) tma_prefetch_desc(&tmap_out);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // set-up above overlaps the previous kernel; global memory only from here

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const int t = u / splits, sk = u - t * splits;
        int mb, nb;
        tile_coords(t, num_m, num_n, shape.group_m, mb, nb);
        const int kb0 = (sk * num_kb) / splits, kb1 = ((sk + 1) * num_kb) / splits;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, kDevTimeoutProducer, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          tma_load_2d(smem_a + stage * Cfg::A_BYTES, &tmap_a, &full_bar[stage], kb * Cfg::BK,
                      mb * Cfg::BM, pol_a);
          tma_load_2d(smem_b + stage * Cfg::B_BYTES, &tmap_b, &full_bar[stage], kb * Cfg::BK,
                      nb * BN, pol_b);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: every issued copy must have landed before the CTA may exit.
      const long long pending = issued < STAGES ? issued : STAGES;
      for (long long i = 0; i < pending; ++i) {
        if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
        uint64_t t0 = globaltimer();
        while (!mbar_test(&full_bar[stage], phase)) {
          if (globaltimer() - t0 > B2F_WAIT_NS) { record_error(kDevTimeoutDrain); break; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = make_idesc_f8(Cfg::BM, BN);
      // Operand descriptors built once (stage 0); each MMA adds an immediate.
      const uint64_t a_desc0 = make_sdesc_sw128(smem_u32(smem_a), 1024);
      const uint64_t b_desc0 = make_sdesc_sw128(smem_u32(smem_b), 1024);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++it) {
        const int sk = u % splits;
        const int kb0 = (sk * num_kb) / splits, kb1 = ((sk + 1) * num_kb) / splits;
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, kDevTimeoutMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, kDevTimeoutMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // descriptor = stage-0 descriptor + (byte offset / 16) in the address field
          const uint64_t ad0 = a_desc0 + uint64_t(stage * (Cfg::A_BYTES >> 4));
          const uint64_t bd0 = b_desc0 + uint64_t(stage * (Cfg::B_BYTES >> 4));
          mma_f8(d_tmem, ad0, bd0, idesc, kb != kb0 ? 1u : 0u);
#pragma unroll
          for (int k = 1; k < Cfg::BK / 32; ++k)
            mma_f8(d_tmem, ad0 + 2 * k, bd0 + 2 * k, idesc, 1u);
          mma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) mma_commit(&tfull_bar[acc]);
      }
      // Drain: wait until every issued MMA retired before TMEM is released.
      mma_commit(drain_bar);
      uint64_t t0 = globaltimer();
      while (!mbar_test(drain_bar, 0)) {
        if (globaltimer() - t0 > B2F_WAIT_NS) { record_error(kDevTimeoutDrain); break; }
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int ew = warp - 2;                 // epilogue warp 0..7
    const int chalf = ew >> 2;               // which half of the tile's columns
    uint8_t* stage = smem_stage + ew * 4096;
    int buf = 0;
    float alpha = ep.alpha;
    if (ep.alpha_ptr != nullptr) alpha *= *ep.alpha_ptr;
    float amax_local = 0.0f;
    int it = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++it) {
      const int t = u / splits;
      int mb, nb;
      tile_coords(t, num_m, num_n, shape.group_m, mb, nb);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      float lbv[BN / 64], lcv[BN / 64];
      {
        const int cb0 = nb * BN + chalf * (BN / 2);
        epi_prefetch_residual<BN / 2>(ep, mb * Cfg::BM + q * 32 + lane, cb0, M, N);
#pragma unroll
        for (int x = 0; x < BN / 64; ++x) epi_lane_vectors(ep, alpha, cb0 + x * 32, N, lbv[x], lcv[x]);
      }
      // tcgen05.ld is warp-collective: the whole warp leaves together or not at all.
      if (!__all_sync(0xffffffffu,
                      mbar_wait(&tfull_bar[acc], acc_phase, kDevTimeoutEpilogue, abort_flag)))
        break;
      tc_fence_after();
      const int row0 = mb * Cfg::BM + q * 32;
      const int row = row0 + lane;
      const int col_base = nb * BN + chalf * (BN / 2);
      float rowsum = 0.0f;
      const uint32_t t_row = tmem_base + (uint32_t(q * 32) << 16) + acc * BN + chalf * (BN / 2);
      bool slice_last = splits == 1;  // this CTA writes the tile's output
      bool drain_tmem = splits == 1;  // the output leaves from this CTA's accumulator
      if (splits == 2) {
        // Two K slices: arrival order is settled first.  The first slice stores its partial
        // tile and then sets the ready bit; the second waits for it (the first is resident
        // and waits on nothing, so the wait ends) and adds that partial to its own
        // accumulator on the way through the epilogue.  counters[t]: +1 per arrival, +4
        // once the partial is visible; the second slice resets it.
        const uint32_t sp = it & 1;
        const int sk = u - t * splits;
        if (ew == 0) {
          if (lane == 0) {
            const unsigned old = splitk_arrive(&ep.counters[t], ep.epoch, 1u);
            *split_last = (old & 3u) == 1u;
            mbar_arrive(split_flag_bar);
          }
          __syncwarp();
        }
        if (!__all_sync(0xffffffffu,
                        mbar_wait(split_flag_bar, sp, kDevTimeoutEpilogue, abort_flag)))
          break;
        slice_last = *split_last;
        if (!slice_last) {
          splitk_store<BN / 2>(ep, t_row, row0, col_base, sk);
          tc_fence_before();
          __threadfence();  // this thread's partials are visible before the ready bit
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&tempty_bar[acc]);
            mbar_arrive(split_done);
          }
          if (ew == 0) {
            const bool okw = mbar_wait(split_done, sp, kDevTimeoutEpilogue, abort_flag);
            if (lane == 0) {
              if (okw) {
                __threadfence();
                splitk_arrive(&ep.counters[t], ep.epoch, 4u);
              }
              mbar_arrive(split_ready);
            }
            __syncwarp();
          }
        } else {
          if (ew == 0) {
            if (lane == 0) {
              int okr = 0;
              const uint64_t t0 = globaltimer();
              while (true) {
                if (splitk_state(&ep.counters[t], ep.epoch) & 4u) { okr = 1; break; }
                if (*abort_flag || globaltimer() - t0 > B2F_WAIT_NS) {
                  record_error(kDevTimeoutEpilogue);
                  *abort_flag = 1;
                  break;
                }
              }
              if (okr) {
                __threadfence();
                ep.counters[t] = 0u;  // both slices arrived and the first is done with it
              }
              *split_ok = okr;
              mbar_arrive(split_ready);
            }
            __syncwarp();
          }
          if (!__all_sync(0xffffffffu,
                          mbar_wait(split_ready, sp, kDevTimeoutEpilogue, abort_flag)) ||
              !*split_ok)
            break;
          __threadfence();
          splitk_accumulate<BN / 2>(ep, t_row, row0, col_base, 1 - sk);
          if (lane == 0) mbar_arrive(split_done);  // (keeps the phase in step with `it`)
          drain_tmem = true;
        }
      } else if (splits > 2) {
        splitk_store<BN / 2>(ep, t_row, row0, col_base, u - t * splits);
        tc_fence_before();
        __threadfence();  // this thread's partials are visible before the tile counter moves
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&tempty_bar[acc]);
          mbar_arrive(split_done);
        }
        const uint32_t sp = it & 1;
        if (ew == 0) {
          bool okw = mbar_wait(split_done, sp, kDevTimeoutEpilogue, abort_flag);
          if (lane == 0) {
            int last = 0;
            if (okw) {
              __threadfence();
              last = splitk_arrive(&ep.counters[t], ep.epoch, 1u) == (unsigned)(splits - 1);
              if (last) {
                __threadfence();
                ep.counters[t] = 0u;  // reset for the next call (every slice has arrived)
              }
            }
            *split_last = last;
            mbar_arrive(split_flag_bar);
          }
          __syncwarp();
        }
        if (!__all_sync(0xffffffffu,
                        mbar_wait(split_flag_bar, sp, kDevTimeoutEpilogue, abort_flag)))
          break;
        slice_last = *split_last;
        if (slice_last) {
          __threadfence();
          epilogue_tile<BN / 2, 1>(ep, &tmap_out, alpha, t_row, row, row0, col_base, M, N,
                                   stage, buf, rowsum, amax_local, lbv, lcv, splits);
        }
      }
      if (drain_tmem) {
        drain_half<BN / 2, (FEAT & kFeatHeadPrep) != 0>(ep, &tmap_out, alpha, t_row, row, row0, col_base, M, N, stage, buf,
                           rowsum, amax_local, lbv, lcv);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      }
      if (ep.mode == kModeRowSum && row < M && slice_last)
        atomicAdd(reinterpret_cast<float*>(ep.out) + row, rowsum * ep.out_inv_scale);
    }
    if (lane == 0) bulk_wait_all();  // output stores complete before the CTA exits
    if (ep.amax != nullptr) {
      amax_local = warp_max(amax_local);
      if (lane == 0) atomic_max_nonneg(ep.amax, amax_local);
    }
  }

  pdl_trigger();  // this CTA's work is issued: the next kernel may be scheduled
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------------------
// CTA-pair variant (cluster of 2, tcgen05 cta_group::2): the pair owns a 256 x BN output
// tile (BN 256, or 128 where 256-wide tiles leave most of a wave idle).  CTA r loads A rows
// [128 r, 128 r + 128) and B rows [BN/2 r, BN/2 (r + 1)) of the tile; the leader (r = 0)
// issues M=256, N=BN, K=32 MMAs that read both CTAs' shared memory, and each CTA's TMEM
// receives its own 128 rows x BN columns.  Per SM this moves
// half the B bytes of the single-CTA kernel for the same MMA work.  TMA loads are plain
// (no multicast); only tcgen05.commit multicasts its arrive to both CTAs.
template <int BN_>
struct Gemm2Cfg {
  static constexpr int BM = 128;   // rows per CTA (256 per pair)
  static constexpr int BN = BN_;   // columns per pair tile (BN / 2 B rows per CTA)
  static constexpr int BK = 128;
  static constexpr int STAGES = BN == 256 ? 6 : 8;
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = (BN / 2) * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 4 * 8192 + 1024 + 256;
  static constexpr int THREADS = 320;  // producer, MMA, 8 epilogue warps
  static_assert(BN == 128 || BN == 256, "pair tiles are 256 x 128 or 256 x 256");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
};

template <int PBN, int FEAT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    gemm_fp8_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                         const __grid_constant__ CUtensorMap tmap_b,
                         const __grid_constant__ CUtensorMap tmap_out, const GemmShape shape,
                         const EpilogueParams ep) {
  using Cfg = Gemm2Cfg<PBN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int BN = Cfg::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * Cfg::A_BYTES;
  uint8_t* smem_stage = smem + STAGES * Cfg::STAGE_BYTES;  // 8 warps x 4 KB
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem_stage + 4 * 8192);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;      // [2]  (leader's are used)
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int M = shape.M, N = shape.N, K = shape.K;
  const int num_m = (M + 2 * Cfg::BM - 1) / (2 * Cfg::BM);
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + Cfg::BK - 1) / Cfg::BK;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 16);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if (ep.out_vec && ep.mode == kModeStore) tma_prefetch_desc(&tmap_out);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // set-up above overlaps the previous kernel; global memory only from here

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer (both CTAs)
      const uint64_t pol = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += num_pairs) {
        int mb, nb;
        tile_coords(t, num_m, num_n, shape.group_m, mb, nb);
        const int row_a = mb * 2 * Cfg::BM + rank * Cfg::BM;
        const int row_b = nb * BN + rank * (BN / 2);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, kDevTimeoutProducer, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = map_to_rank(&full_bar[stage], 0);
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::STAGE_BYTES);
          tma_load_2d_pair(smem_a + stage * Cfg::A_BYTES, &tmap_a, fb, kb * Cfg::BK, row_a, pol);
          tma_load_2d_pair(smem_b + stage * Cfg::B_BYTES, &tmap_b, fb, kb * Cfg::BK, row_b, pol);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (rank == 0) {
        const long long pending = issued < STAGES ? issued : STAGES;
        for (long long i = 0; i < pending; ++i) {
          if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
          const uint64_t t0 = globaltimer();
          while (!mbar_test(&full_bar[stage], phase)) {
            if (globaltimer() - t0 > B2F_WAIT_NS) { record_error(kDevTimeoutDrain); break; }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------------------------------------ MMA issuer (leader)
      constexpr uint32_t idesc = make_idesc_f8(2 * Cfg::BM, BN);
      const uint64_t a_desc0 = make_sdesc_sw128(smem_u32(smem_a), 1024);
      const uint64_t b_desc0 = make_sdesc_sw128(smem_u32(smem_b), 1024);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += num_pairs, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, kDevTimeoutMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, kDevTimeoutMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad0 = a_desc0 + uint64_t(stage * (Cfg::A_BYTES >> 4));
          const uint64_t bd0 = b_desc0 + uint64_t(stage * (Cfg::B_BYTES >> 4));
          mma_f8_pair(d_tmem, ad0, bd0, idesc, kb != 0);
#pragma unroll
          for (int k = 1; k < Cfg::BK / 32; ++k)
            mma_f8_pair(d_tmem, ad0 + 2 * k, bd0 + 2 * k, idesc, 1u);
          mma_commit_pair(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) mma_commit_pair(&tfull_bar[acc]);
      }
      mma_commit_pair(drain_bar);
      const uint64_t t0 = globaltimer();
      while (!mbar_test(drain_bar, 0)) {
        if (globaltimer() - t0 > B2F_WAIT_NS) { record_error(kDevTimeoutDrain); break; }
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue (both CTAs)
    const int q = warp & 3;
    const int ew = warp - 2;                 // epilogue warp 0..7
    const int chalf = ew >> 2;               // which half of the tile's columns
    uint8_t* stage = smem_stage + ew * 4096;
    int buf = 0;
    float alpha = ep.alpha;
    if (ep.alpha_ptr != nullptr) alpha *= *ep.alpha_ptr;
    float amax_local = 0.0f;
    int it = 0;
    for (int t = pair; t < num_tiles; t += num_pairs, ++it) {
      int mb, nb;
      tile_coords(t, num_m, num_n, shape.group_m, mb, nb);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      float lbv[BN / 64], lcv[BN / 64];
      {
        const int cb0 = nb * BN + chalf * (BN / 2);
        epi_prefetch_residual<BN / 2>(ep, mb * 2 * Cfg::BM + rank * Cfg::BM + q * 32 + lane, cb0,
                                      M, N);
#pragma unroll
        for (int x = 0; x < BN / 64; ++x) epi_lane_vectors(ep, alpha, cb0 + x * 32, N, lbv[x], lcv[x]);
      }
      // tcgen05.ld is warp-collective: the whole warp leaves together or not at all.
      if (!__all_sync(0xffffffffu,
                      mbar_wait(&tfull_bar[acc], acc_phase, kDevTimeoutEpilogue, abort_flag)))
        break;
      tc_fence_after();
      const int row0 = mb * 2 * Cfg::BM + rank * Cfg::BM + q * 32;
      const int row = row0 + lane;
      float rowsum = 0.0f;
      const uint32_t t_row = tmem_base + (uint32_t(q * 32) << 16) + acc * BN + chalf * (BN / 2);
      drain_half<BN / 2, (FEAT & kFeatHeadPrep) != 0>(ep, &tmap_out, alpha, t_row, row, row0,
                                                      nb * BN + chalf * (BN / 2), M, N, stage,
                                                      buf, rowsum, amax_local, lbv, lcv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(map_to_rank(&tempty_bar[acc], 0));
      if (ep.mode == kModeRowSum && row < M)
        atomicAdd(reinterpret_cast<float*>(ep.out) + row, rowsum * ep.out_inv_scale);
    }
    if (lane == 0) bulk_wait_all();  // output stores complete before the CTA exits
    if (ep.amax != nullptr) {
      amax_local = warp_max(amax_local);
      if (lane == 0) atomic_max_nonneg(ep.amax, amax_local);
    }
  }

  pdl_trigger();  // this CTA's work is issued: the next kernel may be scheduled
  __syncwarp();
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace b2f
