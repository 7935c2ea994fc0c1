// Attention operand preparation (C ABI: b2f_head_norm_rope, b2f_fp8_to_bf16, b2f_fp8_to_f16).
//
// b2f_head_norm_rope: one warp per token, heads streamed through it:
//   x = stored * in_scale; y = x * rsqrt(mean(x^2) + eps) * (w + w_offset)   (optional)
//   rotate-half RoPE on the first rotary_dim dims with cos/sin[pos], pos = token % seq
//   out = e4m3(y / out_scale) into a dense [T, H * D] tensor.
// Reference: _cute_harness_rms_norm / _cute_harness_apply_rope
// (tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:167-183, applied at :365-376).
//
// b2f_fp8_to_bf16: copies an e4m3 column block to bf16 (the exact image of the e4m3
// values: bf16 holds every e4m3 value), used for the V operand of the P.V MMA.
#include <string>

#include "common.cuh"
#include "host_common.h"

namespace b2f {
namespace {

struct RopeParams {
  const uint8_t* in;
  long long in_ld, in_hstride;
  float in_scale;
  const float* weight;  // [D] f32 or null (no norm)
  float w_offset, eps;
  const float* cos;     // [seq, rotary] f32 or null (no RoPE)
  const float* sin;
  int rotary, seq;
  uint8_t* out;
  long long out_ld;
  float out_inv_scale;
  int rows, heads;
};

// One warp per token: the token's cos / sin row and the norm weights are loaded once (as
// vectors) and reused for every head; the heads stream through HB at a time (their loads
// issued together).  Lane l holds elements [l*E, l*E + E) of a head; the rotate-half
// partner of element i sits in lane l +- (rotary/2)/E.
#ifndef B2F_ROPE_HB
#define B2F_ROPE_HB 4
#endif
template <int D>
__global__ void __launch_bounds__(256) head_norm_rope_kernel(const RopeParams p) {
  pdl_wait();
  constexpr int E = D / 32;  // elements per lane
  constexpr int W = (E + 3) / 4;  // 32-bit words per lane
  // Heads whose loads are in flight together (measured at D = 128, [8192 x 32 heads]:
  // 4 -> 25.6 us, 16 -> 33.2 us, the extra registers costing more occupancy than the
  // deeper loads gain).
  constexpr int HB = B2F_ROPE_HB;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= p.rows) return;
  const int i0 = lane * E;
  float w[E], cs[E], sn[E];
#pragma unroll
  for (int e = 0; e < E; ++e) { w[e] = 1.0f; cs[e] = 1.0f; sn[e] = 0.0f; }
  if (p.weight != nullptr) {
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const float2 v = *reinterpret_cast<const float2*>(p.weight + i0 + e);
      w[e] = v.x + p.w_offset;
      w[e + 1] = v.y + p.w_offset;
    }
  }
  const bool rope = p.cos != nullptr;
  const int half = p.rotary / 2;
  const int off = rope ? half / E : 0;  // lane distance between rotation partners
  if (rope && i0 < p.rotary) {
    const long long base = (long long)(t % p.seq) * p.rotary + i0;
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const float2 c = *reinterpret_cast<const float2*>(p.cos + base + e);
      const float2 sv = *reinterpret_cast<const float2*>(p.sin + base + e);
      cs[e] = c.x; cs[e + 1] = c.y;
      sn[e] = (i0 + e < half) ? -sv.x : sv.x;  // rotate_half sign folded into sin
      sn[e + 1] = (i0 + e + 1 < half) ? -sv.y : sv.y;
    }
  }
  const int src_lane = (i0 < half) ? lane + off : lane - off;
  const uint8_t* row_in = p.in + (long long)t * p.in_ld + i0;
  uint8_t* row_out = p.out + (long long)t * p.out_ld + i0;
  for (int h0 = 0; h0 < p.heads; h0 += HB) {
    uint32_t raw[HB][W];
#pragma unroll
    for (int hb = 0; hb < HB; ++hb) {
      if (h0 + hb < p.heads) {
        const uint8_t* src = row_in + (long long)(h0 + hb) * p.in_hstride;
        if constexpr (E == 2) {
          raw[hb][0] = *reinterpret_cast<const uint16_t*>(src);
        } else if constexpr (E == 4) {
          raw[hb][0] = *reinterpret_cast<const uint32_t*>(src);
        } else {
          const uint2 q = *reinterpret_cast<const uint2*>(src);
          raw[hb][0] = q.x;
          raw[hb][1] = q.y;
        }
      }
    }
#pragma unroll
    for (int hb = 0; hb < HB; ++hb) {
      if (h0 + hb >= p.heads) break;  // warp-uniform
      float x[E];
#pragma unroll
      for (int e = 0; e < E; e += 2) {
        const float2 v = e4m3x2_to_f32x2((raw[hb][e / 4] >> (8 * (e % 4))) & 0xFFFF);
        x[e] = v.x * p.in_scale;
        x[e + 1] = v.y * p.in_scale;
      }
      if (p.weight != nullptr) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) ss += x[e] * x[e];
        ss = warp_sum(ss);
        const float inv = rsqrtf(ss / float(D) + p.eps);
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = x[e] * inv * w[e];
      }
      if (rope) {
        float y[E];
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float partner = __shfl_sync(0xffffffffu, x[e], src_lane & 31);
          y[e] = (i0 + e < p.rotary) ? x[e] * cs[e] + partner * sn[e] : x[e];
        }
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = y[e];
      }
      uint32_t packed[W] = {};
#pragma unroll
      for (int e = 0; e < E; e += 2)
        packed[e / 4] |= uint32_t(f32x2_to_e4m3x2(x[e] * p.out_inv_scale,
                                                  x[e + 1] * p.out_inv_scale))
                         << (8 * (e % 4));
      uint8_t* dst = row_out + (long long)(h0 + hb) * D;
      if constexpr (E == 2) {
        *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(packed[0]);
      } else if constexpr (E == 4) {
        *reinterpret_cast<uint32_t*>(dst) = packed[0];
      } else {
        *reinterpret_cast<uint2*>(dst) = make_uint2(packed[0], packed[1]);
      }
    }
  }
}

// head_dim 128 with full-width (or no) RoPE, heads in groups of four: lane l owns the 16
// elements [16 (l % 8), 16 (l % 8) + 16) of head 4 g + l / 8 in every group g, so one
// 16-byte load per lane moves four heads and the whole token row is in flight before any
// arithmetic; the norm reduces over the 8 lanes of a head and the rotate-half partner
// (element i +- 64) sits in lane l ^ 4.  Same formulas as head_norm_rope_kernel (the
// f32 sum of squares runs in another order).
template <int G>
__device__ __forceinline__ void head_norm_rope128_token(const RopeParams& p, int t, int lane) {
  const int sub = lane & 7;
  const int hg = lane >> 3;
  const int i0 = sub * 16;
  const uint8_t* src = p.in + (long long)t * p.in_ld + (long long)hg * p.in_hstride + i0;
  uint4 raw[G];
#pragma unroll
  for (int g = 0; g < G; ++g)
    raw[g] = *reinterpret_cast<const uint4*>(src + (long long)(4 * g) * p.in_hstride);
  float w[16], cs[16], sn[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) { w[e] = 1.0f; cs[e] = 1.0f; sn[e] = 0.0f; }
  if (p.weight != nullptr) {
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      const float4 v = *reinterpret_cast<const float4*>(p.weight + i0 + e);
      w[e] = v.x + p.w_offset; w[e + 1] = v.y + p.w_offset;
      w[e + 2] = v.z + p.w_offset; w[e + 3] = v.w + p.w_offset;
    }
  }
  const bool rope = p.cos != nullptr;
  if (rope) {
    const long long base = (long long)(t % p.seq) * 128 + i0;
    const float sg = sub < 4 ? -1.0f : 1.0f;  // rotate_half sign folded into sin
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      const float4 c = *reinterpret_cast<const float4*>(p.cos + base + e);
      const float4 sv = *reinterpret_cast<const float4*>(p.sin + base + e);
      cs[e] = c.x; cs[e + 1] = c.y; cs[e + 2] = c.z; cs[e + 3] = c.w;
      sn[e] = sg * sv.x; sn[e + 1] = sg * sv.y; sn[e + 2] = sg * sv.z; sn[e + 3] = sg * sv.w;
    }
  }
  uint8_t* dst = p.out + (long long)t * p.out_ld + (long long)hg * 128 + i0;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float x[16];
    const uint32_t wd[4] = {raw[g].x, raw[g].y, raw[g].z, raw[g].w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 a = e4m3x2_to_f32x2(wd[q] & 0xFFFF);
      const float2 b = e4m3x2_to_f32x2(wd[q] >> 16);
      x[4 * q] = a.x * p.in_scale; x[4 * q + 1] = a.y * p.in_scale;
      x[4 * q + 2] = b.x * p.in_scale; x[4 * q + 3] = b.y * p.in_scale;
    }
    if (p.weight != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) ss += x[e] * x[e];
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      ss += __shfl_xor_sync(0xffffffffu, ss, 4);
      const float inv = rsqrtf(ss / 128.0f + p.eps);
#pragma unroll
      for (int e = 0; e < 16; ++e) x[e] = x[e] * inv * w[e];
    }
    if (rope) {
      float y[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, x[e], 4);
        y[e] = x[e] * cs[e] + partner * sn[e];
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) x[e] = y[e];
    }
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      o[q] = uint32_t(f32x2_to_e4m3x2(x[4 * q] * p.out_inv_scale,
                                      x[4 * q + 1] * p.out_inv_scale)) |
             (uint32_t(f32x2_to_e4m3x2(x[4 * q + 2] * p.out_inv_scale,
                                       x[4 * q + 3] * p.out_inv_scale))
              << 16);
    *reinterpret_cast<uint4*>(dst + (long long)(4 * g) * 128) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int G>
__global__ void __launch_bounds__(256) head_norm_rope128_kernel(const RopeParams p) {
  pdl_wait();
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t < p.rows) head_norm_rope128_token<G>(p, t, threadIdx.x & 31);
}

// q and k of one token in one warp (head_dim 128, rotate-half RoPE over the whole head or
// none): lane (hg = lane / 8, sub = lane % 8) holds elements [8 sub, 8 sub + 8) and their
// rotate-half partners [8 sub + 64, 8 sub + 72) of heads 4 g + hg, so the rotation needs no
// shuffles; the token's cos / sin values are loaded once for the q and the k heads; all
// arithmetic on f32 pairs (fma.rn.f32x2 / mul.rn.f32x2).  The per-head sum of squares runs
// over the lane's 16 values (pairs) and then the 8 lanes of the head.
struct QkLane {
  float2 c[8], sn[8];  // cos / sin of the lane's elements: [0..3] low block, [4..7] high
};

template <int G>
__device__ __forceinline__ void qk_heads128(const RopeParams& p, const QkLane& tb, bool rope,
                                            int t, int hg, int e0) {
  const uint8_t* src = p.in + (long long)t * p.in_ld + (long long)hg * p.in_hstride + e0;
  uint2 lo[G], hi[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    lo[g] = *reinterpret_cast<const uint2*>(src + (long long)(4 * g) * p.in_hstride);
    hi[g] = *reinterpret_cast<const uint2*>(src + (long long)(4 * g) * p.in_hstride + 64);
  }
  float2 w[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) w[u] = make_float2(1.f, 1.f);
  if (p.weight != nullptr) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p.weight + e0));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p.weight + e0 + 4));
    const float4 c = __ldg(reinterpret_cast<const float4*>(p.weight + e0 + 64));
    const float4 d = __ldg(reinterpret_cast<const float4*>(p.weight + e0 + 68));
    const float2 off = make_float2(p.w_offset, p.w_offset);
    w[0] = fadd2(make_float2(a.x, a.y), off); w[1] = fadd2(make_float2(a.z, a.w), off);
    w[2] = fadd2(make_float2(b.x, b.y), off); w[3] = fadd2(make_float2(b.z, b.w), off);
    w[4] = fadd2(make_float2(c.x, c.y), off); w[5] = fadd2(make_float2(c.z, c.w), off);
    w[6] = fadd2(make_float2(d.x, d.y), off); w[7] = fadd2(make_float2(d.z, d.w), off);
  }
  const float2 isc = make_float2(p.in_scale, p.in_scale);
  const float2 osc = make_float2(p.out_inv_scale, p.out_inv_scale);
  uint8_t* dst = p.out + (long long)t * p.out_ld + (long long)hg * 128 + e0;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float2 x[8];
    const uint32_t wd[4] = {lo[g].x, lo[g].y, hi[g].x, hi[g].y};
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      x[2 * q4] = fmul2(e4m3x2_to_f32x2(wd[q4] & 0xFFFF), isc);
      x[2 * q4 + 1] = fmul2(e4m3x2_to_f32x2(wd[q4] >> 16), isc);
    }
    if (p.weight != nullptr) {
      float2 ss = make_float2(0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 8; ++u) ss = ffma2(x[u], x[u], ss);
      float sum = ss.x + ss.y;
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      const float inv = rsqrtf(sum / 128.0f + p.eps);
      const float2 inv2 = make_float2(inv, inv);
#pragma unroll
      for (int u = 0; u < 8; ++u) x[u] = fmul2(fmul2(x[u], inv2), w[u]);
    }
    if (rope) {
      // low element e: x_e cos_e - x_{e+64} sin_e; high element e+64: x_{e+64} cos + x_e sin
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 xl = x[u], xh = x[u + 4];
        x[u] = ffma2(xh, make_float2(-tb.sn[u].x, -tb.sn[u].y), fmul2(xl, tb.c[u]));
        x[u + 4] = ffma2(xl, tb.sn[u + 4], fmul2(xh, tb.c[u + 4]));
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 a = fmul2(x[2 * u], osc), b = fmul2(x[2 * u + 1], osc);
      o[u] = uint32_t(f32x2_to_e4m3x2(a.x, a.y)) | (uint32_t(f32x2_to_e4m3x2(b.x, b.y)) << 16);
    }
    *reinterpret_cast<uint2*>(dst + (long long)(4 * g) * 128) = make_uint2(o[0], o[1]);
    *reinterpret_cast<uint2*>(dst + (long long)(4 * g) * 128 + 64) = make_uint2(o[2], o[3]);
  }
}

template <int GQ, int GK>
__device__ __forceinline__ void qk_token128(const RopeParams& q, const RopeParams& k, int t,
                                            int lane) {
  const int hg = lane >> 3, e0 = (lane & 7) * 8;
  const bool rope = q.cos != nullptr;
  QkLane tb;
  if (rope) {
    const long long base = (long long)(t % q.seq) * 128 + e0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // low block, then the + 64 block
      const float4 c0 = __ldg(reinterpret_cast<const float4*>(q.cos + base + 64 * h));
      const float4 c1 = __ldg(reinterpret_cast<const float4*>(q.cos + base + 64 * h + 4));
      const float4 s0 = __ldg(reinterpret_cast<const float4*>(q.sin + base + 64 * h));
      const float4 s1 = __ldg(reinterpret_cast<const float4*>(q.sin + base + 64 * h + 4));
      tb.c[4 * h] = make_float2(c0.x, c0.y); tb.c[4 * h + 1] = make_float2(c0.z, c0.w);
      tb.c[4 * h + 2] = make_float2(c1.x, c1.y); tb.c[4 * h + 3] = make_float2(c1.z, c1.w);
      tb.sn[4 * h] = make_float2(s0.x, s0.y); tb.sn[4 * h + 1] = make_float2(s0.z, s0.w);
      tb.sn[4 * h + 2] = make_float2(s1.x, s1.y); tb.sn[4 * h + 3] = make_float2(s1.z, s1.w);
    }
  }
  qk_heads128<GQ>(q, tb, rope, t, hg, e0);
  qk_heads128<GK>(k, tb, rope, t, hg, e0);
}

template <bool F16>
__device__ __forceinline__ void fp8_convert8(const uint8_t* in, long long in_ld, uint16_t* out,
                                             long long out_ld, int rows, int cols, float scale,
                                             long long i) {
  const int vec_per_row = cols / 8;
  if (i >= (long long)rows * vec_per_row) return;
  const int r = int(i / vec_per_row);
  const int c = int(i - (long long)r * vec_per_row) * 8;
  const uint2 q = *reinterpret_cast<const uint2*>(in + (long long)r * in_ld + c);
  const float2 a = e4m3x2_to_f32x2(q.x & 0xFFFF), b = e4m3x2_to_f32x2(q.x >> 16),
               cc = e4m3x2_to_f32x2(q.y & 0xFFFF), d = e4m3x2_to_f32x2(q.y >> 16);
  uint4 o;
  if constexpr (F16) {
    o.x = pack_f16x2(a.x * scale, a.y * scale);
    o.y = pack_f16x2(b.x * scale, b.y * scale);
    o.z = pack_f16x2(cc.x * scale, cc.y * scale);
    o.w = pack_f16x2(d.x * scale, d.y * scale);
  } else {
    o.x = pack_bf16x2(a.x * scale, a.y * scale);
    o.y = pack_bf16x2(b.x * scale, b.y * scale);
    o.z = pack_bf16x2(cc.x * scale, cc.y * scale);
    o.w = pack_bf16x2(d.x * scale, d.y * scale);
  }
  *reinterpret_cast<uint4*>(out + (long long)r * out_ld + c) = o;
}

template <bool F16>
__global__ void fp8_to_bf16_kernel(const uint8_t* in, long long in_ld, uint16_t* out,
                                   long long out_ld, int rows, int cols, float scale) {
  pdl_wait();
  fp8_convert8<F16>(in, in_ld, out, out_ld, rows, cols, scale,
                    (long long)blockIdx.x * blockDim.x + threadIdx.x);
}

// The three operand preparations of a gated GQA block in one launch: blocks [0, nq) run
// the q and k head norm + RoPE (one warp per token: GQ and GK four-head groups), the rest
// convert V to f16 / bf16 (none when V was written elsewhere).  One launch instead of
// three: each of them alone is too short to fill the GPU past its ramp and tail.
struct VConvertParams {
  const uint8_t* in;
  long long in_ld;
  uint16_t* out;
  long long out_ld;
  int rows, cols;
  int f16;
};

template <int GQ, int GK>
__global__ void __launch_bounds__(256, 2) attn_prep_kernel(const RopeParams q, const RopeParams k,
                                                        const VConvertParams v, int nq) {
  pdl_wait();
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31;
  if (b < nq) {
    const int t = b * 8 + (threadIdx.x >> 5);
    if (t < q.rows) qk_token128<GQ, GK>(q, k, t, lane);
  } else {
    const long long i = (long long)(b - nq) * blockDim.x + threadIdx.x;
    if (v.f16) fp8_convert8<true>(v.in, v.in_ld, v.out, v.out_ld, v.rows, v.cols, 1.0f, i);
    else fp8_convert8<false>(v.in, v.in_ld, v.out, v.out_ld, v.rows, v.cols, 1.0f, i);
  }
}

// out = e4m3( silu(gate * in_scale) * (up * in_scale) / out_scale ), 8 elements per thread.
__global__ void swiglu_kernel(const uint8_t* gate, long long gate_ld, const uint8_t* up,
                              long long up_ld, uint8_t* out, long long out_ld, int rows, int cols,
                              float in_scale, float out_inv_scale) {
  pdl_wait();
  const int vec_per_row = cols / 8;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)rows * vec_per_row) return;
  const int r = int(i / vec_per_row);
  const int c = int(i - (long long)r * vec_per_row) * 8;
  const uint2 g = *reinterpret_cast<const uint2*>(gate + (long long)r * gate_ld + c);
  const uint2 u = *reinterpret_cast<const uint2*>(up + (long long)r * up_ld + c);
  const uint32_t gw[2] = {g.x, g.y}, uw[2] = {u.x, u.y};
  uint32_t ow[2];
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    float res[4];
#pragma unroll
    for (int hlf = 0; hlf < 2; ++hlf) {
      const float2 gg = e4m3x2_to_f32x2((gw[w] >> (16 * hlf)) & 0xFFFF);
      const float2 uu = e4m3x2_to_f32x2((uw[w] >> (16 * hlf)) & 0xFFFF);
      const float g0 = gg.x * in_scale, g1 = gg.y * in_scale;
      res[2 * hlf] = g0 / (1.0f + expf(-g0)) * (uu.x * in_scale);
      res[2 * hlf + 1] = g1 / (1.0f + expf(-g1)) * (uu.y * in_scale);
    }
    ow[w] = uint32_t(f32x2_to_e4m3x2(res[0] * out_inv_scale, res[1] * out_inv_scale)) |
            (uint32_t(f32x2_to_e4m3x2(res[2] * out_inv_scale, res[3] * out_inv_scale)) << 16);
  }
  *reinterpret_cast<uint2*>(out + (long long)r * out_ld + c) = make_uint2(ow[0], ow[1]);
}

}  // namespace
}  // namespace b2f

extern "C" {

int b2f_swiglu_fp8(const void* gate, long long gate_ld, const void* up, long long up_ld,
                   void* out, long long out_ld, int rows, int cols, float in_scale,
                   float out_scale, b2f_stream_t stream) {
  using namespace b2f;
  if (rows <= 0 || cols <= 0) return fail(B2F_ERR_ARG, "swiglu: empty shape");
  if (gate == nullptr || up == nullptr || out == nullptr) return fail(B2F_ERR_ARG, "swiglu: null tensor");
  if (cols % 8 || gate_ld % 8 || up_ld % 8 || out_ld % 8 || ((uintptr_t)gate & 7) ||
      ((uintptr_t)up & 7) || ((uintptr_t)out & 7))
    return fail(B2F_ERR_ARG, "swiglu: cols/ld multiples of 8, 8-byte aligned tensors required");
  if (!(out_scale > 0.f)) return fail(B2F_ERR_ARG, "swiglu: out_scale must be > 0");
  const long long n = (long long)rows * (cols / 8);
  B2F_CUDA_TRY(launch_pdl(swiglu_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                          (cudaStream_t)stream, reinterpret_cast<const uint8_t*>(gate), gate_ld,
                          reinterpret_cast<const uint8_t*>(up), up_ld,
                          reinterpret_cast<uint8_t*>(out), out_ld, rows, cols, in_scale,
                          1.0f / out_scale));
  return B2F_OK;
}

}  // extern "C"

namespace b2f {
namespace {
// Validates a b2f_head_norm_rope argument block and fills the kernel parameters.
int rope_params(const b2f_rope_args* a, RopeParams& p) {
  if (a == nullptr) return fail(B2F_ERR_ARG, "head_norm_rope: null args");
  if (a->rows <= 0 || a->heads <= 0) return fail(B2F_ERR_ARG, "head_norm_rope: empty shape");
  const int d = a->head_dim;
  if (d != 64 && d != 128 && d != 256)
    return fail(B2F_ERR_UNSUPPORTED, "head_norm_rope: head_dim must be 64, 128 or 256");
  if (a->in == nullptr || a->out == nullptr) return fail(B2F_ERR_ARG, "head_norm_rope: null tensor");
  if (a->cos != nullptr) {
    if (a->sin == nullptr || a->seq <= 0)
      return fail(B2F_ERR_ARG, "head_norm_rope: cos needs sin and seq");
    const int e = d / 32;
    if (a->rotary_dim <= 0 || a->rotary_dim > d || a->rotary_dim % (2 * e) != 0)
      return fail(B2F_ERR_ARG, "head_norm_rope: rotary_dim must be a multiple of 2*head_dim/32");
  }
  const long long al = d / 32;  // bytes per lane: rows and heads must keep lane loads aligned
  if (((a->in_ld | a->in_head_stride | a->out_ld) % al) || ((uintptr_t)a->in % al) ||
      ((uintptr_t)a->out % al))
    return fail(B2F_ERR_ARG, "head_norm_rope: pointers and pitches must be multiples of head_dim/32");
  if (!(a->out_scale > 0.f)) return fail(B2F_ERR_ARG, "head_norm_rope: out_scale must be > 0");
  p.in = reinterpret_cast<const uint8_t*>(a->in);
  p.in_ld = a->in_ld; p.in_hstride = a->in_head_stride; p.in_scale = a->in_scale;
  p.weight = a->weight; p.w_offset = a->weight_offset; p.eps = a->eps;
  p.cos = a->cos; p.sin = a->sin; p.rotary = a->rotary_dim;
  p.seq = a->seq > 0 ? a->seq : a->rows;
  p.out = reinterpret_cast<uint8_t*>(a->out); p.out_ld = a->out_ld;
  p.out_inv_scale = 1.0f / a->out_scale;
  p.rows = a->rows; p.heads = a->heads;
  if ((a->weight != nullptr && (reinterpret_cast<uintptr_t>(a->weight) & 7)) ||
      (a->cos != nullptr && ((reinterpret_cast<uintptr_t>(a->cos) & 7) ||
                             (reinterpret_cast<uintptr_t>(a->sin) & 7) || (a->rotary_dim % 2))))
    return fail(B2F_ERR_ARG, "head_norm_rope: weight / cos / sin must be 8-byte aligned");
  return B2F_OK;
}

bool al16p(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; }

// The 128-wide layout (four heads per 16-byte lane load) applies: head_dim 128, heads a
// multiple of 4, full-width or no RoPE, 16-byte aligned rows, heads and tables.
bool rope128_ok(const b2f_rope_args* a) {
  return a->head_dim == 128 && a->heads % 4 == 0 && a->heads <= 32 &&
         (a->cos == nullptr || a->rotary_dim == 128) && a->in_ld % 16 == 0 &&
         a->in_head_stride % 16 == 0 && a->out_ld % 16 == 0 && al16p(a->in) &&
         al16p(a->out) && (a->weight == nullptr || al16p(a->weight)) &&
         (a->cos == nullptr || (al16p(a->cos) && al16p(a->sin)));
}
}  // namespace
}  // namespace b2f

extern "C" {

int b2f_head_norm_rope(const b2f_rope_args* a, b2f_stream_t stream) {
  using namespace b2f;
  RopeParams p;
  if (int rc = rope_params(a, p)) return rc;
  const int d = a->head_dim;
  const int grid = (a->rows + 7) / 8;  // one warp per token
  cudaStream_t s = (cudaStream_t)stream;
  // 4-head groups pay off from 16 heads (measured [8192 tokens]: 32 heads 25.6 -> 21.1 us;
  // 8 heads 8.0 -> 11.8 us, the extra registers costing more than the wider loads gain)
  const bool fast128 = rope128_ok(a) && a->heads >= 16;
  if (fast128) {
    switch (a->heads / 4) {
      case 4: B2F_CUDA_TRY(launch_pdl(head_norm_rope128_kernel<4>, dim3(grid), dim3(256), 0, s, p)); break;
      case 5: B2F_CUDA_TRY(launch_pdl(head_norm_rope128_kernel<5>, dim3(grid), dim3(256), 0, s, p)); break;
      case 6: B2F_CUDA_TRY(launch_pdl(head_norm_rope128_kernel<6>, dim3(grid), dim3(256), 0, s, p)); break;
      case 7: B2F_CUDA_TRY(launch_pdl(head_norm_rope128_kernel<7>, dim3(grid), dim3(256), 0, s, p)); break;
      default: B2F_CUDA_TRY(launch_pdl(head_norm_rope128_kernel<8>, dim3(grid), dim3(256), 0, s, p)); break;
    }
  } else if (d == 64) B2F_CUDA_TRY(launch_pdl(head_norm_rope_kernel<64>, dim3(grid), dim3(256), 0, s, p));
  else if (d == 128) B2F_CUDA_TRY(launch_pdl(head_norm_rope_kernel<128>, dim3(grid), dim3(256), 0, s, p));
  else B2F_CUDA_TRY(launch_pdl(head_norm_rope_kernel<256>, dim3(grid), dim3(256), 0, s, p));
  B2F_CUDA_TRY(cudaGetLastError());
  return B2F_OK;
}

int b2f_attn_prep(const b2f_rope_args* q, const b2f_rope_args* k, const void* v_in,
                  long long v_in_ld, void* v_out, long long v_out_ld, int v_cols, int v_dtype,
                  b2f_stream_t stream) {
  using namespace b2f;
  if (q == nullptr || k == nullptr) return fail(B2F_ERR_ARG, "attn_prep: null args");
  RopeParams pq, pk;
  if (int rc = rope_params(q, pq)) return rc;
  if (int rc = rope_params(k, pk)) return rc;
  if (!rope128_ok(q) || !rope128_ok(k) || q->rows != k->rows || q->cos != k->cos ||
      q->sin != k->sin || (q->cos != nullptr && pq.seq != pk.seq))
    return fail(B2F_ERR_UNSUPPORTED,
                "attn_prep: q and k need head_dim 128, heads a multiple of 4 (<= 32), full or "
                "no RoPE with the same tables, 16-byte aligned rows, and the same token count");
  const bool has_v = v_in != nullptr || v_out != nullptr || v_cols != 0;
  if (has_v &&
      (v_in == nullptr || v_out == nullptr || v_cols <= 0 || v_cols % 8 || v_in_ld % 8 ||
       v_out_ld % 8 || ((uintptr_t)v_in & 7) || ((uintptr_t)v_out & 15) ||
       (v_dtype != B2F_DTYPE_F16 && v_dtype != B2F_DTYPE_BF16)))
    return fail(B2F_ERR_ARG, "attn_prep: V must be e4m3 -> f16 / bf16, cols and pitches "
                             "multiples of 8, aligned");
  VConvertParams pv{reinterpret_cast<const uint8_t*>(v_in), v_in_ld,
                    reinterpret_cast<uint16_t*>(v_out), v_out_ld, q->rows, v_cols,
                    v_dtype == B2F_DTYPE_F16 ? 1 : 0};
  const int nq = (q->rows + 7) / 8;  // one warp per token does its q and k heads
  const long long nv = has_v ? ((long long)q->rows * (v_cols / 8) + 255) / 256 : 0;
  const int grid = (int)(nq + nv);
  cudaStream_t s = (cudaStream_t)stream;
  const int gq = q->heads / 4, gk = k->heads / 4;
#define B2F_PREP(GQ, GK)                                                        \
  if (gq == GQ && gk == GK) {                                                   \
    B2F_CUDA_TRY(launch_pdl(attn_prep_kernel<GQ, GK>, dim3(grid), dim3(256), 0, s, pq, pk, pv, \
                            nq));                                                   \
    B2F_CUDA_TRY(cudaGetLastError());                                           \
    return B2F_OK;                                                              \
  }
  B2F_PREP(8, 2) B2F_PREP(4, 1) B2F_PREP(8, 1) B2F_PREP(4, 2) B2F_PREP(2, 1) B2F_PREP(8, 8)
  B2F_PREP(4, 4)
#undef B2F_PREP
  return fail(B2F_ERR_UNSUPPORTED, "attn_prep: head counts (q, k) not in the compiled set "
                                   "{(32,8), (16,4), (32,4), (16,8), (8,4), (32,32), (16,16)}");
}

static int fp8_convert(const void* in, long long in_ld, void* out, long long out_ld, int rows,
                       int cols, float scale, bool f16, b2f_stream_t stream) {
  using namespace b2f;
  const char* name = f16 ? "fp8_to_f16" : "fp8_to_bf16";
  if (rows <= 0 || cols <= 0) return fail(B2F_ERR_ARG, std::string(name) + ": empty shape");
  if (in == nullptr || out == nullptr) return fail(B2F_ERR_ARG, std::string(name) + ": null tensor");
  if (cols % 8 || in_ld % 8 || out_ld % 8 || ((uintptr_t)in & 7) || ((uintptr_t)out & 15))
    return fail(B2F_ERR_ARG,
                std::string(name) + ": cols/ld multiples of 8, aligned tensors required");
  const long long n = (long long)rows * (cols / 8);
  const int grid = (int)((n + 255) / 256);
  if (f16)
    B2F_CUDA_TRY(launch_pdl(fp8_to_bf16_kernel<true>, dim3(grid), dim3(256), 0,
                            (cudaStream_t)stream, reinterpret_cast<const uint8_t*>(in), in_ld,
                            reinterpret_cast<uint16_t*>(out), out_ld, rows, cols, scale));
  else
    B2F_CUDA_TRY(launch_pdl(fp8_to_bf16_kernel<false>, dim3(grid), dim3(256), 0,
                            (cudaStream_t)stream, reinterpret_cast<const uint8_t*>(in), in_ld,
                            reinterpret_cast<uint16_t*>(out), out_ld, rows, cols, scale));
  return B2F_OK;
}

int b2f_fp8_to_bf16(const void* in, long long in_ld, void* out, long long out_ld, int rows,
                    int cols, float scale, b2f_stream_t stream) {
  return fp8_convert(in, in_ld, out, out_ld, rows, cols, scale, false, stream);
}

int b2f_fp8_to_f16(const void* in, long long in_ld, void* out, long long out_ld, int rows,
                   int cols, float scale, b2f_stream_t stream) {
  return fp8_convert(in, in_ld, out, out_ld, rows, cols, scale, true, stream);
}

}  // extern "C"
