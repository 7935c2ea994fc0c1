// Fused FP8 attention on 5th-generation tensor cores (C ABI: b2f_attention_fp8).
//
// Per query tile of 128 rows and key tile j:
//   S_j  = Q . K_j^T            tcgen05.mma kind::f8f6f4 (e4m3 x e4m3 -> f32 in TMEM)
//   P_j  = exp2(S_j * scale*log2e - m)  in registers, online softmax with lazy rescaling
//          (the running max only moves when it grows by more than 2^8), P rounded to f16
//          with f16 V (bf16 with bf16 V); P goes back to shared memory (two-tile kernel)
//          or tensor memory over S_j (head_dim 256 kernel)
//   O   += P_j . V_j            tcgen05.mma kind::f16, V (exact bf16 / f16 image of the
//                               e4m3 values) MN-major from shared memory
//   ctx  = e4m3( O / l * sigmoid(gate) / ctx_scale )   fused epilogue
// Two kernels:
//   attention2_kernel<D, VF16> (head_dim 64 / 128): two query tiles per CTA, 128-key
//     tiles, P through shared memory, S released as soon as the softmax loaded it (384
//     threads: TMA producer warp, MMA warp, two idle warps, two softmax warpgroups); the
//     two tiles are GQA head pairs sharing K / V,
//     or two heads with their own K / V at the same query rows (causal, head_dim 64), or
//     causal query tiles (i, n-1-i) of one head; e4m3 gate tiles by TMA.
//   attention_kernel<256> (head_dim 256): one query tile per CTA (192 threads), S
//     double-buffered in TMEM so Q.K_{j+1}^T runs while the softmax of tile j is computed.
// Causal tiles above the diagonal are never visited; GQA maps query head h to KV head
// h / (Hq / Hkv).
//
// Reference math: tasks/model_gpt2_small_transformer_block_fp8/starter.py:428-453 (GPT-2),
// tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:354-392 (Qwen, gated GQA),
// tasks/model_qwen35_4b_vision_block_fp8/starter.py:327-345 (non-causal).
#include <cstring>
#include <string>

#include "common.cuh"
#include "host_common.h"

namespace b2f {
namespace {

struct AttnParams {
  int seq, batch, hq, hkv;
  int causal;
  float qk_scale_log2;  // q_scale * k_scale * sm_scale * log2(e)
  const void* gate;     // optional [T, gate_ld], e4m3 or bf16
  int gate_dtype;
  long long gate_ld;
  long long gate_hstride;
  float gate_scale;
  uint8_t* ctx;         // e4m3 [T, ctx_ld], head h at column h * D
  long long ctx_ld;
  float ctx_inv_scale;
  float v_scale;        // V bf16 values are multiplied by v_scale in the epilogue
  int pair_heads;       // two-tile kernel: the tiles are query heads 2y, 2y+1 (same KV head)
  int pair_kv;          // two-tile kernel, head_dim 64, causal, one KV head per query head:
                        // the tiles are heads 2y, 2y+1 (each with its own K / V) at the same
                        // query rows, both K (V) tiles in one ring stage
  int gate_tma;         // two-tile kernel: e4m3 gate tiles arrive in shared memory by TMA
};

// sigmoid(g) from the hardware exponential and an approximate reciprocal: the product with
// the context is requantised to e4m3 (3 mantissa bits), far coarser than their error.
__device__ __forceinline__ float sigmoid_fast(float g) {
  return __fdividef(1.0f, 1.0f + __expf(-g));
}

__device__ __forceinline__ uint64_t make_sdesc(uint32_t addr, uint32_t layout, uint32_t lbo,
                                               uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFF);
  d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(layout & 7) << 61;
  return d;
}

template <int D>
struct AttnCfg {
  static constexpr int BQ = 128;
  static constexpr int BKV = (D == 256) ? 64 : 128;
  static constexpr int ST = (D == 256) ? 2 : 3;
  // e4m3 operand tiles: rows of min(D,128) bytes, D/128 k-blocks (1 for D=64)
  static constexpr int KB = (D >= 128) ? D / 128 : 1;
  static constexpr int ROWB = (D >= 128) ? 128 : D;
  static constexpr uint32_t LAYOUT8 = (ROWB == 128) ? 2u : 4u;  // SW128 / SW64
  static constexpr uint32_t SBO8 = 8 * ROWB;
  static constexpr int Q_BYTES = BQ * D;
  static constexpr int K_BYTES = BKV * D;
  static constexpr int V_BYTES = BKV * D * 2;  // bf16
  static constexpr int P_BYTES = BQ * BKV * 2;  // bf16
  static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
  static constexpr int SMEM_BYTES = Q_BYTES + ST * STAGE_BYTES + P_BYTES + 1024 + 512;
  static constexpr int S_COLS = BKV;
  static constexpr int O_COL = 2 * BKV;
  static constexpr int TMEM_COLS = 512;
  static_assert(2 * BKV + D <= 512, "TMEM budget");
};

template <int D>
__global__ void __launch_bounds__(192, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const AttnParams p) {
  using C = AttnCfg<D>;
  constexpr int BQ = C::BQ, BKV = C::BKV, ST = C::ST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* skv = sq + C::Q_BYTES;
  uint8_t* sp = skv + ST * C::STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sp + C::P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ST;
  uint64_t* s_full = kv_empty + ST;  // [2]
  uint64_t* s_free = s_full + 2;     // [2]
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 1;
  uint64_t* drain = pv_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.seq + BQ - 1) / BQ;
  const int qt = n_qt - 1 - blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hk = h / (p.hq / p.hkv);
  const int q0 = qt * BQ;
  const int kv_end = p.causal ? min(p.seq, q0 + BQ) : p.seq;
  const int nkv = (kv_end + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // set-up above overlaps the previous kernel; global memory only from here

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      const uint64_t pol = policy_evict_last();
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
      for (int kb = 0; kb < C::KB; ++kb)
        tma_load_3d(sq + kb * BQ * C::ROWB, &tm_q, q_full, h * D + kb * 128, q0, b, pol);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int j = 0; j < nkv; ++j) {
        if (!mbar_wait(&kv_empty[stage], phase ^ 1, kDevTimeoutProducer, abort_flag)) break;
        uint8_t* sk = skv + stage * C::STAGE_BYTES;
        uint8_t* sv = sk + C::K_BYTES;
        mbar_arrive_expect_tx(&kv_full[stage], C::STAGE_BYTES);
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_3d(sk + kb * BKV * C::ROWB, &tm_k, &kv_full[stage], hk * D + kb * 128,
                      j * BKV, b, pol);
        for (int vb = 0; vb < D / 64; ++vb)
          tma_load_3d(sv + vb * BKV * 128, &tm_v, &kv_full[stage], hk * D + vb * 64, j * BKV, b,
                      pol);
        ++issued;
        if (++stage == ST) { stage = 0; phase ^= 1; }
      }
      // drain outstanding copies before the CTA may exit
      const int pending = issued < ST ? issued : ST;
      for (int i = 0; i < pending; ++i) {
        if (--stage < 0) { stage = ST - 1; phase ^= 1; }
        const uint64_t t0 = globaltimer();
        while (!mbar_test(&kv_full[stage], phase))
          if (globaltimer() - t0 > B2F_WAIT_NS) { record_error(kDevTimeoutDrain); break; }
      }
      {
        const uint64_t t0 = globaltimer();
        while (!mbar_test(q_full, 0))
          if (globaltimer() - t0 > B2F_WAIT_NS) { record_error(kDevTimeoutDrain); break; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_s = make_idesc_f8(BQ, BKV);
      constexpr uint32_t idesc_pv = make_idesc_bf16(BQ, D, 1);
      bool ok = mbar_wait(q_full, 0, kDevTimeoutMma, abort_flag);
      const uint32_t q_addr = smem_u32(sq);
      auto issue_s = [&](int j) -> bool {
        const int st = j % ST;
        const uint32_t ph = (j / ST) & 1;
        if (!mbar_wait(&kv_full[st], ph, kDevTimeoutMma, abort_flag)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(skv + st * C::STAGE_BYTES);
        const uint32_t d_s = tmem + (j & 1) * C::S_COLS;
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb) {
#pragma unroll
          for (int k = 0; k < C::ROWB / 32; ++k) {
            const uint64_t ad =
                make_sdesc(q_addr + kb * BQ * C::ROWB + k * 32, C::LAYOUT8, 16, C::SBO8);
            const uint64_t bd =
                make_sdesc(k_addr + kb * BKV * C::ROWB + k * 32, C::LAYOUT8, 16, C::SBO8);
            mma_f8(d_s, ad, bd, idesc_s, (kb | k) != 0);
          }
        }
        mma_commit(&s_full[j & 1]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && nkv > 1) ok = issue_s(1);
      const uint32_t p_addr = smem_u32(sp);
      for (int j = 0; j < nkv && ok; ++j) {
        if (!mbar_wait(p_full, j & 1, kDevTimeoutMma, abort_flag)) break;
        tc_fence_after();
        const int st = j % ST;
        const uint32_t v_addr = smem_u32(skv + st * C::STAGE_BYTES + C::K_BYTES);
#pragma unroll
        for (int kb = 0; kb < BKV / 64; ++kb) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = make_sdesc(p_addr + kb * BQ * 128 + k * 32, 2, 16, 1024);
            const uint64_t bd = make_sdesc(v_addr + (kb * 4 + k) * 2048, 2, BKV * 128, 1024);
            mma_bf16(tmem + C::O_COL, ad, bd, idesc_pv, (j | kb | k) != 0);
          }
        }
        mma_commit(pv_done);
        mma_commit(&kv_empty[st]);
        if (j + 2 < nkv) {
          if (!mbar_wait(&s_free[j & 1], (j >> 1) & 1, kDevTimeoutMma, abort_flag)) break;
          if (!issue_s(j + 2)) break;
        }
      }
      mma_commit(drain);
      const uint64_t t0 = globaltimer();
      while (!mbar_test(drain, 0))
        if (globaltimer() - t0 > B2F_WAIT_NS) { record_error(kDevTimeoutDrain); break; }
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int qd = warp & 3;
    const int r = qd * 32 + lane;  // row within the tile == TMEM lane
    const int qi = q0 + r;         // query index within the sequence
    const uint32_t t_lane = tmem + (uint32_t(qd * 32) << 16);
    float m_used = -INFINITY;
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      // tcgen05.ld/st are warp-collective: every lane must take the same path.
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[j & 1], (j >> 1) & 1, kDevTimeoutEpilogue,
                                             abort_flag));
      if (!ok) break;
      tc_fence_after();
      float s[BKV];
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) {
        uint32_t raw[32];
        tmem_ld32(t_lane + (j & 1) * C::S_COLS + c * 32, raw);
#pragma unroll
        for (int u = 0; u < 32; ++u) s[c * 32 + u] = __uint_as_float(raw[u]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[j & 1]);
      const int k0 = j * BKV;
      const bool need_mask = (k0 + BKV > p.seq) || (p.causal && k0 + BKV - 1 > q0);
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < BKV; ++c) {
        float x = s[c] * p.qk_scale_log2;
        if (need_mask) {
          const int kidx = k0 + c;
          if (kidx >= p.seq || (p.causal && kidx > qi)) x = -INFINITY;
        }
        s[c] = x;
        mt = fmaxf(mt, x);
      }
      // lazy rescaling: keep the reference max unless the row max grew by more than 8
      float corr = 1.0f;
      bool rescale = false;
      if (mt > m_used + 8.0f) {
        if (m_used != -INFINITY) {
          corr = exp2f(m_used - mt);
          rescale = true;
        }
        m_used = mt;
      }
      const float mref = (m_used == -INFINITY) ? 0.0f : m_used;
      float lt = 0.f;
      uint32_t pk[BKV / 2];
#pragma unroll
      for (int c = 0; c < BKV; c += 2) {
        const float e0 = exp2f(s[c] - mref);
        const float e1 = exp2f(s[c + 1] - mref);
        const __nv_bfloat162 bb = __floats2bfloat162_rn(e0, e1);
        // the row sum uses the bf16-rounded weights, exactly what the P.V MMA sees
        const float2 rb = __bfloat1622float2(bb);
        lt += rb.x + rb.y;
        pk[c / 2] = *reinterpret_cast<const uint32_t*>(&bb);
      }
      if (j > 0) {
        ok = __all_sync(0xffffffffu,
                        mbar_wait(pv_done, (j - 1) & 1, kDevTimeoutEpilogue, abort_flag));
        if (!ok) break;
        tc_fence_after();
        // The rescale decision is per row; the TMEM round trip runs for the whole warp
        // (lanes that need no rescale multiply by corr == 1).
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
          for (int c = 0; c < D; c += 16) {
            uint32_t o[16];
            tmem_ld16(t_lane + C::O_COL + c, o);
#pragma unroll
            for (int u = 0; u < 16; ++u) o[u] = __float_as_uint(__uint_as_float(o[u]) * corr);
            tmem_st16(t_lane + C::O_COL + c, o);
          }
          tmem_st_wait();
        }
      }
      l = l * corr + lt;
      // P row -> shared memory, K-major 128B-swizzled bf16 (64 keys per 128-byte row)
#pragma unroll
      for (int g = 0; g < BKV / 8; ++g) {
        const int kb = g >> 3, gi = g & 7;
        uint8_t* dst = sp + kb * BQ * 128 + r * 128 + ((gi ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) =
            make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
      }
      fence_async_shared();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // ---------------------------------------------------------------- epilogue
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (nkv - 1) & 1, kDevTimeoutEpilogue,
                                                  abort_flag));
    if (ok) {
      tc_fence_after();
      const long long row = (long long)b * p.seq + qi;
      const bool valid = qi < p.seq;
      const float inv_l = (l > 0.f) ? p.v_scale / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t o[32];
        tmem_ld32(t_lane + C::O_COL + c, o);
        if (!valid) continue;
        float v[32];
#pragma unroll
        for (int u = 0; u < 32; ++u) v[u] = __uint_as_float(o[u]) * inv_l;
        if (p.gate != nullptr) {
          const long long go = row * p.gate_ld + (long long)h * p.gate_hstride + c;
          if (p.gate_dtype == kE4M3) {
            const uint8_t* gp = reinterpret_cast<const uint8_t*>(p.gate) + go;
#pragma unroll
            for (int u = 0; u < 32; u += 16) {
              const uint4 q = *reinterpret_cast<const uint4*>(gp + u);
              const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const float2 a = e4m3x2_to_f32x2(w[t] & 0xFFFF);
                const float2 bb = e4m3x2_to_f32x2(w[t] >> 16);
                const float gv[4] = {a.x, a.y, bb.x, bb.y};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float gg = gv[e] * p.gate_scale;
                  v[u + 4 * t + e] *= sigmoid_fast(gg);
                }
              }
            }
          } else {
            const __nv_bfloat16* gp = reinterpret_cast<const __nv_bfloat16*>(p.gate) + go;
#pragma unroll
            for (int u = 0; u < 32; ++u) {
              const float gg = __bfloat162float(gp[u]) * p.gate_scale;
              v[u] *= sigmoid_fast(gg);
            }
          }
        }
        uint32_t w[8];
#pragma unroll
        for (int t = 0; t < 8; ++t)
          w[t] = uint32_t(f32x2_to_e4m3x2(v[4 * t] * p.ctx_inv_scale,
                                          v[4 * t + 1] * p.ctx_inv_scale)) |
                 (uint32_t(f32x2_to_e4m3x2(v[4 * t + 2] * p.ctx_inv_scale,
                                           v[4 * t + 3] * p.ctx_inv_scale))
                  << 16);
        uint8_t* dst = p.ctx + row * p.ctx_ld + (long long)h * D + c;
        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(dst + 16) = make_uint4(w[4], w[5], w[6], w[7]);
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------
// Two query tiles per CTA (head_dim 64 / 128).  Query tiles A and B share every K/V tile;
// softmax warpgroup A (warps 2-5) and B (warps 6-9) each own one tile.  Each softmax step
// loads its S row into registers and releases the S columns at once, so the MMA warp
// computes S(j+1) while the exponentials of S(j) run; P(j) goes to a shared-memory tile
// per query tile (once P(j-1).V has retired) and P.V reads both operands from shared
// memory.  A tile's softmax therefore never waits for its own P.V and next QK^T.  With
// causal masking the pair is (i, n-1-i), or, for GQA head pairs, the same query rows of
// two heads sharing K/V.  TMEM: S_A | S_B | O_A | O_B.

__device__ __forceinline__ void sts128(uint32_t addr, const uint32_t (&v)[4]) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
}

__device__ __forceinline__ float ex2_hw(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for a pair, on the FMA and integer pipes instead of the exponential unit (Cody-Waite
// style range reduction + polynomial): x = n + f with n = rint(x) (the round-to-nearest of
// adding 1.5 * 2^23 leaves n in the low mantissa bits), f in [-0.5, 0.5]; 2^f by a cubic
// fitted for minimal relative error on that interval (max 7.5e-5, 2^-13.7, below the 2^-11
// rounding of the f16 weights it feeds); 2^n added to the exponent field.  Inputs are
// clamped to >= -125 (masked keys' -inf gives 2^-125, a weight of zero in f16 and
// negligible against the row sum).
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 t = fadd2(x, make_float2(12582912.0f, 12582912.0f));
  const float2 n = fadd2(t, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = ffma2(n, make_float2(-1.0f, -1.0f), x);
  float2 p = ffma2(make_float2(0.05517132f, 0.05517132f), f,
                   make_float2(0.24261054f, 0.24261054f));
  p = ffma2(p, f, make_float2(0.69326097f, 0.69326097f));
  p = ffma2(p, f, make_float2(0.99992812f, 0.99992812f));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

// sigmoid of a pair, 1 / (1 + 2^(-g log2 e)): the exponential on the FMA pipe (ex2_poly2,
// its argument clamped to <= 126 so 2^x stays finite) and one reciprocal on the exponential
// unit instead of two exponential-unit operations per gate value.
__device__ __forceinline__ float2 sigmoid2(float a, float b) {
  const float2 e = ex2_poly2(make_float2(fminf(a * -1.4426950408889634f, 126.0f),
                                         fminf(b * -1.4426950408889634f, 126.0f)));
  return make_float2(__fdividef(1.0f, 1.0f + e.x), __fdividef(1.0f, 1.0f + e.y));
}

template <int D>
struct Attn2Cfg {
  static constexpr int BQ = 128;
  static constexpr int BKV = 128;
  static constexpr int ROWB = (D >= 128) ? 128 : D;
  static constexpr int KB = (D >= 128) ? D / 128 : 1;
  static constexpr uint32_t LAYOUT8 = (ROWB == 128) ? 2u : 4u;
  static constexpr uint32_t SBO8 = 8 * ROWB;
  static constexpr int Q_BYTES = BQ * D;  // per query tile
  static constexpr int K_BYTES = BKV * D;
  static constexpr int V_BYTES = BKV * D * 2;
  // Separate K and V rings: K(j) is released as soon as both S(j) MMAs are issued.
  // Ring slots of one head's K / V tile; with pair_kv a stage is two slots (both heads).
  static constexpr int KST = (D >= 128) ? 2 : 4;
  static constexpr int VST = (D >= 128) ? 2 : 4;
  // P (16-bit) in shared memory, one tile per query tile: [2 key blocks of 64][128 rows]
  // [128-byte swizzled row], the K-major layout of an MMA operand.  The P.V MMA reads both
  // operands from shared memory (with P in tensor memory that MMA ran at less than half
  // rate while the softmax warps kept the SM's issue slots busy), and the S columns are
  // free as soon as the softmax has loaded them: S(j+1) is computed during the
  // exponentials of S(j).
  static constexpr int P_BYTES = BQ * BKV * 2;
  // e4m3 gate tiles (one per query tile, same shape as Q) for the gated epilogue.
  static constexpr int G_BYTES = Q_BYTES;
  static constexpr int SMEM_BYTES = 2 * Q_BYTES + KST * K_BYTES + VST * V_BYTES +
                                    2 * P_BYTES + 2 * G_BYTES + 1024 + 512;
  static constexpr int S_COL = 0;             // S_X at X * BKV
  static constexpr int O_COL = 2 * BKV;       // O_X at O_COL + X * D
  static constexpr int TMEM_COLS = 512;
  static_assert(D > 128 || 2 * BKV + 2 * D <= 512, "TMEM budget");
  static_assert(D > 128 || SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

template <int D, bool VF16>
__global__ void __launch_bounds__(384, 1)
    attention2_kernel(const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_g, const AttnParams p) {
  using C = Attn2Cfg<D>;
  constexpr int BQ = C::BQ, BKV = C::BKV, KST = C::KST, VST = C::VST;
  constexpr bool kSplitPV = D <= 64;  // P.V issued in two 64-key halves
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sq = smem;                            // [2][Q_BYTES]
  uint8_t* sk = sq + 2 * C::Q_BYTES;             // [KST][K_BYTES]
  uint8_t* sv = sk + KST * C::K_BYTES;           // [VST][V_BYTES]
  uint8_t* sp = sv + VST * C::V_BYTES;           // [2][P_BYTES]
  uint8_t* sg = sp + 2 * C::P_BYTES;             // [2][G_BYTES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sg + 2 * C::G_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + KST;
  uint64_t* v_full = k_empty + KST;
  uint64_t* v_empty = v_full + VST;
  uint64_t* s_full = v_empty + VST;  // [tile]: S(j) landed
  uint64_t* s_free = s_full + 2;     // [tile]: the softmax loaded S(j) into registers
  uint64_t* p_full = s_free + 2;     // [tile]: P(j) stored in shared memory
  uint64_t* pv_done = p_full + 2;    // [tile]: P(j).V retired
  uint64_t* p_half = pv_done + 2;    // [tile]: keys 0-63 of P(j) stored
  uint64_t* drain = p_half + 2;
  uint64_t* g_full = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.seq + BQ - 1) / BQ;
  int qt[2], hx[2];
  bool act[2];
  if (p.pair_heads || p.pair_kv) {
    // GQA: query heads 2y and 2y+1 read the same KV head; both tiles take the same query
    // rows, so both stay active for every key tile and share each K / V load.  (pair_kv:
    // the same for two heads with their own K / V, loaded side by side.)  The grid is
    // (head pairs, batch, query tiles) with the longest causal rows in the first z-slice:
    // CTAs start in grid order, so every long CTA starts before any shorter one and the
    // short ones fill the end (longest-first; with the query tile in x, long CTAs that
    // started late set the kernel's tail).
    qt[0] = qt[1] = n_qt - 1 - blockIdx.z;
    hx[0] = 2 * blockIdx.x;
    hx[1] = hx[0] + 1;
    act[0] = true;
  } else {
    if (p.causal) {
      qt[0] = blockIdx.x;
      qt[1] = n_qt - 1 - blockIdx.x;
    } else {
      qt[0] = 2 * blockIdx.x;
      qt[1] = min(2 * (int)blockIdx.x + 1, n_qt - 1);
    }
    hx[0] = hx[1] = blockIdx.y;
    act[0] = qt[0] < qt[1];
  }
  act[1] = true;
  int nkv[2];
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    const int end = p.causal ? min(p.seq, qt[x] * BQ + BQ) : p.seq;
    nkv[x] = act[x] ? (end + BKV - 1) / BKV : 0;
  }
  const int b = (p.pair_heads || p.pair_kv) ? blockIdx.y : blockIdx.z;
  const int hk = hx[0] / (p.hq / p.hkv);
  const int kv2 = p.pair_kv ? 2 : 1;     // heads per K / V ring stage
  const int hkv[2] = {hk, p.pair_kv ? hx[1] : hk};
  const int ks = KST / kv2, vsn = VST / kv2;  // ring stages

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
      mbar_init(&p_half[i], 4);
    }
    mbar_init(drain, 1);
    mbar_init(g_full, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    if (p.gate_tma) tma_prefetch_desc(&tm_g);
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // set-up above overlaps the previous kernel; global memory only from here
  // Every warp runs at the launch allocation (168 registers).  No `setmaxnreg` split: ptxas
  // ignores it in relocatable (-rdc) code, and in a whole-program build the MMA issuer's
  // unrolled loops needed about 150 registers, so the softmax warpgroups could gain at most
  // 176, which measured slower (170.6 vs 166.5 us at the Qwen shape).

  if (warp == 0) {
    // ---------------------------------------------------------------- producers
    // lane 0: Q once, then the K ring; lane 1: the V ring (independent waits).
    const uint64_t pol = policy_evict_last();
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, (act[0] ? 2 : 1) * C::Q_BYTES);
      for (int x = 0; x < 2; ++x) {
        if (!act[x]) continue;
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_3d(sq + x * C::Q_BYTES + kb * BQ * C::ROWB, &tm_q, q_full, hx[x] * D + kb * 128,
                      qt[x] * BQ, b, pol);
      }
    }
    if (lane < 2) {
      const bool is_k = lane == 0;
      const int NS = is_k ? ks : vsn;
      uint64_t* fullb = is_k ? k_full : v_full;
      uint64_t* emptyb = is_k ? k_empty : v_empty;
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool g_issued = false;
      // The gate tiles follow the second K tile: off the first S's critical path, long
      // before the epilogue reads them.
      const int g_after = min(1, nkv[1] - 1);
      for (int j = 0; j < nkv[1]; ++j) {
        if (!mbar_wait(&emptyb[stage], phase ^ 1, kDevTimeoutProducer, abort_flag)) break;
        if (is_k) {
          mbar_arrive_expect_tx(&fullb[stage], kv2 * C::K_BYTES);
          for (int h = 0; h < kv2; ++h) {
            uint8_t* dst = sk + (stage * kv2 + h) * C::K_BYTES;
            for (int kb = 0; kb < C::KB; ++kb)
              tma_load_3d(dst + kb * BKV * C::ROWB, &tm_k, &fullb[stage], hkv[h] * D + kb * 128,
                          j * BKV, b, pol);
          }
        } else {
          mbar_arrive_expect_tx(&fullb[stage], kv2 * C::V_BYTES);
          for (int h = 0; h < kv2; ++h) {
            uint8_t* dst = sv + (stage * kv2 + h) * C::V_BYTES;
            for (int vb = 0; vb < D / 64; ++vb)
              tma_load_3d(dst + vb * BKV * 128, &tm_v, &fullb[stage], hkv[h] * D + vb * 64,
                          j * BKV, b, pol);
          }
        }
        ++issued;
        if (++stage == NS) { stage = 0; phase ^= 1; }
        if (is_k && p.gate_tma && j == g_after) {
          mbar_arrive_expect_tx(g_full, (act[0] ? 2 : 1) * C::G_BYTES);
          for (int x = 0; x < 2; ++x) {
            if (!act[x]) continue;
            for (int kb = 0; kb < C::KB; ++kb)
              tma_load_3d(sg + x * C::G_BYTES + kb * BQ * C::ROWB, &tm_g, g_full,
                          int(hx[x] * p.gate_hstride) + kb * 128, qt[x] * BQ, b,
                          policy_evict_first());
          }
          g_issued = true;
        }
      }
      // Let the copies still in flight land before the CTA exits.
      const int pending = issued < NS ? issued : NS;
      for (int i = 0; i < pending; ++i) {
        if (--stage < 0) { stage = NS - 1; phase ^= 1; }
        const uint64_t t0 = globaltimer();
        while (!mbar_test(&fullb[stage], phase))
          if (globaltimer() - t0 > B2F_WAIT_NS) { record_error(kDevTimeoutDrain); break; }
      }
      if (is_k) {
        const uint64_t t0 = globaltimer();
        while (!mbar_test(q_full, 0))
          if (globaltimer() - t0 > B2F_WAIT_NS) { record_error(kDevTimeoutDrain); break; }
        while (g_issued && !mbar_test(g_full, 0))
          if (globaltimer() - t0 > B2F_WAIT_NS) { record_error(kDevTimeoutDrain); break; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      // Per key tile j: S_A(j+1), S_B(j+1) as soon as each softmax has loaded S(j) into
      // registers (the exponentials of S(j) then overlap the next QK^T), then P_A(j).V and
      // P_B(j).V once the softmax stored P(j).
      constexpr uint32_t idesc_s = make_idesc_f8(BQ, BKV);
      constexpr uint32_t idesc_pv = VF16 ? make_idesc_f16(BQ, D, 1) : make_idesc_bf16(BQ, D, 1);
      bool ok = mbar_wait(q_full, 0, kDevTimeoutMma, abort_flag);
      // Shared-memory descriptors are built once: a descriptor's low 14 bits hold the
      // address / 16 (every address here is below 256 KB, so adding an offset / 16 never
      // carries out of the field), so each MMA's operands are the base plus an immediate.
      // A lean issue loop matters: with the softmax warps keeping the SM's issue slots
      // busy, descriptor arithmetic between 16-bit MMAs left the tensor core idle.
      const uint64_t q_desc[2] = {make_sdesc(smem_u32(sq), C::LAYOUT8, 16, C::SBO8),
                                  make_sdesc(smem_u32(sq + C::Q_BYTES), C::LAYOUT8, 16, C::SBO8)};
      const uint64_t k_desc0 = make_sdesc(smem_u32(sk), C::LAYOUT8, 16, C::SBO8);
      const uint64_t p_desc[2] = {make_sdesc(smem_u32(sp), 2, 16, 1024),
                                  make_sdesc(smem_u32(sp + C::P_BYTES), 2, 16, 1024)};
      const uint64_t v_desc0 = make_sdesc(smem_u32(sv), 2, BKV * 128, 1024);
      auto issue_s = [&](int x, int j) {
        const uint64_t qd = q_desc[x];
        const uint64_t kd =
            k_desc0 + uint64_t(((j % ks) * kv2 + (p.pair_kv ? x : 0)) * (C::K_BYTES >> 4));
        const uint32_t d = tmem + C::S_COL + x * BKV;
#pragma unroll
        for (int kb = 0; kb < C::KB; ++kb) {
#pragma unroll
          for (int k = 0; k < C::ROWB / 32; ++k)
            mma_f8(d, qd + ((kb * BQ * C::ROWB + k * 32) >> 4),
                   kd + ((kb * BKV * C::ROWB + k * 32) >> 4), idesc_s, (kb | k) != 0);
        }
        mma_commit(&s_full[x]);
      };
      // S(j) of both tiles (tile 0 only while its causal rows still reach key tile j); for
      // j > 0 each waits until its softmax has loaded S(j-1).
      auto issue_s_pair = [&](int j) -> bool {
        if (!mbar_wait(&k_full[j % ks], (j / ks) & 1, kDevTimeoutMma, abort_flag))
          return false;
        if (act[0] && j < nkv[0]) {
          if (j > 0 && !mbar_wait(&s_free[0], (j - 1) & 1, kDevTimeoutMma, abort_flag))
            return false;
          tc_fence_after();
          issue_s(0, j);
        }
        if (j > 0 && !mbar_wait(&s_free[1], (j - 1) & 1, kDevTimeoutMma, abort_flag))
          return false;
        tc_fence_after();
        issue_s(1, j);
        mma_commit(&k_empty[j % ks]);  // both readers of K(j) issued before it
        return true;
      };
      auto issue_pv = [&](int x, int j) -> bool {
        // head_dim 64: the first 64 keys' four MMAs go as soon as that half of P is stored
        // (the softmax is still exponentiating the second half), the other four after all
        // of P (GPT-2 shape 49.2 -> 47.1 us; at head_dim 128 it measured slower, 203 ->
        // 214 us, and P.V waits for all of P).
        if (!mbar_wait(kSplitPV ? &p_half[x] : &p_full[x], j & 1, kDevTimeoutMma, abort_flag))
          return false;
        const int vs = j % vsn;
        if (x == 0 || j >= nkv[0]) {  // first reader of V(j)
          if (!mbar_wait(&v_full[vs], (j / vsn) & 1, kDevTimeoutMma, abort_flag)) return false;
        }
        tc_fence_after();
        // P(j): 128 query rows x 128 keys of 16-bit weights in two 64-key blocks of
        // 128-byte swizzled rows; 16 keys (32 bytes of P, 2 KB of V) per MMA.
        const uint64_t pd = p_desc[x];
        const uint64_t vd =
            v_desc0 + uint64_t((vs * kv2 + (p.pair_kv ? x : 0)) * (C::V_BYTES >> 4));
        const uint32_t o = tmem + C::O_COL + x * D;
        mma_bf16(o, pd, vd, idesc_pv, j != 0);
#pragma unroll
        for (int ks = 1; ks < BKV / 32; ++ks)
          mma_bf16(o, pd + (((ks >> 2) * BQ * 128 + (ks & 3) * 32) >> 4),
                   vd + ((ks * 2048) >> 4), idesc_pv, 1u);
        if (kSplitPV) {
          if (!mbar_wait(&p_full[x], j & 1, kDevTimeoutMma, abort_flag)) return false;
          tc_fence_after();
        }
#pragma unroll
        for (int ks = BKV / 32; ks < BKV / 16; ++ks)
          mma_bf16(o, pd + (((ks >> 2) * BQ * 128 + (ks & 3) * 32) >> 4),
                   vd + ((ks * 2048) >> 4), idesc_pv, 1u);
        mma_commit(&pv_done[x]);
        return true;
      };
      if (ok) ok = issue_s_pair(0);
      for (int j = 0; j < nkv[1] && ok; ++j) {
        if (j + 1 < nkv[1] && !(ok = issue_s_pair(j + 1))) break;
        if (j < nkv[0] && !(ok = issue_pv(0, j))) break;
        if (!(ok = issue_pv(1, j))) break;
        mma_commit(&v_empty[j % vsn]);  // both P.V of this key tile issued before it
      }
      mma_commit(drain);
      const uint64_t t0 = globaltimer();
      while (!mbar_test(drain, 0))
        if (globaltimer() - t0 > B2F_WAIT_NS) { record_error(kDevTimeoutDrain); break; }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax + epilogue
    const int x = (warp - 4) >> 2;   // query tile handled by this warpgroup
    const int qd = warp & 3;         // TMEM lane quadrant
    const int r = qd * 32 + lane;
    const int q0 = qt[x] * BQ;
    const int qi = q0 + r;
    const uint32_t t_lane = tmem + (uint32_t(qd * 32) << 16);
    const uint32_t o_col = C::O_COL + x * D;
    const float c = p.qk_scale_log2;
    float m_used = -INFINITY;
    float l = 0.f;
    bool ok = act[x];
    const uint32_t s_col = C::S_COL + x * BKV;
    // Shared-memory addresses of this row's eight swizzled 16-byte chunks of the P tile
    // (chunk c of row r at position c ^ (r % 8) of the 128-byte row; the second 64-key
    // block is a constant offset away).
    uint32_t p_addr[8];
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8)
      p_addr[c8] = smem_u32(sp + x * C::P_BYTES + r * 128) + ((c8 ^ (r & 7)) << 4);
    for (int j = 0; j < nkv[x] && ok; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[x], j & 1, kDevTimeoutEpilogue, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const int k0 = j * BKV;
      // keys k0 + kk with kk > klim are masked (past the sequence end or, causal, past qi)
      const int klim = min(p.seq - 1, p.causal ? qi : p.seq - 1) - k0;
      const bool need_mask = klim < BKV - 1;
      // The whole S row (128 f32 columns) in registers: four loads in flight, one wait;
      // then the S columns are released for S(j+1).
      uint32_t s0[32], s1[32], s2[32], s3[32];
      tmem_ld32_async(t_lane + s_col, s0);
      tmem_ld32_async(t_lane + s_col + 32, s1);
      tmem_ld32_async(t_lane + s_col + 64, s2);
      tmem_ld32_async(t_lane + s_col + 96, s3);
      tmem_ld_wait_regs(s0);
      reg_fence32(s1);
      reg_fence32(s2);
      reg_fence32(s3);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[x]);
      auto sv = [&](int u) -> uint32_t& {
        return u < 32 ? s0[u] : u < 64 ? s1[u - 32] : u < 96 ? s2[u - 64] : s3[u - 96];
      };
      if (need_mask) {
#pragma unroll
        for (int u = 0; u < BKV; ++u)
          if (u > klim) sv(u) = __float_as_uint(-INFINITY);
      }
      // O *= corr (warp-collective; lanes whose row keeps its reference pass corr = 1).
      auto rescale_o = [&](float corr) {
#pragma unroll 1
        for (int cc = 0; cc < D; cc += 16) {
          uint32_t o[16];
          tmem_ld16(t_lane + o_col + cc, o);
#pragma unroll
          for (int u = 0; u < 16; ++u) o[u] = __float_as_uint(__uint_as_float(o[u]) * corr);
          tmem_st16(t_lane + o_col + cc, o);
        }
        tmem_st_wait();
      };
      float corr = 1.0f, lt, mref;
      bool rescale = false;
      {
        // Row max of S * c: 4 independent partial maxima over 3-input max.
        float mp[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) mp[e] = -INFINITY;
#pragma unroll
        for (int u = 0; u < BKV; u += 2)
          mp[(u >> 1) & 3] = fmax3(mp[(u >> 1) & 3], __uint_as_float(sv(u)),
                                   __uint_as_float(sv(u + 1)));
        const float mt = fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])) * c;
        if (mt > m_used + 8.0f) {
          if (m_used != -INFINITY) {
            corr = ex2_hw(m_used - mt);
            rescale = true;
          }
          m_used = mt;
        }
        mref = (m_used == -INFINITY) ? 0.0f : m_used;
      }
      // P(j-1).V has landed before P(j) overwrites the shared-memory P tile and before O is
      // rescaled (P(j).V is released below).  Waiting here, before the exponentials, lets
      // the first half of P(j) be stored while the second half is computed.
      if (j > 0) {
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&pv_done[x], (j - 1) & 1, kDevTimeoutEpilogue, abort_flag));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) rescale_o(corr);
      }
      {
        // P = 2^(S*c - m) to the shared-memory P tile (the A operand of P.V), 64 keys at a
        // time: row r of the tile is sixteen 16-byte chunks of 8 keys in two 64-key blocks
        // of 128-byte rows, swizzled (chunk c at position c ^ (r % 8) of its row), the
        // layout of a K-major SW128 MMA operand.  Each weight is exponentiated in f32 and
        // rounded to f16 (f16 V; 2^-11 relative, the conversion is not on the exponential
        // unit) or bf16 (bf16 V); the row sum accumulates the f32 weights.  Masked keys
        // hold -inf, whose weight is 0.  Scale, offset and row sum are packed pair
        // operations (half the issue slots of scalar FFMA / FADD: the softmax warps share
        // the SM's issue slots with the MMA warp, and 16-bit MMAs fed late leave the tensor
        // core idle).  The 16-bit pairs overwrite the S registers they came from (pair e
        // goes to S slot e, already consumed), which keeps the row within the register
        // budget.
        const float2 c2 = make_float2(c, c), nm2 = make_float2(-mref, -mref);
        float2 acc2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int hb = 0; hb < BKV / 64; ++hb) {
#pragma unroll
          for (int c8 = hb * 8; c8 < hb * 8 + 8; ++c8) {
            // keys [8 c8, 8 c8 + 8): four pairs packed into one fresh 16-byte vector and
            // stored at once (packing them back into the S registers first cost register
            // moves: ncu counted about 360 extra FMA / ALU-pipe instructions per warp step)
            uint32_t q4[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const int e = 4 * c8 + t;
              const float2 xv = ffma2(make_float2(__uint_as_float(sv(2 * e)),
                                                  __uint_as_float(sv(2 * e + 1))), c2, nm2);
              // Every exponential on the exponential unit: moving three of eight pairs to
              // an FMA-pipe polynomial (ex2_poly2) measured slower here (Qwen shape 223 vs
              // 205 us): the softmax is bound by issue slots, which the polynomial adds.
              const float e0 = ex2_hw(xv.x), e1 = ex2_hw(xv.y);
              acc2[t & 1] = fadd2(acc2[t & 1], make_float2(e0, e1));
              if constexpr (VF16) q4[t] = pack_f16x2(e0, e1);
              else q4[t] = pack_bf16x2(e0, e1);
            }
            sts128(p_addr[c8 & 7] + hb * (BQ * 128), q4);
          }
          if (kSplitPV && hb == 0) {
            fence_async_shared();  // keys 0-63 of P visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_half[x]);
          }
        }
        fence_async_shared();  // generic-proxy writes visible to the tensor core
        lt = (acc2[0].x + acc2[0].y) + (acc2[1].x + acc2[1].y);
      }
      l = l * corr + lt;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
    }
    // ---------------------------------------------------------------- epilogue
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[x], (nkv[x] - 1) & 1,
                                                  kDevTimeoutEpilogue, abort_flag));
    if (ok) {
      tc_fence_after();
      const long long row = (long long)b * p.seq + qi;
      const bool valid = qi < p.seq;
      const float inv_l = (l > 0.f) ? p.v_scale / l : 0.f;
      const bool gate_smem = p.gate_tma != 0;
      if (gate_smem)
        ok = __all_sync(0xffffffffu, mbar_wait(g_full, 0, kDevTimeoutEpilogue, abort_flag));
      // 32 columns at a time, the next chunk's tensor-memory load in flight meanwhile.
      uint32_t oa[32], ob[32];
      if (ok) tmem_ld32_async(t_lane + o_col, oa);
#pragma unroll
      for (int cc = 0; cc < D && ok; cc += 32) {
        uint32_t (&o)[32] = ((cc / 32) & 1) ? ob : oa;
        uint32_t (&on)[32] = ((cc / 32) & 1) ? oa : ob;
        tmem_ld_wait_regs(o);
        if (cc + 32 < D) tmem_ld32_async(t_lane + o_col + cc + 32, on);
        // (rows past the sequence end store nothing; the warp reconverges before the next
        // chunk's warp-collective tensor-memory load)
        if (valid) {
          float v[32];
#pragma unroll
          for (int u = 0; u < 32; ++u) v[u] = __uint_as_float(o[u]) * inv_l;
          if (p.gate != nullptr) {
            if (gate_smem) {
              // Row r of this tile's gate, as the TMA wrote it (16-byte chunks swizzled by
              // the row: 128B pattern for 128-byte rows, 64B pattern for 64-byte rows).
              const uint8_t* gt = sg + x * C::G_BYTES + (cc / C::ROWB) * (BQ * C::ROWB);
#pragma unroll
              for (int h16 = 0; h16 < 2; ++h16) {
                const uint32_t off = uint32_t(r * C::ROWB + (cc % C::ROWB) + h16 * 16);
                const uint32_t sw = off ^ (((off >> 7) & (C::ROWB == 128 ? 7u : 3u)) << 4);
                const uint4 qv = *reinterpret_cast<const uint4*>(gt + sw);
                const uint32_t w4[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                  const float2 a = e4m3x2_to_f32x2(w4[t] & 0xFFFF);
                  const float2 bb = e4m3x2_to_f32x2(w4[t] >> 16);
                  const int u = h16 * 16 + 4 * t;
                  const float2 s01 = sigmoid2(a.x * p.gate_scale, a.y * p.gate_scale);
                  const float2 s23 = sigmoid2(bb.x * p.gate_scale, bb.y * p.gate_scale);
                  v[u] *= s01.x;
                  v[u + 1] *= s01.y;
                  v[u + 2] *= s23.x;
                  v[u + 3] *= s23.y;
                }
              }
            } else {
              const long long go = row * p.gate_ld + (long long)hx[x] * p.gate_hstride + cc;
              if (p.gate_dtype == kE4M3) {
                const uint8_t* gp = reinterpret_cast<const uint8_t*>(p.gate) + go;
#pragma unroll
                for (int u = 0; u < 32; u += 16) {
                  const uint4 qv = *reinterpret_cast<const uint4*>(gp + u);
                  const uint32_t w4[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
                  for (int t = 0; t < 4; ++t) {
                    const float2 a = e4m3x2_to_f32x2(w4[t] & 0xFFFF);
                    const float2 bb = e4m3x2_to_f32x2(w4[t] >> 16);
                    v[u + 4 * t] *= sigmoid_fast(a.x * p.gate_scale);
                    v[u + 4 * t + 1] *= sigmoid_fast(a.y * p.gate_scale);
                    v[u + 4 * t + 2] *= sigmoid_fast(bb.x * p.gate_scale);
                    v[u + 4 * t + 3] *= sigmoid_fast(bb.y * p.gate_scale);
                  }
                }
              } else {
                const __nv_bfloat16* gp = reinterpret_cast<const __nv_bfloat16*>(p.gate) + go;
#pragma unroll
                for (int u = 0; u < 32; ++u)
                  v[u] *= sigmoid_fast(__bfloat162float(gp[u]) * p.gate_scale);
              }
            }
          }
          uint32_t w[8];
#pragma unroll
          for (int t = 0; t < 8; ++t)
            w[t] = uint32_t(f32x2_to_e4m3x2(v[4 * t] * p.ctx_inv_scale,
                                            v[4 * t + 1] * p.ctx_inv_scale)) |
                   (uint32_t(f32x2_to_e4m3x2(v[4 * t + 2] * p.ctx_inv_scale,
                                             v[4 * t + 3] * p.ctx_inv_scale))
                    << 16);
          uint8_t* dst = p.ctx + row * p.ctx_ld + (long long)hx[x] * D + cc;
          *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(dst + 16) = make_uint4(w[4], w[5], w[6], w[7]);
        }
        __syncwarp();
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int D, bool PAIR>
int launch_attention(const b2f_attn_args* a, cudaStream_t stream) {
  using C = AttnCfg<D>;
  constexpr int BKV = PAIR ? Attn2Cfg<D>::BKV : C::BKV;
  constexpr int SMEM = PAIR ? Attn2Cfg<D>::SMEM_BYTES : C::SMEM_BYTES;
  CUtensorMap tq, tk, tv;
  std::string err;
  const CUtensorMapSwizzle sw8 =
      (C::ROWB == 128) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  {
    const unsigned long long dims[3] = {(unsigned long long)a->hq * D, (unsigned long long)a->seq,
                                        (unsigned long long)a->batch};
    const unsigned long long strides[2] = {(unsigned long long)a->q_ld,
                                           (unsigned long long)a->q_ld * a->seq};
    const unsigned int box[3] = {(unsigned int)C::ROWB, (unsigned int)C::BQ, 1};
    if (!encode_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a->q, dims, strides, box, sw8, &err))
      return fail(B2F_ERR_ARG, "attention: Q tensor map: " + err);
  }
  {
    const unsigned long long dims[3] = {(unsigned long long)a->hkv * D, (unsigned long long)a->seq,
                                        (unsigned long long)a->batch};
    const unsigned long long strides[2] = {(unsigned long long)a->k_ld,
                                           (unsigned long long)a->k_ld * a->seq};
    const unsigned int box[3] = {(unsigned int)C::ROWB, (unsigned int)BKV, 1};
    if (!encode_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a->k, dims, strides, box, sw8, &err))
      return fail(B2F_ERR_ARG, "attention: K tensor map: " + err);
  }
  {
    const unsigned long long dims[3] = {(unsigned long long)a->hkv * D, (unsigned long long)a->seq,
                                        (unsigned long long)a->batch};
    const unsigned long long strides[2] = {(unsigned long long)a->v_ld * 2,
                                           (unsigned long long)a->v_ld * 2 * a->seq};
    const unsigned int box[3] = {64, (unsigned int)BKV, 1};
    const CUtensorMapDataType vt = a->v_dtype == B2F_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                               : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if (!encode_tmap(&tv, vt, 3, a->v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, &err))
      return fail(B2F_ERR_ARG, "attention: V tensor map: " + err);
  }
  AttnParams p;
  p.seq = a->seq; p.batch = a->batch; p.hq = a->hq; p.hkv = a->hkv;
  p.causal = a->causal;
  const float sm = a->sm_scale > 0.f ? a->sm_scale : 1.0f / sqrtf((float)D);
  p.qk_scale_log2 = a->q_scale * a->k_scale * sm * 1.4426950408889634f;
  p.gate = a->gate; p.gate_dtype = a->gate_dtype; p.gate_ld = a->gate_ld;
  p.gate_hstride = a->gate_head_stride; p.gate_scale = a->gate_scale;
  p.ctx = reinterpret_cast<uint8_t*>(a->ctx); p.ctx_ld = a->ctx_ld;
  p.ctx_inv_scale = 1.0f / a->ctx_scale;
  p.v_scale = a->v_scale;
  p.pair_heads = 0;
  p.pair_kv = 0;
  p.gate_tma = 0;
  CUtensorMap tg = tq;  // (unused unless gate_tma)
  if (PAIR && a->gate != nullptr && a->gate_dtype == B2F_DTYPE_E4M3) {
    // e4m3 gate tiles [BQ rows x D] by TMA, the same box and swizzle as Q; the column
    // extent ends with the last head's D columns.
    const unsigned long long dims[3] = {
        (unsigned long long)((a->hq - 1) * a->gate_head_stride + D), (unsigned long long)a->seq,
        (unsigned long long)a->batch};
    const unsigned long long strides[2] = {(unsigned long long)a->gate_ld,
                                           (unsigned long long)a->gate_ld * a->seq};
    const unsigned int box[3] = {(unsigned int)C::ROWB, (unsigned int)C::BQ, 1};
    if (!encode_tmap(&tg, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a->gate, dims, strides, box, sw8,
                     &err))
      return fail(B2F_ERR_ARG, "attention: gate tensor map: " + err);
    p.gate_tma = 1;
  }
  static thread_local int attr_dev[2][3] = {{-1, -1, -1}, {-1, -1, -1}};
  const int slot = D == 64 ? 0 : (D == 128 ? 1 : 2);
  int dev = 0;
  B2F_CUDA_TRY(cudaGetDevice(&dev));
  const int n_qt = (a->seq + C::BQ - 1) / C::BQ;
  if constexpr (PAIR) {
    if (attr_dev[1][slot] != dev) {
      B2F_CUDA_TRY(cudaFuncSetAttribute(attention2_kernel<D, false>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
      B2F_CUDA_TRY(cudaFuncSetAttribute(attention2_kernel<D, true>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
      attr_dev[1][slot] = dev;
    }
    p.pair_heads = (a->hq / a->hkv) % 2 == 0;
    // Causal attention with a KV head per query head (GPT-2): pair heads 2y, 2y+1 at the
    // same query tile rather than query tiles (i, n-1-i) of one head, whose shorter tile
    // leaves half of the CTA idle for most key tiles.
    p.pair_kv = !p.pair_heads && D == 64 && a->causal && a->hq == a->hkv && a->hq % 2 == 0;
    const bool two_heads = p.pair_heads || p.pair_kv;
    const dim3 grid = two_heads ? dim3(a->hq / 2, a->batch, n_qt)
                                : dim3((n_qt + 1) / 2, a->hq, a->batch);
    if (a->v_dtype == B2F_DTYPE_F16)
      B2F_CUDA_TRY(launch_pdl(attention2_kernel<D, true>, grid, dim3(384), SMEM, stream, tq, tk,
                              tv, tg, p));
    else
      B2F_CUDA_TRY(launch_pdl(attention2_kernel<D, false>, grid, dim3(384), SMEM, stream, tq,
                              tk, tv, tg, p));
  } else {
    if (attr_dev[0][slot] != dev) {
      B2F_CUDA_TRY(cudaFuncSetAttribute(attention_kernel<D>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
      attr_dev[0][slot] = dev;
    }
    dim3 grid(n_qt, a->hq, a->batch);
    B2F_CUDA_TRY(launch_pdl(attention_kernel<D>, grid, dim3(192), SMEM, stream, tq, tk, tv, p));
  }
  B2F_CUDA_TRY(cudaGetLastError());
  return B2F_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace b2f


extern "C" {

void b2f_attn_args_init(b2f_attn_args* a) {
  if (a == nullptr) return;
  *a = b2f_attn_args{};
  a->causal = 1;
  a->q_scale = a->k_scale = a->v_scale = 1.0f;
  a->gate_dtype = B2F_DTYPE_E4M3;
  a->gate_scale = 1.0f;
  a->ctx_scale = 1.0f;
  a->v_dtype = B2F_DTYPE_BF16;
}

int b2f_attention_fp8(const b2f_attn_args* a, b2f_stream_t stream) {
  using namespace b2f;
  if (a == nullptr) return fail(B2F_ERR_ARG, "attention: null args");
  if (a->batch <= 0 || a->seq <= 0 || a->hq <= 0 || a->hkv <= 0)
    return fail(B2F_ERR_ARG, "attention: empty shape");
  if (a->hq % a->hkv != 0) return fail(B2F_ERR_ARG, "attention: hq must be a multiple of hkv");
  const int d = a->head_dim;
  if (d != 64 && d != 128 && d != 256)
    return fail(B2F_ERR_UNSUPPORTED, "attention: head_dim must be 64, 128 or 256");
  if (a->q == nullptr || a->k == nullptr || a->v == nullptr || a->ctx == nullptr)
    return fail(B2F_ERR_ARG, "attention: null tensor");
  if (!al16(a->q) || !al16(a->k) || !al16(a->v) || !al16(a->ctx))
    return fail(B2F_ERR_ARG, "attention: tensors must be 16-byte aligned");
  if (a->q_ld % 16 || a->k_ld % 16 || (a->v_ld * 2) % 16 || a->ctx_ld % 16 ||
      a->q_ld < (long long)a->hq * d || a->k_ld < (long long)a->hkv * d ||
      a->v_ld < (long long)a->hkv * d || a->ctx_ld < (long long)a->hq * d)
    return fail(B2F_ERR_ARG,
                "attention: row pitches must cover the heads and be 16-byte multiples");
  if (a->gate != nullptr) {
    const int gs = a->gate_dtype == B2F_DTYPE_BF16 ? 2 : 1;
    if (a->gate_dtype != B2F_DTYPE_BF16 && a->gate_dtype != B2F_DTYPE_E4M3)
      return fail(B2F_ERR_ARG, "attention: gate must be e4m3 or bf16");
    if (!al16(a->gate) || (a->gate_ld * gs) % 16 || (a->gate_head_stride * gs) % 16)
      return fail(B2F_ERR_ARG, "attention: gate must be 16-byte aligned");
  }
  if (!(a->ctx_scale > 0.f)) return fail(B2F_ERR_ARG, "attention: ctx_scale must be > 0");
  if (a->v_dtype != B2F_DTYPE_BF16 && a->v_dtype != B2F_DTYPE_F16)
    return fail(B2F_ERR_ARG, "attention: v must be bf16 or f16");
  if (a->v_dtype == B2F_DTYPE_F16 && d == 256)
    return fail(B2F_ERR_UNSUPPORTED, "attention: f16 V needs head_dim 64 or 128");
  cudaStream_t s = (cudaStream_t)stream;
  if (d == 64) return launch_attention<64, true>(a, s);
  if (d == 128) return launch_attention<128, true>(a, s);
  return launch_attention<256, false>(a, s);
}

}  // extern "C"
