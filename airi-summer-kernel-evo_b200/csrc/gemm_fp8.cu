// Host launcher of the tcgen05 e4m3 GEMM (C ABI: b2f_gemm_fp8).
#include <atomic>
#include <cstring>
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "gemm_fp8.cuh"
#include "host_common.h"

namespace b2f {

namespace {

thread_local int g_pair_capacity = 0;
}  // namespace
constexpr int kMaxSplits = 8;  // split-K slices per tile (workspace holds one f32 tile each)
// Split-K workspace layout: a fixed region of per-tile arrival counters first (every call
// leaves its counters at zero, and no call ever writes partial sums there, so calls of any
// shape can share one workspace), then kMaxSplits f32 partial-tile slices.
constexpr long long kCounterBytes = 16384;
constexpr int kMaxSplitTiles = kCounterBytes / 4;
namespace {  // co-resident CTA pairs seen by the last pair launch

// Output tensor map for the epilogue's TMA stores: the output viewed as bytes
// [m, n * esize] with 32-row x 128-byte boxes in the 128B swizzle layout.
// Each epilogue warp drains `half_cols` columns of a tile; its TMA store box is the
// largest of 64 / 128 bytes that fits inside that column range.
int encode_out_map(const b2f_gemm_args* a, EpilogueParams& ep, int half_cols, CUtensorMap* map) {
  std::memset(map, 0, sizeof(*map));
  const int esz = a->out_dtype == B2F_DTYPE_F32 ? 4 : (a->out_dtype == B2F_DTYPE_BF16 ? 2 : 1);
  ep.chunk_bytes = half_cols * esz >= 128 ? 128 : 64;
  if (!ep.out_vec || ep.mode != kModeStore) return B2F_OK;
  const unsigned long long dims[2] = {(unsigned long long)a->n * esz, (unsigned long long)a->m};
  const unsigned long long strides[1] = {(unsigned long long)a->out_ld * esz};
  const unsigned int box[2] = {(unsigned int)ep.chunk_bytes, 32};
  std::string err;
  if (!encode_tmap(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a->out, dims, strides, box,
                   ep.chunk_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                   &err))
    return fail(B2F_ERR_ARG, "gemm_fp8: output tensor map: " + err);
  return B2F_OK;
}

// Split-K calls tag their tile counters with a per-call epoch (24 bits, never 0), so a
// counter left mid-protocol by a call that timed out reads as zero in the next call.
std::atomic<unsigned> g_splitk_epoch{0};

unsigned next_splitk_epoch() {
  unsigned e;
  do {
    e = (g_splitk_epoch.fetch_add(1u, std::memory_order_relaxed) + 1u) & 0xFFFFFFu;
  } while (e == 0u);
  return e;
}

EpilogueParams make_epilogue(const b2f_gemm_args* a) {
  EpilogueParams ep;
  ep.epoch = next_splitk_epoch();
  ep.alpha = a->alpha;
  ep.alpha_ptr = a->alpha_ptr;
  ep.col_scale = a->col_scale;
  ep.bias = a->bias;
  ep.pre_mul = a->pre_mul;
  ep.pre_add = a->pre_add;
  ep.act = a->act;
  ep.act_param = a->act_param;
  ep.post_mul = a->post_mul;
  ep.gate = a->gate;
  ep.gate_dtype = a->gate_dtype;
  ep.gate_ld = a->gate_ld;
  {
    const int gsz = a->gate_dtype == B2F_DTYPE_F32 ? 4 : 2;
    ep.gate_vec = a->gate == nullptr ||
                  ((((uintptr_t)a->gate) % 16 == 0) && ((a->gate_ld * gsz) % 16 == 0));
  }
  ep.residual = a->residual;
  ep.res_dtype = a->residual_dtype;
  ep.res_ld = a->residual_ld;
  ep.res_scale = a->residual_scale;
  ep.out = a->out;
  ep.out_dtype = a->out_dtype;
  ep.out_ld = a->out_ld;
  ep.out_inv_scale = 1.0f / a->out_scale;
  ep.amax = a->amax;
  ep.mode = a->mode;
  ep.ws = nullptr;
  ep.ws_ld = 0;
  ep.ws_slice = 0;
  ep.counters = nullptr;
  ep.hp = HeadPrepParams{};
  const int esz = a->out_dtype == B2F_DTYPE_F32 ? 4 : (a->out_dtype == B2F_DTYPE_BF16 ? 2 : 1);
  const int rsz =
      a->residual_dtype == B2F_DTYPE_F32 ? 4 : (a->residual_dtype == B2F_DTYPE_BF16 ? 2 : 1);
  ep.out_vec = (((uintptr_t)a->out) % 16 == 0) && ((a->out_ld * esz) % 16 == 0);
  ep.res_vec = a->residual == nullptr ||
               ((((uintptr_t)a->residual) % 16 == 0) && ((a->residual_ld * rsz) % 16 == 0));
  return ep;
}

// Row blocks per raster group: at most 16, fewer when the group's A panel (rows x K bytes)
// would pass 32 MB, so that it stays in the 126 MB L2 while the group sweeps the column
// blocks (measured on CTA-pair tiles: 16384^3 2875 -> 2996 TFLOP/s with 8 row blocks; at
// 8192^3 and on the Qwen projections 16 was as good as or better than 8, 24 or 32).
int group_rows(int m, int k, int tile_rows) {
  const int num_m = (m + tile_rows - 1) / tile_rows;
  const long long panel = (long long)tile_rows * k;
  long long g = (32ll << 20) / (panel > 0 ? panel : 1);
  g = g < 4 ? 4 : (g > 16 ? 16 : g);
  return (int)std::min<long long>(g, num_m > 0 ? num_m : 1);
}

template <int BN>
int launch_gemm(const b2f_gemm_args* a, EpilogueParams ep, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  CUtensorMap ta, tb;
  std::string err;
  {
    const unsigned long long dims[2] = {(unsigned long long)a->k, (unsigned long long)a->m};
    const unsigned long long strides[1] = {(unsigned long long)a->lda};
    const unsigned int box[2] = {Cfg::BK, Cfg::BM};
    if (!encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a->a, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B, &err))
      return fail(B2F_ERR_ARG, "gemm_fp8: A tensor map: " + err);
  }
  {
    const unsigned long long dims[2] = {(unsigned long long)a->k, (unsigned long long)a->n};
    const unsigned long long strides[1] = {(unsigned long long)a->ldb};
    const unsigned int box[2] = {Cfg::BK, (unsigned int)BN};
    if (!encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a->b, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B, &err))
      return fail(B2F_ERR_ARG, "gemm_fp8: B tensor map: " + err);
  }
  const int num_tiles = ((a->m + Cfg::BM - 1) / Cfg::BM) * ((a->n + BN - 1) / BN);
  const int num_kb = (a->k + Cfg::BK - 1) / Cfg::BK;
  const int sms = sm_count();
  if (sms <= 0) return fail(B2F_ERR_CUDA, "gemm_fp8: cannot query SM count");
  int splits = a->splits;
  if (splits == 0) {
    // Automatic choice: two K slices when the tiles fill at most half of the SMs, K is
    // long and the caller passed a workspace (M=128, N=K=8192 on B200: 25.7 us unsplit,
    // 23.3 us in two slices, 31.4 us in three -- each extra slice adds a partial-tile
    // store and read); otherwise none.
    const bool ws_ok = a->workspace != nullptr &&
                       a->workspace_bytes >= b2f_gemm_workspace_bytes(a->m, a->n);
    splits = (ws_ok && num_tiles * 2 <= sms && num_kb >= 32) ? 2 : 1;
  }
  if (splits < 1 || splits > num_kb || splits > kMaxSplits)
    return fail(B2F_ERR_ARG, "gemm_fp8: splits must be in [1, min(8, K/128)]");
  if (splits > 1 && num_tiles > kMaxSplitTiles)
    return fail(B2F_ERR_UNSUPPORTED, "gemm_fp8: split-K supports at most 4096 output tiles");
  if (splits > 1) {
    if (a->workspace == nullptr ||
        a->workspace_bytes < b2f_gemm_workspace_bytes(a->m, a->n) ||
        (((uintptr_t)a->workspace) & 15))
      return fail(B2F_ERR_ARG, "gemm_fp8: split-K needs a 16-byte aligned workspace of "
                               "b2f_gemm_workspace_bytes(m, n) bytes");
    const long long ws_ld = (long long)((a->n + 255) / 256) * 256;
    const long long ws_rows = (long long)((a->m + 127) / 128) * 128;
    ep.counters = reinterpret_cast<unsigned int*>(a->workspace);
    ep.ws = reinterpret_cast<float*>(reinterpret_cast<char*>(a->workspace) + kCounterBytes);
    ep.ws_ld = ws_ld;
    ep.ws_slice = ws_rows * ws_ld;
  }
  GemmShape shape{a->m, a->n, a->k, splits, group_rows(a->m, a->k, 128)};
  const int units = num_tiles * splits;
  const int grid = units < sms ? units : sms;
  auto kern = shape.splits > 1 ? gemm_fp8_kernel<BN, kFeatSplitK>
                                : (ep.hp.on ? gemm_fp8_kernel<BN, kFeatHeadPrep>
                                            : gemm_fp8_kernel<BN, 0>);
  static thread_local int attr_dev = -1;
  int dev = 0;
  B2F_CUDA_TRY(cudaGetDevice(&dev));
  if (attr_dev != dev) {
    for (auto k : {gemm_fp8_kernel<BN, 0>, gemm_fp8_kernel<BN, kFeatSplitK>,
                   gemm_fp8_kernel<BN, kFeatHeadPrep>})
      B2F_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        Cfg::SMEM_BYTES));
    attr_dev = dev;
  }
  CUtensorMap to;
  // A warp's half tile must fill the 64-byte store box; narrower halves (e4m3 with
  // 64-column tiles) store directly.
  if ((BN / 2) * (a->out_dtype == B2F_DTYPE_F32 ? 4 : (a->out_dtype == B2F_DTYPE_BF16 ? 2 : 1)) < 64)
    ep.out_vec = 0;
  if (int rc = encode_out_map(a, ep, BN / 2, &to)) return rc;
  B2F_CUDA_TRY(launch_pdl(kern, dim3(grid), dim3(Cfg::THREADS), Cfg::SMEM_BYTES, stream, ta, tb,
                          to, shape, ep));
  B2F_CUDA_TRY(cudaGetLastError());
  return B2F_OK;
}

template <int PBN>
int launch_gemm_pair(const b2f_gemm_args* a, EpilogueParams ep, cudaStream_t stream) {
  using Cfg = Gemm2Cfg<PBN>;
  CUtensorMap ta, tb;
  std::string err;
  {
    const unsigned long long dims[2] = {(unsigned long long)a->k, (unsigned long long)a->m};
    const unsigned long long strides[1] = {(unsigned long long)a->lda};
    const unsigned int box[2] = {Cfg::BK, Cfg::BM};
    if (!encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a->a, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B, &err))
      return fail(B2F_ERR_ARG, "gemm_fp8: A tensor map: " + err);
  }
  {
    const unsigned long long dims[2] = {(unsigned long long)a->k, (unsigned long long)a->n};
    const unsigned long long strides[1] = {(unsigned long long)a->ldb};
    const unsigned int box[2] = {Cfg::BK, Cfg::BN / 2};
    if (!encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a->b, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B, &err))
      return fail(B2F_ERR_ARG, "gemm_fp8: B tensor map: " + err);
  }
  GemmShape shape{a->m, a->n, a->k, 1, group_rows(a->m, a->k, 256)};
  const int num_tiles = ((a->m + 255) / 256) * ((a->n + Cfg::BN - 1) / Cfg::BN);
  auto kern = ep.hp.on ? gemm_fp8_pair_kernel<PBN, kFeatHeadPrep> : gemm_fp8_pair_kernel<PBN, 0>;
  static thread_local int cached_dev = -1, cached_pairs = 0;  // per tile width
  int dev = 0;
  B2F_CUDA_TRY(cudaGetDevice(&dev));
  if (cached_dev != dev) {
    for (auto k : {gemm_fp8_pair_kernel<PBN, 0>, gemm_fp8_pair_kernel<PBN, kFeatHeadPrep>})
      B2F_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        Cfg::SMEM_BYTES));
    cudaLaunchConfig_t probe = {};
    probe.gridDim = dim3(2 * 256, 1, 1);
    probe.blockDim = dim3(Cfg::THREADS, 1, 1);
    probe.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2; attr.val.clusterDim.y = 1; attr.val.clusterDim.z = 1;
    probe.attrs = &attr;
    probe.numAttrs = 1;
    int clusters = 0;
    B2F_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, kern, &probe));
    if (clusters <= 0) return fail(B2F_ERR_UNSUPPORTED, "gemm_fp8: no co-resident CTA pairs");
    cached_pairs = clusters;
    cached_dev = dev;
  }
  g_pair_capacity = cached_pairs;
  const int pairs = num_tiles < cached_pairs ? num_tiles : cached_pairs;
  CUtensorMap to;
  if (int rc = encode_out_map(a, ep, Cfg::BN / 2, &to)) return rc;
  B2F_CUDA_TRY(launch_pdl(kern, dim3(2 * pairs), dim3(Cfg::THREADS), Cfg::SMEM_BYTES, stream,
                          ta, tb, to, shape, ep));
  B2F_CUDA_TRY(cudaGetLastError());
  return B2F_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Automatic tile choice of b2f_gemm_fp8 (tile_n = 0).
int auto_tile_n(const b2f_gemm_args* a) {
  int tn = 0;
  // CTA-pair 256 x 256 tiles for large problems with a long K loop.  Short K loops (the
  // K = 768 GEMMs of the GPT-2 block) run faster on single-CTA tiles (measured QKV 26.3
  // -> 24.4 us, FC 45.4 -> 41.0 us at M=8192); between 128- and 256-wide tiles the
  // choice weighs waves x tile width and takes 128 only when it saves a quarter
  // (out-projection N=768: 21.3 -> 17.5 us).  Few-tile problems use 128-wide tiles to
  // fill the 148 SMs.
  const int sms = sm_count();
  const long long rows128 = (a->m + 127) / 128;
  const long long tiles256 = rows128 * ((a->n + 255) / 256);
  const long long tiles128 = rows128 * ((a->n + 127) / 128);
  const long long pair_tiles = (long long)((a->m + 255) / 256) * ((a->n + 255) / 256);
  if (a->m > 128 && pair_tiles >= sms / 2 && a->k >= 2048) {
    // 256 x 256 pair tiles.  (256 x 128 pair tiles, tile_n -128, would halve the wave
    // quantisation of e.g. the 8192 x 2560 o-projection, but measured 1.5x slower there:
    // 104 vs 70 us.)
    tn = 512;
  } else if (a->workspace != nullptr && a->splits > 1 && tiles256 * 2 <= sms) {
    tn = 256;
  } else if (tiles256 < sms) {
    tn = 128;
  } else {
    const long long w256 = (tiles256 + sms - 1) / sms * 2;
    const long long w128 = (tiles128 + sms - 1) / sms;
    // (a tie goes to 128 for short K loops, where the epilogue dominates, and to 256 for
    // long ones: GPT-2's proj, N=768 K=3072, 33.1 us at 256 vs 38.4 at 128)
    tn = (a->k <= 1024 ? 4 * w128 <= 3 * w256 : 4 * w128 < 3 * w256) ? 128 : 256;
  }
  return tn;
}

int check_gemm_args(const b2f_gemm_args* a) {
  if (a == nullptr) return fail(B2F_ERR_ARG, "gemm_fp8: null args");
  if (a->m <= 0 || a->n <= 0 || a->k <= 0) return fail(B2F_ERR_ARG, "gemm_fp8: empty shape");
  if (a->a == nullptr || a->b == nullptr || a->out == nullptr)
    return fail(B2F_ERR_ARG, "gemm_fp8: null tensor");
  if (a->k % 16 != 0) return fail(B2F_ERR_ARG, "gemm_fp8: k must be a multiple of 16");
  if (a->lda < a->k || a->ldb < a->k || a->lda % 16 || a->ldb % 16)
    return fail(B2F_ERR_ARG, "gemm_fp8: lda/ldb must be >= k and multiples of 16");
  if (!aligned16(a->a) || !aligned16(a->b))
    return fail(B2F_ERR_ARG, "gemm_fp8: A and B must be 16-byte aligned");
  if (a->out_dtype < 0 || a->out_dtype > 2 || a->residual_dtype < 0 || a->residual_dtype > 2)
    return fail(B2F_ERR_ARG, "gemm_fp8: bad dtype");
  if (a->act < 0 || a->act > 4) return fail(B2F_ERR_ARG, "gemm_fp8: bad activation");
  if (a->mode != B2F_GEMM_STORE && a->mode != B2F_GEMM_ROWSUM)
    return fail(B2F_ERR_ARG, "gemm_fp8: bad mode");
  if (a->mode == B2F_GEMM_ROWSUM && a->out_dtype != B2F_DTYPE_F32)
    return fail(B2F_ERR_ARG, "gemm_fp8: ROWSUM needs an f32 output");
  if (a->mode == B2F_GEMM_STORE && a->out_ld < a->n)
    return fail(B2F_ERR_ARG, "gemm_fp8: out_ld < n");
  if (a->out_scale == 0.0f) return fail(B2F_ERR_ARG, "gemm_fp8: out_scale must be non-zero");
  const int esz = a->out_dtype == B2F_DTYPE_F32 ? 4 : (a->out_dtype == B2F_DTYPE_BF16 ? 2 : 1);
  if (((uintptr_t)a->out) % esz != 0) return fail(B2F_ERR_ARG, "gemm_fp8: misaligned out");
  if (a->residual != nullptr && a->residual_ld < a->n)
    return fail(B2F_ERR_ARG, "gemm_fp8: residual_ld < n");
  if (a->gate != nullptr &&
      ((a->gate_dtype != B2F_DTYPE_F32 && a->gate_dtype != B2F_DTYPE_BF16) || a->gate_ld < a->n ||
       ((uintptr_t)a->gate) % (a->gate_dtype == B2F_DTYPE_F32 ? 4 : 2) != 0))
    return fail(B2F_ERR_ARG, "gemm_fp8: gate must be f32 or bf16 with gate_ld >= n");
  if (a->col_scale != nullptr && ((uintptr_t)a->col_scale) % 16 != 0)
    return fail(B2F_ERR_ARG, "gemm_fp8: col_scale must be 16-byte aligned");
  if (a->bias != nullptr && ((uintptr_t)a->bias) % 16 != 0)
    return fail(B2F_ERR_ARG, "gemm_fp8: bias must be 16-byte aligned");
  return B2F_OK;
}


}  // namespace
}  // namespace b2f

extern "C" {

void b2f_gemm_args_init(b2f_gemm_args* a) {
  if (a == nullptr) return;
  *a = b2f_gemm_args{};
  a->alpha = 1.0f;
  a->pre_mul = 1.0f;
  a->pre_add = 0.0f;
  a->act = B2F_ACT_NONE;
  a->act_param = 0.0f;
  a->post_mul = 1.0f;
  a->residual_dtype = B2F_DTYPE_BF16;
  a->residual_scale = 1.0f;
  a->out_dtype = B2F_DTYPE_BF16;
  a->out_scale = 1.0f;
  a->mode = B2F_GEMM_STORE;
  a->tile_n = 0;
  a->gate = nullptr;
  a->gate_dtype = B2F_DTYPE_F32;
  a->gate_ld = 0;
}

int b2f_gemm_fp8_head_prep(const b2f_gemm_args* a, const b2f_head_prep_args* h,
                           b2f_stream_t stream) {
  using namespace b2f;
  if (a == nullptr || h == nullptr) return fail(B2F_ERR_ARG, "gemm_fp8_head_prep: null args");
  if (a->out_dtype != B2F_DTYPE_E4M3 || a->mode != B2F_GEMM_STORE ||
      a->act != B2F_ACT_NONE || a->residual != nullptr || a->gate != nullptr ||
      a->amax != nullptr || a->splits > 1 || a->pre_mul != 1.0f || a->pre_add != 0.0f ||
      a->post_mul != 1.0f)
    return fail(B2F_ERR_ARG, "gemm_fp8_head_prep: e4m3 output with a plain epilogue (alpha, "
                             "column scale, bias), no split-K");
  auto head_ok = [&](int off, int stride, int heads) {
    return heads >= 0 && off >= 0 && off % 128 == 0 && stride % 128 == 0 &&
           (heads == 0 || off + (long long)(heads - 1) * stride + 128 <= a->n);
  };
  // every head must be a whole 128-column half of a 256-column tile: offsets multiples of
  // 128 do that by construction
  if (h->q_heads < 0 || h->k_heads < 0 || h->v_heads < 0 || h->q_head_stride < 128 ||
      !head_ok(h->q_off, h->q_head_stride, h->q_heads) || !head_ok(h->k_off, 128, h->k_heads) ||
      !head_ok(h->v_off, 128, h->v_heads))
    return fail(B2F_ERR_ARG, "gemm_fp8_head_prep: head columns must be 128-aligned and inside n");
  if ((h->q_heads && (h->q_out == nullptr || h->q_ld < 128LL * h->q_heads || h->q_ld % 16 ||
                      ((uintptr_t)h->q_out & 15))) ||
      (h->k_heads && (h->k_out == nullptr || h->k_ld < 128LL * h->k_heads || h->k_ld % 16 ||
                      ((uintptr_t)h->k_out & 15))) ||
      (h->v_heads && (h->v_out == nullptr || h->v_ld < 128LL * h->v_heads || h->v_ld % 8 ||
                      ((uintptr_t)h->v_out & 15))))
    return fail(B2F_ERR_ARG, "gemm_fp8_head_prep: q/k/v outputs: 16-byte aligned rows wide "
                             "enough for their heads");
  if (h->v_dtype != B2F_DTYPE_F16 && h->v_dtype != B2F_DTYPE_BF16)
    return fail(B2F_ERR_ARG, "gemm_fp8_head_prep: v_dtype must be f16 or bf16");
  if ((h->rope_cos == nullptr) != (h->rope_sin == nullptr) ||
      (h->rope_cos != nullptr && (h->seq <= 0 || ((uintptr_t)h->rope_cos & 15) ||
                                  ((uintptr_t)h->rope_sin & 15))))
    return fail(B2F_ERR_ARG, "gemm_fp8_head_prep: rope tables [seq][128], 16-byte aligned");
  if (((uintptr_t)h->q_norm_w & 15) || ((uintptr_t)h->k_norm_w & 15))
    return fail(B2F_ERR_ARG, "gemm_fp8_head_prep: norm weights must be 16-byte aligned");
  if (!(h->out_scale > 0.0f) || !(a->out_scale > 0.0f))
    return fail(B2F_ERR_ARG, "gemm_fp8_head_prep: scales must be positive");
  if (a->col_scale != nullptr && ((uintptr_t)a->col_scale) % 16 != 0)
    return fail(B2F_ERR_ARG, "gemm_fp8: col_scale must be 16-byte aligned");
  // the plain-GEMM argument checks (shape, operands, output)
  b2f_gemm_args plain = *a;
  plain.splits = 1;
  plain.workspace = nullptr;
  if (int rc = check_gemm_args(&plain)) return rc;
  // 256-column tiles (each head one 128-column half): CTA pairs where the plain GEMM would
  // use them, else single-CTA 128 x 256 tiles
  const int auto_tn = auto_tile_n(&plain);
  const bool pair = auto_tn == 512 || auto_tn == -128;
  plain.tile_n = pair ? 512 : 256;
  EpilogueParams ep = make_epilogue(&plain);
  HeadPrepParams& p = ep.hp;
  p.on = 1;
  p.q_off = h->q_off; p.q_hstride = h->q_head_stride; p.q_heads = h->q_heads;
  p.k_off = h->k_off; p.k_heads = h->k_heads;
  p.v_off = h->v_off; p.v_heads = h->v_heads;
  p.v_f16 = h->v_dtype == B2F_DTYPE_F16;
  p.q_out = static_cast<uint8_t*>(h->q_out); p.q_ld = h->q_ld;
  p.k_out = static_cast<uint8_t*>(h->k_out); p.k_ld = h->k_ld;
  p.v_out = static_cast<uint16_t*>(h->v_out); p.v_ld = h->v_ld;
  p.q_w = h->q_norm_w; p.k_w = h->k_norm_w;
  p.w_offset = h->weight_offset; p.eps = h->eps;
  p.cos = h->rope_cos; p.sin = h->rope_sin; p.seq = h->seq;
  p.x_scale = a->out_scale;
  p.out_inv_scale = 1.0f / h->out_scale;
  return pair ? launch_gemm_pair<256>(&plain, ep, (cudaStream_t)stream)
              : launch_gemm<256>(&plain, ep, (cudaStream_t)stream);
}

int b2f_gemm_pair_capacity(void) { return b2f::g_pair_capacity; }

long long b2f_gemm_workspace_bytes(int m, int n) {
  if (m <= 0 || n <= 0) return 0;
  const long long ld = (long long)((n + 255) / 256) * 256;   // column tiles of 256
  const long long rows = (long long)((m + 127) / 128) * 128;  // row tiles of 128
  return b2f::kCounterBytes + b2f::kMaxSplits * rows * ld * 4;
}

int b2f_gemm_fp8(const b2f_gemm_args* a, b2f_stream_t stream) {
  using namespace b2f;
  if (int rc = check_gemm_args(a)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  int tn = a->tile_n;
  if (tn == 0) tn = auto_tile_n(a);
  const EpilogueParams ep = make_epilogue(a);
  if (tn == 512 || tn == -256 || tn == -128) {
    if (a->splits > 1) return fail(B2F_ERR_UNSUPPORTED, "gemm_fp8: split-K uses tile_n 128 or 256");
    return tn == -128 ? launch_gemm_pair<128>(a, ep, s) : launch_gemm_pair<256>(a, ep, s);
  }
  if (tn == 256) return launch_gemm<256>(a, ep, s);
  if (tn == 128) return launch_gemm<128>(a, ep, s);
  if (tn == 64) {
    if (a->splits > 1) return fail(B2F_ERR_UNSUPPORTED, "gemm_fp8: split-K uses tile_n 128 or 256");
    return launch_gemm<64>(a, ep, s);
  }
  return fail(B2F_ERR_ARG,
              "gemm_fp8: tile_n must be 0, 64, 128, 256, or -128 / -256 / 512 (CTA pair)");
}

}  // extern "C"


// ---------------------------------------------------------------------------------------
// Allocation-free split-K GEMM (b2f_gemm_fp8_static).
//
// Some callers cannot allocate device memory at call time: a kernel library loaded as a
// plugin into a host framework that owns every device allocation through its own
// allocator, or a serving loop whose memory plan is fixed at start-up and forbids any
// allocation afterwards.  They cannot hand the split-K GEMM a workspace, so this entry
// point keeps its scratch in a file-scope device array instead.
//
// kStaticScratchBytes (8 MiB of f32 partial tiles + 16 KiB of tile counters) lives on
// every GPU that loads this library until the process exits.  Host code only ever sees
// the array's host-side shadow symbol, which is not a device address: the device address
// is looked up with cudaGetSymbolAddress once per device and context, with that device
// current, on the first call made on the device (so make that first call before any
// stream capture); after a cudaDeviceReset the next call looks it up again.
// Every call shares the one array and keeps the last call's partial tiles; the counters
// that must start at zero are cleared (cudaMemsetAsync on the call's stream) at the start
// of every call.  Calls that overlap on the GPU - on two streams, or from two host
// threads - race on the array and must be serialised by the caller.
namespace b2f {
namespace {

constexpr long long kStaticScratchBytes = kCounterBytes + 8ll * 1024 * 1024;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_static_mu;
// Per device: the device address of g_static_scratch and the context it was looked up in
// (a context reset invalidates both the address and the kernels' shared-memory attribute).
struct StaticSlot {
  unsigned long long ctx = 0;
  void* ptr = nullptr;
  bool attr256 = false, attr128 = false;
};
constexpr int kMaxDevices = 64;
StaticSlot g_static_slots[kMaxDevices];  // fixed storage: callers keep pointers into it

int static_scratch_address(void** out, bool** attr_done, int bn) {
  int dev = 0;
  B2F_CUDA_TRY(cudaGetDevice(&dev));
  const unsigned long long ctx = context_token();
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (dev < 0 || dev >= kMaxDevices) return fail(B2F_ERR_UNSUPPORTED, "gemm_fp8_static: device ordinal");
  StaticSlot& slot = g_static_slots[dev];
  if (slot.ptr == nullptr || slot.ctx != ctx || ctx == 0) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr)
      return cuda_fail(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                       "cudaGetSymbolAddress(g_static_scratch)");
    slot = StaticSlot{};
    slot.ptr = p;
    slot.ctx = ctx;
  }
  *out = slot.ptr;
  *attr_done = bn == 256 ? &slot.attr256 : &slot.attr128;
  return B2F_OK;
}

template <int BN>
int launch_gemm_static(const b2f_gemm_args* a, int splits, void* scratch, bool* attr_done,
                       cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  CUtensorMap ta, tb;
  std::string err;
  {
    const unsigned long long dims[2] = {(unsigned long long)a->k, (unsigned long long)a->m};
    const unsigned long long strides[1] = {(unsigned long long)a->lda};
    const unsigned int box[2] = {Cfg::BK, Cfg::BM};
    if (!encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a->a, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B, &err))
      return fail(B2F_ERR_ARG, "gemm_fp8_static: A tensor map: " + err);
  }
  {
    const unsigned long long dims[2] = {(unsigned long long)a->k, (unsigned long long)a->n};
    const unsigned long long strides[1] = {(unsigned long long)a->ldb};
    const unsigned int box[2] = {Cfg::BK, (unsigned int)BN};
    if (!encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a->b, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B, &err))
      return fail(B2F_ERR_ARG, "gemm_fp8_static: B tensor map: " + err);
  }
  EpilogueParams ep = make_epilogue(a);
  const long long ws_ld = (long long)((a->n + 255) / 256) * 256;
  const long long ws_rows = (long long)((a->m + 127) / 128) * 128;
  ep.counters = reinterpret_cast<unsigned int*>(scratch);
  ep.ws = reinterpret_cast<float*>(reinterpret_cast<char*>(scratch) + kCounterBytes);
  ep.ws_ld = ws_ld;
  ep.ws_slice = ws_rows * ws_ld;
  const int num_tiles = ((a->m + Cfg::BM - 1) / Cfg::BM) * ((a->n + BN - 1) / BN);
  const int sms = sm_count();
  if (sms <= 0) return fail(B2F_ERR_CUDA, "gemm_fp8_static: cannot query SM count");
  GemmShape shape{a->m, a->n, a->k, splits, group_rows(a->m, a->k, 128)};
  const int units = num_tiles * splits;
  const int grid = units < sms ? units : sms;
  if (!*attr_done) {
    B2F_CUDA_TRY(cudaFuncSetAttribute(gemm_fp8_kernel<BN, kFeatSplitK>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      Cfg::SMEM_BYTES));
    *attr_done = true;
  }
  CUtensorMap to;
  if (int rc = encode_out_map(a, ep, BN / 2, &to)) return rc;
  // Tile counters must start at zero: clear them on the call's stream.
  B2F_CUDA_TRY(cudaMemsetAsync(scratch, 0, kCounterBytes, stream));
  gemm_fp8_kernel<BN, kFeatSplitK><<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(ta, tb, to,
                                                                                    shape, ep);
  B2F_CUDA_TRY(cudaGetLastError());
  return B2F_OK;
}

}  // namespace
}  // namespace b2f

extern "C" int b2f_gemm_fp8_static(const b2f_gemm_args* a, b2f_stream_t stream) {
  using namespace b2f;
  if (a == nullptr) return fail(B2F_ERR_ARG, "gemm_fp8_static: null args");
  if (a->m <= 0 || a->n <= 0 || a->k <= 0) return fail(B2F_ERR_ARG, "gemm_fp8_static: empty shape");
  if (a->a == nullptr || a->b == nullptr || a->out == nullptr)
    return fail(B2F_ERR_ARG, "gemm_fp8_static: null tensor");
  if (a->k % 16 != 0 || a->lda < a->k || a->ldb < a->k || a->lda % 16 || a->ldb % 16 ||
      !aligned16(a->a) || !aligned16(a->b))
    return fail(B2F_ERR_ARG, "gemm_fp8_static: k, lda, ldb must be multiples of 16 and A, B "
                             "16-byte aligned");
  if (a->out_dtype < 0 || a->out_dtype > 2 || a->residual_dtype < 0 || a->residual_dtype > 2 ||
      a->act < 0 || a->act > 4 || (a->mode != B2F_GEMM_STORE && a->mode != B2F_GEMM_ROWSUM) ||
      (a->mode == B2F_GEMM_ROWSUM && a->out_dtype != B2F_DTYPE_F32))
    return fail(B2F_ERR_ARG, "gemm_fp8_static: bad dtype, activation or mode");
  if ((a->mode == B2F_GEMM_STORE && a->out_ld < a->n) || a->out_scale == 0.0f ||
      (a->residual != nullptr && a->residual_ld < a->n) ||
      (a->gate != nullptr && ((a->gate_dtype != B2F_DTYPE_F32 && a->gate_dtype != B2F_DTYPE_BF16) ||
                              a->gate_ld < a->n)))
    return fail(B2F_ERR_ARG, "gemm_fp8_static: bad output / residual layout or scale");
  const int esz = a->out_dtype == B2F_DTYPE_F32 ? 4 : (a->out_dtype == B2F_DTYPE_BF16 ? 2 : 1);
  if (((uintptr_t)a->out) % esz != 0 || (a->bias != nullptr && !aligned16(a->bias)) ||
      (a->col_scale != nullptr && !aligned16(a->col_scale)))
    return fail(B2F_ERR_ARG, "gemm_fp8_static: misaligned output, bias or col_scale");
  const int num_kb = (a->k + 127) / 128;
  int splits = a->splits;
  if (splits == 0) splits = 2;  // fastest measured (M=128, N=K=8192: two slices 23.3 us)
  if (splits < 2 || splits > kMaxSplits || splits > num_kb)
    return fail(B2F_ERR_ARG, "gemm_fp8_static: splits must be in [2, min(8, K/128)]");
  const int tn = a->tile_n == 0 ? 256 : a->tile_n;
  if (tn != 128 && tn != 256)
    return fail(B2F_ERR_ARG, "gemm_fp8_static: tile_n must be 0, 128 or 256");
  const long long rows = (long long)((a->m + 127) / 128) * 128;
  const long long ld = (long long)((a->n + 255) / 256) * 256;
  const long long need = kCounterBytes + (long long)splits * rows * ld * 4;
  const long long tiles = (rows / 128) * ((a->n + tn - 1) / tn);
  if (need > kStaticScratchBytes || tiles > kMaxSplitTiles)
    return fail(B2F_ERR_ARG,
                "gemm_fp8_static: splits * ceil(m/128)*128 * ceil(n/256)*256 * 4 bytes = " +
                    std::to_string(need - kCounterBytes) +
                    " exceeds the 8 MiB static scratch; use b2f_gemm_fp8 with a workspace");
  void* scratch = nullptr;
  bool* attr_done = nullptr;
  if (int rc = static_scratch_address(&scratch, &attr_done, tn)) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  if (tn == 256) return launch_gemm_static<256>(a, splits, scratch, attr_done, s);
  return launch_gemm_static<128>(a, splits, scratch, attr_done, s);
}
