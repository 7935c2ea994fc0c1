// Whole decoder blocks behind the C ABI (b2f_gpt2_block, b2f_qwen_block): host code that
// runs this library's kernels in each reference evaluator's dataflow order on one stream,
// with every intermediate carved out of a caller workspace (no allocation here).  The
// sequence and the arguments of each launch are those of the Python blocks in
// b200fp8/blocks.py, so both produce the same bits.
//
// Reference math: tasks/model_gpt2_small_transformer_block_fp8/starter.py:393-488,
// tasks/model_qwen35_4b_vision_block_fp8/starter.py:303-369,
// tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:333-416.
#include <cstring>
#include <string>

#include "host_common.h"

namespace b2f {
namespace {

int esize(int dt) { return dt == B2F_DTYPE_F32 ? 4 : (dt == B2F_DTYPE_E4M3 ? 1 : 2); }

// GEMM alpha = scale_a * scale_b, formed in double and rounded once (as the Python blocks
// form it from Python floats), so both paths pass the same f32 alpha.
float alpha_of(float sa, float sb) { return (float)((double)sa * (double)sb); }

// Bump allocator over the caller workspace (256-byte aligned slices).
struct Carve {
  char* base;
  long long used = 0;
  explicit Carve(void* b) : base(static_cast<char*>(b)) {}
  char* take(long long bytes) {
    char* p = base == nullptr ? nullptr : base + used;
    used += (bytes + 255) / 256 * 256;
    return p;
  }
};

// V operand of the blocks: f16 for head_dim 64 / 128 (P is then rounded to f16, 2^-11
// relative, at the same speed as bf16 P), bf16 for head_dim 256 (the only form that
// kernel takes).  Both hold the e4m3 values exactly.
int v_dtype(int head_dim) { return head_dim <= 128 ? B2F_DTYPE_F16 : B2F_DTYPE_BF16; }

int v_convert(const void* in, long long in_ld, void* out, long long rows, int cols, int dt,
              b2f_stream_t s) {
  return dt == B2F_DTYPE_F16 ? b2f_fp8_to_f16(in, in_ld, out, cols, (int)rows, cols, 1.0f, s)
                             : b2f_fp8_to_bf16(in, in_ld, out, cols, (int)rows, cols, 1.0f, s);
}

struct Gpt2Buffers {
  char *n1, *qkv, *v, *ctx, *r1, *n2, *h, *q_rot, *k_rot;
};

long long gpt2_carve(const b2f_gpt2_block_args* a, void* ws, Gpt2Buffers& b) {
  const long long t = (long long)a->batch * a->seq, d = a->d_model;
  const int hd = a->d_model / a->heads;
  Carve c(ws);
  b.n1 = c.take(t * d);
  b.qkv = c.take(t * 3 * d);
  b.v = c.take(t * d * 2);
  b.ctx = c.take(t * d);
  b.r1 = c.take(t * d * esize(a->residual_dtype));
  b.n2 = c.take(t * d);
  b.h = c.take(t * a->mlp);
  b.q_rot = b.k_rot = nullptr;
  if (a->rope_cos != nullptr) {
    b.q_rot = c.take(t * d);
    b.k_rot = c.take(t * d);
  }
  (void)hd;
  return c.used;
}

struct QwenBuffers {
  char *n1, *proj, *q, *k, *v, *ctx, *r1, *n2, *gu, *act;
};

int qwen_ncat(const b2f_qwen_block_args* a) {
  return 2 * a->heads * a->head_dim + 2 * a->kv_heads * a->head_dim;
}

long long qwen_carve(const b2f_qwen_block_args* a, void* ws, QwenBuffers& b) {
  const long long t = (long long)a->batch * a->seq;
  const long long hq = (long long)a->heads * a->head_dim, hk = (long long)a->kv_heads * a->head_dim;
  Carve c(ws);
  b.n1 = c.take(t * a->hidden);
  b.proj = c.take(t * qwen_ncat(a));
  b.q = c.take(t * hq);
  b.k = c.take(t * hk);
  b.v = c.take(t * hk * 2);
  b.ctx = c.take(t * hq);
  b.r1 = b.n2 = b.gu = b.act = nullptr;
  if (a->mlp_gu_w != nullptr) {
    b.r1 = c.take(t * a->hidden * esize(a->residual_dtype));
    b.n2 = c.take(t * a->hidden);
    b.gu = c.take(t * 2LL * a->inter);
    b.act = c.take(t * (long long)a->inter);
  }
  return c.used;
}

// One GEMM launch of the blocks: A e4m3 [m, k] (dense), B e4m3 [n, k], output row pitch n.
struct Gemm {
  b2f_gemm_args g;
  Gemm(int m, int n, int k, const void* a, const void* b, void* out, int out_dtype) {
    b2f_gemm_args_init(&g);
    g.m = m; g.n = n; g.k = k;
    g.a = a; g.lda = k;
    g.b = b; g.ldb = k;
    g.out = out; g.out_dtype = out_dtype; g.out_ld = n;
  }
};

}  // namespace
}  // namespace b2f

extern "C" {

void b2f_gpt2_block_args_init(b2f_gpt2_block_args* a) {
  if (a == nullptr) return;
  std::memset(a, 0, sizeof(*a));
  a->hidden_dtype = B2F_DTYPE_BF16;
  a->hidden_scale = 1.0f;
  a->eps = 1e-5f;
  a->norm_scale = a->qkv_scale = a->ctx_scale = a->mlp_scale = 1.0f / 64.0f;
  a->causal = 1;
  a->residual_dtype = B2F_DTYPE_BF16;
  a->out_dtype = B2F_DTYPE_BF16;
}

long long b2f_gpt2_block_workspace_bytes(const b2f_gpt2_block_args* a) {
  using namespace b2f;
  if (a == nullptr) return -1;
  Gpt2Buffers b;
  return gpt2_carve(a, nullptr, b);
}

int b2f_gpt2_block(const b2f_gpt2_block_args* a, b2f_stream_t s) {
  using namespace b2f;
  if (a == nullptr) return fail(B2F_ERR_ARG, "gpt2_block: null args");
  if (a->batch <= 0 || a->seq <= 0 || a->d_model <= 0 || a->heads <= 0 || a->mlp <= 0 ||
      a->d_model % a->heads)
    return fail(B2F_ERR_ARG, "gpt2_block: bad shape");
  if (a->hidden == nullptr || a->out == nullptr || a->qkv_w == nullptr || a->out_w == nullptr ||
      a->fc_w == nullptr || a->proj_w == nullptr || a->ln1_w == nullptr || a->ln2_w == nullptr)
    return fail(B2F_ERR_ARG, "gpt2_block: null tensor");
  if ((a->residual_dtype != B2F_DTYPE_BF16 && a->residual_dtype != B2F_DTYPE_F32) ||
      (a->out_dtype != B2F_DTYPE_BF16 && a->out_dtype != B2F_DTYPE_F32))
    return fail(B2F_ERR_ARG, "gpt2_block: residual / out must be bf16 or f32");
  Gpt2Buffers b;
  const long long need = gpt2_carve(a, a->workspace, b);
  if (a->workspace == nullptr || a->workspace_bytes < need ||
      (reinterpret_cast<uintptr_t>(a->workspace) & 255))
    return fail(B2F_ERR_ARG, "gpt2_block: workspace must be 256-byte aligned and hold "
                             "b2f_gpt2_block_workspace_bytes bytes");
  const int t = a->batch * a->seq, d = a->d_model, hd = d / a->heads;
  const float ns = a->norm_scale, qs = a->qkv_scale, cs = a->ctx_scale, ms = a->mlp_scale;
  int rc;
  // LN1 -> n1
  {
    b2f_norm_args n;
    b2f_norm_args_init(&n);
    n.rows = t; n.cols = d;
    n.x = a->hidden; n.x_dtype = a->hidden_dtype; n.x_scale = a->hidden_scale; n.x_ld = a->hidden_ld;
    n.weight = a->ln1_w; n.bias = a->ln1_b; n.weight_dtype = B2F_DTYPE_F32;
    n.kind = B2F_NORM_LAYER; n.eps = a->eps;
    n.q_out = b.n1; n.q_ld = d; n.q_scale = ns;
    if ((rc = b2f_norm_quant(&n, s))) return rc;
  }
  // QKV + bias -> e4m3, the 16-bit V image from the same epilogue where the V columns are
  // whole 128-column blocks, else by a separate conversion
  const int vdt = v_dtype(hd);
  {
    Gemm g(t, 3 * d, d, b.n1, a->qkv_w, b.qkv, B2F_DTYPE_E4M3);
    g.g.alpha = alpha_of(ns, a->qkv_s); g.g.bias = a->qkv_b; g.g.out_scale = qs;
    bool fused = false;
    if (d % 128 == 0) {
      b2f_head_prep_args hp;
      std::memset(&hp, 0, sizeof(hp));
      hp.q_head_stride = 128;
      hp.v_off = 2 * d; hp.v_heads = d / 128;
      hp.v_out = b.v; hp.v_ld = d; hp.v_dtype = vdt;
      hp.out_scale = qs;
      rc = b2f_gemm_fp8_head_prep(&g.g, &hp, s);
      if (rc == B2F_OK) fused = true;
      else if (rc != B2F_ERR_UNSUPPORTED) return rc;
    }
    if (!fused) {
      if ((rc = b2f_gemm_fp8(&g.g, s))) return rc;
      if ((rc = v_convert(b.qkv + 2 * d, 3 * d, b.v, t, d, vdt, s))) return rc;
    }
  }
  const char* q = b.qkv;
  const char* k = b.qkv + d;
  long long q_ld = 3 * d, k_ld = 3 * d;
  if (a->rope_cos != nullptr) {
    for (int which = 0; which < 2; ++which) {
      b2f_rope_args r;
      std::memset(&r, 0, sizeof(r));
      r.rows = t; r.heads = a->heads; r.head_dim = hd;
      r.in = which == 0 ? q : k; r.in_ld = 3 * d; r.in_head_stride = hd; r.in_scale = qs;
      r.weight = nullptr; r.weight_offset = 1.0f; r.eps = 1e-6f;
      r.cos = a->rope_cos; r.sin = a->rope_sin; r.rotary_dim = hd; r.seq = a->seq;
      r.out = which == 0 ? b.q_rot : b.k_rot; r.out_ld = d; r.out_scale = qs;
      if ((rc = b2f_head_norm_rope(&r, s))) return rc;
    }
    q = b.q_rot; k = b.k_rot; q_ld = k_ld = d;
  }
  {
    b2f_attn_args at;
    b2f_attn_args_init(&at);
    at.batch = a->batch; at.seq = a->seq; at.hq = a->heads; at.hkv = a->heads; at.head_dim = hd;
    at.causal = a->causal;
    at.q = q; at.q_ld = q_ld; at.q_scale = qs;
    at.k = k; at.k_ld = k_ld; at.k_scale = qs;
    at.v = b.v; at.v_ld = d; at.v_scale = qs; at.v_dtype = vdt;
    at.ctx = b.ctx; at.ctx_ld = d; at.ctx_scale = cs;
    if ((rc = b2f_attention_fp8(&at, s))) return rc;
  }
  // out-proj + bias + hidden -> r1
  {
    Gemm g(t, d, d, b.ctx, a->out_w, b.r1, a->residual_dtype);
    g.g.alpha = alpha_of(cs, a->out_s); g.g.bias = a->out_b;
    g.g.residual = a->hidden; g.g.residual_dtype = a->hidden_dtype;
    g.g.residual_ld = a->hidden_ld; g.g.residual_scale = a->hidden_scale;
    if ((rc = b2f_gemm_fp8(&g.g, s))) return rc;
  }
  // LN2 -> n2
  {
    b2f_norm_args n;
    b2f_norm_args_init(&n);
    n.rows = t; n.cols = d;
    n.x = b.r1; n.x_dtype = a->residual_dtype; n.x_ld = d;
    n.weight = a->ln2_w; n.bias = a->ln2_b; n.weight_dtype = B2F_DTYPE_F32;
    n.kind = B2F_NORM_LAYER; n.eps = a->eps;
    n.q_out = b.n2; n.q_ld = d; n.q_scale = ns;
    if ((rc = b2f_norm_quant(&n, s))) return rc;
  }
  // FC + bias + GELU-tanh -> e4m3
  {
    Gemm g(t, a->mlp, d, b.n2, a->fc_w, b.h, B2F_DTYPE_E4M3);
    g.g.alpha = alpha_of(ns, a->fc_s); g.g.bias = a->fc_b; g.g.act = B2F_ACT_GELU_TANH; g.g.out_scale = ms;
    if ((rc = b2f_gemm_fp8(&g.g, s))) return rc;
  }
  // proj + bias + r1 -> out
  {
    Gemm g(t, d, a->mlp, b.h, a->proj_w, a->out, a->out_dtype);
    g.g.out_ld = a->out_ld;
    g.g.alpha = alpha_of(ms, a->proj_s); g.g.bias = a->proj_b;
    g.g.residual = b.r1; g.g.residual_dtype = a->residual_dtype; g.g.residual_ld = d;
    if ((rc = b2f_gemm_fp8(&g.g, s))) return rc;
  }
  return B2F_OK;
}

void b2f_qwen_block_args_init(b2f_qwen_block_args* a) {
  if (a == nullptr) return;
  std::memset(a, 0, sizeof(*a));
  a->hidden_dtype = B2F_DTYPE_BF16;
  a->hidden_scale = 1.0f;
  a->eps = 1e-6f;
  a->norm_scale = a->qkv_scale = a->ctx_scale = 1.0f / 64.0f;
  a->mlp_proj_scale = 1.0f / 64.0f;
  a->mlp_act_scale = 1.0f / 32.0f;
  a->add_residual = 1;
  a->residual_dtype = B2F_DTYPE_BF16;
  a->out_dtype = B2F_DTYPE_BF16;
}

long long b2f_qwen_block_workspace_bytes(const b2f_qwen_block_args* a) {
  using namespace b2f;
  if (a == nullptr) return -1;
  QwenBuffers b;
  return qwen_carve(a, nullptr, b);
}

int b2f_qwen_block(const b2f_qwen_block_args* a, b2f_stream_t s) {
  using namespace b2f;
  if (a == nullptr) return fail(B2F_ERR_ARG, "qwen_block: null args");
  if (a->batch <= 0 || a->seq <= 0 || a->hidden <= 0 || a->heads <= 0 || a->kv_heads <= 0 ||
      a->head_dim <= 0 || a->heads % a->kv_heads || a->rotary_dim <= 0 ||
      a->rotary_dim > a->head_dim)
    return fail(B2F_ERR_ARG, "qwen_block: bad shape");
  if (a->hidden_in == nullptr || a->out == nullptr || a->qgkv_w == nullptr ||
      a->qgkv_col_scale == nullptr || a->o_w == nullptr || a->in_norm_w == nullptr ||
      a->q_norm_w == nullptr || a->k_norm_w == nullptr || a->rope_cos == nullptr ||
      a->rope_sin == nullptr)
    return fail(B2F_ERR_ARG, "qwen_block: null tensor");
  const bool mlp = a->mlp_gu_w != nullptr;
  if (mlp && (a->mlp_gu_col_scale == nullptr || a->mlp_down_w == nullptr ||
              a->post_norm_w == nullptr || a->inter <= 0))
    return fail(B2F_ERR_ARG, "qwen_block: incomplete MLP");
  if (mlp && !a->add_residual)
    return fail(B2F_ERR_ARG, "qwen_block: add_residual = 0 needs a block without the MLP");
  if ((a->residual_dtype != B2F_DTYPE_BF16 && a->residual_dtype != B2F_DTYPE_F32) ||
      (a->out_dtype != B2F_DTYPE_BF16 && a->out_dtype != B2F_DTYPE_F32))
    return fail(B2F_ERR_ARG, "qwen_block: residual / out must be bf16 or f32");
  QwenBuffers b;
  const long long need = qwen_carve(a, a->workspace, b);
  if (a->workspace == nullptr || a->workspace_bytes < need ||
      (reinterpret_cast<uintptr_t>(a->workspace) & 255))
    return fail(B2F_ERR_ARG, "qwen_block: workspace must be 256-byte aligned and hold "
                             "b2f_qwen_block_workspace_bytes bytes");
  const int t = a->batch * a->seq, hid = a->hidden, h = a->heads, hk = a->kv_heads;
  const int dh = a->head_dim, ncat = qwen_ncat(a);
  const float ns = a->norm_scale, qs = a->qkv_scale, cs = a->ctx_scale;
  // packed-row offsets of q, gate, k, v within one projected row
  const int q_off = 0, q_hstride = a->interleaved ? 2 * dh : dh;
  const int g_off = a->interleaved ? dh : h * dh;
  const int k_off = 2 * h * dh, v_off = k_off + hk * dh;
  int rc;
  {
    b2f_norm_args n;
    b2f_norm_args_init(&n);
    n.rows = t; n.cols = hid;
    n.x = a->hidden_in; n.x_dtype = a->hidden_dtype; n.x_scale = a->hidden_scale;
    n.x_ld = a->hidden_ld;
    n.weight = a->in_norm_w; n.weight_dtype = B2F_DTYPE_F32; n.weight_offset = 1.0f;
    n.kind = B2F_NORM_RMS; n.eps = a->eps;
    n.q_out = b.n1; n.q_ld = hid; n.q_scale = ns;
    if ((rc = b2f_norm_quant(&n, s))) return rc;
  }
  const int vdt = v_dtype(dh);
  // The 16-bit V image from the projection GEMM's epilogue where the V columns are whole
  // 128-column blocks (the q / k norm + RoPE stay a separate launch: in the epilogue each
  // thread owns one row and its rotary-table loads would not coalesce).
  bool v_done = false;
  if ((long long)hk * dh % 128 == 0 && v_off % 128 == 0) {
    Gemm g(t, ncat, hid, b.n1, a->qgkv_w, b.proj, B2F_DTYPE_E4M3);
    g.g.col_scale = a->qgkv_col_scale; g.g.out_scale = qs;
    b2f_head_prep_args hp;
    std::memset(&hp, 0, sizeof(hp));
    hp.q_head_stride = 128;
    hp.v_off = v_off; hp.v_heads = hk * dh / 128;
    hp.v_out = b.v; hp.v_ld = (long long)hk * dh; hp.v_dtype = vdt;
    hp.out_scale = qs;
    rc = b2f_gemm_fp8_head_prep(&g.g, &hp, s);
    if (rc == B2F_OK) v_done = true;
    else if (rc != B2F_ERR_UNSUPPORTED) return rc;
  }
  if (!v_done) {
    Gemm g(t, ncat, hid, b.n1, a->qgkv_w, b.proj, B2F_DTYPE_E4M3);
    g.g.col_scale = a->qgkv_col_scale; g.g.out_scale = qs;
    if ((rc = b2f_gemm_fp8(&g.g, s))) return rc;
  }
  {
    // q / k head norm + RoPE (and the V conversion unless the GEMM wrote V): one launch
    // when the shapes allow it (head_dim 128, four-head groups), else one per operation.
    b2f_rope_args r[2];
    for (int which = 0; which < 2; ++which) {
      std::memset(&r[which], 0, sizeof(r[which]));
      r[which].rows = t; r[which].heads = which == 0 ? h : hk; r[which].head_dim = dh;
      r[which].in = b.proj + (which == 0 ? q_off : k_off); r[which].in_ld = ncat;
      r[which].in_head_stride = which == 0 ? q_hstride : dh; r[which].in_scale = qs;
      r[which].weight = which == 0 ? a->q_norm_w : a->k_norm_w;
      r[which].weight_offset = 1.0f; r[which].eps = a->eps;
      r[which].cos = a->rope_cos; r[which].sin = a->rope_sin;
      r[which].rotary_dim = a->rotary_dim; r[which].seq = a->seq;
      r[which].out = which == 0 ? b.q : b.k; r[which].out_ld = (which == 0 ? h : hk) * dh;
      r[which].out_scale = qs;
    }
    rc = v_done ? b2f_attn_prep(&r[0], &r[1], nullptr, 0, nullptr, 0, 0, vdt, s)
                : b2f_attn_prep(&r[0], &r[1], b.proj + v_off, ncat, b.v, (long long)hk * dh,
                                hk * dh, vdt, s);
    if (rc == B2F_ERR_UNSUPPORTED) {
      for (int which = 0; which < 2; ++which)
        if ((rc = b2f_head_norm_rope(&r[which], s))) return rc;
      if (!v_done && (rc = v_convert(b.proj + v_off, ncat, b.v, t, hk * dh, vdt, s))) return rc;
    } else if (rc) {
      return rc;
    }
  }
  {
    b2f_attn_args at;
    b2f_attn_args_init(&at);
    at.batch = a->batch; at.seq = a->seq; at.hq = h; at.hkv = hk; at.head_dim = dh;
    at.causal = 1;
    at.q = b.q; at.q_ld = (long long)h * dh; at.q_scale = qs;
    at.k = b.k; at.k_ld = (long long)hk * dh; at.k_scale = qs;
    at.v = b.v; at.v_ld = (long long)hk * dh; at.v_scale = qs; at.v_dtype = vdt;
    at.gate = b.proj + g_off; at.gate_dtype = B2F_DTYPE_E4M3; at.gate_ld = ncat;
    at.gate_head_stride = q_hstride; at.gate_scale = qs;
    at.ctx = b.ctx; at.ctx_ld = (long long)h * dh; at.ctx_scale = cs;
    if ((rc = b2f_attention_fp8(&at, s))) return rc;
  }
  void* r1 = mlp ? static_cast<void*>(b.r1) : a->out;
  const int r1_dt = mlp ? a->residual_dtype : a->out_dtype;
  {
    Gemm g(t, hid, h * dh, b.ctx, a->o_w, r1, r1_dt);
    if (!mlp) g.g.out_ld = a->out_ld;
    g.g.alpha = alpha_of(cs, a->o_s);
    if (a->add_residual) {
      g.g.residual = a->hidden_in; g.g.residual_dtype = a->hidden_dtype;
      g.g.residual_ld = a->hidden_ld; g.g.residual_scale = a->hidden_scale;
    }
    if ((rc = b2f_gemm_fp8(&g.g, s))) return rc;
  }
  if (!mlp) return B2F_OK;
  {
    b2f_norm_args n;
    b2f_norm_args_init(&n);
    n.rows = t; n.cols = hid;
    n.x = b.r1; n.x_dtype = a->residual_dtype; n.x_ld = hid;
    n.weight = a->post_norm_w; n.weight_dtype = B2F_DTYPE_F32; n.weight_offset = 1.0f;
    n.kind = B2F_NORM_RMS; n.eps = a->eps;
    n.q_out = b.n2; n.q_ld = hid; n.q_scale = ns;
    if ((rc = b2f_norm_quant(&n, s))) return rc;
  }
  {
    Gemm g(t, 2 * a->inter, hid, b.n2, a->mlp_gu_w, b.gu, B2F_DTYPE_E4M3);
    g.g.col_scale = a->mlp_gu_col_scale; g.g.out_scale = a->mlp_proj_scale;
    if ((rc = b2f_gemm_fp8(&g.g, s))) return rc;
  }
  if ((rc = b2f_swiglu_fp8(b.gu, 2LL * a->inter, b.gu + a->inter, 2LL * a->inter, b.act,
                           a->inter, t, a->inter, a->mlp_proj_scale, a->mlp_act_scale, s)))
    return rc;
  {
    Gemm g(t, hid, a->inter, b.act, a->mlp_down_w, a->out, a->out_dtype);
    g.g.out_ld = a->out_ld;
    g.g.alpha = alpha_of(a->mlp_act_scale, a->mlp_down_s);
    g.g.residual = b.r1; g.g.residual_dtype = a->residual_dtype; g.g.residual_ld = hid;
    if ((rc = b2f_gemm_fp8(&g.g, s))) return rc;
  }
  return B2F_OK;
}

}  // extern "C"
