/*
 * b200fp8 — C ABI of the B200-native FP8 kernel library (libb200fp8.so).
 *
 * The reference (bulatsharif/airi-summer-kernel-evo) exposes its kernels as CuTe-DSL
 * `@cute.jit` entry points that an evaluator compiles and calls with evaluator-owned
 * tensors.  Each entry point below replaces one of those interfaces; the comment above
 * every function names the reference interface (file:line, relative to the reference
 * repository root).
 *
 * Conventions
 *  - Every pointer is a device pointer owned by the caller (the reference's evaluator
 *    owns every buffer the same way, tasks/model_gpt2_small_transformer_block_fp8/TASK.md:46-49).
 *  - FP8 tensors are raw float8_e4m3fn bytes; a stored byte q means the value q * scale.
 *  - Row-major storage with an explicit leading dimension (elements) per matrix.
 *  - `stream` is a cudaStream_t passed as void*.  Calls are asynchronous on it.
 *  - Return value: B2F_OK or a B2F_ERR_* code; b2f_last_error() gives a message for the
 *    calling thread.  No C++ exception crosses this ABI.
 *  - Kernels never trap.  Every internal wait is bounded; an expired wait sets the device
 *    status word, which b2f_status_read() returns (B2F_DEV_* codes).
 */
#ifndef B200FP8_H_
#define B200FP8_H_

#ifdef __cplusplus
extern "C" {
#endif

#define B2F_ABI_VERSION 1

typedef void* b2f_stream_t;

enum b2f_status {
  B2F_OK = 0,
  B2F_ERR_ARG = 1,
  B2F_ERR_UNSUPPORTED = 2,
  B2F_ERR_CUDA = 3,
  B2F_ERR_TIMEOUT = 4,
  B2F_ERR_NCCL = 5
};

enum b2f_dtype { B2F_DTYPE_F32 = 0, B2F_DTYPE_BF16 = 1, B2F_DTYPE_E4M3 = 2, B2F_DTYPE_F16 = 3 };

enum b2f_act {
  B2F_ACT_NONE = 0,
  B2F_ACT_RELU = 1,
  B2F_ACT_GELU_TANH = 2,
  B2F_ACT_LEAKY_RELU = 3,
  B2F_ACT_SILU = 4
};

enum b2f_gemm_mode { B2F_GEMM_STORE = 0, B2F_GEMM_ROWSUM = 1 };

/* Device status word codes (b2f_status_read). */
enum b2f_dev_status {
  B2F_DEV_OK = 0,
  B2F_DEV_TIMEOUT_PRODUCER = 1,
  B2F_DEV_TIMEOUT_MMA = 2,
  B2F_DEV_TIMEOUT_EPILOGUE = 3,
  B2F_DEV_TIMEOUT_DRAIN = 4,
  B2F_DEV_BAD_ARGS = 5
};

/* Library ABI version (B2F_ABI_VERSION of the build). */
int b2f_version(void);

/* Message describing the last error returned to the calling thread ("" if none). */
const char* b2f_last_error(void);

/* Number of SMs on the current device (cached per device), or -1. */
int b2f_num_sms(void);

/* Read (and with reset != 0, clear) the device status word of the current device. */
int b2f_status_read(int reset);

/* Test hook: launch one kernel that waits on an mbarrier nothing arrives on, with a
 * bounded wait of `wait_ns`; it must record B2F_DEV_TIMEOUT_EPILOGUE and return. */
int b2f_debug_bounded_wait(unsigned long long wait_ns, b2f_stream_t stream);

/* ------------------------------------------------------------------ GEMM
 * out = epilogue(alpha * (A . B^T))
 *   A: e4m3 [m, lda], K-major; B: e4m3 [n, ldb], K-major (the reference's `matrix_b_nk`).
 *   v = (alpha * acc [* *alpha_ptr] [* col_scale[col]] + bias[col]) * pre_mul + pre_add
 *   v = act(v) * post_mul
 *   v += residual[row, col] * residual_scale           (optional)
 *   STORE : out[row, col] = v / out_scale  in out_dtype (e4m3 uses RN + saturation)
 *   ROWSUM: out[row] += sum_col(v) / out_scale  (out is f32 [m], zeroed by the caller)
 *   amax (optional): *amax = max(*amax, |v|) over the written elements.
 * Replaces: square_gemm (tasks/level1_01_square_matrix_multiplication_fp8/starter.py:29-37,
 *   reference math :125-138), gemm_add_relu (tasks/level2_76_gemm_add_relu_fp8/starter.py,
 *   reference math :148-169) and the epilogue family tasks/level2_{09,12,14,40,63}_* /
 *   starter.py:116-126, the QKV projection tasks/model_gpt2_small_qkv_projection_fp8/
 *   starter.py:151-158 and every `_cute_harness_scaled_linear` of the block tasks.
 * Requirements: lda, ldb multiples of 16; k multiple of 16; 16-byte aligned A, B.
 */
typedef struct b2f_gemm_args {
  int m, n, k;
  const void* a;
  long long lda;
  const void* b;
  long long ldb;
  float alpha;
  const float* alpha_ptr;
  const float* col_scale; /* optional f32 [n]: per-column scale (fused multi-weight GEMMs) */
  const float* bias;
  float pre_mul, pre_add;
  int act;
  float act_param;
  float post_mul;
  const void* residual;
  int residual_dtype;
  long long residual_ld;
  float residual_scale;
  void* out;
  int out_dtype;
  long long out_ld;
  float out_scale;
  float* amax;
  int mode;
  int tile_n; /* 0 = automatic; 64, 128 or 256 (one CTA, 128-row tiles); -128 or -256 (CTA pair,
                256-row tiles of 128 or 256 columns; 512 = -256) */
  /* Split-K (few output tiles, long K): `splits` K slices per tile, at most 8 (0 =
   * automatic: two slices when a large-enough workspace is given, the 128 x 128 tiles fill
   * at most half of the SMs and K >= 4096; otherwise none).  The workspace holds a fixed
   * 16 KB region of per-tile arrival counters, then one f32 partial tile per slice; zero-fill
   * the buffer once before its first use.  Each call tags the counters it uses with its own
   * epoch and leaves them zero, and a counter with another call's tag (left by a call that
   * timed out) reads as zero, so one workspace serves calls of any shape (at most 4096
   * tiles).  Slices are summed in a fixed order, so results are bitwise reproducible.
   * Size: b2f_gemm_workspace_bytes(m, n). */
  int splits;
  void* workspace;
  long long workspace_bytes;
  /* Optional elementwise gate, f32 or bf16 [m, gate_ld] (null = none): after post_mul the
   * value is multiplied by gate[row, col], then the residual is added, i.e.
   *   out = (A.B^T * alpha) * gate + residual
   * Replaces the epilogue of gemm_gated_residual (cute_kernels/fused_gemm_gated_residual_fp8/
   * submission.py:234-256, reference check :383-394). */
  const void* gate;
  int gate_dtype;
  long long gate_ld;
} b2f_gemm_args;

/* Fill `args` with neutral defaults (alpha 1, pre_mul 1, post_mul 1, out_scale 1, bf16 out). */
void b2f_gemm_args_init(b2f_gemm_args* args);

int b2f_gemm_fp8(const b2f_gemm_args* args, b2f_stream_t stream);

/* Attention-operand preparation fused into a q / gate / k / v projection GEMM.
 * The GEMM is `args` (e4m3 output; alpha, column scale and bias only: no activation /
 * residual / gate / amax / split-K; 256-column tiles, on CTA pairs where b2f_gemm_fp8 would
 * use them, else on single CTAs).  Of its output columns:
 *   q head h   = [q_off + h * q_head_stride, + 128): RMSNorm over the head (q_norm_w +
 *                weight_offset; skipped when null), RoPE (rope_cos / rope_sin [seq][128],
 *                rotate_half over the whole head, position = row % seq; skipped when null),
 *                stored as e4m3 codes y / out_scale in q_out[row, 128 h ..] (q_ld bytes);
 *   k head h   = [k_off + 128 h, + 128): the same with k_norm_w into k_out;
 *   v head h   = [v_off + 128 h, + 128): the e4m3 codes as f16 / bf16 (v_dtype) into v_out;
 *   the rest   (the attention gate) is stored as the plain GEMM would store it, in args->out.
 * The q / k / v values are first rounded to e4m3 at args->out_scale, exactly the codes the
 * plain GEMM would store, so the result equals b2f_gemm_fp8 followed by b2f_attn_prep up
 * to the f32 rounding of the norm (at most one e4m3 step).  Offsets and head strides are
 * multiples of 256 / 128 such that every head is one 128-column half of a 256-column tile;
 * head_dim 128 only.  Replaces the reference block's q/gate/k/v projection followed by its
 * q/k RMSNorm + RoPE (tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:339-366). */
typedef struct b2f_head_prep_args {
  int q_off, q_head_stride, q_heads;
  int k_off, k_heads;
  int v_off, v_heads;
  void* q_out;
  long long q_ld;
  void* k_out;
  long long k_ld;
  void* v_out;
  long long v_ld; /* elements */
  int v_dtype;    /* B2F_DTYPE_F16 or B2F_DTYPE_BF16 */
  const float* q_norm_w;
  const float* k_norm_w;
  float weight_offset, eps;
  const float* rope_cos;
  const float* rope_sin;
  int seq;
  float out_scale; /* q / k codes = e4m3(y / out_scale) */
} b2f_head_prep_args;

int b2f_gemm_fp8_head_prep(const b2f_gemm_args* args, const b2f_head_prep_args* hp,
                           b2f_stream_t stream);

/* Split-K GEMM that allocates nothing (no counterpart in the reference).
 * For callers that cannot allocate device memory at call time - a library loaded as a
 * plugin into a host framework that owns every device allocation through its own
 * allocator, or a serving loop whose memory plan is fixed at start-up - and so cannot pass
 * b2f_gemm_fp8 a split-K workspace.  Same arguments and results as b2f_gemm_fp8 with
 * split-K (`workspace` / `workspace_bytes` are ignored; `splits` 0 selects 2, else 2..8;
 * `tile_n` 0 / 128 / 256).  The scratch is a file-scope device array of 8 MiB + 16 KiB
 * that every GPU which loads the library holds until the process exits; a call whose
 * splits * ceil(m/128)*128 * ceil(n/256)*256 * 4 bytes exceed 8 MiB is rejected with
 * B2F_ERR_ARG.  The first call on a device looks up the array's device address (make it
 * before any stream capture).  Every call shares the array: calls that overlap on the GPU
 * race, and must be serialised by the caller. */
int b2f_gemm_fp8_static(const b2f_gemm_args* args, b2f_stream_t stream);

/* Bytes of split-K workspace that b2f_gemm_fp8 needs for an m x n output. */
long long b2f_gemm_workspace_bytes(int m, int n);

/* Co-resident CTA pairs the last CTA-pair GEMM launch on this thread used (0 = none yet). */
int b2f_gemm_pair_capacity(void);

/* ------------------------------------------------------------------ norm + quantise
 * h = x * x_scale + residual          (x: bf16 / f32 / e4m3; residual optional, bf16 / f32)
 * RMS  : y = h * rsqrt(mean(h^2) + eps) * (weight + weight_offset)
 * LAYER: y = (h - mean) * rsqrt(var(h) + eps) * weight + bias
 * q = e4m3(y / s): s = q_scale (static) or, with dynamic_scale, s = amax(|bf16(y)|) / 448
 *     written to *scale_out (the kernel also leaves amax(|y|) in *amax).
 * Optional outputs: h_out (the updated residual stream; when bf16 the norm uses the
 * bf16-rounded h), y_out (bf16 normalised rows).
 * Replaces: residual_rmsnorm (cute_kernels/fused_residual_rmsnorm_fp8/submission.py:57-106,
 *   formula :139-145), the Qwen rms_norm step (tasks/model_qwen35_4b_full_attention_block_fp8/
 *   starter.py:167-171, used at :347-348 and :402-403), the GPT-2 LayerNorm steps
 *   (tasks/model_gpt2_small_transformer_block_fp8/starter.py:407-416, 461-470); long rows
 *   such as layer_norm's (tasks/level1_40_layer_norm_fp8) go to b2f_layer_norm_rows.
 * dynamic_scale selects the scale:
 *   B2F_SCALE_STATIC        s = q_scale, one pass;
 *   B2F_SCALE_DYNAMIC       both passes below on this device;
 *   B2F_SCALE_DYNAMIC_STATS pass 1 only: writes h_out, leaves amax(|bf16(y)|) of these rows
 *                           in *amax (zeroed first), stores no q;
 *   B2F_SCALE_DYNAMIC_APPLY pass 2 only: reads *amax (e.g. after a MAX all-reduce of every
 *                           row shard's amax), writes *scale_out and q (and y_out).
 * The STATS / APPLY split lets row shards on several GPUs share one per-tensor scale.
 * schedule: B2F_NORM_SCHEDULE_AUTO streams rows through shared memory with bulk copies
 * (persistent CTAs) whenever every row is a 16-byte multiple, else falls back to
 * B2F_NORM_SCHEDULE_ROWGROUP (one row per thread group, no staging); both give identical bits.
 * Requirements: cols % 8 == 0, cols <= 8192, 16-byte aligned rows.
 */
enum b2f_norm_kind { B2F_NORM_RMS = 0, B2F_NORM_LAYER = 1 };
enum b2f_scale_mode {
  B2F_SCALE_STATIC = 0,
  B2F_SCALE_DYNAMIC = 1,
  B2F_SCALE_DYNAMIC_STATS = 2,
  B2F_SCALE_DYNAMIC_APPLY = 3
};
enum b2f_norm_schedule { B2F_NORM_SCHEDULE_AUTO = 0, B2F_NORM_SCHEDULE_ROWGROUP = 1 };

typedef struct b2f_norm_args {
  int rows, cols;
  const void* x;
  int x_dtype;
  float x_scale;
  long long x_ld;
  const void* residual;
  int residual_dtype;
  long long residual_ld;
  const void* weight;
  const void* bias;
  int weight_dtype;
  float weight_offset;
  int kind;
  float eps;
  void* h_out;
  int h_dtype;
  long long h_ld;
  void* y_out;
  long long y_ld;
  void* q_out;
  long long q_ld;
  float q_scale;
  int dynamic_scale; /* b2f_scale_mode */
  float* amax;
  float* scale_out;
  int schedule; /* b2f_norm_schedule */
  float* row_stats; /* optional f32 [rows][2] scratch (8-byte aligned): with a dynamic scale,
                       pass 1 leaves each row's (mean, rstd) there and pass 2 reads them
                       instead of recomputing (same bits); null: pass 2 recomputes */
} b2f_norm_args;

void b2f_norm_args_init(b2f_norm_args* args);
int b2f_norm_quant(const b2f_norm_args* args, b2f_stream_t stream);

/* Which kernels b2f_norm_quant would run for these arguments (first pass it runs):
 * 0 = streaming schedule (shared-memory ring of rows), 1 = row-group kernels, 2 = one warp per
 * row (short bf16 rows, static scale, no residual), or -code when the arguments are
 * invalid.  Launches nothing; needs the current device. */
int b2f_norm_plan(const b2f_norm_args* args);

/* ------------------------------------------------------------------ long-row LayerNorm
 * y[r, :] = (x[r, :] * x_scale - mean_r) * rsqrt(var_r + eps) [* weight + bias]
 *   over rows of up to millions of columns: every row is cut into 65536-element chunks, one
 *   CTA each (pass 1: chunk sums; pass 2: the row's sums combined in f64, then the chunk
 *   normalised), so a handful of rows still streams through all SMs.
 *   x: e4m3, bf16 or f32 [rows, x_ld]; out: f32 or bf16 [rows, out_ld]; weight / bias
 *   optional f32 [cols]; workspace: b2f_layer_norm_rows_workspace_bytes(rows, cols) bytes,
 *   8-byte aligned (per-chunk f64 sums; no zeroing needed).
 * Replaces: layer_norm of tasks/level1_40_layer_norm_fp8 (evaluator starter.py:84-166,
 *   [16 x 4,194,304] e4m3 at 1/448, eps 1e-5, f32 out; CuTe submission
 *   cute_kernels/level1_40_layer_norm_fp8/submission.py:71-134, one CTA per row).
 */
typedef struct b2f_lnrows_args {
  int rows;
  long long cols;
  const void* x;
  int x_dtype;
  long long x_ld;
  float x_scale;
  const float* weight;
  const float* bias;
  float eps;
  void* out;
  int out_dtype;
  long long out_ld;
  void* workspace;
  long long workspace_bytes;
} b2f_lnrows_args;

void b2f_lnrows_args_init(b2f_lnrows_args* args);
long long b2f_layer_norm_rows_workspace_bytes(int rows, long long cols);
int b2f_layer_norm_rows(const b2f_lnrows_args* args, b2f_stream_t stream);

/* ------------------------------------------------------------------ attention
 * ctx[t, h*D:(h+1)*D] = e4m3( softmax(q_h k_g^T * sm_scale [causal]) v_g * sigmoid(gate) / ctx_scale )
 *   tokens t = b * seq + s (attention stays inside each sequence); g = h / (hq / hkv) (GQA)
 *   q: e4m3 [T, q_ld], head h at column h*D, value = stored * q_scale
 *   k: e4m3 [T, k_ld], head g at column g*D, value = stored * k_scale
 *   v: bf16 or f16 (v_dtype) [T, v_ld], head g at column g*D, value = stored * v_scale;
 *      with f16 V the probabilities P are f16 too (exponentials taken in pairs), with bf16 V
 *      they are bf16
 *   gate (optional): e4m3 or bf16 [T, gate_ld], head h at column h*gate_head_stride,
 *         value = stored * gate_scale
 *   sm_scale <= 0 selects 1/sqrt(D).
 * Replaces: the attention step of gpt2_transformer_block (reference math
 *   tasks/model_gpt2_small_transformer_block_fp8/starter.py:428-453), attention_kernel of
 *   qwen35_full_attention_block (tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:
 *   40-49, reference math :354-392) and the vision block's non-causal attention
 *   (tasks/model_qwen35_4b_vision_block_fp8/starter.py:327-345).
 * Requirements: head_dim 64, 128 or 256; 16-byte aligned rows.
 */
typedef struct b2f_attn_args {
  int batch, seq, hq, hkv, head_dim;
  int causal;
  const void* q;
  long long q_ld;
  float q_scale;
  const void* k;
  long long k_ld;
  float k_scale;
  const void* v;
  long long v_ld;
  float v_scale;
  float sm_scale;
  const void* gate;
  int gate_dtype;
  long long gate_ld;
  long long gate_head_stride;
  float gate_scale;
  void* ctx;
  long long ctx_ld;
  float ctx_scale;
  int v_dtype; /* B2F_DTYPE_BF16 (default) or B2F_DTYPE_F16 (head_dim 64 / 128) */
} b2f_attn_args;

void b2f_attn_args_init(b2f_attn_args* args);
int b2f_attention_fp8(const b2f_attn_args* args, b2f_stream_t stream);

/* ------------------------------------------------------------------ attention operand prep
 * Per (token, head): x = in * in_scale; optional RMSNorm x * rsqrt(mean(x^2)+eps) *
 * (weight + weight_offset); optional rotate-half RoPE on the first rotary_dim dims with
 * cos/sin [seq, rotary_dim] at position token % seq; out = e4m3(y / out_scale) into
 * [rows, out_ld] with head h at column h*D.
 * Replaces: q_headnorm / k_headnorm (kernel_evo_archive/best_kernels/qwen-no-prof/
 *   submission.py:368-449; reference math tasks/model_qwen35_4b_full_attention_block_fp8/
 *   starter.py:167-183 and :365-376).
 */
typedef struct b2f_rope_args {
  int rows, heads, head_dim;
  const void* in;
  long long in_ld;
  long long in_head_stride;
  float in_scale;
  const float* weight;
  float weight_offset;
  float eps;
  const float* cos;
  const float* sin;
  int rotary_dim;
  int seq;
  void* out;
  long long out_ld;
  float out_scale;
} b2f_rope_args;

int b2f_head_norm_rope(const b2f_rope_args* args, b2f_stream_t stream);

/* The three operand preparations of a gated GQA attention in one launch: q and k as
 * b2f_head_norm_rope (head_dim 128, heads a multiple of 4, full or no RoPE, 16-byte aligned
 * rows; the same token count) and V [q->rows, v_cols] e4m3 -> f16 or bf16 (v_dtype,
 * exact; v_in = v_out = null and v_cols = 0 skip it, for a V image already written by
 * b2f_gemm_fp8_head_prep).  B2F_ERR_UNSUPPORTED for other shapes (call the operations
 * separately).
 * Replaces: the q / k normalisation, RoPE and V requantisation steps of
 *   qwen35_full_attention_block (tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:
 *   365-376), fused into one launch. */
int b2f_attn_prep(const b2f_rope_args* q, const b2f_rope_args* k, const void* v_in,
                  long long v_in_ld, void* v_out, long long v_out_ld, int v_cols, int v_dtype,
                  b2f_stream_t stream);

/* out (bf16) = in (e4m3 bytes) * scale, [rows, cols] with row pitches in elements.
 * Produces the bf16 V operand of b2f_attention_fp8 (exact: bf16 holds every e4m3 value). */
int b2f_fp8_to_bf16(const void* in, long long in_ld, void* out, long long out_ld, int rows,
                    int cols, float scale, b2f_stream_t stream);

/* out (f16) = in (e4m3 bytes) * scale; the f16 V operand (exact: f16 holds every e4m3 value). */
int b2f_fp8_to_f16(const void* in, long long in_ld, void* out, long long out_ld, int rows,
                   int cols, float scale, b2f_stream_t stream);

/* ------------------------------------------------------------------ quantise
 * q = e4m3(x / s), x f32 or bf16 [rows, cols] (row pitch x_ld elements, 16-byte aligned
 * rows), q e4m3 bytes (row pitch q_ld, 8-byte aligned rows); IEEE division, RN, saturating.
 * dynamic != 0: s = amax(|x|) / 448 (1 for an all-zero x), reduced into *amax and written to
 * *scale_out; else s = scale.  With scale_mul, *scale_prod_out = s * *scale_mul (the GEMM
 * alpha of two dynamically scaled operands, for b2f_gemm_args.alpha_ptr).
 * Replaces: the per-tensor FP8 quantisation the reference applies to its operands
 *   (`(source / scale).to(torch.float8_e4m3fn)`, e.g.
 *   tasks/level1_01_square_matrix_multiplication_fp8/starter.py:61-99). */
typedef struct b2f_quant_args {
  int rows, cols;
  const void* x;
  int x_dtype;
  long long x_ld;
  void* q;
  long long q_ld;
  int dynamic;
  float scale;
  float* amax;
  float* scale_out;
  const float* scale_mul;
  float* scale_prod_out;
} b2f_quant_args;

void b2f_quant_args_init(b2f_quant_args* args);
int b2f_quantize_fp8(const b2f_quant_args* args, b2f_stream_t stream);

/* out = e4m3( silu(gate * in_scale) * (up * in_scale) / out_scale ); gate, up, out e4m3
 * [rows, cols] with row pitches in elements.
 * Replaces: swiglu_kernel (tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:51-58;
 *   reference math :404-412). */
int b2f_swiglu_fp8(const void* gate, long long gate_ld, const void* up, long long up_ld,
                   void* out, long long out_ld, int rows, int cols, float in_scale,
                   float out_scale, b2f_stream_t stream);

/* ------------------------------------------------------------------ op registry */
typedef struct b2f_op {
  const char* name;      /* e.g. "gemm_fp8" */
  int abi_version;
  void* fn;              /* pointer to the b2f_* entry point */
  const char* signature; /* human-readable argument struct name */
} b2f_op;

/* Look up an op by name; NULL if unknown. */
const b2f_op* b2f_registry_lookup(const char* name);
/* Number of registered ops and indexed access (for enumeration). */
int b2f_registry_size(void);
const b2f_op* b2f_registry_at(int index);


/* ------------------------------------------------------------------ decoder blocks
 * Whole-block entry points: the kernels above in each reference evaluator's dataflow order
 * on one stream; intermediates live in a caller workspace of
 * b2f_*_block_workspace_bytes(args) bytes (256-byte aligned).  Tokens t = b * seq + s.
 * Weights are e4m3 [out, in] with per-tensor scales; biases / norm weights f32.
 *
 * GPT-2 block (also the Qwen vision block with rope_cos / rope_sin and causal = 0):
 *   n1 = e4m3(LN1(hidden) / norm_scale); qkv = e4m3((n1 . Wqkv^T + b) / qkv_scale);
 *   [q, k: RoPE -> e4m3]; ctx = e4m3(attention / ctx_scale);
 *   r1 = hidden + ctx . Wout^T + b  (residual_dtype); n2 = e4m3(LN2(r1) / norm_scale);
 *   h = e4m3(gelu_tanh(n2 . Wfc^T + b) / mlp_scale); out = r1 + h . Wproj^T + b.
 * Replaces: gpt2_transformer_block (tasks/model_gpt2_small_transformer_block_fp8/starter.py:
 *   114-140, reference math :393-488) and the vision block
 *   (tasks/model_qwen35_4b_vision_block_fp8/starter.py:303-369). */
typedef struct b2f_gpt2_block_args {
  int batch, seq, d_model, heads, mlp;
  const void* hidden;
  int hidden_dtype; /* f32, bf16 or e4m3 */
  long long hidden_ld;
  float hidden_scale;
  const void* qkv_w;
  float qkv_s;
  const float* qkv_b;
  const void* out_w;
  float out_s;
  const float* out_b;
  const void* fc_w;
  float fc_s;
  const float* fc_b;
  const void* proj_w;
  float proj_s;
  const float* proj_b;
  const float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
  float eps;
  float norm_scale, qkv_scale, ctx_scale, mlp_scale;
  int causal;
  const float* rope_cos; /* optional f32 [seq, head_dim] */
  const float* rope_sin;
  int residual_dtype; /* r1: f32 or bf16 */
  void* out;
  int out_dtype; /* f32 or bf16 */
  long long out_ld;
  void* workspace;
  long long workspace_bytes;
} b2f_gpt2_block_args;

void b2f_gpt2_block_args_init(b2f_gpt2_block_args* args);
long long b2f_gpt2_block_workspace_bytes(const b2f_gpt2_block_args* args);
int b2f_gpt2_block(const b2f_gpt2_block_args* args, b2f_stream_t stream);

/* Qwen gated full-attention block (optional SwiGLU MLP):
 *   n1 = e4m3(RMSNorm_(1+w)(hidden) / norm_scale);
 *   proj = e4m3(n1 . Wqgkv^T * qgkv_col_scale[col] / qkv_scale)   (one GEMM over the packed
 *     weights; qgkv_col_scale[j] = norm_scale * scale of the weight that row j belongs to);
 *   q, k: per-head RMSNorm (1+w) + rotate-half RoPE on rotary_dim dims -> e4m3;
 *   ctx = e4m3(causal GQA attention * sigmoid(gate) / ctx_scale);
 *   r1 = [hidden] + ctx . Wo^T * (ctx_scale * o_s)   (add_residual = 0 leaves the residual
 *     out: the partial of a heads-parallel o-projection);
 *   MLP: n2 = e4m3(RMSNorm_(1+w)(r1)); gu = e4m3(n2 . [Wgate|Wup]^T * mlp_gu_col_scale /
 *     mlp_proj_scale); act = e4m3(silu(gate) * up / mlp_act_scale); out = r1 + act . Wdown^T.
 * Packed row order: interleaved = 1: [q_h | gate_h] per head, then k, then v (the reference's
 *   q_gate weight); interleaved = 0: [q | gate | k | v].
 * Replaces: qwen35_full_attention_block (tasks/model_qwen35_4b_full_attention_block_fp8/
 *   starter.py:66-98, reference math :333-416). */
typedef struct b2f_qwen_block_args {
  int batch, seq, hidden, heads, kv_heads, head_dim, rotary_dim;
  int interleaved;
  const void* hidden_in;
  int hidden_dtype; /* f32, bf16 or e4m3 */
  long long hidden_ld;
  float hidden_scale;
  const void* qgkv_w;
  const float* qgkv_col_scale;
  const void* o_w;
  float o_s;
  const float *in_norm_w, *q_norm_w, *k_norm_w;
  const float* rope_cos; /* f32 [seq, rotary_dim] */
  const float* rope_sin;
  float eps, norm_scale, qkv_scale, ctx_scale;
  int add_residual;
  const float* post_norm_w; /* MLP (mlp_gu_w null: attention block only) */
  const void* mlp_gu_w;     /* [2 * inter, hidden]: gate rows then up rows */
  const float* mlp_gu_col_scale;
  int inter;
  const void* mlp_down_w;
  float mlp_down_s;
  float mlp_proj_scale, mlp_act_scale;
  int residual_dtype;
  void* out;
  int out_dtype;
  long long out_ld;
  void* workspace;
  long long workspace_bytes;
} b2f_qwen_block_args;

void b2f_qwen_block_args_init(b2f_qwen_block_args* args);
long long b2f_qwen_block_workspace_bytes(const b2f_qwen_block_args* args);
int b2f_qwen_block(const b2f_qwen_block_args* args, b2f_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* B200FP8_H_ */
