/*
 * libsvx: B200 (sm_100a) kernels for StreamVoxel's per-step column-generation hot path, behind a plain C ABI.
 *
 * Conventions
 *   - Every entry point returns an svx_status (0 = SVX_OK). svx_last_error() describes the last failure on the
 *     calling host thread. No C++ exception crosses this boundary.
 *   - All buffers are caller-owned device pointers (the caller is normally PyTorch); sizes are element counts.
 *     The library allocates no device memory; it keeps TMA descriptors in host memory.
 *   - Work is enqueued on the given cudaStream_t (passed as void*); nothing synchronises the host, so every call
 *     is capturable in a CUDA graph (after one warm-up call that configures each kernel's shared memory).
 *   - Per-device settings (each kernel's shared-memory opt-in, occupancy, the no-allocation scratch address) are
 *     made on the first call with that device current and kept for the life of the process: cudaDeviceReset, or
 *     releasing and re-creating a device's primary context, is not supported while the library is loaded.
 *   - Logit layout is the reference's: class-major [slot][V][Y][Z][X] (`streamvoxel/stream/fast_ops.py:307`).
 *   - Tokens are int16 [slot][Y][Z][X]; the mask token id equals V (`streamvoxel/stream/condition.py:25`).
 *
 * The reference (zzf1955/StreamVoxel) is Python + PyTorch; each entry point names the Python function whose
 * work it replaces (path:line in the reference).
 */
#ifndef SVX_H
#define SVX_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SVX_API __attribute__((visibility("default")))
#else
#define SVX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SVX_OK = 0,
  SVX_ERR_INVALID = 1,      /* bad shape / size / alignment / capacity: ValueError in the Python mirror */
  SVX_ERR_CUDA = 2,         /* a CUDA runtime or driver call failed: RuntimeError */
  SVX_ERR_UNSUPPORTED = 3,  /* not built for this device (needs sm_100a): RuntimeError */
} svx_status;

/* Per-slot device status word bits (written by the EASE kernels, read back with the commits). */
#define SVX_STATUS_QUOTA_MISSED   0x1u  /* chosen count != k, or a chosen voxel was not selectable */
#define SVX_STATUS_NAN_LOGITS     0x2u  /* a score or probability was NaN */
#define SVX_STATUS_WAIT_TIMEOUT   0x4u  /* a bounded spin-wait gave up (kernel skipped its work) */

typedef enum { SVX_F32 = 0, SVX_BF16 = 1 } svx_dtype;

SVX_API const char* svx_last_error(void);
SVX_API int svx_version(void);
/* 1 if the current device is sm_100 and the kernels can run on it. */
SVX_API int svx_device_supported(void);
/* Bitwise OR of SVX_STATUS_WAIT_TIMEOUT events recorded by the tensor-core kernels since the library loaded. */
SVX_API uint32_t svx_wait_timeouts(void);

/* ------------------------------------------------------------------------------------------------ EASE sampler */

/* Per-slot scalars of one solid step (host-filled, copied to the device before the step).
 * Replaces the 0-dim device tensors of FastLowEntropyLastSlot.prepare (`streamvoxel/stream/fast_ops.py:519-532`). */
typedef struct {
  int32_t k;          /* quota of this step; 0 = the slot takes no solid step */
  int32_t step;       /* forward index (nfe) of this step, keys the native draw */
  int64_t committed;  /* non-deferred voxels committed before this step */
  double frac;        /* (committed + k) / (total - last_count), float64 as the reference apportions */
  uint64_t seed;      /* slot seed, keys the native draw */
} svx_step_params;

/* Negative entropy per voxel, sum_c p_c log p_c in fp32 (`streamvoxel/sampling/entropy.py:1-4`).
 * logits: [slots][classes][voxels] (dtype), slot stride = logit_slot_stride elements. scores: [slots][voxels] fp32. */
SVX_API int svx_ease_scores(const void* logits, int dtype, int slots, int classes, int voxels,
                            int64_t logit_slot_stride, float* scores, uint32_t* status, void* stream);

/* Marking forward (`streamvoxel/stream/slot.py:124-130` + `streamvoxel/sampling/low_entropy_last.py:8-13`, col=True):
 * air = sum_{a in air_ids} softmax(logits)[a]; bad = air <= float32(1 - last_eps); last = per-(z,x) column top run of
 * not-bad voxels (largest y first). last: [slots][Y][Z][X] uint8 (written), last_count: [slots] int32 (written). */
SVX_API int svx_ease_mark(const void* logits, int dtype, int slots, int classes, int height, int depth, int width,
                          int64_t logit_slot_stride, const int32_t* air_ids, int n_air, double last_eps,
                          uint8_t* last, int32_t* last_count, void* stream);

/* Solid-step selection: `block_quota_select` (`streamvoxel/sampling/block_quota.py:20-38`) in the graph-capturable
 * form of `quota_select_nosync` (`streamvoxel/stream/fast_ops.py:442-473`). Selectable = tokens == mask_id && !last.
 * pos: [slots][blocks] int32 inverse block order. Writes chosen [slots][voxels] uint8, the ascending chosen voxel
 * indexes index_out [slots][index_capacity] int32 (the `nonzero_static` of `fast_ops.py:548`, -1 past the count),
 * chosen_count [slots] and OR-s SVX_STATUS_QUOTA_MISSED into status when the selection does not hold exactly k
 * selectable voxels. workspace: svx_ease_select_workspace_bytes(slots, voxels) bytes of device scratch. */
SVX_API size_t svx_ease_select_workspace_bytes(int slots, int voxels);
SVX_API int svx_ease_select(const float* scores, const int16_t* tokens, const uint8_t* last, const int32_t* pos,
                            const svx_step_params* params, int slots, int height, int depth, int width, int block,
                            int mask_id, uint8_t* chosen, int32_t* index_out, int index_capacity,
                            int32_t* chosen_count, uint32_t* status, void* workspace, void* stream);

/* svx_ease_select for callers that cannot allocate device memory (this entry point has no counterpart in the
 * reference). A host whose device memory belongs entirely to another framework's pool, or that must not allocate
 * while it is running, cannot hand svx_ease_select a workspace; this variant takes none. Its scratch is a fixed
 * array compiled into the library (262,400 bytes, held on every GPU that loads the library until the process exits),
 * so it accepts at most 64 slots and 1024 4^3 blocks per column and returns SVX_ERR_INVALID beyond that. The first call
 * on each device looks the array's device address up (cudaGetSymbolAddress) and keeps it for the life of the process
 * (no device reset, see the conventions above); make that first call before any stream capture. Every call uses the same array: calls whose kernels overlap on the GPU (other streams, other host threads)
 * race and must be serialised by the caller. The kernels overwrite all scratch they read on every call. Outputs,
 * inputs and errors are those of svx_ease_select. */
SVX_API int svx_ease_select_noalloc(const float* scores, const int16_t* tokens, const uint8_t* last, const int32_t* pos,
                                    const svx_step_params* params, int slots, int height, int depth, int width,
                                    int block, int mask_id, uint8_t* chosen, int32_t* index_out, int index_capacity,
                                    int32_t* chosen_count, uint32_t* status, void* stream);

/* ----------------------------------------------------------------------------------------- evaluation decoders */

#define SVX_EVAL_RANDOM    0  /* top_mask(draw, masked, k) */
#define SVX_EVAL_ENTROPY   1  /* top_mask(score, masked, k) */
#define SVX_EVAL_MIXED     2  /* top k by score among the top `candidates` by draw */
#define SVX_EVAL_BLOCK     3  /* linear 4^3 block apportioning of the cumulative count, best scores inside */
#define SVX_EVAL_THRESHOLD 4  /* masked & draw < threshold (native_quarter) */

/* Per-slot scalars of one evaluation-decoder step (host-filled, device array). */
typedef struct {
  int32_t mode;        /* SVX_EVAL_* */
  int32_t k;           /* voxels to reveal (every mode but THRESHOLD): already min(quota, masked count) */
  int32_t candidates;  /* MIXED: min(masked count, ceil(multiplier * k)) */
  int32_t committed;   /* BLOCK: voxels revealed before this step */
  float threshold;     /* THRESHOLD: reveal probability of the step */
  int32_t step;        /* written to commit_step for every chosen voxel (0: commit_step untouched) */
} svx_eval_params;

/* The selections of the evaluation decoders (`streamvoxel/eval/samplers.py:23-64`: random, entropy, mixed, block;
 * the native_quarter threshold of `:98-101`) over the masked voxels (tokens == mask_id) of each slot's column.
 * scores/draw: [slots][Y][Z][X] fp32 (negative entropy; uniform draws); pos: [slots][blocks] rank of each 4^3 block
 * in the seeded order (BLOCK). Writes chosen (uint8), the ascending voxel indices (index_out [slots][capacity],
 * -1 padded), chosen_count [slots], commit_step (optional) and the per-block quota range [slots][2] (BLOCK,
 * optional); the reference's assertions (quota range, count) set SVX_STATUS_QUOTA_MISSED in status. */
SVX_API int svx_eval_select(const float* scores, const float* draw, const int16_t* tokens, const int32_t* pos,
                            const svx_eval_params* params, int slots, int height, int depth, int width, int mask_id,
                            uint8_t* chosen, int32_t* index_out, int index_capacity, int32_t* chosen_count,
                            int32_t* commit_step, int32_t* quota_range, uint32_t* status, void* stream);

/* Categorical draw + token commit for the chosen voxels (`streamvoxel/stream/fast_ops.py:549-551`,
 * `streamvoxel/stream/slot.py:149-151`): p = softmax over classes in fp32, value = argmax(p / q).
 * noise != NULL (parity mode): q = noise[slot][i][classes] fp32, the exponential draws torch.multinomial takes from
 * the slot generator; the softmax reproduces torch's CUDA row softmax reduction order. noise == NULL (native mode,
 * the Gumbel-max form of the same draw): value = argmax x - log(-log u), u = (2 (w >> 9) + 1) 2^-24 from
 * Philox4x32-10 keyed by (params.seed, params.step, voxel, class), both logarithms an atanh series evaluated in
 * single-rounded fp32 operations, so a host restatement reproduces every value bit for bit.
 * Writes tokens[index] = value, values_out [slots][index_capacity] int16. */
SVX_API int svx_ease_sample(const void* logits, int dtype, int slots, int classes, int voxels,
                            int64_t logit_slot_stride, const int32_t* index, const svx_step_params* params,
                            const float* noise, int64_t noise_slot_stride, int index_capacity, int16_t* tokens,
                            int16_t* values_out, uint32_t* status, void* stream);

/* Torch-order row softmax of rows [rows][classes] fp32 (the softmax svx_ease_sample uses in parity mode). */
SVX_API int svx_softmax_rows(const float* x, int rows, int classes, float* out, void* stream);

/* `_finish` (`streamvoxel/stream/slot.py:166-167`): tokens[last] = air_token for each slot with finish[slot] != 0. */
SVX_API int svx_ease_finish(int16_t* tokens, const uint8_t* last, const uint8_t* finish, int slots, int voxels,
                            int air_token, void* stream);

/* ------------------------------------------------------------------------------------------------ forward ops */

/* Patch-4 token embed, both branches in one pass (`streamvoxel/stream/fast_ops.py:58-75` GatherPatch, plus the
 * per-position y-embedding `unconditional_md4_timefree.py:166-168`):
 * out = bf16(bf16(bf16(sum_o T[t_o*64+o]) + bias) + add[p]).
 * tokens [slots][Y][Z][X] int16; table [(classes+1)*64][d] bf16; add [patches][d] bf16; out [slots*patches][d].
 * table_c == NULL skips the control branch. stats_b / stats_c (optional, d % 32 == 0): [d/32][slots*patches]
 * (mean, M2) float pairs of each output row's 32-column chunks, for the LayerNorm fold of the next linear. */
SVX_API int svx_patch_embed(const int16_t* tokens, int slots, int height, int depth, int width, int patch,
                            int classes, int d, const uint16_t* table_b, const uint16_t* bias_b,
                            const uint16_t* add_b, uint16_t* out_b, const uint16_t* table_c, const uint16_t* bias_c,
                            const uint16_t* add_c, uint16_t* out_c, float* stats_b, float* stats_c, void* stream);

/* LayerNorm without affine (fp32) + AdaLN modulate (`unconditional_md4_timefree.py:12-13,53-54`):
 * out = bf16(LN(x) * one_plus_scale + shift); one_plus_scale/shift may be NULL (plain LN). x,out [rows][d] bf16. */
SVX_API int svx_layernorm_modulate(const uint16_t* x, int rows, int d, float eps, const uint16_t* one_plus_scale,
                                   const uint16_t* shift, uint16_t* out, void* stream);

/* The condition encoder's LayerNorms (`streaming_controlnet.py:142-158` `_encode_columns`: `l2_norm` (affine, eps 1e-5)
 * then GELU before the 4^3 down-conv; `:158,167-168,217-218`: + type + size embeddings, then `context_norm` (no
 * affine, eps 1e-6)), in fp32: out = bf16(g(LN(x + pre) * weight + bias)), g = GELU(erf) when gelu != 0. pre [d] fp32
 * (16-byte aligned), weight/bias [d] fp32, each may be NULL (weight and bias together). x,out [rows][d] bf16, 16-byte
 * aligned, out may be x; d % 8 == 0, d <= 1536. Replaces `F.layer_norm` / `F.gelu` of `FastSlotForward.encode` (`fast_ops.py:228-239`). */
SVX_API int svx_layernorm_affine(const uint16_t* x, int rows, int d, float eps, const float* pre,
                                 const float* weight, const float* bias, int gelu, uint16_t* out, void* stream);

/* Epilogues of svx_gemm. out = f(acc + bias) with acc = A[M,K] . W[N,K]^T in fp32, every step rounded to bf16 as
 * eager autocast rounds it (`streamvoxel/models/unconditional_md4_timefree.py:37-63`). */
typedef enum {
  SVX_EPI_BIAS = 0,          /* out = bf16(acc + b) */
  SVX_EPI_BIAS_GELU = 1,     /* out = bf16(gelu_erf(bf16(acc + b))) */
  SVX_EPI_GATE_RESIDUAL = 2, /* out = bf16(res + bf16(gate[n] * bf16(acc + b)))  (AdaLN-gated residual) */
  SVX_EPI_RESIDUAL = 3,      /* out = bf16(res + bf16(acc + b)) */
  SVX_EPI_ROPE = 4,          /* out = bf16(acc + b), then axial RoPE on columns < rope_cols (q|k heads of 96) */
  SVX_EPI_CLASS_MAJOR = 5,   /* out = bf16(acc + b) scattered to class-major [slot][V][Y][Z][X] logits */
} svx_epilogue;

typedef struct {
  int epilogue;
  const uint16_t* bias;      /* [N] bf16 */
  const uint16_t* gate;      /* [N] bf16 (GATE_RESIDUAL) */
  const uint16_t* residual;  /* [M][N] bf16 (GATE_RESIDUAL, RESIDUAL); may equal out */
  const uint16_t* rope_sin;  /* [rows_per_slot][head_dim/2] bf16 (ROPE) */
  const uint16_t* rope_cos;
  int rope_cols;             /* ROPE: columns [0, rope_cols) rotate */
  int rows_per_slot;         /* ROPE / CLASS_MAJOR: patches per slot */
  int head_dim;              /* ROPE: 96 */
  int classes;               /* CLASS_MAJOR: V; W rows are ordered n = v*64 + o */
  int height, depth, width, patch; /* CLASS_MAJOR geometry */
  /* LayerNorm fold (bias, GELU, RoPE, class-major epilogues): A holds the raw rows x and W the modulated weights
   * W'[n][k] = W[n][k] (1 + scale[k]); out = epilogue(r (acc - mu u[n]) + v[n]) with mu, r = 1/sqrt(var + ln_eps)
   * of each A row from ln_stats_in ([K/32][M] (mean, M2) pairs of its 32-column chunks, chunk-major),
   * u[n] = sum_k W'[n][k], v[n] = b[n] + sum_k W[n][k] shift[k] (fp32). Replaces LayerNorm + modulate + linear
   * (`unconditional_md4_timefree.py:12-13,53-63`). */
  const float* ln_stats_in;  /* NULL: out = epilogue(acc + b) */
  const float* ln_u;
  const float* ln_v;
  float ln_eps;
  float* ln_stats_out;       /* optional (residual epilogues) [N/32][M] (mean, M2) of the bf16 output rows' chunks */
} svx_epilogue_args;

/* D = A . W^T with a fused epilogue on the tcgen05 tensor cores (TMA-fed, TMEM accumulator).
 * A [M][K] bf16 row-major, W [N][K] bf16 row-major (nn.Linear weight). M % 128 == 0, N % 64 == 0, K % 64 == 0.
 * Replaces the bf16 nn.Linear calls of the block (`unconditional_md4_timefree.py:37-57`) and the head (`:175`). */
SVX_API int svx_gemm(const uint16_t* A, const uint16_t* W, uint16_t* out, int M, int N, int K,
                     const svx_epilogue_args* epi, void* stream);

/* Two independent gated-residual GEMMs with row statistics (epilogue SVX_EPI_GATE_RESIDUAL, ln_stats_out set, no
 * LayerNorm fold) of the same M, N, K in one launch: out_i = bf16(res_i + bf16(gate_i[n] bf16(A_i W_i^T + b_i))).
 * M % 256 == 0. A gate of ones gives the plain residual of SVX_EPI_RESIDUAL bit for bit. The engine runs a control
 * layer's cross-attention projection (`streaming_controlnet.py:61`) with its backbone block's attention projection
 * (`unconditional_md4_timefree.py:62`) this way: both follow the joint attention launch. */
SVX_API int svx_gemm_group(const uint16_t* A0, const uint16_t* W0, uint16_t* out0, const svx_epilogue_args* epi0,
                           const uint16_t* A1, const uint16_t* W1, uint16_t* out1, const svx_epilogue_args* epi1,
                           int M, int N, int K, void* stream);

/* Non-causal attention, head_dim 96, per (slot, head): out = softmax(Q K^T / sqrt(96)) V over keys < length[slot].
 * Q rows: q + (slot*queries + i)*q_row_stride + head*96; K/V: kv + slot*kv_slot_stride + head*kv_head_stride +
 * key*kv_row_stride. out [slot*queries + i][heads*96]. lengths == NULL: every slot has `keys` keys.
 * Replaces SDPA (`unconditional_md4_timefree.py:46`) and the packed FlexAttention (`fast_ops.py:104-108`). */
SVX_API int svx_attention(const uint16_t* q, int64_t q_row_stride, const uint16_t* k, const uint16_t* v,
                          int64_t kv_slot_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                          const int32_t* lengths, int slots, int heads, int queries, int keys, uint16_t* out,
                          const int32_t* plan, int plan_ctas, void* stream);
/* Work-unit assignment for svx_attention (plan, device copy) on plan_ctas CTAs. A unit is two 128-query tiles of one
 * (slot, head); units go longest first to the least-loaded CTA (cost: key tiles + 2), which balances slots of unequal
 * key lengths. plan = [G + 1 offsets][units natural ids (slot*heads + head)*pairs + pair], G = min(ctas, units).
 * The plan affects only which CTA computes a unit, never the result: a plan built for other lengths stays correct.
 * lengths: host array [slots] or NULL (all `keys`). plan_ints returns the ints a plan takes (0: bad shape).
 * No reference counterpart (FlexAttention schedules its own blocks, `fast_ops.py:104-108`). */
SVX_API int svx_attention_plan_ints(int slots, int heads, int queries, int ctas);
SVX_API int svx_attention_plan(const int32_t* lengths, int slots, int heads, int queries, int keys, int ctas,
                               int32_t* plan, int capacity);

/* One attention problem, in svx_attention's layouts. */
typedef struct {
  const uint16_t *q, *k, *v;
  int64_t q_row_stride, kv_slot_stride, kv_head_stride, kv_row_stride;
  const int32_t* lengths;    /* device [slots] or NULL (all `keys`) */
  int keys;
  uint16_t* out;
} svx_attention_problem;

/* One or two independent attention problems over the same slots, heads and queries in one persistent launch: the
 * engine runs a control layer's cross-attention together with its backbone layer's self-attention, so that the
 * short self-attention units fill the CTAs the long cross-attention units leave idle. Two problems need a plan
 * from svx_attention_multi_plan (unit ids problem-major); each problem's output equals its own svx_attention.
 * lengths: host arrays per problem (entries may be NULL). No reference counterpart (the reference launches SDPA and
 * FlexAttention separately, `timefree.py:46`, `fast_ops.py:104-108`). */
SVX_API int svx_attention_multi(const svx_attention_problem* problems, int count, int slots, int heads, int queries,
                                const int32_t* plan, int plan_ctas, void* stream);
SVX_API int svx_attention_multi_plan_ints(int problems, int slots, int heads, int queries, int ctas);
SVX_API int svx_attention_multi_plan(const int32_t* const* lengths, const int* keys, int problems, int slots,
                                     int heads, int queries, int ctas, int32_t* plan, int capacity);

/* ------------------------------------------------------------------------------------------------ the engine */

/* Per-layer weights of one time-free AdaLN block. AdaLN vectors are the constant-time ada outputs
 * (`unconditional_md4_timefree.py:58,120-121`), precomputed in bf16; one_plus_scale = bf16(1 + scale). */
typedef struct {
  const uint16_t *qkv_w, *qkv_b, *proj_w, *proj_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
  const uint16_t *shift1, *one_plus_scale1, *gate1, *shift2, *one_plus_scale2, *gate2;
  /* LayerNorm fold of the two linears that follow a LayerNorm (see svx_epilogue_args): qkv_w and fc1_w hold the
   * modulated weights W (1 + scale), u = their row sums, v = b + W shift (fp32 [N]). */
  const float *qkv_u, *qkv_v, *fc1_u, *fc1_v;
} svx_block_weights;

typedef struct {
  const uint16_t *query_w, *query_b, *proj_w, *proj_b, *zero_w, *zero_b;
  const uint16_t *k, *v;     /* packed cached K/V of this layer: [slots][heads][key_capacity][96] bf16, RoPE applied */
  const float *query_u, *query_v; /* LayerNorm fold of the query linear (no affine): row sums of W, v = b (fp32) */
} svx_cross_weights;

typedef struct {
  int slots, height, depth, width, patch, classes, d, heads, mlp, depth_layers;
  int key_capacity;
  int n_control;             /* control layers; control layer j feeds backbone layer layer_index[j] */
  const int32_t* layer_index;/* host array [n_control], strictly increasing */
} svx_engine_config;

typedef struct {
  const uint16_t *table_b, *bias_b, *yadd_b;   /* backbone embed: gather table, bias, per-patch y-embedding */
  const uint16_t *table_c, *bias_c, *yadd_c;   /* control embed */
  const svx_block_weights* backbone;            /* [depth_layers] (host array) */
  const svx_block_weights* control;             /* [n_control] */
  const svx_cross_weights* cross;               /* [n_control] */
  const uint16_t *final_shift, *final_one_plus_scale, *head_w, *head_b; /* head_w rows ordered n = v*64 + o */
  const uint16_t *rope_sin, *rope_cos;          /* self-attention RoPE tables [patches][48] */
  const uint16_t *cross_sin, *cross_cos;        /* cross-attention query RoPE tables [patches][48] */
  const int32_t* lengths;                       /* [slots] valid packed keys per slot (device) */
  const float *head_u, *head_v;                 /* LayerNorm fold of the head: head_w = W (1 + final scale) */
} svx_engine_weights;

typedef struct {
  uint16_t *xb, *xc, *h, *qkv, *attn, *mlp;     /* [slots*patches][d], [..][d], [..][d], [..][3d], [..][d], [..][mlp] */
  uint16_t *qx, *ax;                            /* cross-attention query and output [slots*patches][d] */
  float *stats_b, *stats_c;                     /* row statistics of xb, xc: (mean, M2) [d/32][n*patches] */
} svx_engine_workspace;

typedef struct svx_engine svx_engine;

/* Replaces FastSlotForward's construction (`streamvoxel/stream/fast_ops.py:168-224`): validates shapes and builds
 * the TMA descriptors for every weight and workspace operand. Pointers must stay valid for the handle's life. */
SVX_API int svx_engine_create(const svx_engine_config* config, const svx_engine_weights* weights,
                              const svx_engine_workspace* workspace, svx_engine** out);
/* One slot-batched forward of the first n slots (`FastSlotForward.forward`, `fast_ops.py:274-308`):
 * tokens [n][Y][Z][X] int16 -> logits [n][V][Y][Z][X] bf16. */
SVX_API int svx_engine_forward(svx_engine* engine, int n, const int16_t* tokens, uint16_t* logits, void* stream);
/* Host key lengths of every slot [slots] (the values written to weights->lengths): rebuilds the cross-attention
 * work plans of every bucket and copies them to the engine's device table on `stream` (stream-ordered before later
 * forwards). Optional: without it the plans stay those of equal lengths, which is correct but less balanced.
 * Called where `FastSlotForward._write` stores a slot's length (`fast_ops.py:241-250`). */
SVX_API int svx_engine_set_lengths(svx_engine* engine, const int32_t* lengths, void* stream);
/* Number of kernel launches one svx_engine_forward(n) enqueues. */
SVX_API int svx_engine_launches(const svx_engine* engine, int n);
SVX_API void svx_engine_destroy(svx_engine* engine);

#ifdef __cplusplus
}
#endif
#endif /* SVX_H */
