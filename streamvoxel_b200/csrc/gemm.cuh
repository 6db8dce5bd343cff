// Host-side entry points shared by the C-ABI wrappers and the engine (TMA descriptors are built once per operand).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace svx {

struct EpiParams {
  int epilogue;
  const uint16_t* bias;
  const uint16_t* gate;
  const uint16_t* residual;
  const uint16_t* rope_sin;
  const uint16_t* rope_cos;
  int rope_cols, rows_per_slot, head_dim, classes, height, depth, width, patch;
  // LayerNorm fold (consumer): with ln_stats_in the epilogue computes r (acc - mu u[n]) + v[n] in place of
  // acc + bias, mu and r = 1/sqrt(var + ln_eps) merged from the row's 32-column chunk statistics (A is the raw row x,
  // W the modulated weights W'[n][k] = W[n][k] (1 + scale[k]), u[n] = sum_k W'[n][k], v[n] = b[n] + sum_k W[n][k]
  // shift[k]), so that no LayerNorm kernel runs between a residual GEMM and the next linear.
  const float2* ln_stats_in;   // [ln_chunks][M] (mean, M2) of the input rows' 32-column chunks (chunk-major)
  const float* ln_u;           // [N] fp32
  const float* ln_v;           // [N] fp32
  int ln_chunks;
  float ln_inv_chunks;         // 1 / ln_chunks
  float ln_eps;
  // LayerNorm statistics for the next linear (producer): (mean, M2) of each 32-column chunk of the bf16 output row.
  float2* ln_stats_out;        // [N / 32][M] (chunk-major)
};

struct GemmPlan {
  CUtensorMap a, b;      // A boxes of 128 rows, W boxes of `bn` rows (one CTA per tile)
  CUtensorMap b_half;    // W boxes of pair_bn / 2 rows (CTA pairs, 256-row tiles)
  int M, N, K, bn, pair_bn;
};

int gemm_plan(GemmPlan* plan, const uint16_t* A, const uint16_t* W, int M, int N, int K, int bn);
int gemm_run(const GemmPlan& plan, int M, uint16_t* out, const EpiParams& ep, cudaStream_t stream);
int gemm_run_group(const GemmPlan& p0, uint16_t* out0, const EpiParams& e0, const GemmPlan& p1, uint16_t* out1,
                   const EpiParams& e1, int M, cudaStream_t stream);
// 3-D bf16 tensor map (inner, groups, rows), box (box_inner, 1, box_rows), 128B swizzle (box_inner 64) or 64B swizzle
// (box_inner 32); elements past `inner` read 0.
int make_map_3d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t groups, uint64_t rows,
                uint64_t group_stride_bytes, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);
uint32_t attention_timeouts();
int epi_from_args(const svx_epilogue_args* e, EpiParams* ep, int N, int K);
int attention_run(const uint16_t* q, int64_t q_row_stride, const uint16_t* k, const uint16_t* v,
                  int64_t kv_slot_stride, int64_t kv_head_stride, int64_t kv_row_stride, const int32_t* lengths,
                  int slots, int heads, int queries, int keys, uint16_t* out, const int32_t* plan, int plan_ctas,
                  cudaStream_t stream);
// One or two attention problems over the same slots, heads and queries in one persistent launch (two need a plan).
int attention_launch(const svx_attention_problem* problems, int count, int slots, int heads, int queries,
                     const int32_t* plan, int plan_ctas, cudaStream_t stream);
// Host-side assignment of the attention work units of 1-2 problems to CTAs (layout in attention.cu); ints it takes.
int attention_plan_ints(int problems, int slots, int heads, int queries, int ctas);
int attention_plan(const int32_t* const* lengths, const int* keys, int problems, int slots, int heads, int queries,
                   int ctas, int32_t* plan, int capacity);
int patch_embed_run(const int16_t* tokens, int slots, int height, int depth, int width, int classes, int d,
                    const uint16_t* table_b, const uint16_t* bias_b, const uint16_t* add_b, uint16_t* out_b,
                    const uint16_t* table_c, const uint16_t* bias_c, const uint16_t* add_c, uint16_t* out_c,
                    float* stats_b, float* stats_c, cudaStream_t stream);
int layernorm_run(const uint16_t* x, int rows, int d, float eps, const uint16_t* ops, const uint16_t* shift,
                  uint16_t* out, cudaStream_t stream);
int layernorm_affine_run(const uint16_t* x, int rows, int d, float eps, const float* pre, const float* weight,
                         const float* bias, int gelu, uint16_t* out, cudaStream_t stream);

}  // namespace svx
