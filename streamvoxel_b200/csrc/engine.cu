// The slot-batched forward of the time-free DiT backbone + compact ControlNet as one host-driven launch sequence.
//
// Replaces `FastSlotForward.forward` (`streamvoxel/stream/fast_ops.py:274-308`), i.e.
// `CompactStreamingControlNet.forward` (`streamvoxel/models/compact_controlnet.py:100-159`) over cached packed K/V:
//   b, c = embed(tokens) + y_embed
//   for i in layers: if i feeds control layer j: c = block_c(c); c = c + cross_j(c); b = block_b(b) + zero_j(c)
//                    else:                      b = block_b(b)
// The cross-attention of control layer j and the self-attention of backbone layer i are independent, so they run
// as one attention launch (LN, query, LN, qkv first; proj, cross proj after), with one work plan over both.
//   logits = head(modulate(LN(b)))  in class-major [slot][V][Y][Z][X]
// Every TMA descriptor is built once in svx_engine_create; svx_engine_forward only enqueues kernels, so it can be
// captured in a CUDA graph per slot bucket. No LayerNorm kernel runs: every residual-stream producer (the embed and
// the residual GEMM epilogues) writes the row statistics of its bf16 output, and every linear that follows a
// LayerNorm + AdaLN modulate takes the raw stream with the modulation folded into its weights and the normalisation
// into its epilogue (r (acc - mu u) + v).
#include <vector>

#include "common.cuh"
#include "gemm.cuh"

struct svx_engine {
  svx_engine_config cfg;
  std::vector<int> layer_map;  // backbone layer -> control layer or -1
  svx_engine_weights w;
  std::vector<svx_block_weights> backbone, control;
  std::vector<svx_cross_weights> cross;
  svx_engine_workspace ws;
  int patches, rows_max;
  // GEMM plans: per backbone layer [qkv, proj, fc1, fc2]; per control layer [qkv, proj, fc1, fc2, query, cproj, zero].
  std::vector<svx::GemmPlan> bplan, cplan;
  svx::GemmPlan head;
  // Work plans of the joint cross + self attention launch (svx::attention_plan, two problems, on plan_ctas CTAs),
  // one row of plan_stride ints per bucket n = 1..slots, rebuilt on the host by svx_engine_set_lengths.
  int32_t* plan_dev = nullptr;
  int plan_stride = 0, plan_ctas = 0;
  std::vector<int32_t> plan_host;
  // bf16 ones [d]: the gate that makes the cross projection's plain residual a gated one, so that it runs in one
  // launch with the backbone's attention projection (svx::gemm_run_group)
  uint16_t* ones = nullptr;
  ~svx_engine() {
    if (plan_dev) cudaFree(plan_dev);
    if (ones) cudaFree(ones);
  }
};

namespace svx {
namespace {

constexpr int HD = 96;

// x: the block's residual stream, the A operand of its qkv and fc1 linears (LayerNorm folded in).
int plan_block(std::vector<GemmPlan>& plans, const svx_block_weights& bw, const svx_engine_workspace& ws,
               const uint16_t* x, int rows, int d, int mlp) {
  GemmPlan p;
  int rc;
  if ((rc = gemm_plan(&p, x, bw.qkv_w, rows, 3 * d, d, 0))) return rc;
  plans.push_back(p);
  if ((rc = gemm_plan(&p, ws.attn, bw.proj_w, rows, d, d, 0))) return rc;
  plans.push_back(p);
  if ((rc = gemm_plan(&p, x, bw.fc1_w, rows, mlp, d, 0))) return rc;
  plans.push_back(p);
  if ((rc = gemm_plan(&p, ws.mlp, bw.fc2_w, rows, d, mlp, 0))) return rc;
  plans.push_back(p);
  return SVX_OK;
}

EpiParams epi(int kind, const uint16_t* bias) {
  EpiParams e{};
  e.epilogue = kind;
  e.bias = bias;
  return e;
}

float2* stats_of(const svx_engine& E, const uint16_t* x) {
  return reinterpret_cast<float2*>(x == E.ws.xb ? E.ws.stats_b : E.ws.stats_c);
}

// The LayerNorm (eps 1e-6, `unconditional_md4_timefree.py:53-54`) of x folded into a linear's epilogue.
void fold(EpiParams& e, const svx_engine& E, const uint16_t* x, const float* u, const float* v) {
  e.ln_stats_in = stats_of(E, x);
  e.ln_u = u;
  e.ln_v = v;
  e.ln_chunks = E.cfg.d / 32;
  e.ln_inv_chunks = 32.f / (float)E.cfg.d;
  e.ln_eps = 1e-6f;
}

// The self-attention problem of a block: q, k, v interleaved in the qkv workspace, out to the attn workspace.
svx_attention_problem self_problem(const svx_engine& E) {
  const svx_engine_workspace& ws = E.ws;
  const int d = E.cfg.d;
  const int64_t ld = 3 * d;
  return svx_attention_problem{ws.qkv, ws.qkv + d, ws.qkv + 2 * d, ld, (int64_t)E.patches * ld, HD, ld, nullptr,
                               E.patches, ws.attn};
}

// The first half of a block: qkv = RoPE(modulate(LN(x)) W_qkv^T + b), the LayerNorm folded into the epilogue.
int run_block_qkv(const svx_engine& E, const svx_block_weights& bw, const GemmPlan* plans, uint16_t* x, int n,
                  cudaStream_t s) {
  const int d = E.cfg.d, rows = n * E.patches;
  const svx_engine_workspace& ws = E.ws;
  EpiParams e = epi(SVX_EPI_ROPE, bw.qkv_b);
  fold(e, E, x, bw.qkv_u, bw.qkv_v);
  e.rope_sin = E.w.rope_sin; e.rope_cos = E.w.rope_cos;
  e.rope_cols = 2 * d; e.rows_per_slot = E.patches; e.head_dim = HD;
  return gemm_run(plans[0], rows, ws.qkv, e, s);
}

// x += g1 proj(attn), with the row statistics of the new x.
EpiParams proj_epi(const svx_engine& E, const svx_block_weights& bw, uint16_t* x) {
  EpiParams e = epi(SVX_EPI_GATE_RESIDUAL, bw.proj_b);
  e.gate = bw.gate1; e.residual = x; e.ln_stats_out = stats_of(E, x);
  return e;
}

// The MLP half: x += g2 fc2(GELU(fc1(modulate(LN(x))))).
int run_block_mlp(const svx_engine& E, const svx_block_weights& bw, const GemmPlan* plans, uint16_t* x, int n,
                  cudaStream_t s) {
  const int rows = n * E.patches;
  const svx_engine_workspace& ws = E.ws;
  int rc;
  EpiParams e = epi(SVX_EPI_BIAS_GELU, bw.fc1_b);
  fold(e, E, x, bw.fc1_u, bw.fc1_v);
  if ((rc = gemm_run(plans[2], rows, ws.mlp, e, s))) return rc;
  e = epi(SVX_EPI_GATE_RESIDUAL, bw.fc2_b);
  e.gate = bw.gate2; e.residual = x; e.ln_stats_out = stats_of(E, x);
  return gemm_run(plans[3], rows, x, e, s);
}

// The second half, after the attention: x += g1 proj(attn), then the MLP half.
int run_block_rest(const svx_engine& E, const svx_block_weights& bw, const GemmPlan* plans, uint16_t* x, int n,
                   cudaStream_t s) {
  int rc;
  if ((rc = gemm_run(plans[1], n * E.patches, x, proj_epi(E, bw, x), s))) return rc;
  return run_block_mlp(E, bw, plans, x, n, s);
}

// One time-free AdaLN block on x (`UnconditionalBlock.forward`, `unconditional_md4_timefree.py:60-63`).
int run_block(const svx_engine& E, const svx_block_weights& bw, const GemmPlan* plans, uint16_t* x, int n,
              cudaStream_t s) {
  int rc;
  if ((rc = run_block_qkv(E, bw, plans, x, n, s))) return rc;
  const svx_attention_problem a = self_problem(E);
  if ((rc = attention_launch(&a, 1, n, E.cfg.heads, E.patches, nullptr, 0, s))) return rc;
  return run_block_rest(E, bw, plans, x, n, s);
}

// Control layer j with backbone layer i (`RotaryCrossAttention.forward`, `streaming_controlnet.py:37-61`, as
// `cross_flex` `fast_ops.py:104-108`, and `compact_controlnet.py:100-159`): c = block_c(c); qx = RoPE(LN(c) Wq);
// qkv = block_b's first half; [cross-attention of qx over the slot's packed keys -> ax, self-attention -> attn]
// in one launch; c += proj(ax); block_b's second half; b += zero(c).
int run_control_layer(const svx_engine& E, int i, int j, int n, cudaStream_t s) {
  const int d = E.cfg.d, rows = n * E.patches;
  const svx_engine_workspace& ws = E.ws;
  const svx_cross_weights& cw = E.cross[j];
  const GemmPlan* cp = &E.cplan[(size_t)j * 7];
  const GemmPlan* bp = &E.bplan[(size_t)i * 4];
  int rc;
  if ((rc = run_block(E, E.control[j], cp, ws.xc, n, s))) return rc;
  EpiParams e = epi(SVX_EPI_ROPE, cw.query_b);
  fold(e, E, ws.xc, cw.query_u, cw.query_v);   // LayerNorm without affine (`streaming_controlnet.py:44`)
  e.rope_sin = E.w.cross_sin; e.rope_cos = E.w.cross_cos;
  e.rope_cols = d; e.rows_per_slot = E.patches; e.head_dim = HD;
  if ((rc = gemm_run(cp[4], rows, ws.qx, e, s))) return rc;
  if ((rc = run_block_qkv(E, E.backbone[i], bp, ws.xb, n, s))) return rc;
  const int64_t cap = E.cfg.key_capacity;
  const svx_attention_problem both[2] = {
      {ws.qx, cw.k, cw.v, d, (int64_t)E.cfg.heads * cap * HD, cap * HD, HD, E.w.lengths, E.cfg.key_capacity, ws.ax},
      self_problem(E)};
  const int units = 2 * n * E.cfg.heads * ((E.patches / 128 + 1) / 2);
  const int32_t* plan = E.plan_dev + (size_t)(n - 1) * E.plan_stride;
  if ((rc = attention_launch(both, 2, n, E.cfg.heads, E.patches, plan, std::min(E.plan_ctas, units), s))) return rc;
  // c += proj(ax) (a residual: its gate is ones) and b += g1 proj(attn) in one launch, then block_b's MLP half
  e = epi(SVX_EPI_GATE_RESIDUAL, cw.proj_b);
  e.gate = E.ones; e.residual = ws.xc; e.ln_stats_out = stats_of(E, ws.xc);
  if (rows % 256 == 0) {
    rc = gemm_run_group(cp[5], ws.xc, e, bp[1], ws.xb, proj_epi(E, E.backbone[i], ws.xb), rows, s);
  } else {
    rc = gemm_run(cp[5], rows, ws.xc, e, s);
    if (!rc) rc = gemm_run(bp[1], rows, ws.xb, proj_epi(E, E.backbone[i], ws.xb), s);
  }
  if (rc) return rc;
  if ((rc = run_block_mlp(E, E.backbone[i], bp, ws.xb, n, s))) return rc;
  e = epi(SVX_EPI_RESIDUAL, cw.zero_b);
  e.residual = ws.xb; e.ln_stats_out = stats_of(E, ws.xb);
  return gemm_run(cp[6], rows, ws.xb, e, s);
}

// Joint cross + self attention plans of every bucket n = 1..slots for the host key lengths (NULL: all slots at the
// key capacity).
int build_plans(svx_engine& E, const int32_t* lengths) {
  const int32_t* lens[2] = {lengths, nullptr};
  const int keys[2] = {E.cfg.key_capacity, E.patches};
  for (int n = 1; n <= E.cfg.slots; ++n) {
    const int rc = attention_plan(lens, keys, 2, n, E.cfg.heads, E.patches, E.plan_ctas,
                                  E.plan_host.data() + (size_t)(n - 1) * E.plan_stride, E.plan_stride);
    if (rc) return rc;
  }
  return SVX_OK;
}

}  // namespace
}  // namespace svx

using namespace svx;

extern "C" int svx_engine_create(const svx_engine_config* config, const svx_engine_weights* weights,
                                 const svx_engine_workspace* workspace, svx_engine** out) {
  SVX_REQUIRE(config && weights && workspace && out, "svx_engine_create: null argument");
  const svx_engine_config& c = *config;
  SVX_REQUIRE(c.patch == 4, "svx_engine_create: patch must be 4");
  SVX_REQUIRE(c.height % 4 == 0 && c.depth % 4 == 0 && c.width % 4 == 0, "svx_engine_create: bad voxel shape");
  SVX_REQUIRE(c.heads > 0 && c.d == c.heads * HD, "svx_engine_create: head_dim must be 96 (d = heads * 96)");
  SVX_REQUIRE(workspace->stats_b && workspace->stats_c && weights->head_u && weights->head_v,
              "svx_engine_create: the LayerNorm fold needs the row-statistics workspace and the head's u and v");
  for (int i = 0; i < c.depth_layers; ++i)
    SVX_REQUIRE(weights->backbone[i].qkv_u && weights->backbone[i].qkv_v && weights->backbone[i].fc1_u &&
                    weights->backbone[i].fc1_v,
                "svx_engine_create: every block needs the LayerNorm fold's u and v");
  for (int j = 0; j < c.n_control; ++j)
    SVX_REQUIRE(weights->control[j].qkv_u && weights->control[j].qkv_v && weights->control[j].fc1_u &&
                    weights->control[j].fc1_v && weights->cross[j].query_u && weights->cross[j].query_v,
                "svx_engine_create: every control layer needs the LayerNorm fold's u and v");
  SVX_REQUIRE(c.slots > 0 && c.depth_layers > 0 && c.n_control >= 0 && c.n_control <= c.depth_layers,
              "svx_engine_create: bad layer counts");
  SVX_REQUIRE(c.n_control == 0 || (c.layer_index && c.key_capacity > 0 && c.key_capacity % 64 == 0),
              "svx_engine_create: control layers need layer indexes and a key capacity (multiple of 64)");
  auto* e = new svx_engine();
  e->cfg = c;
  e->w = *weights;
  e->ws = *workspace;
  e->patches = (c.height / 4) * (c.depth / 4) * (c.width / 4);
  e->rows_max = c.slots * e->patches;
  e->layer_map.assign(c.depth_layers, -1);
  for (int j = 0; j < c.n_control; ++j) {
    const int i = c.layer_index[j];
    if (i < 0 || i >= c.depth_layers || (j > 0 && i <= c.layer_index[j - 1])) {
      delete e;
      return fail(SVX_ERR_INVALID, "svx_engine_create: layer indexes must be increasing and within the backbone");
    }
    e->layer_map[i] = j;
  }
  e->cfg.layer_index = nullptr;
  e->backbone.assign(weights->backbone, weights->backbone + c.depth_layers);
  if (c.n_control) {
    e->control.assign(weights->control, weights->control + c.n_control);
    e->cross.assign(weights->cross, weights->cross + c.n_control);
  }
  e->w.backbone = nullptr; e->w.control = nullptr; e->w.cross = nullptr;
  int rc = SVX_OK;
  for (int i = 0; i < c.depth_layers && !rc; ++i)
    rc = plan_block(e->bplan, e->backbone[i], e->ws, e->ws.xb, e->rows_max, c.d, c.mlp);
  for (int j = 0; j < c.n_control && !rc; ++j) {
    rc = plan_block(e->cplan, e->control[j], e->ws, e->ws.xc, e->rows_max, c.d, c.mlp);
    GemmPlan p;
    if (!rc) rc = gemm_plan(&p, e->ws.xc, e->cross[j].query_w, e->rows_max, c.d, c.d, 0);
    if (!rc) e->cplan.push_back(p);
    if (!rc) rc = gemm_plan(&p, e->ws.ax, e->cross[j].proj_w, e->rows_max, c.d, c.d, 0);
    if (!rc) e->cplan.push_back(p);
    if (!rc) rc = gemm_plan(&p, e->ws.xc, e->cross[j].zero_w, e->rows_max, c.d, c.d, 0);
    if (!rc) e->cplan.push_back(p);
  }
  if (!rc) rc = gemm_plan(&e->head, e->ws.xb, weights->head_w, e->rows_max, c.classes * 64, c.d, 0);
  if (!rc && c.n_control) {
    int device = 0, sms = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err == cudaSuccess) err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (err == cudaSuccess) {
      e->plan_ctas = sms;
      e->plan_stride = attention_plan_ints(2, c.slots, c.heads, e->patches, sms);
      e->plan_host.assign((size_t)c.slots * e->plan_stride, 0);
      rc = e->plan_stride > 0 ? build_plans(*e, nullptr) : fail(SVX_ERR_INVALID, "svx_engine_create: bad plan shape");
      if (!rc) err = cudaMalloc(&e->plan_dev, e->plan_host.size() * sizeof(int32_t));
      if (!rc && err == cudaSuccess)
        err = cudaMemcpy(e->plan_dev, e->plan_host.data(), e->plan_host.size() * sizeof(int32_t),
                         cudaMemcpyHostToDevice);
      const std::vector<uint16_t> ones((size_t)c.d, 0x3F80);   // bf16 1.0
      if (!rc && err == cudaSuccess) err = cudaMalloc(&e->ones, ones.size() * sizeof(uint16_t));
      if (!rc && err == cudaSuccess)
        err = cudaMemcpy(e->ones, ones.data(), ones.size() * sizeof(uint16_t), cudaMemcpyHostToDevice);
    }
    if (!rc && err != cudaSuccess) rc = fail(SVX_ERR_CUDA, cudaGetErrorString(err));
  }
  if (rc) {
    delete e;
    return rc;
  }
  *out = e;
  return SVX_OK;
}

extern "C" int svx_engine_forward(svx_engine* E, int n, const int16_t* tokens, uint16_t* logits, void* stream) {
  SVX_REQUIRE(E && tokens && logits, "svx_engine_forward: null argument");
  SVX_REQUIRE(n >= 1 && n <= E->cfg.slots, "svx_engine_forward: n must be in 1..slots");
  cudaStream_t s = as_stream(stream);
  const svx_engine_config& c = E->cfg;
  const svx_engine_workspace& ws = E->ws;
  const int rows = n * E->patches;
  int rc = patch_embed_run(tokens, n, c.height, c.depth, c.width, c.classes, c.d, E->w.table_b, E->w.bias_b,
                           E->w.yadd_b, ws.xb, c.n_control ? E->w.table_c : nullptr, E->w.bias_c, E->w.yadd_c, ws.xc,
                           ws.stats_b, c.n_control ? ws.stats_c : nullptr, s);
  if (rc) return rc;
  for (int i = 0; i < c.depth_layers; ++i) {
    const int j = E->layer_map[i];
    rc = j >= 0 ? run_control_layer(*E, i, j, n, s)
                : run_block(*E, E->backbone[i], &E->bplan[(size_t)i * 4], ws.xb, n, s);
    if (rc) return rc;
  }
  EpiParams e{};
  e.epilogue = SVX_EPI_CLASS_MAJOR;
  e.bias = E->w.head_b;
  fold(e, *E, ws.xb, E->w.head_u, E->w.head_v);   // final LN + modulate (`unconditional_md4_timefree.py:172-175`)
  e.rows_per_slot = E->patches;
  e.classes = c.classes;
  e.height = c.height; e.depth = c.depth; e.width = c.width; e.patch = 4;
  return gemm_run(E->head, rows, logits, e, s);
}

extern "C" int svx_engine_set_lengths(svx_engine* E, const int32_t* lengths, void* stream) {
  SVX_REQUIRE(E && lengths, "svx_engine_set_lengths: null argument");
  if (!E->plan_dev) return SVX_OK;   // no cross-attention layers
  const int rc = build_plans(*E, lengths);
  if (rc) return rc;
  // Pageable source: the runtime stages it before returning, so plan_host may be rebuilt by the next call.
  SVX_CHECK_CUDA(cudaMemcpyAsync(E->plan_dev, E->plan_host.data(), E->plan_host.size() * sizeof(int32_t),
                                 cudaMemcpyHostToDevice, as_stream(stream)));
  return SVX_OK;
}

extern "C" int svx_engine_launches(const svx_engine* E, int n) {
  if (!E || n < 1) return 0;
  const int per_block = 5;   // qkv, attention, proj, fc1, fc2 (LayerNorms folded into qkv and fc1)
  // query, zero (+ proj when it cannot share the backbone projection's launch); the attention shares the backbone
  // block's launch
  const int per_cross = (n * E->patches) % 256 == 0 ? 2 : 3;
  return 1 + E->cfg.depth_layers * per_block + E->cfg.n_control * (per_block + per_cross) + 1;
}

extern "C" void svx_engine_destroy(svx_engine* E) { delete E; }
