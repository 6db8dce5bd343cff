// Patch-4 token embed (both branches in one pass) and LayerNorm + AdaLN modulate.
#include <math.h>

#include "common.cuh"
#include "gemm.cuh"

namespace svx {
namespace {

// acc[j] += bf16 element j of the 16 bytes (element 2i in the low half of word i), each add the fp32 add of the
// exactly widened bf16 value, rounded to nearest even. sm_100's mixed-precision add (`add.rn.f32.bf16`) takes the bf16
// half straight from the packed word: one instruction per element instead of a shift or mask plus an fp32 add, which
// takes ~15% off the embed, whose time does not follow the bytes it gathers (all-MASK columns, whose 64 rows repeat in
// every patch, take as long as random ones; skipping repeated rows did not help).
__device__ __forceinline__ void add_bf16x8(float (&a)[8], uint4 r) {
  asm("{\n\t.reg .b16 l0, h0, l1, h1, l2, h2, l3, h3;\n\t"
      "mov.b32 {l0, h0}, %8;\n\tmov.b32 {l1, h1}, %9;\n\tmov.b32 {l2, h2}, %10;\n\tmov.b32 {l3, h3}, %11;\n\t"
      "add.rn.f32.bf16 %0, l0, %0;\n\tadd.rn.f32.bf16 %1, h0, %1;\n\tadd.rn.f32.bf16 %2, l1, %2;\n\t"
      "add.rn.f32.bf16 %3, h1, %3;\n\tadd.rn.f32.bf16 %4, l2, %4;\n\tadd.rn.f32.bf16 %5, h2, %5;\n\t"
      "add.rn.f32.bf16 %6, l3, %6;\n\tadd.rn.f32.bf16 %7, h3, %7;\n\t}"
      : "+f"(a[0]), "+f"(a[1]), "+f"(a[2]), "+f"(a[3]), "+f"(a[4]), "+f"(a[5]), "+f"(a[6]), "+f"(a[7])
      : "r"(r.x), "r"(r.y), "r"(r.z), "r"(r.w));
}

__device__ __forceinline__ void unpack_bf16x8(uint4 raw, float (&v)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[2 * j] = __uint_as_float(w[j] << 16);
    v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
  }
}

// Two values rounded to bf16 (nearest even) and widened back: one paired conversion instead of two single ones.
__device__ __forceinline__ float2 round_bf16_pair(float a, float b) {
  return __bfloat1622float2(__floats2bfloat162_rn(a, b));
}

__device__ __forceinline__ uint4 pack_bf16x8(const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
    w[j] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// out[p] = bf16(bf16(bf16(sum_o T[t_o * 64 + o]) + bias) + add[p]): the gather form of the one-hot Conv3d
// (`streamvoxel/stream/fast_ops.py:69-75`: fp32 accumulation over the 64 patch offsets, the conv bias added in bf16),
// then the per-position y-embedding (`fast_ops.py:282-283`). One CTA per patch, 8 channels per thread. With stats
// buffers it also writes (mean, M2) of every 32-column chunk of the bf16 output row (four adjacent lanes), chunk-major
// ([d/32][rows]), the statistics the first LayerNorm of each branch takes from the GEMM that follows.
__global__ void patch_embed_kernel(const int16_t* __restrict__ tokens, int height, int depth, int width, int classes,
                                   int d, int total_rows, const uint16_t* __restrict__ table_b,
                                   const uint16_t* __restrict__ bias_b, const uint16_t* __restrict__ add_b,
                                   uint16_t* __restrict__ out_b, const uint16_t* __restrict__ table_c,
                                   const uint16_t* __restrict__ bias_c, const uint16_t* __restrict__ add_c,
                                   uint16_t* __restrict__ out_c, float2* __restrict__ stats_b,
                                   float2* __restrict__ stats_c) {
  constexpr int P = 4, P3 = 64;
  grid_launch_dependents();
  grid_dependency_wait();
  const int gz = depth / P, gx = width / P;
  const int patches = (height / P) * gz * gx;
  const int row = blockIdx.x;  // slot * patches + p
  __shared__ int rows[P3];
  for (int o = threadIdx.x; o < P3; o += blockDim.x) {
    const int slot = row / patches, p = row % patches;
    const int py = p / (gz * gx), pz = (p / gx) % gz, px = p % gx;
    const int oy = o >> 4, oz = (o >> 2) & 3, ox = o & 3;
    const int64_t voxel = (((int64_t)slot * height + py * P + oy) * depth + pz * P + oz) * width + px * P + ox;
    int t = tokens[voxel];
    t = t < 0 ? 0 : (t > classes ? classes : t);  // out-of-vocabulary ids clamp instead of reading out of bounds
    rows[o] = t * P3 + o;
  }
  __syncthreads();
  const int c0 = threadIdx.x * 8;
  if (c0 >= d) return;
  for (int branch = 0; branch < 2; ++branch) {
    if (!(branch ? table_c : table_b)) continue;
    const uint16_t* table = (branch ? table_c : table_b) + c0;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int o = 0; o < P3; ++o) add_bf16x8(acc, *reinterpret_cast<const uint4*>(table + (int64_t)rows[o] * d));
    float bias[8], add[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>((branch ? bias_c : bias_b) + c0), bias);
    unpack_bf16x8(*reinterpret_cast<const uint4*>((branch ? add_c : add_b) + (int64_t)(row % patches) * d + c0), add);
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      float2 r = round_bf16_pair(acc[j], acc[j + 1]);
      r = round_bf16_pair(r.x + bias[j], r.y + bias[j + 1]);
      r = round_bf16_pair(r.x + add[j], r.y + add[j + 1]);
      acc[j] = r.x;
      acc[j + 1] = r.y;
    }
    *reinterpret_cast<uint4*>((branch ? out_c : out_b) + (int64_t)row * d + c0) = pack_bf16x8(acc);
    float2* stats = branch ? stats_c : stats_b;
    if (stats) {   // d % 32 == 0: the four lanes of a chunk are all active (lanes past d have returned)
      const unsigned group = 0xFu << (threadIdx.x & 28);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += acc[j];
      sum += __shfl_xor_sync(group, sum, 1);
      sum += __shfl_xor_sync(group, sum, 2);
      const float mean = sum * (1.f / 32.f);
      float m2 = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) m2 = fmaf(acc[j] - mean, acc[j] - mean, m2);
      m2 += __shfl_xor_sync(group, m2, 1);
      m2 += __shfl_xor_sync(group, m2, 2);
      if ((threadIdx.x & 3) == 0) stats[(int64_t)(threadIdx.x / 4) * total_rows + row] = make_float2(mean, m2);
    }
  }
}

// LayerNorm (no affine; fp32 statistics, `unconditional_md4_timefree.py:53-54`) and the AdaLN modulate
// x * (1 + scale) + shift in fp32 (`:12-13`), rounded to bf16 where the next linear casts its input.
// One warp per row; lane L holds the 8-channel chunks L, L+32, ... (d % 8 == 0, at most 32*PER chunks).
template <int PER>
__global__ void layernorm_modulate_kernel(const uint16_t* __restrict__ x, int rows, int d, float eps,
                                          const uint16_t* __restrict__ ops, const uint16_t* __restrict__ shift,
                                          uint16_t* __restrict__ out) {
  grid_launch_dependents();
  grid_dependency_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + warp_id();
  if (row >= rows) return;
  const int lane = lane_id();
  const int chunks = d >> 3;
  const uint16_t* src = x + (int64_t)row * d;
  float v[PER][8];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = i * 32 + lane;
    if (c < chunks) {
      unpack_bf16x8(*reinterpret_cast<const uint4*>(src + c * 8), v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += v[i][j];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / d;
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    if (i * 32 + lane < chunks) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float c = v[i][j] - mean;
        var += c * c;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
  const float rstd = rsqrtf(var / d + eps);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = i * 32 + lane;
    if (c >= chunks) continue;
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = (v[i][j] - mean) * rstd;
    if (ops) {
      float s[8], b[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(ops + c * 8), s);
      unpack_bf16x8(*reinterpret_cast<const uint4*>(shift + c * 8), b);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = __fadd_rn(__fmul_rn(y[j], s[j]), b[j]);
    }
    *reinterpret_cast<uint4*>(out + (int64_t)row * d + c * 8) = pack_bf16x8(y);
  }
}

// LayerNorm of the condition encoder (`streamvoxel/models/streaming_controlnet.py:142-158,160-169,218`) in fp32:
// v = x + pre (pre: the fp32 type + size embeddings, `:158,217`; optional), y = (v - mean) * rstd, then
// y * weight + bias (fp32 affine of `l2_norm`, `:147`; optional) and GELU(erf) (`:147`; optional), stored bf16
// (the cast the next linear or conv makes under autocast). One warp per row, as above; a warp reads its whole row
// before it writes, so out may be x (in place).
template <int PER>
__global__ void layernorm_affine_kernel(const uint16_t* x, int rows, int d, float eps, const float* __restrict__ pre,
                                        const float* __restrict__ weight, const float* __restrict__ bias, int gelu,
                                        uint16_t* out) {
  grid_launch_dependents();
  grid_dependency_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + warp_id();
  if (row >= rows) return;
  const int lane = lane_id();
  const int chunks = d >> 3;
  const uint16_t* src = x + (int64_t)row * d;
  float v[PER][8];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = i * 32 + lane;
    if (c < chunks) {
      unpack_bf16x8(*reinterpret_cast<const uint4*>(src + c * 8), v[i]);
      if (pre) {
        const float4 a = *reinterpret_cast<const float4*>(pre + c * 8);
        const float4 b = *reinterpret_cast<const float4*>(pre + c * 8 + 4);
        v[i][0] += a.x; v[i][1] += a.y; v[i][2] += a.z; v[i][3] += a.w;
        v[i][4] += b.x; v[i][5] += b.y; v[i][6] += b.z; v[i][7] += b.w;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += v[i][j];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum / d;
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    if (i * 32 + lane < chunks) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float c = v[i][j] - mean;
        var += c * c;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
  const float rstd = rsqrtf(var / d + eps);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = i * 32 + lane;
    if (c >= chunks) continue;
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = (v[i][j] - mean) * rstd;
    if (weight) {
      const float w[8] = {weight[c * 8], weight[c * 8 + 1], weight[c * 8 + 2], weight[c * 8 + 3],
                          weight[c * 8 + 4], weight[c * 8 + 5], weight[c * 8 + 6], weight[c * 8 + 7]};
      const float b[8] = {bias[c * 8], bias[c * 8 + 1], bias[c * 8 + 2], bias[c * 8 + 3],
                          bias[c * 8 + 4], bias[c * 8 + 5], bias[c * 8 + 6], bias[c * 8 + 7]};
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = fmaf(y[j], w[j], b[j]);
    }
    if (gelu) {
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = 0.5f * y[j] * (1.f + erff(y[j] * 0.7071067811865476f));
    }
    *reinterpret_cast<uint4*>(out + (int64_t)row * d + c * 8) = pack_bf16x8(y);
  }
}

}  // namespace

int patch_embed_run(const int16_t* tokens, int slots, int height, int depth, int width, int classes, int d,
                    const uint16_t* table_b, const uint16_t* bias_b, const uint16_t* add_b, uint16_t* out_b,
                    const uint16_t* table_c, const uint16_t* bias_c, const uint16_t* add_c, uint16_t* out_c,
                    float* stats_b, float* stats_c, cudaStream_t stream) {
  SVX_REQUIRE((!stats_b && !stats_c) || d % 32 == 0, "patch_embed: row statistics need d % 32 == 0");
  const int patches = (height / 4) * (depth / 4) * (width / 4);
  int threads = ((d / 8 + 31) / 32) * 32;
  if (threads < 64) threads = 64;
  return launch_dependent("patch_embed_kernel", patch_embed_kernel, dim3(slots * patches), dim3(threads), 0, stream,
                          tokens, height, depth, width, classes, d, slots * patches, table_b, bias_b, add_b, out_b,
                          table_c, bias_c, add_c, out_c, reinterpret_cast<float2*>(stats_b),
                          reinterpret_cast<float2*>(stats_c));
}

int layernorm_run(const uint16_t* x, int rows, int d, float eps, const uint16_t* ops, const uint16_t* shift,
                  uint16_t* out, cudaStream_t stream) {
  const int warps = 8;
  const int grid = (rows + warps - 1) / warps;
  const dim3 g(grid), b(warps * 32);
  const char* what = "layernorm_modulate_kernel";
  switch ((d / 8 + 31) / 32) {
    case 1: return launch_dependent(what, layernorm_modulate_kernel<1>, g, b, 0, stream, x, rows, d, eps, ops, shift, out);
    case 2: return launch_dependent(what, layernorm_modulate_kernel<2>, g, b, 0, stream, x, rows, d, eps, ops, shift, out);
    case 3: return launch_dependent(what, layernorm_modulate_kernel<3>, g, b, 0, stream, x, rows, d, eps, ops, shift, out);
    case 4: return launch_dependent(what, layernorm_modulate_kernel<4>, g, b, 0, stream, x, rows, d, eps, ops, shift, out);
    case 5: return launch_dependent(what, layernorm_modulate_kernel<5>, g, b, 0, stream, x, rows, d, eps, ops, shift, out);
    case 6: return launch_dependent(what, layernorm_modulate_kernel<6>, g, b, 0, stream, x, rows, d, eps, ops, shift, out);
    default: return fail(SVX_ERR_INVALID, "layernorm: d must be at most 1536");
  }
}

int layernorm_affine_run(const uint16_t* x, int rows, int d, float eps, const float* pre, const float* weight,
                         const float* bias, int gelu, uint16_t* out, cudaStream_t stream) {
  using Kernel = void (*)(const uint16_t*, int, int, float, const float*, const float*, const float*, int, uint16_t*);
  static const Kernel kernels[] = {layernorm_affine_kernel<1>, layernorm_affine_kernel<2>, layernorm_affine_kernel<3>,
                                   layernorm_affine_kernel<4>, layernorm_affine_kernel<5>, layernorm_affine_kernel<6>};
  const int per = (d / 8 + 31) / 32;
  if (per < 1 || per > 6) return fail(SVX_ERR_INVALID, "layernorm_affine: d must be at most 1536");
  const int warps = 8;
  return launch_dependent("layernorm_affine_kernel", kernels[per - 1], dim3((rows + warps - 1) / warps),
                          dim3(warps * 32), 0, stream, x, rows, d, eps, pre, weight, bias, gelu, out);
}

}  // namespace svx

using namespace svx;

extern "C" int svx_patch_embed(const int16_t* tokens, int slots, int height, int depth, int width, int patch,
                               int classes, int d, const uint16_t* table_b, const uint16_t* bias_b,
                               const uint16_t* add_b, uint16_t* out_b, const uint16_t* table_c,
                               const uint16_t* bias_c, const uint16_t* add_c, uint16_t* out_c, float* stats_b,
                               float* stats_c, void* stream) {
  SVX_REQUIRE(patch == 4, "svx_patch_embed: only patch 4 is implemented");
  SVX_REQUIRE(height % 4 == 0 && depth % 4 == 0 && width % 4 == 0 && slots > 0, "svx_patch_embed: bad shape");
  SVX_REQUIRE(d % 8 == 0 && d <= 8192, "svx_patch_embed: d must be a multiple of 8");
  SVX_REQUIRE(tokens && table_b && bias_b && add_b && out_b, "svx_patch_embed: null backbone operand");
  SVX_REQUIRE(!table_c || (bias_c && add_c && out_c), "svx_patch_embed: incomplete control operands");
  SVX_REQUIRE(!stats_c || table_c, "svx_patch_embed: control statistics without the control branch");
  return patch_embed_run(tokens, slots, height, depth, width, classes, d, table_b, bias_b, add_b, out_b, table_c,
                         bias_c, add_c, out_c, stats_b, stats_c, as_stream(stream));
}

extern "C" int svx_layernorm_modulate(const uint16_t* x, int rows, int d, float eps, const uint16_t* one_plus_scale,
                                      const uint16_t* shift, uint16_t* out, void* stream) {
  SVX_REQUIRE(x && out && rows > 0, "svx_layernorm_modulate: bad arguments");
  SVX_REQUIRE((one_plus_scale == nullptr) == (shift == nullptr), "svx_layernorm_modulate: scale and shift go together");
  SVX_REQUIRE(d % 8 == 0 && d <= 1536, "svx_layernorm_modulate: d must be a multiple of 8, at most 1536");
  return layernorm_run(x, rows, d, eps, one_plus_scale, shift, out, as_stream(stream));
}

extern "C" int svx_layernorm_affine(const uint16_t* x, int rows, int d, float eps, const float* pre,
                                    const float* weight, const float* bias, int gelu, uint16_t* out, void* stream) {
  SVX_REQUIRE(x && out && rows > 0, "svx_layernorm_affine: bad arguments");
  SVX_REQUIRE((weight == nullptr) == (bias == nullptr), "svx_layernorm_affine: weight and bias go together");
  SVX_REQUIRE(d % 8 == 0 && d <= 1536, "svx_layernorm_affine: d must be a multiple of 8, at most 1536");
  SVX_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
                reinterpret_cast<uintptr_t>(pre)) & 15) == 0,
              "svx_layernorm_affine: x, out and pre must be 16-byte aligned");
  return layernorm_affine_run(x, rows, d, eps, pre, weight, bias, gelu, out, as_stream(stream));
}
