// Non-causal attention with head_dim 96 over per-slot variable-length keys (FlashAttention-2 style online softmax).
//
// One CTA = 128 queries of one (slot, head); 8 warps x 16 query rows. K/V tiles of 64 keys are double-buffered in
// shared memory with cp.async (rows past the slot length are zero-filled and masked to -inf), so a slot pays only for
// ceil(length / 64) key tiles: the packed-key FlexAttention block mask of `streamvoxel/stream/fast_ops.py:149-159`.
// S = Q K^T and O = P V run on mma.sync m16n8k16 (bf16 in, fp32 accumulate); P is rounded to bf16 for the second
// product like SDPA's flash kernel; O is normalised in fp32 and written as bf16.
#include <math.h>

#include "common.cuh"
#include "gemm.cuh"

namespace svx {
namespace {

constexpr int HD = 96;             // head dim
constexpr int LDS = HD + 8;        // padded smem row (208 B): conflict-free ldmatrix
constexpr int BQ = 128, BKEY = 64;
constexpr int kWarps = 8, kThreads = kWarps * 32;

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  return (uint32_t)f32_to_bf16(lo) | ((uint32_t)f32_to_bf16(hi) << 16);
}

// Load rows [row0, row0+ROWS) x 96 dims of a row-major operand into smem (zero-fill rows >= valid).
template <int ROWS>
__device__ __forceinline__ void load_tile(uint16_t* dst, const uint16_t* src, int64_t row_stride, int row0, int valid) {
  constexpr int CHUNKS = ROWS * (HD / 8);
  for (int c = threadIdx.x; c < CHUNKS; c += kThreads) {
    const int r = c / (HD / 8), k = (c % (HD / 8)) * 8;
    const bool ok = row0 + r < valid;
    const uint16_t* s = src + (int64_t)(ok ? row0 + r : 0) * row_stride + k;
    cp_async16(dst + r * LDS + k, s, ok);
  }
}

__global__ void __launch_bounds__(kThreads) attention_kernel(const uint16_t* __restrict__ q, int64_t q_row_stride,
                                                              const uint16_t* __restrict__ k,
                                                              const uint16_t* __restrict__ v, int64_t kv_slot_stride,
                                                              int64_t kv_head_stride, int64_t kv_row_stride,
                                                              const int32_t* __restrict__ lengths, int heads,
                                                              int queries, int keys, uint16_t* __restrict__ out,
                                                              float scale_log2) {
  extern __shared__ __align__(16) uint16_t sm[];
  uint16_t* sq = sm;                       // [BQ][LDS]
  uint16_t* sk = sq + BQ * LDS;            // [2][BKEY][LDS]
  uint16_t* sv = sk + 2 * BKEY * LDS;      // [2][BKEY][LDS]
  const int slot = blockIdx.z, head = blockIdx.y, q0 = blockIdx.x * BQ;
  const int warp = warp_id(), lane = lane_id();
  const int length = lengths ? min(lengths[slot], keys) : keys;

  const uint16_t* qbase = q + ((int64_t)slot * queries) * q_row_stride + head * HD;
  const uint16_t* kbase = k + slot * kv_slot_stride + head * kv_head_stride;
  const uint16_t* vbase = v + slot * kv_slot_stride + head * kv_head_stride;
  const int tiles = (length + BKEY - 1) / BKEY;

  load_tile<BQ>(sq, qbase, q_row_stride, q0, queries);
  if (tiles > 0) {
    load_tile<BKEY>(sk, kbase, kv_row_stride, 0, length);
    load_tile<BKEY>(sv, vbase, kv_row_stride, 0, length);
  }
  cp_commit();

  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  uint32_t qa[HD / 16][4];

  for (int t = 0; t < tiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < tiles) {
      load_tile<BKEY>(sk + (buf ^ 1) * BKEY * LDS, kbase, kv_row_stride, (t + 1) * BKEY, length);
      load_tile<BKEY>(sv + (buf ^ 1) * BKEY * LDS, vbase, kv_row_stride, (t + 1) * BKEY, length);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (t == 0) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk)
        ldsm_x4(qa[kk], sq + (warp * 16 + (lane & 15)) * LDS + kk * 16 + (lane >> 4) * 8);
    }
    const uint16_t* kt = sk + buf * BKEY * LDS;
    const uint16_t* vt = sv + buf * BKEY * LDS;
    // S = Q K^T for this warp's 16 rows x 64 keys.
    float s[BKEY / 8][4];
#pragma unroll
    for (int j = 0; j < BKEY / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int j = 0; j < BKEY / 8; j += 2) {
        uint32_t b[4];
        const int mi = lane >> 3;
        ldsm_x4(b, kt + (j * 8 + (mi >> 1) * 8 + (lane & 7)) * LDS + kk * 16 + (mi & 1) * 8);
        mma_bf16(s[j], qa[kk], b[0], b[1]);
        mma_bf16(s[j + 1], qa[kk], b[2], b[3]);
      }
    }
    // Mask keys past the slot length, then the online softmax update (log2 domain).
    const int key0 = t * BKEY;
#pragma unroll
    for (int j = 0; j < BKEY / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + j * 8 + (lane & 3) * 2 + (e & 1);
        s[j][e] = key < length ? s[j][e] * scale_log2 : -INFINITY;
      }
    }
    float mx[2] = {m[0], m[1]};
#pragma unroll
    for (int j = 0; j < BKEY / 8; ++j) {
      mx[0] = fmaxf(mx[0], fmaxf(s[j][0], s[j][1]));
      mx[1] = fmaxf(mx[1], fmaxf(s[j][2], s[j][3]));
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      alpha[r] = exp2f(m[r] - mx[r]);  // m = -inf on the first tile: alpha = 0
      m[r] = mx[r];
    }
    uint32_t pa[BKEY / 16][4];
#pragma unroll
    for (int j = 0; j < BKEY / 8; ++j) {
      const float p0 = exp2f(s[j][0] - m[0]), p1 = exp2f(s[j][1] - m[0]);
      const float p2 = exp2f(s[j][2] - m[1]), p3 = exp2f(s[j][3] - m[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      pa[j >> 1][(j & 1) * 2 + 0] = pack_bf16(p0, p1);
      pa[j >> 1][(j & 1) * 2 + 1] = pack_bf16(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l[r] = l[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= alpha[0]; o[i][1] *= alpha[0];
      o[i][2] *= alpha[1]; o[i][3] *= alpha[1];
    }
    // O += P V: the A fragments of P are the S accumulators of key columns 16c..16c+15.
#pragma unroll
    for (int c = 0; c < BKEY / 16; ++c) {
#pragma unroll
      for (int i = 0; i < HD / 8; i += 2) {
        uint32_t b[4];
        const int mi = lane >> 3;
        ldsm_x4_t(b, vt + (c * 16 + (mi & 1) * 8 + (lane & 7)) * LDS + i * 8 + (mi >> 1) * 8);
        mma_bf16(o[i], pa[c], b[0], b[1]);
        mma_bf16(o[i + 1], pa[c], b[2], b[3]);
      }
    }
    __syncthreads();
  }
  cp_wait<0>();
  // Normalise and store: rows g and g+8 of the warp, dims i*8 + 2*(lane&3) + {0,1}.
  const int g = lane >> 2;
  const float inv0 = l[0] > 0.f ? 1.f / l[0] : 0.f, inv1 = l[1] > 0.f ? 1.f / l[1] : 0.f;
  const int row0 = q0 + warp * 16 + g;
  uint16_t* out0 = out + ((int64_t)slot * queries + row0) * (heads * HD) + head * HD;
  uint16_t* out1 = out0 + 8 * (int64_t)(heads * HD);
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) {
    const int d = i * 8 + (lane & 3) * 2;
    if (row0 < queries) *reinterpret_cast<uint32_t*>(out0 + d) = pack_bf16(o[i][0] * inv0, o[i][1] * inv0);
    if (row0 + 8 < queries) *reinterpret_cast<uint32_t*>(out1 + d) = pack_bf16(o[i][2] * inv1, o[i][3] * inv1);
  }
}

constexpr size_t kSmem = (size_t)(BQ + 4 * BKEY) * LDS * sizeof(uint16_t);

}  // namespace

int attention_run(const uint16_t* q, int64_t q_row_stride, const uint16_t* k, const uint16_t* v,
                  int64_t kv_slot_stride, int64_t kv_head_stride, int64_t kv_row_stride, const int32_t* lengths,
                  int slots, int heads, int queries, int keys, uint16_t* out, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    SVX_CHECK_CUDA(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
    configured = true;
  }
  dim3 grid((queries + BQ - 1) / BQ, heads, slots);
  const float scale_log2 = (1.0f / sqrtf((float)HD)) * 1.4426950408889634f;
  attention_kernel<<<grid, kThreads, kSmem, stream>>>(q, q_row_stride, k, v, kv_slot_stride, kv_head_stride,
                                                      kv_row_stride, lengths, heads, queries, keys, out, scale_log2);
  return launch_status("attention_kernel");
}

}  // namespace svx

using namespace svx;

extern "C" int svx_attention(const uint16_t* q, int64_t q_row_stride, const uint16_t* k, const uint16_t* v,
                             int64_t kv_slot_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                             const int32_t* lengths, int slots, int heads, int queries, int keys, uint16_t* out,
                             void* stream) {
  SVX_REQUIRE(q && k && v && out && slots > 0 && heads > 0 && queries > 0 && keys > 0, "svx_attention: bad arguments");
  SVX_REQUIRE(q_row_stride % 8 == 0 && kv_row_stride % 8 == 0 && kv_head_stride % 8 == 0 && kv_slot_stride % 8 == 0,
              "svx_attention: strides must be multiples of 8 elements");
  const uintptr_t align = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                          reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
  SVX_REQUIRE((align & 15u) == 0, "svx_attention: operands must be 16-byte aligned");
  return attention_run(q, q_row_stride, k, v, kv_slot_stride, kv_head_stride, kv_row_stride, lengths, slots, heads,
                       queries, keys, out, as_stream(stream));
}
