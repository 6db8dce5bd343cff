// Non-causal attention, head_dim 96, over per-slot variable-length keys, on the 5th-generation tensor cores.
//
// One CTA = 128 queries of one (slot, head). Key tiles of 128 are streamed by TMA (two 64-dim 128B-swizzled boxes per
// operand; the tensor maps' inner extent is 96, so dims 96..127 of a box read as zero and cost no DRAM traffic) into a
// two-stage ring, and only the ceil(length / 128) tiles of a slot are loaded: the packed-key block mask of
// `streamvoxel/stream/fast_ops.py:149-159`.
//
// Warp roles (256 threads): warp 0 loads Q and the K ring, warp 2 the V ring (TMA); warp 1 owns TMEM and one thread
// issues tcgen05.mma:
//   S(t) = Q K(t)^T    M=128, N=128, K=96  -> TMEM columns [128 (t%2), +128)   (double buffered)
//   O   += P(t) V(t)   M=128, N=96,  K=128 -> TMEM columns [256, 352)           (V read MN-major)
// Warps 4-7 are the softmax warps, one query row per thread (TMEM lane): each reads its row of S(t) once with
// tcgen05.ld, frees the S buffer, and writes P(t) = 2^(S*scale - m) as bf16 into a 128B-swizzled K-major tile in shared
// memory (the A operand of the P.V product). The exponent base m is raised lazily: only when a row's max grows by more
// than 8 (a factor 256, so P <= 256 stays exact in the fp32 sums), and then the warp rescales its O rows and running
// sums in TMEM/registers after the previous P.V has completed -- exact, since P, O and the sum always share one m.
// S(t+1) runs on the tensor core while the softmax of S(t) runs. P is rounded to bf16 before P.V and the row sums stay
// fp32, as in SDPA's flash kernels; the output is normalised in fp32 and written as bf16.
// Every mbarrier wait is bounded (tc::wait); a timeout raises a CTA-wide abort, sets SVX_STATUS_WAIT_TIMEOUT in the
// library's timeout word and skips the rest of the CTA's work.
#include <math.h>

#include "common.cuh"
#include "gemm.cuh"
#include "tc.cuh"

namespace svx {

__device__ uint32_t g_svx_attention_timeouts = 0;

namespace {

constexpr int TQ = 128, TK = 128, HD = 96;
constexpr uint32_t ATOM = 128 * 128;  // one 128-row x 128 B swizzle atom column block (16 KB)
constexpr uint32_t TILE = 2 * ATOM;   // a 128 x 128 bf16 operand tile (dims or keys 0-63, 64-127)
constexpr uint32_t TMEM_COLS = 512;
constexpr int kThreads = 256;
constexpr size_t kSmem = 1024 + TILE + 2 * TILE + 2 * TILE + 2 * TILE + 18 * 8 + 16;

struct AttnParams {
  int heads, queries, keys, kv_mode;  // kv_mode 0: K/V groups = heads, rows = slot*keys + key; 1: groups = slot*heads + head
  const int32_t* lengths;
  uint16_t* out;
  float scale_log2;
};

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  return (uint32_t)f32_to_bf16(lo) | ((uint32_t)f32_to_bf16(hi) << 16);
}

__global__ void __launch_bounds__(kThreads, 1) attention_tc_kernel(const __grid_constant__ CUtensorMap mq,
                                                                   const __grid_constant__ CUtensorMap mk,
                                                                   const __grid_constant__ CUtensorMap mv,
                                                                   const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* sk = sq + TILE;                 // K ring (2 tiles)
  uint8_t* sv = sk + 2 * TILE;             // V ring (2 tiles)
  uint8_t* sp = sv + 2 * TILE;             // P buffers (2 tiles)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sp + 2 * TILE);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 3;
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 7;
  uint64_t* s_full = bars + 9;
  uint64_t* s_free = bars + 11;
  uint64_t* p_full = bars + 13;
  uint64_t* o_full = bars + 15;   // P.V of the tile in P buffer b has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = warp_id(), lane = lane_id();
  const int slot = blockIdx.z, head = blockIdx.y, q0 = blockIdx.x * TQ;
  const int length = p.lengths ? min(p.lengths[slot], p.keys) : p.keys;
  const int tiles = (length + TK - 1) / TK;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(k_full + i, 1); mbar_init(k_empty + i, 1);
      mbar_init(v_full + i, 1); mbar_init(v_empty + i, 1);
      mbar_init(s_full + i, 1); mbar_init(s_free + i, 128);
      mbar_init(p_full + i, 128); mbar_init(o_full + i, 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc::prefetch_map(&mq); tc::prefetch_map(&mk); tc::prefetch_map(&mv);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, TMEM_COLS);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_o = tmem + 256;
  const int kg = p.kv_mode == 0 ? head : slot * p.heads + head;
  const int kr0 = p.kv_mode == 0 ? slot * p.keys : 0;

  if (warp == 0) {
    if (lane == 0 && tiles > 0) {
      const int qr = slot * p.queries + q0;
      mbar_expect_tx(q_full, TILE);
      tc::tma_load_3d(sq, &mq, 0, head, qr, q_full);
      tc::tma_load_3d(sq + ATOM, &mq, 64, head, qr, q_full);
      for (int t = 0; t < tiles; ++t) {
        const int s = t & 1;
        if (t >= 2 && !tc::wait(k_empty + s, ((t - 2) >> 1) & 1, abort_flag)) break;
        mbar_expect_tx(k_full + s, TILE);
        tc::tma_load_3d(sk + s * TILE, &mk, 0, kg, kr0 + t * TK, k_full + s);
        tc::tma_load_3d(sk + s * TILE + ATOM, &mk, 64, kg, kr0 + t * TK, k_full + s);
      }
    }
  } else if (warp == 2) {
    if (lane == 0 && tiles > 0) {
      for (int t = 0; t < tiles; ++t) {
        const int s = t & 1;
        if (t >= 2 && !tc::wait(v_empty + s, ((t - 2) >> 1) & 1, abort_flag)) break;
        mbar_expect_tx(v_full + s, TILE);
        tc::tma_load_3d(sv + s * TILE, &mv, 0, kg, kr0 + t * TK, v_full + s);
        tc::tma_load_3d(sv + s * TILE + ATOM, &mv, 64, kg, kr0 + t * TK, v_full + s);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && tiles > 0) {
      constexpr uint32_t idesc_s = tc::instr_desc(TQ, TK, false);
      constexpr uint32_t idesc_o = tc::instr_desc(TQ, HD, true);
      bool ok = tc::wait(q_full, 0, abort_flag);
      const uint32_t qa = smem_addr(sq);
      for (int t = 0; ok && t <= tiles; ++t) {
        if (t < tiles) {
          const int s = t & 1;
          ok = tc::wait(k_full + s, (t >> 1) & 1, abort_flag);
          if (ok && t >= 2) ok = tc::wait(s_free + s, ((t - 2) >> 1) & 1, abort_flag);
          if (!ok) break;
          tc::fence_after();
          const uint32_t kb = smem_addr(sk + s * TILE);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * ATOM + (kk & 3) * 32;
            tc::umma(tmem + s * 128, tc::sw128_desc(qa + off), tc::sw128_desc(kb + off), idesc_s, kk > 0);
          }
          tc::commit(s_full + s);
          tc::commit(k_empty + s);
        }
        if (t >= 1) {
          const int u = t - 1, su = u & 1;
          ok = tc::wait(v_full + su, (u >> 1) & 1, abort_flag);
          if (ok) ok = tc::wait(p_full + su, (u >> 1) & 1, abort_flag);
          if (!ok) break;
          tc::fence_after();
          const uint32_t pa = smem_addr(sp + su * TILE), vb = smem_addr(sv + su * TILE);
#pragma unroll
          for (int kk = 0; kk < TK / 16; ++kk) {
            const uint32_t aoff = (kk >> 2) * ATOM + (kk & 3) * 32;
            tc::umma(tmem_o, tc::sw128_desc(pa + aoff), tc::sw128_desc(vb + kk * 2048, ATOM, 1024), idesc_o,
                     (u > 0 || kk > 0) ? 1u : 0u);
          }
          tc::commit(o_full + su);
          tc::commit(v_empty + su);
        }
      }
    }
  } else if (warp >= 4) {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    const float sl2 = p.scale_log2;
    float m_used = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int t = 0; t < tiles; ++t) {
      const int s = t & 1;
      if (!tc::wait(s_full + s, (t >> 1) & 1, abort_flag)) { ok = false; break; }
      tc::fence_after();
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::ld32(tmem + lanes + s * 128 + c * 32, r[c]);
      tc::wait_ld();
      tc::fence_before();
      tc::mbar_arrive(s_free + s);
      const int key0 = t * TK;
      const bool full = key0 + TK <= length;
      if (!full) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (key0 + c * 32 + j >= length) r[c][j] = __float_as_uint(-INFINITY);
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int j = 0; j < 32; ++j) mx = fmaxf(mx, __uint_as_float(r[c][j]));
      mx *= sl2;
      // Raise the exponent base only when the row max outgrows it by more than 8 (warp-uniform rescale of O).
      const bool raise = mx > m_used + 8.f;
      if (__any_sync(0xffffffffu, raise)) {
        const float m_new = raise ? mx : m_used;
        const float alpha = tc::ex2(m_used - m_new);   // m_used = -inf on the first tile: alpha = 0
        l_run *= alpha;
        m_used = m_new;
        if (t >= 1) {
          // O holds the P.V products of tiles < t; the last one (t-1) must have completed.
          const int u = t - 1;
          if (!tc::wait(o_full + (u & 1), (u >> 1) & 1, abort_flag)) { ok = false; break; }
          tc::fence_after();
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            tc::ld32(tmem_o + lanes + c * 32, o);
            tc::wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
            tc::st32(tmem_o + lanes + c * 32, o);
          }
          tc::wait_st();
        }
      }
      // P buffer s was last read by the P.V of tile t-2.
      if (t >= 2 && !tc::wait(o_full + s, ((t - 2) >> 1) & 1, abort_flag)) { ok = false; break; }
      const float base = m_used;
      float sum = 0.f;
      uint8_t* pb = sp + s * TILE;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float p0 = tc::ex2(__uint_as_float(r[c][j]) * sl2 - base);
          const float p1 = tc::ex2(__uint_as_float(r[c][j + 1]) * sl2 - base);
          sum += p0 + p1;
          packed[j >> 1] = pack_bf16(p0, p1);
        }
        // keys c*32 .. c*32+31: swizzle atom c/2, 16-byte chunks (c%2)*4 .. +3, chunk index XOR (row % 8)
        uint8_t* rowp = pb + (c >> 1) * ATOM + row * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = ((c & 1) * 4 + q) ^ (row & 7);
          *reinterpret_cast<uint4*>(rowp + chunk * 16) =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
      }
      l_run += sum;
      tc::fence_before();
      tc::fence_async_smem();
      tc::mbar_arrive(p_full + s);
    }
    const int qrow = q0 + row;
    if (ok && tiles > 0) {
      const int u = tiles - 1;
      ok = tc::wait(o_full + (u & 1), (u >> 1) & 1, abort_flag);
      if (ok) {
        tc::fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(p.out + ((int64_t)slot * p.queries + qrow) * (p.heads * HD) + head * HD);
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tc::ld32(tmem_o + lanes + c * 32, o);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float* f = reinterpret_cast<const float*>(o) + 8 * i;
            dst[c * 4 + i] = make_uint4(pack_bf16(f[0] * inv, f[1] * inv), pack_bf16(f[2] * inv, f[3] * inv),
                                        pack_bf16(f[4] * inv, f[5] * inv), pack_bf16(f[6] * inv, f[7] * inv));
          }
        }
      }
    } else if (ok && qrow < p.queries) {
      uint4* dst = reinterpret_cast<uint4*>(p.out + ((int64_t)slot * p.queries + qrow) * (p.heads * HD) + head * HD);
      for (int i = 0; i < HD / 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
    }
    if (!ok && lane == 0) atomicOr(&g_svx_attention_timeouts, SVX_STATUS_WAIT_TIMEOUT);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

int attention_run(const uint16_t* q, int64_t q_row_stride, const uint16_t* k, const uint16_t* v,
                  int64_t kv_slot_stride, int64_t kv_head_stride, int64_t kv_row_stride, const int32_t* lengths,
                  int slots, int heads, int queries, int keys, uint16_t* out, cudaStream_t stream) {
  SVX_REQUIRE(queries % TQ == 0, "attention: queries must be a multiple of 128");
  int kv_mode;
  uint64_t groups, rows, group_stride, row_stride;
  if (kv_slot_stride == (int64_t)keys * kv_row_stride) {          // [slot*keys + key][.. head*stride ..]
    kv_mode = 0; groups = heads; rows = (uint64_t)slots * keys;
    group_stride = kv_head_stride * 2; row_stride = kv_row_stride * 2;
  } else if (kv_slot_stride == (int64_t)heads * kv_head_stride) {  // [slot][head][key][dim]
    kv_mode = 1; groups = (uint64_t)slots * heads; rows = keys;
    group_stride = kv_head_stride * 2; row_stride = kv_row_stride * 2;
  } else {
    return fail(SVX_ERR_INVALID, "attention: K/V strides must be [slot*keys][head] or [slot][head][key] layouts");
  }
  CUtensorMap mq, mk, mv;
  int rc = make_map_3d(&mq, q, HD, heads, (uint64_t)slots * queries, HD * 2, q_row_stride * 2, 64, TQ);
  if (!rc) rc = make_map_3d(&mk, k, HD, groups, rows, group_stride, row_stride, 64, TK);
  if (!rc) rc = make_map_3d(&mv, v, HD, groups, rows, group_stride, row_stride, 64, TK);
  if (rc) return rc;
  static bool configured = false;
  if (!configured) {
    SVX_CHECK_CUDA(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
    configured = true;
  }
  AttnParams prm{heads, queries, keys, kv_mode, lengths, out, (1.0f / sqrtf((float)HD)) * 1.4426950408889634f};
  dim3 grid(queries / TQ, heads, slots);
  attention_tc_kernel<<<grid, kThreads, kSmem, stream>>>(mq, mk, mv, prm);
  return launch_status("attention_tc_kernel");
}

uint32_t attention_timeouts() {
  uint32_t v = 0;
  if (cudaMemcpyFromSymbol(&v, g_svx_attention_timeouts, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  return v;
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
