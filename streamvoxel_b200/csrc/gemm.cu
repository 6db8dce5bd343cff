// Dense bf16 GEMM with fused epilogues on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA.
//
// D[M,N] = A[M,K] . W[N,K]^T, both operands K-major (activations row-major, nn.Linear weights as stored).
// Persistent: one CTA per SM walks the 128 x BN output tiles round-robin. Warp 0 streams A/W k-blocks through a
// STAGES-deep ring of 128B-swizzled shared-memory tiles that runs continuously across tiles; warp 1 owns TMEM and one
// elected thread issues tcgen05.mma (M=128, N=BN, K=16) into one of two TMEM accumulators (2 x BN fp32 columns),
// committing each stage back to the producer and each finished tile to the epilogue; warps 4-19 are the epilogue:
// four warps per 32-lane TMEM quarter (32-column chunks dealt round-robin) read the accumulator with tcgen05.ld, run
// the fused epilogue (paired fp32 arithmetic, one bf16x2 conversion per pair) and release the accumulator, so the
// epilogue of tile i overlaps the main loop of tile i+1. Every warp runs on the launch's 96 registers: ptxas compiles
// each role within them regardless of setmaxnreg, and a decrease in the producer branch only made it spill.
// Every mbarrier wait is bounded; a timeout sets SVX_STATUS_WAIT_TIMEOUT in g_svx_timeouts and skips the work.
#include <cuda.h>
#include <math.h>

#include "common.cuh"
#include "gemm.cuh"
#include "tc.cuh"

namespace svx {

__device__ uint32_t g_svx_timeouts = 0;

namespace {

constexpr int BM = 128, BK = 64;
constexpr int kThreads = 640;  // warps 0-1 producer/MMA, 2-3 idle, 4-19 epilogue
constexpr int kEpilogueWarps = 16;
constexpr uint32_t A_BYTES = BM * BK * 2;
// Kernel variants: the epilogue (svx_epilogue, bits 0-2) | kFold (LayerNorm folded into this GEMM's epilogue) |
// kStats (row statistics for the next LayerNorm written by this epilogue) | kGroup (two independent problems of the
// same shape in one launch: the second problem's tiles follow the first's, with their own operands and epilogue).
constexpr int kFold = 8, kStats = 16, kGroup = 32;

__device__ __forceinline__ void record_timeout() { atomicOr(&g_svx_timeouts, SVX_STATUS_WAIT_TIMEOUT); }

__device__ __forceinline__ float2 unpack2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// Round a pair to bf16 (nearest-even) and back to fp32.
__device__ __forceinline__ float2 round2(float2 v) { return unpack2(tc::pack_bf16x2(v.x, v.y)); }

__device__ __forceinline__ void store_bf16x32(uint16_t* p, const float (&v)[32]) {
  uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    q[i] = make_uint4(tc::pack_bf16x2(v[8 * i], v[8 * i + 1]), tc::pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                      tc::pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), tc::pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU (erf form) of a pair, x * 0.5 * (1 + erf(x / sqrt 2)), with erf from Abramowitz & Stegun 7.1.28
// (|error| <= 3e-7): for a = |x| / sqrt 2, erf(a) = 1 - 1 / p^16 with p = 1 + c1 a + ... + c6 a^6, so
// erfc(a) = 1 / p^16 (four squarings and one reciprocal; p^16 overflows to inf, and erfc to 0, beyond a ~ 12), and
// 1 + erf = 2 - erfc for x >= 0, erfc for x < 0. Branch-free, one MUFU operation per value (7.1.26 takes a reciprocal
// and an exponential, and the fc1 epilogue is bound by that pipe). Its bf16 outputs equal ATen's erff-based GELU for
// x >= -3 (checked on 4M bf16 inputs); below, where |GELU| < 4e-3, they differ by at most 1.6e-5.
__device__ __forceinline__ float2 gelu_erf2(float2 x) {
  constexpr float c1 = 0.0705230784f, c2 = 0.0422820123f, c3 = 0.0092705272f, c4 = 0.0001520143f,
                  c5 = 0.0002765672f, c6 = 0.0000430638f;
  constexpr float rs2 = 0.70710678118654752440f;
  const float2 a = __fmul2_rn(make_float2(fabsf(x.x), fabsf(x.y)), make_float2(rs2, rs2));
  float2 p = __ffma2_rn(make_float2(c6, c6), a, make_float2(c5, c5));
  p = __ffma2_rn(p, a, make_float2(c4, c4));
  p = __ffma2_rn(p, a, make_float2(c3, c3));
  p = __ffma2_rn(p, a, make_float2(c2, c2));
  p = __ffma2_rn(p, a, make_float2(c1, c1));
  p = __ffma2_rn(p, a, make_float2(1.f, 1.f));
  p = __fmul2_rn(p, p);
  p = __fmul2_rn(p, p);
  p = __fmul2_rn(p, p);
  p = __fmul2_rn(p, p);
  const float2 erfc = make_float2(rcp_approx(p.x), rcp_approx(p.y));
  const float2 h = __fmul2_rn(__fmul2_rn(x, make_float2(0.5f, 0.5f)), erfc);
  return make_float2(x.x >= 0.f ? x.x - h.x : h.x, x.y >= 0.f ? x.y - h.y : h.y);
}

__device__ __forceinline__ void unpack8(uint4 raw, float* v) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = unpack2(w[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

// Operands an epilogue chunk reads from global memory, fetched before the accumulator is ready (bf16, packed).
struct Operands {
  uint4 bias[4];
  uint4 extra[4];   // gate (GATE_RESIDUAL) | sin, cos (ROPE: 2 + 2)
  uint4 res[4];     // residual row slice (GATE_RESIDUAL, RESIDUAL)
  float u, v;       // LayerNorm fold: u[n + lane], v[n + lane], staged through shared memory for the whole warp
};

// GLOBAL_RES = false: the residual comes from a staging box in shared memory instead.
template <int E, bool GLOBAL_RES = true>
__device__ __forceinline__ void prefetch32(const EpiParams& ep, int N, int row, int n, Operands& o) {
  constexpr int EPI = E & 7;
  [[maybe_unused]] constexpr bool LN_FOLD = (E & kFold) != 0, LN_STATS = (E & kStats) != 0;
  if constexpr (LN_FOLD) {   // this lane's u and v in place of the bias, which v holds
    o.u = __ldg(ep.ln_u + n + lane_id());
    o.v = __ldg(ep.ln_v + n + lane_id());
  } else {
    const uint4* b = reinterpret_cast<const uint4*>(ep.bias + n);
#pragma unroll
    for (int i = 0; i < 4; ++i) o.bias[i] = b[i];
  }
  if constexpr (EPI == SVX_EPI_GATE_RESIDUAL) {
    const uint4* g = reinterpret_cast<const uint4*>(ep.gate + n);
#pragma unroll
    for (int i = 0; i < 4; ++i) o.extra[i] = g[i];
  }
  if constexpr ((EPI == SVX_EPI_GATE_RESIDUAL || EPI == SVX_EPI_RESIDUAL) && GLOBAL_RES) {
    const uint4* r = reinterpret_cast<const uint4*>(ep.residual + (int64_t)row * N + n);
#pragma unroll
    for (int i = 0; i < 4; ++i) o.res[i] = r[i];
  }
  if constexpr (EPI == SVX_EPI_ROPE) {
    if (n < ep.rope_cols) {
      const int p = row % ep.rows_per_slot;
      const int half = ep.head_dim >> 1;
      const int64_t t = (int64_t)p * half + ((n % ep.head_dim) >> 1);   // 16 consecutive table entries, 16-byte aligned
      const uint4* sn = reinterpret_cast<const uint4*>(ep.rope_sin + t);
      const uint4* cs = reinterpret_cast<const uint4*>(ep.rope_cos + t);
      o.extra[0] = sn[0]; o.extra[1] = sn[1]; o.extra[2] = cs[0]; o.extra[3] = cs[1];
    }
  }
}

// Mean and 1/sqrt(var + eps) of a row from its 32-column chunk statistics (var: the biased variance of layer_norm).
// Shifted sums about the first chunk's mean m0 (no division, and no cancellation when |mean| >> std):
// mean = m0 + sum_c d_c / C and var = sum_c (M2_c + 32 d_c^2) / (32 C) - (sum_c d_c / C)^2 with d_c = mean_c - m0.
// Statistics are chunk-major ([chunk][M]), so a warp's 32 consecutive rows read one 256-byte run per chunk; 12
// chunks are loaded together so that their latencies overlap.
__device__ __forceinline__ float2 row_norm(const EpiParams& ep, int row, int M) {
  const float2* st = ep.ln_stats_in + row;
  const float m0 = __ldg(st).x;
  float s1 = 0.f, s2 = 0.f;
  for (int c0 = 0; c0 < ep.ln_chunks; c0 += 12) {
    float2 q[12];
#pragma unroll
    for (int i = 0; i < 12; ++i)
      q[i] = c0 + i < ep.ln_chunks ? __ldg(st + (int64_t)(c0 + i) * M) : make_float2(m0, 0.f);
#pragma unroll
    for (int i = 0; i < 12; ++i) {
      const float d = q[i].x - m0;
      s1 += d;
      s2 += fmaf(32.f * d, d, q[i].y);
    }
  }
  const float dm = s1 * ep.ln_inv_chunks;
  const float var = fmaxf(fmaf(-dm, dm, s2 * ep.ln_inv_chunks * (1.f / 32.f)), 0.f);
  return make_float2(m0 + dm, rsqrtf(var + ep.ln_eps));
}

// (mean, M2) of the 32 bf16 values a thread stores for its row: the statistics of the next LayerNorm.
__device__ __forceinline__ void chunk_stats(const EpiParams& ep, int M, int row, int n, const float (&y)[32]) {
  float r[32];
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float2 q = round2(make_float2(y[j], y[j + 1]));
    r[j] = q.x;
    r[j + 1] = q.y;
  }
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) sum += r[j];
  const float mean = sum * (1.f / 32.f);
  float m2 = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float d = r[j] - mean;
    m2 = fmaf(d, d, m2);
  }
  ep.ln_stats_out[(int64_t)(n / 32) * M + row] = make_float2(mean, m2);   // chunk-major [N / 32][M]
}

// The same statistics from the 16 packed bf16 pairs the epilogue stores (unpacking is exact and takes no conversion).
__device__ __forceinline__ void chunk_stats_packed(const EpiParams& ep, int M, int row, int n,
                                                   const uint32_t (&pk)[16]) {
  float2 s = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 16; ++j) s = __fadd2_rn(s, unpack2(pk[j]));
  const float mean = (s.x + s.y) * (1.f / 32.f);
  const float2 nm = make_float2(-mean, -mean);
  float2 m2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float2 d = __fadd2_rn(unpack2(pk[j]), nm);
    m2 = __ffma2_rn(d, d, m2);
  }
  ep.ln_stats_out[(int64_t)(n / 32) * M + row] = make_float2(mean, m2.x + m2.y);
}

// Epilogue arithmetic of one row x 32 columns [n, n+32) of the tile; acc holds fp32 accumulators, o the bias, gate,
// RoPE table and residual words of the row; nr the row's (mean, 1/std) when the LayerNorm is folded in.
// uv: the warp's 32 u then 32 v values of this chunk in shared memory (LayerNorm fold; nullptr: read them from
// global memory).
template <int E>
__device__ __forceinline__ void epilogue_math(const EpiParams& ep, int row, int n, const uint32_t (&acc)[32],
                                              const Operands& o, float2 nr, float (&y)[32],
                                              const float* uv = nullptr) {
  constexpr int EPI = E & 7;
  [[maybe_unused]] constexpr bool LN_FOLD = (E & kFold) != 0, LN_STATS = (E & kStats) != 0;
  if constexpr (LN_FOLD) {
    const float2 ra = make_float2(nr.y, nr.y), rb = make_float2(-nr.x * nr.y, -nr.x * nr.y);
    const float4* up = reinterpret_cast<const float4*>(uv ? uv : ep.ln_u + n);
    const float4* vp = reinterpret_cast<const float4*>(uv ? uv + 32 : ep.ln_v + n);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 uq = up[q], vq = vp[q];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = 2 * q + h;
        const float2 u2 = h ? make_float2(uq.z, uq.w) : make_float2(uq.x, uq.y);
        const float2 v2 = h ? make_float2(vq.z, vq.w) : make_float2(vq.x, vq.y);
        const float2 a = make_float2(__uint_as_float(acc[2 * j]), __uint_as_float(acc[2 * j + 1]));
        const float2 v = round2(__ffma2_rn(a, ra, __ffma2_rn(rb, u2, v2)));
        y[2 * j] = v.x;
        y[2 * j + 1] = v.y;
      }
    }
  } else {
    const uint32_t* bw = reinterpret_cast<const uint32_t*>(o.bias);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float2 v = round2(__fadd2_rn(make_float2(__uint_as_float(acc[2 * j]), __uint_as_float(acc[2 * j + 1])),
                                         unpack2(bw[j])));
      y[2 * j] = v.x;
      y[2 * j + 1] = v.y;
    }
  }
  if constexpr (EPI == SVX_EPI_BIAS_GELU) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float2 g = gelu_erf2(make_float2(y[2 * j], y[2 * j + 1]));
      y[2 * j] = g.x;
      y[2 * j + 1] = g.y;
    }
  } else if constexpr (EPI == SVX_EPI_GATE_RESIDUAL || EPI == SVX_EPI_RESIDUAL) {
    const uint32_t* rw = reinterpret_cast<const uint32_t*>(o.res);
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(o.extra);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float2 v = make_float2(y[2 * j], y[2 * j + 1]);
      if constexpr (EPI == SVX_EPI_GATE_RESIDUAL) v = round2(__fmul2_rn(unpack2(gw[j]), v));
      v = __fadd2_rn(unpack2(rw[j]), v);
      y[2 * j] = v.x;
      y[2 * j + 1] = v.y;
    }
  } else if constexpr (EPI == SVX_EPI_ROPE) {
    if (n < ep.rope_cols) {
      // Axial RoPE (`unconditional_md4_timefree.py:24-30`): pair (2f, 2f+1) of a head rotates by table entry f;
      // a*cos, b*sin, ... are bf16 ops, so every product and sum rounds to bf16.
      float sn[16], cs[16];
      unpack8(o.extra[0], sn); unpack8(o.extra[1], sn + 8);
      unpack8(o.extra[2], cs); unpack8(o.extra[3], cs + 8);
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float sv = sn[j >> 1], cv = cs[j >> 1];
        const float a = y[j], b = y[j + 1];
        // (a cos, a sin) and (b sin, b cos), each product rounded, then a cos - b sin and a sin + b cos rounded:
        // three paired conversions instead of six single ones (qkv launch 31.1 -> 27.1 us on B200).
        const float2 pa = round2(__fmul2_rn(make_float2(a, a), make_float2(cv, sv)));
        const float2 pb = round2(__fmul2_rn(make_float2(b, b), make_float2(sv, cv)));
        const float2 r = round2(__fadd2_rn(pa, make_float2(-pb.x, pb.y)));
        y[j] = r.x;
        y[j + 1] = r.y;
      }
    }
  }
}

// Epilogue of one row x 32 columns [n, n+32) of the tile, stored straight to global memory.
template <int E>
__device__ __forceinline__ void epilogue32(const EpiParams& ep, uint16_t* out, int M, int N, int row, int n,
                                           const uint32_t (&acc)[32], const Operands& o, float2 nr,
                                           const float* uv = nullptr) {
  constexpr int EPI = E & 7;
  [[maybe_unused]] constexpr bool LN_FOLD = (E & kFold) != 0, LN_STATS = (E & kStats) != 0;
  float y[32];
  epilogue_math<E>(ep, row, n, acc, o, nr, y, uv);
  if constexpr (LN_STATS && EPI != SVX_EPI_CLASS_MAJOR) chunk_stats(ep, M, row, n, y);
  if constexpr (EPI == SVX_EPI_CLASS_MAJOR) {
    // W rows are ordered n = v * 64 + o, so the 32 columns are one class v and offsets o..o+31 of one patch.
    constexpr int P = 4, P3 = 64;
    const int v = n / P3, o0 = n % P3;
    const int slot = row / ep.rows_per_slot, p = row % ep.rows_per_slot;
    const int gz = ep.depth / P, gx = ep.width / P;
    const int py = p / (gz * gx), pz = (p / gx) % gz, px = p % gx;
    uint16_t* base = out + ((int64_t)slot * ep.classes + v) * ((int64_t)ep.height * ep.depth * ep.width);
#pragma unroll
    for (int j = 0; j < 32; j += 4) {  // four consecutive x voxels per 8-byte store
      const int oo = o0 + j;
      const int oy = oo >> 4, oz = (oo >> 2) & 3;
      const int64_t idx = ((int64_t)(py * P + oy) * ep.depth + (pz * P + oz)) * ep.width + px * P;
      *reinterpret_cast<uint2*>(base + idx) =
          make_uint2(tc::pack_bf16x2(y[j], y[j + 1]), tc::pack_bf16x2(y[j + 2], y[j + 3]));
    }
  } else {
    store_bf16x32(out + (int64_t)row * N + n, y);
  }
}

template <int BN, int STAGES, int E>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                           const __grid_constant__ CUtensorMap tmB,
                                                           uint16_t* __restrict__ out, int M, int N, int K,
                                                           const EpiParams ep) {
  [[maybe_unused]] constexpr int EPI = E & 7;
  [[maybe_unused]] constexpr bool LN_FOLD = (E & kFold) != 0, LN_STATS = (E & kStats) != 0;
  constexpr uint32_t B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_s = smem;
  uint8_t* b_s = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(b_s + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = warp_id(), lane = lane_id();
  const int kblocks = K / BK;
  const int n_tiles = N / BN;
  const int tiles = (M / BM) * n_tiles;
  grid_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(acc_full + b, 1); mbar_init(acc_empty + b, kEpilogueWarps); }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc::prefetch_map(&tmA);
    tc::prefetch_map(&tmB);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, TMEM_COLS);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  grid_dependency_wait();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    if (warp == 0 && lane == 0) {
      int it = 0;  // ring position across all tiles of this CTA
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES, round = it / STAGES;
          if (round > 0 && !tc::wait(empty + s, (round - 1) & 1, abort_flag)) { record_timeout(); ok = false; break; }
          mbar_expect_tx(full + s, A_BYTES + B_BYTES);
          tc::tma_load_2d(a_s + s * A_BYTES, &tmA, kb * BK, m0, full + s);
          tc::tma_load_2d(b_s + s * B_BYTES, &tmB, kb * BK, n0, full + s);
        }
      }
    } else if (warp == 1 && lane == 0) {
      constexpr uint32_t idesc = tc::instr_desc(BM, BN);
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++local) {
        const int buf = local & 1, use = local >> 1;
        if (use > 0 && !tc::wait(acc_empty + buf, (use - 1) & 1, abort_flag)) { record_timeout(); break; }
        tc::fence_after();
        const uint32_t acc = tmem + buf * BN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES, round = it / STAGES;
          if (!tc::wait(full + s, round & 1, abort_flag)) { record_timeout(); ok = false; break; }
          tc::fence_after();
          const uint32_t a0 = smem_addr(a_s + s * A_BYTES), b0 = smem_addr(b_s + s * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc::umma(acc, tc::sw128_desc(a0 + kk * 32), tc::sw128_desc(b0 + kk * 32), idesc, (kb | kk) != 0);
          tc::commit(empty + s);
        }
        if (ok) tc::commit(acc_full + buf);
      }
    }
    // Teardown: the TMEM owner frees the columns once all 20 warps are past their last TMEM access.
    tc::fence_before();
    __syncwarp();
    asm volatile("barrier.sync 1, %0;" ::"n"(kThreads) : "memory");
    if (warp == 1) {
      tc::fence_after();
      tc::tmem_dealloc(*tmem_slot, TMEM_COLS);
    }
  } else {
    // Epilogue warps 4..19: TMEM lane quarter (warp % 4) = rows 32*(warp%4) .. +31; 32-column chunks
    // group, group + 4, ... of the tile, group = (warp - 4) / 4.
    const int quarter = warp & 3, group = (warp - 4) >> 2;
    constexpr int CHUNKS = BN / 32;
    int local = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
      const int m0 = (tile / n_tiles) * BM, n0 = (tile % n_tiles) * BN;
      const int buf = local & 1, use = local >> 1;
      const int row = m0 + quarter * 32 + lane;
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * BN);
      // The first chunk's operands are fetched while the main loop still runs.
      float2 nr = make_float2(0.f, 1.f);
      if constexpr (LN_FOLD) {
        if (row < M && group < CHUNKS) nr = row_norm(ep, row, M);
      }
      Operands ops;
      if (group < CHUNKS) prefetch32<E>(ep, N, row, n0 + group * 32, ops);
      if (!tc::wait(acc_full + buf, use & 1, abort_flag)) { record_timeout(); break; }
      tc::fence_after();
#pragma unroll
      for (int c = 0; c < (CHUNKS + 3) / 4; ++c) {
        const int chunk = group + 4 * c;
        if (chunk < CHUNKS) {
          if (c > 0) prefetch32<E>(ep, N, row, n0 + chunk * 32, ops);
          uint32_t acc[32];
          tc::ld32(taddr + chunk * 32, acc);
          tc::wait_ld();
          if (row < M) epilogue32<E>(ep, out, M, N, row, n0 + chunk * 32, acc, ops, nr);
        }
      }
      tc::fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(acc_empty + buf);
    }
    tc::fence_before();
    __syncwarp();
    asm volatile("barrier.arrive 1, %0;" ::"n"(kThreads) : "memory");
  }
}

// CTA-pair variant (cluster of 2, tcgen05 cta_group::2): a pair owns 256 x BN output tiles. CTA r of the pair streams
// rows [128 r, +128) of the A slice and rows [BN/2 r, +BN/2) of the W slice into its own ring, counting both CTAs'
// bytes on the even CTA's full barrier; the even CTA issues M=256 products that read each CTA's A rows and both W
// halves, so every W byte crosses shared memory once per pair (a 128 x BN tile per SM reads 1.5x the operand bytes
// per product, which leaves one SM's tensor core waiting on shared-memory bandwidth). Stage and accumulator
// commits arrive on both CTAs' barriers; each CTA's epilogue reads its own 128 TMEM lanes and releases the
// accumulator on the even CTA's barrier.
// Epilogue through shared memory: each epilogue warp owns two 32 x 32 staging boxes (64B-swizzled, so a row per
// thread reads and writes them without bank conflicts). The residual tile of its chunk is TMA-loaded into the box
// while the main loop still runs; the warp combines it with the accumulator in place and TMA-stores the box, so
// global memory sees whole lines instead of one 16-byte piece per row and instruction. The class-major head keeps
// the direct scatter.
constexpr int PM = 256;
constexpr uint32_t BOX = 32 * 32 * 2;   // one staging box: 32 rows x 32 bf16

template <int BN, int STAGES, int E>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmR,
                     uint16_t* __restrict__ out, int M, int N, int K, const __grid_constant__ EpiParams ep,
                     const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                     const __grid_constant__ CUtensorMap tmO2, const __grid_constant__ CUtensorMap tmR2,
                     const __grid_constant__ EpiParams ep2) {
  constexpr int EPI = E & 7;
  [[maybe_unused]] constexpr bool LN_FOLD = (E & kFold) != 0, LN_STATS = (E & kStats) != 0;
  constexpr bool GROUP = (E & kGroup) != 0;   // tiles [per, 2 per) are the second problem's (tmA2 ... ep2)
  constexpr uint32_t HB_BYTES = (BN / 2) * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256 : 512;   // allocations are powers of two
  constexpr bool STAGED = EPI != SVX_EPI_CLASS_MAJOR;
  constexpr bool RES = EPI == SVX_EPI_GATE_RESIDUAL || EPI == SVX_EPI_RESIDUAL;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_s = smem;
  uint8_t* b_s = smem + STAGES * A_BYTES;
  uint8_t* stage_s = b_s + STAGES * HB_BYTES;                      // 2 boxes per epilogue warp
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_s + kEpilogueWarps * 2 * BOX);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* res_full = acc_empty + 2;                              // per epilogue warp and box
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_full + 2 * kEpilogueWarps);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  float* uv_stage = reinterpret_cast<float*>(tmem_slot + 4);      // LayerNorm fold: 32 u + 32 v per epilogue warp

  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = tc::cluster_rank();
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int kblocks = K / BK;
  const int n_tiles = N / BN;
  const int per = (M / PM) * n_tiles;
  const int tiles = GROUP ? 2 * per : per;
  // Tiles of this pair: round-robin (tile = pair + k * pairs), or, with the LayerNorm fold, a contiguous run, so that
  // consecutive tiles share their rows and the rows' statistics are merged once per row block (same makespan).
  int t_first = pair, t_step = pairs, t_count = tiles > pair ? (tiles - pair + pairs - 1) / pairs : 0;
  if constexpr (LN_FOLD) {
    const int base = tiles / pairs, extra = tiles % pairs;
    t_first = pair * base + min(pair, extra);
    t_step = 1;
    t_count = base + (pair < extra ? 1 : 0);
  }
  grid_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(acc_full + b, 1); mbar_init(acc_empty + b, 2 * kEpilogueWarps); }
    for (int b = 0; b < 2 * kEpilogueWarps; ++b) mbar_init(res_full + b, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc::prefetch_map(&tmA);
    tc::prefetch_map(&tmB);
    if (STAGED) tc::prefetch_map(&tmO);
    if (RES) tc::prefetch_map(&tmR);
    if (GROUP) {
      tc::prefetch_map(&tmA2);
      tc::prefetch_map(&tmB2);
      if (STAGED) tc::prefetch_map(&tmO2);
      if (RES) tc::prefetch_map(&tmR2);
    }
  }
  if (warp == 1) tc::tmem_alloc_pair(tmem_slot, TMEM_COLS);
  tc::fence_before();
  __syncthreads();
  tc::cluster_sync();   // both CTAs' barriers initialised and TMEM allocated before any cross-CTA signal
  tc::fence_after();
  grid_dependency_wait();   // A and the residual come from the previous kernel
  const uint32_t tmem = *tmem_slot;
  const uint32_t full0 = tc::cluster_addr(full, 0);        // the even CTA's full barriers
  const uint32_t acc_empty0 = tc::cluster_addr(acc_empty, 0);

  if (warp < 4) {
    if (warp == 0) {
      int it = 0;
      bool ok = true;
      for (int k = 0; ok && k < t_count; ++k) {
        const int tile = t_first + k * t_step;
        const bool second = GROUP && tile >= per;
        const int lt = second ? tile - per : tile;
        const CUtensorMap* map_a = second ? &tmA2 : &tmA;
        const CUtensorMap* map_b = second ? &tmB2 : &tmB;
        const int m0 = (lt / n_tiles) * PM + (int)rank * BM, n0 = (lt % n_tiles) * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES, round = it / STAGES;
          if (round > 0 && !tc::wait_w(empty + s, (round - 1) & 1, abort_flag)) { record_timeout(); ok = false; break; }
          if (rank == 0) tc::expect_tx_w(full + s, 2 * (A_BYTES + HB_BYTES));
          tc::tma_load_2d_pair_w(a_s + s * A_BYTES, map_a, kb * BK, m0, full0 + 8 * s);
          tc::tma_load_2d_pair_w(b_s + s * HB_BYTES, map_b, kb * BK, n0, full0 + 8 * s);
        }
      }
    } else if (warp == 1 && rank == 0) {
      constexpr uint32_t idesc = tc::instr_desc(PM, BN);
      int it = 0, local = 0;
      bool ok = true;
      for (int k = 0; ok && k < t_count; ++k, ++local) {   // the tiles' order is the producer's; only their count
        const int buf = local & 1, use = local >> 1;
        if (use > 0 && !tc::wait_w(acc_empty + buf, (use - 1) & 1, abort_flag)) { record_timeout(); break; }
        tc::fence_after();
        const uint32_t acc = tmem + buf * BN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES, round = it / STAGES;
          if (!tc::wait_w(full + s, round & 1, abort_flag)) { record_timeout(); ok = false; break; }
          tc::fence_after();
          const uint32_t a0 = smem_addr(a_s + s * A_BYTES), b0 = smem_addr(b_s + s * HB_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc::umma_pair_w(acc, tc::sw128_desc(a0 + kk * 32), tc::sw128_desc(b0 + kk * 32), idesc, (kb | kk) != 0);
          tc::commit_pair_w(empty + s, 0x3);
        }
        if (ok) tc::commit_pair_w(acc_full + buf, 0x3);
      }
    }
    tc::fence_before();
    __syncwarp();
    tc::cluster_sync();   // no cross-CTA signal is pending once every thread of both CTAs is here
    if (warp == 1) {
      tc::fence_after();
      tc::tmem_dealloc_pair(*tmem_slot, TMEM_COLS);
    }
  } else {
    const int quarter = warp & 3, group = (warp - 4) >> 2, ws = warp - 4;
    constexpr int CHUNKS = BN / 32;
    constexpr int MINE = (CHUNKS + 3) / 4;   // 32-column chunks of this warp per tile: group, group + 4
    uint8_t* wbox = stage_s + ws * 2 * BOX;
    // Row `lane` of a 64B-swizzled 32 x 32 box: 16-byte piece q sits at q ^ ((lane / 2) % 4).
    const int swz = (lane >> 1) & 3;
    int local = 0;
    int norm_block = -1;   // row block whose statistics nr holds
    float2 nr = make_float2(0.f, 1.f);
    for (int k = 0; k < t_count; ++k, ++local) {
      const int tile = t_first + k * t_step;
      const bool second = GROUP && tile >= per;
      const int lt = second ? tile - per : tile;
      const EpiParams& e = second ? ep2 : ep;
      const CUtensorMap* map_o = second ? &tmO2 : &tmO;
      const CUtensorMap* map_r = second ? &tmR2 : &tmR;
      const int m0 = (lt / n_tiles) * PM + (int)rank * BM, n0 = (lt % n_tiles) * BN;
      const int buf = local & 1, use = local >> 1;
      const int row0 = m0 + quarter * 32, row = row0 + lane;
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * BN);
      if constexpr (STAGED) {
        if (lane == 0) {
          tc::bulk_wait_read();   // the previous tile's stores have left this warp's boxes
          if constexpr (RES) {
#pragma unroll
            for (int j = 0; j < MINE; ++j) {
              const int chunk = group + 4 * j;
              if (chunk < CHUNKS) {
                mbar_expect_tx(res_full + 2 * ws + j, BOX);
                tc::tma_load_2d(wbox + j * BOX, map_r, n0 + chunk * 32, row0, res_full + 2 * ws + j);
              }
            }
          }
        }
        __syncwarp();
      }
      if constexpr (LN_FOLD) {
        if (group < CHUNKS && lt / n_tiles != norm_block) {
          nr = row_norm(e, row, M);
          norm_block = lt / n_tiles;
        }
      }
      Operands ops;
      if (group < CHUNKS) prefetch32<E, !STAGED>(e, N, row, n0 + group * 32, ops);
      if (!tc::wait(acc_full + buf, use & 1, abort_flag)) { record_timeout(); break; }
      tc::fence_after();
      bool ok = true;
#pragma unroll
      for (int j = 0; j < MINE; ++j) {
        const int chunk = group + 4 * j;
        if (chunk < CHUNKS) {
          if (j > 0) prefetch32<E, !STAGED>(e, N, row, n0 + chunk * 32, ops);
          uint32_t acc[32];
          tc::ld32(taddr + chunk * 32, acc);
          tc::wait_ld();
          if constexpr (STAGED) {
            uint4* rb = reinterpret_cast<uint4*>(wbox + j * BOX + lane * 64);
            if constexpr (RES) {
              if (!tc::wait(res_full + 2 * ws + j, local & 1, abort_flag)) { record_timeout(); ok = false; break; }
#pragma unroll
              for (int q = 0; q < 4; ++q) ops.res[q] = rb[q ^ swz];
            }
            float y[32];
            float* uv = uv_stage + ws * 64;
            if constexpr (LN_FOLD) {
              __syncwarp();   // the previous chunk's reads of uv are done
              uv[lane] = ops.u;
              uv[32 + lane] = ops.v;
              __syncwarp();
            }
            epilogue_math<E>(e, row, n0 + chunk * 32, acc, ops, nr, y, LN_FOLD ? uv : nullptr);
            uint32_t pk[16];
#pragma unroll
            for (int w = 0; w < 16; ++w) pk[w] = tc::pack_bf16x2(y[2 * w], y[2 * w + 1]);
            if constexpr (LN_STATS) chunk_stats_packed(e, M, row, n0 + chunk * 32, pk);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              rb[q ^ swz] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
            tc::fence_async_smem();
            __syncwarp();
            if (lane == 0) {
              tc::tma_store_2d(map_o, n0 + chunk * 32, row0, wbox + j * BOX);
              tc::bulk_commit();
            }
          } else {
            float* uv = uv_stage + ws * 64;
            if constexpr (LN_FOLD) {
              __syncwarp();
              uv[lane] = ops.u;
              uv[32 + lane] = ops.v;
              __syncwarp();
            }
            if (row < M) epilogue32<E>(e, out, M, N, row, n0 + chunk * 32, acc, ops, nr, LN_FOLD ? uv : nullptr);
          }
        }
      }
      tc::fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cluster(acc_empty0 + 8 * buf);
      if (!ok) break;
    }
    if constexpr (STAGED) {
      if (lane == 0) tc::bulk_wait_all();   // every store of this warp is complete before the CTA ends
    }
    tc::fence_before();
    __syncwarp();
    tc::cluster_sync();
  }
}

template <int BN, int STAGES>
constexpr size_t pair_smem_bytes() {
  return 1024 + STAGES * (A_BYTES + (size_t)(BN / 2) * BK * 2) + (size_t)kEpilogueWarps * 2 * BOX +
         (2 * STAGES + 4 + 2 * kEpilogueWarps) * 8 + 16 + kEpilogueWarps * 64 * 4;
}

// One launch of the pair kernel; with kGroup in EPI, a second problem of the same M, N, K (a2 ... ep2) whose tiles
// follow the first's (without it the second set repeats the first and is not read).
template <int BN, int STAGES, int EPI>
int launch_pair_tile(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& o, const CUtensorMap& r,
                     uint16_t* out, int M, int N, int K, const EpiParams& ep, cudaStream_t stream,
                     const CUtensorMap* a2 = nullptr, const CUtensorMap* b2 = nullptr, const CUtensorMap* o2 = nullptr,
                     const CUtensorMap* r2 = nullptr, const EpiParams* ep2 = nullptr) {
  constexpr size_t bytes = pair_smem_bytes<BN, STAGES>();
  static PerDevice<int> pairs_per_device;
  int max_pairs = 0;
  const int rc = pairs_per_device.get(&max_pairs, [](int, int* clusters) -> int {
    SVX_CHECK_CUDA(cudaFuncSetAttribute(gemm_pair_kernel<BN, STAGES, EPI>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = bytes;
    SVX_CHECK_CUDA(cudaOccupancyMaxActiveClusters(clusters, gemm_pair_kernel<BN, STAGES, EPI>, &cfg));
    SVX_REQUIRE(*clusters > 0, "gemm: no CTA pair fits on this device");
    return SVX_OK;
  });
  if (rc) return rc;
  const int tiles = (N / BN) * (M / PM) * ((EPI & kGroup) ? 2 : 1);
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  return launch_dependent("gemm_pair_kernel", gemm_pair_kernel<BN, STAGES, EPI>, dim3(2 * pairs), dim3(kThreads),
                          bytes, stream, a, b, o, r, out, M, N, K, ep, a2 ? *a2 : a, b2 ? *b2 : b, o2 ? *o2 : o,
                          r2 ? *r2 : r, ep2 ? *ep2 : ep);
}

template <int BN, int STAGES>
constexpr size_t smem_bytes() {
  return 1024 + STAGES * (A_BYTES + (size_t)BN * BK * 2) + (2 * STAGES + 4) * 8 + 16;
}

template <int BN, int STAGES, int EPI>
int launch_tile(const CUtensorMap& a, const CUtensorMap& b, uint16_t* out, int M, int N, int K, const EpiParams& ep,
                cudaStream_t stream) {
  constexpr size_t bytes = smem_bytes<BN, STAGES>();
  static PerDevice<int> sms_per_device;
  int sms = 0;
  const int rc = sms_per_device.get(&sms, [](int device, int* count) -> int {
    SVX_CHECK_CUDA(cudaFuncSetAttribute(gemm_kernel<BN, STAGES, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)bytes));
    SVX_CHECK_CUDA(cudaDeviceGetAttribute(count, cudaDevAttrMultiProcessorCount, device));
    return SVX_OK;
  });
  if (rc) return rc;
  const int tiles = (N / BN) * (M / BM);
  return launch_dependent("gemm_kernel", gemm_kernel<BN, STAGES, EPI>, dim3(tiles < sms ? tiles : sms), dim3(kThreads),
                          bytes, stream, a, b, out, M, N, K, ep);
}

template <int EPI>
int launch_pair_epi(const CUtensorMap& a, const CUtensorMap& b_half, const CUtensorMap& o, const CUtensorMap& r,
                    int bn, uint16_t* out, int M, int N, int K, const EpiParams& ep, cudaStream_t stream) {
  switch (bn) {
    case 256: return launch_pair_tile<256, 4, EPI>(a, b_half, o, r, out, M, N, K, ep, stream);
    case 192: return launch_pair_tile<192, 5, EPI>(a, b_half, o, r, out, M, N, K, ep, stream);
    case 128: return launch_pair_tile<128, 5, EPI>(a, b_half, o, r, out, M, N, K, ep, stream);
    default: return fail(SVX_ERR_INVALID, "gemm: pair tile width must be 128, 192 or 256");
  }
}

template <int EPI>
int launch_epi(const CUtensorMap& a, const CUtensorMap& b, int bn, uint16_t* out, int M, int N, int K,
               const EpiParams& ep, cudaStream_t stream) {
  switch (bn) {
    case 256: return launch_tile<256, 4, EPI>(a, b, out, M, N, K, ep, stream);
    case 128: return launch_tile<128, 6, EPI>(a, b, out, M, N, K, ep, stream);
    case 64: return launch_tile<64, 8, EPI>(a, b, out, M, N, K, ep, stream);
    default: return fail(SVX_ERR_INVALID, "gemm: tile width must be 64, 128 or 256");
  }
}

}  // namespace

// ------------------------------------------------------------------------------------------- host side

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(ptr);
  }
  return fn;
}

static int make_kmajor_map(CUtensorMap* map, const void* ptr, int rows, int cols, int box_rows) {
  EncodeTiled encode = encode_fn();
  if (!encode) return fail(SVX_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  SVX_REQUIRE((reinterpret_cast<uintptr_t>(ptr) & 15u) == 0, "gemm operand must be 16-byte aligned");
  SVX_REQUIRE(cols % BK == 0 && rows % box_rows == 0, "gemm operand shape must tile by the box");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, elem,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SVX_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return SVX_OK;
}

int make_map_3d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t groups, uint64_t rows,
                uint64_t group_stride_bytes, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                CUtensorMapSwizzle swizzle) {
  EncodeTiled encode = encode_fn();
  if (!encode) return fail(SVX_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  SVX_REQUIRE((reinterpret_cast<uintptr_t>(ptr) & 15u) == 0, "TMA operand must be 16-byte aligned");
  SVX_REQUIRE(group_stride_bytes % 16 == 0 && row_stride_bytes % 16 == 0, "TMA strides must be multiples of 16 bytes");
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)groups, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)group_stride_bytes, (cuuint64_t)row_stride_bytes};
  cuuint32_t box[3] = {box_inner, 1, box_rows};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, elem,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SVX_ERR_CUDA, "cuTensorMapEncodeTiled (3d) failed: " + std::to_string((int)r));
  return SVX_OK;
}

// Tile width for the persistent grid. A CTA streams the 128-row A slice and the BN-row W slice of every tile it owns,
// so a tile costs about (128 + BN) operand rows of traffic: pick the smallest (tiles per SM, rounded up) x (128 + BN),
// the wider tile on ties (measured on B200 at M = 8192: BN 64 reaches ~420 TFLOP/s, BN 256 ~800-980).
static int pick_bn(int M, int N) {
  int sms = 148;
  int device = 0;
  if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  int best = 0;
  long best_cost = 0;
  for (int bn : {256, 128, 64}) {
    if (N % bn) continue;
    const long tiles = (long)(N / bn) * (M / BM);
    const long cost = ((tiles + sms - 1) / sms) * (BM + bn);
    if (!best || cost < best_cost) { best = bn; best_cost = cost; }
  }
  return best;
}

// Tile width for CTA pairs (256-row tiles, 74 pairs on 148 SMs). A tile's main loop is bound by its products, which
// scale with BN, plus a per-tile cost (epilogue, accumulator hand-off) that the fused epilogues (LayerNorm fold, row
// statistics, RoPE, GELU) make worth about 200 columns: the cost of a width is (rounds of tiles over the pairs) x
// (BN + 200); the wider tile on ties. Measured on B200 at M = 8192 with the engine's epilogues (us, BN 256/192/128):
// qkv 36.5/42.2/43.7, fc1 43.8/44.8/54.6, fc2 43.4/35.9/46.0, d x d 19.0/17.0/19.6, head 187.0/-/240.0.
static int pick_pair_bn(int M, int N) {
  int sms = 148;
  int device = 0;
  if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int pairs = sms / 2;
  int best = 0;
  long best_cost = 0;
  for (int bn : {256, 192, 128}) {
    if (N % bn) continue;
    const long tiles = (long)(N / bn) * (M / PM);
    const long cost = ((tiles + pairs - 1) / pairs) * (bn + 200);
    if (!best || cost < best_cost) { best = bn; best_cost = cost; }
  }
  return best;
}

int gemm_plan(GemmPlan* plan, const uint16_t* A, const uint16_t* W, int M, int N, int K, int bn) {
  SVX_REQUIRE(M > 0 && M % BM == 0, "gemm: M must be a positive multiple of 128");
  SVX_REQUIRE(N > 0 && N % 64 == 0 && K > 0 && K % BK == 0, "gemm: N and K must be multiples of 64");
  plan->M = M; plan->N = N; plan->K = K;
  plan->bn = bn > 0 ? bn : pick_bn(M, N);
  SVX_REQUIRE(N % plan->bn == 0, "gemm: N must be a multiple of the tile width");
  int rc = make_kmajor_map(&plan->a, A, M, K, BM);
  if (rc) return rc;
  rc = make_kmajor_map(&plan->b, W, N, K, plan->bn);
  if (rc) return rc;
  // CTA pairs for row counts that tile by 256, unless the caller fixed a single-CTA tile width.
  plan->pair_bn = (bn <= 0 && M % PM == 0) ? pick_pair_bn(M, N) : 0;
  if (plan->pair_bn) return make_kmajor_map(&plan->b_half, W, N, K, plan->pair_bn / 2);
  return SVX_OK;
}

// 2-D bf16 map over a row-major [rows, cols] matrix: 32 x 32 boxes, 64B swizzle (the epilogue staging boxes).
static int make_box_map(CUtensorMap* map, const void* ptr, int rows, int cols) {
  EncodeTiled encode = encode_fn();
  if (!encode) return fail(SVX_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  SVX_REQUIRE((reinterpret_cast<uintptr_t>(ptr) & 15u) == 0 && cols % 32 == 0 && rows % 32 == 0,
              "gemm: epilogue operand must be 16-byte aligned and tile by 32 x 32");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, elem,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SVX_ERR_CUDA, "cuTensorMapEncodeTiled (box) failed: " + std::to_string((int)r));
  return SVX_OK;
}

template <int E>
static int run_epi(const GemmPlan& plan, int M, uint16_t* out, const EpiParams& ep, cudaStream_t stream) {
  constexpr int EPI = E & 7;
  if (plan.pair_bn && M % PM == 0) {
    CUtensorMap o{}, r{};
    if (EPI != SVX_EPI_CLASS_MAJOR) {
      int rc = make_box_map(&o, out, M, plan.N);
      if (!rc && (EPI == SVX_EPI_GATE_RESIDUAL || EPI == SVX_EPI_RESIDUAL)) {
        SVX_REQUIRE(ep.residual, "gemm: residual epilogue needs a residual");
        rc = make_box_map(&r, ep.residual, M, plan.N);
      }
      if (rc) return rc;
    }
    return launch_pair_epi<E>(plan.a, plan.b_half, o, r, plan.pair_bn, out, M, plan.N, plan.K, ep, stream);
  }
  return launch_epi<E>(plan.a, plan.b, plan.bn, out, M, plan.N, plan.K, ep, stream);
}

int gemm_run(const GemmPlan& plan, int M, uint16_t* out, const EpiParams& ep, cudaStream_t stream) {
  SVX_REQUIRE(M > 0 && M <= plan.M && M % BM == 0, "gemm: run rows must be a multiple of 128 within the plan");
  // The LayerNorm fold is built for the linears that follow a LayerNorm (bias, GELU, RoPE, class-major epilogues),
  // the row statistics for the residual epilogues that produce the normalised streams.
  const bool fold = ep.ln_stats_in != nullptr, stats = ep.ln_stats_out != nullptr;
  SVX_REQUIRE(!fold || (ep.ln_u && ep.ln_v && ep.ln_chunks > 0 && plan.K == 32 * ep.ln_chunks),
              "gemm: the LayerNorm fold needs u, v and K / 32 statistics per row");
  switch (ep.epilogue | (fold ? kFold : 0) | (stats ? kStats : 0)) {
    case SVX_EPI_BIAS: return run_epi<SVX_EPI_BIAS>(plan, M, out, ep, stream);
    case SVX_EPI_BIAS_GELU: return run_epi<SVX_EPI_BIAS_GELU>(plan, M, out, ep, stream);
    case SVX_EPI_GATE_RESIDUAL: return run_epi<SVX_EPI_GATE_RESIDUAL>(plan, M, out, ep, stream);
    case SVX_EPI_RESIDUAL: return run_epi<SVX_EPI_RESIDUAL>(plan, M, out, ep, stream);
    case SVX_EPI_ROPE: return run_epi<SVX_EPI_ROPE>(plan, M, out, ep, stream);
    case SVX_EPI_CLASS_MAJOR: return run_epi<SVX_EPI_CLASS_MAJOR>(plan, M, out, ep, stream);
    case SVX_EPI_BIAS | kFold: return run_epi<SVX_EPI_BIAS | kFold>(plan, M, out, ep, stream);
    case SVX_EPI_BIAS_GELU | kFold: return run_epi<SVX_EPI_BIAS_GELU | kFold>(plan, M, out, ep, stream);
    case SVX_EPI_ROPE | kFold: return run_epi<SVX_EPI_ROPE | kFold>(plan, M, out, ep, stream);
    case SVX_EPI_CLASS_MAJOR | kFold: return run_epi<SVX_EPI_CLASS_MAJOR | kFold>(plan, M, out, ep, stream);
    case SVX_EPI_GATE_RESIDUAL | kStats: return run_epi<SVX_EPI_GATE_RESIDUAL | kStats>(plan, M, out, ep, stream);
    case SVX_EPI_RESIDUAL | kStats: return run_epi<SVX_EPI_RESIDUAL | kStats>(plan, M, out, ep, stream);
    default:
      return fail(SVX_ERR_INVALID, "gemm: unknown epilogue, or a LayerNorm fold / row statistics it does not take");
  }
}

// Two independent gated-residual GEMMs with row statistics (E = GATE_RESIDUAL | kStats) of the same shape in one
// CTA-pair launch: one launch's fixed cost and tail instead of two. Both plans must take the same pair tile width.
static int check_group(const EpiParams& e0, const EpiParams& e1, int M) {
  SVX_REQUIRE(M > 0 && M % PM == 0, "gemm group: rows must be a positive multiple of 256");
  for (const EpiParams* e : {&e0, &e1})
    SVX_REQUIRE(e->epilogue == SVX_EPI_GATE_RESIDUAL && e->bias && e->gate && e->residual && e->ln_stats_out &&
                    !e->ln_stats_in,
                "gemm group: both problems are gated residuals with row statistics (no LayerNorm fold)");
  return SVX_OK;
}

int gemm_run_group(const GemmPlan& p0, uint16_t* out0, const EpiParams& e0, const GemmPlan& p1, uint16_t* out1,
                   const EpiParams& e1, int M, cudaStream_t stream) {
  int rc = check_group(e0, e1, M);
  if (rc) return rc;
  SVX_REQUIRE(M <= p0.M && M <= p1.M, "gemm group: rows beyond a plan");
  SVX_REQUIRE(p0.N == p1.N && p0.K == p1.K && p0.pair_bn && p0.pair_bn == p1.pair_bn,
              "gemm group: both problems need the same N, K and pair tile width");
  CUtensorMap o0{}, r0{}, o1{}, r1{};
  rc = make_box_map(&o0, out0, M, p0.N);
  if (!rc) rc = make_box_map(&r0, e0.residual, M, p0.N);
  if (!rc) rc = make_box_map(&o1, out1, M, p1.N);
  if (!rc) rc = make_box_map(&r1, e1.residual, M, p1.N);
  if (rc) return rc;
  constexpr int E = SVX_EPI_GATE_RESIDUAL | kStats | kGroup;
  switch (p0.pair_bn) {
    case 256: return launch_pair_tile<256, 4, E>(p0.a, p0.b_half, o0, r0, out0, M, p0.N, p0.K, e0, stream, &p1.a,
                                                 &p1.b_half, &o1, &r1, &e1);
    case 192: return launch_pair_tile<192, 5, E>(p0.a, p0.b_half, o0, r0, out0, M, p0.N, p0.K, e0, stream, &p1.a,
                                                 &p1.b_half, &o1, &r1, &e1);
    case 128: return launch_pair_tile<128, 5, E>(p0.a, p0.b_half, o0, r0, out0, M, p0.N, p0.K, e0, stream, &p1.a,
                                                 &p1.b_half, &o1, &r1, &e1);
    default: return fail(SVX_ERR_INVALID, "gemm group: pair tile width must be 128, 192 or 256");
  }
}

int epi_from_args(const svx_epilogue_args* e, EpiParams* ep, int N, int K) {
  SVX_REQUIRE(e && (e->bias || e->ln_stats_in), "gemm: epilogue needs a bias (or the LayerNorm fold's u and v)");
  *ep = EpiParams{};
  ep->epilogue = e->epilogue;
  ep->bias = e->bias;
  ep->gate = e->gate;
  ep->residual = e->residual;
  ep->rope_sin = e->rope_sin;
  ep->rope_cos = e->rope_cos;
  ep->rope_cols = e->rope_cols;
  ep->rows_per_slot = e->rows_per_slot;
  ep->head_dim = e->head_dim;
  ep->classes = e->classes;
  ep->height = e->height; ep->depth = e->depth; ep->width = e->width; ep->patch = e->patch;
  ep->ln_stats_in = reinterpret_cast<const float2*>(e->ln_stats_in);
  ep->ln_u = e->ln_u;
  ep->ln_v = e->ln_v;
  ep->ln_chunks = K / 32;
  ep->ln_inv_chunks = K >= 32 ? 32.f / (float)K : 0.f;
  ep->ln_eps = e->ln_eps;
  ep->ln_stats_out = reinterpret_cast<float2*>(e->ln_stats_out);
  if (e->ln_stats_in)
    SVX_REQUIRE(e->ln_u && e->ln_v && K % 32 == 0 && (reinterpret_cast<uintptr_t>(e->ln_u) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(e->ln_v) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(e->ln_stats_in) & 7) == 0,
                "gemm: the LayerNorm fold needs K % 32 == 0, 16-byte aligned u and v, 8-byte aligned statistics");
  if (e->ln_stats_out)
    SVX_REQUIRE(e->epilogue != SVX_EPI_CLASS_MAJOR && (reinterpret_cast<uintptr_t>(e->ln_stats_out) & 7) == 0,
                "gemm: row statistics need a row-major output and an 8-byte aligned buffer");
  if (e->epilogue == SVX_EPI_GATE_RESIDUAL) SVX_REQUIRE(e->gate && e->residual, "gemm: gated residual needs gate+res");
  if (e->epilogue == SVX_EPI_RESIDUAL) SVX_REQUIRE(e->residual, "gemm: residual epilogue needs the residual");
  if (e->epilogue == SVX_EPI_ROPE)
    SVX_REQUIRE(e->rope_sin && e->rope_cos && e->rows_per_slot > 0 && e->head_dim > 0 && e->head_dim % 32 == 0 &&
                    e->rope_cols % 32 == 0,
                "gemm: bad RoPE epilogue arguments");
  if (e->epilogue == SVX_EPI_CLASS_MAJOR)
    SVX_REQUIRE(e->patch == 4 && e->classes > 0 && N == e->classes * 64 &&
                    e->rows_per_slot == (e->height / 4) * (e->depth / 4) * (e->width / 4),
                "gemm: bad class-major epilogue arguments");
  return SVX_OK;
}

}  // namespace svx

using namespace svx;

extern "C" int svx_gemm(const uint16_t* A, const uint16_t* W, uint16_t* out, int M, int N, int K,
                        const svx_epilogue_args* epi, void* stream) {
  SVX_REQUIRE(A && W && out, "svx_gemm: null operand");
  EpiParams ep;
  int rc = epi_from_args(epi, &ep, N, K);
  if (rc) return rc;
  GemmPlan plan;
  rc = gemm_plan(&plan, A, W, M, N, K, 0);
  if (rc) return rc;
  return gemm_run(plan, M, out, ep, as_stream(stream));
}

extern "C" int svx_gemm_group(const uint16_t* A0, const uint16_t* W0, uint16_t* out0, const svx_epilogue_args* epi0,
                              const uint16_t* A1, const uint16_t* W1, uint16_t* out1, const svx_epilogue_args* epi1,
                              int M, int N, int K, void* stream) {
  SVX_REQUIRE(A0 && W0 && out0 && A1 && W1 && out1, "svx_gemm_group: null operand");
  EpiParams e0, e1;
  int rc = epi_from_args(epi0, &e0, N, K);
  if (!rc) rc = epi_from_args(epi1, &e1, N, K);
  if (!rc) rc = check_group(e0, e1, M);   // before any CUDA call
  if (rc) return rc;
  GemmPlan p0, p1;
  rc = gemm_plan(&p0, A0, W0, M, N, K, 0);
  if (!rc) rc = gemm_plan(&p1, A1, W1, M, N, K, 0);
  if (rc) return rc;
  return gemm_run_group(p0, out0, e0, p1, out1, e1, M, as_stream(stream));
}

extern "C" uint32_t svx_wait_timeouts(void) {
  uint32_t v = 0;
  if (cudaMemcpyFromSymbol(&v, g_svx_timeouts, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  return v | attention_timeouts();
}
