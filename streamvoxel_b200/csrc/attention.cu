// Non-causal attention, head_dim 96, over per-slot variable-length keys, on the 5th-generation tensor cores.
//
// A launch runs one attention problem, or two independent ones over the same slots, heads and queries (the engine
// pairs a control layer's cross-attention with its backbone layer's self-attention). A persistent CTA per SM takes
// work units of two 128-query tiles of one (problem, slot, head): from a host-built plan (attention_plan: longest
// units first onto the least-loaded CTA, refined by MULTIFIT, so that CTAs finish together when slot lengths differ)
// or, for one problem without a plan, longest slots first in boustrophedon passes. Key tiles
// of 96 are streamed by TMA into four-stage K and V rings, and only the ceil(length / 96) tiles of a slot are loaded:
// the packed-key block mask of `streamvoxel/stream/fast_ops.py:149-159`. Q and K tiles are exactly 96 dims wide: dims
// 0-63 as a 128B-swizzled part (128-byte rows) and dims 64-95 as a 64B-swizzled part (64-byte rows). V tiles are two
// 128B-swizzled 64-dim boxes (dims 96-127 read as zero, no memory traffic) so that P V is one N=96 product per 16 keys.
//
// Tensor memory per query tile i: S_i fp32 at [128 i, +96), O_i fp32 at [256 + 128 i, +96), and P_i (bf16 pairs, 48
// columns) in the two tails: keys 0-63 at [128 i + 96, +32), keys 64-95 at [256 + 128 i + 96, +16) (the products take
// P per 16-key step, so it need not be contiguous). S, P and O are separate, so nothing serialises a query tile's chain but the data
// itself: S_i(t+1) is computed as soon as the softmax has read S_i(t), while it still computes exponentials, and
// P_i(t) V(t) runs while the softmax works on tile t+1. The softmax therefore runs back to back and bounds the step
// together with the tensor core (with 128-key tiles P must share S's columns, and S(t+1) then waits for P(t) V(t)).
//
// Warp roles (384 threads): warp 0 loads Q and the K ring, warp 2 the V ring; warp 1 (which owns TMEM) issues the
// products of query tile 0 and warp 3 those of tile 1 (each loop warp-converged, one elected lane issuing):
//   S_i  = Q_i K(t)^T     M=128, N=96, K=96          (once the softmax has read S_i(t-1))
//   O_i += P_i(t) V(t)    M=128, N=96, K=96          (A = P_i in TMEM, V read MN-major)
// Warps 4-7 run the softmax of tile 0 and warps 8-11 that of tile 1, one query row per thread (TMEM lane): read the
// row of S_i with tcgen05.ld, release S_i, compute P_i = 2^(S*scale - m), and once P_i(t-1) V(t-1) has completed write
// P_i with tcgen05.st and signal the MMA warp. A quarter of the exponentials are evaluated on the FMA pipe (a fitted
// polynomial, relative error 2.7e-6) and the rest on the MUFU, which alone would bound the softmax. The exponent base
// m is raised lazily: only when a row's max grows by more than 8 (a factor 256, so P <= 256 stays exact in the fp32
// sums), and then the warp rescales its O rows in TMEM (after P_i(t-1) V(t-1) has completed, before P_i(t) V(t) is
// issued) -- exact, since P, O and the sum share one m. P is rounded to bf16 before P.V and the row sums stay fp32, as
// in SDPA's flash kernels; the output is normalised in fp32 and written as bf16.
// Every mbarrier wait is bounded (tc::wait); a timeout raises a CTA-wide abort, sets SVX_STATUS_WAIT_TIMEOUT in the
// library's timeout word and skips the rest of the CTA's work.
#include <math.h>

#include <algorithm>
#include <queue>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"
#include "tc.cuh"

namespace svx {

__device__ uint32_t g_svx_attention_timeouts = 0;

namespace {

constexpr int TQ = 128, TK = 96, HD = 96;
constexpr int STAGES = 4;                      // K and V ring depth
constexpr uint32_t QWIDE = TQ * 128;           // Q tile dims 0-63: 128 rows x 128 B (128B swizzle)
constexpr uint32_t QOPER = QWIDE + TQ * 64;    // + dims 64-95: 128 rows x 64 B (64B swizzle)
constexpr uint32_t KWIDE = TK * 128;           // K tile dims 0-63: 96 rows x 128 B
constexpr uint32_t KOPER = KWIDE + TK * 64;    // + dims 64-95
constexpr uint32_t VWIDE = TK * 128;           // one 64-dim atom of a V tile: 96 keys x 128 B
constexpr uint32_t VOPER = 2 * VWIDE;          // one V tile: two atoms along N
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t S_COL = 0, O_COL = 256;      // + 128 i; P_i in the 32-column tails of both (S_COL/O_COL + 96)
constexpr int kThreads = 384;
constexpr int kBars = 2 + 4 * STAGES + 8;
constexpr int kMaxSlots = 512;                 // slot ranking table in shared memory
constexpr size_t kSmem = 1024 + 2 * QOPER + STAGES * (KOPER + VOPER) + kBars * 8 + 16 + kMaxSlots * 4;
// Of every 8 pairs of exponentials, this many go to the FMA pipe (measured on B200: 2 of 8 is the balance point).
constexpr int kFmaPairs = 2;

// 2^x on the FMA pipe for a pair: x = j + f with j = rint(x) from the 1.5 * 2^23 magic sum and f in [-0.5, 0.5], a
// degree-4 polynomial for 2^f (coefficients fitted for least relative error on [-0.5, 0.5]: 2.7e-6), and j added to
// the exponent field. x is clamped at -125.5 so that the result stays a normal float (2^-125.5 where the MUFU would
// give 0 or a denormal; both vanish against the row sum, which is at least 1).
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
  x.x = fmaxf(x.x, -125.5f);
  x.y = fmaxf(x.y, -125.5f);
  const float2 t = __fadd2_rn(x, make_float2(12582912.f, 12582912.f));
  const float2 j = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = __ffma2_rn(j, make_float2(-1.f, -1.f), x);
  float2 q = __ffma2_rn(make_float2(0.009570068679749966f, 0.009570068679749966f), f,
                        make_float2(0.055917806923389435f, 0.055917806923389435f));
  q = __ffma2_rn(q, f, make_float2(0.240247443318367f, 0.240247443318367f));
  q = __ffma2_rn(q, f, make_float2(0.6931218504905701f, 0.6931218504905701f));
  q = __ffma2_rn(q, f, make_float2(0.9999992847442627f, 0.9999992847442627f));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// One attention problem of a launch. A launch runs one or two problems over the same slots, heads and queries (the
// cross-attention of a control layer together with the independent self-attention of its backbone layer).
struct AttnProblem {
  int keys, units;
  int kv_mode;  // 0: K/V groups = heads, rows = slot*keys + key; 1: groups = slot*heads + head, rows = key
  const int32_t* lengths;
  uint16_t* out;
};

// The tensor maps of one problem: Q dims 0-63 (128B swizzle) and 64-95 (64B), K likewise, V as 64-dim boxes.
struct AttnMaps {
  CUtensorMap m[2][5];
};

struct AttnParams {
  int slots, heads, queries, pairs, units, problems;   // units: over all problems
  AttnProblem pr[2];
  // Optional unit assignment built on the host (attention_plan): [G + 1] offsets into the unit list that follows,
  // CTA c taking units [plan[c], plan[c + 1]); ids are natural, problem-major: units of problem 0, then problem 1,
  // each (slot * heads + head) * pairs + pair. Null (one problem only): the boustrophedon passes over the
  // longest-first numbering.
  const int32_t* plan;
  float scale_log2;
};

// One work unit: two 128-query tiles of one (slot, head). Without a plan, units are numbered longest slot first; with
// one, naturally. A tile index past the slot's queries (odd tile counts) repeats the last tile, whose result is not
// stored.
struct Unit {
  int prob, slot, head, q0, nq, length, tiles, kg, kr0;
  __device__ __forceinline__ Unit(const AttnParams& p, const int* rank_slot, int w) {
    prob = w >= p.pr[0].units;
    if (prob) w -= p.pr[0].units;
    // Field selects rather than p.pr[prob]: a dynamic index into the parameters would copy them to local memory.
    const int keys = prob ? p.pr[1].keys : p.pr[0].keys;
    const int kv_mode = prob ? p.pr[1].kv_mode : p.pr[0].kv_mode;
    const int32_t* lengths = prob ? p.pr[1].lengths : p.pr[0].lengths;
    const int per_slot = p.heads * p.pairs;
    const int rem = w % per_slot;
    slot = p.plan ? w / per_slot : rank_slot[w / per_slot];
    head = rem / p.pairs;
    q0 = (rem % p.pairs) * 2 * TQ;
    nq = min(2, (p.queries - q0) / TQ);
    length = lengths ? max(0, min(lengths[slot], keys)) : keys;
    tiles = (length + TK - 1) / TK;
    kg = kv_mode == 0 ? head : slot * p.heads + head;
    kr0 = kv_mode == 0 ? slot * keys : 0;
  }
};

// The k-th unit of CTA c in a grid of G: passes over the longest-first unit list alternate direction (c, then
// 2G - 1 - c, ...), which balances the summed lengths of the CTAs; -1 for a pass that has no unit for c.
__device__ __forceinline__ int unit_of(int c, int k, int G, int units) {
  const int w = k * G + ((k & 1) ? G - 1 - c : c);
  return w < units ? w : -1;
}

// How many units CTA c takes (an upper bound of passes without a plan), and its k-th unit (-1: none). Plan entries
// are clamped to the unit range, so a malformed plan can drop or repeat units but never index out of bounds.
__device__ __forceinline__ int units_of(const AttnParams& p, int c, int G) {
  if (!p.plan) return (p.units + G - 1) / G;
  const int b = min(max(__ldg(p.plan + c), 0), p.units);
  const int e = min(max(__ldg(p.plan + c + 1), b), p.units);
  return e - b;
}

__device__ __forceinline__ int unit_at(const AttnParams& p, int c, int k, int G) {
  if (!p.plan) return unit_of(c, k, G, p.units);
  const int b = min(max(__ldg(p.plan + c), 0), p.units);
  const int w = __ldg(p.plan + G + 1 + b + k);
  return (w >= 0 && w < p.units) ? w : -1;
}

__global__ void __launch_bounds__(kThreads, 1) attention_tc_kernel(const __grid_constant__ AttnMaps maps,
                                                                   const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;                      // Q tiles 0, 1
  uint8_t* sk = sq + 2 * QOPER;            // K ring
  uint8_t* sv = sk + STAGES * KOPER;       // V ring
  uint64_t* bars = reinterpret_cast<uint64_t*>(sv + STAGES * VOPER);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;          // both chains' last S of a unit completed: Q may be replaced
  uint64_t* k_full = bars + 2;
  uint64_t* k_empty = k_full + STAGES;
  uint64_t* v_full = k_empty + STAGES;
  uint64_t* v_empty = v_full + STAGES;
  uint64_t* s_full = v_empty + STAGES;   // per query tile: S_i computed
  uint64_t* s_empty = s_full + 2;        // per query tile, 128 arrivals: S_i has been read
  uint64_t* p_full = s_empty + 2;        // per query tile, 128 arrivals: P_i written (and O_i rescaled)
  uint64_t* pv_done = p_full + 2;        // per query tile: P_i V completed (P_i free, O_i quiescent)
  uint32_t* misc = reinterpret_cast<uint32_t*>(bars + kBars);
  uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;
  int* rank_slot = reinterpret_cast<int*>(misc + 4);

  const int warp = warp_id(), lane = lane_id();
  const int G = gridDim.x, c = blockIdx.x;
  grid_launch_dependents();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 2);
    for (int i = 0; i < STAGES; ++i) {   // a K/V stage is released by the products of both query tiles
      mbar_init(k_full + i, 1); mbar_init(k_empty + i, 2);
      mbar_init(v_full + i, 1); mbar_init(v_empty + i, 2);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full + i, 1); mbar_init(s_empty + i, 128); mbar_init(p_full + i, 128); mbar_init(pv_done + i, 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int pb = 0; pb < p.problems; ++pb)
      for (int j = 0; j < 5; ++j) tc::prefetch_map(&maps.m[pb][j]);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, TMEM_COLS);
  grid_dependency_wait();   // Q, K, V and the lengths come from earlier kernels
  if (warp == 3) {
    // Slots in descending key-length order (ties by slot index): rank_slot[rank] = slot.
    for (int s = lane; s < p.slots; s += 32) {
      int r = s;
      if (p.pr[0].lengths) {
        const int ls = max(0, min(p.pr[0].lengths[s], p.pr[0].keys));
        r = 0;
        for (int u = 0; u < p.slots; ++u) {
          const int lu = max(0, min(p.pr[0].lengths[u], p.pr[0].keys));
          r += (lu > ls) || (lu == ls && u < s);
        }
      }
      rank_slot[r] = s;
    }
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;

  // No register split between the roles: ptxas compiles every role within the launch's 168 registers a thread
  // anyway, and a setmaxnreg decrease in the load/MMA branch made it spill values that the softmax reloads per tile.
  if (warp < 4) {
    if (warp == 0) {   // Q and the K ring
      int T = 0, qn = 0;
      bool ok = true;
      const int nk = units_of(p, c, G);
      for (int k = 0; ok && k < nk; ++k) {
        const int w = unit_at(p, c, k, G);
        if (w < 0) continue;
        const Unit U(p, rank_slot, w);
        if (U.tiles == 0) continue;
        if (qn >= 1 && !tc::wait_w(q_empty, (qn - 1) & 1, abort_flag)) break;
        tc::expect_tx_w(q_full, 2 * QOPER);
        for (int i = 0; i < 2; ++i) {
          const int qr = U.slot * p.queries + U.q0 + min(i, U.nq - 1) * TQ;
          tc::tma_load_3d_w(sq + i * QOPER, &maps.m[U.prob][0], 0, U.head, qr, q_full);
          tc::tma_load_3d_w(sq + i * QOPER + QWIDE, &maps.m[U.prob][1], 64, U.head, qr, q_full);
        }
        for (int t = 0; t < U.tiles; ++t) {
          const int g = T + t, s = g % STAGES;
          if (g >= STAGES && !tc::wait_w(k_empty + s, (g / STAGES - 1) & 1, abort_flag)) { ok = false; break; }
          tc::expect_tx_w(k_full + s, KOPER);
          tc::tma_load_3d_w(sk + s * KOPER, &maps.m[U.prob][2], 0, U.kg, U.kr0 + t * TK, k_full + s);
          tc::tma_load_3d_w(sk + s * KOPER + KWIDE, &maps.m[U.prob][3], 64, U.kg, U.kr0 + t * TK, k_full + s);
        }
        T += U.tiles;
        ++qn;
      }
    } else if (warp == 2) {   // the V ring
      int T = 0;
      bool ok = true;
      const int nk = units_of(p, c, G);
      for (int k = 0; ok && k < nk; ++k) {
        const int w = unit_at(p, c, k, G);
        if (w < 0) continue;
        const Unit U(p, rank_slot, w);
        for (int t = 0; t < U.tiles; ++t) {
          const int g = T + t, s = g % STAGES;
          if (g >= STAGES && !tc::wait_w(v_empty + s, (g / STAGES - 1) & 1, abort_flag)) { ok = false; break; }
          tc::expect_tx_w(v_full + s, VOPER);
          tc::tma_load_3d_w(sv + s * VOPER, &maps.m[U.prob][4], 0, U.kg, U.kr0 + t * TK, v_full + s);
          tc::tma_load_3d_w(sv + s * VOPER + VWIDE, &maps.m[U.prob][4], 64, U.kg, U.kr0 + t * TK, v_full + s);
        }
        T += U.tiles;
      }
    } else {   // warp 1: products of query tile 0; warp 3: of query tile 1
      const int i = warp == 1 ? 0 : 1;
      constexpr uint32_t idesc_s = tc::instr_desc(TQ, TK, false);
      constexpr uint32_t idesc_o = tc::instr_desc(TQ, HD, true);
      const uint32_t qa = smem_addr(sq + i * QOPER);
      const uint32_t s_tmem = tmem + S_COL + 128 * i, o_tmem = tmem + O_COL + 128 * i;
      int T = 0, qn = 0;
      bool ok = true;
      const int nk = units_of(p, c, G);
      for (int k = 0; ok && k < nk; ++k) {
        const int w = unit_at(p, c, k, G);
        if (w < 0) continue;
        const Unit U(p, rank_slot, w);
        if (U.tiles == 0) continue;
        if (!tc::wait_w(q_full, qn & 1, abort_flag)) break;
        for (int t = 0; t <= U.tiles; ++t) {
          if (t < U.tiles) {   // S(t): its K tile has landed and the softmax has read S(t-1)
            const int g = T + t, ks = g % STAGES;
            ok = tc::wait_w(k_full + ks, (g / STAGES) & 1, abort_flag) &&
                 (g == 0 || tc::wait_w(s_empty + i, (g - 1) & 1, abort_flag));
            if (!ok) break;
            tc::fence_after();
            const uint32_t kb = smem_addr(sk + ks * KOPER);
            tc::mma_qk96_w(s_tmem, tc::sw128_desc(qa), tc::sw128_desc(kb), tc::sw64_desc(qa + QWIDE),
                           tc::sw64_desc(kb + KWIDE), idesc_s);
            tc::commit_w(s_full + i);
            tc::commit_w(k_empty + ks);
            if (t == U.tiles - 1) tc::commit_w(q_empty);
          }
          if (t >= 1) {   // O += P(t-1) V(t-1); the unit's first product starts O afresh
            const int g = T + t - 1, vs = g % STAGES;
            ok = tc::wait_w(v_full + vs, (g / STAGES) & 1, abort_flag) && tc::wait_w(p_full + i, g & 1, abort_flag);
            if (!ok) break;
            tc::fence_after();
            tc::mma_pv96_w(o_tmem, s_tmem + 96, o_tmem + 96, tc::sw128_desc(smem_addr(sv + vs * VOPER), VWIDE, 1024),
                           idesc_o, t > 1 ? 1u : 0u);
            tc::commit_w(pv_done + i);
            tc::commit_w(v_empty + vs);
          }
        }
        T += U.tiles;
        ++qn;
      }
    }
    // Teardown: the TMEM owner frees the columns once all 12 warps are past their last TMEM access.
    tc::fence_before();
    __syncwarp();
    asm volatile("barrier.sync 1, %0;" ::"n"(kThreads) : "memory");
    if (warp == 1) {
      tc::fence_after();
      tc::tmem_dealloc(*tmem_slot, TMEM_COLS);
    }
  } else {
    const int i = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    const uint32_t ts = tmem + lanes + S_COL + 128 * i, to = tmem + lanes + O_COL + 128 * i;
    const float sl2 = p.scale_log2;
    int T = 0;
    bool ok = true;
    const int nk = units_of(p, c, G);
    for (int k = 0; ok && k < nk; ++k) {
      const int w = unit_at(p, c, k, G);
      if (w < 0) continue;
      const Unit U(p, rank_slot, w);
      // The output row of this thread, computed where it is written so that it is not live across the tile loop.
      auto out_row = [&](const Unit& V) {
        return reinterpret_cast<uint4*>((V.prob ? p.pr[1].out : p.pr[0].out) +
                                        ((int64_t)V.slot * p.queries + V.q0 + i * TQ + row) * (p.heads * HD) +
                                        V.head * HD);
      };
      if (U.tiles == 0) {
        if (i < U.nq) {
          uint4* dst = out_row(U);
          for (int k8 = 0; k8 < HD / 8; ++k8) dst[k8] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      float m_used = -INFINITY, l_run = 0.f;
      for (int t = 0; t < U.tiles; ++t) {
        const int g = T + t;
        if (!tc::wait(s_full + i, g & 1, abort_flag)) { ok = false; break; }
        tc::fence_after();
        uint32_t r[3][32];
#pragma unroll
        for (int c3 = 0; c3 < 3; ++c3) tc::ld32(ts + c3 * 32, r[c3]);
        tc::wait_ld();
        tc::fence_before();
        tc::mbar_arrive(s_empty + i);   // S_i(t+1) may now be computed into the same columns
        const int key0 = t * TK;
        if (key0 + TK > U.length) {
#pragma unroll
          for (int c3 = 0; c3 < 3; ++c3)
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (key0 + c3 * 32 + j >= U.length) r[c3][j] = __float_as_uint(-INFINITY);
        }
        float mc[3];
#pragma unroll
        for (int c3 = 0; c3 < 3; ++c3) {
          float a = __uint_as_float(r[c3][0]), b = __uint_as_float(r[c3][1]);
#pragma unroll
          for (int j = 2; j < 32; j += 4) {
            a = tc::fmax3(a, __uint_as_float(r[c3][j]), __uint_as_float(r[c3][j + 1]));
            b = tc::fmax3(b, __uint_as_float(r[c3][j + 2]), __uint_as_float(r[c3][j + 3]));
          }
          mc[c3] = fmaxf(a, b);
        }
        const float mx = tc::fmax3(mc[0], mc[1], mc[2]) * sl2;
        // Raise the exponent base only when the row max outgrows it by more than 8 (warp-uniform rescale of O).
        const bool raise = mx > m_used + 8.f;
        const bool any_raise = __any_sync(0xffffffffu, raise);
        float alpha = 1.f;
        if (any_raise) {
          const float m_new = raise ? mx : m_used;
          alpha = tc::ex2(m_used - m_new);   // m_used = -inf on the first tile: alpha = 0
          m_used = m_new;
        }
        // P = 2^(S*scale - m) as bf16 pairs: keys 2j, 2j+1 -> P column j (0-31 after S_i, 32-47 after O_i).
        const float2 scale2 = make_float2(sl2, sl2), nbase2 = make_float2(-m_used, -m_used);
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        uint32_t packed[48];
#pragma unroll
        for (int j = 0; j < TK; j += 2) {
          const int c3 = j >> 5, jj = j & 31;
          const float2 x = __ffma2_rn(make_float2(__uint_as_float(r[c3][jj]), __uint_as_float(r[c3][jj + 1])), scale2,
                                      nbase2);
          const float2 e = ((j >> 1) & 7) < kFmaPairs ? exp2_fma2(x) : make_float2(tc::ex2(x.x), tc::ex2(x.y));
          acc[(j >> 1) & 3] = __fadd2_rn(acc[(j >> 1) & 3], e);
          packed[j >> 1] = tc::pack_bf16x2(e.x, e.y);
        }
        // P_i(t-1) V(t-1) has completed: P_i may be overwritten and O_i holds the products of tiles < t.
        if (g >= 1 && !tc::wait(pv_done + i, (g - 1) & 1, abort_flag)) { ok = false; break; }
        tc::fence_after();
        if (any_raise && t >= 1) {
#pragma unroll
          for (int c3 = 0; c3 < HD / 32; ++c3) {
            uint32_t o[32];
            tc::ld32(to + c3 * 32, o);
            tc::wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
            tc::st32(to + c3 * 32, o);
          }
        }
        {
          uint32_t lo[32], hi[16];
#pragma unroll
          for (int j = 0; j < 32; ++j) lo[j] = packed[j];
#pragma unroll
          for (int j = 0; j < 16; ++j) hi[j] = packed[32 + j];
          tc::st32(ts + 96, lo);
          tc::st16(to + 96, hi);
        }
        tc::wait_st();
        const float2 s01 = __fadd2_rn(acc[0], acc[1]), s23 = __fadd2_rn(acc[2], acc[3]);
        l_run = l_run * alpha + ((s01.x + s01.y) + (s23.x + s23.y));
        tc::fence_before();
        tc::mbar_arrive(p_full + i);
      }
      if (ok) ok = tc::wait(pv_done + i, (T + U.tiles - 1) & 1, abort_flag);
      if (!ok) break;
      tc::fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      const Unit V(p, rank_slot, w);
      uint4* dst = out_row(V);
#pragma unroll
      for (int c3 = 0; c3 < HD / 32; ++c3) {
        uint32_t o[32];
        tc::ld32(to + c3 * 32, o);
        tc::wait_ld();
        if (i < V.nq) {
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const float* f = reinterpret_cast<const float*>(o) + 8 * k4;
            dst[c3 * 4 + k4] = make_uint4(tc::pack_bf16x2(f[0] * inv, f[1] * inv),
                                          tc::pack_bf16x2(f[2] * inv, f[3] * inv),
                                          tc::pack_bf16x2(f[4] * inv, f[5] * inv),
                                          tc::pack_bf16x2(f[6] * inv, f[7] * inv));
          }
        }
      }
      // O_i has been read (tcgen05.wait::ld above); the next unit's first P V, which overwrites it, is issued only
      // after this warpgroup's next p_full arrival.
      T += U.tiles;
    }
    if (!ok && lane == 0) atomicOr(&g_svx_attention_timeouts, SVX_STATUS_WAIT_TIMEOUT);
    // Teardown: every TMEM access of this warpgroup is done; the TMEM owner frees the columns after all 12 warps.
    tc::fence_before();
    __syncwarp();
    asm volatile("barrier.arrive 1, %0;" ::"n"(kThreads) : "memory");
  }
}

}  // namespace

int attention_plan_ints(int problems, int slots, int heads, int queries, int ctas) {
  if (problems < 1 || problems > 2 || slots <= 0 || heads <= 0 || queries <= 0 || queries % TQ || ctas <= 0) return 0;
  const int64_t units = (int64_t)problems * slots * heads * ((queries / TQ + 1) / 2);
  if (units > (1 << 28)) return 0;
  return (int)(std::min<int64_t>(ctas, units) + 1 + units);
}

int attention_plan(const int32_t* const* lengths, const int* keys, int problems, int slots, int heads, int queries,
                   int ctas, int32_t* plan, int capacity) {
  const int need = attention_plan_ints(problems, slots, heads, queries, ctas);
  SVX_REQUIRE(need > 0 && keys, "attention_plan: bad shape");
  for (int pb = 0; pb < problems; ++pb) SVX_REQUIRE(keys[pb] > 0, "attention_plan: bad key count");
  SVX_REQUIRE(plan && capacity >= need, "attention_plan: plan buffer too small");
  const int pairs = (queries / TQ + 1) / 2, per_slot = heads * pairs, per_prob = slots * per_slot;
  const int units = problems * per_prob;
  const int G = std::min(ctas, units);
  // Cost of a unit in quarter key tiles: its tiles plus two tiles of per-unit work (Q load, ring fill, epilogue; the
  // joint launch measured on B200 at the bench's lengths: 1 tile 176.3 us, 2 tiles 173.1, 3-6 tiles the same as 2);
  // a unit without keys only writes zeros.
  std::vector<int64_t> cost(units);
  for (int u = 0; u < units; ++u) {
    const int pb = u / per_prob, slot = (u % per_prob) / per_slot;
    const int len = lengths && lengths[pb] ? std::max(0, std::min(lengths[pb][slot], keys[pb])) : keys[pb];
    const int tiles = (len + TK - 1) / TK;
    cost[u] = tiles ? 4 * (int64_t)tiles + 8 : 1;
  }
  std::vector<int> order(units);
  for (int u = 0; u < units; ++u) order[u] = u;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost[a] > cost[b]; });
  // Longest processing time first (LPT): each unit to the least-loaded CTA (lowest index on ties).
  std::priority_queue<std::pair<int64_t, int>, std::vector<std::pair<int64_t, int>>, std::greater<>> heap;
  for (int c = 0; c < G; ++c) heap.emplace(0, c);
  std::vector<int> owner(units), trial(units);
  int64_t best = 0, total = 0;
  for (int u : order) {
    auto [load, c] = heap.top();
    heap.pop();
    owner[u] = c;
    heap.emplace(load + cost[u], c);
    best = std::max(best, load + cost[u]);
    total += cost[u];
  }
  // MULTIFIT: the smallest capacity at which first-fit decreasing packs the units into G CTAs, by bisection between
  // the lower bound and the LPT makespan; kept when it beats LPT (a few long slots among many short ones).
  std::vector<int64_t> bin(G);
  auto first_fit = [&](int64_t cap) {
    std::fill(bin.begin(), bin.end(), 0);
    int open = 0;
    for (int u : order) {
      int c = 0;
      while (c < open && bin[c] + cost[u] > cap) ++c;
      if (c == open) {
        if (open == G) return false;
        ++open;
      }
      bin[c] += cost[u];
      trial[u] = c;
    }
    return true;
  };
  int64_t lo = std::max<int64_t>(cost[order[0]], (total + G - 1) / G), hi = best - 1;
  while (lo <= hi) {
    const int64_t mid = lo + (hi - lo) / 2;
    if (first_fit(mid)) {
      owner = trial;
      best = mid;
      hi = mid - 1;
    } else {
      lo = mid + 1;
    }
  }
  std::vector<int> count(G + 1, 0);
  for (int u = 0; u < units; ++u) ++count[owner[u]];
  plan[0] = 0;
  for (int c = 0; c < G; ++c) plan[c + 1] = plan[c] + count[c];
  std::vector<int> fill(plan, plan + G);
  for (int u : order) plan[G + 1 + fill[owner[u]]++] = u;   // each CTA's units longest first
  return SVX_OK;
}

int attention_launch(const svx_attention_problem* probs, int problems, int slots, int heads, int queries,
                     const int32_t* plan, int plan_ctas, cudaStream_t stream) {
  SVX_REQUIRE(problems == 1 || (problems == 2 && plan), "attention: one problem, or two with a plan");
  SVX_REQUIRE(queries % TQ == 0, "attention: queries must be a multiple of 128");
  SVX_REQUIRE(slots <= kMaxSlots, "attention: at most 512 slots");
  const int pairs = (queries / TQ + 1) / 2;
  const int per_prob = slots * heads * pairs, units = problems * per_prob;
  AttnMaps maps;
  AttnParams prm{};
  prm.slots = slots; prm.heads = heads; prm.queries = queries; prm.pairs = pairs; prm.units = units;
  prm.problems = problems; prm.plan = plan;
  prm.scale_log2 = (1.0f / sqrtf((float)HD)) * 1.4426950408889634f;
  constexpr CUtensorMapSwizzle SW64 = CU_TENSOR_MAP_SWIZZLE_64B;
  for (int pb = 0; pb < 2; ++pb) {
    const svx_attention_problem& a = probs[pb < problems ? pb : 0];
    const int keys = a.keys;
    SVX_REQUIRE(keys > 0, "attention: keys must be positive");
    int kv_mode;
    uint64_t groups, rows;
    if (a.kv_slot_stride == (int64_t)keys * a.kv_row_stride) {          // [slot*keys + key][.. head*stride ..]
      kv_mode = 0; groups = heads; rows = (uint64_t)slots * keys;
    } else if (a.kv_slot_stride == (int64_t)heads * a.kv_head_stride) {  // [slot][head][key][dim]
      kv_mode = 1; groups = (uint64_t)slots * heads; rows = keys;
    } else {
      return fail(SVX_ERR_INVALID, "attention: K/V strides must be [slot*keys][head] or [slot][head][key] layouts");
    }
    const uint64_t gs = a.kv_head_stride * 2, rs = a.kv_row_stride * 2, qrows = (uint64_t)slots * queries;
    CUtensorMap* m = maps.m[pb];
    int rc = make_map_3d(&m[0], a.q, HD, heads, qrows, HD * 2, a.q_row_stride * 2, 64, TQ);
    if (!rc) rc = make_map_3d(&m[1], a.q, HD, heads, qrows, HD * 2, a.q_row_stride * 2, 32, TQ, SW64);
    if (!rc) rc = make_map_3d(&m[2], a.k, HD, groups, rows, gs, rs, 64, TK);
    if (!rc) rc = make_map_3d(&m[3], a.k, HD, groups, rows, gs, rs, 32, TK, SW64);
    if (!rc) rc = make_map_3d(&m[4], a.v, HD, groups, rows, gs, rs, 64, TK);
    if (rc) return rc;
    prm.pr[pb] = AttnProblem{keys, per_prob, kv_mode, a.lengths, a.out};
  }
  static PerDevice<int> sms_per_device;
  int sms = 0;
  const int rc = sms_per_device.get(&sms, [](int device, int* count) -> int {
    SVX_CHECK_CUDA(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
    SVX_CHECK_CUDA(cudaDeviceGetAttribute(count, cudaDevAttrMultiProcessorCount, device));
    return SVX_OK;
  });
  if (rc) return rc;
  SVX_REQUIRE(!plan || (plan_ctas >= 1 && plan_ctas <= units), "attention: a plan needs 1 <= ctas <= units");
  const int grid = plan ? plan_ctas : (units < sms ? units : sms);
  return launch_dependent("attention_tc_kernel", attention_tc_kernel, dim3(grid), dim3(kThreads), kSmem, stream,
                          maps, prm);
}

int attention_run(const uint16_t* q, int64_t q_row_stride, const uint16_t* k, const uint16_t* v,
                  int64_t kv_slot_stride, int64_t kv_head_stride, int64_t kv_row_stride, const int32_t* lengths,
                  int slots, int heads, int queries, int keys, uint16_t* out, const int32_t* plan, int plan_ctas,
                  cudaStream_t stream) {
  const svx_attention_problem a{q, k, v, q_row_stride, kv_slot_stride, kv_head_stride, kv_row_stride, lengths, keys,
                                out};
  return attention_launch(&a, 1, slots, heads, queries, plan, plan_ctas, stream);
}

uint32_t attention_timeouts() {
  uint32_t v = 0;
  if (cudaMemcpyFromSymbol(&v, g_svx_attention_timeouts, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  return v;
}

}  // namespace svx

using namespace svx;

extern "C" int svx_attention_plan_ints(int slots, int heads, int queries, int ctas) {
  return attention_plan_ints(1, slots, heads, queries, ctas);
}

extern "C" int svx_attention_plan(const int32_t* lengths, int slots, int heads, int queries, int keys, int ctas,
                                  int32_t* plan, int capacity) {
  return attention_plan(&lengths, &keys, 1, slots, heads, queries, ctas, plan, capacity);
}

extern "C" int svx_attention_multi_plan_ints(int problems, int slots, int heads, int queries, int ctas) {
  return attention_plan_ints(problems, slots, heads, queries, ctas);
}

extern "C" int svx_attention_multi_plan(const int32_t* const* lengths, const int* keys, int problems, int slots,
                                        int heads, int queries, int ctas, int32_t* plan, int capacity) {
  return attention_plan(lengths, keys, problems, slots, heads, queries, ctas, plan, capacity);
}

namespace {
int check_problem(const svx_attention_problem& a) {
  SVX_REQUIRE(a.q && a.k && a.v && a.out && a.keys > 0, "svx_attention: bad arguments");
  SVX_REQUIRE(a.q_row_stride % 8 == 0 && a.kv_row_stride % 8 == 0 && a.kv_head_stride % 8 == 0 &&
                  a.kv_slot_stride % 8 == 0,
              "svx_attention: strides must be multiples of 8 elements");
  const uintptr_t align = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                          reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.out);
  SVX_REQUIRE((align & 15u) == 0, "svx_attention: operands must be 16-byte aligned");
  return SVX_OK;
}
}  // namespace

extern "C" int svx_attention(const uint16_t* q, int64_t q_row_stride, const uint16_t* k, const uint16_t* v,
                             int64_t kv_slot_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                             const int32_t* lengths, int slots, int heads, int queries, int keys, uint16_t* out,
                             const int32_t* plan, int plan_ctas, void* stream) {
  SVX_REQUIRE(slots > 0 && heads > 0 && queries > 0, "svx_attention: bad arguments");
  const svx_attention_problem a{q, k, v, q_row_stride, kv_slot_stride, kv_head_stride, kv_row_stride, lengths, keys,
                                out};
  if (const int rc = check_problem(a)) return rc;
  return attention_launch(&a, 1, slots, heads, queries, plan, plan_ctas, as_stream(stream));
}

extern "C" int svx_attention_multi(const svx_attention_problem* problems, int count, int slots, int heads,
                                   int queries, const int32_t* plan, int plan_ctas, void* stream) {
  SVX_REQUIRE(problems && (count == 1 || count == 2) && slots > 0 && heads > 0 && queries > 0,
              "svx_attention_multi: one or two problems over positive shapes");
  for (int i = 0; i < count; ++i)
    if (const int rc = check_problem(problems[i])) return rc;
  return attention_launch(problems, count, slots, heads, queries, plan, plan_ctas, as_stream(stream));
}
