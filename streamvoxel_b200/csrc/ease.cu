// EASE sampler kernels: entropy scores, low-entropy-last marking, 4^3 block-quota selection, categorical draw.
//
// Logits are class-major per slot, [classes][voxels] (the reference's [V,Y,Z,X], `streamvoxel/stream/fast_ops.py:307`),
// so a warp reading one class for 32 x VPT consecutive voxels issues fully coalesced 16-byte loads.
#include <math.h>

#include <type_traits>

#include <limits.h>

#include "common.cuh"
#include "tc.cuh"

namespace svx {
namespace {

constexpr int kScoreThreads = 256;
// Entropy and marking kernels: 4 voxels per lane, 2 lanes per voxel group, 8 class rows in flight per lane (the best
// of the shapes measured on B200; more rows per lane or wider loads lower the occupancy more than they add).
constexpr int kStatVoxels = 4, kStatSplit = 2, kStatRows = 8;
constexpr int kSelectThreads = 1024;

// ----------------------------------------------------------------------------------------------- scores

template <typename T, int VPT> struct Vec;
template <> struct Vec<uint16_t, 4> {
  static __device__ __forceinline__ void load(const uint16_t* p, float (&x)[4]) {
    uint2 raw = *reinterpret_cast<const uint2*>(p);
    x[0] = __uint_as_float(raw.x << 16);
    x[1] = __uint_as_float(raw.x & 0xFFFF0000u);
    x[2] = __uint_as_float(raw.y << 16);
    x[3] = __uint_as_float(raw.y & 0xFFFF0000u);
  }
};
template <> struct Vec<float, 4> {
  static __device__ __forceinline__ void load(const float* p, float (&x)[4]) {
    float4 raw = *reinterpret_cast<const float4*>(p);
    x[0] = raw.x; x[1] = raw.y; x[2] = raw.z; x[3] = raw.w;
  }
};

__device__ __forceinline__ float fast_exp2(float x) { return tc::ex2(x); }

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.69314718055994531f;

// Online softmax statistics of one voxel over the class axis, in base 2: b = a reference near the running max logit
// times log2(e), s = sum 2^z and t = sum 2^z z with z = x log2(e) - b, so p = 2^z / s and sum_c p ln p = ln2 t/s - ln s
// for any b. Moving to a larger reference b' is the exact identity s' = 2^d s, t' = 2^d (t + d s) with d = b - b'. The
// move is lazy: it happens only when a logit exceeds b by more than kRebaseSlack, so z <= kRebaseSlack and every term
// stays below 2^kRebaseSlack (the conditional rescaling of FlashAttention-4); after the first rows it is rarely taken.
constexpr float kRebaseSlack = 8.f;

__device__ __forceinline__ void rebase(float& b, float& s, float& t, float nb) {
  if (nb > b + kRebaseSlack) {
    if (b != -INFINITY) {
      const float d = b - nb;
      const float e = fast_exp2(d);
      t = e * fmaf(d, s, t);
      s = e * s;
    }
    b = nb;
  }
}

// Merge another lane's statistics (b2, s2, t2) into (b, s, t).
__device__ __forceinline__ void merge(float& b, float& s, float& t, float b2, float s2, float t2) {
  const float nb = fmaxf(b, b2);
  float ns = 0.f, nt = 0.f;
  if (b != -INFINITY) {
    const float d = b - nb, e = fast_exp2(d);
    ns = e * s;
    nt = e * fmaf(d, s, t);
  }
  if (b2 != -INFINITY) {
    const float d = b2 - nb, e = fast_exp2(d);
    ns = fmaf(e, s2, ns);
    nt = fmaf(e, fmaf(d, s2, t2), nt);
  }
  b = nb;
  s = ns;
  t = nt;
}

// The statistics of VPT voxels starting at `base` (class-major rows `voxels` apart). SPLIT adjacent lanes share the
// voxels and take every SPLIT-th class row each, CH rows in flight per lane, so one warp load covers 32/SPLIT x VPT
// contiguous voxels of SPLIT rows; on return every lane of the group holds the merged statistics of all classes.
// Base-2 exponentials on the MUFU and paired fp32 arithmetic keep it near 7 instructions per logit, so the kernels
// stay close to the HBM time of reading the logits once (measured on B200 for [8, 256, 65536] bf16: 57.5 us, against
// 45 us for the same reads without the arithmetic).
template <typename T, int VPT, int SPLIT, int CH, bool ENTROPY>
__device__ __forceinline__ void class_stats(const T* base, int classes, int voxels, int q, bool valid,
                                            float (&b)[VPT], float (&s)[VPT], float (&t)[VPT]) {
  static_assert(VPT % 2 == 0 && CH >= 2, "voxel pairs");
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    b[v] = -INFINITY;
    s[v] = t[v] = 0.f;
  }
  const float2 l2e = make_float2(kLog2e, kLog2e);
  // Folds rows x[0..R) into the statistics: one (lazy) rebase per voxel, then 2^z on voxel pairs.
  auto fold = [&](auto& x, auto rows) {
    constexpr int R = decltype(rows)::value;
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      float mx = x[0][v];
#pragma unroll
      for (int j = 1; j + 1 < R; j += 2) mx = tc::fmax3(mx, x[j][v], x[j + 1][v]);
      if (R % 2 == 0) mx = fmaxf(mx, x[R - 1][v]);
      rebase(b[v], s[v], t[v], mx * kLog2e);
    }
#pragma unroll
    for (int v = 0; v < VPT; v += 2) {
      const float2 nb = make_float2(-b[v], -b[v + 1]);
      float2 sv = make_float2(s[v], s[v + 1]), tv = make_float2(t[v], t[v + 1]);
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const float2 z = __ffma2_rn(make_float2(x[j][v], x[j][v + 1]), l2e, nb);
        const float2 e = make_float2(fast_exp2(z.x), fast_exp2(z.y));
        sv = __fadd2_rn(sv, e);
        if (ENTROPY) tv = __ffma2_rn(e, z, tv);
      }
      s[v] = sv.x; s[v + 1] = sv.y;
      t[v] = tv.x; t[v + 1] = tv.y;
    }
  };
  int c = q;
  if (valid) {
    for (; c + (CH - 1) * SPLIT < classes; c += CH * SPLIT) {
      float x[CH][VPT];
#pragma unroll
      for (int j = 0; j < CH; ++j) Vec<T, VPT>::load(base + (int64_t)(c + j * SPLIT) * voxels, x[j]);
      fold(x, std::integral_constant<int, CH>());
    }
    for (; c < classes; c += SPLIT) {
      float x[1][VPT];
      Vec<T, VPT>::load(base + (int64_t)c * voxels, x[0]);
      fold(x, std::integral_constant<int, 1>());
    }
  }
#pragma unroll
  for (int off = 1; off < SPLIT; off <<= 1) {
#pragma unroll
    for (int v = 0; v < VPT; ++v) {
      const float b2 = __shfl_xor_sync(0xffffffffu, b[v], off);
      const float s2 = __shfl_xor_sync(0xffffffffu, s[v], off);
      const float t2 = __shfl_xor_sync(0xffffffffu, t[v], off);
      merge(b[v], s[v], t[v], b2, s2, t2);
    }
  }
}

// Negative entropy sum_c p log p (== `(logp.exp()*logp).sum(0)`, `sampling/entropy.py:3-4`), in nats.
template <typename T, int VPT, int SPLIT, int CH>
__global__ void __launch_bounds__(kScoreThreads) ease_scores_kernel(const T* __restrict__ logits, int classes,
                                                                    int voxels, int64_t slot_stride,
                                                                    float* __restrict__ scores,
                                                                    uint32_t* __restrict__ status) {
  const int slot = blockIdx.y;
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  const int q = g % SPLIT;
  const int n0 = (g / SPLIT) * VPT;
  const bool valid = n0 < voxels;
  float b[VPT], s[VPT], t[VPT];
  class_stats<T, VPT, SPLIT, CH, true>(logits + slot * slot_stride + (valid ? n0 : 0), classes, voxels, q, valid, b,
                                       s, t);
  if (!valid || q != 0) return;
  bool nan = false;
  float out[VPT];
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    out[v] = kLn2 * (t[v] / s[v]) - logf(s[v]);
    nan |= isnan(out[v]);
  }
  float* dst = scores + (int64_t)slot * voxels + n0;
#pragma unroll
  for (int v = 0; v < VPT; v += 4)
    *reinterpret_cast<float4*>(dst + v) = make_float4(out[v], out[v + 1], out[v + 2], out[v + 3]);
  if (nan && status) atomicOr(status + slot, SVX_STATUS_NAN_LOGITS);
}

// ----------------------------------------------------------------------------------------------- marking

// good[n] = !(air(n) <= threshold), air = sum over air ids of softmax(logits)[a] (`stream/slot.py:126`): the softmax
// denominator from the same class statistics, then the air probabilities summed in id order.
template <typename T, int VPT, int SPLIT, int CH>
__global__ void __launch_bounds__(kScoreThreads) ease_air_kernel(const T* __restrict__ logits, int classes, int voxels,
                                                                 int64_t slot_stride, const int32_t* __restrict__ air_ids,
                                                                 int n_air, float threshold, uint8_t* __restrict__ good) {
  static_assert(VPT == 4, "one 32-bit store of 4 flags");
  const int slot = blockIdx.y;
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  const int q = g % SPLIT;
  const int n0 = (g / SPLIT) * VPT;
  const bool valid = n0 < voxels;
  const T* base = logits + slot * slot_stride + (valid ? n0 : 0);
  float b[VPT], s[VPT], t[VPT];
  class_stats<T, VPT, SPLIT, CH, false>(base, classes, voxels, q, valid, b, s, t);
  if (!valid || q != 0) return;
  float air[VPT] = {};
  for (int a = 0; a < n_air; ++a) {
    float x[VPT];
    Vec<T, VPT>::load(base + (int64_t)air_ids[a] * voxels, x);
#pragma unroll
    for (int v = 0; v < VPT; ++v) air[v] += fast_exp2(fmaf(x[v], kLog2e, -b[v])) / s[v];
  }
  uint32_t flags = 0;
#pragma unroll
  for (int v = 0; v < VPT; ++v) flags |= (uint32_t)!(air[v] <= threshold) << (8 * v);
  *reinterpret_cast<uint32_t*>(good + (int64_t)slot * voxels + n0) = flags;
}

// last[y,z,x] = good[y'..] for all y' >= y: the per-column top run (`low_entropy_last.py:11-13`, col=True).
__global__ void ease_column_run_kernel(uint8_t* __restrict__ last, int height, int columns, int32_t* last_count) {
  const int slot = blockIdx.x;
  uint8_t* col = last + (int64_t)slot * height * columns;
  int count = 0;
  for (int c = threadIdx.x; c < columns; c += blockDim.x) {
    bool run = true;
    for (int y = height - 1; y >= 0; --y) {
      run = run && col[(int64_t)y * columns + c];
      col[(int64_t)y * columns + c] = run;
      count += run;
    }
  }
  __shared__ int total;
  if (threadIdx.x == 0) total = 0;
  __syncthreads();
  atomicAdd(&total, count);
  __syncthreads();
  if (threadIdx.x == 0) last_count[slot] = total;
}

// ----------------------------------------------------------------------------------------------- selection

struct BlockGeom {
  int height, depth, width, nbz, nbx, blocks;
  __device__ __forceinline__ int voxel(int j, int i) const {  // block j (YZX), in-block offset i (YZX, b = 4)
    int by = j / (nbz * nbx), bz = (j / nbx) % nbz, bx = j % nbx;
    int dy = i >> 4, dz = (i >> 2) & 3, dx = i & 3;
    return ((by * 4 + dy) * depth + bz * 4 + dz) * width + bx * 4 + dx;
  }
};

// Non-deferred (nt) and selectable (lg) voxels of 4^3 block j: one 32-bit load of `last` and one 64-bit load of the
// tokens per 4-voxel x-row (a row starts at a multiple of 4 voxels; the entry points check the alignment).
__device__ __forceinline__ void block_counts(const BlockGeom& g, const uint8_t* lst, const int16_t* tok, int mask_id,
                                             int j, int& nt, int& lg) {
  nt = 0;
  lg = 0;
#pragma unroll 4
  for (int r = 0; r < 16; ++r) {
    const int n = g.voxel(j, r * 4);
    const uint32_t l4 = *reinterpret_cast<const uint32_t*>(lst + n);
    const uint2 t4 = *reinterpret_cast<const uint2*>(tok + n);
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      const bool nl = ((l4 >> (8 * x)) & 0xFFu) == 0;
      const int16_t t = (int16_t)(((x < 2 ? t4.x : t4.y) >> (16 * (x & 1))) & 0xFFFFu);
      nt += nl;
      lg += nl && t == mask_id;
    }
  }
}

// Per-block quota (`block_quota.py:24-30` / `fast_ops.py:451-463`): float64 apportioning of the step goal over
// blocks, the remainder to the blocks with the largest fractional part (seeded order `pos` breaks ties).
__global__ void __launch_bounds__(kSelectThreads) ease_quota_kernel(const int16_t* __restrict__ tokens,
                                                                    const uint8_t* __restrict__ last,
                                                                    const int32_t* __restrict__ pos,
                                                                    const svx_step_params* __restrict__ params,
                                                                    BlockGeom g, int mask_id, int32_t* __restrict__ quota,
                                                                    int32_t* __restrict__ got) {
  const int slot = blockIdx.x;
  const int j = threadIdx.x;
  const int voxels = g.height * g.depth * g.width;
  const svx_step_params p = params[slot];
  __shared__ double keys[kSelectThreads];
  __shared__ int ids[kSelectThreads];
  __shared__ unsigned long long base_sum;
  if (j == 0) { base_sum = 0; got[slot] = 0; }
  __syncthreads();
  long long base = 0;
  double key = INFINITY;
  const int16_t* tok = tokens + (int64_t)slot * voxels;
  const uint8_t* lst = last + (int64_t)slot * voxels;
  if (j < g.blocks && p.k > 0) {
    int ntot = 0, unused = 0;
    block_counts(g, lst, tok, mask_id, j, ntot, unused);
    double ideal = p.frac * (double)ntot;
    base = (long long)floor(ideal + 1e-9);
    key = -(ideal - (double)base) * 1e6 + (double)pos[(int64_t)slot * g.blocks + j];
  }
  atomicAdd(&base_sum, (unsigned long long)base);
  keys[j] = key;
  ids[j] = j;
  __syncthreads();
  // Bitonic sort of (key, id) ascending over the power-of-two padded block count.
  int size = 1;
  while (size < g.blocks) size <<= 1;
  for (int k = 2; k <= size; k <<= 1) {
    for (int stride = k >> 1; stride > 0; stride >>= 1) {
      int partner = j ^ stride;
      if (j < size && partner > j && partner < size) {
        bool up = (j & k) == 0;
        double ka = keys[j], kb = keys[partner];
        int ia = ids[j], ib = ids[partner];
        bool greater = ka > kb || (ka == kb && ia > ib);
        if (greater == up) {
          keys[j] = kb; keys[partner] = ka;
          ids[j] = ib; ids[partner] = ia;
        }
      }
      __syncthreads();
    }
  }
  long long extra = (long long)p.committed + p.k - (long long)base_sum;
  if (extra < 0) extra = 0;
  // ids[r] is the block of rank r; blocks with rank < extra get one more voxel.
  if (j < g.blocks && p.k > 0) {
    const int block = ids[j];
    int lg = 0, nt = 0;
    block_counts(g, lst, tok, mask_id, block, nt, lg);
    long long b = (long long)floor(p.frac * (double)nt + 1e-9);
    long long target = b + (j < extra ? 1 : 0);
    long long q = target - (nt - lg);
    q = q < 0 ? 0 : q;
    q = q > lg ? lg : q;
    quota[(int64_t)slot * g.blocks + block] = (int32_t)q;
  } else if (j < g.blocks) {
    quota[(int64_t)slot * g.blocks + j] = 0;
  }
}

// In-block ranking (`block_quota.py:31-33`): a warp per 4^3 block; voxel i is chosen when fewer than quota selectable
// voxels of its block beat it (higher score, or equal score and lower in-block index: a stable descending sort).
__global__ void ease_block_select_kernel(const float* __restrict__ scores, const int16_t* __restrict__ tokens,
                                         const uint8_t* __restrict__ last, const int32_t* __restrict__ quota,
                                         const svx_step_params* __restrict__ params, BlockGeom g, int mask_id,
                                         uint8_t* __restrict__ chosen, int32_t* __restrict__ got) {
  const int slot = blockIdx.y;
  const int j = blockIdx.x * (blockDim.x >> 5) + warp_id();
  if (j >= g.blocks) return;
  const int lane = lane_id();
  const int voxels = g.height * g.depth * g.width;
  const int64_t off = (int64_t)slot * voxels;
  const int q = params[slot].k > 0 ? quota[(int64_t)slot * g.blocks + j] : 0;
  int n[2];
  float sm[2];
  bool sel[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    n[h] = g.voxel(j, lane + 32 * h);
    sel[h] = !last[off + n[h]] && tokens[off + n[h]] == mask_id;
    sm[h] = sel[h] ? scores[off + n[h]] : -INFINITY;
  }
  int rank[2] = {0, 0};
#pragma unroll 4
  for (int l = 0; l < 64; ++l) {
    float other = __shfl_sync(0xffffffffu, l < 32 ? sm[0] : sm[1], l & 31);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int i = lane + 32 * h;
      rank[h] += (other > sm[h]) || (other == sm[h] && l < i);
    }
  }
  int count = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    bool c = sel[h] && rank[h] < q;
    chosen[off + n[h]] = c;
    count += c;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) count += __shfl_xor_sync(0xffffffffu, count, o);
  if (lane == 0 && count) atomicAdd(got + slot, count);
}

// Total order of (score descending, voxel index ascending) as one unsigned key. -0.0 and +0.0 compare equal in the
// reference's sort, so both map to the key of +0.0 and tie-break on the index.
__device__ __forceinline__ uint64_t order_key(float score, int n) {
  uint32_t u = score == 0.0f ? 0u : __float_as_uint(score);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (uint64_t(u) << 32) | uint64_t(0xFFFFFFFFu - uint32_t(n));
}

// Radix select over a 64-bit order key inside one CTA: the key of the c-th best candidate (c >= 1; with fewer than
// c candidates 0, so that every candidate is at or above it). Keys are unique (the voxel index is in the low word),
// so exactly min(c, candidates) candidates have key >= the result. 8-bit digits from the top; a digit whose bucket
// holds exactly the remaining count ends the search early.
template <typename Cand, typename Key>
__device__ uint64_t cta_select_key(int voxels, int c, Cand cand, Key key, uint32_t* hist, unsigned long long* sh) {
  const int t = threadIdx.x;
  unsigned long long& prefix = sh[0];
  unsigned long long& mask = sh[1];
  unsigned long long& rem = sh[2];
  unsigned long long& done = sh[3];
  if (t == 0) { prefix = 0; mask = 0; rem = (unsigned long long)c; done = 0; }
  __syncthreads();
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int i = t; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    if (!done) {
      for (int n = t; n < voxels; n += blockDim.x) {
        if (!cand(n)) continue;
        const uint64_t k = key(n);
        if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
      }
    }
    __syncthreads();
    if (t == 0 && !done) {
      unsigned long long acc = 0;
      int d = 255;
      for (; d >= 0; --d) {
        if (acc + hist[d] >= rem) break;
        acc += hist[d];
      }
      if (d < 0) {   // fewer candidates than c: all of them
        prefix = 0; mask = ~0ull; done = 1;
      } else {
        rem -= acc;
        prefix |= (unsigned long long)d << shift;
        mask |= 255ull << shift;
        if (hist[d] == rem) done = 1;   // the whole bucket is taken: its smallest key is the threshold
      }
    }
    __syncthreads();
  }
  const uint64_t result = prefix;
  __syncthreads();
  return result;
}

// Global trim / top-up (`block_quota.py:34-37`, `top_mask` `:4-12`) when the clamped block quotas miss k, then the
// ascending compaction of the chosen voxels (`nonzero_static`, `fast_ops.py:548`) and the quota check (`:540`).
// The fix-up is a radix select over the 64-bit key (score order, then lower voxel index first).
__global__ void __launch_bounds__(kSelectThreads) ease_fixup_compact_kernel(
    const float* __restrict__ scores, const int16_t* __restrict__ tokens, const uint8_t* __restrict__ last,
    const svx_step_params* __restrict__ params, int voxels, int mask_id, uint8_t* __restrict__ chosen,
    int32_t* __restrict__ got, int32_t* __restrict__ index_out, int index_capacity, int32_t* __restrict__ chosen_count,
    uint32_t* __restrict__ status) {
  const int slot = blockIdx.x;
  const int t = threadIdx.x;
  const int64_t off = (int64_t)slot * voxels;
  const int k = params[slot].k;
  const int have = got[slot];
  __shared__ uint32_t hist[256];
  __shared__ unsigned long long prefix, sel_sh[4];
  __shared__ int remaining, candidates;
  __shared__ int scan[kSelectThreads];
  if (k > 0 && have != k) {
    const bool trim = have > k;  // trim: keep the best k of the chosen; top-up: add the best k-have of the rest
    if (t == 0) { prefix = 0; remaining = trim ? k : k - have; candidates = 0; }
    __syncthreads();
    int mine = 0;
    for (int n = t; n < voxels; n += blockDim.x) {
      bool sel = !last[off + n] && tokens[off + n] == mask_id;
      bool cand = trim ? (bool)chosen[off + n] : (sel && !chosen[off + n]);
      mine += cand;
    }
    atomicAdd(&candidates, mine);
    __syncthreads();
    const bool take_all = remaining >= candidates;
    if (!take_all && remaining > 0) {
      auto cand = [&](int n) {
        const bool sel = !last[off + n] && tokens[off + n] == mask_id;
        return trim ? (bool)chosen[off + n] : (sel && !chosen[off + n]);
      };
      auto key = [&](int n) { return order_key(scores[off + n], n); };
      const uint64_t thr = cta_select_key(voxels, remaining, cand, key, hist, sel_sh);
      if (t == 0) prefix = thr;
      __syncthreads();
    }
    // prefix is now the key of the remaining-th best candidate; candidates at or above it are taken.
    for (int n = t; n < voxels; n += blockDim.x) {
      bool sel = !last[off + n] && tokens[off + n] == mask_id;
      bool cand = trim ? (bool)chosen[off + n] : (sel && !chosen[off + n]);
      bool take = cand && (take_all || (remaining > 0 && order_key(scores[off + n], n) >= prefix));
      if (trim && cand && !take) chosen[off + n] = 0;
      if (!trim && take) chosen[off + n] = 1;
    }
    __syncthreads();
  }
  // Ascending compaction: thread t owns voxels [t*per, (t+1)*per), read 16 flags per load when per % 16 == 0.
  const int per = (voxels + blockDim.x - 1) / blockDim.x;
  const int lo = min(voxels, t * per), hi = min(voxels, lo + per);
  const bool wide = per % 16 == 0 && voxels % per == 0 && (reinterpret_cast<uintptr_t>(chosen + off) & 15) == 0;
  int count = 0;
  bool bad = false;
  if (wide) {
    for (int n0 = lo; n0 < hi; n0 += 16) {
      const uint4 c = *reinterpret_cast<const uint4*>(chosen + off + n0);
      if (!(c.x | c.y | c.z | c.w)) continue;
      const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        count += (int)((w[q] * 0x01010101u) >> 24);   // flags are 0 or 1
        for (int b = 0; b < 4; ++b)
          if ((w[q] >> (8 * b)) & 0xFFu) {
            const int n = n0 + 4 * q + b;
            bad |= last[off + n] || tokens[off + n] != mask_id;
          }
      }
    }
  } else {
    for (int n = lo; n < hi; ++n) {
      if (chosen[off + n]) {
        ++count;
        bad |= last[off + n] || tokens[off + n] != mask_id;
      }
    }
  }
  scan[t] = count;
  __syncthreads();
  for (int s = 1; s < (int)blockDim.x; s <<= 1) {  // Hillis-Steele inclusive scan
    int v = t >= s ? scan[t - s] : 0;
    __syncthreads();
    scan[t] += v;
    __syncthreads();
  }
  int w = scan[t] - count;
  if (wide) {
    for (int n0 = lo; n0 < hi && count; n0 += 16) {
      const uint4 c = *reinterpret_cast<const uint4*>(chosen + off + n0);
      if (!(c.x | c.y | c.z | c.w)) continue;
      const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int q = 0; q < 4; ++q)
        for (int b = 0; b < 4; ++b)
          if ((wd[q] >> (8 * b)) & 0xFFu) {
            if (w < index_capacity) index_out[(int64_t)slot * index_capacity + w] = n0 + 4 * q + b;
            ++w;
          }
    }
  } else {
    for (int n = lo; n < hi; ++n)
      if (chosen[off + n]) {
        if (w < index_capacity) index_out[(int64_t)slot * index_capacity + w] = n;
        ++w;
      }
  }
  const int total = scan[blockDim.x - 1];
  for (int i = total + t; i < index_capacity; i += blockDim.x) index_out[(int64_t)slot * index_capacity + i] = -1;
  bad = __syncthreads_or(bad);
  if (t == 0) {
    chosen_count[slot] = total;
    got[slot] = total;
    if ((bad || total != k) && status) atomicOr(status + slot, SVX_STATUS_QUOTA_MISSED);
  }
}

// ----------------------------------------------------------------------------------------------- eval selection

// The evaluation decoders' selections (`streamvoxel/eval/samplers.py:23-64`), one CTA per slot over the masked voxels
// (tokens == mask_id): RANDOM/ENTROPY = top_mask of the draw / the score (`block_quota.py:4-12`: largest first, lower
// flat index on ties); MIXED = top k by score among the top `candidates` by draw (`samplers.py:23-28`); BLOCK = the
// linear block apportioning of `block_select` (`samplers.py:31-48`): target q (+1 for the first rem blocks of the
// seeded order) of the cumulative after = committed + k, quota = target - already committed, then the quota's
// best-scored masked voxels of each 4^3 block (stable descending); THRESHOLD = masked & draw < threshold (the
// native_quarter schedule, `samplers.py:98-101`). Then the ascending index list, the commit step of every chosen
// voxel, and the reference's assertions as SVX_STATUS_QUOTA_MISSED.
__global__ void __launch_bounds__(kSelectThreads) ease_eval_select_kernel(
    const float* __restrict__ scores, const float* __restrict__ draw, const int16_t* __restrict__ tokens,
    const int32_t* __restrict__ pos, const svx_eval_params* __restrict__ params, BlockGeom g, int mask_id,
    uint8_t* __restrict__ chosen, int32_t* __restrict__ index_out, int index_capacity, int32_t* __restrict__ count_out,
    int32_t* __restrict__ commit_step, int32_t* __restrict__ quota_range, uint32_t* __restrict__ status) {
  const int slot = blockIdx.x;
  const int t = threadIdx.x;
  const int voxels = g.height * g.depth * g.width;
  const int64_t off = (int64_t)slot * voxels;
  const svx_eval_params P = params[slot];
  const int16_t* tok = tokens + off;
  const float* sc = scores + off;
  const float* dr = draw + off;
  uint8_t* ch = chosen + off;
  __shared__ uint32_t hist[256];
  __shared__ unsigned long long sh[4];
  __shared__ int quota[kSelectThreads];
  __shared__ int scan[kSelectThreads];
  __shared__ int qsum, qmin, qmax, qbad;
  auto masked = [&](int n) { return tok[n] == mask_id; };
  bool bad = false;
  if (P.mode == SVX_EVAL_THRESHOLD) {
    for (int n = t; n < voxels; n += blockDim.x) ch[n] = masked(n) && dr[n] < P.threshold;
  } else if (P.mode == SVX_EVAL_RANDOM || P.mode == SVX_EVAL_ENTROPY || P.mode == SVX_EVAL_MIXED) {
    const float* first = P.mode != SVX_EVAL_ENTROPY ? dr : sc;
    const int c = P.mode == SVX_EVAL_MIXED ? P.candidates : P.k;
    auto key1 = [&](int n) { return order_key(first[n], n); };
    const uint64_t thr = c > 0 ? cta_select_key(voxels, c, masked, key1, hist, sh) : ~0ull;
    for (int n = t; n < voxels; n += blockDim.x) ch[n] = c > 0 && masked(n) && key1(n) >= thr;
    __syncthreads();
    if (P.mode == SVX_EVAL_MIXED) {   // the best k scores among the candidates
      auto cand = [&](int n) { return ch[n] != 0; };
      auto key2 = [&](int n) { return order_key(sc[n], n); };
      const uint64_t thr2 = P.k > 0 ? cta_select_key(voxels, P.k, cand, key2, hist, sh) : ~0ull;
      for (int n = t; n < voxels; n += blockDim.x) ch[n] = P.k > 0 && ch[n] && key2(n) >= thr2;
    }
  } else if (P.mode == SVX_EVAL_BLOCK) {
    if (t == 0) { qsum = 0; qmin = INT_MAX; qmax = INT_MIN; qbad = 0; }
    __syncthreads();
    const long long after = (long long)P.committed + P.k;
    const long long q = after / g.blocks, rem = after % g.blocks;
    for (int j = t; j < g.blocks; j += blockDim.x) {
      int legal = 0;
      for (int i = 0; i < 64; ++i) legal += masked(g.voxel(j, i));
      const long long target = q + (pos[(int64_t)slot * g.blocks + j] < rem ? 1 : 0);
      const long long qj = target - (64 - legal);
      if (qj < 0 || qj > legal) atomicOr(&qbad, 1);
      const int qc = (int)max(0ll, min(qj, (long long)legal));
      quota[j] = qc;
      atomicAdd(&qsum, qc);
      atomicMin(&qmin, (int)qj);
      atomicMax(&qmax, (int)qj);
    }
    __syncthreads();
    bad = qbad || qsum != P.k;
    // In-block ranking: a warp per block, voxel i chosen when fewer than quota masked voxels beat it.
    const int warp = warp_id(), lane = lane_id(), warps = blockDim.x >> 5;
    for (int j = warp; j < g.blocks; j += warps) {
      int n[2];
      float sm[2];
      bool sel[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        n[h] = g.voxel(j, lane + 32 * h);
        sel[h] = masked(n[h]);
        sm[h] = sel[h] ? sc[n[h]] : -INFINITY;
      }
      int rank[2] = {0, 0};
#pragma unroll 4
      for (int l = 0; l < 64; ++l) {
        const float other = __shfl_sync(0xffffffffu, l < 32 ? sm[0] : sm[1], l & 31);
#pragma unroll
        for (int h = 0; h < 2; ++h) rank[h] += (other > sm[h]) || (other == sm[h] && l < lane + 32 * h);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) ch[n[h]] = sel[h] && rank[h] < quota[j];
    }
    if (quota_range && t == 0) {
      quota_range[2 * slot] = qmin;
      quota_range[2 * slot + 1] = qmax;
    }
  } else {
    bad = true;
    for (int n = t; n < voxels; n += blockDim.x) ch[n] = 0;
  }
  __syncthreads();
  // Ascending compaction (thread t owns voxels [t*per, (t+1)*per)) and the commit step.
  const int per = (voxels + blockDim.x - 1) / blockDim.x;
  const int lo = min(voxels, t * per), hi = min(voxels, lo + per);
  int count = 0;
  for (int n = lo; n < hi; ++n) count += ch[n] != 0;
  scan[t] = count;
  __syncthreads();
  for (int s = 1; s < (int)blockDim.x; s <<= 1) {
    const int v = t >= s ? scan[t - s] : 0;
    __syncthreads();
    scan[t] += v;
    __syncthreads();
  }
  int w = scan[t] - count;
  for (int n = lo; n < hi; ++n)
    if (ch[n]) {
      if (w < index_capacity) index_out[(int64_t)slot * index_capacity + w] = n;
      if (commit_step && P.step) commit_step[off + n] = P.step;
      ++w;
    }
  const int total = scan[blockDim.x - 1];
  for (int i = total + t; i < index_capacity; i += blockDim.x) index_out[(int64_t)slot * index_capacity + i] = -1;
  bad = __syncthreads_or(bad);
  if (t == 0) {
    count_out[slot] = total;
    const bool exact = P.mode != SVX_EVAL_THRESHOLD;
    if ((bad || (exact && total != P.k) || total > index_capacity) && status)
      atomicOr(status + slot, SVX_STATUS_QUOTA_MISSED);
  }
}

// ----------------------------------------------------------------------------------------------- sampling

// Row softmax in torch's CUDA order (persistent warp softmax for rows of <= 1024 fp32 elements): W = min(npot, 32)
// lanes, element it*W + lane in register it, per-lane max then butterfly max, per-lane sum of expf(x - max) in
// register order then butterfly sum, p = e / sum.
template <int ITER>
__device__ __forceinline__ void torch_softmax_lane(const float (&x)[ITER], int width, float (&p)[ITER]) {
  float m = x[0];
#pragma unroll
  for (int it = 1; it < ITER; ++it) m = (m > x[it]) ? m : x[it];
  for (int o = width >> 1; o > 0; o >>= 1) {
    float b = __shfl_xor_sync(0xffffffffu, m, o, width);
    m = (m < b) ? b : m;
  }
  float s = 0.f;
  float e[ITER];
#pragma unroll
  for (int it = 0; it < ITER; ++it) {
    e[it] = expf(x[it] - m);
    s += e[it];
  }
  for (int o = width >> 1; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o, width);
#pragma unroll
  for (int it = 0; it < ITER; ++it) p[it] = e[it] / s;
}

__device__ __forceinline__ void argmax_merge(float& val, int& idx, float v2, int i2) {
  bool better = (v2 > val) || (v2 == val && i2 < idx) || (isnan(v2) && !isnan(val));
  if (better) { val = v2; idx = i2; }
}

template <typename T, int ITER>
__global__ void ease_sample_parity_kernel(const T* __restrict__ logits, int classes, int voxels, int64_t slot_stride,
                                          const int32_t* __restrict__ index, const svx_step_params* __restrict__ params,
                                          const float* __restrict__ noise, int64_t noise_slot_stride, int index_capacity,
                                          int width, int16_t* __restrict__ tokens, int16_t* __restrict__ values_out,
                                          uint32_t* __restrict__ status) {
  const int slot = blockIdx.y;
  const int warps = blockDim.x >> 5;
  const int i = blockIdx.x * warps + warp_id();
  const int k = params[slot].k;
  if (i >= k || i >= index_capacity) return;
  const int lane = lane_id();
  const int n = index[(int64_t)slot * index_capacity + i];
  if (n < 0) return;
  const T* col = logits + slot * slot_stride + n;
  const float* q = noise + slot * noise_slot_stride + (int64_t)i * classes;
  float x[ITER], p[ITER];
#pragma unroll
  for (int it = 0; it < ITER; ++it) {
    int c = it * width + lane;
    x[it] = (lane < width && c < classes) ? load_as_f32(col + (int64_t)c * voxels) : -INFINITY;
  }
  torch_softmax_lane<ITER>(x, width, p);
  float best = -INFINITY;
  int arg = 0x7fffffff;
  bool nan = false;
#pragma unroll
  for (int it = 0; it < ITER; ++it) {
    int c = it * width + lane;
    if (lane < width && c < classes) {
      float r = p[it] / q[c];
      nan |= isnan(p[it]);
      argmax_merge(best, arg, r, c);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float b = __shfl_xor_sync(0xffffffffu, best, o);
    int a = __shfl_xor_sync(0xffffffffu, arg, o);
    argmax_merge(best, arg, b, a);
  }
  nan = __any_sync(0xffffffffu, nan);
  if (lane == 0) {
    tokens[(int64_t)slot * voxels + n] = (int16_t)arg;
    values_out[(int64_t)slot * index_capacity + i] = (int16_t)arg;
    if (nan && status) atomicOr(status + slot, SVX_STATUS_NAN_LOGITS);
  }
}

// Philox4x32-10 (Salmon et al., SC 2011): ten rounds, key bumped by the Weyl constants between rounds.
__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) { k0 += 0x9E3779B9u; k1 += 0xBB67AE85u; }
    uint32_t hi0 = __umulhi(0xD2511F53u, c[0]), lo0 = 0xD2511F53u * c[0];
    uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]), lo1 = 0xCD9E8D57u * c[2];
    uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
  }
}

constexpr uint32_t kNativeStream = 0x53564F58u;

// Natural logarithm of a positive normal fp32 value from the atanh series: a = m 2^e with m in [sqrt(1/2), sqrt(2)),
// log a = e ln 2 + 2 atanh(s), s = (m - 1) / (m + 1), atanh(s) = s (1 + z/3 + z^2/5 + ... + z^5/11), z = s^2
// (|s| <= 0.1716, so the first omitted term is below 1e-10 relative). Every step is one IEEE round-to-nearest fp32
// operation (the __f*_rn intrinsics are never contracted into FMAs), so a host restatement that performs the same
// operations in the same order returns the same bits; that makes the native draw reproducible off the device.
__device__ __forceinline__ float series_log(float a) {
  int bits = __float_as_int(a);
  int e = (bits >> 23) - 127;
  int mbits = (bits & 0x007FFFFF) | 0x3F800000;
  if (mbits > 0x3FB504F3) {  // m > sqrt(2): halve m
    mbits -= 0x00800000;
    e += 1;
  }
  const float m = __int_as_float(mbits);
  const float s = __fdiv_rn(__fsub_rn(m, 1.f), __fadd_rn(m, 1.f));
  const float z = __fmul_rn(s, s);
  // 1/11, 1/9, 1/7, 1/5, 1/3 and ln 2, each the nearest fp32 value, written out in hexadecimal
  float t = 0x1.745d18p-4f;
  t = __fadd_rn(0x1.c71c72p-4f, __fmul_rn(z, t));
  t = __fadd_rn(0x1.24924ap-3f, __fmul_rn(z, t));
  t = __fadd_rn(0x1.99999ap-3f, __fmul_rn(z, t));
  t = __fadd_rn(0x1.555556p-2f, __fmul_rn(z, t));
  t = __fadd_rn(1.f, __fmul_rn(z, t));
  return __fadd_rn(__fmul_rn((float)e, 0x1.62e430p-1f), __fmul_rn(__fmul_rn(2.f, s), t));
}

// Native draw (Gumbel-max): argmax_v x_v - log E_v with E_v = -log u_v, which is distributed as
// multinomial(softmax(x), 1). u_v = (2 (w >> 9) + 1) 2^-24 (odd multiples of 2^-24, exactly representable, never 0
// or 1) from Philox keyed by (seed, step, voxel, class); the logs are `series_log`, the subtraction one fp32 op, ties
// go to the lower class. Lane L owns class groups g = L, L+32, ... of 4 consecutive classes, so each Philox call
// feeds 4 classes.
template <typename T>
__global__ void ease_sample_native_kernel(const T* __restrict__ logits, int classes, int voxels, int64_t slot_stride,
                                          const int32_t* __restrict__ index, const svx_step_params* __restrict__ params,
                                          int index_capacity, int16_t* __restrict__ tokens,
                                          int16_t* __restrict__ values_out, uint32_t* __restrict__ status) {
  const int slot = blockIdx.y;
  const int warps = blockDim.x >> 5;
  const int i = blockIdx.x * warps + warp_id();
  const svx_step_params p = params[slot];
  if (i >= p.k || i >= index_capacity) return;
  const int lane = lane_id();
  const int n = index[(int64_t)slot * index_capacity + i];
  if (n < 0) return;
  const T* col = logits + slot * slot_stride + n;
  const int groups = (classes + 3) >> 2;
  float best = -INFINITY;
  int arg = 0x7fffffff;
  bool nan = false;
  for (int g = lane; g < groups; g += 32) {
    uint32_t w[4] = {(uint32_t)g, (uint32_t)n, (uint32_t)p.step, kNativeStream};
    philox4x32_10(w, (uint32_t)p.seed, (uint32_t)(p.seed >> 32));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int c = g * 4 + j;
      if (c >= classes) break;
      const float u = (float)(((w[j] >> 9) << 1) | 1u) * 5.9604644775390625e-08f;  // 2^-24
      const float x = load_as_f32(col + (int64_t)c * voxels);
      nan |= isnan(x);
      argmax_merge(best, arg, __fsub_rn(x, series_log(-series_log(u))), c);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float b = __shfl_xor_sync(0xffffffffu, best, o);
    int a = __shfl_xor_sync(0xffffffffu, arg, o);
    argmax_merge(best, arg, b, a);
  }
  nan = __any_sync(0xffffffffu, nan);
  if (lane == 0) {
    tokens[(int64_t)slot * voxels + n] = (int16_t)arg;
    values_out[(int64_t)slot * index_capacity + i] = (int16_t)arg;
    if (nan && status) atomicOr(status + slot, SVX_STATUS_NAN_LOGITS);
  }
}

template <int ITER>
__global__ void softmax_rows_kernel(const float* __restrict__ x, int rows, int classes, int width,
                                    float* __restrict__ out) {
  const int row = blockIdx.x * (blockDim.x >> 5) + warp_id();
  if (row >= rows) return;
  const int lane = lane_id();
  float v[ITER], p[ITER];
#pragma unroll
  for (int it = 0; it < ITER; ++it) {
    int c = it * width + lane;
    v[it] = (lane < width && c < classes) ? x[(int64_t)row * classes + c] : -INFINITY;
  }
  torch_softmax_lane<ITER>(v, width, p);
#pragma unroll
  for (int it = 0; it < ITER; ++it) {
    int c = it * width + lane;
    if (lane < width && c < classes) out[(int64_t)row * classes + c] = p[it];
  }
}

__global__ void ease_finish_kernel(int16_t* __restrict__ tokens, const uint8_t* __restrict__ last,
                                   const uint8_t* __restrict__ finish, int voxels, int air_token) {
  const int slot = blockIdx.y;
  if (!finish[slot]) return;
  const int64_t off = (int64_t)slot * voxels;
  for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < voxels; n += gridDim.x * blockDim.x)
    if (last[off + n]) tokens[off + n] = (int16_t)air_token;
}

// Torch's persistent softmax geometry for a row of `classes` elements: lanes and registers per lane.
void softmax_geometry(int classes, int& width, int& iters) {
  int npot = 1;
  while (npot < classes) npot <<= 1;
  width = npot < 32 ? npot : 32;
  iters = npot / width;
}

template <typename T, int VPT, int SPLIT, int CH>
void launch_scores(const void* logits, int slots, int classes, int voxels, int64_t slot_stride, float* scores,
                   uint32_t* status, cudaStream_t s) {
  dim3 grid((voxels / VPT * SPLIT + kScoreThreads - 1) / kScoreThreads, slots);
  ease_scores_kernel<T, VPT, SPLIT, CH><<<grid, kScoreThreads, 0, s>>>(static_cast<const T*>(logits), classes,
                                                                       voxels, slot_stride, scores, status);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace svx

using namespace svx;

extern "C" int svx_ease_scores(const void* logits, int dtype, int slots, int classes, int voxels,
                               int64_t logit_slot_stride, float* scores, uint32_t* status, void* stream) {
  SVX_REQUIRE(logits && scores && slots > 0 && classes > 0 && voxels > 0, "svx_ease_scores: bad arguments");
  SVX_REQUIRE(aligned16(logits) && aligned16(scores), "svx_ease_scores: logits and scores must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  if (dtype == SVX_BF16) {
    SVX_REQUIRE(voxels % 8 == 0 && logit_slot_stride % 8 == 0, "svx_ease_scores: voxels must be a multiple of 8");
    launch_scores<uint16_t, kStatVoxels, kStatSplit, kStatRows>(logits, slots, classes, voxels, logit_slot_stride,
                                                                scores, status, s);
  } else if (dtype == SVX_F32) {
    SVX_REQUIRE(voxels % 4 == 0 && logit_slot_stride % 4 == 0, "svx_ease_scores: voxels must be a multiple of 4");
    launch_scores<float, kStatVoxels, kStatSplit, kStatRows>(logits, slots, classes, voxels, logit_slot_stride, scores,
                                                             status, s);
  } else {
    return fail(SVX_ERR_INVALID, "svx_ease_scores: dtype must be SVX_F32 or SVX_BF16");
  }
  return launch_status("ease_scores_kernel");
}

extern "C" int svx_ease_mark(const void* logits, int dtype, int slots, int classes, int height, int depth, int width,
                             int64_t logit_slot_stride, const int32_t* air_ids, int n_air, double last_eps,
                             uint8_t* last, int32_t* last_count, void* stream) {
  SVX_REQUIRE(height > 0 && depth > 0 && width > 0 && (int64_t)height * depth * width <= INT32_MAX,
              "svx_ease_mark: the column must hold between 1 and 2^31 - 1 voxels");
  const int voxels = height * depth * width;
  SVX_REQUIRE(logits && last && last_count && air_ids && n_air > 0 && slots > 0,
              "svx_ease_mark: bad arguments");
  SVX_REQUIRE(aligned16(logits), "svx_ease_mark: logits must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  const float threshold = (float)(1.0 - last_eps);  // torch compares the fp32 tensor with the scalar cast to fp32
  SVX_REQUIRE((reinterpret_cast<uintptr_t>(last) & 3u) == 0, "svx_ease_mark: last must be 4-byte aligned");
  dim3 grid((voxels / kStatVoxels * kStatSplit + kScoreThreads - 1) / kScoreThreads, slots);
  if (dtype == SVX_BF16) {
    SVX_REQUIRE(voxels % 8 == 0 && logit_slot_stride % 8 == 0, "svx_ease_mark: voxels must be a multiple of 8");
    ease_air_kernel<uint16_t, kStatVoxels, kStatSplit, kStatRows><<<grid, kScoreThreads, 0, s>>>(
        static_cast<const uint16_t*>(logits), classes, voxels, logit_slot_stride, air_ids, n_air, threshold, last);
  } else if (dtype == SVX_F32) {
    SVX_REQUIRE(voxels % 4 == 0 && logit_slot_stride % 4 == 0, "svx_ease_mark: voxels must be a multiple of 4");
    ease_air_kernel<float, kStatVoxels, kStatSplit, kStatRows><<<grid, kScoreThreads, 0, s>>>(
        static_cast<const float*>(logits), classes, voxels, logit_slot_stride, air_ids, n_air, threshold, last);
  } else {
    return fail(SVX_ERR_INVALID, "svx_ease_mark: dtype must be SVX_F32 or SVX_BF16");
  }
  int rc = launch_status("ease_air_kernel");
  if (rc) return rc;
  ease_column_run_kernel<<<slots, 256, 0, s>>>(last, height, depth * width, last_count);
  return launch_status("ease_column_run_kernel");
}

extern "C" size_t svx_ease_select_workspace_bytes(int slots, int voxels) {
  return (size_t)slots * (voxels / 64 + 1) * sizeof(int32_t);
}

extern "C" int svx_ease_select(const float* scores, const int16_t* tokens, const uint8_t* last, const int32_t* pos,
                               const svx_step_params* params, int slots, int height, int depth, int width, int block,
                               int mask_id, uint8_t* chosen, int32_t* index_out, int index_capacity,
                               int32_t* chosen_count, uint32_t* status, void* workspace, void* stream) {
  SVX_REQUIRE(block == 4, "svx_ease_select: only 4^3 blocks are implemented");
  SVX_REQUIRE(height % 4 == 0 && depth % 4 == 0 && width % 4 == 0 && height > 0 && depth > 0 && width > 0,
              "svx_ease_select: shape must be a positive multiple of 4");
  SVX_REQUIRE((int64_t)height * depth * width <= (int64_t)kSelectThreads * 64,
              "svx_ease_select: at most 1024 blocks per column");
  const int voxels = height * depth * width;
  BlockGeom g{height, depth, width, depth / 4, width / 4, voxels / 64};
  SVX_REQUIRE(g.blocks <= kSelectThreads, "svx_ease_select: at most 1024 blocks per column");
  SVX_REQUIRE(scores && tokens && last && pos && params && chosen && index_out && chosen_count && workspace &&
                  slots > 0 && index_capacity > 0,
              "svx_ease_select: bad arguments");
  SVX_REQUIRE((reinterpret_cast<uintptr_t>(tokens) & 7) == 0 && (reinterpret_cast<uintptr_t>(last) & 3) == 0,
              "svx_ease_select: tokens must be 8-byte and last 4-byte aligned");
  cudaStream_t s = as_stream(stream);
  int32_t* quota = static_cast<int32_t*>(workspace);
  int32_t* got = quota + (size_t)slots * g.blocks;
  ease_quota_kernel<<<slots, kSelectThreads, 0, s>>>(tokens, last, pos, params, g, mask_id, quota, got);
  int rc = launch_status("ease_quota_kernel");
  if (rc) return rc;
  const int warps = 8;
  dim3 grid((g.blocks + warps - 1) / warps, slots);
  ease_block_select_kernel<<<grid, warps * 32, 0, s>>>(scores, tokens, last, quota, params, g, mask_id, chosen, got);
  rc = launch_status("ease_block_select_kernel");
  if (rc) return rc;
  ease_fixup_compact_kernel<<<slots, kSelectThreads, 0, s>>>(scores, tokens, last, params, voxels, mask_id, chosen, got,
                                                            index_out, index_capacity, chosen_count, status);
  return launch_status("ease_fixup_compact_kernel");
}

extern "C" int svx_eval_select(const float* scores, const float* draw, const int16_t* tokens, const int32_t* pos,
                               const svx_eval_params* params, int slots, int height, int depth, int width,
                               int mask_id, uint8_t* chosen, int32_t* index_out, int index_capacity,
                               int32_t* chosen_count, int32_t* commit_step, int32_t* quota_range, uint32_t* status,
                               void* stream) {
  SVX_REQUIRE(scores && draw && tokens && pos && params && chosen && index_out && chosen_count && slots > 0 &&
                  index_capacity > 0,
              "svx_eval_select: bad arguments (scores, draw and pos are required whatever the mode)");
  SVX_REQUIRE(height % 4 == 0 && depth % 4 == 0 && width % 4 == 0 && height > 0 && depth > 0 && width > 0,
              "svx_eval_select: the column must tile by 4^3 blocks");
  SVX_REQUIRE((int64_t)height * depth * width <= (int64_t)kSelectThreads * 64,
              "svx_eval_select: at most 1024 blocks per column");
  BlockGeom g{height, depth, width, depth / 4, width / 4, (height / 4) * (depth / 4) * (width / 4)};
  SVX_REQUIRE(g.blocks <= kSelectThreads, "svx_eval_select: at most 1024 blocks per column");
  ease_eval_select_kernel<<<slots, kSelectThreads, 0, as_stream(stream)>>>(
      scores, draw, tokens, pos, params, g, mask_id, chosen, index_out, index_capacity, chosen_count, commit_step,
      quota_range, status);
  return launch_status("ease_eval_select_kernel");
}

template <typename T>
static int launch_parity(const T* logits, int classes, int voxels, int64_t stride, const int32_t* index,
                         const svx_step_params* params, const float* noise, int64_t noise_stride, int cap, int slots,
                         int16_t* tokens, int16_t* values, uint32_t* status, cudaStream_t s) {
  int width, iters;
  softmax_geometry(classes, width, iters);
  const int warps = 8;
  dim3 grid((cap + warps - 1) / warps, slots);
#define SVX_PARITY(I)                                                                                            \
  case I:                                                                                                        \
    ease_sample_parity_kernel<T, I><<<grid, warps * 32, 0, s>>>(logits, classes, voxels, stride, index, params,  \
                                                                noise, noise_stride, cap, width, tokens, values, \
                                                                status);                                         \
    break;
  switch (iters) {
    SVX_PARITY(1) SVX_PARITY(2) SVX_PARITY(4) SVX_PARITY(8) SVX_PARITY(16) SVX_PARITY(32)
    default: return fail(SVX_ERR_INVALID, "svx_ease_sample: at most 1024 classes");
  }
#undef SVX_PARITY
  return launch_status("ease_sample_parity_kernel");
}

extern "C" int svx_ease_sample(const void* logits, int dtype, int slots, int classes, int voxels,
                               int64_t logit_slot_stride, const int32_t* index, const svx_step_params* params,
                               const float* noise, int64_t noise_slot_stride, int index_capacity, int16_t* tokens,
                               int16_t* values_out, uint32_t* status, void* stream) {
  SVX_REQUIRE(logits && index && params && tokens && values_out && slots > 0 && classes > 0 && classes <= 1024 &&
                  index_capacity > 0,
              "svx_ease_sample: bad arguments");
  cudaStream_t s = as_stream(stream);
  if (noise) {
    if (dtype == SVX_BF16)
      return launch_parity(static_cast<const uint16_t*>(logits), classes, voxels, logit_slot_stride, index, params,
                           noise, noise_slot_stride, index_capacity, slots, tokens, values_out, status, s);
    if (dtype == SVX_F32)
      return launch_parity(static_cast<const float*>(logits), classes, voxels, logit_slot_stride, index, params, noise,
                           noise_slot_stride, index_capacity, slots, tokens, values_out, status, s);
    return fail(SVX_ERR_INVALID, "svx_ease_sample: dtype must be SVX_F32 or SVX_BF16");
  }
  const int warps = 8;
  dim3 grid((index_capacity + warps - 1) / warps, slots);
  if (dtype == SVX_BF16)
    ease_sample_native_kernel<uint16_t><<<grid, warps * 32, 0, s>>>(static_cast<const uint16_t*>(logits), classes,
                                                                   voxels, logit_slot_stride, index, params,
                                                                   index_capacity, tokens, values_out, status);
  else if (dtype == SVX_F32)
    ease_sample_native_kernel<float><<<grid, warps * 32, 0, s>>>(static_cast<const float*>(logits), classes, voxels,
                                                                logit_slot_stride, index, params, index_capacity,
                                                                tokens, values_out, status);
  else
    return fail(SVX_ERR_INVALID, "svx_ease_sample: dtype must be SVX_F32 or SVX_BF16");
  return launch_status("ease_sample_native_kernel");
}

extern "C" int svx_softmax_rows(const float* x, int rows, int classes, float* out, void* stream) {
  SVX_REQUIRE(x && out && rows > 0 && classes > 0 && classes <= 1024, "svx_softmax_rows: bad arguments");
  int width, iters;
  softmax_geometry(classes, width, iters);
  const int warps = 8;
  const int grid = (rows + warps - 1) / warps;
  cudaStream_t s = as_stream(stream);
  switch (iters) {
    case 1: softmax_rows_kernel<1><<<grid, warps * 32, 0, s>>>(x, rows, classes, width, out); break;
    case 2: softmax_rows_kernel<2><<<grid, warps * 32, 0, s>>>(x, rows, classes, width, out); break;
    case 4: softmax_rows_kernel<4><<<grid, warps * 32, 0, s>>>(x, rows, classes, width, out); break;
    case 8: softmax_rows_kernel<8><<<grid, warps * 32, 0, s>>>(x, rows, classes, width, out); break;
    case 16: softmax_rows_kernel<16><<<grid, warps * 32, 0, s>>>(x, rows, classes, width, out); break;
    case 32: softmax_rows_kernel<32><<<grid, warps * 32, 0, s>>>(x, rows, classes, width, out); break;
    default: return fail(SVX_ERR_INVALID, "svx_softmax_rows: at most 1024 classes");
  }
  return launch_status("softmax_rows_kernel");
}

extern "C" int svx_ease_finish(int16_t* tokens, const uint8_t* last, const uint8_t* finish, int slots, int voxels,
                               int air_token, void* stream) {
  SVX_REQUIRE(tokens && last && finish && slots > 0 && voxels > 0, "svx_ease_finish: bad arguments");
  dim3 grid(64, slots);
  ease_finish_kernel<<<grid, 256, 0, as_stream(stream)>>>(tokens, last, finish, voxels, air_token);
  return launch_status("ease_finish_kernel");
}

// ------------------------------------------------------------------------------------- selection without allocation
//
// Some hosts cannot give this library device memory for its selection scratch: a plugin whose process leaves all
// device memory to another framework's pool, or a caller inside a region where allocating would synchronise the
// device. For them svx_ease_select_noalloc runs the same three selection kernels on a fixed scratch array that lives
// in the library's own device image. Every GPU that loads the library holds this array until the process exits.
#include <mutex>

namespace svx {
namespace {
constexpr int kNoAllocMaxSlots = 64;
constexpr int kNoAllocMaxBlocks = kSelectThreads;  // 4^3 blocks per column, as svx_ease_select allows
}  // namespace
}  // namespace svx

// Per-call scratch of the selection: block quotas [slots][blocks] and per-slot counters [slots] (int32).
// 64 * (1024 + 1) * 4 = 262,400 bytes on each device.
static __device__ __align__(256) int32_t g_select_scratch[svx::kNoAllocMaxSlots * (svx::kNoAllocMaxBlocks + 1)];

namespace svx {
namespace {
PerDevice<void*> g_scratch_address;

// Device address of g_select_scratch on the current device, looked up once per device (the address stays valid while
// the device's primary context lives, which is why the library does not support a device reset). In host code the
// array's name only stands in for the symbol; a kernel must be given the address cudaGetSymbolAddress returns.
int scratch_address(void** out) {
  return g_scratch_address.get(out, [](int, void** address) -> int {
    cudaError_t e = cudaGetSymbolAddress(address, g_select_scratch);
    if (e != cudaSuccess)
      return fail(SVX_ERR_CUDA, std::string("svx_ease_select_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    return SVX_OK;
  });
}
}  // namespace
}  // namespace svx

extern "C" int svx_ease_select_noalloc(const float* scores, const int16_t* tokens, const uint8_t* last,
                                       const int32_t* pos, const svx_step_params* params, int slots, int height,
                                       int depth, int width, int block, int mask_id, uint8_t* chosen,
                                       int32_t* index_out, int index_capacity, int32_t* chosen_count,
                                       uint32_t* status, void* stream) {
  SVX_REQUIRE(slots > 0 && slots <= kNoAllocMaxSlots,
              "svx_ease_select_noalloc: at most 64 slots per call (the fixed scratch holds 64 x 1025 int32)");
  SVX_REQUIRE(height > 0 && depth > 0 && width > 0 && height % 4 == 0 && depth % 4 == 0 && width % 4 == 0 &&
                  (int64_t)(height / 4) * (depth / 4) * (width / 4) <= kNoAllocMaxBlocks,
              "svx_ease_select_noalloc: at most 1024 4^3 blocks per column");
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  // The first selection kernel zeroes the per-slot counters and writes every block quota before the later kernels
  // read them, so nothing left in the array by an earlier call is ever read.
  return svx_ease_select(scores, tokens, last, pos, params, slots, height, depth, width, block, mask_id, chosen,
                         index_out, index_capacity, chosen_count, status, scratch, stream);
}
