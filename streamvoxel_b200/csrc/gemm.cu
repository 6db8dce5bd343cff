// Dense bf16 GEMM with fused epilogues on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA.
//
// D[M,N] = A[M,K] . W[N,K]^T, both operands K-major (activations row-major, nn.Linear weights as stored).
// One 128 x BN output tile per CTA. Warp roles: warp 0 issues TMA loads into a STAGES-deep shared-memory ring
// (128B-swizzled tiles), warp 1 allocates TMEM and one elected thread issues tcgen05.mma (M=128, N=BN, K=16) into an
// fp32 TMEM accumulator, committing each stage back to the producer; warps 2-5 wait for the final commit, read the
// accumulator with tcgen05.ld (each warp owns its 32-lane TMEM quarter = 32 output rows) and run the epilogue.
// Every mbarrier wait is bounded; a timeout sets SVX_STATUS_WAIT_TIMEOUT in g_svx_timeouts and skips the work.
#include <cuda.h>
#include <math.h>

#include "common.cuh"
#include "gemm.cuh"

namespace svx {

__device__ uint32_t g_svx_timeouts = 0;

namespace {

constexpr int BM = 128, BK = 64;
constexpr int kThreads = 192;
constexpr uint32_t A_BYTES = BM * BK * 2;

__device__ __forceinline__ void record_timeout() { atomicOr(&g_svx_timeouts, SVX_STATUS_WAIT_TIMEOUT); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

// UMMA shared-memory descriptor of a K-major tile in the canonical 128B-swizzle layout (8-row atoms of 128 B,
// 1024 B apart): start address >> 4, LBO = 1 (unused for swizzled K-major), SBO = 1024 B, version 1, SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t instr_desc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void load_bf16x32(const uint16_t* p, float (&v)[32]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 raw = q[i];
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
      v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  }
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return (uint32_t)f32_to_bf16(lo) | ((uint32_t)f32_to_bf16(hi) << 16);
}

__device__ __forceinline__ void store_bf16x32(uint16_t* p, const float (&v)[32]) {
  uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    q[i] = make_uint4(pack2(v[8 * i], v[8 * i + 1]), pack2(v[8 * i + 2], v[8 * i + 3]),
                      pack2(v[8 * i + 4], v[8 * i + 5]), pack2(v[8 * i + 6], v[8 * i + 7]));
}

// GELU (erf form), in the operation order of ATen's GeluCUDAKernelImpl: x * 0.5 * (1 + erf(x * sqrt(1/2))).
__device__ __forceinline__ float gelu_erf(float x) { return x * 0.5f * (1.0f + erff(x * 0.70710678118654752440f)); }

// Epilogue of one row x 32 columns [n, n+32) of the tile; acc holds fp32 accumulators.
template <int EPI>
__device__ __forceinline__ void epilogue32(const EpiParams& ep, uint16_t* out, int N, int row, int n,
                                           const uint32_t (&acc)[32]) {
  float bias[32], y[32];
  load_bf16x32(ep.bias + n, bias);
#pragma unroll
  for (int j = 0; j < 32; ++j) y[j] = round_bf16(__uint_as_float(acc[j]) + bias[j]);
  if constexpr (EPI == SVX_EPI_BIAS_GELU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) y[j] = gelu_erf(y[j]);
  } else if constexpr (EPI == SVX_EPI_GATE_RESIDUAL || EPI == SVX_EPI_RESIDUAL) {
    float res[32];
    load_bf16x32(ep.residual + (int64_t)row * N + n, res);
    if constexpr (EPI == SVX_EPI_GATE_RESIDUAL) {
      float gate[32];
      load_bf16x32(ep.gate + n, gate);
#pragma unroll
      for (int j = 0; j < 32; ++j) y[j] = round_bf16(gate[j] * y[j]);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) y[j] = res[j] + y[j];
  } else if constexpr (EPI == SVX_EPI_ROPE) {
    if (n < ep.rope_cols) {
      // Axial RoPE (`unconditional_md4_timefree.py:24-30`): pair (2f, 2f+1) of a head rotates by table entry f;
      // a*cos, b*sin, ... are bf16 ops, so every product and sum rounds to bf16.
      const int p = row % ep.rows_per_slot;
      const int half = ep.head_dim >> 1;
      const int dim0 = n % ep.head_dim;
      const uint16_t* sn = ep.rope_sin + (int64_t)p * half + (dim0 >> 1);
      const uint16_t* cs = ep.rope_cos + (int64_t)p * half + (dim0 >> 1);
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float s = bf16_to_f32(sn[j >> 1]), c = bf16_to_f32(cs[j >> 1]);
        float a = y[j], b = y[j + 1];
        y[j] = round_bf16(round_bf16(a * c) - round_bf16(b * s));
        y[j + 1] = round_bf16(round_bf16(a * s) + round_bf16(b * c));
      }
    }
  }
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
      const int o = o0 + j;
      const int oy = o >> 4, oz = (o >> 2) & 3;
      const int64_t idx = ((int64_t)(py * P + oy) * ep.depth + (pz * P + oz)) * ep.width + px * P;
      *reinterpret_cast<uint2*>(base + idx) = make_uint2(pack2(y[j], y[j + 1]), pack2(y[j + 2], y[j + 3]));
    }
  } else {
    store_bf16x32(out + (int64_t)row * N + n, y);
  }
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                           const __grid_constant__ CUtensorMap tmB,
                                                           uint16_t* __restrict__ out, int M, int N, int K,
                                                           const EpiParams ep) {
  constexpr uint32_t B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_s = smem;
  uint8_t* b_s = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(b_s + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = warp_id(), lane = lane_id();
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int kblocks = K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    mbar_init(accum, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < kblocks; ++kb) {
        const int s = kb % STAGES, round = kb / STAGES;
        if (round > 0 && !mbar_wait(empty + s, (round - 1) & 1)) { *abort_flag = 1; record_timeout(); break; }
        if (*abort_flag) break;
        mbar_expect_tx(full + s, A_BYTES + B_BYTES);
        tma_load_2d(a_s + s * A_BYTES, &tmA, kb * BK, m0, full + s);
        tma_load_2d(b_s + s * B_BYTES, &tmB, kb * BK, n0, full + s);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(BN);
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        const int s = kb % STAGES, round = kb / STAGES;
        if (!mbar_wait(full + s, round & 1)) { *abort_flag = 1; record_timeout(); ok = false; break; }
        fence_after();
        const uint32_t a0 = smem_addr(a_s + s * A_BYTES), b0 = smem_addr(b_s + s * B_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          umma(tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), idesc, (kb | kk) != 0);
        umma_commit(empty + s);
      }
      if (ok) umma_commit(accum);
    }
  } else {
    // Epilogue warps 2..5: TMEM lane quarter (warp % 4) holds rows 32*(warp%4) .. +31 of the tile.
    const int quarter = warp & 3;
    const int row = m0 + quarter * 32 + lane;
    if (mbar_wait(accum, 0)) {
      fence_after();
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t acc[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(c * 32), acc);
        if (row < M) epilogue32<EPI>(ep, out, N, row, n0 + c * 32, acc);
      }
    } else {
      record_timeout();
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

template <int BN, int STAGES>
constexpr size_t smem_bytes() {
  return 1024 + STAGES * (A_BYTES + (size_t)BN * BK * 2) + (2 * STAGES + 1) * 8 + 16;
}

template <int BN, int STAGES, int EPI>
int launch_tile(const CUtensorMap& a, const CUtensorMap& b, uint16_t* out, int M, int N, int K, const EpiParams& ep,
                cudaStream_t stream) {
  constexpr size_t bytes = smem_bytes<BN, STAGES>();
  static bool configured = false;
  if (!configured) {
    SVX_CHECK_CUDA(cudaFuncSetAttribute(gemm_kernel<BN, STAGES, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)bytes));
    configured = true;
  }
  dim3 grid(N / BN, M / BM);
  gemm_kernel<BN, STAGES, EPI><<<grid, kThreads, bytes, stream>>>(a, b, out, M, N, K, ep);
  return launch_status("gemm_kernel");
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
                uint64_t group_stride_bytes, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows) {
  EncodeTiled encode = encode_fn();
  if (!encode) return fail(SVX_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  SVX_REQUIRE((reinterpret_cast<uintptr_t>(ptr) & 15u) == 0, "TMA operand must be 16-byte aligned");
  SVX_REQUIRE(group_stride_bytes % 16 == 0 && row_stride_bytes % 16 == 0, "TMA strides must be multiples of 16 bytes");
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)groups, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)group_stride_bytes, (cuuint64_t)row_stride_bytes};
  cuuint32_t box[3] = {box_inner, 1, box_rows};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, elem,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SVX_ERR_CUDA, "cuTensorMapEncodeTiled (3d) failed: " + std::to_string((int)r));
  return SVX_OK;
}

static int pick_bn(int M, int N) {
  if (N % 256 == 0 && (long)(N / 256) * (M / BM) >= 148) return 256;
  if (N % 128 == 0) return 128;
  return 64;
}

int gemm_plan(GemmPlan* plan, const uint16_t* A, const uint16_t* W, int M, int N, int K, int bn) {
  SVX_REQUIRE(M > 0 && M % BM == 0, "gemm: M must be a positive multiple of 128");
  SVX_REQUIRE(N > 0 && N % 64 == 0 && K > 0 && K % BK == 0, "gemm: N and K must be multiples of 64");
  plan->M = M; plan->N = N; plan->K = K;
  plan->bn = bn > 0 ? bn : pick_bn(M, N);
  SVX_REQUIRE(N % plan->bn == 0, "gemm: N must be a multiple of the tile width");
  int rc = make_kmajor_map(&plan->a, A, M, K, BM);
  if (rc) return rc;
  return make_kmajor_map(&plan->b, W, N, K, plan->bn);
}

int gemm_run(const GemmPlan& plan, int M, uint16_t* out, const EpiParams& ep, cudaStream_t stream) {
  SVX_REQUIRE(M > 0 && M <= plan.M && M % BM == 0, "gemm: run rows must be a multiple of 128 within the plan");
  switch (ep.epilogue) {
    case SVX_EPI_BIAS: return launch_epi<SVX_EPI_BIAS>(plan.a, plan.b, plan.bn, out, M, plan.N, plan.K, ep, stream);
    case SVX_EPI_BIAS_GELU:
      return launch_epi<SVX_EPI_BIAS_GELU>(plan.a, plan.b, plan.bn, out, M, plan.N, plan.K, ep, stream);
    case SVX_EPI_GATE_RESIDUAL:
      return launch_epi<SVX_EPI_GATE_RESIDUAL>(plan.a, plan.b, plan.bn, out, M, plan.N, plan.K, ep, stream);
    case SVX_EPI_RESIDUAL:
      return launch_epi<SVX_EPI_RESIDUAL>(plan.a, plan.b, plan.bn, out, M, plan.N, plan.K, ep, stream);
    case SVX_EPI_ROPE: return launch_epi<SVX_EPI_ROPE>(plan.a, plan.b, plan.bn, out, M, plan.N, plan.K, ep, stream);
    case SVX_EPI_CLASS_MAJOR:
      return launch_epi<SVX_EPI_CLASS_MAJOR>(plan.a, plan.b, plan.bn, out, M, plan.N, plan.K, ep, stream);
    default: return fail(SVX_ERR_INVALID, "gemm: unknown epilogue");
  }
}

int epi_from_args(const svx_epilogue_args* e, EpiParams* ep, int N) {
  SVX_REQUIRE(e && e->bias, "gemm: epilogue needs a bias");
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
  int rc = epi_from_args(epi, &ep, N);
  if (rc) return rc;
  GemmPlan plan;
  rc = gemm_plan(&plan, A, W, M, N, K, 0);
  if (rc) return rc;
  return gemm_run(plan, M, out, ep, as_stream(stream));
}

extern "C" uint32_t svx_wait_timeouts(void) {
  uint32_t v = 0;
  if (cudaMemcpyFromSymbol(&v, g_svx_timeouts, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
  return v | attention_timeouts();
}
