// Projection GEMMs of the decode step on tcgen05:  D[M, N] = A[M, K] . B[N, K]^T  (bf16 in,
// fp32 accumulate in TMEM, bf16 out) — the nn.Linear products of the Qwen3 layers
// (mini_vllm/layers/linear.py: qkv_proj, o_proj, gate_up_proj, down_proj, and the LM head,
// embed_head.py:56-66), where A is the activation (M = the decode batch, <= a few hundred rows)
// and B the weight in its checkpoint layout [out_features, in_features].
//
// Tile: 128 rows of A x BN rows of B, K in 64-element steps (one 128-byte swizzle atom), both
// operands K-major straight from TMA; one thread issues tcgen05.mma (M = 128, N = BN, K = 16) into
// a BN-column TMEM accumulator.  With few output tiles (N = 1024 projections at M = 256) the K
// range is split over CTAs and the last CTA of a tile adds the fp32 partials (ticket).
// Epilogues: plain bf16 store, or SiLU(gate) * up when B holds the gate rows [0, N) and the up
// rows [N, 2N) (MergedColumnParallelLinear + SiluAndMul, activation.py:12-16): each CTA then
// accumulates both halves for its columns and writes the activated product only.
//
// Programmatic dependent launch: the kernel lets its successor launch early and waits for its
// predecessor (griddepcontrol) only before reading A, so the first weight tiles stream in while
// the previous kernel drains.
#include "hl_common.cuh"

#include <cuda.h>

namespace hl {
namespace {

constexpr int kGBM = 128;
constexpr int kGBK = 64;
constexpr int kGThreads = 192;  // warp 0 TMA, warp 1 TMEM + MMA, warps 2-5 epilogue
constexpr int kGATile = kGBM * kGBK * 2;  // 16 KiB

template <int BN, bool SILU>
struct GemmCfg {
  static constexpr int kBRows = SILU ? 2 * BN : BN;           // gate + up rows for SILU
  static constexpr int kBTile = kBRows * kGBK * 2;
  static constexpr int kStageBytes = kGATile + kBTile;
  static constexpr int kStages = (200 * 1024) / kStageBytes < 8 ? (200 * 1024) / kStageBytes : 8;
  static constexpr int kOffBar = kStages * kStageBytes;
  static constexpr int kSmem = kOffBar + 256 + 1024;
  static constexpr uint32_t kTmemCols = SILU ? 2 * BN : BN;   // accumulator columns
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t(BN) >> 3) << 17) |
                                     ((uint32_t(kGBM) >> 4) << 24);
  static_assert(kStageBytes % 1024 == 0, "stages must keep 1024-byte alignment");
};

struct GemmParams {
  CUtensorMap ta;
  CUtensorMap tb;
  __nv_bfloat16* d;
  int64_t ldd;
  int M, N, K;
  int splits;      // K split over gridDim.z
  int silu_rows;   // SILU: row offset of the up half in B (= N)
  float* partial;  // split-K fp32 partial tiles
  int* tickets;
  int* err;
};

__device__ __forceinline__ uint64_t gdesc(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t(1) << 16;            // leading byte offset (unused for swizzled K-major)
  d |= uint64_t(1024 >> 4) << 32;    // 8 rows x 128 B between row groups
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;            // 128-byte swizzle
  return d;
}

__device__ __forceinline__ void tma2(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void g_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void g_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void g_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ float silu_mul(float g, float u) {
  // bf16(bf16(silu(g)) * u): the reference's SiluAndMul rounding (silu output is bf16 first)
  const float gb = __bfloat162float(__float2bfloat16_rn(g));
  const float ub = __bfloat162float(__float2bfloat16_rn(u));
  const float s = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(gb, __fadd_rn(1.0f, expf(-gb)))));
  return __fmul_rn(s, ub);
}

template <int BN, bool SILU>
__global__ void __launch_bounds__(kGThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmParams p) {
  using C = GemmCfg<BN, SILU>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* full = bars;                  // [kStages]
  uint64_t* empty = bars + C::kStages;    // [kStages]
  uint64_t* acc_full = bars + 2 * C::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * C::kStages + 1);
  int* flag = reinterpret_cast<int*>(bars + 2 * C::kStages + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN;
  const int m0 = blockIdx.y * kGBM;
  const int split = blockIdx.z;
  const int nk = p.K / kGBK;
  const int kb0 = int(int64_t(nk) * split / p.splits);
  const int kb1 = int(int64_t(nk) * (split + 1) / p.splits);
  const int nkb = kb1 - kb0;

  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && nkb > 0) {
      auto load_b = [&](int i) {
        const uint32_t st = sbase + (i % C::kStages) * C::kStageBytes + kGATile;
        const uint32_t bar = smem_u32(&full[i % C::kStages]);
        tma2(st, &p.tb, (kb0 + i) * kGBK, n0, bar);
        if constexpr (SILU) tma2(st + BN * kGBK * 2, &p.tb, (kb0 + i) * kGBK, p.silu_rows + n0, bar);
      };
      // Weights do not depend on the previous kernel: fetch the first stages before waiting.
      const int pre = nkb < C::kStages ? nkb : C::kStages;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], C::kStageBytes);
        load_b(i);
      }
      pdl_wait();
      for (int i = 0; i < nkb; ++i) {
        const int st = i % C::kStages;
        if (i >= C::kStages) {
          if (!mbar_wait(&empty[st], ((i / C::kStages) - 1) & 1)) {
            atomicOr(p.err, 1);
            break;
          }
          mbar_arrive_expect_tx(&full[st], C::kStageBytes);
          load_b(i);
        }
        tma2(sbase + st * C::kStageBytes, &p.ta, (kb0 + i) * kGBK, m0, smem_u32(&full[st]));
      }
    } else if (nkb > 0) {
      pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0 && nkb > 0) {
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        const int st = i % C::kStages;
        if (!mbar_wait(&full[st], (i / C::kStages) & 1)) {
          atomicOr(p.err, 1);
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a = sbase + st * C::kStageBytes;
        const uint32_t b = a + kGATile;
#pragma unroll
        for (int kk = 0; kk < kGBK / 16; ++kk) {
          g_mma(tmem, gdesc(a + kk * 32), gdesc(b + kk * 32), C::kIdesc, (i > 0 || kk > 0) ? 1u : 0u);
          if constexpr (SILU)
            g_mma(tmem + BN, gdesc(a + kk * 32), gdesc(b + BN * kGBK * 2 + kk * 32), C::kIdesc,
                  (i > 0 || kk > 0) ? 1u : 0u);
        }
        g_commit(smem_u32(&empty[st]));
      }
      g_commit(smem_u32(acc_full));
      if (!ok) mbar_wait(acc_full, 0);
    }
  } else {
    pdl_wait();
    // Epilogue: thread = output row (TMEM lane); columns in chunks of 16.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int row = m0 + r;
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    const bool have = nkb > 0 && mbar_wait(acc_full, 0);
    if (nkb > 0 && !have) atomicOr(p.err, 1);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    if (p.splits == 1) {
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        float v[16];
        g_ld16(lane_base + c, v);
        if constexpr (SILU) {
          float u[16];
          g_ld16(lane_base + BN + c, u);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = silu_mul(v[i], u[i]);
        }
        if (row < p.M && n0 + c < p.N) {
          __nv_bfloat16* dst = p.d + int64_t(row) * p.ldd + n0 + c;
          if (n0 + c + 16 <= p.N) {
            uint32_t w[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
              w[i] = *reinterpret_cast<uint32_t*>(&h);
            }
            reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
            reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
          } else {
            for (int i = 0; i < 16 && n0 + c + i < p.N; ++i) dst[i] = __float2bfloat16_rn(v[i]);
          }
        }
      }
    } else {
      // Split K: publish this CTA's fp32 tile, the last CTA of the tile sums and stores.
      float* part = p.partial + (int64_t(tile) * p.splits + split) * kGBM * C::kTmemCols;
#pragma unroll 1
      for (int c = 0; c < int(C::kTmemCols); c += 16) {
        float v[16];
        if (have) {
          g_ld16(lane_base + c, v);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.f;
        }
        float4* dst = reinterpret_cast<float4*>(part + int64_t(r) * C::kTmemCols + c);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (r == 0) *flag = atomicAdd(&p.tickets[tile], 1) == p.splits - 1;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (*flag) {
        __threadfence();
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          float v[16], u[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = u[i] = 0.f;
          for (int s = 0; s < p.splits; ++s) {
            const float* src = p.partial + (int64_t(tile) * p.splits + s) * kGBM * C::kTmemCols + int64_t(r) * C::kTmemCols;
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] += __ldcg(src + c + i);
            if constexpr (SILU) {
#pragma unroll
              for (int i = 0; i < 16; ++i) u[i] += __ldcg(src + BN + c + i);
            }
          }
          if constexpr (SILU) {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = silu_mul(v[i], u[i]);
          }
          if (row < p.M) {
            for (int i = 0; i < 16 && n0 + c + i < p.N; ++i)
              p.d[int64_t(row) * p.ldd + n0 + c + i] = __float2bfloat16_rn(v[i]);
          }
        }
        if (r == 0) p.tickets[tile] = 0;
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
  }
}

typedef CUresult (*EncodeFnG)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFnG encode_fn_g() {
  static EncodeFnG fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFnG>(ptr);
  }
  return fn;
}

// Row-major [rows, K] bf16 with row stride ld (elements) -> boxes of 64 (K) x box_rows.
bool encode2(CUtensorMap* map, const void* base, uint64_t rows, uint64_t k, uint64_t ld, uint32_t box_rows) {
  EncodeFnG fn = encode_fn_g();
  if (!fn) return false;
  const cuuint64_t dims[2] = {k, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {uint32_t(kGBK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                  cudaSuccess)
      sms = 148;
  }
  return sms;
}

template <int BN, bool SILU>
int launch_gemm(const GemmParams& prm, dim3 grid, cudaStream_t stream) {
  using C = GemmCfg<BN, SILU>;
  static bool configured = false;  // first call happens before any graph capture
  if (!configured) {
    cudaError_t e =
        cudaFuncSetAttribute(gemm_tc_kernel<BN, SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) {
      set_error("hl_gemm_bf16: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return HL_ERR_CUDA;
    }
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kGThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, SILU>, prm);
  if (e != cudaSuccess) {
    set_error("hl_gemm_bf16: launch failed: %s", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  return HL_OK;
}

constexpr int kGBN = 64;

// Split K until the grid covers the SMs (at most 8 ways, each part at least 4 K steps).
int gemm_splits(int M, int N, int K) {
  const int mt = (M + kGBM - 1) / kGBM, nt = (N + kGBN - 1) / kGBN, nk = K / kGBK;
  int splits = 1;
  while (splits < 8 && mt * nt * splits * 2 <= num_sms() && nk / (splits * 2) >= 4) splits *= 2;
  return splits;
}

}  // namespace
}  // namespace hl

using namespace hl;

extern "C" int64_t hl_gemm_workspace_size(int M, int N, int K, int epilogue) {
  if (M <= 0 || N <= 0 || K <= 0) return -1;
  const int64_t tiles = int64_t((M + kGBM - 1) / kGBM) * ((N + kGBN - 1) / kGBN);
  const int splits = gemm_splits(M, N, K);
  const int64_t cols = epilogue == HL_GEMM_SILU_MUL ? 2 * kGBN : kGBN;
  return 256 + ((tiles * 4 + 255) & ~int64_t(255)) + (splits > 1 ? tiles * splits * kGBM * cols * 4 : 0);
}

extern "C" int hl_gemm_bf16(const void* a, int64_t lda, const void* b, int64_t ldb, void* d, int64_t ldd, int M,
                            int N, int K, int epilogue, void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  if (M == 0 || N == 0) return HL_OK;
  HL_CHECK_ARG(a && b && d && M > 0 && N > 0 && K > 0, "hl_gemm_bf16: bad arguments");
  HL_CHECK_ARG(K % kGBK == 0, "hl_gemm_bf16: K must be a multiple of 64");
  HL_CHECK_ARG(epilogue == HL_GEMM_PLAIN || epilogue == HL_GEMM_SILU_MUL, "hl_gemm_bf16: bad epilogue");
  HL_CHECK_ARG(aligned16(a) && aligned16(b) && aligned16(d) && lda % 8 == 0 && ldb % 8 == 0 && ldd % 8 == 0,
               "hl_gemm_bf16: 16-byte aligned operands and row strides required");
  const int64_t need = hl_gemm_workspace_size(M, N, K, epilogue);
  HL_CHECK_ARG(workspace && workspace_bytes >= need && aligned16(workspace),
               "hl_gemm_bf16: workspace of %lld bytes needed", (long long)need);
  const bool silu = epilogue == HL_GEMM_SILU_MUL;
  constexpr int BN = kGBN;
  const int mt = (M + kGBM - 1) / kGBM, nt = (N + BN - 1) / BN;
  HL_CHECK_ARG(mt <= 65535, "hl_gemm_bf16: M too large");
  const int splits = gemm_splits(M, N, K);
  GemmParams prm;
  memset(&prm, 0, sizeof(prm));
  const uint64_t b_rows = silu ? uint64_t(2) * N : uint64_t(N);
  if (!encode2(&prm.ta, a, M, K, lda, kGBM) || !encode2(&prm.tb, b, b_rows, K, ldb, BN)) {
    set_error("hl_gemm_bf16: cuTensorMapEncodeTiled failed");
    return HL_ERR_CUDA;
  }
  prm.d = static_cast<__nv_bfloat16*>(d);
  prm.ldd = ldd;
  prm.M = M;
  prm.N = N;
  prm.K = K;
  prm.splits = splits;
  prm.silu_rows = N;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  prm.err = reinterpret_cast<int*>(ws);
  prm.tickets = reinterpret_cast<int*>(ws + 256);
  prm.partial = reinterpret_cast<float*>(ws + 256 + ((int64_t(mt) * nt * 4 + 255) & ~int64_t(255)));
  const dim3 grid(nt, mt, splits);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return silu ? launch_gemm<BN, true>(prm, grid, s) : launch_gemm<BN, false>(prm, grid, s);
}
