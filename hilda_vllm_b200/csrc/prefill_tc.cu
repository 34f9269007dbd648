// Varlen causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Semantics: flash_attn_varlen_func(q, k | k_cache, v | v_cache, cu_seqlens_q, cu_seqlens_k,
// max_seqlen_q, max_seqlen_k, softmax_scale, causal=True, block_table) as the reference calls it
// (mini_vllm/layers/attention.py:120-131,149-160): for sequence s with Lq queries and Lk keys,
// query i sees keys j <= i + (Lk - Lq) (bottom-right causal), j < Lk; rows with no visible key
// are zero.  With a block table, key j of sequence s is slot block_table[s, j / BS] * BS + j % BS
// of the paged cache, so a cached prefix and the chunk being prefilled are read the same way.
//
// One CTA = 128 query rows of one query head of one sequence.  Warp roles:
//   warp 0    TMA producer: Q once, then K and V tiles of 128 keys (two 64-dimension boxes each,
//             128-byte swizzled, i.e. the canonical K-major / MN-major UMMA layouts) into a
//             2-stage ring.  A 128-key tile never crosses a 256-token page.
//   warp 1    allocates 512 TMEM columns, and one thread issues the MMAs:
//             S = Q K^T (M=128 queries, N=128 keys, K=128, BF16 in, FP32 in TMEM, double-buffered
//             S so the next tile's S overlaps this tile's softmax), then O += P V (M=128, N=128
//             head dims, K=128 keys; V read MN-major straight from the TMA layout) with O resident
//             in TMEM for the whole sequence.  Completion is signalled with tcgen05.commit on
//             mbarriers.
//   warps 2-5 softmax: thread = query row = TMEM lane; reads its S row (tcgen05.ld), applies the
//             causal / length mask, online softmax in base 2, rescales its O row in TMEM when the
//             running max grows, writes P (bf16, swizzled K-major) to shared memory, and finally
//             normalises O and stores it.
// Every mbarrier wait is bounded; a timeout records an error bit and makes the roles leave their
// loops, after which the CTA frees its TMEM and returns.  No cluster launch, no multicast.
#include "hl_common.cuh"

#include <cuda.h>

namespace hl {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kD = 128;
constexpr int kThreads = 192;
constexpr int kHalf = 128 * 128;      // one [128 rows x 64 bf16] swizzled block (16 KiB)
constexpr int kTile = 2 * kHalf;      // 128 x 128 bf16 (32 KiB)
constexpr int kStages = 2;
constexpr uint32_t kTmemCols = 512;   // S0 [0,128) S1 [128,256) O [256,384)
constexpr uint32_t kColO = 256;

// Shared-memory map (offsets from a 1024-aligned base).
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTile;                 // + stage * 2 * kTile
constexpr int kOffP = kOffK + kStages * 2 * kTile;   // V of stage s at kOffK + s*2*kTile + kTile
constexpr int kOffPlo = kOffP + kTile;               // low part of P (split mode)
constexpr int kOffBar = kOffPlo + kTile;
constexpr int kSmemBytes = kOffBar + 256 + 1024;     // + alignment slack (226.3 KiB)

constexpr float kLog2e = 1.4426950408889634f;

// UMMA instruction descriptor (kind::f16): D fp32, A and B bf16, M=128, N=128.
constexpr uint32_t idesc_bf16(bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((128u >> 3) << 17) |
         ((128u >> 4) << 24);
}
constexpr uint32_t kIdescS = idesc_bf16(false);
constexpr uint32_t kIdescPV = idesc_bf16(true);

struct TcParams {
  CUtensorMap tq;
  CUtensorMap tk;
  CUtensorMap tv;
  const int32_t* cu_q;
  const int32_t* cu_k;
  const int32_t* block_tables;
  int64_t bt_stride;
  int64_t num_blocks;
  int paged;
  int block_size;
  int num_q_heads;
  int num_kv_heads;
  float scale_log2;
  __nv_bfloat16* out;
  int64_t out_row_stride;
};

__device__ int g_prefill_errors;  // bit 0: an mbarrier wait timed out; bit 1: a block id out of range

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm_100 version bits.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
      "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
      "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
      "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
      "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (*abort_flag) return false;
  if (mbar_wait(bar, parity)) return true;
  *abort_flag = 1;
  atomicOr(&g_prefill_errors, 1);
  return false;
}

// SPLIT_P: P is written as two bf16 matrices, hi = bf16(p) and lo = bf16(p - hi), and O gets
// both products (P_hi V + P_lo V), so the probabilities enter the MMA with ~16 significant bits
// instead of bf16's 8 (bf16-rounded P alone is what flash-attn does; it misses an fp32
// reference's rtol 2e-2 / atol 2e-3 on a few outputs with heavy cancellation).
template <bool SPLIT_P>
__global__ void __launch_bounds__(kThreads, 1) varlen_prefill_tc_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* o_done = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 13);

  const int tile = blockIdx.x;
  const int hq = blockIdx.y;
  const int s = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.num_q_heads / p.num_kv_heads;
  const int hk = hq / G;

  const int q_begin = p.cu_q[s];
  const int Lq = p.cu_q[s + 1] - q_begin;
  const int k_begin = p.cu_k[s];
  const int Lk = p.cu_k[s + 1] - k_begin;
  const int q0 = tile * kBM;
  if (q0 >= Lq) return;  // uniform per CTA
  const int shift = Lk - Lq;
  int k_needed = min(Lk, q0 + kBM + shift);
  if (k_needed < 0) k_needed = 0;
  const int n_tiles = (k_needed + kBN - 1) / kBN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);   // producer arrive.expect_tx + TMA bytes
      mbar_init(&kv_empty[i], 1);  // tcgen05.commit after the tile's PV
      mbar_init(&s_full[i], 1);    // tcgen05.commit after the tile's S
      mbar_init(&s_free[i], 128);  // every softmax thread has read its S row
    }
    mbar_init(p_full, 128);        // every softmax thread has written its P row
    mbar_init(o_done, 1);          // tcgen05.commit after the tile's PV
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0 && n_tiles > 0) {
      mbar_arrive_expect_tx(q_full, kTile);
      tma_load_3d(sbase + kOffQ, &p.tq, 0, hq, q_begin + q0, smem_u32(q_full));
      tma_load_3d(sbase + kOffQ + kHalf, &p.tq, 64, hq, q_begin + q0, smem_u32(q_full));
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j & 1;
        if (j >= 2 && !wait_or_abort(&kv_empty[st], ((j - 2) >> 1) & 1, abort_flag)) break;
        const int kj = j * kBN;
        int row;
        if (p.paged) {
          const int blk = p.block_tables[int64_t(s) * p.bt_stride + kj / p.block_size];
          // An out-of-range block reads zeros (TMA fill) and is recorded (error bit 1).
          if (blk < 0 || blk >= p.num_blocks) atomicOr(&g_prefill_errors, 2);
          row = blk * p.block_size + (kj % p.block_size);
        } else {
          row = k_begin + kj;
        }
        const uint32_t kdst = sbase + kOffK + st * 2 * kTile;
        const uint32_t vdst = kdst + kTile;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTile);
        tma_load_3d(kdst, &p.tk, 0, hk, row, smem_u32(&kv_full[st]));
        tma_load_3d(kdst + kHalf, &p.tk, 64, hk, row, smem_u32(&kv_full[st]));
        tma_load_3d(vdst, &p.tv, 0, hk, row, smem_u32(&kv_full[st]));
        tma_load_3d(vdst + kHalf, &p.tv, 64, hk, row, smem_u32(&kv_full[st]));
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && n_tiles > 0) {
      bool ok = wait_or_abort(q_full, 0, abort_flag);
      auto issue_pv = [&](int i) -> bool {
        if (!wait_or_abort(p_full, i & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t pbase = sbase + kOffP;
        const uint32_t vbase = sbase + kOffK + (i & 1) * 2 * kTile + kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = smem_desc(pbase + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
          const uint64_t b = smem_desc(vbase + kk * 16 * 128, kHalf, 1024);
          umma_bf16(tmem + kColO, a, b, kIdescPV, (i > 0 || kk > 0) ? 1u : 0u);
        }
        if constexpr (SPLIT_P) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t a = smem_desc(sbase + kOffPlo + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
            const uint64_t b = smem_desc(vbase + kk * 16 * 128, kHalf, 1024);
            umma_bf16(tmem + kColO, a, b, kIdescPV, 1u);
          }
        }
        umma_commit(smem_u32(o_done));
        umma_commit(smem_u32(&kv_empty[i & 1]));
        return true;
      };
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int st = j & 1;
        if (!wait_or_abort(&kv_full[st], (j >> 1) & 1, abort_flag)) break;
        if (j >= 2 && !wait_or_abort(&s_free[st], ((j - 2) >> 1) & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t kbase = sbase + kOffK + st * 2 * kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = smem_desc(sbase + kOffQ + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
          const uint64_t b = smem_desc(kbase + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
          umma_bf16(tmem + st * 128, a, b, kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(smem_u32(&s_full[st]));
        if (j >= 1 && !issue_pv(j - 1)) break;
      }
      if (!*abort_flag) issue_pv(n_tiles - 1);
    }
  } else {
    // ---------------------------------------------------------------- softmax + epilogue
    // TMEM loads/stores are warp-collective (.sync.aligned): every branch around them is made
    // warp-uniform, per-row differences are carried in the values instead.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile = TMEM lane
    const int qi = q0 + r;              // query index within the sequence
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    float m = -INFINITY, l = 0.f;
    const int limit = qi + shift;  // keys j <= limit are visible (and j < Lk)
    bool alive = n_tiles > 0;
    for (int j = 0; alive && j < n_tiles; ++j) {
      const int sb = j & 1;
      if (!__all_sync(0xffffffffu, wait_or_abort(&s_full[sb], (j >> 1) & 1, abort_flag))) {
        alive = false;
        break;
      }
      tc_fence_after();
      float sv[kBN];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float chunk[32];
        tmem_ld32(lane_base + sb * 128 + c * 32, chunk);
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c * 32 + i] = chunk[i];
      }
      tc_fence_before();
      mbar_arrive(&s_free[sb]);

      const int j0 = j * kBN;
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < kBN; ++c) {
        const int kj = j0 + c;
        const bool ok = kj < Lk && kj <= limit;
        sv[c] = ok ? sv[c] * p.scale_log2 : -INFINITY;
        mt = fmaxf(mt, sv[c]);
      }
      const float mn = fmaxf(m, mt);
      const float corr = (mn == -INFINITY) ? 1.f : exp2f(m - mn);

      if (j >= 1) {
        // PV of the previous tile must be done before O is rescaled and P is overwritten.
        if (!__all_sync(0xffffffffu, wait_or_abort(o_done, (j - 1) & 1, abort_flag))) {
          alive = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32(lane_base + kColO + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= corr;
            tmem_st32(lane_base + kColO + c * 32, o);
          }
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
      }
      m = mn;

      if (j0 + kBN > Lk) {
        // Last, partial tile: zero the V rows past the sequence so that P = 0 never meets a
        // non-finite cache value inside the MMA.
        if (!__all_sync(0xffffffffu, wait_or_abort(&kv_full[j & 1], (j >> 1) & 1, abort_flag))) {
          alive = false;
          break;
        }
        if (j0 + r >= Lk) {
          uint4* v0 = reinterpret_cast<uint4*>(smem + kOffK + (j & 1) * 2 * kTile + kTile + r * 128);
          uint4* v1 = reinterpret_cast<uint4*>(smem + kOffK + (j & 1) * 2 * kTile + kTile + kHalf + r * 128);
#pragma unroll
          for (int c = 0; c < 8; ++c) v0[c] = v1[c] = make_uint4(0, 0, 0, 0);
        }
      }
      // P row r as bf16, 128 keys = two 64-key swizzled blocks: 16-byte chunk c of block h
      // goes to chunk (c ^ (r & 7)) of row r.
      float ps = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint32_t w[4], wl[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float a = (mn == -INFINITY) ? 0.f : exp2f(sv[8 * c + 2 * t] - mn);
          const float b = (mn == -INFINITY) ? 0.f : exp2f(sv[8 * c + 2 * t + 1] - mn);
          ps += a + b;
          __nv_bfloat162 h2 = __floats2bfloat162_rn(a, b);
          w[t] = *reinterpret_cast<uint32_t*>(&h2);
          if constexpr (SPLIT_P) {
            const float2 hf = __bfloat1622float2(h2);
            __nv_bfloat162 l2 = __floats2bfloat162_rn(a - hf.x, b - hf.y);
            wl[t] = *reinterpret_cast<uint32_t*>(&l2);
          }
        }
        const int h = c >> 3, cc = c & 7;
        const int off = h * kHalf + r * 128 + ((cc ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(smem + kOffP + off) = make_uint4(w[0], w[1], w[2], w[3]);
        if constexpr (SPLIT_P) *reinterpret_cast<uint4*>(smem + kOffPlo + off) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
      }
      l = l * corr + ps;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // Epilogue: O / l -> bf16 rows of the output (rows past the sequence load but do not store).
    const bool have_o =
        __all_sync(0xffffffffu, alive && n_tiles > 0 && wait_or_abort(o_done, (n_tiles - 1) & 1, abort_flag));
    if (have_o) tc_fence_after();
    __nv_bfloat16* orow = p.out + int64_t(q_begin + qi) * p.out_row_stride + hq * kD;
    const float inv = (have_o && l > 0.f) ? 1.f / l : 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float o[32];
      if (have_o) {
        tmem_ld32(lane_base + kColO + c * 32, o);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0.f;
      }
      if (qi < Lq) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t w[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            __nv_bfloat162 h2 = __floats2bfloat162_rn(o[v * 8 + 2 * t] * inv, o[v * 8 + 2 * t + 1] * inv);
            w[t] = *reinterpret_cast<uint32_t*>(&h2);
          }
          *reinterpret_cast<uint4*>(orow + c * 32 + v * 8) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------------- head pairs
// The production kernel when Hq / Hk is even: one CTA = 128 query rows of the TWO query heads
// 2p and 2p+1, which share one KV head, so every K/V tile brought in by TMA feeds twice the
// MMAs.  TMEM holds S_a, S_b (128 columns each) and O_a, O_b (128 each) = all 512 columns; the
// probabilities are written back over their own S columns as bf16 (P_hi in the first 64
// columns, P_lo in the next 64 with SPLIT_P) and the PV product reads them straight from TMEM
// as the A operand (tcgen05.mma with [a-tmem]), so P never touches shared memory.
//   warp 0     TMA producer (both Q tiles once, then K+V tiles into a 2-stage ring)
//   warp 1     TMEM allocator; its lane 0 alone is the MMA issuer, in ping-pong order per key
//              tile j:  PV_a(j), QK_a(j+1), PV_b(j), QK_b(j+1)
//              so the tensor core works on one head while the other head's softmax runs.  The
//              tensor pipe takes an M128 x N128 x K16 instruction every 64 cycles, so the issuer
//              does as little as possible between MMAs: descriptors are built once and a K step
//              adds a constant to the start-address field.
//   warps 2-3  zero the V rows past the sequence in the last key tile
//   warps 4-7  softmax of head a (thread = query row = TMEM lane; warp w reads TMEM lanes
//              32 * (w % 4) ..), warps 8-11 softmax of head b.
// Waiting roles sleep in mbarrier.try_wait with a suspend-time hint instead of spinning, which
// leaves the issue slots (and the power budget: the kernel runs at the 1 kW cap when timed for
// more than a few ms) to the warps that work.
// Registers: the kernel launches with 168 per thread (384 x 168 = 64512 of the SM's 65536);
// warpgroup 0 (warps 0-3) gives back down to 120 with setmaxnreg.dec and the two softmax
// warpgroups take them with setmaxnreg.inc to 192 (128 x 120 + 256 x 192 = 64512), so a whole
// 128-key S row stays in registers.
// O is rescaled lazily: the running reference max only moves when a tile's max exceeds it by
// more than kRescaleLog2 (probabilities then stay <= 2^kRescaleLog2, exact in bf16 range),
// which skips almost every O read-modify-write of TMEM.  Since tcgen05.commit tracks every
// earlier MMA of the issuing thread, "S_a(j) is ready" also means PV_a(j-1) has finished, so
// the softmax warps may touch O_a then.  CTAs run heaviest query tile first (blockIdx.z is
// the reversed tile index) to shorten the causal tail.
constexpr int kThreads2 = 384;
constexpr int kOff2Qa = 0;
constexpr int kOff2Qb = kTile;
constexpr int kOff2K = 2 * kTile;                        // + stage * 2 * kTile; V at + kTile
constexpr int kOff2Bar = kOff2K + kStages * 2 * kTile;   // 192 KiB
constexpr int kSmem2Bytes = kOff2Bar + 256 + 1024;
constexpr float kRescaleLog2 = 8.f;

__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                             uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// 2^x on the MUFU unit (ex2.approx.ftz: 2^-inf = +0, relative error ~2^-22).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

constexpr uint32_t kSuspendHintNs = 100000;        // longest sleep of one try_wait
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // a wait gives up after 2 s

// Bounded mbarrier wait: the thread sleeps inside try_wait until the phase completes (or the
// hint elapses), so waiting warps take no issue slots.  Gives up as soon as another role has
// raised the abort flag, or after kWaitLimitNs of global time (error bit 0).
__device__ __forceinline__ bool wait2(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint32_t addr = smem_u32(bar);
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    if (done) return true;
    if ((i & 15u) == 15u) {
      if (*abort_flag) return false;
      const uint64_t now = global_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitLimitNs) {
        break;
      }
    }
  }
  *abort_flag = 1;
  atomicOr(&g_prefill_errors, 1);
  return false;
}

template <bool SPLIT_P>
__global__ void __launch_bounds__(kThreads2, 1) varlen_prefill_pair_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOff2Bar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2] stages
  uint64_t* kv_empty = bars + 3;  // [2] stages
  uint64_t* s_full = bars + 5;    // [2] heads
  uint64_t* p_full = bars + 7;    // [2] heads
  uint64_t* o_done = bars + 9;
  uint64_t* v_land = bars + 10;   // the last key tile's TMA landed (MMA issuer -> warps 2-3)
  uint64_t* v_zero = bars + 11;   // its V rows past the sequence are zeroed (warps 2-3 -> issuer)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 13);

  const int pair = blockIdx.x;
  const int s = blockIdx.y;
  const int tile = gridDim.z - 1 - blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.num_q_heads / p.num_kv_heads;
  const int hq0 = 2 * pair;
  const int hk = hq0 / G;

  const int q_begin = p.cu_q[s];
  const int Lq = p.cu_q[s + 1] - q_begin;
  const int k_begin = p.cu_k[s];
  const int Lk = p.cu_k[s + 1] - k_begin;
  const int q0 = tile * kBM;
  if (q0 >= Lq) return;  // uniform per CTA
  const int shift = Lk - Lq;
  int k_needed = min(Lk, q0 + kBM + shift);
  if (k_needed < 0) k_needed = 0;
  const int n_tiles = (k_needed + kBN - 1) / kBN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);    // producer arrive.expect_tx + TMA bytes
      mbar_init(&kv_empty[i], 1);   // tcgen05.commit after the tile's last MMA
      mbar_init(&s_full[i], 1);     // tcgen05.commit after QK of head i
      mbar_init(&p_full[i], 128);   // every softmax thread of head i wrote its P row
    }
    mbar_init(o_done, 1);
    mbar_init(v_land, 1);
    mbar_init(v_zero, 64);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 120;");
  }
  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0 && n_tiles > 0) {
      mbar_arrive_expect_tx(q_full, 2 * kTile);
      tma_load_3d(sbase + kOff2Qa, &p.tq, 0, hq0, q_begin + q0, smem_u32(q_full));
      tma_load_3d(sbase + kOff2Qa + kHalf, &p.tq, 64, hq0, q_begin + q0, smem_u32(q_full));
      tma_load_3d(sbase + kOff2Qb, &p.tq, 0, hq0 + 1, q_begin + q0, smem_u32(q_full));
      tma_load_3d(sbase + kOff2Qb + kHalf, &p.tq, 64, hq0 + 1, q_begin + q0, smem_u32(q_full));
      int issued = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j & 1;
        if (j >= 2 && !wait2(&kv_empty[st], ((j - 2) >> 1) & 1, abort_flag)) break;
        const int kj = j * kBN;
        int row;
        if (p.paged) {
          const int blk = p.block_tables[int64_t(s) * p.bt_stride + kj / p.block_size];
          // An out-of-range block reads zeros (TMA fill) and is recorded (error bit 1).
          if (blk < 0 || blk >= p.num_blocks) atomicOr(&g_prefill_errors, 2);
          row = blk * p.block_size + (kj % p.block_size);
        } else {
          row = k_begin + kj;
        }
        const uint32_t kdst = sbase + kOff2K + st * 2 * kTile;
        const uint32_t vdst = kdst + kTile;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTile);
        tma_load_3d(kdst, &p.tk, 0, hk, row, smem_u32(&kv_full[st]));
        tma_load_3d(kdst + kHalf, &p.tk, 64, hk, row, smem_u32(&kv_full[st]));
        tma_load_3d(vdst, &p.tv, 0, hk, row, smem_u32(&kv_full[st]));
        tma_load_3d(vdst + kHalf, &p.tv, 64, hk, row, smem_u32(&kv_full[st]));
        issued = j + 1;
      }
      // Drain: no copy into this CTA's shared memory may still be in flight at exit (the
      // normal path returns at once, every tile having been consumed).
      mbar_wait(q_full, 0);
      for (int t = issued >= 2 ? issued - 2 : 0; t < issued; ++t) mbar_wait(&kv_full[t & 1], (t >> 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (lane 0)
    if (n_tiles > 0 && lane == 0) {
      // A 16-wide K step only moves a descriptor's start-address field (bits 0-13 = address
      // >> 4; every address here is below 256 KiB, so the field never carries), so each MMA
      // adds a compile-time constant to one of these.
      const uint64_t dq0 = smem_desc(sbase + kOff2Qa, 16, 1024), dq1 = smem_desc(sbase + kOff2Qb, 16, 1024);
      const uint64_t dk0 = smem_desc(sbase + kOff2K, 16, 1024), dk1 = smem_desc(sbase + kOff2K + 2 * kTile, 16, 1024);
      const uint64_t dv0 = smem_desc(sbase + kOff2K + kTile, kHalf, 1024);
      const uint64_t dv1 = smem_desc(sbase + kOff2K + 3 * kTile, kHalf, 1024);
      auto qk = [&](int j, int h) {
        const uint64_t a0 = h ? dq1 : dq0;
        const uint64_t b0 = (j & 1) ? dk1 : dk0;
        const uint32_t d = tmem + h * 128;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t off = uint64_t(((kk >> 2) * kHalf + (kk & 3) * 32) >> 4);
          umma_bf16(d, a0 + off, b0 + off, kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(smem_u32(&s_full[h]));
      };
      auto pv = [&](int j, int h) {
        const uint64_t b0 = (j & 1) ? dv1 : dv0;
        const uint32_t pcol = tmem + h * 128;
        const uint32_t ocol = tmem + kColO + h * 128;
        const uint32_t first = j > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16_ts(ocol, pcol + kk * 8, b0 + uint64_t((kk * 16 * 128) >> 4), kIdescPV, kk > 0 ? 1u : first);
        if constexpr (SPLIT_P) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16_ts(ocol, pcol + 64 + kk * 8, b0 + uint64_t((kk * 16 * 128) >> 4), kIdescPV, 1u);
        }
      };
      // The last key tile reaches past the sequence: warps 2-3 zero its V rows past Lk once its
      // TMA has landed (signalled here), and PV waits for that.
      const bool tail_partial = (n_tiles - 1) * kBN + kBN > Lk;
      auto landed = [&](int t) {
        if (tail_partial && t == n_tiles - 1) mbar_arrive(v_land);
      };
      bool ok = wait2(q_full, 0, abort_flag) && wait2(&kv_full[0], 0, abort_flag);
      if (ok) {
        landed(0);
        tc_fence_after();
        qk(0, 0);
        qk(0, 1);
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int st = j & 1;
        ok = wait2(&p_full[0], j & 1, abort_flag);
        if (!ok) break;
        if (tail_partial && j == n_tiles - 1) {
          ok = wait2(v_zero, 0, abort_flag);
          if (!ok) break;
        }
        tc_fence_after();
        pv(j, 0);
        if (j + 1 < n_tiles) {
          ok = wait2(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, abort_flag);
          if (!ok) break;
          landed(j + 1);
          qk(j + 1, 0);
        }
        ok = wait2(&p_full[1], j & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        pv(j, 1);
        umma_commit(smem_u32(&kv_empty[st]));
        if (j + 1 < n_tiles) qk(j + 1, 1);
      }
      umma_commit(smem_u32(o_done));
      if (!ok) mbar_wait(o_done, 0);  // let issued MMAs finish before TMEM is freed
    }
    __syncwarp();
  } else if (warp == 2 || warp == 3) {
    // ---------------------------------------------------------------- tail V rows
    // Zero the V rows past the sequence in the last, partial key tile so that P = 0 never
    // meets a non-finite cache value inside the MMA (rows of a cache block nobody wrote).
    const int jl = n_tiles - 1;
    if (n_tiles > 0 && jl * kBN + kBN > Lk) {
      if (wait2(v_land, 0, abort_flag)) {
        uint8_t* vs = smem + kOff2K + (jl & 1) * 2 * kTile + kTile;
        for (int rr = max(Lk - jl * kBN, 0) + (threadIdx.x - 64); rr < kBN; rr += 64) {
          uint4* v0 = reinterpret_cast<uint4*>(vs + rr * 128);
          uint4* v1 = reinterpret_cast<uint4*>(vs + kHalf + rr * 128);
#pragma unroll
          for (int c = 0; c < 8; ++c) v0[c] = v1[c] = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      mbar_arrive(v_zero);
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- softmax + epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 192;");
    const int h = (warp - 4) >> 2;   // 0: head a, 1: head b
    const int quarter = warp & 3;    // TMEM lanes [32 * quarter, +32) belong to this warp
    const int r = quarter * 32 + lane;
    const int qi = q0 + r;
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    const uint32_t s_col = lane_base + h * 128;
    const uint32_t o_col = lane_base + kColO + h * 128;
    const int limit = qi + shift;  // keys j <= limit are visible (and j < Lk)
    const float sc = p.scale_log2;
    float m_ref = -INFINITY, l = 0.f;
    bool alive = n_tiles > 0;
    for (int j = 0; alive && j < n_tiles; ++j) {
      if (!__all_sync(0xffffffffu, wait2(&s_full[h], j & 1, abort_flag))) {
        alive = false;
        break;
      }
      tc_fence_after();
      uint32_t raw[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32_async(s_col + c * 32, raw[c]);
      tmem_wait_ld();
      float sv[kBN];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(raw[c][i]);
      const int j0 = j * kBN;
      // Rows of this tile see every key of it unless the tile reaches the diagonal or Lk.
      if (j0 + kBN - 1 > q0 + shift || j0 + kBN > Lk) {
        const int lim = min(limit, Lk - 1) - j0;  // visible columns c <= lim
#pragma unroll
        for (int c = 0; c < kBN; ++c) sv[c] = c <= lim ? sv[c] : -INFINITY;
      }
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < kBN; c += 4) {
        mx[0] = fmaxf(mx[0], sv[c]);
        mx[1] = fmaxf(mx[1], sv[c + 1]);
        mx[2] = fmaxf(mx[2], sv[c + 2]);
        mx[3] = fmaxf(mx[3], sv[c + 3]);
      }
      const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sc;
      float corr = 1.f;
      if (mt > m_ref + kRescaleLog2) {
        if (m_ref != -INFINITY) corr = ex2(m_ref - mt);
        m_ref = mt;
      }
      if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
        // PV_h(j-1) has completed (it was issued before QK_h(j), whose commit we waited for).
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t o[16];
          tmem_ld16_async(o_col + c * 16, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
          tmem_st16(o_col + c * 16, o);
        }
      }
      l *= corr;
      // p = 2^(s * scale_log2 - m_ref); masked keys (-inf) give 0; a row with nothing visible
      // yet (m_ref = -inf) gives all zeros.
      const float msub = m_ref == -INFINITY ? 0.f : m_ref;
      const float2 sc2 = make_float2(sc, sc);
      const float2 nm2 = make_float2(-msub, -msub);
      float2 rs = make_float2(0.f, 0.f);
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const float2 x = __ffma2_rn(make_float2(sv[ch * 16 + 2 * t], sv[ch * 16 + 2 * t + 1]), sc2, nm2);
          const float2 e = make_float2(ex2(x.x), ex2(x.y));
          rs = __fadd2_rn(rs, e);
          __nv_bfloat162 h2 = __floats2bfloat162_rn(e.x, e.y);
          hi[t] = *reinterpret_cast<uint32_t*>(&h2);
          if constexpr (SPLIT_P) {
            const float2 hf = __bfloat1622float2(h2);
            __nv_bfloat162 l2 = __floats2bfloat162_rn(e.x - hf.x, e.y - hf.y);
            lo[t] = *reinterpret_cast<uint32_t*>(&l2);
          }
        }
        tmem_st8(s_col + ch * 8, hi);
        if constexpr (SPLIT_P) tmem_st8(s_col + 64 + ch * 8, lo);
      }
      l += rs.x + rs.y;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[h]);
    }
    // Epilogue: O / l -> bf16 rows of the output (rows past the sequence load but do not store).
    const bool have_o = __all_sync(0xffffffffu, alive && n_tiles > 0 && wait2(o_done, 0, abort_flag));
    if (have_o) tc_fence_after();
    __nv_bfloat16* orow = p.out + int64_t(q_begin + qi) * p.out_row_stride + (hq0 + h) * kD;
    const float inv = (have_o && l > 0.f) ? 1.f / l : 0.f;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t o[32];
      if (have_o) {
        tmem_ld32_async(o_col + c * 32, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (qi < Lq) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t w[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            __nv_bfloat162 h2 = __floats2bfloat162_rn(__uint_as_float(o[v * 8 + 2 * t]) * inv,
                                                      __uint_as_float(o[v * 8 + 2 * t + 1]) * inv);
            w[t] = *reinterpret_cast<uint32_t*>(&h2);
          }
          *reinterpret_cast<uint4*>(orow + c * 32 + v * 8) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// [rows, heads, 128] bf16 with the given byte strides -> box of 128 rows x 1 head x 64 dims.
bool make_map(CUtensorMap* map, const void* base, uint64_t heads, uint64_t rows, uint64_t head_stride_bytes,
              uint64_t row_stride_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {kD, heads, rows};
  const cuuint64_t strides[2] = {head_stride_bytes, row_stride_bytes};
  const cuuint32_t box[3] = {64, 1, 128};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace
}  // namespace hl

using namespace hl;

template <bool SPLIT_P>
int launch_pair(const TcParams& prm, int max_seqlen_q, int num_q_heads, int num_seqs, cudaStream_t stream) {
  static bool configured = false;  // first call happens before any graph capture
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(varlen_prefill_pair_kernel<SPLIT_P>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem2Bytes);
    if (e != cudaSuccess) {
      set_error("hl_varlen_prefill: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return HL_ERR_CUDA;
    }
    configured = true;
  }
  dim3 grid(num_q_heads / 2, num_seqs, (max_seqlen_q + kBM - 1) / kBM);
  varlen_prefill_pair_kernel<SPLIT_P><<<grid, kThreads2, kSmem2Bytes, stream>>>(prm);
  HL_CHECK_LAUNCH("hl_varlen_prefill");
  return HL_OK;
}

template <bool SPLIT_P>
int launch_tc(const TcParams& prm, int max_seqlen_q, int num_q_heads, int num_seqs, cudaStream_t stream) {
  static bool configured = false;  // first call happens before any graph capture
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(varlen_prefill_tc_kernel<SPLIT_P>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) {
      set_error("hl_varlen_prefill: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return HL_ERR_CUDA;
    }
    configured = true;
  }
  dim3 grid((max_seqlen_q + kBM - 1) / kBM, num_q_heads, num_seqs);
  varlen_prefill_tc_kernel<SPLIT_P><<<grid, kThreads, kSmemBytes, stream>>>(prm);
  HL_CHECK_LAUNCH("hl_varlen_prefill");
  return HL_OK;
}

extern "C" int hl_varlen_prefill(const void* q, int64_t q_row_stride, int64_t total_q, const void* k,
                                    const void* v, int64_t k_row_stride, int64_t v_row_stride, int64_t total_k,
                                    const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                                    const int32_t* block_tables, int64_t bt_stride, int num_seqs, int max_seqlen_q,
                                    int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                                    int64_t num_blocks, float softmax_scale, void* out, int64_t out_row_stride,
                                    int precise_p, void* stream) {
  clear_error();
  HL_CHECK_ARG(num_seqs >= 0 && max_seqlen_q >= 0, "hl_varlen_prefill: negative size");
  if (num_seqs == 0 || max_seqlen_q == 0) return HL_OK;
  HL_CHECK_ARG(q && k && v && cu_seqlens_q && cu_seqlens_k && out, "hl_varlen_prefill: null pointer");
  HL_CHECK_ARG(head_dim == kD, "hl_varlen_prefill: head_dim %d != 128", head_dim);
  HL_CHECK_ARG(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0, "hl_varlen_prefill: Hq %% Hk != 0");
  HL_CHECK_ARG(num_seqs <= 65535 && num_q_heads <= 65535, "hl_varlen_prefill: grid too large");
  HL_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out) && q_row_stride % 8 == 0 &&
                   out_row_stride % 8 == 0,
               "hl_varlen_prefill: q/k/v/out must be 16-byte aligned with row strides %% 8 == 0");
  HL_CHECK_ARG(total_q > 0 && total_q < (int64_t(1) << 31), "hl_varlen_prefill: bad total_q");
  TcParams prm;
  memset(&prm, 0, sizeof(prm));
  const uint64_t hs = uint64_t(head_dim) * 2;
  bool ok = make_map(&prm.tq, q, num_q_heads, total_q, hs, uint64_t(q_row_stride) * 2);
  if (block_tables) {
    HL_CHECK_ARG(block_size > 0 && block_size % kBN == 0 && bt_stride > 0 && num_blocks > 0,
                 "hl_varlen_prefill: block_size must be a multiple of 128");
    HL_CHECK_ARG(num_blocks * block_size < (int64_t(1) << 31), "hl_varlen_prefill: cache too large");
    const uint64_t rows = uint64_t(num_blocks) * block_size;
    const uint64_t rs = uint64_t(num_kv_heads) * head_dim * 2;
    ok = ok && make_map(&prm.tk, k, num_kv_heads, rows, hs, rs) && make_map(&prm.tv, v, num_kv_heads, rows, hs, rs);
  } else {
    HL_CHECK_ARG(k_row_stride % 8 == 0 && v_row_stride % 8 == 0 && total_k > 0 && total_k < (int64_t(1) << 31),
                 "hl_varlen_prefill: bad k/v layout");
    ok = ok && make_map(&prm.tk, k, num_kv_heads, total_k, hs, uint64_t(k_row_stride) * 2) &&
         make_map(&prm.tv, v, num_kv_heads, total_k, hs, uint64_t(v_row_stride) * 2);
  }
  if (!ok) {
    set_error("hl_varlen_prefill: cuTensorMapEncodeTiled failed");
    return HL_ERR_CUDA;
  }
  prm.cu_q = cu_seqlens_q;
  prm.cu_k = cu_seqlens_k;
  prm.block_tables = block_tables;
  prm.bt_stride = bt_stride;
  prm.num_blocks = block_tables ? num_blocks : 0;
  prm.paged = block_tables != nullptr;
  prm.block_size = block_size;
  prm.num_q_heads = num_q_heads;
  prm.num_kv_heads = num_kv_heads;
  prm.scale_log2 = softmax_scale * kLog2e;
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.out_row_stride = out_row_stride;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool split = (precise_p & 1) != 0;
  const bool pairs = (num_q_heads / num_kv_heads) % 2 == 0 && !(precise_p & HL_PREFILL_ONE_HEAD_PER_CTA);
  HL_CHECK_ARG((max_seqlen_q + kBM - 1) / kBM <= 65535, "hl_varlen_prefill: max_seqlen_q too large");
  if (pairs) {
    if (split) return launch_pair<true>(prm, max_seqlen_q, num_q_heads, num_seqs, st);
    return launch_pair<false>(prm, max_seqlen_q, num_q_heads, num_seqs, st);
  }
  if (split) return launch_tc<true>(prm, max_seqlen_q, num_q_heads, num_seqs, st);
  return launch_tc<false>(prm, max_seqlen_q, num_q_heads, num_seqs, st);
}

extern "C" int hl_varlen_prefill_read_errors(int32_t* errors_out) {
  clear_error();
  HL_CHECK_ARG(errors_out, "hl_varlen_prefill_read_errors: null pointer");
  cudaError_t e = cudaMemcpyFromSymbol(errors_out, g_prefill_errors, sizeof(int32_t));
  if (e != cudaSuccess) {
    set_error("hl_varlen_prefill_read_errors: %s", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  return HL_OK;
}

extern "C" int hl_varlen_prefill_copy_errors_async(int32_t* dst, void* stream) {
  clear_error();
  HL_CHECK_ARG(dst, "hl_varlen_prefill_copy_errors_async: null pointer");
  cudaError_t e = cudaMemcpyFromSymbolAsync(dst, g_prefill_errors, sizeof(int32_t), 0, cudaMemcpyDefault,
                                            static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("hl_varlen_prefill_copy_errors_async: %s", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  return HL_OK;
}

extern "C" int hl_varlen_prefill_clear_errors(void* stream) {
  clear_error();
  const int32_t zero = 0;
  cudaError_t e = cudaMemcpyToSymbolAsync(g_prefill_errors, &zero, sizeof(int32_t), 0, cudaMemcpyHostToDevice,
                                          static_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("hl_varlen_prefill_clear_errors: %s", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  return HL_OK;
}
