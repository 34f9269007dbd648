// Paged decode attention for B200 (sm_100a): split-K flash-decoding over a paged KV cache
// with an in-kernel last-CTA reduction.
//
// Semantics (mini_vllm/layers/attention.py:162-170, flash_attn_with_kvcache with one query
// token, causal=True, cache_seqlens=context_lens, block_table=block_tables):
//   out[b, hq] = softmax_j(scale * q[b, hq] . K[b, j, hq / G]) @ V[b, j, hq / G],  j < L_b,
//   token j of sequence b lives at slot block_tables[b, j / BS] * BS + j % BS,
//   G = Hq / Hk (grouped-query attention).  L_b == 0 gives zeros.
// FP8 variant (attention.py:134-141): K/V bytes are e4m3, dequantised in registers as
// value * scale[h]; k_scale is folded into q and v_scale into the output.
//
// Work decomposition.  One CTA = one (split, sequence): SPLIT consecutive tokens of one page,
// all local KV heads.  Because the cache is [block, offset, Hk, D], the K (and V) rows of a
// run of tokens inside one page are one contiguous byte range, so each pipeline stage is a
// single 16 KiB cp.async.bulk (TMA engine) per K and per V, completion tracked by an mbarrier.
// 8 warps: warp w owns KV head w % Hk and a 1/(8/Hk) slice of each tile's tokens; within a
// warp each half-warp takes one token at a time and its 16 lanes split D = 128 into 8-element
// (16-byte) slices, so shared-memory reads are conflict-free 256-byte rows.  All G query
// heads of the KV head are kept in registers, so every K/V byte is read from HBM once and
// used G times.  Splits of one sequence are combined by the CTA that finishes last (atomic
// ticket in the workspace); sequences that fit in one split write the output directly.
//
// Kernel choice (hl_paged_decode): this CUDA-core kernel serves GQA ratios 1 and 2; ratios >= 4
// (with at most 2048 sequences) go to the tcgen05 kernel of paged_decode_tc.cu, whose cost does
// not grow with the number of query heads per KV head.
#include "hl_common.cuh"

#include <atomic>
#include <mutex>

namespace hl {
namespace {

constexpr int kDecodeThreads = 256;
constexpr int kHeadDim = 128;
#ifndef HL_DECODE_SPLIT
#define HL_DECODE_SPLIT 128
#endif
constexpr int kSplit = HL_DECODE_SPLIT;  // tokens per CTA (divides every supported block size)
constexpr int kTileBytes = 16384;      // bytes per K (and per V) pipeline stage
constexpr int kStages = 2;
constexpr int kMaxBatch = 4096;        // capacity of the ticket array in the workspace
constexpr int64_t kWsErrOff = 0;       // int32 error word(s)
constexpr int64_t kWsTicketOff = 256;  // int32 tickets[kMaxBatch]
constexpr int64_t kWsMlOff = kWsTicketOff + 4 * kMaxBatch + 256;  // float2 (m, l) [B][S][Hq]

constexpr float kLog2e = 1.4426950408889634f;
// Smallest GQA ratio that hl_paged_decode hands to the tensor-core kernel.
constexpr int kTcMinGroupBf16 = 4;
constexpr int kTcMinGroupFp8 = 4;
constexpr int kMaxDecodeDevices = 64;

__host__ __device__ constexpr int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

struct DecodeParams {
  const __nv_bfloat16* q;
  int64_t q_row_stride;
  const uint8_t* k_cache;
  const uint8_t* v_cache;
  const float* k_scale;
  const float* v_scale;
  const int32_t* block_tables;
  int64_t bt_stride;
  int max_blocks;
  const int32_t* context_lens;
  int batch;
  int block_size;
  int64_t num_blocks;
  int max_splits;
  float scale_log2;  // softmax_scale * log2(e)
  __nv_bfloat16* out;
  int64_t out_row_stride;
  uint8_t* ws;
};

template <bool FP8, int G>
constexpr int ctas_per_sm() { return G <= 2 ? 3 : (G <= 4 ? 2 : 1); }

template <bool FP8, int HK, int SPLIT = kSplit>
struct Traits {
  static constexpr int kElem = FP8 ? 1 : 2;
  static constexpr int kTileB = kTileBytes;  // bytes per K (and per V) stage
  static constexpr int kRowBytes = HK * kHeadDim * kElem;  // one token, all local KV heads
  static constexpr int kT = kTileB / kRowBytes < SPLIT ? kTileB / kRowBytes : SPLIT;  // tokens per tile
  static constexpr int kPhases = 8 / HK;                    // warps sharing one KV head
  static constexpr int kTPW = kT / kPhases;                 // tokens per warp per tile
  static constexpr int kTPH = kTPW / 2;                     // tokens per half-warp per tile
  static_assert(SPLIT % kT == 0, "split must be a whole number of tiles");
  static_assert(kTPH >= 1, "tile too small");
};

// Load this lane's 8 consecutive K or V elements (its D-slice) from shared memory as four
// float2 pairs of adjacent dimensions, ready for the packed fp32x2 FMA of sm_100.
template <bool FP8>
__device__ __forceinline__ void load8x2(const uint8_t* p, float2 (&x)[4]) {
  if constexpr (FP8) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    x[0] = e4m3x2_to_float2(static_cast<uint16_t>(v.x & 0xffffu));
    x[1] = e4m3x2_to_float2(static_cast<uint16_t>(v.x >> 16));
    x[2] = e4m3x2_to_float2(static_cast<uint16_t>(v.y & 0xffffu));
    x[3] = e4m3x2_to_float2(static_cast<uint16_t>(v.y >> 16));
  } else {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    x[0] = make_float2(bf16lo(v.x), bf16hi(v.x));
    x[1] = make_float2(bf16lo(v.y), bf16hi(v.y));
    x[2] = make_float2(bf16lo(v.z), bf16hi(v.z));
    x[3] = make_float2(bf16lo(v.w), bf16hi(v.w));
  }
}

// Sums NV per-lane partial values over the 16 lanes of each half-warp so that every lane ends
// with all NV totals.  A butterfly reduce-scatter (each level halves the values a lane keeps,
// exchanging the other half with its partner) followed by an all-gather costs about
// 3*NV + log2(16) shuffles and adds instead of 4*NV for NV independent shuffle trees.
template <int NV>
__device__ __forceinline__ void halfwarp_allreduce(float (&v)[NV], int ln, int hw) {
  if constexpr (NV > 16) {
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1)
#pragma unroll
      for (int k = 0; k < NV; ++k) v[k] += __shfl_xor_sync(0xffffffffu, v[k], off);
  } else {
#pragma unroll
    for (int lvl = 0; lvl < 4; ++lvl) {
      const int off = 8 >> lvl;
      const int cur = NV >> lvl;  // values still held before this level (compile-time after unrolling)
      if (cur >= 2) {
        const bool upper = (ln & off) != 0;
#pragma unroll
        for (int k = 0; k < (NV >> (lvl + 1)); ++k) {
          const float lo = v[k], hi = v[k + (NV >> (lvl + 1))];
          const float send = upper ? lo : hi;
          const float keep = upper ? hi : lo;
          v[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      } else {
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
      }
    }
    // Lane ln now holds total number (ln >> (4 - log2 NV)); gather all of them.
    constexpr int kShift = NV == 1 ? 4 : NV == 2 ? 3 : NV == 4 ? 2 : NV == 8 ? 1 : 0;
    const float mine = v[0];
#pragma unroll
    for (int k = 0; k < NV; ++k) v[k] = __shfl_sync(0xffffffffu, mine, hw * 16 + (k << kShift));
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float (&x)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Merge softmax state (m2, l2, a2) into (m, l, a).  m == -inf means "empty".
template <int G>
__device__ __forceinline__ void merge_state(float (&m)[G], float (&l)[G], float2 (&a)[G][4], const float (&m2)[G],
                                            const float (&l2)[G], const float2 (&a2)[G][4]) {
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const float mn = fmaxf(m[j], m2[j]);
    if (mn == -INFINITY) continue;
    const float c1 = exp2f(m[j] - mn);
    const float c2 = exp2f(m2[j] - mn);
    l[j] = l[j] * c1 + l2[j] * c2;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      a[j][c] = __ffma2_rn(a[j][c], make_float2(c1, c1), __fmul2_rn(a2[j][c], make_float2(c2, c2)));
    m[j] = mn;
  }
}

template <bool B>
struct BoolTag {
  static constexpr bool value = B;
};

// Softmax reference maximum moves only when a tile's maximum exceeds it by more than this (log2
// units): probabilities stay <= 2^8 (exact range in fp32) and the accumulators are rescaled in
// few tiles instead of every one.
constexpr float kLazyLog2 = 8.f;

// One staged tile of kT tokens for this warp's KV head: the half-warp's kTPH tokens, all G query
// heads.  kFull: every token of the tile is inside the context (no per-token checks).
template <bool FP8, int G, int HK, int SPLIT, class FullTag>
__device__ __forceinline__ void decode_tile(FullTag, const uint8_t* Ks, int tile_tok0, int tok1, int phase, int hw,
                                            int ln, int h, const float2 (&qs)[G][4], float (&m)[G], float (&l)[G],
                                            float2 (&acc)[G][4]) {
  constexpr bool kFull = FullTag::value;
  using Tr = Traits<FP8, HK, SPLIT>;
  constexpr int kTPW = Tr::kTPW;
  constexpr int kTPH = Tr::kTPH;
  constexpr int kRow = Tr::kRowBytes;
  const uint8_t* Vs = Ks + Tr::kTileB;
  // Partial q.k over this lane's 8 dimensions, packed fp32x2 FMAs; sc[j * kTPH + i].
  float sc[G * kTPH];
  bool valid[kTPH];
#pragma unroll
  for (int i = 0; i < kTPH; ++i) {
    const int tt = phase * kTPW + 2 * i + hw;
    valid[i] = kFull || tile_tok0 + tt < tok1;
    float2 kx[4];
    load8x2<FP8>(Ks + tt * kRow + (h * kHeadDim + 8 * ln) * Tr::kElem, kx);
#pragma unroll
    for (int j = 0; j < G; ++j) {
      float2 a = __fmul2_rn(qs[j][0], kx[0]);
      a = __ffma2_rn(qs[j][1], kx[1], a);
      a = __ffma2_rn(qs[j][2], kx[2], a);
      a = __ffma2_rn(qs[j][3], kx[3], a);
      sc[j * kTPH + i] = a.x + a.y;
    }
  }
  halfwarp_allreduce<G * kTPH>(sc, ln, hw);

  float pr[G][kTPH];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    float mt = -INFINITY;
#pragma unroll
    for (int i = 0; i < kTPH; ++i)
      if (valid[i]) mt = fmaxf(mt, sc[j * kTPH + i]);
    if (mt > m[j] + kLazyLog2) {  // also the first tile with a token (m = -inf)
      const float corr = exp2f(m[j] - mt);
      l[j] *= corr;
      const float2 c2 = make_float2(corr, corr);
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[j][c] = __fmul2_rn(acc[j][c], c2);
      m[j] = mt;
    }
    if (m[j] == -INFINITY) {
#pragma unroll
      for (int i = 0; i < kTPH; ++i) pr[j][i] = 0.f;
      continue;
    }
    float ps = 0.f;
#pragma unroll
    for (int i = 0; i < kTPH; ++i) {
      pr[j][i] = valid[i] ? exp2f(sc[j * kTPH + i] - m[j]) : 0.f;
      ps += pr[j][i];
    }
    l[j] += ps;
  }
#pragma unroll
  for (int i = 0; i < kTPH; ++i) {
    if (!valid[i]) continue;  // never touch V rows past the context (may hold NaN bits)
    const int tt = phase * kTPW + 2 * i + hw;
    float2 vx[4];
    load8x2<FP8>(Vs + tt * kRow + (h * kHeadDim + 8 * ln) * Tr::kElem, vx);
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const float2 p2 = make_float2(pr[j][i], pr[j][i]);
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[j][c] = __ffma2_rn(p2, vx[c], acc[j][c]);
    }
  }
}

template <bool FP8, int G, int HK, int SPLIT>
__global__ void __launch_bounds__(kDecodeThreads, ctas_per_sm<FP8, G>())
paged_decode_kernel(const DecodeParams p) {
  using Tr = Traits<FP8, HK, SPLIT>;
  constexpr int kTileBytes = Tr::kTileB;
  constexpr int kT = Tr::kT;
  constexpr int kRow = Tr::kRowBytes;
  constexpr int kHq = HK * G;

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * 2 * kTileBytes);
  int* flag_smem = reinterpret_cast<int*>(full + kStages);

  const int split = blockIdx.x;
  const int b = blockIdx.y;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int ln = lane & 15;  // D-slice: elements [8*ln, 8*ln + 8)
  const int hw = lane >> 4;  // half-warp
  const int h = warp % HK;   // local KV head of this warp
  const int phase = warp / HK;

  int32_t* ws_err = reinterpret_cast<int32_t*>(p.ws + kWsErrOff);
  int32_t* tickets = reinterpret_cast<int32_t*>(p.ws + kWsTicketOff);
  float2* ws_ml = reinterpret_cast<float2*>(p.ws + kWsMlOff);
  float* ws_o = reinterpret_cast<float*>(
      p.ws + kWsMlOff + align256(int64_t(p.batch) * p.max_splits * kHq * sizeof(float2)));

  // Launched as a programmatic dependent of the previous kernel in the stream: the CTAs may be
  // scheduled while it finishes, but nothing earlier kernels wrote (context lengths, block
  // tables, q, the cache) is read before griddepcontrol.wait, so any predecessor is safe.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int L = p.context_lens[b];
  const int Lmax = p.max_blocks * p.block_size;
  L = L < 0 ? 0 : (L > Lmax ? Lmax : L);
  const int n_splits = (L + SPLIT - 1) / SPLIT;
  __nv_bfloat16* out_b = p.out + int64_t(b) * p.out_row_stride;

  if (split >= n_splits) {
    if (split == 0) {  // empty sequence (padding row): finite zeros, like an empty softmax
      for (int i = tid; i < kHq * kHeadDim / 8; i += kDecodeThreads)
        reinterpret_cast<uint4*>(out_b)[i] = make_uint4(0, 0, 0, 0);
    }
    return;
  }

  const int tok0 = split * SPLIT;
  const int tok1 = min(L, tok0 + SPLIT);
  const int page = tok0 / p.block_size;
  const int64_t block = p.block_tables[int64_t(b) * p.bt_stride + page];
  const bool bad_block = block < 0 || block >= p.num_blocks;
  const int ntiles = (tok1 - tok0 + kT - 1) / kT;
  const int64_t base_slot = block * p.block_size + (tok0 % p.block_size);
  const uint8_t* kbase = p.k_cache + base_slot * kRow;
  const uint8_t* vbase = p.v_cache + base_slot * kRow;

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
    *flag_smem = 0;
  }
  __syncthreads();

  if (bad_block) {
    if (tid == 0) atomicOr(ws_err, 2);
  } else if (tid == 0) {
    const int npre = ntiles < kStages ? ntiles : kStages;
    for (int i = 0; i < npre; ++i) {
      mbar_arrive_expect_tx(&full[i], 2 * kT * kRow);
      bulk_g2s(smem + i * 2 * kTileBytes, kbase + int64_t(i) * kT * kRow, kT * kRow, &full[i]);
      bulk_g2s(smem + i * 2 * kTileBytes + kTileBytes, vbase + int64_t(i) * kT * kRow, kT * kRow, &full[i]);
    }
  }

  // Query slice of the G query heads that share KV head h, pre-scaled so that the
  // softmax runs in base 2 (and, for FP8, with k_scale folded in).
  float2 qs[G][4];
  {
    const float ks = (FP8 && p.k_scale) ? p.k_scale[h] : 1.0f;
    const float f = p.scale_log2 * ks;
    const __nv_bfloat16* qb = p.q + int64_t(b) * p.q_row_stride;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(qb + (h * G + j) * kHeadDim + 8 * ln);
      qs[j][0] = make_float2(bf16lo(v.x) * f, bf16hi(v.x) * f);
      qs[j][1] = make_float2(bf16lo(v.y) * f, bf16hi(v.y) * f);
      qs[j][2] = make_float2(bf16lo(v.z) * f, bf16hi(v.z) * f);
      qs[j][3] = make_float2(bf16lo(v.w) * f, bf16hi(v.w) * f);
    }
  }

  float m[G], l[G];
  float2 acc[G][4];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[j][c] = make_float2(0.f, 0.f);
  }

  bool timed_out = false;
  if (!bad_block) {
    for (int t = 0; t < ntiles; ++t) {
      const int stage = t % kStages;
      // A wait that gives up is made warp-uniform here and CTA-uniform at the barrier
      // below, so no thread is left alone in a shuffle or a __syncthreads.
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], (t / kStages) & 1));
      if (ok) {
        const uint8_t* Ks = smem + stage * 2 * kTileBytes;
        const int tile_tok0 = tok0 + t * kT;
        if (tile_tok0 + kT <= tok1)
          decode_tile<FP8, G, HK, SPLIT>(BoolTag<true>{}, Ks, tile_tok0, tok1, phase, hw, ln, h, qs, m, l, acc);
        else
          decode_tile<FP8, G, HK, SPLIT>(BoolTag<false>{}, Ks, tile_tok0, tok1, phase, hw, ln, h, qs, m, l, acc);
      }  // ok
      // Every warp is done with this stage: refill it (or leave together on a timeout).
      if (__syncthreads_or(!ok)) {
        timed_out = true;
        break;
      }
      if (tid == 0 && t + kStages < ntiles) {
        const int nt = t + kStages;
        mbar_arrive_expect_tx(&full[stage], 2 * kT * kRow);
        bulk_g2s(smem + stage * 2 * kTileBytes, kbase + int64_t(nt) * kT * kRow, kT * kRow, &full[stage]);
        bulk_g2s(smem + stage * 2 * kTileBytes + kTileBytes, vbase + int64_t(nt) * kT * kRow, kT * kRow,
                 &full[stage]);
      }
    }
  }
  if (timed_out) {
    if (tid == 0) {
      atomicOr(ws_err, 1);
      // Give copies still in flight a second bounded chance to land before the CTA's
      // shared memory is released.
      for (int i = 0; i < kStages; ++i) mbar_wait(&full[i], 0), mbar_wait(&full[i], 1);
    }
    return;
  }

  // Merge the two half-warps (they hold disjoint token subsets of the same D-slice).
  {
    float m2[G], l2[G];
    float2 a2[G][4];
#pragma unroll
    for (int j = 0; j < G; ++j) {
      m2[j] = __shfl_xor_sync(0xffffffffu, m[j], 16);
      l2[j] = __shfl_xor_sync(0xffffffffu, l[j], 16);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        a2[j][c] = make_float2(__shfl_xor_sync(0xffffffffu, acc[j][c].x, 16),
                               __shfl_xor_sync(0xffffffffu, acc[j][c].y, 16));
    }
    merge_state<G>(m, l, acc, m2, l2, a2);
  }

  // Merge warps that share a KV head (only when Hk < 8).  Stage buffers are free: every
  // issued bulk copy has been waited for.
  if constexpr (Tr::kPhases > 1) {
    __syncthreads();
    float* scr = reinterpret_cast<float*>(smem);  // [warp][j][lane 0..15][10]
    if (phase > 0 && hw == 0) {
#pragma unroll
      for (int j = 0; j < G; ++j) {
        float* e = scr + ((warp * G + j) * 16 + ln) * 10;
        e[0] = m[j];
        e[1] = l[j];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          e[2 + 2 * c] = acc[j][c].x;
          e[3 + 2 * c] = acc[j][c].y;
        }
      }
    }
    __syncthreads();
    if (phase == 0) {
      for (int ph = 1; ph < Tr::kPhases; ++ph) {
        const int w2 = ph * HK + h;
        float m2[G], l2[G];
        float2 a2[G][4];
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const float* e = scr + ((w2 * G + j) * 16 + ln) * 10;
          m2[j] = e[0];
          l2[j] = e[1];
#pragma unroll
          for (int c = 0; c < 4; ++c) a2[j][c] = make_float2(e[2 + 2 * c], e[3 + 2 * c]);
        }
        merge_state<G>(m, l, acc, m2, l2, a2);
      }
    }
  }

  const float vs = (FP8 && p.v_scale) ? p.v_scale[h] : 1.0f;
  if (n_splits == 1) {
    if (phase == 0 && hw == 0) {
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const float inv = l[j] > 0.f ? vs / l[j] : 0.f;
        float o[8];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          o[2 * c] = acc[j][c].x * inv;
          o[2 * c + 1] = acc[j][c].y * inv;
        }
        *reinterpret_cast<uint4*>(out_b + (h * G + j) * kHeadDim + 8 * ln) = pack_bf16x8(o);
      }
    }
    return;
  }

  // Write this split's partial state, then take a ticket; the last CTA combines.
  if (phase == 0 && hw == 0) {
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int hq = h * G + j;
      const int64_t row = (int64_t(b) * p.max_splits + split) * kHq + hq;
      float* o = ws_o + row * kHeadDim + 8 * ln;
      reinterpret_cast<float4*>(o)[0] =
          make_float4(acc[j][0].x * vs, acc[j][0].y * vs, acc[j][1].x * vs, acc[j][1].y * vs);
      reinterpret_cast<float4*>(o)[1] =
          make_float4(acc[j][2].x * vs, acc[j][2].y * vs, acc[j][3].x * vs, acc[j][3].y * vs);
      if (ln == 0) ws_ml[row] = make_float2(m[j], l[j]);
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(&tickets[b], 1);
    *flag_smem = (prev == n_splits - 1);
  }
  __syncthreads();
  if (!*flag_smem) return;
  __threadfence();

  // Last CTA of sequence b: combine the n_splits partials.  Each thread produces 8
  // consecutive output elements of one query head.
  for (int idx = tid; idx < kHq * (kHeadDim / 8); idx += kDecodeThreads) {
    const int hq = idx / (kHeadDim / 8);
    const int d0 = (idx % (kHeadDim / 8)) * 8;
    const int64_t row0 = int64_t(b) * p.max_splits * kHq + hq;
    float mx = -INFINITY;
    for (int s = 0; s < n_splits; ++s) mx = fmaxf(mx, __ldcg(&ws_ml[row0 + int64_t(s) * kHq]).x);
    float lsum = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (mx != -INFINITY) {
      for (int s = 0; s < n_splits; ++s) {
        const int64_t row = row0 + int64_t(s) * kHq;
        const float2 ml = __ldcg(&ws_ml[row]);
        if (ml.x == -INFINITY) continue;
        const float c = exp2f(ml.x - mx);
        lsum += ml.y * c;
        const float4* src = reinterpret_cast<const float4*>(ws_o + row * kHeadDim + d0);
        const float4 a = __ldcg(src), bq = __ldcg(src + 1);
        o[0] += a.x * c;
        o[1] += a.y * c;
        o[2] += a.z * c;
        o[3] += a.w * c;
        o[4] += bq.x * c;
        o[5] += bq.y * c;
        o[6] += bq.z * c;
        o[7] += bq.w * c;
      }
    }
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
#pragma unroll
    for (int d = 0; d < 8; ++d) o[d] *= inv;
    *reinterpret_cast<uint4*>(out_b + hq * kHeadDim + d0) = pack_bf16x8(o);
  }
  if (tid == 0) tickets[b] = 0;  // ready for the next launch
}

template <bool FP8, int G, int HK, int SPLIT>
int launch_decode(const DecodeParams& p, cudaStream_t stream) {
  constexpr size_t smem = size_t(kStages) * 2 * Traits<FP8, HK>::kTileB + kStages * sizeof(uint64_t) + 16;
  // The shared-memory opt-in is per device; the first call on a device happens before any graph
  // capture (the engine's eager warm-up).
  static std::atomic<bool> configured[kMaxDecodeDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDecodeDevices) {
    set_error("hl_paged_decode: no usable current device");
    return HL_ERR_CUDA;
  }
  if (!configured[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(paged_decode_kernel<FP8, G, HK, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(smem));
    if (e != cudaSuccess) {
      set_error("hl_paged_decode: cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return HL_ERR_CUDA;
    }
    configured[dev].store(true, std::memory_order_release);
  }
  // Launched as a programmatic dependent of the previous kernel in the stream (see the kernel's
  // griddepcontrol.wait placement).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.max_splits, p.batch);
  cfg.blockDim = dim3(kDecodeThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, paged_decode_kernel<FP8, G, HK, SPLIT>, p);
  if (e != cudaSuccess) {
    set_error("hl_paged_decode: launch failed: %s", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  return HL_OK;
}

template <bool FP8, int G, int SPLIT>
int dispatch_hk(int hk, const DecodeParams& p, cudaStream_t s) {
  switch (hk) {
    case 1: return launch_decode<FP8, G, 1, SPLIT>(p, s);
    case 2: return launch_decode<FP8, G, 2, SPLIT>(p, s);
    case 4: return launch_decode<FP8, G, 4, SPLIT>(p, s);
    case 8: return launch_decode<FP8, G, 8, SPLIT>(p, s);
  }
  set_error("hl_paged_decode: num_kv_heads=%d not in {1,2,4,8}", hk);
  return HL_ERR_UNSUPPORTED;
}

template <bool FP8, int SPLIT>
int dispatch_g(int g, int hk, const DecodeParams& p, cudaStream_t s) {
  switch (g) {
    case 1: return dispatch_hk<FP8, 1, SPLIT>(hk, p, s);
    case 2: return dispatch_hk<FP8, 2, SPLIT>(hk, p, s);
    case 4: return dispatch_hk<FP8, 4, SPLIT>(hk, p, s);
    case 8: return dispatch_hk<FP8, 8, SPLIT>(hk, p, s);
  }
  set_error("hl_paged_decode: Hq/Hk=%d not in {1,2,4,8}", g);
  return HL_ERR_UNSUPPORTED;
}

int64_t max_splits_for(int max_blocks, int block_size, int split = kSplit) {
  return (int64_t(max_blocks) * block_size + split - 1) / split;
}

// Small launches (a few sequences) run with 32-token splits: the grid of 128-token splits would
// leave most SMs idle (config 1: 8 sequences of up to 1024 tokens = 64 CTAs on 148 SMs), and a
// split streams its tokens at the rate one CTA's pipeline allows.  The choice depends only on the
// batch size and the block-table width, so a CUDA graph replays the same grid.
constexpr int kSmallSplit = 32;
constexpr int kSmallGridCtas = 296;  // 2 x the SMs of a B200


}  // namespace
}  // namespace hl

namespace hl {
int64_t decode_tc_workspace_bytes(int batch, int num_q_heads);
int64_t tc_ticket_end(int batch, int num_q_heads);
int decode_tc_launch(const void* q, int64_t q_row_stride, const void* k_cache, const void* v_cache, bool fp8,
                     const float* k_scale, const float* v_scale, const int32_t* block_tables, int64_t bt_stride,
                     int max_blocks, const int32_t* context_lens, int batch, int num_q_heads, int num_kv_heads,
                     int block_size, int64_t num_blocks, float scale_log2, void* out, int64_t out_row_stride, void* ws,
                     cudaStream_t stream);
bool decode_tc_supported(int batch, int num_q_heads, int num_kv_heads, int block_size, bool fp8);
}  // namespace hl

using namespace hl;

extern "C" int64_t hl_paged_decode_workspace_size(int batch, int num_q_heads, int head_dim, int max_blocks_per_seq,
                                                  int block_size) {
  if (batch <= 0 || num_q_heads <= 0 || head_dim <= 0 || max_blocks_per_seq <= 0 || block_size <= 0) return -1;
  // (sequence, split) partial slots: the 128-token grid's, or the small grid's, which runs only
  // while batch x 128-token splits < kSmallGridCtas (bounded so the size grows with the batch).
  const int64_t units = int64_t(batch) * max_splits_for(max_blocks_per_seq, block_size);
  const int64_t units_small = int64_t(batch) * max_splits_for(max_blocks_per_seq, block_size, kSmallSplit);
  const int64_t cap_small = int64_t(kSmallGridCtas) * (kSplit / kSmallSplit);
  const int64_t u = units > (units_small < cap_small ? units_small : cap_small)
                        ? units : (units_small < cap_small ? units_small : cap_small);
  const int64_t rows = u * num_q_heads;
  const int64_t simt = kWsMlOff + align256(rows * int64_t(sizeof(float2))) + rows * head_dim * int64_t(sizeof(float));
  const int64_t tc = decode_tc_workspace_bytes(batch, num_q_heads);
  return simt > tc ? simt : tc;
}

namespace {
int paged_decode_impl(bool allow_tc, const void* q, int64_t q_row_stride, const void* k_cache, const void* v_cache,
                      int kv_dtype, const float* k_scale, const float* v_scale, const int32_t* block_tables,
                      int64_t bt_stride, int max_blocks_per_seq, const int32_t* context_lens, int batch,
                      int num_q_heads, int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                      float softmax_scale, void* out, int64_t out_row_stride, void* workspace, int64_t workspace_bytes,
                      void* stream);
}

extern "C" int hl_paged_decode(const void* q, int64_t q_row_stride, const void* k_cache, const void* v_cache,
                               int kv_dtype, const float* k_scale, const float* v_scale, const int32_t* block_tables,
                               int64_t bt_stride, int max_blocks_per_seq, const int32_t* context_lens, int batch,
                               int num_q_heads, int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                               float softmax_scale, void* out, int64_t out_row_stride, void* workspace,
                               int64_t workspace_bytes, void* stream) {
  return paged_decode_impl(false, q, q_row_stride, k_cache, v_cache, kv_dtype, k_scale, v_scale, block_tables,
                           bt_stride, max_blocks_per_seq, context_lens, batch, num_q_heads, num_kv_heads, head_dim,
                           block_size, num_blocks, softmax_scale, out, out_row_stride, workspace, workspace_bytes,
                           stream);
}

extern "C" int hl_paged_decode_tc(const void* q, int64_t q_row_stride, const void* k_cache, const void* v_cache,
                                    int kv_dtype, const float* k_scale, const float* v_scale,
                                    const int32_t* block_tables, int64_t bt_stride, int max_blocks_per_seq,
                                    const int32_t* context_lens, int batch, int num_q_heads, int num_kv_heads,
                                    int head_dim, int block_size, int64_t num_blocks, float softmax_scale, void* out,
                                    int64_t out_row_stride, void* workspace, int64_t workspace_bytes, void* stream) {
  return paged_decode_impl(true, q, q_row_stride, k_cache, v_cache, kv_dtype, k_scale, v_scale, block_tables,
                           bt_stride, max_blocks_per_seq, context_lens, batch, num_q_heads, num_kv_heads, head_dim,
                           block_size, num_blocks, softmax_scale, out, out_row_stride, workspace, workspace_bytes,
                           stream);
}

namespace {

int paged_decode_impl(bool allow_tc, const void* q, int64_t q_row_stride, const void* k_cache, const void* v_cache,
                      int kv_dtype, const float* k_scale, const float* v_scale, const int32_t* block_tables,
                      int64_t bt_stride, int max_blocks_per_seq, const int32_t* context_lens, int batch,
                      int num_q_heads, int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                      float softmax_scale, void* out, int64_t out_row_stride, void* workspace, int64_t workspace_bytes,
                      void* stream) {
  clear_error();
  HL_CHECK_ARG(batch >= 0, "hl_paged_decode: batch < 0");
  if (batch == 0) return HL_OK;
  HL_CHECK_ARG(batch <= kMaxBatch, "hl_paged_decode: batch %d > %d", batch, kMaxBatch);
  HL_CHECK_ARG(q && k_cache && v_cache && block_tables && context_lens && out, "hl_paged_decode: null pointer");
  HL_CHECK_ARG(head_dim == kHeadDim, "hl_paged_decode: head_dim %d != 128", head_dim);
  HL_CHECK_ARG(block_size > 0 && block_size % 256 == 0, "hl_paged_decode: block_size %% 256 != 0");
  HL_CHECK_ARG(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0, "hl_paged_decode: Hq %% Hk != 0");
  HL_CHECK_ARG(kv_dtype == HL_KV_BF16 || kv_dtype == HL_KV_FP8_E4M3, "hl_paged_decode: bad kv_dtype");
  HL_CHECK_ARG(max_blocks_per_seq > 0 && bt_stride >= max_blocks_per_seq, "hl_paged_decode: bad block table width");
  HL_CHECK_ARG(aligned16(q) && q_row_stride % 8 == 0 && q_row_stride >= int64_t(num_q_heads) * head_dim,
               "hl_paged_decode: q must be 16-byte aligned with row stride %% 8 == 0");
  HL_CHECK_ARG(aligned16(out) && out_row_stride % 8 == 0 && out_row_stride >= int64_t(num_q_heads) * head_dim,
               "hl_paged_decode: out must be 16-byte aligned with row stride %% 8 == 0");
  HL_CHECK_ARG(aligned16(k_cache) && aligned16(v_cache), "hl_paged_decode: caches must be 16-byte aligned");
  const int64_t need =
      hl_paged_decode_workspace_size(batch, num_q_heads, head_dim, max_blocks_per_seq, block_size);
  if (!workspace || workspace_bytes < need || !aligned16(workspace)) {
    set_error("hl_paged_decode: workspace of %lld bytes needed (got %lld)", (long long)need,
              (long long)workspace_bytes);
    return HL_ERR_WORKSPACE;
  }
  const bool small = int64_t(batch) * max_splits_for(max_blocks_per_seq, block_size) < kSmallGridCtas;
  const int64_t S = max_splits_for(max_blocks_per_seq, block_size, small ? kSmallSplit : kSplit);
  HL_CHECK_ARG(S <= 65535, "hl_paged_decode: too many splits");

  DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_row_stride = q_row_stride;
  p.k_cache = static_cast<const uint8_t*>(k_cache);
  p.v_cache = static_cast<const uint8_t*>(v_cache);
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.block_tables = block_tables;
  p.bt_stride = bt_stride;
  p.max_blocks = max_blocks_per_seq;
  p.context_lens = context_lens;
  p.batch = batch;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.max_splits = int(S);
  p.scale_log2 = softmax_scale * kLog2e;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_row_stride = out_row_stride;
  p.ws = static_cast<uint8_t*>(workspace);

  const int g = num_q_heads / num_kv_heads;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool fp8 = kv_dtype == HL_KV_FP8_E4M3;
  // With four or more query heads per KV head (two or more for e4m3 bytes) the CUDA-core
  // kernel spends two or more FMAs per cache byte plus the half-warp score reductions and runs
  // out of issue slots well below the HBM rate (BF16 at 256 x 900 tokens: G = 4 0.59 of the copy
  // peak, G = 8 0.24; e4m3 G = 4 0.28), while the tcgen05 kernel puts the G heads on the MMA's
  // N = 16 columns at no extra cost.  For BF16 G <= 2 the CUDA-core kernel is the faster one at
  // every measured length.
  const bool tc_fits = decode_tc_supported(batch, num_q_heads, num_kv_heads, block_size, fp8) &&
                       num_blocks * block_size < (int64_t(1) << 31);
  // One KV head per GPU (tensor parallelism over all 8 heads): the CUDA-core kernel keeps only 8
  // warps' worth of one head per CTA and the tensor-core kernel is ahead already at GQA 2
  // (Hq 2 / Hk 1, 256 x U[65, 1087] tokens: 25.8 vs 28.1 us).
  const bool tc_preferred = g >= (fp8 ? kTcMinGroupFp8 : kTcMinGroupBf16) || (!fp8 && num_kv_heads == 1 && g == 2);
  if (allow_tc || (tc_preferred && tc_fits)) {
    if (!decode_tc_supported(batch, num_q_heads, num_kv_heads, block_size, fp8)) {
      set_error("hl_paged_decode_tc: needs batch <= 2048, Hq/Hk in {1,2,4,8,16} (BF16) or {1,2,4,8} (FP8), "
                "block_size %% 128 == 0");
      return HL_ERR_UNSUPPORTED;
    }
    HL_CHECK_ARG(tc_fits, "hl_paged_decode_tc: cache too large");
    return decode_tc_launch(q, q_row_stride, k_cache, v_cache, fp8, k_scale, v_scale, block_tables, bt_stride,
                            max_blocks_per_seq, context_lens, batch, num_q_heads, num_kv_heads, block_size,
                            num_blocks, p.scale_log2, out, out_row_stride, workspace, s);
  }
  if (small) return fp8 ? dispatch_g<true, kSmallSplit>(g, num_kv_heads, p, s)
                        : dispatch_g<false, kSmallSplit>(g, num_kv_heads, p, s);
  return fp8 ? dispatch_g<true, kSplit>(g, num_kv_heads, p, s) : dispatch_g<false, kSplit>(g, num_kv_heads, p, s);
}

}  // namespace

extern "C" int hl_paged_decode_read_errors(const void* workspace, int32_t* errors_out, void* stream) {
  clear_error();
  HL_CHECK_ARG(workspace && errors_out, "hl_paged_decode_read_errors: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(errors_out, static_cast<const uint8_t*>(workspace) + kWsErrOff, sizeof(int32_t),
                                  cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    set_error("hl_paged_decode_read_errors: %s", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  return HL_OK;
}

// ------------------------------------------------------------------------------------------
// Allocation-free variant of the decode entry point.
//
// Some callers cannot hand us a workspace: hosts that bind this library through a foreign-
// function interface and have no device allocator of their own, serving loops whose memory
// is fully carved out up front and that must not call cudaMalloc (it synchronises the device
// and can fail under memory pressure), and plugins that may only touch the buffers their
// host passes in.  For them the split-K scratch lives in this file-scope device array, which
// every GPU that loads the library reserves once, until the process exits.
// ------------------------------------------------------------------------------------------
namespace hl {
namespace {

constexpr int64_t kNoAllocScratchBytes = int64_t(32) << 20;  // 32 MiB per GPU
static __device__ __align__(256) uint8_t g_decode_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::atomic<uint8_t*> g_scratch_ptr[kMaxDevices];
std::mutex g_scratch_mutex;

// Device address of g_decode_scratch on the current device (host code only holds a host-side
// stand-in for the symbol, so the address must be looked up per device).
int scratch_for_current_device(uint8_t** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("hl_paged_decode_noalloc: no usable current device (%s)", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  uint8_t* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    p = g_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      void* addr = nullptr;
      e = cudaGetSymbolAddress(&addr, g_decode_scratch);
      if (e != cudaSuccess || addr == nullptr) {
        set_error("hl_paged_decode_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        return HL_ERR_CUDA;
      }
      p = static_cast<uint8_t*>(addr);
      g_scratch_ptr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return HL_OK;
}

}  // namespace
}  // namespace hl

extern "C" int64_t hl_paged_decode_noalloc_capacity(void) { return hl::kNoAllocScratchBytes; }

extern "C" int hl_paged_decode_noalloc(const void* q, int64_t q_row_stride, const void* k_cache, const void* v_cache,
                                       int kv_dtype, const float* k_scale, const float* v_scale,
                                       const int32_t* block_tables, int64_t bt_stride, int max_blocks_per_seq,
                                       const int32_t* context_lens, int batch, int num_q_heads, int num_kv_heads,
                                       int head_dim, int block_size, int64_t num_blocks, float softmax_scale,
                                       void* out, int64_t out_row_stride, void* stream) {
  clear_error();
  HL_CHECK_ARG(batch >= 0, "hl_paged_decode_noalloc: batch < 0");
  if (batch == 0) return HL_OK;
  HL_CHECK_ARG(num_q_heads > 0 && head_dim > 0 && max_blocks_per_seq > 0 && block_size > 0,
               "hl_paged_decode_noalloc: bad shape");
  const int64_t need =
      hl_paged_decode_workspace_size(batch, num_q_heads, head_dim, max_blocks_per_seq, block_size);
  if (need < 0 || need > kNoAllocScratchBytes) {
    set_error("hl_paged_decode_noalloc: this shape needs %lld bytes of scratch, more than the built-in %lld "
              "(use hl_paged_decode with a caller-provided workspace)",
              (long long)need, (long long)kNoAllocScratchBytes);
    return HL_ERR_UNSUPPORTED;
  }
  uint8_t* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc != HL_OK) return rc;
  // The array keeps whatever the previous call left: zero the error word and the tickets,
  // which the kernel expects to find at zero (the partials are always written before read).
  // (both kernels keep the error word at 0 and their tickets right after it).
  const int64_t zero_bytes = kWsMlOff > tc_ticket_end(batch, num_q_heads) ? kWsMlOff : tc_ticket_end(batch, num_q_heads);
  cudaError_t e = cudaMemsetAsync(scratch, 0, size_t(zero_bytes), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("hl_paged_decode_noalloc: cudaMemsetAsync failed: %s", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  return hl_paged_decode(q, q_row_stride, k_cache, v_cache, kv_dtype, k_scale, v_scale, block_tables, bt_stride,
                         max_blocks_per_seq, context_lens, batch, num_q_heads, num_kv_heads, head_dim, block_size,
                         num_blocks, softmax_scale, out, out_row_stride, scratch, kNoAllocScratchBytes, stream);
}

// Error bits the most recent hl_paged_decode_noalloc call on the current device left in the
// scratch array's error word (each call starts it from zero).  Synchronises `stream`.
extern "C" int hl_paged_decode_noalloc_read_errors(int32_t* errors_out, void* stream) {
  clear_error();
  HL_CHECK_ARG(errors_out, "hl_paged_decode_noalloc_read_errors: null pointer");
  uint8_t* scratch = nullptr;
  int rc = hl::scratch_for_current_device(&scratch);
  if (rc != HL_OK) return rc;
  return hl_paged_decode_read_errors(scratch, errors_out, stream);
}
