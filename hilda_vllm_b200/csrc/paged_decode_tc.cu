// Paged decode attention on the 5th-generation tensor cores (BF16 or FP8 e4m3 KV cache).
//
// Semantics: as paged_decode.cu (flash_attn_with_kvcache with one query token per sequence,
// mini_vllm/layers/attention.py:162-170): out[b, hq] = softmax_j(scale q[b,hq].K[b,j,hq/G])
// V[b,j,hq/G] over j < L_b, key j at slot block_tables[b, j/BS]*BS + j%BS; L_b == 0 gives zeros.
//
// The CUDA-core kernel spends two FMAs per cache byte and query head plus the cross-lane score
// reductions, so with four or more query heads per KV head it runs out of issue slots; here the
// two products run on tcgen05 with the G query heads of a KV head as the (padded) N dimension:
//     S^T [128 tokens x 16] = K_tile [128 x 128] . Q_h^T        (A = K tile, K-major)
//     O^T [128 dims  x 16] += V_tile^T [128 x 128] . P^T          (A = V tile read MN-major)
// both with M = 128, N = 16, K = 16 steps, fp32 in TMEM.  The K and V tiles arrive by TMA in the
// same 128-byte-swizzled layout the prefill kernel uses; Q (G rows of the head, rest zero) comes
// with each tile.  Softmax: thread = token = TMEM lane of S^T, the per-head max and sum across
// the 128 tokens by warp shuffles and a 4-warp exchange in shared memory; P^T (bf16 hi + lo,
// ~16 significant bits; for 2G <= 16 the two parts are rows [0, G) and [G, 2G) of one operand,
// so one PV pass gives both) goes to shared memory in the K-major layout of the B operand.  O is
// rescaled lazily (the reference maximum moves only when a tile exceeds it by 2^8).  V rows past
// the context are zeroed before the PV product (P is 0 there; the cache may hold NaN bits).
// FP8 caches: QK in kind::f8f6f4 on the staged e4m3 K bytes with Q as two exact e4m3 terms, and
// converter warps 10-13 turning V into f16 (details with the constants below).
//
// Work: a unit is (sequence b, KV head h, 128-token tile t), 64 KiB of K+V.  The grid is one CTA
// per SM; CTA c takes the contiguous unit range [c*upc, (c+1)*upc) of the (b, h, t)-ordered list
// (upc = ceil(units / grid)), so every CTA streams the same number of bytes and the TMA pipeline
// (3 stages) runs across sequence boundaries.  A (b, h) pair cut by a range boundary is finished
// by the last of its CTAs to arrive (ticket), which merges the partial (m, l, O) of the others.
// Warp 0 issues TMA, warp 1 owns TMEM and issues the MMAs, warps 2-5 run the softmax, warps 6-9
// the per-(b, h) epilogues (normalise O and store, or publish a partial and merge), so a pair
// boundary never stalls the softmax; FP8 adds warps 10-13 (Q split, V conversion).
// Every wait is bounded; no cluster launch, no multicast.
#include "hl_common.cuh"

#include <atomic>

#include <cuda.h>

namespace hl {

int64_t decode_tc_workspace_bytes(int batch, int num_q_heads);
int64_t tc_ticket_end(int batch, int num_q_heads);
int decode_tc_launch(const void* q, int64_t q_row_stride, const void* k_cache, const void* v_cache, bool fp8,
                     const float* k_scale, const float* v_scale, const int32_t* block_tables, int64_t bt_stride,
                     int max_blocks, const int32_t* context_lens, int batch, int num_q_heads, int num_kv_heads,
                     int block_size, int64_t num_blocks, float scale_log2, void* out, int64_t out_row_stride, void* ws,
                     cudaStream_t stream);
bool decode_tc_supported(int batch, int num_q_heads, int num_kv_heads, int block_size, bool fp8);

namespace {

constexpr int kUT = 128;                    // tokens per unit
constexpr int kThreadsTc = 320;
constexpr int kStagesTc = 3;
constexpr int kHalfKV = 128 * 128;          // [128 rows x 64 bf16] swizzled block
constexpr int kKV = 2 * kHalfKV;            // one head's 128-token K (or V) tile: 32 KiB
constexpr int kHalfQ = 16 * 128;            // [16 rows x 64 bf16]
constexpr int kQ = 2 * kHalfQ;
constexpr int kStage = 2 * kKV + kQ;        // 68 KiB (a multiple of 1024)
constexpr int kHalfP = 16 * 128;
constexpr int kP = 2 * kHalfP;
constexpr int kOffP = kStagesTc * kStage;   // P^T hi [2]
constexpr int kOffPlo = kOffP + 2 * kP;     // P^T lo [2]
constexpr int kOffRed = kOffPlo + 2 * kP;   // float [2][4][16]
constexpr int kOffEp = kOffRed + 2 * 4 * 16 * 4;  // softmax -> epilogue: (m[16], l[16]) [4], flag
constexpr int kOffBarTc = kOffEp + 1024;
constexpr int kBarBytes = 512;
constexpr int kSmemTc = kOffBarTc + kBarBytes + 1024;

// FP8 (e4m3) caches.  TMA brings each unit's K and V bytes (128 tokens x 128 B of one head,
// 16 KiB each, 128-byte swizzled) and its bf16 Q rows into a 3-deep staging ring.
//   S^T = K Q^T runs as kind::f8f6f4 straight from the staged K bytes.  Q, after an exact
//   power-of-two shift that puts its largest |q| in [2^7, 2^8), is split into two e4m3 terms,
//   q1 = q truncated to 4 significant bits and q2 = q - q1 (the other <= 4 bits of a bf16), so
//   the two terms reproduce every component within 2^8 of the head's largest exactly; smaller
//   ones lose low bits to the e4m3 subnormal grid, at most 2^-16 of the largest.
//   O^T += V^T P^T needs P with f16 range and precision, so four converter warps turn each V
//   row into f16 (e4m3 -> f16 x 2^-8, exact, by bit placement) in a double-buffered tile, and
//   the product runs as kind::f16.
constexpr int kThreads8 = 448;             // + warps 10-13: Q split (once per pair), V conversion
constexpr int kStages8 = 3;
constexpr int kHalf8 = 128 * 128;           // [128 tokens x 128 e4m3]
constexpr int kStage8 = 2 * kHalf8 + kQ;    // K, V, then the bf16 Q rows: 36 KiB
constexpr int kOffV16 = kStages8 * kStage8; // V f16 [2]
constexpr int kQ8 = 16 * 128;              // Q e4m3 terms: q1 in rows [0, G), q2 in rows [G, 2G)
constexpr int kOffQ8 = kOffV16 + 2 * kKV;   // Q e4m3 terms [2]
constexpr int kOffP16 = kOffQ8 + 2 * kQ8;   // P^T f16 [2]
constexpr int kOffRed8 = kOffP16 + 2 * kP;
constexpr int kOffEp8 = kOffRed8 + 2 * 4 * 16 * 4;  // ep[4][32], flag, qf[4], qmax[2][4]
constexpr int kOffBar8 = kOffEp8 + 1024;
constexpr int kSmem8 = kOffBar8 + kBarBytes + 1024;
static_assert(kSmemTc <= 227 * 1024 && kSmem8 <= 227 * 1024, "shared memory");

constexpr int kMaxBatchTc = 2048;
constexpr int kMaxGridTc = 256;
constexpr int kMaxDevicesTc = 64;
constexpr uint32_t kTmemColsTc = 64;        // S0 [0,16) S1 [16,32) O0 [32,48) O1 [48,64)
constexpr float kRescale = 8.f;

// kind::f16 instruction descriptor: fp32 accumulate, A and B both bf16 (or both f16), M = 128,
// N = 16, B K-major, A K-major or MN-major.
__host__ __device__ constexpr uint32_t idesc_n16(bool a_mn_major, bool f16) {
  return (1u << 4) | ((f16 ? 0u : 1u) << 7) | ((f16 ? 0u : 1u) << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((16u >> 3) << 17) | ((128u >> 4) << 24);
}

struct TcDecodeParams {
  CUtensorMap tq;
  CUtensorMap tk;
  CUtensorMap tv;
  const float* k_scale;    // FP8 path, per KV head, may be null
  const float* v_scale;
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* context_lens;
  int batch;
  int max_blocks;
  int block_size;
  int num_kv_heads;
  int64_t num_blocks;
  float scale_log2;
  __nv_bfloat16* out;
  int64_t out_row_stride;
  uint8_t* ws;
};

// Workspace: [0] error word, [256] tickets[batch * Hk], then per CTA two partial slots of
// (m[G], l[G], O[G][128]) fp32.
constexpr int64_t kTcTicketOff = 256;
__host__ __device__ inline int64_t tc_part_off(int batch, int hk) {
  return kTcTicketOff + ((int64_t(batch) * hk * 4 + 255) & ~int64_t(255));
}

__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

__device__ __forceinline__ void tma3(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// A and B both e4m3 (instruction descriptor formats 0), fp32 accumulate.
__device__ __forceinline__ void mma_ss_e4m3(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// e4m3 byte of a value that e4m3 holds exactly, or of its truncation to the subnormal grid
// (multiples of 2^-9) below 2^-6; |x| < 2^8.  Branch-free.
__device__ __forceinline__ uint32_t e4m3_byte(float x) {
  const uint32_t u = __float_as_uint(x);
  const uint32_t sign = (u >> 24) & 0x80u;
  const int e = int((u >> 23) & 0xffu) - 120;  // e4m3 biased exponent
  const uint32_t m = (u >> 20) & 7u;
  const int sh = 1 - e;                        // subnormal: (1.m) >> (1 - e), zero below 2^-9
  const uint32_t sub = sh <= 4 ? (8u | m) >> sh : 0u;
  return sign | (e >= 1 ? (uint32_t(e) << 3) | m : sub);
}

// The larger e4m3 term of x: x truncated to 4 significant bits, or to the subnormal grid.
__device__ __forceinline__ float e4m3_head(float x) {
  const float a = fabsf(x);
  const float t = a >= 0.015625f ? __uint_as_float(__float_as_uint(a) & 0xfff00000u) : floorf(a * 512.f) * 0.001953125f;
  return copysignf(t, x);
}

__device__ __forceinline__ void commit_to(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float fast_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void softmax_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void epilogue_bar() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

__device__ __forceinline__ bool epilogue_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.and.pred p, 2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v))
      : "memory");
  return r != 0;
}

// AND over the 128 softmax threads (a barrier among them): every softmax warp leaves the loop
// together, so none is left alone at a later bar.sync.
__device__ __forceinline__ bool softmax_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.and.pred p, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v))
      : "memory");
  return r != 0;
}

__device__ __forceinline__ bool waitb(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < kMaxWaitPolls; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 63u) == 63u && *abort_flag) return false;
  }
  *abort_flag = 1;
  atomicOr(err, 1);
  return false;
}

// Walks the (b, h, t)-ordered unit list; every role keeps its own copy.
struct Cursor {
  int b, h, t, tiles, L;
  int64_t base;  // index of unit (b, 0, 0)
  __device__ __forceinline__ int64_t pair_first() const { return base + int64_t(h) * tiles; }
  __device__ __forceinline__ int64_t pair_last() const { return base + int64_t(h) * tiles + tiles - 1; }
};

__device__ __forceinline__ int seq_len(const TcDecodeParams& p, int b) {
  int L = p.context_lens[b];
  const int lmax = p.max_blocks * p.block_size;
  return L < 0 ? 0 : (L > lmax ? lmax : L);
}

__device__ __forceinline__ void advance(const TcDecodeParams& p, Cursor& c) {
  if (++c.t < c.tiles) return;
  c.t = 0;
  if (++c.h < p.num_kv_heads) return;
  c.h = 0;
  c.base += int64_t(p.num_kv_heads) * c.tiles;
  do {
    ++c.b;
    c.L = c.b < p.batch ? seq_len(p, c.b) : 0;
    c.tiles = (c.L + kUT - 1) / kUT;
  } while (c.b < p.batch && c.tiles == 0);
}

__device__ __forceinline__ bool convert_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.and.pred p, 3, 128, p;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v))
      : "memory");
  return r != 0;
}

// Four e4m3 bytes (dims d .. d+3, low byte first) -> f16x2 words {d, d+1} and {d+2, d+3}, every
// value multiplied by 2^-8, exactly.  Each byte goes to the high byte of its 16-bit half
// (sign at bit 15, exponent at 11-14, mantissa at 8-10); one right shift puts exponent and
// mantissa into the low four exponent bits and top three mantissa bits of the f16, so an e4m3
// value 2^(e-7) (1 + m/8) reads as 2^(e-15) (1 + m/8) and a subnormal m 2^-9 as the f16
// subnormal m 2^-17; the add carries the sign from bit 14 on to bit 15.  Four ALU operations
// per pair instead of the conversion instruction, which issues on the much narrower XU pipe.
// (The byte 0x7F / 0xFF, e4m3's NaN, reads as 480 x 2^-8; the store kernels never write it.)
__device__ __forceinline__ void e4m3x4_to_f16x2_lo(uint32_t w, uint32_t& a, uint32_t& b) {
  uint32_t x = __byte_perm(w, 0u, 0x1404u) >> 1;  // b0 -> bits 7-14, b1 -> bits 23-30
  uint32_t y = __byte_perm(w, 0u, 0x3424u) >> 1;  // b2, b3
  a = x + (x & 0x40004000u);
  b = y + (y & 0x40004000u);
}

// Loads token row r of a staged e4m3 tile (128 B, 128-byte swizzle): 8 chunks of 16 dims.
__device__ __forceinline__ void load_row8(const uint8_t* src, int r, uint4 (&w)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) w[j] = *reinterpret_cast<const uint4*>(src + r * 128 + ((j ^ (r & 7)) << 4));
}

// Writes token row r (loaded by load_row8) into an f16 operand tile (two [128 x 64] halves,
// 128-byte swizzle), values x 2^-8, or zeros when `zero`.
__device__ __forceinline__ void store_row_f16(const uint4 (&w)[8], uint8_t* dst, int r, bool zero) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {  // dims [16j, 16j + 16)
    uint32_t o[8];
    e4m3x4_to_f16x2_lo(w[j].x, o[0], o[1]);
    e4m3x4_to_f16x2_lo(w[j].y, o[2], o[3]);
    e4m3x4_to_f16x2_lo(w[j].z, o[4], o[5]);
    e4m3x4_to_f16x2_lo(w[j].w, o[6], o[7]);
    if (zero) {
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = 0u;
    }
    uint8_t* half = dst + (j >> 2) * kHalfKV + r * 128;
    const int c = 2 * (j & 3);
    *reinterpret_cast<uint4*>(half + ((c ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(half + (((c + 1) ^ (r & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

template <int G, bool FP8>
__global__ void __launch_bounds__(FP8 ? kThreads8 : kThreadsTc, 1)
    paged_decode_tc_kernel(const __grid_constant__ TcDecodeParams p) {
  constexpr int kStages = FP8 ? kStages8 : kStagesTc;
  constexpr int kOffBars = FP8 ? kOffBar8 : kOffBarTc;
  constexpr int kOffEpX = FP8 ? kOffEp8 : kOffEp;
  constexpr int kOffRedX = FP8 ? kOffRed8 : kOffRed;
  constexpr uint32_t kIdescQK = idesc_n16(false, FP8);
  constexpr uint32_t kIdescPV = idesc_n16(true, FP8);
  // BF16 with 2G <= 16: P_hi and P_lo share one B operand (rows [0, G) and [G, 2G)), so the PV
  // product is one pass of 8 MMAs and O^T columns g and G + g add up in the epilogue.
  constexpr bool kMergedP = !FP8 && 2 * G <= 16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint64_t* full = bars + 0;      // [kStages] TMA landed
  uint64_t* empty = bars + 4;     // [kStages] stage consumed (BF16: after the unit's PV; FP8: converted)
  uint64_t* s_full = bars + 8;    // [2] S^T ready
  uint64_t* p_full = bars + 10;   // [2] P^T written (128 arrivals)
  uint64_t* o_ready = bars + 12;  // [2] O^T of a finished pair ready
  uint64_t* o_free = bars + 14;   // [2] O^T read by the epilogue (128 arrivals)
  uint64_t* pv_done = bars + 16;  // one completion per PV
  uint64_t* ep_full = bars + 17;  // [4] (m, l) of a finished pair handed to the epilogue
  uint64_t* k_ready = bars + 21;  // FP8 [2]: Q e4m3 terms of a pair written (128 arrivals)
  uint64_t* v_ready = bars + 23;  // FP8 [2]: V f16 tile written (128 arrivals)
  uint64_t* k_free = bars + 25;   // FP8 [2]: the products of the pair that read Q buffer [k & 1] completed
  uint64_t* v_free = bars + 27;   // FP8 [2]: the PV that read V buffer [i & 1] completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 29);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 30);
  int* s_start = reinterpret_cast<int*>(bars + 31);  // b, h, t, tiles, L, flag
  int64_t* s_base = reinterpret_cast<int64_t*>(bars + 34);
  int64_t* s_range = reinterpret_cast<int64_t*>(bars + 35);  // start, end, upc
  float* red = reinterpret_cast<float*>(smem + kOffRedX);
  float* ep = reinterpret_cast<float*>(smem + kOffEpX);                    // [4][32]
  volatile int* ep_flag = reinterpret_cast<volatile int*>(smem + kOffEpX + 512);
  float* qf = reinterpret_cast<float*>(smem + kOffEpX + 576);              // FP8: [4] S multiplier per pair
  float* qmax = reinterpret_cast<float*>(smem + kOffEpX + 640);            // FP8: [2][4]
  int* err = reinterpret_cast<int*>(p.ws);
  int* tickets = reinterpret_cast<int*>(p.ws + kTcTicketOff);
  float* parts = reinterpret_cast<float*>(p.ws + tc_part_off(p.batch, p.num_kv_heads));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int grid = gridDim.x;
  constexpr int kThreads = FP8 ? kThreads8 : kThreadsTc;
  constexpr uint32_t kCols = kTmemColsTc;

  // ---------------------------------------------------------------- setup
  if (warp == 0) {
    // Units per sequence (Hk * tiles), scanned over lane-contiguous chunks of the batch.
    const int chunk = (p.batch + 31) / 32;
    const int b0 = lane * chunk, b1 = min(p.batch, b0 + chunk);
    int64_t mine = 0;
    for (int b = b0; b < b1; ++b) mine += int64_t(p.num_kv_heads) * ((seq_len(p, b) + kUT - 1) / kUT);
    int64_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int64_t total = __shfl_sync(0xffffffffu, incl, 31);
    const int64_t upc = total > 0 ? (total + grid - 1) / grid : 1;
    const int64_t start = min(total, int64_t(cta) * upc);
    const int64_t end = min(total, start + upc);
    const int64_t excl = incl - mine;
    if (lane == 0) {
      s_range[0] = start;
      s_range[1] = end;
      s_range[2] = upc;
      s_start[5] = 0;
    }
    __syncwarp();
    if (start < end && excl <= start && start < incl) {
      int64_t cum = excl;
      for (int b = b0; b < b1; ++b) {
        const int L = seq_len(p, b);
        const int tiles = (L + kUT - 1) / kUT;
        const int64_t n = int64_t(p.num_kv_heads) * tiles;
        if (start < cum + n) {
          const int64_t off = start - cum;
          s_start[0] = b;
          s_start[1] = int(off / tiles);
          s_start[2] = int(off % tiles);
          s_start[3] = tiles;
          s_start[4] = L;
          s_base[0] = cum;
          break;
        }
        cum += n;
      }
    }
    // Sequences of length 0 (padding rows) get zeros; CTA c writes rows b = c (mod grid).
    for (int b = cta; b < p.batch; b += grid) {
      if (seq_len(p, b) != 0) continue;
      __nv_bfloat16* o = p.out + int64_t(b) * p.out_row_stride;
      const int n = p.num_kv_heads * G * 128 / 8;
      for (int i = lane; i < n; i += 32) reinterpret_cast<uint4*>(o)[i] = make_uint4(0, 0, 0, 0);
    }
  }
  if (threadIdx.x == 32) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], FP8 ? 129 : 1);  // FP8: 128 converter threads + the QK commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_ready[i], 1);
      mbar_init(&o_free[i], 128);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&ep_full[i], 1);
    mbar_init(pv_done, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_ready[i], 128);
      mbar_init(&v_ready[i], 128);
      mbar_init(&k_free[i], 1);
      mbar_init(&v_free[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Zero the padded rows of every Q and P^T buffer (only rows < G are ever written).
  if constexpr (FP8) {
    for (int i = threadIdx.x; i < (2 * kQ8 + 2 * kP) / 16; i += kThreads)
      *reinterpret_cast<uint4*>(smem + kOffQ8 + i * 16) = make_uint4(0, 0, 0, 0);
  } else {
    for (int i = threadIdx.x; i < (kStagesTc * kQ + 4 * kP) / 16; i += kThreads) {
      const int byte = i * 16;
      uint8_t* dst = byte < kStagesTc * kQ ? smem + (byte / kQ) * kStage + 2 * kKV + byte % kQ
                                           : smem + kOffP + (byte - kStagesTc * kQ);
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
  fence_proxy_async_smem();
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const int64_t start = s_range[0], end = s_range[1], upc = s_range[2];
  const int n_units = int(end - start);
  Cursor c0;
  c0.b = s_start[0];
  c0.h = s_start[1];
  c0.t = s_start[2];
  c0.tiles = s_start[3];
  c0.L = s_start[4];
  c0.base = s_base[0];

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0 && n_units > 0) {
      Cursor c = c0;
      int issued = 0;
      for (int i = 0; i < n_units; ++i, advance(p, c)) {
        const int st = i % kStages;
        if (i >= kStages && !waitb(&empty[st], ((i / kStages) - 1) & 1, abort_flag, err)) break;
        const int tok0 = c.t * kUT;
        const int blk = p.block_tables[int64_t(c.b) * p.bt_stride + tok0 / p.block_size];
        if (blk < 0 || blk >= p.num_blocks) atomicOr(err, 2);
        const int row = blk * p.block_size + tok0 % p.block_size;  // out of range reads zeros
        const uint32_t bar = smem_u32(&full[st]);
        if constexpr (FP8) {
          const uint32_t k = sbase + st * kStage8;
          const uint32_t q = k + 2 * kHalf8;
          mbar_arrive_expect_tx(&full[st], 2 * kHalf8 + 2 * G * 128);
          tma3(k, &p.tk, 0, c.h, row, bar);
          tma3(k + kHalf8, &p.tv, 0, c.h, row, bar);
          tma3(q, &p.tq, 0, c.h * G, c.b, bar);
          tma3(q + kHalfQ, &p.tq, 64, c.h * G, c.b, bar);
        } else {
          const uint32_t k = sbase + st * kStage;
          const uint32_t v = k + kKV;
          const uint32_t q = k + 2 * kKV;
          mbar_arrive_expect_tx(&full[st], 2 * kKV + 2 * G * 128);
          tma3(k, &p.tk, 0, c.h, row, bar);
          tma3(k + kHalfKV, &p.tk, 64, c.h, row, bar);
          tma3(v, &p.tv, 0, c.h, row, bar);
          tma3(v + kHalfKV, &p.tv, 64, c.h, row, bar);
          tma3(q, &p.tq, 0, c.h * G, c.b, bar);
          tma3(q + kHalfQ, &p.tq, 64, c.h * G, c.b, bar);
        }
        issued = i + 1;
      }
      // No copy into this CTA's shared memory may be in flight at exit.
      for (int i = issued >= kStages ? issued - kStages : 0; i < issued; ++i)
        mbar_wait(&full[i % kStages], (i / kStages) & 1);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (n_units > 0) {
      auto qk = [&](int i, int qp) {
        if constexpr (FP8) {
          // 8-bit K-major, 128-byte swizzle: 32 dims (32 bytes) per k-step; the two Q terms are
          // N rows [0, G) and [G, 2G), so S^T columns g and G + g add up to the product.
          const uint32_t k = sbase + (i % kStages) * kStage8;
          const uint32_t q = sbase + kOffQ8 + (qp & 1) * kQ8;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t a = sdesc(k + kk * 32, 16, 1024);
            const uint64_t b = sdesc(q + kk * 32, 16, 1024);
            mma_ss_e4m3(tmem + (i & 1) * 16, a, b, kIdescQK, kk > 0 ? 1u : 0u);
          }
          commit_to(smem_u32(&s_full[i & 1]));
          commit_to(smem_u32(&empty[i % kStages]));  // the staged K bytes are read
        } else {
          const uint32_t k = sbase + (i % kStages) * kStage;
          const uint32_t q = k + 2 * kKV;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t a = sdesc(k + (kk >> 2) * kHalfKV + (kk & 3) * 32, 16, 1024);
            const uint64_t b = sdesc(q + (kk >> 2) * kHalfQ + (kk & 3) * 32, 16, 1024);
            mma_ss(tmem + (i & 1) * 16, a, b, kIdescQK, kk > 0 ? 1u : 0u);
          }
          commit_to(smem_u32(&s_full[i & 1]));
        }
      };
      // The unit's K and Q operands are in place (FP8: Q of pair qp, split once per pair).
      auto k_landed = [&](int i, int qp) {
        return waitb(&full[i % kStages], (i / kStages) & 1, abort_flag, err) &&
               (!FP8 || waitb(&k_ready[qp & 1], (qp >> 1) & 1, abort_flag, err));
      };
      Cursor c = c0;
      bool ok = __all_sync(0xffffffffu, k_landed(0, 0));
      if (ok && lane == 0) {
        fence_after();
        qk(0, 0);
      }
      __syncwarp();
      int pc = 0;  // pairs started
      for (int i = 0; ok && i < n_units; ++i, advance(p, c)) {
        const bool first = (i == 0) || c.t == 0;
        const bool last = (i == n_units - 1) || c.t == c.tiles - 1;
        if (i + 1 < n_units) {
          const int qp = pc + (last ? 1 : 0);  // pair of unit i + 1
          ok = __all_sync(0xffffffffu, k_landed(i + 1, qp));
          if (!ok) break;
          if (lane == 0) {
            fence_after();
            qk(i + 1, qp);
          }
        }
        if (first && pc >= 2) {
          ok = __all_sync(0xffffffffu, waitb(&o_free[pc & 1], ((pc - 2) >> 1) & 1, abort_flag, err));
          if (!ok) break;
        }
        ok = __all_sync(0xffffffffu, waitb(&p_full[i & 1], (i >> 1) & 1, abort_flag, err));
        if (ok && FP8) ok = __all_sync(0xffffffffu, waitb(&v_ready[i & 1], (i >> 1) & 1, abort_flag, err));
        if (!ok) break;
        if (lane == 0) {
          fence_after();
          const uint32_t o = tmem + 32 + (pc & 1) * 16;
          if constexpr (FP8) {
            const uint32_t v = sbase + kOffV16 + (i & 1) * kKV;
            const uint32_t ph = sbase + kOffP16 + (i & 1) * kP;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t a = sdesc(v + kk * 16 * 128, kHalfKV, 1024);
              const uint64_t b = sdesc(ph + (kk >> 2) * kHalfP + (kk & 3) * 32, 16, 1024);
              mma_ss(o, a, b, kIdescPV, (first && kk == 0) ? 0u : 1u);
            }
            commit_to(smem_u32(&v_free[i & 1]));
          } else {
            const uint32_t v = sbase + (i % kStages) * kStage + kKV;
            const uint32_t ph = sbase + kOffP + (i & 1) * kP;
            const uint32_t pl = sbase + kOffPlo + (i & 1) * kP;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t a = sdesc(v + kk * 16 * 128, kHalfKV, 1024);
              const uint64_t b = sdesc(ph + (kk >> 2) * kHalfP + (kk & 3) * 32, 16, 1024);
              mma_ss(o, a, b, kIdescPV, (first && kk == 0) ? 0u : 1u);
            }
            if constexpr (!kMergedP) {
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {
                const uint64_t a = sdesc(v + kk * 16 * 128, kHalfKV, 1024);
                const uint64_t b = sdesc(pl + (kk >> 2) * kHalfP + (kk & 3) * 32, 16, 1024);
                mma_ss(o, a, b, kIdescPV, 1u);
              }
            }
            commit_to(smem_u32(&empty[i % kStages]));
          }
          commit_to(smem_u32(pv_done));
          if (last) commit_to(smem_u32(&o_ready[pc & 1]));
          if (FP8 && last) commit_to(smem_u32(&k_free[pc & 1]));  // every QK of the pair is done
        }
        __syncwarp();
        if (last) ++pc;
      }
      if (lane == 0 && !ok) {
        // Let issued MMAs finish before TMEM is released.
        commit_to(smem_u32(pv_done));
        mbar_wait(pv_done, 0), mbar_wait(pv_done, 1);
      }
      __syncwarp();
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------------- softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // token of S^T / dimension of O^T = TMEM lane
    const int wq = warp - 2;            // index into the 4-warp exchange
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    float m_ref[G], l_run[G];
    Cursor c = c0;
    int pc = 0;
    bool alive = true;
    for (int i = 0; alive && i < n_units; ++i, advance(p, c)) {
      const bool first = (i == 0) || c.t == 0;
      const bool last = (i == n_units - 1) || c.t == c.tiles - 1;
      if (!softmax_all(waitb(&s_full[i & 1], (i >> 1) & 1, abort_flag, err))) {
        alive = false;
        break;
      }
      fence_after();
      uint32_t raw[16];
      ld16(lane_base + (i & 1) * 16, raw);
      const bool valid = c.t * kUT + r < c.L;
      // FP8: the converters' per-pair multiplier (k_scale and the Q shift folded in).  Its slot
      // (pair mod 4) is rewritten only for pair + 4, after the last product of pair + 2, which
      // follows this pair's last P^T.
      const float mult = FP8 ? qf[pc & 3] : p.scale_log2;
      float x[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float sraw = __uint_as_float(raw[g]);
        if constexpr (FP8) sraw += __uint_as_float(raw[G + g]);  // q1 and q2 columns
        x[g] = valid ? sraw * mult : -INFINITY;
      }
      if (!FP8 && !valid) {
        // V rows past the context enter the PV product with P = 0; clear them so that
        // whatever bits the cache holds there (NaN included) contribute nothing.
        uint8_t* vrow = smem + (i % kStages) * kStage + kKV + r * 128;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          *reinterpret_cast<uint4*>(vrow + k * 16) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(vrow + kHalfKV + k * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      if (first) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          m_ref[g] = -INFINITY;
          l_run[g] = 0.f;
        }
      }
      // tile maximum per head over the 128 tokens
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float v = x[g];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red[(0 * 4 + wq) * 16 + g] = v;
      }
      softmax_bar();
      float corr[G];
      bool rescale = false;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float mt = fmaxf(fmaxf(red[g], red[16 + g]), fmaxf(red[32 + g], red[48 + g]));
        corr[g] = 1.f;
        if (mt > m_ref[g] + kRescale) {
          if (m_ref[g] != -INFINITY) {
            corr[g] = fast_ex2(m_ref[g] - mt);
            rescale = true;
          }
          m_ref[g] = mt;
        }
      }
      rescale = rescale && !first;
      float pr[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        pr[g] = fast_ex2(x[g] - (m_ref[g] == -INFINITY ? 0.f : m_ref[g]));
        float v = pr[g];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[(1 * 4 + wq) * 16 + g] = v;
      }
      // P^T (row g, token r) in the swizzled K-major layout: BF16 as hi + lo (~16 significant
      // bits), FP8 as one f16 (11 bits; the f16 products of the e4m3 path)
      {
        const int half = r >> 6, cc = r & 63;
        if constexpr (FP8) {
          uint8_t* ph = smem + kOffP16 + (i & 1) * kP + half * kHalfP;
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const int off = g * 128 + (((cc >> 3) ^ (g & 7)) << 4) + (cc & 7) * 2;
            *reinterpret_cast<__half*>(ph + off) = __float2half_rn(pr[g]);
          }
        } else {
          uint8_t* ph = smem + kOffP + (i & 1) * kP + half * kHalfP;
          uint8_t* pl = smem + kOffPlo + (i & 1) * kP + half * kHalfP;
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const int off = g * 128 + (((cc >> 3) ^ (g & 7)) << 4) + (cc & 7) * 2;
            const __nv_bfloat16 hi = __float2bfloat16_rn(pr[g]);
            const __nv_bfloat16 lo = __float2bfloat16_rn(pr[g] - __bfloat162float(hi));
            *reinterpret_cast<__nv_bfloat16*>(ph + off) = hi;
            if constexpr (kMergedP) {
              const int gl = G + g;  // P_lo as row G + g of the same operand
              *reinterpret_cast<__nv_bfloat16*>(ph + gl * 128 + (((cc >> 3) ^ (gl & 7)) << 4) + (cc & 7) * 2) = lo;
            } else {
              *reinterpret_cast<__nv_bfloat16*>(pl + off) = lo;
            }
          }
        }
      }
      softmax_bar();
#pragma unroll
      for (int g = 0; g < G; ++g)
        l_run[g] = l_run[g] * corr[g] + ((red[64 + g] + red[80 + g]) + (red[96 + g] + red[112 + g]));
      if (rescale) {
        // O^T holds PV of the earlier tiles of this pair: wait for the last one, then scale.
        if (!softmax_all(waitb(pv_done, (i - 1) & 1, abort_flag, err))) {
          alive = false;
          break;
        }
        fence_after();
        uint32_t o[16];
        ld16(lane_base + 32 + (pc & 1) * 16, o);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          o[g] = __float_as_uint(__uint_as_float(o[g]) * corr[g]);
          if constexpr (kMergedP) o[G + g] = __float_as_uint(__uint_as_float(o[G + g]) * corr[g]);
        }
        st16(lane_base + 32 + (pc & 1) * 16, o);
      }
      fence_proxy_async_smem();
      fence_before();
      mbar_arrive(&p_full[i & 1]);

      if (last) {
        if (r == 0) {
#pragma unroll
          for (int g = 0; g < G; ++g) {
            ep[(pc & 3) * 32 + g] = m_ref[g];
            ep[(pc & 3) * 32 + 16 + g] = l_run[g];
          }
          mbar_arrive(&ep_full[pc & 3]);
        }
        ++pc;
      }
    }
  } else if (warp < 10) {
    // ---------------------------------------------------------------- pair epilogues
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // dimension of O^T = TMEM lane
    const uint32_t lane_base = tmem + (uint32_t(quarter * 32) << 16);
    Cursor c = c0;
    int pc = 0;
    for (int i = 0; i < n_units; ++i, advance(p, c)) {
      const bool last = (i == n_units - 1) || c.t == c.tiles - 1;
      if (!last) continue;
      if (!epilogue_all(waitb(&ep_full[pc & 3], (pc >> 2) & 1, abort_flag, err) &&
                        waitb(&o_ready[pc & 1], (pc >> 1) & 1, abort_flag, err)))
        break;
      fence_after();
      float m_ref[G], l_run[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        m_ref[g] = ep[(pc & 3) * 32 + g];
        l_run[g] = ep[(pc & 3) * 32 + 16 + g];
      }
      uint32_t o[16];
      ld16(lane_base + 32 + (pc & 1) * 16, o);
      fence_before();
      mbar_arrive(&o_free[pc & 1]);
      if constexpr (kMergedP) {  // O = V^T P_hi + V^T P_lo
#pragma unroll
        for (int g = 0; g < G; ++g) o[g] = __float_as_uint(__uint_as_float(o[g]) + __uint_as_float(o[G + g]));
      }
      // FP8: V was converted x 2^-8.
      const float vs = FP8 ? (p.v_scale ? p.v_scale[c.h] : 1.f) * 256.f : 1.f;
      const int64_t pf = c.pair_first(), pl_ = c.pair_last();
      __nv_bfloat16* orow = p.out + int64_t(c.b) * p.out_row_stride + int64_t(c.h) * G * 128;
      if (pf >= start && pl_ < end) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float inv = l_run[g] > 0.f ? vs / l_run[g] : 0.f;
          orow[g * 128 + r] = __float2bfloat16_rn(__uint_as_float(o[g]) * inv);
        }
      } else {
        // Partial pair: publish (m, l, O) in this CTA's slot, the last CTA of the pair merges.
        const int slot = pf < start ? 0 : 1;  // 0: the pair began before this range
        float* part = parts + (int64_t(cta) * 2 + slot) * (130 * G);
#pragma unroll
        for (int g = 0; g < G; ++g) part[2 * G + g * 128 + r] = __uint_as_float(o[g]);
        if (r == 0) {
#pragma unroll
          for (int g = 0; g < G; ++g) {
            part[g] = m_ref[g];
            part[G + g] = l_run[g];
          }
        }
        __threadfence();
        epilogue_bar();
        const int pair = c.b * p.num_kv_heads + c.h;
        const int c_first = int(pf / upc), c_last = int(pl_ / upc);
        if (r == 0) *ep_flag = atomicAdd(&tickets[pair], 1) == c_last - c_first;
        epilogue_bar();
        const bool merger = *ep_flag != 0;
        epilogue_bar();  // ep_flag is reused by the next pair
        if (merger) {
          __threadfence();
          float mx[G], ls[G], acc[G];
#pragma unroll
          for (int g = 0; g < G; ++g) {
            mx[g] = -INFINITY;
            ls[g] = 0.f;
            acc[g] = 0.f;
          }
          for (int cc = c_first; cc <= c_last; ++cc) {
            const int sl = pf < int64_t(cc) * upc ? 0 : 1;
            const float* q = parts + (int64_t(cc) * 2 + sl) * (130 * G);
#pragma unroll
            for (int g = 0; g < G; ++g) mx[g] = fmaxf(mx[g], __ldcg(q + g));
          }
          for (int cc = c_first; cc <= c_last; ++cc) {
            const int sl = pf < int64_t(cc) * upc ? 0 : 1;
            const float* q = parts + (int64_t(cc) * 2 + sl) * (130 * G);
#pragma unroll
            for (int g = 0; g < G; ++g) {
              const float m = __ldcg(q + g);
              if (m == -INFINITY) continue;
              const float f = fast_ex2(m - mx[g]);
              ls[g] += __ldcg(q + G + g) * f;
              acc[g] += __ldcg(q + 2 * G + g * 128 + r) * f;
            }
          }
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float inv = ls[g] > 0.f ? vs / ls[g] : 0.f;
            orow[g * 128 + r] = __float2bfloat16_rn(acc[g] * inv);
          }
          if (r == 0) tickets[pair] = 0;  // ready for the next launch
        }
      }
      ++pc;
    }
  } else if constexpr (FP8) {
    // ---------------------------------------------------------------- Q split, V e4m3 -> f16
    // Thread = token row r of a unit for V; Q elements [G r, G r + G) of the pair's G x 128 bf16
    // rows at the pair's first unit.  Q is shifted by an exact power of two so that its largest
    // |q| lies in [2^7, 2^8), then split into two e4m3 terms (q1 = q truncated to 4 significant
    // bits, q2 = q - q1); 2^-shift and k_scale go into the softmax multiplier.
    const int r = (warp - 10) * 32 + lane;
    const int wq = warp - 10;
    const int g = (r * G) >> 7, d0 = (r * G) & 127;
    Cursor c = c0;
    int pc = 0;  // pairs started
    for (int i = 0; i < n_units; ++i, advance(p, c)) {
      const int st = i % kStages;
      const int bf = i & 1;
      const bool first = (i == 0) || c.t == 0;
      const bool last = (i == n_units - 1) || c.t == c.tiles - 1;
      if (!convert_all(waitb(&full[st], (i / kStages) & 1, abort_flag, err))) break;
      const uint8_t* stage = smem + st * kStage8;
      uint4 vw[8];
      load_row8(stage + kHalf8, r, vw);
      if (first) {
        float qv[G];
        {
          const int qoff = (d0 >> 6) * kHalfQ + g * 128 + (((((d0 & 63) >> 3) ^ (g & 7))) << 4) + (d0 & 7) * 2;
          const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(stage + 2 * kHalf8 + qoff);
#pragma unroll
          for (int k = 0; k < G; ++k) qv[k] = __bfloat162float(src[k]);
        }
        float amax = 0.f;
#pragma unroll
        for (int k = 0; k < G; ++k) amax = fmaxf(amax, fabsf(qv[k]));
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (lane == 0) qmax[(pc & 1) * 4 + wq] = amax;
        // Q buffer (pc & 1) is free once every product of pair pc - 2 has completed (the
        // barrier also publishes qmax to all four warps).
        if (!convert_all(pc < 2 || waitb(&k_free[pc & 1], ((pc - 2) >> 1) & 1, abort_flag, err))) break;
        fence_after();
        const float* qm = qmax + (pc & 1) * 4;
        amax = fmaxf(fmaxf(qm[0], qm[1]), fmaxf(qm[2], qm[3]));
        const int e = int((__float_as_uint(amax) >> 23) & 0xffu) - 127;
        int shift = amax > 0.f ? 7 - e : 0;  // largest |q| * 2^shift in [2^7, 2^8)
        shift = shift > 126 ? 126 : shift;   // -120 <= 7 - e for every finite float
        const float up = __uint_as_float(uint32_t(shift + 127) << 23);
        const float down = __uint_as_float(uint32_t(127 - shift) << 23);
        // row g, dims [d0, d0 + G) of both terms (G <= 8 bytes inside one 16-byte chunk)
        uint8_t* qb = smem + kOffQ8 + (pc & 1) * kQ8;
        uint8_t* t1 = qb + g * 128 + ((((d0 >> 4) ^ (g & 7))) << 4) + (d0 & 15);
        uint8_t* t2 = qb + (G + g) * 128 + ((((d0 >> 4) ^ ((G + g) & 7))) << 4) + (d0 & 15);
#pragma unroll
        for (int k = 0; k < G; ++k) {
          const float x = qv[k] * up;
          const float h = e4m3_head(x);
          t1[k] = uint8_t(e4m3_byte(h));
          t2[k] = uint8_t(e4m3_byte(x - h));
        }
        if (r == 0) {
          const float ks = p.k_scale ? p.k_scale[c.h] : 1.f;
          qf[pc & 3] = p.scale_log2 * ks * down;
        }
        fence_proxy_async_smem();
        mbar_arrive(&k_ready[pc & 1]);
      }
      if (!convert_all(i < 2 || waitb(&v_free[bf], ((i - 2) >> 1) & 1, abort_flag, err))) break;
      mbar_arrive(&empty[st]);  // this thread's staged bytes are in registers
      // V rows past the context are written as zeros (P is 0 there; the cache may hold NaN bits).
      store_row_f16(vw, smem + kOffV16 + bf * kKV, r, c.t * kUT + r >= c.L);
      fence_proxy_async_smem();
      mbar_arrive(&v_ready[bf]);
      if (last) ++pc;
    }
  }

  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
  }
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_tiled() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  }
  return fn;
}

// [outer, heads, 128] bf16 -> boxes of (64 dims x box_heads x box_outer), 128-byte swizzle.
bool encode3(CUtensorMap* map, const void* base, uint64_t heads, uint64_t outer, uint64_t head_stride_bytes,
             uint64_t outer_stride_bytes, uint32_t box_heads, uint32_t box_outer) {
  EncodeFn fn = encode_tiled();
  if (!fn) return false;
  const cuuint64_t dims[3] = {128, heads, outer};
  const cuuint64_t strides[2] = {head_stride_bytes, outer_stride_bytes};
  const cuuint32_t box[3] = {64, box_heads, box_outer};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [rows, heads, 128] e4m3 bytes -> boxes of (128 bytes x 1 head x 128 rows), 128-byte swizzle.
bool encode_e4m3(CUtensorMap* map, const void* base, uint64_t heads, uint64_t rows, uint64_t row_stride_bytes) {
  EncodeFn fn = encode_tiled();
  if (!fn) return false;
  const cuuint64_t dims[3] = {128, heads, rows};
  const cuuint64_t strides[2] = {128, row_stride_bytes};
  const cuuint32_t box[3] = {128, 1, uint32_t(kUT)};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int G, bool FP8>
int launch_g(const TcDecodeParams& prm, cudaStream_t stream) {
  // Per device: the shared-memory opt-in is a per-device attribute.  The first call on a device
  // happens before any graph capture (the engine's eager warm-up).
  static std::atomic<int> grid_of[kMaxDevicesTc];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevicesTc) {
    set_error("hl_paged_decode: no usable current device");
    return HL_ERR_CUDA;
  }
  constexpr int kSmem = FP8 ? kSmem8 : kSmemTc;
  int grid = grid_of[dev].load(std::memory_order_acquire);
  if (grid == 0) {
    int sms = 0;
    e = cudaFuncSetAttribute(paged_decode_tc_kernel<G, FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
      set_error("hl_paged_decode: tensor-core kernel setup: %s", cudaGetErrorString(e));
      return HL_ERR_CUDA;
    }
    grid = sms < kMaxGridTc ? sms : kMaxGridTc;
    grid_of[dev].store(grid, std::memory_order_release);
  }
  paged_decode_tc_kernel<G, FP8><<<grid, FP8 ? kThreads8 : kThreadsTc, kSmem, stream>>>(prm);
  HL_CHECK_LAUNCH("hl_paged_decode");
  return HL_OK;
}

}  // namespace

int64_t tc_ticket_end(int batch, int num_q_heads) { return tc_part_off(batch, num_q_heads); }

int64_t decode_tc_workspace_bytes(int batch, int num_q_heads) {
  // tickets for up to batch * Hq pairs, two partial slots of (m, l, O) per CTA for G <= Hq.
  return tc_part_off(batch, num_q_heads) + int64_t(kMaxGridTc) * 2 * 130 * num_q_heads * 4;
}

bool decode_tc_supported(int batch, int num_q_heads, int num_kv_heads, int block_size, bool fp8) {
  const int g = num_q_heads / num_kv_heads;
  const bool g_ok = fp8 ? (g == 1 || g == 2 || g == 4 || g == 8) : (g == 1 || g == 2 || g == 4 || g == 8 || g == 16);
  return batch <= kMaxBatchTc && block_size % kUT == 0 && g_ok;
}

int decode_tc_launch(const void* q, int64_t q_row_stride, const void* k_cache, const void* v_cache, bool fp8,
                     const float* k_scale, const float* v_scale, const int32_t* block_tables, int64_t bt_stride,
                     int max_blocks, const int32_t* context_lens, int batch, int num_q_heads, int num_kv_heads,
                     int block_size, int64_t num_blocks, float scale_log2, void* out, int64_t out_row_stride, void* ws,
                     cudaStream_t stream) {
  const int g = num_q_heads / num_kv_heads;
  TcDecodeParams prm;
  memset(&prm, 0, sizeof(prm));
  const uint64_t rows = uint64_t(num_blocks) * block_size;
  bool ok = encode3(&prm.tq, q, num_q_heads, batch, 256, uint64_t(q_row_stride) * 2, g, 1);
  if (fp8) {
    const uint64_t rs = uint64_t(num_kv_heads) * 128;
    ok = ok && encode_e4m3(&prm.tk, k_cache, num_kv_heads, rows, rs) &&
         encode_e4m3(&prm.tv, v_cache, num_kv_heads, rows, rs);
  } else {
    const uint64_t rs = uint64_t(num_kv_heads) * 128 * 2;
    ok = ok && encode3(&prm.tk, k_cache, num_kv_heads, rows, 256, rs, 1, kUT) &&
         encode3(&prm.tv, v_cache, num_kv_heads, rows, 256, rs, 1, kUT);
  }
  if (!ok) {
    set_error("hl_paged_decode: cuTensorMapEncodeTiled failed");
    return HL_ERR_CUDA;
  }
  prm.k_scale = fp8 ? k_scale : nullptr;
  prm.v_scale = fp8 ? v_scale : nullptr;
  prm.block_tables = block_tables;
  prm.bt_stride = bt_stride;
  prm.context_lens = context_lens;
  prm.batch = batch;
  prm.max_blocks = max_blocks;
  prm.block_size = block_size;
  prm.num_kv_heads = num_kv_heads;
  prm.num_blocks = num_blocks;
  prm.scale_log2 = scale_log2;
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.out_row_stride = out_row_stride;
  prm.ws = static_cast<uint8_t*>(ws);
  if (fp8) {
    switch (g) {
      case 1: return launch_g<1, true>(prm, stream);
      case 2: return launch_g<2, true>(prm, stream);
      case 4: return launch_g<4, true>(prm, stream);
      case 8: return launch_g<8, true>(prm, stream);
    }
  } else {
    switch (g) {
      case 1: return launch_g<1, false>(prm, stream);
      case 2: return launch_g<2, false>(prm, stream);
      case 4: return launch_g<4, false>(prm, stream);
      case 8: return launch_g<8, false>(prm, stream);
      case 16: return launch_g<16, false>(prm, stream);
    }
  }
  set_error("hl_paged_decode: Hq/Hk=%d not supported by the tensor-core kernel", g);
  return HL_ERR_UNSUPPORTED;
}

}  // namespace hl
