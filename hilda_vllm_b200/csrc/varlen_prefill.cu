// Varlen causal prefill attention on CUDA cores (hl_varlen_prefill_simt; the engine uses the
// tensor-core kernel in prefill_tc.cu).
//
// Semantics (mini_vllm/layers/attention.py:120-131,149-160: flash_attn_varlen_func with
// causal=True and, when a prefix is cached or the prompt is chunked, block_table set so K/V
// come from the paged cache): for sequence s with Lq = cu_q[s+1]-cu_q[s] query rows and
// Lk = cu_k[s+1]-cu_k[s] keys, query row i attends keys j <= i + (Lk - Lq) (causal mask
// aligned to the bottom-right corner) with j < Lk.  A row with no admissible key is zero.
//
// This kernel is the small-prompt path: one CTA = 64 query rows x one query head of one
// sequence; 4 threads per row each own 32 of the 128 dimensions; K/V tiles of 64 keys are
// staged in shared memory (key rows are read by every query row as a broadcast).  The grid
// is (ceil(max_seqlen_q/64), Hq, num_seqs) so it never depends on device values.
#include "hl_common.cuh"

namespace hl {
namespace {

constexpr int kD = 128;
constexpr int kRows = 64;     // query rows per CTA
constexpr int kKeys = 64;     // keys per shared-memory tile
constexpr int kTPR = 4;       // threads per query row
constexpr int kDPT = kD / kTPR;  // 32 dims per thread
constexpr int kThreads = kRows * kTPR;  // 256
constexpr int kChunk = 16;    // keys scored per softmax update
constexpr float kLog2e = 1.4426950408889634f;

struct PrefillParams {
  const __nv_bfloat16* q;
  int64_t q_row_stride;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t k_row_stride;  // contiguous mode: elements between key rows; paged: Hk*D
  int64_t v_row_stride;
  const int32_t* cu_q;
  const int32_t* cu_k;
  const int32_t* block_tables;  // null: contiguous K/V
  int64_t bt_stride;
  int num_q_heads;
  int num_kv_heads;
  int block_size;
  int64_t num_blocks;
  float scale_log2;
  __nv_bfloat16* out;
  int64_t out_row_stride;
};

__global__ void __launch_bounds__(kThreads) varlen_prefill_simt_kernel(const PrefillParams p) {
  __shared__ __align__(16) __nv_bfloat16 Ks[kKeys][kD];
  __shared__ __align__(16) __nv_bfloat16 Vs[kKeys][kD];

  const int tile = blockIdx.x;
  const int hq = blockIdx.y;
  const int s = blockIdx.z;
  const int G = p.num_q_heads / p.num_kv_heads;
  const int hk = hq / G;
  const int q_begin = p.cu_q[s];
  const int Lq = p.cu_q[s + 1] - q_begin;
  const int k_begin = p.cu_k[s];
  const int Lk = p.cu_k[s + 1] - k_begin;
  const int r0 = tile * kRows;
  if (r0 >= Lq) return;
  const int shift = Lk - Lq;  // bottom-right causal alignment

  const int tid = threadIdx.x;
  const int row = tid / kTPR;  // query row within the tile
  const int part = tid % kTPR; // which 32-dim slice
  const int i = r0 + row;      // query row within the sequence
  const bool row_ok = i < Lq;

  float qv[kDPT];
  {
    const int ii = row_ok ? i : 0;
    const __nv_bfloat16* qp = p.q + int64_t(q_begin + ii) * p.q_row_stride + hq * kD + part * kDPT;
#pragma unroll
    for (int c = 0; c < kDPT / 8; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(qp + 8 * c);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        qv[8 * c + 2 * t] = bf16lo(w[t]) * p.scale_log2;
        qv[8 * c + 2 * t + 1] = bf16hi(w[t]) * p.scale_log2;
      }
    }
  }
  float o[kDPT];
#pragma unroll
  for (int d = 0; d < kDPT; ++d) o[d] = 0.f;
  float m = -INFINITY, l = 0.f;

  // Keys needed by this tile: j <= (last row) + shift.
  const int last_row = min(Lq, r0 + kRows) - 1;
  int k_end = min(Lk, last_row + shift + 1);
  if (k_end < 0) k_end = 0;
  const int row_limit = i + shift;  // admissible keys: j <= row_limit

  for (int k0 = 0; k0 < k_end; k0 += kKeys) {
    __syncthreads();
    // Cooperative tile load: 64 keys x 128 dims x 2 (K, V), 16-byte vectors.
    for (int e = tid; e < kKeys * (kD / 8); e += kThreads) {
      const int kr = e / (kD / 8);
      const int c = e % (kD / 8);
      const int j = k0 + kr;
      uint4 kvec = make_uint4(0, 0, 0, 0), vvec = make_uint4(0, 0, 0, 0);
      if (j < k_end) {
        int64_t krow, vrow;
        bool ok = true;
        if (p.block_tables) {
          const int64_t blk = p.block_tables[int64_t(s) * p.bt_stride + j / p.block_size];
          ok = blk >= 0 && blk < p.num_blocks;
          const int64_t slot = blk * p.block_size + j % p.block_size;
          krow = slot * p.k_row_stride;
          vrow = slot * p.v_row_stride;
        } else {
          krow = int64_t(k_begin + j) * p.k_row_stride;
          vrow = int64_t(k_begin + j) * p.v_row_stride;
        }
        if (ok) {
          kvec = *reinterpret_cast<const uint4*>(p.k + krow + hk * kD + 8 * c);
          vvec = *reinterpret_cast<const uint4*>(p.v + vrow + hk * kD + 8 * c);
        }
      }
      *reinterpret_cast<uint4*>(&Ks[kr][8 * c]) = kvec;
      *reinterpret_cast<uint4*>(&Vs[kr][8 * c]) = vvec;
    }
    __syncthreads();

    for (int c0 = 0; c0 < kKeys && k0 + c0 < k_end; c0 += kChunk) {
      float sc[kChunk];
#pragma unroll
      for (int t = 0; t < kChunk; ++t) {
        const __nv_bfloat16* kr = &Ks[c0 + t][part * kDPT];
        float acc = 0.f;
#pragma unroll
        for (int c = 0; c < kDPT / 8; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(kr + 8 * c);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            acc = fmaf(qv[8 * c + 2 * u], bf16lo(w[u]), acc);
            acc = fmaf(qv[8 * c + 2 * u + 1], bf16hi(w[u]), acc);
          }
        }
        sc[t] = acc;
      }
#pragma unroll
      for (int t = 0; t < kChunk; ++t) {
        sc[t] += __shfl_xor_sync(0xffffffffu, sc[t], 1);
        sc[t] += __shfl_xor_sync(0xffffffffu, sc[t], 2);
      }
      float mt = -INFINITY;
#pragma unroll
      for (int t = 0; t < kChunk; ++t) {
        const int j = k0 + c0 + t;
        const bool ok = row_ok && j < k_end && j <= row_limit;
        if (!ok) sc[t] = -INFINITY;
        mt = fmaxf(mt, sc[t]);
      }
      const float mn = fmaxf(m, mt);
      if (mn == -INFINITY) continue;
      const float corr = exp2f(m - mn);
      l *= corr;
#pragma unroll
      for (int d = 0; d < kDPT; ++d) o[d] *= corr;
#pragma unroll
      for (int t = 0; t < kChunk; ++t) {
        if (sc[t] == -INFINITY) continue;
        const float pr = exp2f(sc[t] - mn);
        l += pr;
        const __nv_bfloat16* vr = &Vs[c0 + t][part * kDPT];
#pragma unroll
        for (int c = 0; c < kDPT / 8; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(vr + 8 * c);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            o[8 * c + 2 * u] = fmaf(pr, bf16lo(w[u]), o[8 * c + 2 * u]);
            o[8 * c + 2 * u + 1] = fmaf(pr, bf16hi(w[u]), o[8 * c + 2 * u + 1]);
          }
        }
      }
      m = mn;
    }
  }

  if (!row_ok) return;
  const float inv = l > 0.f ? 1.f / l : 0.f;
  __nv_bfloat16* op = p.out + int64_t(q_begin + i) * p.out_row_stride + hq * kD + part * kDPT;
#pragma unroll
  for (int c = 0; c < kDPT / 8; ++c) {
    uint32_t w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      __nv_bfloat162 h2 = __floats2bfloat162_rn(o[8 * c + 2 * u] * inv, o[8 * c + 2 * u + 1] * inv);
      w[u] = *reinterpret_cast<uint32_t*>(&h2);
    }
    *reinterpret_cast<uint4*>(op + 8 * c) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace
}  // namespace hl

using namespace hl;

extern "C" int hl_varlen_prefill_simt(const void* q, int64_t q_row_stride, const void* k, const void* v,
                                 int64_t k_row_stride, int64_t v_row_stride, const int32_t* cu_seqlens_q,
                                 const int32_t* cu_seqlens_k, const int32_t* block_tables, int64_t bt_stride,
                                 int num_seqs, int max_seqlen_q, int max_seqlen_k, int num_q_heads,
                                 int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                                 float softmax_scale, void* out, int64_t out_row_stride, void* stream) {
  clear_error();
  (void)max_seqlen_k;
  HL_CHECK_ARG(num_seqs >= 0 && max_seqlen_q >= 0, "hl_varlen_prefill_simt: negative size");
  if (num_seqs == 0 || max_seqlen_q == 0) return HL_OK;
  HL_CHECK_ARG(q && k && v && cu_seqlens_q && cu_seqlens_k && out, "hl_varlen_prefill_simt: null pointer");
  HL_CHECK_ARG(head_dim == kD, "hl_varlen_prefill_simt: head_dim %d != 128", head_dim);
  HL_CHECK_ARG(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0, "hl_varlen_prefill_simt: Hq %% Hk != 0");
  HL_CHECK_ARG(num_seqs <= 65535 && num_q_heads <= 65535, "hl_varlen_prefill_simt: grid too large");
  HL_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out) && q_row_stride % 8 == 0 &&
                   out_row_stride % 8 == 0,
               "hl_varlen_prefill_simt: q/k/v/out must be 16-byte aligned with row strides %% 8 == 0");
  PrefillParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_row_stride = q_row_stride;
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  if (block_tables) {
    HL_CHECK_ARG(block_size > 0 && bt_stride > 0, "hl_varlen_prefill_simt: bad block table");
    p.k_row_stride = int64_t(num_kv_heads) * head_dim;
    p.v_row_stride = int64_t(num_kv_heads) * head_dim;
  } else {
    HL_CHECK_ARG(k_row_stride % 8 == 0 && v_row_stride % 8 == 0, "hl_varlen_prefill_simt: k/v row stride %% 8 != 0");
    p.k_row_stride = k_row_stride;
    p.v_row_stride = v_row_stride;
  }
  p.cu_q = cu_seqlens_q;
  p.cu_k = cu_seqlens_k;
  p.block_tables = block_tables;
  p.bt_stride = bt_stride;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.scale_log2 = softmax_scale * kLog2e;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_row_stride = out_row_stride;
  dim3 grid((max_seqlen_q + kRows - 1) / kRows, num_q_heads, num_seqs);
  varlen_prefill_simt_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  HL_CHECK_LAUNCH("hl_varlen_prefill_simt");
  return HL_OK;
}
