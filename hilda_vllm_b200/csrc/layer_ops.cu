// Elementwise / row-reduction kernels around attention, written to reproduce the
// reference's eager PyTorch arithmetic step by step (each intermediate rounded where the
// reference rounds it), so the decode step needs no Inductor/Triton kernels:
//   RMSNorm            mini_vllm/layers/layernorm.py:18-28   (rms_forward)
//   add + RMSNorm      mini_vllm/layers/layernorm.py:30-42   (add_rms_forward)
//   QK-RMSNorm + RoPE  mini_vllm/models/qwen3.py:82-85, layers/rotary_embedding.py:8-16,39-50
//   SiLU * mul         mini_vllm/layers/activation.py:12-16
//   greedy argmax      logits.argmax(-1) (first index among equal maxima)
#include "hl_common.cuh"

namespace hl {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w), computed per row by one warp.
// If `res` is given: x = in + res (fp32), res := bf16(x) first (the add_rms_forward order).
// NV = hidden / 256 vectors of 8 elements per lane, so the row stays in registers.
template <bool ADD, int NV>
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ res,
                               const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int rows,
                               int hidden, int64_t in_stride, int64_t out_stride, float eps) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const __nv_bfloat16* x = in + int64_t(warp) * in_stride;
  __nv_bfloat16* r = ADD ? res + int64_t(warp) * hidden : nullptr;
  __nv_bfloat16* y = out + int64_t(warp) * out_stride;
  float buf[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NV; ++c) {
    const int vi = lane + 32 * c;
    const uint4 a = *reinterpret_cast<const uint4*>(x + 8 * vi);
    const uint32_t wa[4] = {a.x, a.y, a.z, a.w};
    float v[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      v[2 * t] = bf16lo(wa[t]);
      v[2 * t + 1] = bf16hi(wa[t]);
    }
    if (ADD) {
      const uint4 b = *reinterpret_cast<const uint4*>(r + 8 * vi);
      const uint32_t wb[4] = {b.x, b.y, b.z, b.w};
      uint32_t ro[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        v[2 * t] = __fadd_rn(v[2 * t], bf16lo(wb[t]));
        v[2 * t + 1] = __fadd_rn(v[2 * t + 1], bf16hi(wb[t]));
        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * t], v[2 * t + 1]);
        ro[t] = *reinterpret_cast<uint32_t*>(&h2);
      }
      *reinterpret_cast<uint4*>(r + 8 * vi) = make_uint4(ro[0], ro[1], ro[2], ro[3]);
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      buf[c][t] = v[t];
      ss = fmaf(v[t], v[t], ss);
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / float(hidden) + eps);
#pragma unroll
  for (int c = 0; c < NV; ++c) {
    const int vi = lane + 32 * c;
    const uint4 wv = *reinterpret_cast<const uint4*>(w + 8 * vi);
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float a = __fmul_rn(bf16_round(__fmul_rn(buf[c][2 * t], inv)), bf16lo(ww[t]));
      const float b = __fmul_rn(bf16_round(__fmul_rn(buf[c][2 * t + 1], inv)), bf16hi(ww[t]));
      __nv_bfloat162 h2 = __floats2bfloat162_rn(a, b);
      o[t] = *reinterpret_cast<uint32_t*>(&h2);
    }
    *reinterpret_cast<uint4*>(y + 8 * vi) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// In-place QK-RMSNorm (over head_dim = 128) + NeoX RoPE on the q and k parts of the fused
// qkv rows: qkv[t] = [q (Hq*128) | k (Hk*128) | v (Hk*128)].  One half-warp per (token,
// head); lane ln owns dims [8ln, 8ln+8) and its RoPE partner dims live in lane ln ^ 8.
// cos_sin[pos] = [cos(pos*f_0..63) | sin(pos*f_0..63)] fp32 (the reference's cos_sin_cache).
//
// KV != kNoStore also fuses the KV-cache store (store_kvcache, mini_vllm/layers/attention.py:
// 59-90, and its FP8 twin): the (token, head) space then covers the v heads too, and for a
// token whose slot is in range the post-RoPE k head and the v head are written to row `slot`
// of the paged cache, as bf16 bytes (kStoreBf16) or as e4m3 of x / scale[h] (kStoreFp8) —
// the same bytes the separate store kernels write from the rotated qkv rows.
// kStoreFp8Mirror writes the e4m3 rows and, in the same pass, the bf16 rows into a second pair
// of caches (the FP8 mode's BF16 prefill cache), so that cache holds every token's K/V too.
constexpr int kNoStore = 0;
constexpr int kStoreBf16 = 1;
constexpr int kStoreFp8 = 2;
constexpr int kStoreFp8Mirror = 3;

template <int KV>
__global__ void qk_norm_rope_kernel(__nv_bfloat16* __restrict__ qkv, int64_t row_stride, int num_tokens,
                                    int num_q_heads, int num_kv_heads, const __nv_bfloat16* __restrict__ qw,
                                    const __nv_bfloat16* __restrict__ kw, const float* __restrict__ cos_sin,
                                    const int64_t* __restrict__ positions, float eps, void* __restrict__ k_cache,
                                    void* __restrict__ v_cache, const int32_t* __restrict__ slot_mapping,
                                    int64_t num_slots, const float* __restrict__ k_scale,
                                    const float* __restrict__ v_scale, __nv_bfloat16* __restrict__ k_mirror,
                                    __nv_bfloat16* __restrict__ v_mirror) {
  // Let the next kernel (the decode attention, launched as a programmatic dependent) start its
  // prologue now; it waits for this grid's writes before it reads q or the newest K/V slot.
  asm volatile("griddepcontrol.launch_dependents;");
  const int heads = num_q_heads + (KV == kNoStore ? 1 : 2) * num_kv_heads;
  const int64_t gid = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 4;  // (token, head) index
  const int ln = threadIdx.x & 15;
  const bool active = gid < int64_t(num_tokens) * heads;
  const int64_t tok = active ? gid / heads : 0;
  const int hh = active ? int(gid % heads) : 0;
  const bool is_q = hh < num_q_heads;
  __nv_bfloat16* x = qkv + tok * row_stride + int64_t(hh) * 128 + 8 * ln;
  const int row_elems = num_kv_heads * 128;
  if constexpr (KV != kNoStore) {
    // v heads: a copy into the cache; the half-warp is uniform in hh, so it leaves together.
    if (hh >= num_q_heads + num_kv_heads) {
      if (!active) return;
      const int64_t slot = slot_mapping[tok];
      if (slot < 0 || slot >= num_slots) return;
      const int hv = hh - num_q_heads - num_kv_heads;
      const uint4 a = *reinterpret_cast<const uint4*>(x);
      const int64_t off = slot * row_elems + hv * 128 + 8 * ln;
      if constexpr (KV == kStoreBf16) {
        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(v_cache) + off) = a;
      } else {
        *reinterpret_cast<uint2*>(static_cast<uint8_t*>(v_cache) + off) = quant8_e4m3(a, v_scale ? v_scale[hv] : 1.f);
        if constexpr (KV == kStoreFp8Mirror) *reinterpret_cast<uint4*>(v_mirror + off) = a;
      }
      return;
    }
  }
  float v[8];
  {
    const uint4 a = active ? *reinterpret_cast<const uint4*>(x) : make_uint4(0, 0, 0, 0);
    const uint32_t wa[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      v[2 * t] = bf16lo(wa[t]);
      v[2 * t + 1] = bf16hi(wa[t]);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int t = 0; t < 8; ++t) ss = fmaf(v[t], v[t], ss);
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / 128.f + eps);
  const __nv_bfloat16* w = is_q ? qw : kw;
  float nv[8];
  {
    const uint4 wv = *reinterpret_cast<const uint4*>(w + 8 * ln);
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      nv[2 * t] = bf16_round(__fmul_rn(bf16_round(__fmul_rn(v[2 * t], inv)), bf16lo(ww[t])));
      nv[2 * t + 1] = bf16_round(__fmul_rn(bf16_round(__fmul_rn(v[2 * t + 1], inv)), bf16hi(ww[t])));
    }
  }
  float pv[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) pv[t] = __shfl_xor_sync(0xffffffffu, nv[t], 8);
  if (!active) return;
  const int64_t pos = positions[tok];
  const int f0 = (ln & 7) * 8;  // frequency index of this lane's first element
  const float* cs = cos_sin + pos * 128;
  const bool first_half = ln < 8;
  uint32_t o[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    float r[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int e = 2 * t + u;
      const float c = cs[f0 + e];
      const float s = cs[64 + f0 + e];
      // first half: y1 = x1*cos - x2*sin ; second half: y2 = x2*cos + x1*sin
      r[u] = first_half ? __fsub_rn(__fmul_rn(nv[e], c), __fmul_rn(pv[e], s))
                        : __fadd_rn(__fmul_rn(nv[e], c), __fmul_rn(pv[e], s));
    }
    __nv_bfloat162 h2 = __floats2bfloat162_rn(r[0], r[1]);
    o[t] = *reinterpret_cast<uint32_t*>(&h2);
  }
  const uint4 rot = make_uint4(o[0], o[1], o[2], o[3]);
  *reinterpret_cast<uint4*>(x) = rot;
  if constexpr (KV != kNoStore) {
    if (!is_q) {
      const int64_t slot = slot_mapping[tok];
      if (slot >= 0 && slot < num_slots) {
        const int hk = hh - num_q_heads;
        const int64_t off = slot * row_elems + hk * 128 + 8 * ln;
        if constexpr (KV == kStoreBf16) {
          *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(k_cache) + off) = rot;
        } else {
          *reinterpret_cast<uint2*>(static_cast<uint8_t*>(k_cache) + off) = quant8_e4m3(rot, k_scale ? k_scale[hk] : 1.f);
          if constexpr (KV == kStoreFp8Mirror) *reinterpret_cast<uint4*>(k_mirror + off) = rot;
        }
      }
    }
  }
}

// out[t, i] = bf16(bf16(silu(x[t, i])) * y[t, i]) with x = in[t, :I], y = in[t, I:2I].
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, int rows,
                                int inter, int64_t in_stride, int64_t out_stride) {
  const int64_t vid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nvec = inter / 8;
  if (vid >= int64_t(rows) * nvec) return;
  const int64_t r = vid / nvec;
  const int c = int(vid % nvec);
  const uint4 a = *reinterpret_cast<const uint4*>(in + r * in_stride + 8 * c);
  const uint4 b = *reinterpret_cast<const uint4*>(in + r * in_stride + inter + 8 * c);
  const uint32_t wa[4] = {a.x, a.y, a.z, a.w};
  const uint32_t wb[4] = {b.x, b.y, b.z, b.w};
  uint32_t o[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    float xs[2] = {bf16lo(wa[t]), bf16hi(wa[t])};
    float ys[2] = {bf16lo(wb[t]), bf16hi(wb[t])};
    float rr[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float sx = bf16_round(__fdiv_rn(xs[u], __fadd_rn(1.0f, expf(-xs[u]))));
      rr[u] = __fmul_rn(sx, ys[u]);
    }
    __nv_bfloat162 h2 = __floats2bfloat162_rn(rr[0], rr[1]);
    o[t] = *reinterpret_cast<uint32_t*>(&h2);
  }
  *reinterpret_cast<uint4*>(out + r * out_stride + 8 * c) = make_uint4(o[0], o[1], o[2], o[3]);
}

// Greedy sampling: per row, index of the maximum (lowest index among ties; NaN never wins).
// One CTA per row; writes the token both to out_tokens[row] and, when given, to
// next_tokens[slot_of_row[row]] so the next decode step can read it on the device.
__global__ void argmax_kernel(const __nv_bfloat16* __restrict__ logits, int64_t row_stride, int vocab,
                              int64_t index_offset, int64_t* __restrict__ out_tokens, float* __restrict__ out_values) {
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + int64_t(row) * row_stride;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  // 16-byte loads (8 logits) when the row allows it; each thread walks its indices in
  // increasing order, so a strict '>' keeps the lowest index among equal values.
  int head = 0;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
    head = vocab & ~7;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    for (int i = threadIdx.x; i < (head >> 3); i += blockDim.x) {
      const uint4 v = __ldg(xv + i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float a = bf16lo(w[t]), b = bf16hi(w[t]);
        if (a > best) {
          best = a;
          bi = 8 * i + 2 * t;
        }
        if (b > best) {
          best = b;
          bi = 8 * i + 2 * t + 1;
        }
      }
    }
  }
  for (int i = head + threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = __bfloat162float(x[i]);
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sb[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (lane == 0) {
      out_tokens[row] = index_offset + ((bi == 0x7fffffff) ? 0 : bi);
      if (out_values) out_values[row] = best;
    }
  }
}

// ---------------------------------------------------------------------------- sampling
// Temperature sampling on the device by the Gumbel-max trick: token = argmax_i (logit_i / T + g_i)
// with g_i = -log(-log u_i), u_i uniform in (0, 1).  This is the same distribution as the
// reference's exponential race argmax_i softmax(logit / T)_i / E_i, E_i ~ Exp(1)
// (mini_vllm/layers/sampler.py:12-25 with top_k = -1, top_p = 1): -log E is Gumbel distributed
// and the softmax normaliser does not move the argmax.  u_i is a counter-based hash of (seed,
// step, row, global vocabulary index): SplitMix64's finaliser (Steele, Lea & Flood, "Fast
// splittable pseudorandom number generators", OOPSLA 2014), so the noise does not depend on how
// the vocabulary is sharded over ranks.  Rows with T <= 0 take the plain argmax.
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ float gumbel(uint64_t key, int64_t index) {
  const uint64_t h = splitmix64(key ^ (uint64_t(index) * 0xd1b54a32d192ed03ull));
  const float u = (float(uint32_t(h >> 40)) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
  return -__logf(-__logf(u));
}

// Per-thread best (value, index) over a row, threads strided over it with 16-byte loads when the
// row is aligned: x_i / T + Gumbel noise when hot, else x_i; the lowest index among equals.
__device__ __forceinline__ void row_best_strided(const __nv_bfloat16* __restrict__ x, int vocab, int64_t index_offset,
                                                 bool hot, float inv_t, uint64_t key, float& best, int& bi) {
  best = -INFINITY;
  bi = 0x7fffffff;
  int head = 0;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
    head = vocab & ~7;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    for (int i = threadIdx.x; i < (head >> 3); i += blockDim.x) {
      const uint4 v = __ldg(xv + i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t4 = 0; t4 < 4; ++t4) {
        float a = bf16lo(w[t4]), b = bf16hi(w[t4]);
        const int ia = 8 * i + 2 * t4;
        if (hot) {
          a = __fmaf_rn(a, inv_t, gumbel(key, index_offset + ia));
          b = __fmaf_rn(b, inv_t, gumbel(key, index_offset + ia + 1));
        }
        if (a > best) {
          best = a;
          bi = ia;
        }
        if (b > best) {
          best = b;
          bi = ia + 1;
        }
      }
    }
  }
  for (int i = head + threadIdx.x; i < vocab; i += blockDim.x) {
    float v = __bfloat162float(x[i]);
    if (hot) v = __fmaf_rn(v, inv_t, gumbel(key, index_offset + i));
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
}

__global__ void sample_kernel(const __nv_bfloat16* __restrict__ logits, int64_t row_stride, int vocab,
                              int64_t index_offset, const float* __restrict__ temperatures, uint64_t seed,
                              unsigned long long* __restrict__ step_state, int rows, int64_t* __restrict__ out_tokens,
                              float* __restrict__ out_values) {
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + int64_t(row) * row_stride;
  const float t = temperatures ? temperatures[row] : 0.f;
  const bool hot = t > 0.f;
  const float inv_t = hot ? 1.0f / t : 1.0f;
  __shared__ unsigned long long s_step;
  if (threadIdx.x == 0) s_step = step_state ? step_state[0] : 0ull;
  __syncthreads();
  const uint64_t key = splitmix64(seed ^ splitmix64(s_step * 0x9e3779b97f4a7c15ull + uint64_t(row)));
  float best;
  int bi;
  row_best_strided(x, vocab, index_offset, hot, inv_t, key, best, bi);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sb[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (lane == 0) {
      out_tokens[row] = index_offset + ((bi == 0x7fffffff) ? 0 : bi);
      if (out_values) out_values[row] = best;
      if (step_state) {
        // The last row to finish advances the step for the next launch (every row has read it).
        __threadfence();
        if (atomicAdd(&step_state[1], 1ull) == (unsigned long long)(rows - 1)) {
          step_state[1] = 0;
          step_state[0] = s_step + 1;
        }
      }
    }
  }
}


// ---------------------------------------------------------------------------------------------
// Sampling with top-k / top-p on the device (mini_vllm/layers/sampler.py:13-49): per row
// x = logits / temperature; top-k keeps the k largest x; top-p then keeps, in descending order
// of x, the tokens whose inclusive cumulative softmax probability (over the top-k set) is below
// top_p, and always the first; the token is a draw from the softmax over what is kept, taken
// as the Gumbel-max argmax(x + g) with the noise of hl_sample (so a row without top-k / top-p
// gets exactly hl_sample's token).  Tokens of equal value are ordered by index (lowest first)
// wherever the boundary of a filter cuts through them; torch.sort leaves that order unspecified.
//
// One CTA per row.  x's order is the order of the bf16 logits, so the selections work on a
// 16-bit order-preserving key of the logit bits with two 256-bin histograms (high byte, then
// the low byte inside the chosen bin): counts for top-k, softmax mass for top-p.  Each thread
// owns a contiguous range of the row, so "first m by index" is a block-wide scan of counts.
// ---------------------------------------------------------------------------------------------
constexpr int kFilterThreads = 1024;
constexpr float kLog2eF = 1.4426950408889634f;

__device__ __forceinline__ uint32_t order_key(uint32_t b16) {
  return (b16 & 0x8000u) ? (~b16 & 0xffffu) : (b16 | 0x8000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  const uint32_t b = (k & 0x8000u) ? (k & 0x7fffu) : (~k & 0xffffu);
  return __uint_as_float(b << 16);
}

template <typename T>
__device__ __forceinline__ T warp_incl_scan(T v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// Warp 0: scanning the 256 bins from the top, the bin b where the running total reaches
// `target` (above < target <= above + h[b]); -1 when the total stays below it.
template <typename T>
__device__ int find_from_top(const T* h, T target, T* above_out) {
  const int lane = threadIdx.x & 31;
  T part[8];
  T sum = T(0);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    part[j] = h[255 - (lane * 8 + j)];
    sum += part[j];
  }
  const T incl = warp_incl_scan(sum, lane);
  const T excl = incl - sum;
  const unsigned m = __ballot_sync(0xffffffffu, excl < target && target <= incl);
  int res = -1;
  T above = T(0);
  if (m) {
    const int src = __ffs(m) - 1;
    if (lane == src) {
      T c = excl;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (res < 0 && target <= c + part[j]) {
          res = 255 - (lane * 8 + j);
          above = c;
        }
        c += part[j];
      }
    }
    res = __shfl_sync(0xffffffffu, res, src);
    above = __shfl_sync(0xffffffffu, above, src);
  }
  *above_out = above;
  return res;
}

struct FilterShared {
  unsigned hc[256];
  float hm[256];
  unsigned wsum[32];
  float wsumf[32];
  int ires[2];
  float fres[4];
  unsigned ures[4];
};

// Block-wide exclusive scan of one count per thread; also returns the total.
__device__ __forceinline__ unsigned block_excl_scan(unsigned v, unsigned* total, FilterShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned incl = warp_incl_scan(v, lane);
  if (lane == 31) sh.wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const unsigned w = sh.wsum[lane];
    const unsigned wi = warp_incl_scan(w, lane);
    sh.wsum[lane] = wi - w;
    if (lane == 31) sh.ures[3] = wi;
  }
  __syncthreads();
  const unsigned r = sh.wsum[warp] + incl - v;
  *total = sh.ures[3];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float block_sum(float v, FilterShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) sh.wsumf[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = sh.wsumf[lane];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
    if (lane == 0) sh.fres[3] = w;
  }
  __syncthreads();
  const float r = sh.fres[3];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kFilterThreads) sample_filtered_kernel(
    const __nv_bfloat16* __restrict__ logits, int64_t row_stride, int vocab, const float* __restrict__ temperatures,
    const int32_t* __restrict__ top_ks, const float* __restrict__ top_ps, uint64_t seed,
    unsigned long long* __restrict__ step_state, int rows, int64_t* __restrict__ out_tokens) {
  __shared__ FilterShared sh;
  __shared__ unsigned long long s_step;
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint16_t* xr = reinterpret_cast<const uint16_t*>(logits + int64_t(row) * row_stride);
  const float t = temperatures ? temperatures[row] : 0.f;
  const bool hot = t > 0.f;
  const float inv_t = hot ? 1.0f / t : 1.0f;
  const int k = top_ks ? top_ks[row] : 0;
  const float top_p = top_ps ? top_ps[row] : 1.f;
  const bool filt_k = hot && k > 0 && k < vocab;
  const bool filt_p = hot && top_p < 1.f;
  if (tid == 0) s_step = step_state ? step_state[0] : 0ull;
  __syncthreads();
  const uint64_t key = splitmix64(seed ^ splitmix64(s_step * 0x9e3779b97f4a7c15ull + uint64_t(row)));
  const int seg = (vocab + kFilterThreads - 1) / kFilterThreads;
  const int begin = min(vocab, tid * seg), end = min(vocab, begin + seg);

  // Kept set: K = {key > kap} + the first m_k (by index) with key == kap; F = K filtered the same
  // way by (vp, idx_p).  Defaults keep everything.
  uint32_t kap = 0, vp = 0;
  int idx_k = INT_MAX, idx_p = INT_MAX;
  auto in_k = [&](int i, uint32_t kk) { return kk > kap || (kk == kap && i <= idx_k); };
  auto in_f = [&](int i, uint32_t kk) { return in_k(i, kk) && (kk > vp || (kk == vp && i <= idx_p)); };
  // Index of the m-th (1-based, index order) element of the row satisfying pred; INT_MAX if none.
  auto nth_index = [&](auto pred, unsigned m) {
    unsigned c = 0;
    for (int i = begin; i < end; ++i) c += pred(i, order_key(__ldg(xr + i))) ? 1u : 0u;
    unsigned total;
    const unsigned ex = block_excl_scan(c, &total, sh);
    if (tid == 0) sh.ires[0] = INT_MAX;
    __syncthreads();
    if (ex < m && m <= ex + c) {
      unsigned seen = ex;
      for (int i = begin; i < end; ++i) {
        if (pred(i, order_key(__ldg(xr + i))) && ++seen == m) {
          sh.ires[0] = i;
          break;
        }
      }
    }
    __syncthreads();
    const int r = sh.ires[0];
    __syncthreads();
    return r;
  };

  if (filt_k || filt_p) {
    // High-byte counts and the maximum key.
    for (int i = tid; i < 256; i += kFilterThreads) sh.hc[i] = 0u;
    __syncthreads();
    uint32_t kmax = 0;
    for (int i = begin; i < end; ++i) {
      const uint32_t kk = order_key(__ldg(xr + i));
      kmax = max(kmax, kk);
      if (filt_k) atomicAdd(&sh.hc[kk >> 8], 1u);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
    if (lane == 0) sh.wsum[warp] = kmax;
    __syncthreads();
    if (warp == 0) {
      uint32_t w = sh.wsum[lane];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) w = max(w, __shfl_xor_sync(0xffffffffu, w, o));
      if (lane == 0) sh.ures[0] = w;
    }
    __syncthreads();
    kmax = sh.ures[0];

    if (filt_k) {
      // k-th largest key: high byte, then low byte inside that bin.
      if (warp == 0) {
        unsigned above;
        const int b1 = find_from_top(sh.hc, unsigned(k), &above);
        if (lane == 0) {
          sh.ires[1] = b1;
          sh.ures[1] = above;
        }
      }
      __syncthreads();
      const int b1 = sh.ires[1];
      const unsigned above1 = sh.ures[1];
      __syncthreads();
      for (int i = tid; i < 256; i += kFilterThreads) sh.hc[i] = 0u;
      __syncthreads();
      for (int i = begin; i < end; ++i) {
        const uint32_t kk = order_key(__ldg(xr + i));
        if (int(kk >> 8) == b1) atomicAdd(&sh.hc[kk & 0xffu], 1u);
      }
      __syncthreads();
      if (warp == 0) {
        unsigned above;
        const int b2 = find_from_top(sh.hc, unsigned(k) - above1, &above);
        if (lane == 0) {
          sh.ires[1] = b2;
          sh.ures[1] = above1 + above;
          sh.ures[2] = b2 >= 0 ? sh.hc[b2] : 0u;
        }
      }
      __syncthreads();
      kap = (uint32_t(b1) << 8) | uint32_t(sh.ires[1]);
      const unsigned m_k = unsigned(k) - sh.ures[1];  // ties at kap to keep, >= 1
      const unsigned n_tie = sh.ures[2];
      __syncthreads();
      if (m_k < n_tie) idx_k = nth_index([&](int, uint32_t kk) { return kk == kap; }, m_k);
    }

    if (filt_p) {
      // Softmax mass over K by high byte; the top token (key kmax, lowest index) is always in K.
      const float vmax = key_float(kmax) * inv_t;
      for (int i = tid; i < 256; i += kFilterThreads) sh.hm[i] = 0.f;
      __syncthreads();
      float z = 0.f;
      for (int i = begin; i < end; ++i) {
        const uint32_t kk = order_key(__ldg(xr + i));
        if (!in_k(i, kk)) continue;
        const float e = exp2f((key_float(kk) * inv_t - vmax) * kLog2eF);
        z += e;
        atomicAdd(&sh.hm[kk >> 8], e);
      }
      z = block_sum(z, sh);
      // top_p <= 0 keeps only the first token, as the reference's "cumsum < top_p, first always
      // kept" does; z >= 1 (the top token's term), so the floor stays positive.
      const float thr = fmaxf(top_p, 1e-30f) * z;
      if (warp == 0) {
        float above;
        const int c1 = find_from_top(sh.hm, thr, &above);
        if (lane == 0) {
          sh.ires[1] = c1;
          sh.fres[0] = above;
        }
      }
      __syncthreads();
      const int c1 = sh.ires[1];
      const float above1 = sh.fres[0];
      __syncthreads();
      if (c1 >= 0) {
        for (int i = tid; i < 256; i += kFilterThreads) {
          sh.hm[i] = 0.f;
          sh.hc[i] = 0u;
        }
        __syncthreads();
        for (int i = begin; i < end; ++i) {
          const uint32_t kk = order_key(__ldg(xr + i));
          if (int(kk >> 8) != c1 || !in_k(i, kk)) continue;
          atomicAdd(&sh.hm[kk & 0xffu], exp2f((key_float(kk) * inv_t - vmax) * kLog2eF));
          atomicAdd(&sh.hc[kk & 0xffu], 1u);
        }
        __syncthreads();
        if (warp == 0) {
          float above;
          int c2 = find_from_top(sh.hm, thr - above1, &above);
          if (c2 < 0) {  // rounding: the crossing is the lowest non-empty bin
            above = 0.f;
            c2 = -1;
            float acc = 0.f;
            for (int b = 255; b >= 0; --b) {
              if (sh.hc[b] != 0u) {
                c2 = b;
                above = acc;
              }
              acc += sh.hm[b];
            }
          }
          if (lane == 0) {
            sh.ires[1] = c2;
            sh.fres[1] = above1 + above;
            sh.ures[2] = c2 >= 0 ? sh.hc[c2] : 0u;
          }
        }
        __syncthreads();
        const int c2 = sh.ires[1];
        const float cum_gt = sh.fres[1];
        const unsigned n_tie = sh.ures[2];
        __syncthreads();
        if (c2 >= 0) {
          vp = (uint32_t(c1) << 8) | uint32_t(c2);
          const float e_v = exp2f((key_float(vp) * inv_t - vmax) * kLog2eF);
          // tie r (0-based) is kept iff cum_gt + (r + 1) e_v < thr
          float mf = ceilf((thr - cum_gt) / e_v) - 1.f;
          unsigned m_p = mf <= 0.f ? 0u : (mf >= float(n_tie) ? n_tie : unsigned(mf));
          if (vp == kmax && m_p == 0u) m_p = 1u;  // the first token is always kept
          if (m_p < n_tie)
            idx_p = m_p == 0u ? -1 : nth_index([&](int i, uint32_t kk) { return kk == vp && in_k(i, kk); }, m_p);
        }
      }
    }
  }

  // Gumbel-max (or argmax for a greedy row) over the kept tokens; lowest index among equals.
  // Rows without a filter take hl_sample's scan, so their token (and cost) is hl_sample's.
  float best = -INFINITY;
  int bi = 0x7fffffff;
  if (!(filt_k || filt_p)) {
    row_best_strided(logits + int64_t(row) * row_stride, vocab, 0, hot, inv_t, key, best, bi);
  } else {
    for (int i = begin; i < end; ++i) {
      const uint32_t raw = __ldg(xr + i);
      if (!in_f(i, order_key(raw))) continue;
      float v = __uint_as_float(raw << 16);
      if (hot) v = __fmaf_rn(v, inv_t, gumbel(key, i));
      if (v > best) {
        best = v;
        bi = i;
      }
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  if (lane == 0) {
    sh.wsumf[warp] = best;
    sh.wsum[warp] = unsigned(bi);
  }
  __syncthreads();
  if (warp == 0) {
    best = sh.wsumf[lane];
    bi = int(sh.wsum[lane]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (lane == 0) {
      out_tokens[row] = (bi == 0x7fffffff) ? 0 : bi;
      if (step_state) {
        __threadfence();
        if (atomicAdd(&step_state[1], 1ull) == (unsigned long long)(rows - 1)) {
          step_state[1] = 0;
          step_state[0] = s_step + 1;
        }
      }
    }
  }
}

}  // namespace
}  // namespace hl

using namespace hl;

extern "C" int hl_sample(const void* logits, int64_t row_stride, int rows, int vocab, int64_t index_offset,
                         const float* temperatures, uint64_t seed, void* step_state, int64_t* out_tokens,
                         float* out_values, void* stream) {
  clear_error();
  if (rows == 0) return HL_OK;
  HL_CHECK_ARG(logits && out_tokens && rows > 0 && vocab > 0, "hl_sample: bad arguments");
  sample_kernel<<<rows, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
      (const __nv_bfloat16*)logits, row_stride, vocab, index_offset, temperatures, seed,
      static_cast<unsigned long long*>(step_state), rows, out_tokens, out_values);
  HL_CHECK_LAUNCH("hl_sample");
  return HL_OK;
}

extern "C" int hl_sample_filtered(const void* logits, int64_t row_stride, int rows, int vocab,
                                  const float* temperatures, const int32_t* top_ks, const float* top_ps,
                                  uint64_t seed, void* step_state, int64_t* out_tokens, void* stream) {
  clear_error();
  if (rows == 0) return HL_OK;
  HL_CHECK_ARG(logits && out_tokens && rows > 0 && vocab > 0 && row_stride >= vocab,
               "hl_sample_filtered: bad arguments");
  sample_filtered_kernel<<<rows, kFilterThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      (const __nv_bfloat16*)logits, row_stride, vocab, temperatures, top_ks, top_ps, seed,
      static_cast<unsigned long long*>(step_state), rows, out_tokens);
  HL_CHECK_LAUNCH("hl_sample_filtered");
  return HL_OK;
}

extern "C" int hl_rmsnorm(const void* in, int64_t in_stride, void* residual, const void* weight, void* out,
                          int64_t out_stride, int rows, int hidden, float eps, void* stream) {
  clear_error();
  if (rows == 0) return HL_OK;
  HL_CHECK_ARG(in && weight && out && rows > 0, "hl_rmsnorm: bad arguments");
  HL_CHECK_ARG(hidden % 256 == 0 && hidden <= 8192, "hl_rmsnorm: hidden must be a multiple of 256, <= 8192");
  HL_CHECK_ARG(aligned16(in) && aligned16(out) && aligned16(weight) && in_stride % 8 == 0 && out_stride % 8 == 0 &&
                   (!residual || aligned16(residual)),
               "hl_rmsnorm: 16-byte alignment required");
  const int threads = 256;
  const int blocks = (rows * 32 + threads - 1) / threads;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __nv_bfloat16* x = (const __nv_bfloat16*)in;
  __nv_bfloat16* r = (__nv_bfloat16*)residual;
  const __nv_bfloat16* wt = (const __nv_bfloat16*)weight;
  __nv_bfloat16* y = (__nv_bfloat16*)out;
#define HL_RMS_CASE(NV)                                                                                  \
  case NV:                                                                                               \
    if (r)                                                                                               \
      rmsnorm_kernel<true, NV><<<blocks, threads, 0, s>>>(x, r, wt, y, rows, hidden, in_stride, out_stride, eps); \
    else                                                                                                 \
      rmsnorm_kernel<false, NV><<<blocks, threads, 0, s>>>(x, r, wt, y, rows, hidden, in_stride, out_stride, eps); \
    break;
  switch (hidden / 256) {
    HL_RMS_CASE(1) HL_RMS_CASE(2) HL_RMS_CASE(3) HL_RMS_CASE(4) HL_RMS_CASE(5) HL_RMS_CASE(6) HL_RMS_CASE(8)
    HL_RMS_CASE(10) HL_RMS_CASE(12) HL_RMS_CASE(14) HL_RMS_CASE(16) HL_RMS_CASE(20) HL_RMS_CASE(24)
    HL_RMS_CASE(28) HL_RMS_CASE(32)
    default:
      set_error("hl_rmsnorm: hidden=%d not supported", hidden);
      return HL_ERR_UNSUPPORTED;
  }
#undef HL_RMS_CASE
  HL_CHECK_LAUNCH("hl_rmsnorm");
  return HL_OK;
}

extern "C" int hl_qk_norm_rope(void* qkv, int64_t row_stride, int num_tokens, int num_q_heads, int num_kv_heads,
                               int head_dim, const void* q_weight, const void* k_weight, const float* cos_sin,
                               const int64_t* positions, float eps, void* stream) {
  return hl_qk_norm_rope_store(qkv, row_stride, num_tokens, num_q_heads, num_kv_heads, head_dim, q_weight, k_weight,
                               cos_sin, positions, eps, nullptr, nullptr, 0, nullptr, 0, nullptr, nullptr, stream);
}

extern "C" int hl_qk_norm_rope_store(void* qkv, int64_t row_stride, int num_tokens, int num_q_heads,
                                     int num_kv_heads, int head_dim, const void* q_weight, const void* k_weight,
                                     const float* cos_sin, const int64_t* positions, float eps, void* k_cache,
                                     void* v_cache, int kv_dtype, const int32_t* slot_mapping, int64_t num_slots,
                                     const float* k_scale, const float* v_scale, void* stream) {
  return hl_qk_norm_rope_store_mirrored(qkv, row_stride, num_tokens, num_q_heads, num_kv_heads, head_dim, q_weight,
                                        k_weight, cos_sin, positions, eps, k_cache, v_cache, kv_dtype, slot_mapping,
                                        num_slots, k_scale, v_scale, nullptr, nullptr, stream);
}

extern "C" int hl_qk_norm_rope_store_mirrored(void* qkv, int64_t row_stride, int num_tokens, int num_q_heads,
                                              int num_kv_heads, int head_dim, const void* q_weight,
                                              const void* k_weight, const float* cos_sin, const int64_t* positions,
                                              float eps, void* k_cache, void* v_cache, int kv_dtype,
                                              const int32_t* slot_mapping, int64_t num_slots, const float* k_scale,
                                              const float* v_scale, void* k_mirror, void* v_mirror, void* stream) {
  clear_error();
  if (num_tokens == 0) return HL_OK;
  HL_CHECK_ARG(qkv && q_weight && k_weight && cos_sin && positions && num_tokens > 0, "hl_qk_norm_rope: bad args");
  HL_CHECK_ARG(head_dim == 128, "hl_qk_norm_rope: head_dim must be 128");
  HL_CHECK_ARG(aligned16(qkv) && row_stride % 8 == 0, "hl_qk_norm_rope: 16-byte alignment required");
  const bool store = k_cache != nullptr;
  const bool mirror = k_mirror != nullptr || v_mirror != nullptr;
  if (store) {
    HL_CHECK_ARG(v_cache && slot_mapping && num_slots > 0, "hl_qk_norm_rope_store: cache arguments missing");
    HL_CHECK_ARG(kv_dtype == HL_KV_BF16 || kv_dtype == HL_KV_FP8_E4M3, "hl_qk_norm_rope_store: bad kv_dtype");
    HL_CHECK_ARG(aligned16(k_cache) && aligned16(v_cache), "hl_qk_norm_rope_store: 16-byte aligned caches required");
  } else {
    HL_CHECK_ARG(!v_cache, "hl_qk_norm_rope_store: v_cache without k_cache");
  }
  if (mirror) {
    HL_CHECK_ARG(store && kv_dtype == HL_KV_FP8_E4M3 && k_mirror && v_mirror,
                 "hl_qk_norm_rope_store_mirrored: bf16 mirror caches go with an FP8 store (both k and v)");
    HL_CHECK_ARG(aligned16(k_mirror) && aligned16(v_mirror), "hl_qk_norm_rope_store_mirrored: 16-byte alignment");
  }
  const int heads = num_q_heads + (store ? 2 : 1) * num_kv_heads;
  const int64_t groups = int64_t(num_tokens) * heads;
  const int threads = 256;
  const int64_t blocks = (groups * 16 + threads - 1) / threads;
  HL_CHECK_ARG(blocks < (1ll << 31), "hl_qk_norm_rope: grid too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto q = (__nv_bfloat16*)qkv;
  auto qwt = (const __nv_bfloat16*)q_weight;
  auto kwt = (const __nv_bfloat16*)k_weight;
  if (!store) {
    qk_norm_rope_kernel<kNoStore><<<(unsigned)blocks, threads, 0, s>>>(
        q, row_stride, num_tokens, num_q_heads, num_kv_heads, qwt, kwt, cos_sin, positions, eps, nullptr, nullptr,
        nullptr, 0, nullptr, nullptr, nullptr, nullptr);
  } else if (kv_dtype == HL_KV_BF16) {
    qk_norm_rope_kernel<kStoreBf16><<<(unsigned)blocks, threads, 0, s>>>(
        q, row_stride, num_tokens, num_q_heads, num_kv_heads, qwt, kwt, cos_sin, positions, eps, k_cache, v_cache,
        slot_mapping, num_slots, nullptr, nullptr, nullptr, nullptr);
  } else if (!mirror) {
    qk_norm_rope_kernel<kStoreFp8><<<(unsigned)blocks, threads, 0, s>>>(
        q, row_stride, num_tokens, num_q_heads, num_kv_heads, qwt, kwt, cos_sin, positions, eps, k_cache, v_cache,
        slot_mapping, num_slots, k_scale, v_scale, nullptr, nullptr);
  } else {
    qk_norm_rope_kernel<kStoreFp8Mirror><<<(unsigned)blocks, threads, 0, s>>>(
        q, row_stride, num_tokens, num_q_heads, num_kv_heads, qwt, kwt, cos_sin, positions, eps, k_cache, v_cache,
        slot_mapping, num_slots, k_scale, v_scale, static_cast<__nv_bfloat16*>(k_mirror),
        static_cast<__nv_bfloat16*>(v_mirror));
  }
  HL_CHECK_LAUNCH("hl_qk_norm_rope");
  return HL_OK;
}

extern "C" int hl_silu_mul(const void* in, int64_t in_stride, void* out, int64_t out_stride, int rows,
                           int intermediate, void* stream) {
  clear_error();
  if (rows == 0) return HL_OK;
  HL_CHECK_ARG(in && out && rows > 0 && intermediate % 8 == 0, "hl_silu_mul: bad arguments");
  HL_CHECK_ARG(aligned16(in) && aligned16(out) && in_stride % 8 == 0 && out_stride % 8 == 0,
               "hl_silu_mul: 16-byte alignment required");
  const int64_t n = int64_t(rows) * (intermediate / 8);
  const int threads = 256;
  silu_mul_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      (const __nv_bfloat16*)in, (__nv_bfloat16*)out, rows, intermediate, in_stride, out_stride);
  HL_CHECK_LAUNCH("hl_silu_mul");
  return HL_OK;
}

extern "C" int hl_argmax(const void* logits, int64_t row_stride, int rows, int vocab, int64_t* out_tokens,
                         void* stream) {
  clear_error();
  if (rows == 0) return HL_OK;
  HL_CHECK_ARG(logits && out_tokens && rows > 0 && vocab > 0, "hl_argmax: bad arguments");
  argmax_kernel<<<rows, 1024, 0, static_cast<cudaStream_t>(stream)>>>((const __nv_bfloat16*)logits, row_stride, vocab,
                                                                       0, out_tokens, nullptr);
  HL_CHECK_LAUNCH("hl_argmax");
  return HL_OK;
}

extern "C" int hl_argmax_shard(const void* logits, int64_t row_stride, int rows, int vocab, int64_t index_offset,
                               int64_t* out_tokens, float* out_values, void* stream) {
  clear_error();
  if (rows == 0) return HL_OK;
  HL_CHECK_ARG(logits && out_tokens && out_values && rows > 0 && vocab > 0, "hl_argmax_shard: bad arguments");
  argmax_kernel<<<rows, 1024, 0, static_cast<cudaStream_t>(stream)>>>((const __nv_bfloat16*)logits, row_stride, vocab,
                                                                       index_offset, out_tokens, out_values);
  HL_CHECK_LAUNCH("hl_argmax_shard");
  return HL_OK;
}
