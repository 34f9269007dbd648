// KV-cache store kernels: scatter new K/V rows into the paged cache by slot_mapping
// (BF16 copy and FP8 e4m3 quantising store), and the BF16 -> FP8 prefill-to-decode copy.
//
// Semantics follow mini_vllm/layers/attention.py:59-90 (store_kvcache_kernel: token i with
// slot != -1 writes key[i] / value[i], num_kv_heads*head_dim contiguous elements, to
// k_cache[slot] / v_cache[slot]) and :51-56 (the FP8 store and the FP8 copy whose source is
// not in the reference tree; here they quantise as round-to-nearest-even e4m3 of x/scale[h]
// with saturation at +-448).
//
// One CTA per token row, 16-byte vectors: a row of Hk*D bf16 is Hk*D/8 vectors, so for
// Qwen3 (Hk*D = 1024) 128 threads move the K row and the V row with one 16-byte load and
// one 16-byte store each.  The kernels are HBM/latency bound; the grid is sized by tokens.
#include "hl_common.cuh"

namespace hl {
namespace {

constexpr int kStoreThreads = 128;

__device__ __forceinline__ bool slot_ok(int64_t slot, int64_t num_slots) { return slot >= 0 && slot < num_slots; }

// ------------------------------------------------------------------ BF16 store
__global__ void __launch_bounds__(kStoreThreads) store_kv_bf16_vec(
    const __nv_bfloat16* __restrict__ key, const __nv_bfloat16* __restrict__ value, int64_t key_stride,
    int64_t value_stride, __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
    const int32_t* __restrict__ slot_mapping, int64_t num_slots, int row_elems) {
  const int64_t tok = blockIdx.x;
  const int64_t slot = slot_mapping[tok];
  if (!slot_ok(slot, num_slots)) return;
  const int nvec = row_elems >> 3;
  const uint4* ks = reinterpret_cast<const uint4*>(key + tok * key_stride);
  const uint4* vs = reinterpret_cast<const uint4*>(value + tok * value_stride);
  uint4* kd = reinterpret_cast<uint4*>(k_cache + slot * row_elems);
  uint4* vd = reinterpret_cast<uint4*>(v_cache + slot * row_elems);
  for (int i = threadIdx.x; i < nvec; i += kStoreThreads) {
    uint4 a = __ldg(ks + i);
    uint4 b = __ldg(vs + i);
    kd[i] = a;
    vd[i] = b;
  }
}

__global__ void __launch_bounds__(kStoreThreads) store_kv_bf16_scalar(
    const __nv_bfloat16* __restrict__ key, const __nv_bfloat16* __restrict__ value, int64_t key_stride,
    int64_t value_stride, __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
    const int32_t* __restrict__ slot_mapping, int64_t num_slots, int row_elems) {
  const int64_t tok = blockIdx.x;
  const int64_t slot = slot_mapping[tok];
  if (!slot_ok(slot, num_slots)) return;
  for (int i = threadIdx.x; i < row_elems; i += kStoreThreads) {
    k_cache[slot * row_elems + i] = key[tok * key_stride + i];
    v_cache[slot * row_elems + i] = value[tok * value_stride + i];
  }
}

// ------------------------------------------------------------------ FP8 quantisation
__global__ void __launch_bounds__(kStoreThreads) store_kv_fp8_vec(
    const __nv_bfloat16* __restrict__ key, const __nv_bfloat16* __restrict__ value, int64_t key_stride,
    int64_t value_stride, uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
    const int32_t* __restrict__ slot_mapping, int64_t num_slots, int row_elems, int head_dim,
    const float* __restrict__ k_scale, const float* __restrict__ v_scale) {
  const int64_t tok = blockIdx.x;
  const int64_t slot = slot_mapping[tok];
  if (!slot_ok(slot, num_slots)) return;
  const int nvec = row_elems >> 3;
  const uint4* ks = reinterpret_cast<const uint4*>(key + tok * key_stride);
  const uint4* vs = reinterpret_cast<const uint4*>(value + tok * value_stride);
  uint2* kd = reinterpret_cast<uint2*>(k_cache + slot * row_elems);
  uint2* vd = reinterpret_cast<uint2*>(v_cache + slot * row_elems);
  for (int i = threadIdx.x; i < nvec; i += kStoreThreads) {
    const int h = (i * 8) / head_dim;
    const float sk = k_scale ? k_scale[h] : 1.0f;
    const float sv = v_scale ? v_scale[h] : 1.0f;
    kd[i] = quant8_e4m3(__ldg(ks + i), sk);
    vd[i] = quant8_e4m3(__ldg(vs + i), sv);
  }
}

__global__ void __launch_bounds__(kStoreThreads) store_kv_fp8_scalar(
    const __nv_bfloat16* __restrict__ key, const __nv_bfloat16* __restrict__ value, int64_t key_stride,
    int64_t value_stride, uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
    const int32_t* __restrict__ slot_mapping, int64_t num_slots, int row_elems, int head_dim,
    const float* __restrict__ k_scale, const float* __restrict__ v_scale) {
  const int64_t tok = blockIdx.x;
  const int64_t slot = slot_mapping[tok];
  if (!slot_ok(slot, num_slots)) return;
  for (int i = threadIdx.x; i < row_elems; i += kStoreThreads) {
    const int h = i / head_dim;
    const float sk = k_scale ? k_scale[h] : 1.0f;
    const float sv = v_scale ? v_scale[h] : 1.0f;
    k_cache[slot * row_elems + i] =
        float_to_e4m3_sat(__fdiv_rn(__bfloat162float(key[tok * key_stride + i]), sk));
    v_cache[slot * row_elems + i] =
        float_to_e4m3_sat(__fdiv_rn(__bfloat162float(value[tok * value_stride + i]), sv));
  }
}

// ------------------------------------------------------------------ BF16 -> FP8 copy
// grid (num_tokens, num_layers): each CTA converts one slot's K and V rows of one layer.
__global__ void __launch_bounds__(kStoreThreads) copy_kv_bf16_to_fp8_kernel(
    const __nv_bfloat16* __restrict__ src_k, const __nv_bfloat16* __restrict__ src_v, uint8_t* __restrict__ dst_k,
    uint8_t* __restrict__ dst_v, const int32_t* __restrict__ slot_mapping, int64_t num_slots, int row_elems,
    int head_dim, const float* __restrict__ k_scale, const float* __restrict__ v_scale, int64_t src_layer_stride,
    int64_t dst_layer_stride, int64_t scale_layer_stride) {
  const int64_t tok = blockIdx.x;
  const int64_t layer = blockIdx.y;
  const int64_t slot = slot_mapping[tok];
  if (!slot_ok(slot, num_slots)) return;
  const int nvec = row_elems >> 3;
  const uint4* ks = reinterpret_cast<const uint4*>(src_k + layer * src_layer_stride + slot * row_elems);
  const uint4* vs = reinterpret_cast<const uint4*>(src_v + layer * src_layer_stride + slot * row_elems);
  uint2* kd = reinterpret_cast<uint2*>(dst_k + layer * dst_layer_stride + slot * row_elems);
  uint2* vd = reinterpret_cast<uint2*>(dst_v + layer * dst_layer_stride + slot * row_elems);
  const float* ksc = k_scale ? k_scale + layer * scale_layer_stride : nullptr;
  const float* vsc = v_scale ? v_scale + layer * scale_layer_stride : nullptr;
  for (int i = threadIdx.x; i < nvec; i += kStoreThreads) {
    const int h = (i * 8) / head_dim;
    kd[i] = quant8_e4m3(__ldg(ks + i), ksc ? ksc[h] : 1.0f);
    vd[i] = quant8_e4m3(__ldg(vs + i), vsc ? vsc[h] : 1.0f);
  }
}

bool vec_ok(const void* a, const void* b, int64_t sa, int64_t sb, const void* c, const void* d) {
  return aligned16(a) && aligned16(b) && aligned16(c) && aligned16(d) && (sa % 8 == 0) && (sb % 8 == 0);
}

}  // namespace
}  // namespace hl

using namespace hl;

extern "C" int hl_store_kv_bf16(const void* key, const void* value, int64_t key_row_stride, int64_t value_row_stride,
                                void* k_cache, void* v_cache, const int32_t* slot_mapping, int64_t num_tokens,
                                int64_t num_slots, int num_kv_heads, int head_dim, void* stream) {
  clear_error();
  HL_CHECK_ARG(num_tokens >= 0, "hl_store_kv_bf16: num_tokens < 0");
  if (num_tokens == 0) return HL_OK;
  HL_CHECK_ARG(key && value && k_cache && v_cache && slot_mapping, "hl_store_kv_bf16: null pointer");
  HL_CHECK_ARG(num_kv_heads > 0 && head_dim > 0, "hl_store_kv_bf16: bad head shape");
  HL_CHECK_ARG(num_tokens <= 0x7fffffff, "hl_store_kv_bf16: too many tokens");
  const int row = num_kv_heads * head_dim;
  HL_CHECK_ARG(key_row_stride >= row && value_row_stride >= row, "hl_store_kv_bf16: row stride < Hk*D");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (row % 8 == 0 && vec_ok(key, value, key_row_stride, value_row_stride, k_cache, v_cache)) {
    store_kv_bf16_vec<<<(unsigned)num_tokens, kStoreThreads, 0, s>>>(
        (const __nv_bfloat16*)key, (const __nv_bfloat16*)value, key_row_stride, value_row_stride,
        (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, slot_mapping, num_slots, row);
  } else {
    store_kv_bf16_scalar<<<(unsigned)num_tokens, kStoreThreads, 0, s>>>(
        (const __nv_bfloat16*)key, (const __nv_bfloat16*)value, key_row_stride, value_row_stride,
        (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, slot_mapping, num_slots, row);
  }
  HL_CHECK_LAUNCH("hl_store_kv_bf16");
  return HL_OK;
}

extern "C" int hl_store_kv_fp8(const void* key, const void* value, int64_t key_row_stride, int64_t value_row_stride,
                               void* k_cache, void* v_cache, const int32_t* slot_mapping, int64_t num_tokens,
                               int64_t num_slots, int num_kv_heads, int head_dim, const float* k_scale,
                               const float* v_scale, void* stream) {
  clear_error();
  HL_CHECK_ARG(num_tokens >= 0, "hl_store_kv_fp8: num_tokens < 0");
  if (num_tokens == 0) return HL_OK;
  HL_CHECK_ARG(key && value && k_cache && v_cache && slot_mapping, "hl_store_kv_fp8: null pointer");
  HL_CHECK_ARG(num_kv_heads > 0 && head_dim > 0, "hl_store_kv_fp8: bad head shape");
  HL_CHECK_ARG(num_tokens <= 0x7fffffff, "hl_store_kv_fp8: too many tokens");
  const int row = num_kv_heads * head_dim;
  HL_CHECK_ARG(key_row_stride >= row && value_row_stride >= row, "hl_store_kv_fp8: row stride < Hk*D");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = (head_dim % 8 == 0) && aligned16(key) && aligned16(value) && (key_row_stride % 8 == 0) &&
                   (value_row_stride % 8 == 0) && ((reinterpret_cast<uintptr_t>(k_cache) & 7u) == 0) &&
                   ((reinterpret_cast<uintptr_t>(v_cache) & 7u) == 0);
  if (vec) {
    store_kv_fp8_vec<<<(unsigned)num_tokens, kStoreThreads, 0, s>>>(
        (const __nv_bfloat16*)key, (const __nv_bfloat16*)value, key_row_stride, value_row_stride, (uint8_t*)k_cache,
        (uint8_t*)v_cache, slot_mapping, num_slots, row, head_dim, k_scale, v_scale);
  } else {
    store_kv_fp8_scalar<<<(unsigned)num_tokens, kStoreThreads, 0, s>>>(
        (const __nv_bfloat16*)key, (const __nv_bfloat16*)value, key_row_stride, value_row_stride, (uint8_t*)k_cache,
        (uint8_t*)v_cache, slot_mapping, num_slots, row, head_dim, k_scale, v_scale);
  }
  HL_CHECK_LAUNCH("hl_store_kv_fp8");
  return HL_OK;
}

extern "C" int hl_copy_kv_bf16_to_fp8(const void* src_k, const void* src_v, void* dst_k, void* dst_v,
                                      const int32_t* slot_mapping, int64_t num_tokens, int64_t num_slots,
                                      int num_kv_heads, int head_dim, const float* k_scale, const float* v_scale,
                                      int num_layers, int64_t src_layer_stride, int64_t dst_layer_stride,
                                      int64_t scale_layer_stride, void* stream) {
  clear_error();
  HL_CHECK_ARG(num_tokens >= 0 && num_layers >= 0, "hl_copy_kv_bf16_to_fp8: negative size");
  if (num_tokens == 0 || num_layers == 0) return HL_OK;
  HL_CHECK_ARG(src_k && src_v && dst_k && dst_v && slot_mapping, "hl_copy_kv_bf16_to_fp8: null pointer");
  HL_CHECK_ARG(num_kv_heads > 0 && head_dim > 0 && head_dim % 8 == 0, "hl_copy_kv_bf16_to_fp8: head_dim % 8 != 0");
  HL_CHECK_ARG(num_tokens <= 0x7fffffff && num_layers <= 65535, "hl_copy_kv_bf16_to_fp8: grid too large");
  HL_CHECK_ARG(aligned16(src_k) && aligned16(src_v) && src_layer_stride % 8 == 0,
               "hl_copy_kv_bf16_to_fp8: source must be 16-byte aligned");
  HL_CHECK_ARG(((reinterpret_cast<uintptr_t>(dst_k) | reinterpret_cast<uintptr_t>(dst_v)) & 7u) == 0 &&
                   dst_layer_stride % 8 == 0,
               "hl_copy_kv_bf16_to_fp8: destination must be 8-byte aligned");
  const int row = num_kv_heads * head_dim;
  dim3 grid((unsigned)num_tokens, (unsigned)num_layers);
  copy_kv_bf16_to_fp8_kernel<<<grid, kStoreThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      (const __nv_bfloat16*)src_k, (const __nv_bfloat16*)src_v, (uint8_t*)dst_k, (uint8_t*)dst_v, slot_mapping,
      num_slots, row, head_dim, k_scale, v_scale, src_layer_stride, dst_layer_stride, scale_layer_stride);
  HL_CHECK_LAUNCH("hl_copy_kv_bf16_to_fp8");
  return HL_OK;
}
