// Tensor-parallel all-reduce over NVLink peer memory, fused with the residual add + RMSNorm
// that follows every all-reduce of the Qwen3 decoder.
//
// The reference sums the o_proj and down_proj partial outputs with an NCCL all-reduce
// (mini_vllm/layers/linear.py:176-178) and then runs add + RMSNorm on the result
// (post_attention_layernorm / the next layer's input_layernorm / the final norm,
// mini_vllm/layers/layernorm.py:30-42, models/qwen3.py:150-157).  Here one kernel does both:
// every rank keeps its partial sums in a buffer that the other ranks mapped through CUDA IPC,
// a CTA meets the same CTA of every peer at a flag barrier (relaxed peer stores, acquire polls of
// its own flags), then
// reads its rows from all ranks' buffers over NVLink with plain loads, sums them in fp32 in
// rank order (so every rank computes bit-identical results), rounds to bf16 (the all-reduce
// result, as NCCL returns it) and applies the reference's add + RMSNorm arithmetic.
//
// Reuse: the o_proj and down_proj partials live in two different buffers that alternate, so
// when a rank is at call k+2 (writing buffer A again with its GEMM), every peer has passed the
// start barrier of call k+1 and therefore finished reading buffer A of call k (kernels of a
// stream run in order) — one barrier per call is enough.  Flags carry a per-CTA epoch that
// grows by one per call (compared with >=, so a peer running one call ahead is harmless).
//
// Every wait is bounded by time (globaltimer): on expiry the CTA records HL_AR_TIMEOUT in the
// rank's error word, skips the peer reads (treats the partial sums as zero) and finishes the
// add + RMSNorm; the host reads the word.
// No multicast, no NVLS: peer memory is only touched by ordinary loads and stores.
#include "hl_common.cuh"

namespace hl {
namespace {

constexpr int kArMaxRanks = 8;
constexpr int kArMaxBlocks = 128;
constexpr int kArThreads = 128;

struct ArParams {
  const __nv_bfloat16* data[kArMaxRanks];  // rank p's partial sums [rows, hidden]
  __nv_bfloat16* result[kArMaxRanks];      // two-shot: rank p's reduced rows [rows, hidden]
  int* signal[kArMaxRanks];                // rank p's flags [2][kArMaxBlocks][kArMaxRanks]
  int world;
  int rank;
  int rows;
  int hidden;
  __nv_bfloat16* residual;  // [rows, hidden], updated in place
  const __nv_bfloat16* weight;
  __nv_bfloat16* out;
  int64_t out_stride;
  float eps;
  int* epochs;      // this rank's per-CTA call counters [kArMaxBlocks]
  int* error_word;  // this rank's error bits
  unsigned long long timeout_ns;
};

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The flag store needs no release: the partial sums it announces were written by an earlier
// kernel of this stream and are complete in this GPU's memory before this kernel starts.  The
// poll keeps acquire semantics so that the peer-buffer loads after it cannot be served from
// copies older than the flag.
__device__ __forceinline__ void store_flag_sys(int* p, int v) {
  asm volatile("st.relaxed.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Publishes this thread's earlier stores, and those it has observed (the CTA's, through the
// __syncthreads before it), at system scope before the flag: the two-shot barrier announces rows
// that this kernel itself pushed into the peers' memory.
__device__ __forceinline__ void store_flag_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int load_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Barrier of this CTA with the same CTA of every peer on flag bank `bank`: thread t < world
// (t != rank) writes the epoch into peer t's slot for this rank and polls its own slot for peer t.
// Returns false (and records HL_AR_TIMEOUT) if a peer did not arrive in time.
template <bool kRelease>
__device__ __forceinline__ bool cta_barrier(const ArParams& p, int bank, int epoch, int* s_ok) {
  const int blk = blockIdx.x;
  const int tid = threadIdx.x;
  if (tid < p.world && tid != p.rank) {
    int* slot = p.signal[tid] + (bank * kArMaxBlocks + blk) * kArMaxRanks + p.rank;
    if constexpr (kRelease)
      store_flag_release_sys(slot, epoch);
    else
      store_flag_sys(slot, epoch);
    const int* mine = p.signal[p.rank] + (bank * kArMaxBlocks + blk) * kArMaxRanks + tid;
    const unsigned long long t0 = global_ns();
    bool arrived = false;
    for (uint32_t it = 0;; ++it) {
      if (load_acquire_sys(mine) >= epoch) {
        arrived = true;
        break;
      }
      if ((it & 255u) == 255u && global_ns() - t0 > p.timeout_ns) break;
    }
    if (!arrived) {
      *s_ok = 0;
      atomicOr(p.error_word, HL_AR_TIMEOUT);
    }
  }
  __syncthreads();
  return *s_ok != 0;
}

// Work split.  The peer reads are done in units of 1024 elements of one row (32 lanes x 4
// 16-byte vectors); a warp issues the loads of a unit from every rank at once, so a unit costs one
// NVLink round trip whatever the rank count.  A CTA takes a group of rows_per_cta() rows and its
// four warps share the group's units; the add + RMSNorm then runs one warp per row, with the
// row in registers in the add + RMSNorm kernel's layout and order (lane owns the vectors
// lane + 32 c), so one rank reproduces that kernel bit for bit.
constexpr int kUnitElems = 1024;

__host__ __device__ constexpr int rows_per_cta(int hidden) { return hidden <= 1024 ? 4 : (hidden <= 2048 ? 2 : 1); }

// bf16(sum over ranks, in rank order, in fp32) of the ncv 8-element vectors this lane owns in one
// unit; `off` = row * hidden + unit * 1024 + 8 * lane.  Peer partials change between calls at the
// same addresses: no L1 caching.
__device__ __forceinline__ void reduce_unit(const ArParams& p, int64_t off, int ncv, uint4 (&sum)[4]) {
  uint4 a[kArMaxRanks][4];
#pragma unroll
  for (int r = 0; r < kArMaxRanks; ++r)
    if (r < p.world)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c < ncv) a[r][c] = __ldcv(reinterpret_cast<const uint4*>(p.data[r] + off + 256 * c));
  float buf[4][8];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int t = 0; t < 8; ++t) buf[c][t] = 0.f;
#pragma unroll
  for (int r = 0; r < kArMaxRanks; ++r)
    if (r < p.world)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c < ncv) {
          const uint32_t w[4] = {a[r][c].x, a[r][c].y, a[r][c].z, a[r][c].w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            buf[c][2 * t] = __fadd_rn(buf[c][2 * t], bf16lo(w[t]));
            buf[c][2 * t + 1] = __fadd_rn(buf[c][2 * t + 1], bf16hi(w[t]));
          }
        }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      __nv_bfloat162 h2 = __floats2bfloat162_rn(buf[c][2 * t], buf[c][2 * t + 1]);
      o[t] = *reinterpret_cast<uint32_t*>(&h2);
    }
    sum[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// residual[row] := bf16(sums + residual[row]) (fp32 add); out[row] = bf16(bf16(x * rsqrt(mean(x^2)
// + eps)) * weight), x the fp32 sum: the add_rms_forward order.  `sums` points at the row's
// all-reduced bf16 values (shared memory, or the two-shot result buffer, read past L1); `zero`
// treats them as zeros (a peer wait timed out).
template <int NV>
__device__ __forceinline__ void add_rmsnorm_row(const ArParams& p, int row, const __nv_bfloat16* sums,
                                                bool from_global, bool zero) {
  const int lane = threadIdx.x & 31;
  const int64_t base = int64_t(row) * p.hidden + 8 * lane;
  float buf[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NV; ++c) {
    const uint4 rv = *reinterpret_cast<const uint4*>(p.residual + base + 256 * c);
    const uint4* sp = reinterpret_cast<const uint4*>(sums + 8 * lane + 256 * c);
    const uint4 sv = zero ? make_uint4(0, 0, 0, 0) : (from_global ? __ldcv(sp) : *sp);
    const uint32_t w[4] = {sv.x, sv.y, sv.z, sv.w};
    const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
    uint32_t ro[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      buf[c][2 * t] = __fadd_rn(bf16lo(w[t]), bf16lo(rw[t]));
      buf[c][2 * t + 1] = __fadd_rn(bf16hi(w[t]), bf16hi(rw[t]));
      __nv_bfloat162 h2 = __floats2bfloat162_rn(buf[c][2 * t], buf[c][2 * t + 1]);
      ro[t] = *reinterpret_cast<uint32_t*>(&h2);
    }
    *reinterpret_cast<uint4*>(p.residual + base + 256 * c) = make_uint4(ro[0], ro[1], ro[2], ro[3]);
#pragma unroll
    for (int t = 0; t < 8; ++t) ss = fmaf(buf[c][t], buf[c][t], ss);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / float(p.hidden) + p.eps);
#pragma unroll
  for (int c = 0; c < NV; ++c) {
    const int col = 8 * (lane + 32 * c);
    const uint4 wv = *reinterpret_cast<const uint4*>(p.weight + col);
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float a = __fmul_rn(bf16_round(__fmul_rn(buf[c][2 * t], inv)), bf16lo(ww[t]));
      const float b = __fmul_rn(bf16_round(__fmul_rn(buf[c][2 * t + 1], inv)), bf16hi(ww[t]));
      __nv_bfloat162 h2 = __floats2bfloat162_rn(a, b);
      o[t] = *reinterpret_cast<uint32_t*>(&h2);
    }
    *reinterpret_cast<uint4*>(p.out + int64_t(row) * p.out_stride + col) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// One-shot: every rank reads every rank's partial sums of all rows.  The units of a row group
// are reduced into shared memory (bf16 sums, [rows_per_cta][hidden]), then one warp per row
// applies the add + RMSNorm.
template <int NV>
__global__ void __launch_bounds__(kArThreads) ar_add_rmsnorm_kernel(const __grid_constant__ ArParams p) {
  extern __shared__ __align__(16) __nv_bfloat16 s_sums[];
  __shared__ int s_epoch;
  __shared__ int s_ok;
  const int blk = blockIdx.x;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (tid == 0) {
    s_epoch = p.epochs[blk] + 1;
    s_ok = 1;
  }
  __syncthreads();
  const int epoch = s_epoch;
  const bool ok = cta_barrier<false>(p, 0, epoch, &s_ok);
  if (tid == 0) p.epochs[blk] = epoch;

  const int rpc = rows_per_cta(p.hidden);
  const int units = (p.hidden + kUnitElems - 1) / kUnitElems;
  for (int row0 = blk * rpc; row0 < p.rows; row0 += gridDim.x * rpc) {
    const int nr = min(rpc, p.rows - row0);
    if (ok) {
      for (int w = warp; w < nr * units; w += kArThreads / 32) {
        const int rl = w / units;
        const int u = w - rl * units;
        const int ncv = min(4, (p.hidden - u * kUnitElems) / 256);
        uint4 sum[4];
        reduce_unit(p, int64_t(row0 + rl) * p.hidden + u * kUnitElems + 8 * lane, ncv, sum);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (c < ncv)
            *reinterpret_cast<uint4*>(s_sums + rl * p.hidden + u * kUnitElems + 8 * lane + 256 * c) = sum[c];
      }
    }
    __syncthreads();
    if (warp < nr) add_rmsnorm_row<NV>(p, row0 + warp, s_sums + warp * p.hidden, false, !ok);
    __syncthreads();  // the next group reuses s_sums
  }
}

// Two-shot variant for more than two ranks: each rank reduces only the rows it owns (row r is
// owned by rank r % world), reading them from every rank, and pushes the bf16 sum into every
// rank's result buffer; after a second barrier (released at system scope, because it announces
// this kernel's own remote stores) every rank reads all rows' sums from its local result buffer
// and applies the add + RMSNorm.  Per call and rank the NVLink traffic is 2 (world - 1) / world
// of the rows instead of the one-shot's (world - 1) x the rows, for one more barrier.  The sums
// are taken in rank order, as in the one-shot kernel, so both give bit-identical results.  A CTA
// works on the same row groups in both phases, so the second barrier is again between equal CTA
// indices.
template <int NV>
__global__ void __launch_bounds__(kArThreads) ar2_add_rmsnorm_kernel(const __grid_constant__ ArParams p) {
  __shared__ int s_epoch;
  __shared__ int s_ok;
  const int blk = blockIdx.x;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (tid == 0) {
    s_epoch = p.epochs[blk] + 1;
    s_ok = 1;
  }
  __syncthreads();
  const int epoch = s_epoch;
  // The partial sums were written by an earlier kernel of this stream: relaxed flags suffice.
  bool ok = cta_barrier<false>(p, 0, epoch, &s_ok);
  if (tid == 0) p.epochs[blk] = epoch;

  const int rpc = rows_per_cta(p.hidden);
  const int units = (p.hidden + kUnitElems - 1) / kUnitElems;
  // ---------------------------------------------------------------- phase 1: owned rows
  if (ok) {
    for (int row0 = blk * rpc; row0 < p.rows; row0 += gridDim.x * rpc) {
      const int nr = min(rpc, p.rows - row0);
      for (int w = warp; w < nr * units; w += kArThreads / 32) {
        const int rl = w / units;
        const int u = w - rl * units;
        const int row = row0 + rl;
        if (row % p.world != p.rank) continue;
        const int ncv = min(4, (p.hidden - u * kUnitElems) / 256);
        const int64_t off = int64_t(row) * p.hidden + u * kUnitElems + 8 * lane;
        uint4 sum[4];
        reduce_unit(p, off, ncv, sum);
        for (int r = 0; r < p.world; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (c < ncv) *reinterpret_cast<uint4*>(p.result[r] + off + 256 * c) = sum[c];
      }
    }
  }
  __syncthreads();
  ok = ok && cta_barrier<true>(p, 1, epoch, &s_ok);

  // ---------------------------------------------------------------- phase 2: add + RMSNorm
  // Sums pushed by the rows' owners in this call: read past L1.
  for (int row0 = blk * rpc; row0 < p.rows; row0 += gridDim.x * rpc) {
    const int nr = min(rpc, p.rows - row0);
    if (warp < nr) {
      const int row = row0 + warp;
      add_rmsnorm_row<NV>(p, row, p.result[p.rank] + int64_t(row) * p.hidden, true, !ok);
    }
  }
}

}  // namespace
}  // namespace hl

using namespace hl;

extern "C" int hl_device_alloc(int64_t bytes, void** ptr_out) {
  clear_error();
  HL_CHECK_ARG(bytes > 0 && ptr_out, "hl_device_alloc: bad arguments");
  cudaError_t e = cudaMalloc(ptr_out, size_t(bytes));
  if (e == cudaSuccess) e = cudaMemset(*ptr_out, 0, size_t(bytes));
  if (e != cudaSuccess) {
    set_error("hl_device_alloc: %s", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  return HL_OK;
}

extern "C" int hl_device_free(void* ptr) {
  clear_error();
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_error("hl_device_free: %s", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  return HL_OK;
}

extern "C" int hl_ipc_get_handle(void* dev_ptr, void* handle_out) {
  clear_error();
  HL_CHECK_ARG(dev_ptr && handle_out, "hl_ipc_get_handle: bad arguments");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, dev_ptr);
  if (e != cudaSuccess) {
    set_error("hl_ipc_get_handle: %s", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  return HL_OK;
}

extern "C" int hl_ipc_open_handle(const void* handle, void** dev_ptr_out) {
  clear_error();
  HL_CHECK_ARG(handle && dev_ptr_out, "hl_ipc_open_handle: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("hl_ipc_open_handle: %s", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  return HL_OK;
}

extern "C" int hl_ipc_close_handle(void* dev_ptr) {
  clear_error();
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) {
    set_error("hl_ipc_close_handle: %s", cudaGetErrorString(e));
    return HL_ERR_CUDA;
  }
  return HL_OK;
}

// Two flag banks (the two-shot kernel's second barrier uses bank 1).
extern "C" int64_t hl_allreduce_signal_bytes(void) { return int64_t(2) * kArMaxBlocks * kArMaxRanks * sizeof(int); }

namespace {
int allreduce_launch(void* const* peer_data, void* const* peer_result, void* const* peer_signal, int world, int rank,
                     int rows, int hidden, void* residual, const void* weight, void* out, int64_t out_stride,
                     float eps, int* epochs, int* error_word, int64_t timeout_ns, void* stream);
}

extern "C" int hl_allreduce_add_rmsnorm(void* const* peer_data, void* const* peer_signal, int world, int rank,
                                        int rows, int hidden, void* residual, const void* weight, void* out,
                                        int64_t out_stride, float eps, int* epochs, int* error_word,
                                        int64_t timeout_ns, void* stream) {
  clear_error();
  return allreduce_launch(peer_data, nullptr, peer_signal, world, rank, rows, hidden, residual, weight, out,
                          out_stride, eps, epochs, error_word, timeout_ns, stream);
}

extern "C" int hl_allreduce_add_rmsnorm_2shot(void* const* peer_data, void* const* peer_result,
                                              void* const* peer_signal, int world, int rank, int rows, int hidden,
                                              void* residual, const void* weight, void* out, int64_t out_stride,
                                              float eps, int* epochs, int* error_word, int64_t timeout_ns,
                                              void* stream) {
  clear_error();
  HL_CHECK_ARG(peer_result, "hl_allreduce_add_rmsnorm_2shot: result buffers missing");
  return allreduce_launch(peer_data, peer_result, peer_signal, world, rank, rows, hidden, residual, weight, out,
                          out_stride, eps, epochs, error_word, timeout_ns, stream);
}

namespace {
int allreduce_launch(void* const* peer_data, void* const* peer_result, void* const* peer_signal, int world, int rank,
                     int rows, int hidden, void* residual, const void* weight, void* out, int64_t out_stride,
                     float eps, int* epochs, int* error_word, int64_t timeout_ns, void* stream) {
  if (rows == 0) return HL_OK;
  HL_CHECK_ARG(peer_data && peer_signal && residual && weight && out && epochs && error_word && rows > 0,
               "hl_allreduce_add_rmsnorm: bad arguments");
  HL_CHECK_ARG(world >= 1 && world <= kArMaxRanks && rank >= 0 && rank < world,
               "hl_allreduce_add_rmsnorm: world must be 1..8");
  HL_CHECK_ARG(hidden % 256 == 0 && hidden <= 8192, "hl_allreduce_add_rmsnorm: hidden must be a multiple of 256, <= 8192");
  HL_CHECK_ARG(aligned16(residual) && aligned16(weight) && aligned16(out) && out_stride % 8 == 0,
               "hl_allreduce_add_rmsnorm: 16-byte alignment required");
  HL_CHECK_ARG(timeout_ns > 0, "hl_allreduce_add_rmsnorm: timeout must be positive");
  // Decode batches: the flag barrier and the row groups are per CTA, at most kArMaxBlocks CTAs.
  HL_CHECK_ARG(!peer_result || rows <= 512, "hl_allreduce_add_rmsnorm_2shot: at most 512 rows");
  ArParams prm;
  memset(&prm, 0, sizeof(prm));
  for (int r = 0; r < world; ++r) {
    HL_CHECK_ARG(peer_data[r] && peer_signal[r] && aligned16(peer_data[r]),
                 "hl_allreduce_add_rmsnorm: null or misaligned peer pointer");
    prm.data[r] = static_cast<const __nv_bfloat16*>(peer_data[r]);
    prm.signal[r] = static_cast<int*>(peer_signal[r]);
    if (peer_result) {
      HL_CHECK_ARG(peer_result[r] && aligned16(peer_result[r]), "hl_allreduce_add_rmsnorm_2shot: bad result pointer");
      prm.result[r] = static_cast<__nv_bfloat16*>(peer_result[r]);
    }
  }
  prm.world = world;
  prm.rank = rank;
  prm.rows = rows;
  prm.hidden = hidden;
  prm.residual = static_cast<__nv_bfloat16*>(residual);
  prm.weight = static_cast<const __nv_bfloat16*>(weight);
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.out_stride = out_stride;
  prm.eps = eps;
  prm.epochs = epochs;
  prm.error_word = error_word;
  prm.timeout_ns = static_cast<unsigned long long>(timeout_ns);
  const int rpc = rows_per_cta(hidden);
  const int groups = (rows + rpc - 1) / rpc;
  const int blocks = groups < kArMaxBlocks ? groups : kArMaxBlocks;
  const size_t sums_bytes = size_t(rpc) * hidden * sizeof(__nv_bfloat16);  // <= 16 KiB
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define HL_AR_CASE(NV)                                                          \
  case NV:                                                                      \
    if (peer_result)                                                            \
      ar2_add_rmsnorm_kernel<NV><<<blocks, kArThreads, 0, s>>>(prm);            \
    else                                                                        \
      ar_add_rmsnorm_kernel<NV><<<blocks, kArThreads, sums_bytes, s>>>(prm);    \
    break;
  switch (hidden / 256) {
    HL_AR_CASE(1) HL_AR_CASE(2) HL_AR_CASE(3) HL_AR_CASE(4) HL_AR_CASE(5) HL_AR_CASE(6) HL_AR_CASE(8)
    HL_AR_CASE(10) HL_AR_CASE(12) HL_AR_CASE(14) HL_AR_CASE(16) HL_AR_CASE(20) HL_AR_CASE(24) HL_AR_CASE(28)
    HL_AR_CASE(32)
    default:
      set_error("hl_allreduce_add_rmsnorm: hidden=%d not supported", hidden);
      return HL_ERR_UNSUPPORTED;
  }
#undef HL_AR_CASE
  HL_CHECK_LAUNCH("hl_allreduce_add_rmsnorm");
  return HL_OK;
}
}  // namespace
