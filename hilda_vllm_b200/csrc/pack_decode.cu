// Decode-batch packing on the GPU: rebuilds the persistent decode graph buffers
// (input_ids, positions, context_lens, slot_mapping, block-table rows) in place.
//
// Device restatement of ModelRunner.prepare_decode (mini_vllm/engine/model_runner.py:652-720)
// and its block-table row bookkeeping (:551-584).  The reference rebuilds every slot on the
// host each step and issues one host->device copy per changed block-table row; here the
// device keeps, per slot, the owning sequence id and its block-table length (the reference's
// decode_slot_seq_ids / decode_slot_block_table_lens) next to the graph buffers, and the host
// sends only the slots whose state is not "same owner, one more token":
//   - padding slot with an owner     -> row := -1, owner := -1 (_clear_decode_block_table_slot)
//   - owner changed or table shrank  -> full row rewrite, -1 padded (_copy_decode_block_table_row)
//   - table grew                     -> tail entries only (_sync_decode_block_table_row, :573-581)
//   - explicit length / token        -> scalars (new owner, or a length that is not previous+1)
// Every other slot below `batch` with an owner advances by one token and takes the token the
// sampler left in next_tokens[slot].  Per slot i < batch the outputs are exactly the
// reference's: input_ids = last token, positions = len-1, context_lens = len,
// slot_mapping = row[bt_len-1]*BS + (len-1) % BS; padding slots get 0, 0, 0, -1.  Slots in
// [batch, graph_batch) get positions 0, context_lens 0, slot_mapping -1 (:709-712).
//
// The per-step packet (header, events, block-id pool) is read from device memory, so the
// launch can sit inside the decode CUDA graph.  One CTA, one thread per slot; a slot's row
// update is a short serial loop (<= bt_stride).
#include "hl_common.cuh"

namespace hl {
namespace {

constexpr int kMaxGraphBatch = 1024;

__global__ void __launch_bounds__(kMaxGraphBatch) pack_decode_kernel(
    const uint8_t* __restrict__ packet, int64_t packet_bytes, int graph_batch, int block_size,
    int64_t* __restrict__ slot_seq_ids, int32_t* __restrict__ slot_bt_lens, const int64_t* __restrict__ next_tokens,
    int64_t* __restrict__ input_ids, int64_t* __restrict__ positions, int32_t* __restrict__ slot_mapping,
    int32_t* __restrict__ context_lens, int32_t* __restrict__ block_tables, int64_t bt_stride, int max_blocks) {
  __shared__ int ev_of_slot[kMaxGraphBatch];
  const hl_pack_header hdr = *reinterpret_cast<const hl_pack_header*>(packet);
  const int batch = hdr.batch < 0 ? 0 : (hdr.batch > graph_batch ? graph_batch : hdr.batch);
  int64_t max_events = (packet_bytes - int64_t(sizeof(hl_pack_header))) / int64_t(sizeof(hl_pack_event));
  const int num_events = hdr.num_events < 0 ? 0 : int(hdr.num_events < max_events ? hdr.num_events : max_events);
  const hl_pack_event* events = reinterpret_cast<const hl_pack_event*>(packet + sizeof(hl_pack_header));
  int64_t pool_len = 0;
  const int32_t* pool = nullptr;
  if (hdr.pool_offset >= 0 && (hdr.pool_offset & 3) == 0 && hdr.pool_offset <= packet_bytes && hdr.pool_len > 0) {
    pool = reinterpret_cast<const int32_t*>(packet + hdr.pool_offset);
    const int64_t room = (packet_bytes - hdr.pool_offset) / 4;
    pool_len = hdr.pool_len < room ? hdr.pool_len : room;
  }

  const int i = threadIdx.x;
  ev_of_slot[i] = -1;
  __syncthreads();
  for (int e = i; e < num_events; e += blockDim.x) {
    const int s = events[e].slot;
    if (s >= 0 && s < batch) ev_of_slot[s] = e;
  }
  __syncthreads();
  if (i >= graph_batch) return;
  if (i >= batch) {
    positions[i] = 0;
    context_lens[i] = 0;
    slot_mapping[i] = -1;
    return;
  }

  int32_t* row = block_tables + int64_t(i) * bt_stride;
  bool have_scalars = false;
  int32_t ctx = 0;
  int64_t token = 0;
  const int e = ev_of_slot[i];
  if (e >= 0) {
    const hl_pack_event ev = events[e];
    if (ev.flags & HL_EV_CLEAR) {
      for (int k = 0; k < max_blocks; ++k) row[k] = -1;
      slot_seq_ids[i] = -1;
      slot_bt_lens[i] = 0;
    }
    if (ev.flags & HL_EV_ROW) {
      const int start = ev.row_start < 0 ? 0 : ev.row_start;
      for (int k = 0; k < ev.row_count; ++k) {
        const int idx = start + k;
        const int64_t src = int64_t(ev.pool_off) + k;
        if (idx < max_blocks && src >= 0 && src < pool_len) row[idx] = pool[src];
      }
      if (ev.flags & HL_EV_ROW_FILL)
        for (int k = start + ev.row_count; k < max_blocks; ++k) row[k] = -1;
      slot_bt_lens[i] = ev.bt_len;
    }
    if (ev.flags & HL_EV_SCALARS) {
      have_scalars = true;
      ctx = ev.ctx_len;
      token = ev.token;
      slot_seq_ids[i] = ev.seq_id;
      slot_bt_lens[i] = ev.bt_len;
    }
  }
  if (!have_scalars) {
    if (slot_seq_ids[i] == -1) {  // padding slot
      input_ids[i] = 0;
      positions[i] = 0;
      context_lens[i] = 0;
      slot_mapping[i] = -1;
      return;
    }
    ctx = context_lens[i] + 1;  // continuing sequence: one token appended since last step
    token = next_tokens[i];
  }
  input_ids[i] = token;
  positions[i] = ctx - 1;
  context_lens[i] = ctx;
  const int bt_len = slot_bt_lens[i];
  int32_t sm = -1;
  if (bt_len > 0 && bt_len <= max_blocks && ctx > 0) {
    const int32_t last = row[bt_len - 1];
    sm = last * block_size + (ctx - 1) % block_size;
  }
  slot_mapping[i] = sm;
}

}  // namespace
}  // namespace hl

using namespace hl;

extern "C" int hl_pack_decode_batch(const void* packet, int64_t packet_bytes, int graph_batch, int block_size,
                                    int64_t* slot_seq_ids, int32_t* slot_bt_lens, const int64_t* next_tokens,
                                    int64_t* input_ids, int64_t* positions, int32_t* slot_mapping,
                                    int32_t* context_lens, int32_t* block_tables, int64_t bt_stride,
                                    int max_blocks_per_seq, void* stream) {
  clear_error();
  HL_CHECK_ARG(graph_batch >= 0 && graph_batch <= kMaxGraphBatch, "hl_pack_decode_batch: graph_batch not in [0, %d]",
               kMaxGraphBatch);
  if (graph_batch == 0) return HL_OK;
  HL_CHECK_ARG(packet && packet_bytes >= int64_t(sizeof(hl_pack_header)) && aligned16(packet),
               "hl_pack_decode_batch: packet must be a 16-byte aligned buffer of >= 16 bytes");
  HL_CHECK_ARG(slot_seq_ids && slot_bt_lens && next_tokens && input_ids && positions && slot_mapping &&
                   context_lens && block_tables,
               "hl_pack_decode_batch: null pointer");
  HL_CHECK_ARG(block_size > 0 && max_blocks_per_seq > 0 && bt_stride >= max_blocks_per_seq,
               "hl_pack_decode_batch: bad block table shape");
  pack_decode_kernel<<<1, kMaxGraphBatch, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(packet), packet_bytes, graph_batch, block_size, slot_seq_ids, slot_bt_lens,
      next_tokens, input_ids, positions, slot_mapping, context_lens, block_tables, bt_stride, max_blocks_per_seq);
  HL_CHECK_LAUNCH("hl_pack_decode_batch");
  return HL_OK;
}
