"""Host side of the GPU decode-batch packing (hl_pack_decode_batch).

The reference rebuilds the persistent decode batch on the host every step
(ModelRunner.prepare_decode, mini_vllm/engine/model_runner.py:652-720: one Python loop over all
slots writing five pinned staging tensors, plus a host->device copy per changed block-table
row, :551-584).  Here the device keeps that state itself, and this class keeps a mirror of
what the device holds, so that each step it only emits events for slots whose state is not
"same sequence, one more token":

  padding slot that still has an owner      -> CLEAR             (_clear_decode_block_table_slot)
  new owner, or block table shrank          -> ROW|ROW_FILL      (_copy_decode_block_table_row)
  same owner, block table grew              -> ROW (tail only)   (_sync_decode_block_table_row)
  new owner / length not previous+1 / token the device does not hold -> SCALARS

The device holds slot i's input token when the previous step sampled it there: either the host
read it back (note_sampled) or the step was launched without reading it yet (note_launched,
overlapped decode), in which case the host's copy of the sequence ends with PLACEHOLDER.

Everything is serialised into one packet (header, events, block-id pool) that the runner
copies to the device with a single host->device copy.  The block-table decisions are the
reference's, so the device buffers end up bit-identical to the reference's graph buffers.
"""
from __future__ import annotations

import numpy as np

from hilda_vllm_b200.engine.sequence import PLACEHOLDER, SequenceStatus

EV_SCALARS = 1
EV_ROW = 2
EV_ROW_FILL = 4
EV_CLEAR = 8

HEADER_DTYPE = np.dtype([("num_events", "<i4"), ("batch", "<i4"), ("pool_offset", "<i4"), ("pool_len", "<i4")])
EVENT_DTYPE = np.dtype([
    ("flags", "<i4"), ("slot", "<i4"), ("ctx_len", "<i4"), ("bt_len", "<i4"),
    ("seq_id", "<i8"), ("token", "<i8"),
    ("row_start", "<i4"), ("row_count", "<i4"), ("pool_off", "<i4"), ("reserved", "<i4"),
])
assert HEADER_DTYPE.itemsize == 16 and EVENT_DTYPE.itemsize == 48

_UNKNOWN = object()


def packet_capacity_bytes(max_bs: int, max_blocks: int) -> int:
    """Worst case: one full-row event per slot."""
    return HEADER_DTYPE.itemsize + max_bs * EVENT_DTYPE.itemsize + max_bs * max_blocks * 4 + 16


class DecodePacker:
    """Builds decode packets and mirrors the device's per-slot state."""

    def __init__(self, max_bs: int, max_blocks: int, buffer: np.ndarray | None = None):
        self.max_bs = max_bs
        self.max_blocks = max_blocks
        self.capacity = packet_capacity_bytes(max_bs, max_blocks)
        if buffer is None:
            buffer = np.zeros(self.capacity, dtype=np.uint8)
        assert buffer.dtype == np.uint8 and buffer.size >= self.capacity
        self.buffer = buffer
        self.owner = [-1] * max_bs       # slot_seq_ids on the device
        self.bt_len = [0] * max_bs       # slot_bt_lens on the device
        self.ctx = [0] * max_bs          # context_lens on the device
        self.token: list[object] = [_UNKNOWN] * max_bs  # next_tokens on the device
        self.last_num_events = 0

    def note_sampled(self, batch: int, tokens: list[int]) -> None:
        """Records that the device's next_tokens[0:batch] now hold `tokens` and that rows
        beyond batch hold unknown values."""
        for i in range(batch):
            self.token[i] = tokens[i]
        for i in range(batch, self.max_bs):
            self.token[i] = _UNKNOWN

    def forget_tokens(self) -> None:
        self.token = [_UNKNOWN] * self.max_bs

    def note_launched(self, batch: int, scheduled_seqs) -> None:
        """Records that a decode step was launched whose sampled tokens stay on the device: slot
        i's next_tokens then holds the token at position len(seq) of the sequence it ran (the host
        learns its value later)."""
        for i in range(batch):
            seq = scheduled_seqs[i].seq
            self.token[i] = _UNKNOWN if seq is None else ("dev", seq.seq_id, seq.num_tokens)
        for i in range(batch, self.max_bs):
            self.token[i] = _UNKNOWN

    def _device_holds(self, i: int, seq) -> bool:
        tok = self.token[i]
        if isinstance(tok, tuple):
            return tok == ("dev", seq.seq_id, seq.num_tokens - 1)
        return tok is not _UNKNOWN and seq.last_token != PLACEHOLDER and tok == seq.last_token

    def needs_host_tokens(self, scheduled_seqs) -> bool:
        """True when building this step's packet would need a token the host has not read back
        yet (a sequence whose last token is still on the GPU, in another slot or for an earlier
        owner of its slot).  build() must not be called then."""
        for i, sched in enumerate(scheduled_seqs):
            seq = sched.seq
            if seq is None or seq.status == SequenceStatus.WAITING or seq.last_token != PLACEHOLDER:
                continue
            if self.owner[i] != seq.seq_id or self.ctx[i] + 1 != seq.num_tokens or not self._device_holds(i, seq):
                return True
        return False

    def build(self, scheduled_seqs, graph_bs: int) -> int:
        """Serialises the packet for this step into self.buffer; returns its size in bytes."""
        bs = len(scheduled_seqs)
        assert bs <= graph_bs <= self.max_bs
        events: list[tuple] = []
        pool: list[int] = []
        owner, bt_len, ctx, token = self.owner, self.bt_len, self.ctx, self.token
        for i, sched in enumerate(scheduled_seqs):
            slot = sched.slot_index if sched.slot_index >= 0 else i
            assert slot == i, "decode scheduling is expected to follow slot order"
            seq = sched.seq
            if seq is None or seq.status == SequenceStatus.WAITING:
                if owner[i] != -1 or bt_len[i] != 0:
                    events.append((EV_CLEAR, i, 0, 0, -1, 0, 0, 0, 0, 0))
                    owner[i] = -1
                    bt_len[i] = 0
                ctx[i] = 0
                continue
            table = seq.block_table
            if not table:
                raise RuntimeError(
                    f"decode sequence has empty block_table: seq_id={seq.seq_id}, status={seq.status}, "
                    f"num_tokens={seq.num_tokens}, num_computed_tokens={seq.num_computed_tokens}, slot_index={i}")
            n = len(table)
            length = seq.num_tokens
            flags = 0
            row_start = row_count = pool_off = 0
            same_owner = owner[i] == seq.seq_id
            if not same_owner or n < bt_len[i]:
                flags = EV_ROW | EV_ROW_FILL
                row_count = n
                pool_off = len(pool)
                pool.extend(table)
            elif n > bt_len[i]:
                flags = EV_ROW
                row_start = bt_len[i]
                row_count = n - row_start
                pool_off = len(pool)
                pool.extend(table[row_start:])
            if not same_owner or ctx[i] + 1 != length or not self._device_holds(i, seq):
                if seq.last_token == PLACEHOLDER:
                    raise RuntimeError("decode packet needs a token that is still on the GPU")
                flags |= EV_SCALARS
            if flags:
                events.append((flags, i, length, n, seq.seq_id, seq.last_token, row_start, row_count, pool_off, 0))
            owner[i] = seq.seq_id
            bt_len[i] = n
            ctx[i] = length
        for i in range(bs, graph_bs):
            ctx[i] = 0
        return self._serialise(events, pool, bs)

    def _serialise(self, events: list[tuple], pool: list[int], bs: int) -> int:
        buf = self.buffer
        ne = len(events)
        ev_bytes = ne * EVENT_DTYPE.itemsize
        pool_offset = HEADER_DTYPE.itemsize + ev_bytes
        total = pool_offset + 4 * len(pool)
        if total > self.capacity:
            raise RuntimeError("decode packet exceeds its buffer")
        hdr = buf[: HEADER_DTYPE.itemsize].view(HEADER_DTYPE)
        hdr[0] = (ne, bs, pool_offset, len(pool))
        if ne:
            buf[HEADER_DTYPE.itemsize:pool_offset].view(EVENT_DTYPE)[:] = events
        if pool:
            buf[pool_offset:total].view(np.int32)[:] = pool
        self.last_num_events = ne
        # Round up to 16 bytes so copies stay vector-aligned.
        return (total + 15) & ~15
