"""Decode-batch packing restatements (TEST ORACLE ONLY).

ReferenceDecodeBuffers restates ModelRunner.prepare_decode and its block-table row bookkeeping
(mini_vllm/engine/model_runner.py:504-584 and :652-720) on numpy arrays: the persistent graph
buffers input_ids / positions / slot_mapping / context_lens / block_tables plus the per-slot
(seq_id, block-table length) record that decides between a full row copy, a tail copy and a
clear.  tests/golden/ pins it against the reference's own ModelRunner methods.

apply_packet restates what hl_pack_decode_batch does with a packet (header, events, block-id
pool) on the device state, so the host packet builder can be checked on the CPU.
"""
from __future__ import annotations

import numpy as np

EV_SCALARS, EV_ROW, EV_ROW_FILL, EV_CLEAR = 1, 2, 4, 8


class ReferenceDecodeBuffers:

    def __init__(self, max_bs: int, max_blocks: int, block_size: int):
        self.block_size = block_size
        self.max_blocks = max_blocks
        self.input_ids = np.zeros(max_bs, np.int64)
        self.positions = np.zeros(max_bs, np.int64)
        self.slot_mapping = np.full(max_bs, -1, np.int32)   # model_runner.py:527
        self.context_lens = np.zeros(max_bs, np.int32)      # :528
        self.block_tables = np.full((max_bs, max_blocks), -1, np.int32)  # :529
        self.slot_seq_ids = [-1] * max_bs                   # :522
        self.slot_bt_lens = [0] * max_bs                    # :523

    def _clear(self, i):  # :551-556
        if self.slot_seq_ids[i] == -1 and self.slot_bt_lens[i] == 0:
            return
        self.block_tables[i].fill(-1)
        self.slot_seq_ids[i] = -1
        self.slot_bt_lens[i] = 0

    def _sync_row(self, i, seq_id, table):  # :565-584
        n = len(table)
        prev_id, prev_n = self.slot_seq_ids[i], self.slot_bt_lens[i]
        if prev_id != seq_id or n < prev_n:
            self.block_tables[i].fill(-1)
            self.block_tables[i, :n] = table
        elif n > prev_n:
            self.block_tables[i, prev_n:n] = table[prev_n:n]
        self.slot_seq_ids[i] = seq_id
        self.slot_bt_lens[i] = n

    def prepare(self, rows, graph_bs: int):
        """rows: one entry per scheduled slot, None for padding or a tuple
        (seq_id, num_tokens, last_token, block_table, waiting)."""
        bs = len(rows)
        ids = np.zeros(bs, np.int64)
        pos = np.zeros(bs, np.int64)
        ctx = np.zeros(bs, np.int32)
        sm = np.full(bs, -1, np.int32)
        for i, row in enumerate(rows):
            if row is None or row[4]:
                self._clear(i)
                continue
            seq_id, n_tok, last, table, _ = row
            n_blocks = -(-n_tok // self.block_size)
            ids[i] = last
            pos[i] = n_tok - 1
            ctx[i] = n_tok
            sm[i] = table[-1] * self.block_size + (n_tok - (n_blocks - 1) * self.block_size) - 1
            self._sync_row(i, seq_id, table)
        self.input_ids[:bs] = ids
        self.positions[:bs] = pos
        self.context_lens[:bs] = ctx
        self.slot_mapping[:bs] = sm
        if graph_bs > bs:  # :709-712
            self.positions[bs:graph_bs] = 0
            self.context_lens[bs:graph_bs] = 0
            self.slot_mapping[bs:graph_bs] = -1

    def snapshot(self, n: int) -> dict[str, np.ndarray]:
        return {"input_ids": self.input_ids[:n].copy(), "positions": self.positions[:n].copy(),
                "slot_mapping": self.slot_mapping[:n].copy(), "context_lens": self.context_lens[:n].copy(),
                "block_tables": self.block_tables[:n].copy()}


class DeviceDecodeState:
    """The device buffers hl_pack_decode_batch reads and writes."""

    def __init__(self, max_bs: int, max_blocks: int, block_size: int):
        self.block_size = block_size
        self.max_blocks = max_blocks
        self.input_ids = np.zeros(max_bs, np.int64)
        self.positions = np.zeros(max_bs, np.int64)
        self.slot_mapping = np.full(max_bs, -1, np.int32)
        self.context_lens = np.zeros(max_bs, np.int32)
        self.block_tables = np.full((max_bs, max_blocks), -1, np.int32)
        self.slot_seq_ids = np.full(max_bs, -1, np.int64)
        self.slot_bt_lens = np.zeros(max_bs, np.int32)
        self.next_tokens = np.zeros(max_bs, np.int64)

    def snapshot(self, n: int) -> dict[str, np.ndarray]:
        return {"input_ids": self.input_ids[:n].copy(), "positions": self.positions[:n].copy(),
                "slot_mapping": self.slot_mapping[:n].copy(), "context_lens": self.context_lens[:n].copy(),
                "block_tables": self.block_tables[:n].copy()}


HEADER = np.dtype([("num_events", "<i4"), ("batch", "<i4"), ("pool_offset", "<i4"), ("pool_len", "<i4")])
EVENT = np.dtype([("flags", "<i4"), ("slot", "<i4"), ("ctx_len", "<i4"), ("bt_len", "<i4"), ("seq_id", "<i8"),
                  ("token", "<i8"), ("row_start", "<i4"), ("row_count", "<i4"), ("pool_off", "<i4"),
                  ("reserved", "<i4")])


def apply_packet(st: DeviceDecodeState, packet: np.ndarray, graph_bs: int) -> None:
    hdr = packet[:16].view(HEADER)[0]
    batch = min(max(int(hdr["batch"]), 0), graph_bs)
    ne = int(hdr["num_events"])
    events = packet[16:16 + ne * EVENT.itemsize].view(EVENT)
    pool = packet[int(hdr["pool_offset"]):int(hdr["pool_offset"]) + 4 * int(hdr["pool_len"])].view(np.int32)
    ev_of = {}
    for e, ev in enumerate(events):
        if 0 <= ev["slot"] < batch:
            ev_of[int(ev["slot"])] = ev
    for i in range(graph_bs):
        if i >= batch:
            st.positions[i] = 0
            st.context_lens[i] = 0
            st.slot_mapping[i] = -1
            continue
        have = False
        ev = ev_of.get(i)
        if ev is not None:
            if ev["flags"] & EV_CLEAR:
                st.block_tables[i].fill(-1)
                st.slot_seq_ids[i] = -1
                st.slot_bt_lens[i] = 0
            if ev["flags"] & EV_ROW:
                start = max(int(ev["row_start"]), 0)
                for k in range(int(ev["row_count"])):
                    if start + k < st.max_blocks:
                        st.block_tables[i, start + k] = pool[int(ev["pool_off"]) + k]
                if ev["flags"] & EV_ROW_FILL:
                    st.block_tables[i, start + int(ev["row_count"]):] = -1
                st.slot_bt_lens[i] = ev["bt_len"]
            if ev["flags"] & EV_SCALARS:
                have = True
                ctx, tok = int(ev["ctx_len"]), int(ev["token"])
                st.slot_seq_ids[i] = ev["seq_id"]
                st.slot_bt_lens[i] = ev["bt_len"]
        if not have:
            if st.slot_seq_ids[i] == -1:
                st.input_ids[i] = 0
                st.positions[i] = 0
                st.context_lens[i] = 0
                st.slot_mapping[i] = -1
                continue
            ctx, tok = int(st.context_lens[i]) + 1, int(st.next_tokens[i])
        st.input_ids[i] = tok
        st.positions[i] = ctx - 1
        st.context_lens[i] = ctx
        n = int(st.slot_bt_lens[i])
        st.slot_mapping[i] = (st.block_tables[i, n - 1] * st.block_size + (ctx - 1) % st.block_size
                              if 0 < n <= st.max_blocks and ctx > 0 else -1)
