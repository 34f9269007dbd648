"""Continuous-batching scheduler with a persistent, compacted decode batch.

Decisions are those of mini_vllm/engine/scheduler.py:30-362, step for step, so block ids,
decode-slot indices and compaction moves are identical to the reference's:
  - a sequence that finishes prefill takes the lowest free decode slot (min-heap);
  - when a slot is freed, the last occupied slot above it moves into the hole and the
    vacated index returns to the heap; the batch high-water mark then shrinks over trailing
    empty slots (this is the "dense slot compaction" the GPU pack kernel replays);
  - prefill is chunked with an adaptive limit under decode pressure and tile-aligned chunks;
  - decode is preferred right after a prefill step when the running set is >= half full;
  - on KV exhaustion the longest other running sequence is preempted.
"""
import heapq
import os
from collections import deque
from dataclasses import dataclass

from hilda_vllm_b200.engine.block_manager import BlockManager
from hilda_vllm_b200.engine.sequence import PLACEHOLDER, Sequence, SequenceStatus


@dataclass
class ScheduledSequence:
    seq: Sequence | None  # None = padding slot
    token_chunk_size: int
    slot_index: int = -1

    @property
    def is_padding(self):
        return self.seq is None

    @property
    def num_computed_tokens_after(self):
        return self.seq.num_computed_tokens + self.token_chunk_size

    @property
    def requires_sampling(self):
        return self.num_computed_tokens_after >= len(self.seq)


class Scheduler:

    def __init__(self, config):
        Sequence.block_size = config.kvcache_block_size
        self.max_num_seqs = config.max_num_seqs
        self.max_num_batched_tokens = config.max_num_batched_tokens
        self.eos = config.eos
        self.drop_preempted_decode_token = bool(getattr(config, "drop_preempted_decode_token", False))
        self.unblock_prefill_head = bool(getattr(config, "unblock_prefill_head", True))
        self.enable_chunked_prefill = config.enable_chunked_prefill
        self.chunked_prefill_size = config.chunked_prefill_size
        self.chunked_prefill_min_size = config.chunked_prefill_min_size
        self.chunked_prefill_tile_size = config.chunked_prefill_tile_size
        self.block_manager = BlockManager(config.num_kvcache_blocks, config.kvcache_block_size)
        self.waiting: deque[Sequence] = deque()
        self.running: set[Sequence] = set()
        self.last_step_was_prefill = False
        self.decode_slots: list[Sequence | None] = [None] * self.max_num_seqs
        self.free_slot_indices: list[int] = list(range(self.max_num_seqs))
        self.persistent_batch_size = 0
        self.debug_persistent_batching = os.getenv("HILDA_DEBUG_PB", "0") == "1"
        self.debug_prefill = os.getenv("HILDA_DEBUG_PREFILL", "0") == "1"
        self.reset_diagnostics()

    def is_finished(self):
        return not self.waiting and not self.running

    def reset_diagnostics(self):
        self.prefill_allocation_blocked_steps = 0
        self.prefill_no_schedulable_steps = 0
        self.min_free_blocks_observed = len(self.block_manager.free_block_ids)

    def get_diagnostics(self):
        bm = self.block_manager
        return {
            "prefill_allocation_blocked_steps": self.prefill_allocation_blocked_steps,
            "prefill_no_schedulable_steps": self.prefill_no_schedulable_steps,
            "min_free_blocks_observed": self.min_free_blocks_observed,
            "kv_num_blocks": len(bm.blocks),
            "kv_free_blocks": len(bm.free_block_ids),
            "kv_used_blocks": len(bm.used_block_ids),
        }

    def add(self, seq: Sequence):
        self.waiting.append(seq)

    # ------------------------------------------------------------------ decode slots
    def _assign_decode_slot(self, seq: Sequence):
        idx = heapq.heappop(self.free_slot_indices)
        self.decode_slots[idx] = seq
        seq.decode_slot_index = idx
        self.persistent_batch_size = max(self.persistent_batch_size, idx + 1)

    def _free_decode_slot(self, seq: Sequence):
        hole = seq.decode_slot_index
        if hole < 0:
            return
        tail = self.persistent_batch_size - 1
        while tail > hole and self.decode_slots[tail] is None:
            tail -= 1
        if tail > hole:
            mover = self.decode_slots[tail]
            assert mover is not None
            self.decode_slots[hole] = mover
            mover.decode_slot_index = hole
            self.decode_slots[tail] = None
            heapq.heappush(self.free_slot_indices, tail)
        else:
            self.decode_slots[hole] = None
            heapq.heappush(self.free_slot_indices, hole)
        seq.decode_slot_index = -1

    def _maybe_shrink_batch(self):
        while self.persistent_batch_size > 0 and self.decode_slots[self.persistent_batch_size - 1] is None:
            self.persistent_batch_size -= 1
        if not self.running:
            assert all(slot is None for slot in self.decode_slots)
            self.persistent_batch_size = 0
            self.free_slot_indices = list(range(self.max_num_seqs))

    # ------------------------------------------------------------------ chunking
    def _compute_chunk_limit(self):
        if not self.enable_chunked_prefill or not self.running:
            return self.max_num_batched_tokens
        pressure = len(self.running) / max(1, self.max_num_seqs)
        limit = self.chunked_prefill_size
        if pressure >= 0.75:
            limit = max(self.chunked_prefill_min_size, limit // 4)
        elif pressure >= 0.5:
            limit = max(self.chunked_prefill_min_size, limit // 2)
        return min(limit, self.max_num_batched_tokens)

    def _align_chunk_size(self, chunk_size: int, remaining_tokens: int):
        if not self.enable_chunked_prefill:
            return chunk_size
        if remaining_tokens <= chunk_size:
            return remaining_tokens
        tile = self.chunked_prefill_tile_size
        if chunk_size <= tile:
            return chunk_size
        aligned = (chunk_size // tile) * tile
        return aligned if aligned > 0 else chunk_size

    # ------------------------------------------------------------------ scheduling
    def _schedule_prefill(self, skip_blocked: bool = False) -> list[ScheduledSequence]:
        """skip_blocked: a sequence that cannot get its blocks is passed over instead of ending the
        scan, so sequences behind it that already hold blocks (chunked prefills in progress) can run."""
        out: list[ScheduledSequence] = []
        admitted = 0
        active = len(self.running)
        batched = 0
        limit = self._compute_chunk_limit()
        self.min_free_blocks_observed = min(self.min_free_blocks_observed, len(self.block_manager.free_block_ids))
        for seq in list(self.waiting):
            if active + admitted >= self.max_num_seqs:
                break
            if not seq.block_table:
                if not self.block_manager.can_allocate(seq):
                    self.prefill_allocation_blocked_steps += 1
                    if self.debug_prefill:
                        print(f"[PREFILL] blocked on allocation: seq_id={seq.seq_id} len={len(seq)} "
                              f"free_blocks={len(self.block_manager.free_block_ids)} required_blocks={seq.num_blocks}")
                    if skip_blocked:
                        continue
                    break
                self.block_manager.allocate(seq)
                seq.num_computed_tokens = seq.num_cached_tokens
            remaining = seq.num_uncomputed_tokens
            if remaining <= 0:
                self._append_waiting(seq)
                continue
            available = min(limit, self.max_num_batched_tokens - batched)
            if available <= 0:
                break
            chunk = self._align_chunk_size(min(remaining, available), remaining)
            if chunk <= 0:
                self._append_waiting(seq)
                continue
            admitted += 1
            batched += chunk
            self.block_manager.mark_computed(seq, seq.num_computed_tokens + chunk)
            out.append(ScheduledSequence(seq, chunk))
        return out

    def _schedule_decode(self) -> list[ScheduledSequence]:
        if self.persistent_batch_size == 0:
            return []
        out: list[ScheduledSequence] = []
        any_real = False
        bm = self.block_manager
        for i in range(self.persistent_batch_size):
            seq = self.decode_slots[i]
            if seq is None:
                out.append(ScheduledSequence(None, 0, slot_index=i))
                continue
            if not seq.block_table:
                self.preempt(seq)
                out.append(ScheduledSequence(None, 0, slot_index=i))
                continue
            if not bm.can_append(seq):
                victim = self._find_preempt_victim(exclude=seq)
                if victim is not None:
                    self.preempt(victim)
                if not bm.can_append(seq):
                    self.preempt(seq)
                    out.append(ScheduledSequence(None, 0, slot_index=i))
                    continue
            bm.may_append(seq)
            out.append(ScheduledSequence(seq, 1, slot_index=i))
            any_real = True
        return out if any_real else []

    def _find_preempt_victim(self, exclude: Sequence | None = None) -> Sequence | None:
        best = None
        for seq in self.running:
            if seq is exclude:
                continue
            if best is None or len(seq) > len(best):
                best = seq
        return best

    def schedule(self) -> tuple[list[ScheduledSequence], bool]:
        pressure = len(self.running) / max(1, self.max_num_seqs)
        prefer_decode = (self.enable_chunked_prefill and self.running and self.waiting
                         and self.last_step_was_prefill and pressure >= 0.5)
        if prefer_decode:
            scheduled = self._schedule_decode()
            if scheduled:
                self.last_step_was_prefill = False
                return scheduled, False
        scheduled = self._schedule_prefill()
        if scheduled:
            self.last_step_was_prefill = True
            return scheduled, True
        if self.waiting:
            self.prefill_no_schedulable_steps += 1
        scheduled = self._schedule_decode()
        if not scheduled and self.waiting and self.unblock_prefill_head:
            # The head of the queue cannot get its blocks while nothing runs, but chunked prefills
            # further back hold theirs: the reference stops here (the error below); let those
            # finish instead, which frees blocks for the head once they complete.
            scheduled = self._schedule_prefill(skip_blocked=True)
            if scheduled:
                self.last_step_was_prefill = True
                return scheduled, True
        if not scheduled:
            raise RuntimeError("scheduler found no runnable prefill or decode work: "
                               f"running={len(self.running)} waiting={len(self.waiting)} "
                               f"persistent_batch_size={self.persistent_batch_size}")
        self.last_step_was_prefill = False
        return scheduled, False

    def preempt(self, seq: Sequence):
        seq.status = SequenceStatus.WAITING
        self.block_manager.deallocate(seq)
        seq.num_computed_tokens = 0
        self.running.discard(seq)
        self._free_decode_slot(seq)
        self._maybe_shrink_batch()
        self.waiting.appendleft(seq)

    def _append_waiting(self, seq: Sequence):
        self.waiting.remove(seq)
        self.waiting.append(seq)

    def _finish(self, seq: Sequence):
        seq.status = SequenceStatus.FINISHED
        self.block_manager.deallocate(seq)
        self.running.discard(seq)
        self._free_decode_slot(seq)

    def _is_done(self, seq: Sequence, token_id: int) -> bool:
        return (not seq.ignore_eos and token_id == self.eos) or seq.num_completion_tokens == seq.max_tokens

    def _skip_row(self, sched: ScheduledSequence) -> bool:
        """Rows of a decode batch whose token is not appended.  A sequence preempted as a victim
        after it was put in the batch is WAITING: the decode buffers treat it as padding, so its
        row's token is not its own; the reference appends it anyway (scheduler.py:326-340), and so
        does this scheduler unless config.drop_preempted_decode_token is set."""
        if sched.is_padding:
            return True
        return self.drop_preempted_decode_token and sched.seq.status == SequenceStatus.WAITING

    # ------------------------------------------------------------------ overlapped decode
    # A decode step whose sampled tokens stay on the GPU until the next step has been launched.
    # Used only while no running sequence can stop on EOS, so every stop is known from lengths
    # alone and reading the tokens back later never changes a scheduling decision.
    def eos_cannot_stop(self) -> bool:
        return self.eos < 0 or all(seq.ignore_eos for seq in self.running)

    def postprocess_launched(self, seqs: list[ScheduledSequence]) -> tuple[list[tuple[Sequence, int, int]],
                                                                          list[Sequence]]:
        """postprocess() for a launched decode step whose tokens are not read yet: each real
        sequence gets a PLACEHOLDER token and sequences reaching max_tokens finish now.
        Returns the (sequence, token position, batch row) triples to fill later and the
        finished sequences."""
        pending: list[tuple[Sequence, int, int]] = []
        finished: list[Sequence] = []
        for slot, sched in enumerate(seqs):
            if self._skip_row(sched):
                continue
            seq = sched.seq
            seq.num_computed_tokens += 1
            pending.append((seq, seq.num_tokens, slot))
            seq.append_token(PLACEHOLDER)
            if seq.num_completion_tokens == seq.max_tokens:
                self._finish(seq)
                finished.append(seq)
        self._maybe_shrink_batch()
        return pending, finished

    def resolve_tokens(self, pending: list[tuple[Sequence, int, int]], token_ids: list[int]) -> None:
        """Fills the placeholders of a launched step with the tokens read back from the GPU
        (token_ids: one per batch row)."""
        for seq, pos, row in pending:
            tok = token_ids[row]
            assert seq.token_ids[pos] == PLACEHOLDER
            seq.token_ids[pos] = tok
            if pos == seq.num_tokens - 1:
                seq.last_token = tok
        self.block_manager.resolve_deferred()

    def postprocess(self, seqs: list[ScheduledSequence], token_ids: list[int | None], is_prefill: bool):
        if not is_prefill:
            for sched, token_id in zip(seqs, token_ids):
                if self._skip_row(sched):
                    continue
                seq = sched.seq
                assert token_id is not None
                seq.num_computed_tokens += 1
                seq.append_token(token_id)
                if self._is_done(seq, token_id):
                    self._finish(seq)
            self._maybe_shrink_batch()
            return

        for sched, token_id in zip(seqs, token_ids):
            seq = sched.seq
            reached_end = seq.num_computed_tokens + sched.token_chunk_size >= len(seq)
            seq.num_computed_tokens = min(len(seq), seq.num_computed_tokens + sched.token_chunk_size)
            if not reached_end:
                self._append_waiting(seq)
                continue
            self.waiting.remove(seq)
            seq.status = SequenceStatus.RUNNING
            self._assign_decode_slot(seq)
            self.running.add(seq)
            assert token_id is not None
            seq.append_token(token_id)
            if self._is_done(seq, token_id):
                self._finish(seq)
                self._maybe_shrink_batch()
