"""Paged KV block allocator with a chained-hash prefix cache.

Behaviour (and therefore every block id it hands out) is that of
mini_vllm/engine/block_manager.py:8-115: blocks are taken from the head of a FIFO free list,
freed blocks go to its tail, a full block's hash is xxh64(previous block hash as 8
little-endian bytes || token ids as int64 bytes), and a cached block is reused only when its
stored token ids equal the request's.

One departure, in what a reused block counts for: the reference registers a block's hash when
the block is allocated, before any of its KV rows exist, and counts every hit as computed
(block_manager.py:58-80, then scheduler.py:184 starts the prefill after the hits).  With chunked
prefill the owner may not have reached that block yet, so a second sequence with the same prefix
would start its prefill after rows nobody has written.  Here each block records whether its rows
are written (or are written by a chunk scheduled earlier in the same step: the KV store of a step
runs before its attention in every layer); hits still share the same block ids, but
num_cached_tokens only counts the leading run of written blocks, and the sequence computes the
rest itself, into the shared blocks.
"""
from collections import deque

import numpy as np
import xxhash

from hilda_vllm_b200.engine.sequence import PLACEHOLDER, Sequence


class Block:

    def __init__(self, block_id: int):
        self.block_id = block_id
        self.ref_count = 0
        self.hash = -1
        self.token_ids: list[int] = []
        self.computed = False  # every row of the block is written (or scheduled to be, this step)

    def update(self, hash: int, token_ids: list[int]):
        self.hash = hash
        self.token_ids = token_ids

    def reset(self):
        self.ref_count = 1
        self.hash = -1
        self.token_ids = []
        self.computed = False


class BlockManager:

    def __init__(self, num_blocks: int, block_size: int, count_unwritten_hits: bool = False):
        self.block_size = block_size
        # True reproduces the reference: every hit counts as computed, written or not.
        self.count_unwritten_hits = count_unwritten_hits
        self.unwritten_hits = 0  # hits that were not counted (diagnostics)
        self.blocks: list[Block] = [Block(i) for i in range(num_blocks)]
        self.hash_to_block_id: dict[int, int] = {}
        self.deferred_hashes: list[tuple] = []  # (seq, page index, block id)
        self.free_block_ids: deque[int] = deque(range(num_blocks))
        self.used_block_ids: set[int] = set()

    @classmethod
    def compute_hash(cls, token_ids: list[int], prefix: int = -1) -> int:
        hasher = xxhash.xxh64()
        if prefix != -1:
            hasher.update(prefix.to_bytes(8, "little"))
        hasher.update(np.asarray(token_ids, dtype=np.int64).tobytes())
        return hasher.intdigest()

    def _allocate_block(self, block_id: int) -> Block:
        block = self.blocks[block_id]
        assert block.ref_count == 0
        block.reset()
        self.free_block_ids.remove(block_id)
        self.used_block_ids.add(block_id)
        return block

    def _deallocate_block(self, block_id: int) -> None:
        assert self.blocks[block_id].ref_count == 0
        self.used_block_ids.remove(block_id)
        self.free_block_ids.append(block_id)

    def can_allocate(self, seq: Sequence) -> bool:
        return len(self.free_block_ids) >= seq.num_blocks

    def allocate(self, seq: Sequence) -> None:
        assert not seq.block_table
        prev_hash = -1
        missed = False
        counting = True  # hits still count as computed tokens (no unwritten block before them)
        for i in range(seq.num_blocks):
            token_ids = seq.block(i)
            full = len(token_ids) == self.block_size
            prev_hash = self.compute_hash(token_ids, prev_hash) if full else -1
            cached_id = self.hash_to_block_id.get(prev_hash, -1)
            if cached_id == -1 or self.blocks[cached_id].token_ids != token_ids:
                missed = True
            if missed:
                block = self._allocate_block(self.free_block_ids[0])
            else:
                if counting and not self.blocks[cached_id].computed and not self.count_unwritten_hits:
                    counting = False
                    self.unwritten_hits += 1
                if counting:
                    seq.num_cached_tokens += self.block_size
                if cached_id in self.used_block_ids:
                    block = self.blocks[cached_id]
                    block.ref_count += 1
                else:
                    written = self.blocks[cached_id].computed  # a freed block keeps its rows
                    block = self._allocate_block(cached_id)
                    block.computed = written
            if prev_hash != -1:
                block.update(prev_hash, token_ids)
                self.hash_to_block_id[prev_hash] = block.block_id
            seq.block_table.append(block.block_id)

    def allocate_uncached(self, seq: Sequence) -> None:
        """Fresh blocks for every page of `seq`, outside the prefix cache (no lookup, no hash
        registered): for one-off scoring passes that must neither reuse nor publish rows."""
        assert not seq.block_table
        for _ in range(seq.num_blocks):
            seq.block_table.append(self._allocate_block(self.free_block_ids[0]).block_id)

    def deallocate(self, seq: Sequence) -> None:
        for block_id in reversed(seq.block_table):
            block = self.blocks[block_id]
            block.ref_count -= 1
            if block.ref_count == 0:
                self._deallocate_block(block_id)
        seq.num_cached_tokens = 0
        seq.decode_cache_ready = False
        seq.block_table.clear()

    def can_append(self, seq: Sequence) -> bool:
        needs_block = len(seq) % self.block_size == 1
        return len(self.free_block_ids) >= needs_block

    def mark_computed(self, seq: Sequence, end: int) -> None:
        """Blocks of `seq` wholly below token `end` have their rows written once this step runs
        (called when a prefill chunk ending at `end` is scheduled)."""
        table = seq.block_table
        for i in range(seq.num_computed_tokens // self.block_size, min(end // self.block_size, len(table))):
            self.blocks[table[i]].computed = True

    def may_append(self, seq: Sequence) -> None:
        table = seq.block_table
        last = self.blocks[table[-1]]
        phase = len(seq) % self.block_size
        if phase == 1:
            # The newest token starts a new page.
            block = self._allocate_block(self.free_block_ids[0])
            table.append(block.block_id)
        elif phase == 0:
            # The newest token, written by this decode step, completes the last page.
            last.computed = True
        if phase == 0 and last.hash == -1:
            # The last page just filled up: register it in the prefix cache.
            token_ids = seq.block(seq.num_blocks - 1)
            if PLACEHOLDER in token_ids:
                # Its last token is still on the GPU (overlapped decode): hash it once known.
                self.deferred_hashes.append((seq, seq.num_blocks - 1, last.block_id))
                return
            self._register_full_block(table, len(table) - 1, token_ids)

    def _register_full_block(self, table: list[int], i: int, token_ids: list[int]) -> None:
        block = self.blocks[table[i]]
        prefix = self.blocks[table[i - 1]].hash if i > 0 else -1
        h = self.compute_hash(token_ids, prefix)
        block.update(h, token_ids)
        self.hash_to_block_id[h] = block.block_id

    def resolve_deferred(self) -> None:
        """Registers the pages whose hashing waited for a token read back from the GPU (the same
        hash may_append computes, one step later); pages no longer owned are dropped."""
        keep = []
        for seq, i, block_id in self.deferred_hashes:
            table = seq.block_table
            if i >= len(table) or table[i] != block_id or self.blocks[block_id].hash != -1:
                continue
            token_ids = seq.block(i)
            if PLACEHOLDER in token_ids:
                keep.append((seq, i, block_id))
                continue
            self._register_full_block(table, i, token_ids)
        self.deferred_hashes = keep
