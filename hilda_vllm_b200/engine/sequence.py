"""Request state: token ids, prefill progress, block table, decode slot.

Same attributes, properties and pickle protocol as mini_vllm/engine/sequence.py:14-132, so a
Sequence can be handed to, or received from, code written for the reference.
"""
from copy import copy
from enum import Enum, auto
from itertools import count

from hilda_vllm_b200.sampling_params import SamplingParams


# Stands for a decode token that the GPU has sampled but the host has not read back yet
# (overlapped decode steps); replaced by the real id one step later.
PLACEHOLDER = -1


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


class Sequence:
    block_size = 256
    counter = count()

    def __init__(self, token_ids: list[int], sampling_params: SamplingParams = SamplingParams()):
        self.seq_id = next(Sequence.counter)
        self.status = SequenceStatus.WAITING
        self.token_ids = copy(token_ids)
        self.last_token = token_ids[-1]
        self.num_tokens = len(self.token_ids)
        self.num_prompt_tokens = len(token_ids)
        self.num_cached_tokens = 0
        self.num_computed_tokens = 0
        self.block_table: list[int] = []
        self.temperature = sampling_params.temperature
        self.max_tokens = sampling_params.max_tokens
        self.ignore_eos = sampling_params.ignore_eos
        self.top_k = sampling_params.top_k
        self.top_p = sampling_params.top_p
        self.greedy = getattr(sampling_params, "greedy", False)
        self.decode_cache_ready = False
        self.decode_slot_index = -1

    def __len__(self):
        return self.num_tokens

    def __getitem__(self, key):
        return self.token_ids[key]

    @property
    def is_finished(self):
        return self.status == SequenceStatus.FINISHED

    @property
    def num_completion_tokens(self):
        return self.num_tokens - self.num_prompt_tokens

    @property
    def num_uncomputed_tokens(self):
        return self.num_tokens - self.num_computed_tokens

    @property
    def prompt_token_ids(self):
        return self.token_ids[: self.num_prompt_tokens]

    @property
    def completion_token_ids(self):
        return self.token_ids[self.num_prompt_tokens:]

    @property
    def num_prompt_tokens_remaining(self):
        return max(0, self.num_prompt_tokens - self.num_computed_tokens)

    @property
    def is_prefill_done(self):
        return self.num_computed_tokens >= self.num_prompt_tokens

    @property
    def num_cached_blocks(self):
        return self.num_cached_tokens // self.block_size

    @property
    def num_blocks(self):
        return -(-self.num_tokens // self.block_size)

    @property
    def last_block_num_tokens(self):
        return self.num_tokens - (self.num_blocks - 1) * self.block_size

    def block(self, i):
        assert 0 <= i < self.num_blocks
        start = i * self.block_size
        return self.token_ids[start: start + self.block_size]

    def append_token(self, token_id: int):
        self.token_ids.append(token_id)
        self.last_token = token_id
        self.num_tokens += 1

    # Pickle protocol (sequence.py:91-132): a sequence that has generated tokens ships only its
    # last token; one still in prefill ships its full token list.
    def _ships_all_tokens(self) -> bool:
        return self.status == SequenceStatus.WAITING or self.num_completion_tokens == 0

    def __getstate__(self):
        tokens = self.token_ids if self._ships_all_tokens() else self.last_token
        return (self.seq_id, self.status, self.num_tokens, self.num_prompt_tokens, self.num_cached_tokens,
                self.num_computed_tokens, self.block_table, self.temperature, self.max_tokens, self.ignore_eos,
                self.top_k, self.top_p, self.decode_cache_ready, self.decode_slot_index, tokens, self.greedy)

    def __setstate__(self, state):
        (self.seq_id, self.status, self.num_tokens, self.num_prompt_tokens, self.num_cached_tokens,
         self.num_computed_tokens, self.block_table, self.temperature, self.max_tokens, self.ignore_eos,
         self.top_k, self.top_p, self.decode_cache_ready, self.decode_slot_index, tokens, self.greedy) = state
        if self._ships_all_tokens():
            self.token_ids = tokens
            self.last_token = tokens[-1]
        else:
            self.last_token = tokens
