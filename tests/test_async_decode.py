"""Overlapped decode (LLMEngine.step with async_decode) against the synchronous engine, on CPU.

The model runner is replaced by a stand-in whose "device" is the oracle's restatement of the
decode pack kernel (oracle/decode_pack.py) and whose model says the token at position p of
sequence s is a fixed function tok(s, p).  Every decode step then checks that the buffers the
packet produces on the device hold exactly the right input token, position, context length and
slot mapping for every live slot — in particular that a token still "on the GPU" (PLACEHOLDER on
the host) is the one the device feeds back.  The overlapped engine must finish every request with
the same tokens and the same block-level decisions as the synchronous one, under churn
(staggered lengths, slot compaction, preemption from a small pool, prefix caching).
"""
from types import SimpleNamespace

import numpy as np
import pytest

from hilda_vllm_b200.engine.decode_packer import DecodePacker
from hilda_vllm_b200.engine.llm_engine import LLMEngine
from hilda_vllm_b200.engine.model_runner import decode_sampling, device_sampleable
from hilda_vllm_b200.engine.scheduler import Scheduler
from hilda_vllm_b200.engine.sequence import PLACEHOLDER, Sequence, SequenceStatus
from hilda_vllm_b200.sampling_params import SamplingParams
from oracle.decode_pack import DeviceDecodeState, apply_packet


@pytest.fixture(autouse=True)
def _restore_sequence_globals():
    bs, counter = Sequence.block_size, Sequence.counter
    yield
    Sequence.block_size, Sequence.counter = bs, counter


def tok(seq_id: int, pos: int) -> int:
    return (seq_id * 7919 + pos * 104729) % 5000 + 3


class FakeRunner:
    def __init__(self, max_bs: int, block_size: int, max_model_len: int, device_filters: bool = False):
        self.device_filters = device_filters  # ModelRunner: True on one GPU (hl_sample_filtered)
        self.max_blocks = -(-max_model_len // block_size)
        self.block_size = block_size
        self.packer = DecodePacker(max_bs, self.max_blocks)
        self.dev = DeviceDecodeState(max_bs, self.max_blocks, block_size)
        self.last_decode_batch_info = None
        self.prompts: dict[int, list[int]] = {}
        self.steps = 0
        self.launched = 0

    def truth(self, seq, pos):
        prompt = self.prompts[seq.seq_id]
        return prompt[pos] if pos < len(prompt) else tok(seq.seq_id, pos)

    def _device_step(self, scheduled):
        bs = len(scheduled)
        nbytes = self.packer.build(scheduled, bs)
        apply_packet(self.dev, self.packer.buffer[:nbytes].copy(), bs)
        self.last_decode_batch_info = {"scheduled_bs": bs, "graph_bs": bs,
                                       "active_seqs": sum(not s.is_padding for s in scheduled),
                                       "padded_slots": sum(s.is_padding for s in scheduled), "pack_events": 0}
        tokens = []
        for i, sched in enumerate(scheduled):
            seq = sched.seq
            if seq is None or seq.status == SequenceStatus.WAITING:  # padding, or preempted after scheduling
                assert self.dev.context_lens[i] == 0 and self.dev.slot_mapping[i] == -1
                self.dev.next_tokens[i] = 999_999  # whatever a padding row's argmax gives
                tokens.append(999_999)
                continue
            n = seq.num_tokens
            assert self.dev.context_lens[i] == n and self.dev.positions[i] == n - 1
            assert self.dev.input_ids[i] == self.truth(seq, n - 1), (i, seq.seq_id, n)
            table = seq.block_table
            assert list(self.dev.block_tables[i, :len(table)]) == table
            want_slot = table[(n - 1) // self.block_size] * self.block_size + (n - 1) % self.block_size
            assert self.dev.slot_mapping[i] == want_slot
            t = tok(seq.seq_id, n)
            self.dev.next_tokens[i] = t
            tokens.append(t)
        self.steps += 1
        return tokens

    # -- the ModelRunner surface LLMEngine uses
    def run(self, scheduled, is_prefill):
        if is_prefill:
            out = []
            for s in scheduled:
                if s.requires_sampling:
                    out.append(tok(s.seq.seq_id, s.seq.num_tokens))
                else:
                    out.append(None)
            return out
        tokens = self._device_step(scheduled)
        self.packer.note_sampled(len(scheduled), tokens)
        return [None if s.is_padding else t for s, t in zip(scheduled, tokens)]

    def samples_on_device(self, seq):
        return device_sampleable(seq, self.device_filters)

    def can_launch_decode(self, scheduled):
        return (decode_sampling(scheduled, self.device_filters) is not None
                and not self.packer.needs_host_tokens(scheduled))

    def launch_decode(self, scheduled):
        tokens = self._device_step(scheduled)
        self.packer.note_launched(len(scheduled), scheduled)
        self.launched += 1
        return tokens

    def collect_decode(self, handle):
        return handle


def make_engine(async_decode: bool, num_blocks: int, max_num_seqs: int = 8, block_size: int = 16,
                max_model_len: int = 256, drop_victim_token: bool = True, device_filters: bool = False):
    cfg = SimpleNamespace(kvcache_block_size=block_size, max_num_seqs=max_num_seqs, max_num_batched_tokens=128,
                          eos=-1, enable_chunked_prefill=True, chunked_prefill_size=64, chunked_prefill_min_size=16,
                          chunked_prefill_tile_size=16, num_kvcache_blocks=num_blocks, async_decode=async_decode,
                          kv_cache_dtype="auto", max_model_len=max_model_len,
                          drop_preempted_decode_token=drop_victim_token)
    eng = LLMEngine.__new__(LLMEngine)
    eng.config = cfg
    eng.scheduler = Scheduler(cfg)
    eng.model_runner = FakeRunner(max_num_seqs, block_size, max_model_len, device_filters)
    eng._inflight = None
    eng.last_step_diagnostics = None
    return eng


def drive(eng, prompts, max_tokens, greedy=True, top_k=-1):
    seqs = []
    for p, m in zip(prompts, max_tokens):
        seq = Sequence(p, SamplingParams(max_tokens=m, ignore_eos=True, greedy=greedy, top_k=top_k))
        eng.model_runner.prompts[seq.seq_id] = list(p)
        eng.scheduler.add(seq)
        seqs.append(seq)
    outputs = {}
    guard = 0
    while not eng.is_finished():
        out, *_ = eng.step()
        for seq_id, toks in out:
            assert seq_id not in outputs
            assert PLACEHOLDER not in toks
            outputs[seq_id] = list(toks)
        guard += 1
        assert guard < 10_000
    return seqs, outputs


@pytest.mark.parametrize("num_blocks,drop_victim_token", [(200, True), (24, True), (24, False), (40, False)])
def test_overlapped_decode_matches_synchronous(num_blocks, drop_victim_token):
    """With drop_victim_token the tokens are exactly the model's; with the reference's behaviour
    (a preempted victim keeps its padding row's token) only sync == overlapped is required."""
    rng = np.random.default_rng(num_blocks)
    prompts = [rng.integers(0, 4000, int(n)).tolist() for n in rng.integers(1, 60, 20)]
    max_tokens = [int(m) for m in rng.integers(1, 90, 20)]
    results = {}
    for mode in (False, True):
        Sequence.counter = iter(range(10_000))  # same seq ids in both runs
        eng = make_engine(mode, num_blocks, drop_victim_token=drop_victim_token)
        seqs, outputs = drive(eng, prompts, max_tokens)
        assert len(outputs) == len(prompts)
        for seq in seqs:
            want = [tok(seq.seq_id, len(seq.prompt_token_ids) + k) for k in range(seq.max_tokens)]
            if drop_victim_token:
                assert outputs[seq.seq_id] == want
            else:
                assert len(outputs[seq.seq_id]) == len(want)
        results[mode] = (outputs, eng.model_runner.steps, eng.model_runner.launched)
        assert not eng.scheduler.block_manager.deferred_hashes or mode
    assert results[False][0] == results[True][0]
    assert results[True][2] > 0  # the overlapped path actually ran
    assert results[False][2] == 0


@pytest.mark.parametrize("top_k,device_filters,overlapped", [(-1, False, True), (5, False, False), (5, True, True)])
def test_which_sampled_sequences_overlap(top_k, device_filters, overlapped):
    """Plain temperature sampling runs on the device and overlaps; top-k overlaps too where the
    device sampler has the whole vocabulary (one GPU), else it needs the host sampler and those
    steps run synchronously."""
    Sequence.counter = iter(range(10_000))
    eng = make_engine(True, 200, device_filters=device_filters)
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 4000, 10).tolist() for _ in range(4)]
    seqs, outputs = drive(eng, prompts, [12] * 4, greedy=False, top_k=top_k)
    assert (eng.model_runner.launched > 0) == overlapped and len(outputs) == 4


def test_deferred_page_hash_equals_synchronous_hash():
    """A page that fills up with a token still on the GPU is hashed one step later, with the
    same value the synchronous engine registers at once."""
    hashes = {}
    for mode in (False, True):
        Sequence.counter = iter(range(10_000))
        eng = make_engine(mode, 200)
        eng.model_runner.prompts = {}
        seq = Sequence(list(range(5)), SamplingParams(max_tokens=40, ignore_eos=True, greedy=True))
        eng.model_runner.prompts[seq.seq_id] = list(range(5))
        eng.scheduler.add(seq)
        bm = eng.scheduler.block_manager
        registered = []
        while not eng.is_finished():
            eng.step()
            registered.append(sorted(bm.hash_to_block_id.items()))
        hashes[mode] = registered[-1]
    assert hashes[True] == hashes[False] and len(hashes[True]) >= 2


def test_decode_sampling_settings_encoding():
    """Per-row device sampler settings: greedy and padding rows are (T 0, k 0, p 1); top_k travels
    as int32 bits in the float32 block (-1 -> 0, no filter); rows with filters make the whole
    batch host-sampled unless the device has the full vocabulary."""
    from hilda_vllm_b200.engine.model_runner import ModelRunner

    Sequence.counter = iter(range(10_000))
    mk = lambda **kw: Sequence([1, 2, 3], SamplingParams(max_tokens=4, **kw))
    seqs = [mk(greedy=True), mk(temperature=0.7), mk(temperature=1.2, top_k=7, top_p=0.9), None]
    sched = [SimpleNamespace(seq=s, is_padding=s is None) for s in seqs]
    assert decode_sampling(sched, filters=False) is None
    out = decode_sampling(sched, filters=True)
    assert out.dtype == np.float32 and out.shape == (3, 4)
    np.testing.assert_array_equal(out[0], np.array([0.0, 0.7, 1.2, 0.0], np.float32))
    np.testing.assert_array_equal(out[1].view(np.int32), [0, 0, 7, 0])
    np.testing.assert_array_equal(out[2], np.array([1.0, 1.0, 0.9, 1.0], np.float32))
    plain = decode_sampling(sched[:2], filters=False)
    np.testing.assert_array_equal(plain[1].view(np.int32), [0, 0])

    # upload only on change: the mirror starts as "greedy, unfiltered" everywhere
    runner = SimpleNamespace(samp_host=np.zeros((3, 8), np.float32))
    runner.samp_host[2] = 1.0
    change = ModelRunner._temps_change
    assert change(runner, decode_sampling(sched[:1], True), 1) is None  # greedy: nothing to send
    block = change(runner, out, 4)
    assert block is not None and block.shape == (3, 8)
    np.testing.assert_array_equal(block[:, :4].view(np.uint32), out.view(np.uint32))
    assert change(runner, out, 4) is None  # the device already holds it
    assert change(runner, out[:, :2].copy(), 4) is not None  # rows 2, 3 go back to greedy
    np.testing.assert_array_equal(runner.samp_host[1, :4].view(np.int32), [0, 0, 0, 0])
