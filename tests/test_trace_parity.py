"""Replays churn traces recorded from the reference engine (tests/golden/sched_trace_*.json,
made by tests/golden/make_golden.py from mini_vllm's Scheduler, BlockManager and ModelRunner)
through this package's host code and checks, bit for bit:
  - every scheduling decision (prefill/decode, slot order, chunk sizes, padding slots),
    block ids, free lists, decode slots, compaction and preemption;
  - the prefill batch metadata (prefill_metadata vs the reference prepare_prefill);
  - the decode graph buffers: DecodePacker packets applied with the oracle's restatement of
    the pack kernel == the reference prepare_decode buffers (and the oracle's restatement of
    prepare_decode == the recorded reference buffers, which pins that restatement)."""
import json
from types import SimpleNamespace

import numpy as np
import pytest

from hilda_vllm_b200.engine.decode_packer import DecodePacker
from hilda_vllm_b200.engine.model_runner import prefill_metadata
from hilda_vllm_b200.engine.scheduler import Scheduler
from hilda_vllm_b200.engine.sequence import Sequence, SequenceStatus
from hilda_vllm_b200.sampling_params import SamplingParams
from oracle.decode_pack import DeviceDecodeState, ReferenceDecodeBuffers, apply_packet

TRACES = ["sched_trace_churn", "sched_trace_prefix", "sched_trace_complete"]


def _load(golden_dir, name):
    with open(golden_dir / f"{name}.json") as f:
        return json.load(f)


def _replay(trace, seq_block_size, on_step=None):
    meta = trace["meta"]
    seq_block_size(meta["block_size"])
    # The reference stops with "no runnable work" where this scheduler would let held chunked
    # prefills proceed; the traces pin the reference's behaviour, so that escape is off here.
    cfg = SimpleNamespace(**meta["cfg"], unblock_prefill_head=False)
    sched = Scheduler(cfg)
    prompts, params = meta["prompts"], meta["params"]
    seqs = {}
    next_prompt = 0
    for rec in trace["steps"]:
        while next_prompt < len(rec["admitted"]):
            mt, ign = params[next_prompt]
            s = Sequence(prompts[next_prompt], SamplingParams(max_tokens=mt, ignore_eos=ign))
            assert s.seq_id == rec["admitted"][next_prompt]
            seqs[s.seq_id] = s
            sched.add(s)
            next_prompt += 1
        if "error" in rec:
            with pytest.raises(RuntimeError, match="no runnable prefill or decode work"):
                sched.schedule()
            return seqs
        scheduled, is_prefill = sched.schedule()
        assert is_prefill == rec["is_prefill"]
        got = [[s.slot_index, -1 if s.seq is None else s.seq.seq_id, s.token_chunk_size] for s in scheduled]
        assert got == rec["sched"]
        if on_step is not None:
            on_step(rec, scheduled, is_prefill)
        sched.postprocess(scheduled, rec["tokens"], is_prefill)
        after = rec["after"]
        assert [-1 if s is None else s.seq_id for s in sched.decode_slots] == after["decode_slots"]
        assert sched.persistent_batch_size == after["persistent_batch_size"]
        assert sorted(sched.free_slot_indices) == after["free_slots"]
        assert list(sched.block_manager.free_block_ids) == after["free_blocks"]
        assert [s.seq_id for s in sched.waiting] == after["waiting"]
        assert {str(k): v.block_table for k, v in seqs.items() if v.block_table} == after["block_tables"]
        assert sorted(k for k, v in seqs.items() if v.is_finished) == after["finished"]
    return seqs


@pytest.mark.parametrize("name", TRACES)
def test_scheduler_matches_reference_trace(golden_dir, seq_block_size, name):
    _replay(_load(golden_dir, name), seq_block_size)


@pytest.mark.parametrize("name", TRACES)
def test_prefill_metadata_matches_reference(golden_dir, seq_block_size, name):
    trace = _load(golden_dir, name)
    bs = trace["meta"]["block_size"]
    n = [0]

    def check(rec, scheduled, is_prefill):
        if not is_prefill:
            return
        m = prefill_metadata(scheduled, bs)
        ref = rec["prefill"]
        assert m["input_ids"].tolist() == ref["input_ids"]
        assert m["positions"].tolist() == ref["positions"]
        assert m["cu_seqlens_q"].tolist() == ref["cu_q"] and m["cu_seqlens_k"].tolist() == ref["cu_k"]
        assert (m["max_seqlen_q"], m["max_seqlen_k"]) == (ref["max_q"], ref["max_k"])
        assert m["slot_mapping"].tolist() == ref["slot_mapping"]
        assert (None if m["block_tables"] is None else m["block_tables"].tolist()) == ref["block_tables"]
        n[0] += 1

    _replay(trace, seq_block_size, check)
    assert n[0] > 0


@pytest.mark.parametrize("name", TRACES)
def test_decode_packing_matches_reference(golden_dir, seq_block_size, name):
    trace = _load(golden_dir, name)
    meta = trace["meta"]
    bs = meta["block_size"]
    max_bs = meta["max_bs"]
    mb = -(-meta["max_model_len"] // bs)
    packer = DecodePacker(max_bs, mb)
    dev = DeviceDecodeState(max_bs, mb, bs)
    ref = ReferenceDecodeBuffers(max_bs, mb, bs)
    prev_tokens = {}
    n = [0, 0]

    def check(rec, scheduled, is_prefill):
        if is_prefill:
            return
        graph_bs = rec["graph_bs"]
        rows = [None if s.seq is None else (s.seq.seq_id, len(s.seq), s.seq.last_token, list(s.seq.block_table),
                                            s.seq.status == SequenceStatus.WAITING) for s in scheduled]
        # Pin the oracle restatement of prepare_decode on the reference's own buffers.
        ref.prepare(rows, graph_bs)
        want = {k: np.asarray(v) for k, v in rec["decode"].items()}
        snap = ref.snapshot(graph_bs)
        for k in want:
            np.testing.assert_array_equal(snap[k], want[k], err_msg=f"oracle prepare_decode {k}")
        # The device path: packet from the host packer, applied as hl_pack_decode_batch does.
        nbytes = packer.build(scheduled, graph_bs)
        apply_packet(dev, packer.buffer[:nbytes], graph_bs)
        got = dev.snapshot(graph_bs)
        for k in want:
            np.testing.assert_array_equal(got[k], want[k], err_msg=f"packed {k}")
        n[0] += 1
        n[1] += packer.last_num_events
        # The sampler writes this step's tokens into next_tokens on the device.
        toks = [0 if t is None else t for t in rec["tokens"]]
        dev.next_tokens[: len(toks)] = toks
        packer.note_sampled(len(toks), toks)

    _replay(trace, seq_block_size, check)
    assert n[0] > 10
    # Most slots continue without an event: the packet is much smaller than the batch.
    assert n[1] < sum(1 for _ in range(n[0])) * max_bs
