"""Tensor-parallel host logic with two gloo ranks on the CPU: sharded linear layers and their
weight loaders (the reference's TP layout, mini_vllm/layers/linear.py), the all-reduce after
o_proj/down_proj, the vocabulary-sharded LM head gather (embed_head.py:56-66), the greedy
(max, index) merge that replaces the logits gather, and the torchrun-mode control plane."""
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=world, rank=rank)
        torch.manual_seed(0)
        from transformers import Qwen3Config

        from hilda_vllm_b200.engine.control_plane import ShmChannel
        from hilda_vllm_b200.engine.model_runner import merge_shard_argmax
        from hilda_vllm_b200.layers.embed_head import ParallelLMHead
        from hilda_vllm_b200.layers.linear import MergedColumnParallelLinear, QKVParallelLinear, RowParallelLinear
        from hilda_vllm_b200.utils.loader import random_weights

        cfg = Qwen3Config(hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2,
                          head_dim=128, num_hidden_layers=1, vocab_size=512, tie_word_embeddings=False)
        w = dict(random_weights(cfg, seed=5, std=0.02, device="cpu", dtype=torch.float32))
        p = "model.layers.0."
        torch.set_default_dtype(torch.float32)
        qkv = QKVParallelLinear(256, 128, 4, 2)
        for sid in "qkv":
            qkv.weight.weight_loader(qkv.weight, w[p + f"self_attn.{sid}_proj.weight"], sid)
        o = RowParallelLinear(4 * 128, 256)
        o.weight.weight_loader(o.weight, w[p + "self_attn.o_proj.weight"])
        gu = MergedColumnParallelLinear(256, [512, 512])
        gu.weight.weight_loader(gu.weight, w[p + "mlp.gate_proj.weight"], 0)
        gu.weight.weight_loader(gu.weight, w[p + "mlp.up_proj.weight"], 1)
        down = RowParallelLinear(512, 256)
        down.weight.weight_loader(down.weight, w[p + "mlp.down_proj.weight"])
        head = ParallelLMHead(512, 256)
        head.weight.weight_loader(head.weight, w["lm_head.weight"])

        x = torch.randn(5, 256, generator=torch.Generator().manual_seed(1))
        with torch.no_grad():
            # attention projections: this rank's heads only, then the o_proj all-reduce
            y = qkv(x)
            hq, hk = 4 // world, 2 // world
            q = y[:, :hq * 128]
            attn_out = q  # stand-in for attention output of this rank's heads
            z = o(attn_out)
            g, u = gu(x).chunk(2, -1)
            m = down(torch.nn.functional.silu(g) * u)
            logits = head.local_logits(x)
            parts = [torch.empty_like(logits) for _ in range(world)]
            dist.all_gather(parts, logits)
            full_logits = torch.cat(parts, -1)
            # greedy merge of per-shard (max, index) pairs
            val, idx = logits.max(-1)
            idx = idx + head.vocab_start_idx
            all_val = [torch.empty_like(val) for _ in range(world)]
            all_idx = [torch.empty_like(idx) for _ in range(world)]
            dist.all_gather(all_val, val)
            dist.all_gather(all_idx, idx)
            merged = merge_shard_argmax(torch.stack(all_val), torch.stack(all_idx))
        # control plane (torchrun mode): the segment name crosses once over gloo, calls through it
        group = dist.new_group(backend="gloo")
        box = [None]
        if rank == 0:
            chan = ShmChannel.create(world, size=1 << 20)
            box = [chan.name]
        dist.broadcast_object_list(box, src=0, group=group)
        if rank > 0:
            chan = ShmChannel.attach(box[0], rank, world)
        dist.barrier(group=group)
        if rank == 0:
            chan.send("run", [1, 2, 3], {"a": 1})
            msg = ("run", [[1, 2, 3], {"a": 1}])
        else:
            method, args = chan.recv()
            msg = (method, args)
        dist.barrier(group=group)
        chan.close()
        queue.put((rank, z, m, full_logits, merged, msg))
        dist.destroy_process_group()
    except Exception as exc:  # pragma: no cover - surfaced by the parent
        queue.put((rank, repr(exc)))
        raise


def _reference_outputs():
    from transformers import Qwen3Config

    from hilda_vllm_b200.utils.loader import random_weights

    cfg = Qwen3Config(hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=128, num_hidden_layers=1, vocab_size=512, tie_word_embeddings=False)
    w = dict(random_weights(cfg, seed=5, std=0.02, device="cpu", dtype=torch.float32))
    p = "model.layers.0."
    x = torch.randn(5, 256, generator=torch.Generator().manual_seed(1))
    q = x @ w[p + "self_attn.q_proj.weight"].t()
    g = x @ w[p + "mlp.gate_proj.weight"].t()
    u = x @ w[p + "mlp.up_proj.weight"].t()
    m = (torch.nn.functional.silu(g) * u) @ w[p + "mlp.down_proj.weight"].t()
    logits = x @ w["lm_head.weight"].t()
    return w, q, m, logits


def _run_ranks(world):
    """Runs _worker on `world` spawned gloo ranks; returns {rank: result} or raises with the first
    failing rank's message."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            item = queue.get(timeout=240)
            if len(item) <= 2:
                raise RuntimeError(f"rank {item[0]} failed: {item[1]}")
            results[item[0]] = item
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    if any(p.exitcode != 0 for p in procs):
        raise RuntimeError(f"rank exit codes {[p.exitcode for p in procs]}")
    return results


def test_tensor_parallel_layers_two_gloo_ranks():
    world = 2
    # The rendezvous port is picked free and then bound by the ranks a moment later, so another
    # process on the host can take it in between: one retry on a fresh port.
    try:
        results = _run_ranks(world)
    except RuntimeError:
        results = _run_ranks(world)
    w, q, m, logits = _reference_outputs()
    # o_proj over the concatenated per-rank head outputs == full o_proj (sum of the two shards)
    o_full = q @ w["model.layers.0.self_attn.o_proj.weight"].t()
    for r in range(world):
        _, z, m_r, full_logits, merged, msg = results[r]
        assert torch.allclose(z, o_full, atol=1e-5, rtol=1e-4)
        assert torch.allclose(m_r, m, atol=1e-5, rtol=1e-4)
        assert torch.allclose(full_logits, logits, atol=1e-6)
        assert torch.equal(merged, logits.argmax(-1))
        assert msg == ("run", [[1, 2, 3], {"a": 1}])


def test_merge_shard_argmax_ties_pick_lowest_global_index():
    from hilda_vllm_b200.engine.model_runner import merge_shard_argmax

    logits = torch.tensor([[1.0, 5.0, 5.0, 0.0], [2.0, 0.0, 0.0, 2.0], [0.0, 1.0, 3.0, 3.0]])
    shards = logits.chunk(2, -1)
    vals, idxs = [], []
    for s, sh in enumerate(shards):
        v, i = sh.max(-1)
        vals.append(v)
        idxs.append(i + 2 * s)
    merged = merge_shard_argmax(torch.stack(vals), torch.stack(idxs))
    assert merged.tolist() == logits.argmax(-1).tolist() == [1, 0, 2]


def test_all_reduce_kernel_choice_follows_measured_costs():
    """One-shot vs two-shot fused all-reduce, against the B200 measurements at 8 ranks (us per
    call, one-shot / two-shot): the choice is the faster kernel, or within 2 % of it."""
    from hilda_vllm_b200.layers.nvlink_allreduce import prefer_two_shot

    measured = {  # (world, rows, hidden): (one-shot us, two-shot us), 8 B200s
        (8, 64, 1024): (10.1, 16.2), (8, 256, 1024): (14.6, 16.7), (8, 64, 4096): (17.9, 22.6),
        (8, 256, 4096): (37.2, 35.1),
    }
    for (world, rows, hidden), (one, two) in measured.items():
        chosen = two if prefer_two_shot(world, rows, hidden) else one
        assert chosen <= 1.02 * min(one, two), (world, rows, hidden)
    assert not prefer_two_shot(1, 512, 8192) and not prefer_two_shot(2, 512, 8192)
