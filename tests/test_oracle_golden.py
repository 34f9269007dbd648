"""Pins the CPU oracle against fixtures produced by the reference's own code
(tests/golden/make_golden.py) and against torch's float8_e4m3fn cast."""
import json

import numpy as np
import torch

from oracle import attention as oattn
from oracle import kv_store
from oracle.build import load as load_oracle_c
from oracle.qwen3_model import Qwen3Oracle, decode_context, prefill_context


def bf(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)


def test_store_oracle_matches_reference_triton_kernel(golden_dir):
    g = np.load(golden_dir / "store_kv.npz")
    n, hq, hk, d, nb, bs = g["shape"].tolist()
    qkv = bf(g["qkv"])
    key = qkv[:, hq * d:(hq + hk) * d].view(n, hk, d)
    value = qkv[:, (hq + hk) * d:].view(n, hk, d)
    kc = torch.zeros(nb, bs, hk, d, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    kv_store.store_kvcache(key, value, kc, vc, torch.from_numpy(g["slot_mapping"]))
    rows = torch.from_numpy(g["touched_slots"])
    assert torch.equal(kc.view(-1, hk * d)[rows].view(torch.int16), torch.from_numpy(g["k_rows"]))
    assert torch.equal(vc.view(-1, hk * d)[rows].view(torch.int16), torch.from_numpy(g["v_rows"]))
    nz = torch.nonzero(kc.view(-1, hk * d).float().abs().sum(1)).flatten()
    assert nz.tolist() == g["k_nonzero_rows"].tolist()  # slot -1 skipped, nothing else touched


def test_e4m3_c_oracle_matches_torch_exhaustively():
    lib = load_oracle_c()
    allb = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    vals = allb[torch.isfinite(allb.float())]
    src = vals.view(torch.int16).numpy().copy()
    for scale in (1.0, 0.37, 3.5, 1e-3):
        out = np.zeros(len(vals), np.uint8)
        sc = np.array([scale], np.float32)
        lib.oracle_quantize_rows(src.ctypes.data, 1, 1, len(vals), sc.ctypes.data, out.ctypes.data)
        ref = torch.clamp(vals.float() / torch.tensor(scale, dtype=torch.float32), -448, 448)
        ref = ref.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        assert (out == ref).all(), scale
    dec = np.array([lib.oracle_e4m3_to_float(i) for i in range(256)], np.float32)
    tdec = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    both_nan = np.isnan(dec) & np.isnan(tdec)
    assert ((dec == tdec) | both_nan).all()


def test_e4m3_torch_quantiser_equals_c_oracle():
    """quantize_e4m3_torch (the GPU-resident oracle's quantiser) equals the C restatement on every
    finite bf16 value, with per-head scales."""
    allb = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    vals = allb[torch.isfinite(allb.float())]
    n = vals.numel() // 4 * 4
    x = vals[:n].view(-1, 4, 1).expand(-1, 4, 16).contiguous().view(-1, 4, 16)
    for sc in (None, torch.tensor([1.0, 0.37, 3.5, 1e-3])):
        assert torch.equal(kv_store.quantize_e4m3_torch(x, sc), kv_store.quantize_e4m3(x, sc))


def test_fp8_store_and_copy_oracles_agree():
    g = torch.Generator().manual_seed(5)
    key = (torch.randn(6, 2, 128, generator=g) * 40).bfloat16()
    value = torch.randn(6, 2, 128, generator=g).bfloat16()
    ks, vs = torch.tensor([0.5, 2.0]), torch.tensor([0.01, 1.0])
    kc = torch.zeros(2, 8, 2, 128, dtype=torch.uint8)
    vc = torch.zeros_like(kc)
    sm = torch.tensor([0, 3, -1, 9, 15, 4], dtype=torch.int32)
    kv_store.store_kvcache_fp8(key, value, kc, vc, sm, ks, vs)
    # copy path: BF16 cache -> FP8 cache at the same slots gives the same bytes
    kb = torch.zeros(2, 8, 2, 128, dtype=torch.bfloat16)
    vb = torch.zeros_like(kb)
    kv_store.store_kvcache(key, value, kb, vb, sm)
    kc2 = torch.zeros_like(kc)
    vc2 = torch.zeros_like(vc)
    kv_store.copy_kvcache_fp8(kb, vb, kc2, vc2, sm, ks, vs)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    want = torch.clamp(key[1].float() / ks.view(2, 1), -448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(kc.view(-1, 2, 128)[3], want)


def test_attention_oracle_edge_cases():
    g = torch.Generator().manual_seed(6)
    kc = torch.randn(4, 256, 2, 128, generator=g).bfloat16()
    vc = torch.randn(4, 256, 2, 128, generator=g).bfloat16()
    q = torch.randn(3, 4, 128, generator=g).bfloat16()
    bt = torch.tensor([[2, 0, -1], [1, -1, -1], [3, 2, 1]], dtype=torch.int32)
    lens = torch.tensor([300, 0, 1], dtype=torch.int32)
    out = oattn.paged_decode(q, kc, vc, bt, lens, 128 ** -0.5)
    assert torch.all(out[1] == 0)  # empty row
    # one cached token: softmax of one element = 1, output = that V row (slot 3*256+0)
    assert torch.allclose(out[2], vc.view(-1, 2, 128)[768].float().repeat_interleave(2, 0))
    # decode of a sequence equals the last row of its causal prefill
    k = kc.view(-1, 2, 128)[torch.cat([torch.arange(512, 768), torch.arange(0, 44)])]
    v = vc.view(-1, 2, 128)[torch.cat([torch.arange(512, 768), torch.arange(0, 44)])]
    qs = torch.randn(300, 4, 128, generator=g).bfloat16()
    qs[-1] = q[0]
    cu = torch.tensor([0, 300], dtype=torch.int32)
    pre = oattn.varlen_prefill(qs, k, v, cu, cu, 128 ** -0.5)
    assert torch.allclose(pre[-1], out[0], atol=1e-5, rtol=1e-5)
    # keys fewer than queries: rows with no visible key are zero
    cuk = torch.tensor([0, 10], dtype=torch.int32)
    cuq = torch.tensor([0, 12], dtype=torch.int32)
    short = oattn.varlen_prefill(qs[:12], k[:10], v[:10], cuq, cuk, 128 ** -0.5)
    assert torch.all(short[:2] == 0) and torch.all(short[2:].abs().sum(-1) > 0)


def test_layer_restatements_match_reference_modules(golden_dir):
    g = np.load(golden_dir / "layers.npz")
    from types import SimpleNamespace

    cfg = SimpleNamespace(num_attention_heads=4, num_key_value_heads=2, head_dim=128, hidden_size=512,
                          rms_norm_eps=1e-6, rope_theta=1000000.0, rope_scaling=None, max_position_embeddings=4096,
                          num_hidden_layers=0)
    o = Qwen3Oracle(cfg, {"model.embed_tokens.weight": torch.zeros(2, 2)}, 1, 256)
    x, r, w = bf(g["rms_x"]), bf(g["rms_r"]), bf(g["rms_w"])
    assert torch.equal(o.rms(x, w).view(torch.int16), torch.from_numpy(g["rms_y"]))
    y2, r2 = o.add_rms(x, r, w)
    assert torch.equal(y2.view(torch.int16), torch.from_numpy(g["add_y"]))
    assert torch.equal(r2.view(torch.int16), torch.from_numpy(g["add_r"]))
    q = bf(g["rope_q"])
    out = o.rope(o.rms(q, bf(g["rope_w"])), torch.from_numpy(g["rope_pos"]))
    assert torch.equal(out.view(torch.int16), torch.from_numpy(g["rope_out"]))
    a = bf(g["silu_in"])
    gate, up = a.chunk(2, -1)
    assert torch.equal((torch.nn.functional.silu(gate) * up).view(torch.int16), torch.from_numpy(g["silu_out"]))


def test_oracle_model_matches_reference_modules_greedy(golden_dir):
    """Tiny Qwen3 through the oracle reproduces the reference modules' greedy tokens."""
    from transformers import Qwen3Config

    from hilda_vllm_b200.models.qwen3 import Qwen3ForCausalLM  # noqa: F401  (weights only)
    from hilda_vllm_b200.utils.loader import checkpoint_tensor_shapes
    import zlib

    gold = json.loads((golden_dir / "tiny_model_greedy.json").read_text())
    cfg = Qwen3Config(**gold["config"])
    weights = {}
    for name, shape, is_norm in checkpoint_tensor_shapes(cfg):
        if is_norm:
            weights[name] = torch.ones(shape, dtype=torch.bfloat16)
        else:
            gen = torch.Generator().manual_seed((gold["seed"] * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFF_FFFF_FFFF_FFFF)
            weights[name] = (torch.randn(shape, generator=gen, dtype=torch.float32) * 0.02).bfloat16()
    bs = 256
    model = Qwen3Oracle(cfg, weights, 16, bs)
    prompts = gold["prompts"]
    tables = [[0], [1], [2, 3]]
    ids, pos, ctx = prefill_context(prompts, [0] * 3, [len(p) for p in prompts], tables, bs)
    with torch.no_grad():
        logits = model.logits(model.forward(ids, pos, ctx), ctx)
    toks = logits.argmax(-1).tolist()
    assert toks == gold["steps"][0]["tokens"]
    seqs = [p + [t] for p, t in zip(prompts, toks)]
    for step in gold["steps"][1:]:
        for s, t in zip(seqs, tables):
            if (len(s) - 1) // bs >= len(t):
                t.append(max(max(x) for x in tables) + 1)
        lens = [len(s) for s in seqs]
        ids, pos, ctx = decode_context(lens, [s[-1] for s in seqs], tables, bs, 4)
        with torch.no_grad():
            toks = model.logits(model.forward(ids, pos, ctx), ctx).argmax(-1).tolist()
        assert toks == step["tokens"]
        seqs = [s + [t] for s, t in zip(seqs, toks)]


def _seeded_weights(cfg, seed):
    """This repository's seeded random init (hilda_vllm_b200.utils.loader), restated: norms 1,
    every other tensor N(0, 0.02) from a generator seeded by (seed, crc32 of its name)."""
    import zlib

    from hilda_vllm_b200.utils.loader import checkpoint_tensor_shapes

    weights = {}
    for name, shape, is_norm in checkpoint_tensor_shapes(cfg):
        if is_norm:
            weights[name] = torch.ones(shape, dtype=torch.bfloat16)
        else:
            gen = torch.Generator().manual_seed((seed * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFF_FFFF_FFFF_FFFF)
            weights[name] = (torch.randn(shape, generator=gen, dtype=torch.float32) * 0.02).bfloat16()
    return weights


def _bf16_ulp(x: float) -> float:
    import math
    return 2.0 ** (math.floor(math.log2(abs(x))) - 7) if x != 0 else 2.0 ** -133


def test_oracle_0_6b_matches_reference_modules_32_greedy_steps(golden_dir):
    """The Qwen3-0.6B configuration (28 layers, vocab 151,936) through the oracle, teacher-forced
    on the greedy tokens that the reference's own modules produced free-running for 32 decode
    steps after a 64-token prefill (tests/golden/qwen3_0_6b_greedy_32.json): every step's argmax
    must be the reference's token, except where the reference's own top-2 gap is within 2 bf16
    ulps of its top logit (a tie that bf16 rounding order may flip)."""
    from transformers import AutoConfig

    from pathlib import Path

    gold = json.loads((golden_dir / "qwen3_0_6b_greedy_32.json").read_text())
    root = Path(__file__).resolve().parent.parent
    cfg = AutoConfig.from_pretrained(root / gold["config_dir"])
    bs = 256
    model = Qwen3Oracle(cfg, _seeded_weights(cfg, gold["seed"]), 4, bs)
    prompts = gold["prompts"]
    tables = [[0], [1], [2], [3]]
    ids, pos, ctx = prefill_context(prompts, [0] * 4, [len(p) for p in prompts], tables, bs)
    with torch.no_grad():
        got = [model.logits(model.forward(ids, pos, ctx), ctx).argmax(-1).tolist()]
    seqs = [p + [t] for p, t in zip(prompts, gold["steps"][0]["tokens"])]
    for step in gold["steps"][1:]:
        lens = [len(x) for x in seqs]
        ids, pos, ctx = decode_context(lens, [x[-1] for x in seqs], tables, bs, 1)
        with torch.no_grad():
            got.append(model.logits(model.forward(ids, pos, ctx), ctx).argmax(-1).tolist())
        seqs = [x + [t] for x, t in zip(seqs, step["tokens"])]
    exact = ties = 0
    for mine, step in zip(got, gold["steps"]):
        for m, t, top1, gap in zip(mine, step["tokens"], step["top1"], step["gap"]):
            if m == t:
                exact += 1
            else:
                assert gap <= 2 * _bf16_ulp(top1), (m, t, top1, gap)
                ties += 1
    assert exact + ties == 4 * len(gold["steps"])
    assert exact >= 0.9 * (exact + ties)


def test_e4m3_to_f16_bit_placement_is_exact():
    """The tensor-core FP8 decode converts e4m3 to f16 by bit placement (byte to the high byte of
    a 16-bit half, shift right by one, carry the sign from bit 14 to 15), giving value x 2^-8;
    restated here over all 256 bytes against torch's e4m3 decoding."""
    b = np.arange(256, dtype=np.uint32)
    x = (b << 8) >> 1
    h = ((x + (x & 0x4000)) & 0xFFFF).astype(np.uint16)
    got = torch.from_numpy(h.view(np.int16)).view(torch.float16).float()
    want = torch.from_numpy(b.astype(np.uint8)).view(torch.float8_e4m3fn).float() / 256
    finite = ~torch.isnan(want)
    assert torch.equal(got[finite], want[finite])
    assert int(finite.sum()) == 254


def test_sampler_filter_oracle_matches_reference_golden(golden_dir):
    """oracle/sampler.kept_set against the reference Sampler's own _apply_top_k / _apply_top_p
    masks (tests/golden/sampler_filters.npz, rows without equal logits)."""
    from oracle.sampler import kept_set

    g = np.load(golden_dir / "sampler_filters.npz")
    logits = torch.from_numpy(g["logits"])
    for r in range(logits.shape[0]):
        mine = kept_set(logits[r], float(g["temps"][r]), int(g["top_ks"][r]), float(g["top_ps"][r]))
        ref = torch.from_numpy(g["keep"][r])
        if float(g["top_ps"][r]) < 1.0:
            assert torch.equal(mine, ref), r
        else:
            # The reference skips _apply_top_p only when no row of the batch filters; here a
            # top_p = 1 row is filtered anyway and loses exactly the top-k tokens whose float32
            # inclusive cumsum reaches 1.0 (often the last kept one, whatever its probability).
            # The restatement (and hl_sample_filtered) keep per-row semantics: no top-p filter.
            x = logits[r] / torch.tensor(g["temps"][r])
            order = torch.sort(x, descending=True, stable=True).indices
            order = order[mine[order]]
            cum = torch.cumsum(torch.softmax(x[order], 0), 0)
            dropped = torch.zeros_like(mine)
            dropped[order[cum >= 1.0]] = True
            dropped[order[0]] = False
            assert torch.equal(ref, mine & ~dropped), r
    assert (g["keep"].sum(1) < logits.shape[1]).sum() > 20  # most rows actually filter something


def _e4m3_head(x: np.ndarray) -> np.ndarray:
    """x truncated to 4 significant bits (>= 2^-6) or to the 2^-9 grid (below): the larger e4m3
    term of the tensor-core FP8 decode's Q split (restated bit for bit)."""
    a = np.abs(x).astype(np.float32)
    big = (a.view(np.uint32) & np.uint32(0xFFF00000)).view(np.float32)
    small = (np.floor(a * np.float32(512)) * np.float32(1 / 512)).astype(np.float32)
    return np.copysign(np.where(a >= np.float32(0.015625), big, small), x).astype(np.float32)


def _e4m3_byte(x: np.ndarray) -> np.ndarray:
    """e4m3 byte of a value on the e4m3 grid (truncating below it), |x| < 2^8 (restated)."""
    u = x.astype(np.float32).view(np.uint32).astype(np.int64)
    sign = (u >> 24) & 0x80
    e = ((u >> 23) & 0xFF) - 120
    m = (u >> 20) & 7
    sh = 1 - e
    sub = np.where(sh <= 4, (8 | m) >> np.clip(sh, 0, 31), 0)
    return (sign | np.where(e >= 1, (e << 3) | m, sub)).astype(np.uint8)


def test_fp8_decode_q_split_is_exact():
    """The tensor-core FP8 decode feeds Q to a kind::f8f6f4 MMA as two e4m3 terms: after a
    power-of-two shift putting the head's largest |q| in [2^7, 2^8), q1 = q truncated to 4
    significant bits and q2 = q - q1.  Over every finite bf16 value (as the largest component,
    and as a component 2^k below it): q1 + q2 reproduces q exactly whenever q >= 2^-1 after the
    shift (8 of a bf16's bits fit in two 4-bit terms), and within 2^-9 below that."""
    bits = np.arange(65536, dtype=np.uint32)
    vals = (bits << 16).view(np.float32)
    vals = vals[np.isfinite(vals) & (vals != 0)]
    e4 = lambda b: torch.from_numpy(b).view(torch.float8_e4m3fn).float().numpy()
    for k in (0, 3, 7, 12, 20):  # the component sits 2^k below the head's largest |q|
        e = np.floor(np.log2(np.abs(vals))).astype(np.int64)
        x = np.ldexp(np.abs(vals) / np.exp2(e), 7 - k).astype(np.float32) * np.sign(vals)  # same mantissa
        h = _e4m3_head(x)
        rec = e4(_e4m3_byte(h)) + e4(_e4m3_byte((x - h).astype(np.float32)))
        err = np.abs(rec - x.astype(np.float64))
        exact = np.abs(x) >= 0.5
        assert np.all(err[exact] == 0), k
        assert np.all(err <= 2.0 ** -9), (k, float(err.max()))
