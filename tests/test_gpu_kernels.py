"""GPU parity of every kernel behind the C ABI against the CPU oracle (and the reference's
golden fixtures).  Tolerances: integer / byte outputs bit-exact; BF16 attention within
rtol 2e-2 / atol 2e-3 of the fp32 oracle, FP8-KV attention within atol 6e-2 (BASELINE
north_star); elementwise layer kernels within 1 bf16 ulp of the reference modules."""

import numpy as np
import pytest
import torch

from hilda_vllm_b200 import kernels
from oracle import attention as oattn
from oracle import kv_store

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_TOL = dict(rtol=2e-2, atol=2e-3)


def bf(a):
    return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)


def assert_close(got, want, rtol, atol, what=""):
    got, want = got.float().cpu(), want.float().cpu()
    err = (got - want).abs()
    bad = err > atol + rtol * want.abs()
    assert not bad.any(), f"{what}: {int(bad.sum())} / {bad.numel()} out of tolerance, max err {err.max():.3e}"


def make_paged(g, b, hk, d, nb, bs, lens, dtype=torch.bfloat16):
    k = torch.randn(nb, bs, hk, d, generator=g).to(dtype)
    v = torch.randn(nb, bs, hk, d, generator=g).to(dtype)
    mb = max(1, max(-(-n // bs) for n in lens))
    perm = torch.randperm(nb, generator=g).tolist()
    tables, off = [], 0
    for n in lens:
        nblk = -(-n // bs)
        tables.append(perm[off:off + nblk] + [-1] * (mb - nblk))
        off += nblk
    assert off <= nb
    return k, v, torch.tensor(tables, dtype=torch.int32), torch.tensor(lens, dtype=torch.int32)


# ----------------------------------------------------------------------------- store
def test_store_bf16_matches_reference_golden(golden_dir):
    g = np.load(golden_dir / "store_kv.npz")
    n, hq, hk, d, nb, bs = g["shape"].tolist()
    qkv = bf(g["qkv"]).to(DEV)
    key = qkv[:, hq * d:(hq + hk) * d].view(n, hk, d)
    value = qkv[:, (hq + hk) * d:].view(n, hk, d)
    kc = torch.zeros(nb, bs, hk, d, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    kernels.store_kvcache(key, value, kc, vc, torch.from_numpy(g["slot_mapping"]).to(DEV))
    rows = torch.from_numpy(g["touched_slots"]).to(DEV)
    assert torch.equal(kc.view(-1, hk * d)[rows].view(torch.int16).cpu(), torch.from_numpy(g["k_rows"]))
    assert torch.equal(vc.view(-1, hk * d)[rows].view(torch.int16).cpu(), torch.from_numpy(g["v_rows"]))
    nz = torch.nonzero(kc.view(-1, hk * d).float().abs().sum(1)).flatten().cpu()
    assert nz.tolist() == g["k_nonzero_rows"].tolist()


@pytest.mark.parametrize("n,hk", [(1, 8), (256, 8), (3000, 8), (77, 1), (64, 4)])
def test_store_bf16_random(n, hk):
    g = torch.Generator().manual_seed(n)
    d, nb, bs = 128, 64, 256
    qkv = torch.randn(n, (2 * hk + 2 * hk) * d, generator=g).bfloat16()
    key = qkv[:, 2 * hk * d:3 * hk * d].view(n, hk, d)
    value = qkv[:, 3 * hk * d:].view(n, hk, d)
    slots = torch.randperm(nb * bs, generator=g)[:n].to(torch.int32)
    slots[::7] = -1
    kc = torch.randn(nb, bs, hk, d, generator=g).bfloat16()
    vc = torch.randn(nb, bs, hk, d, generator=g).bfloat16()
    kd, vd = kc.to(DEV), vc.to(DEV)
    qd = qkv.to(DEV)  # strided key/value views into a fused projection, as in the model
    kernels.store_kvcache(qd[:, 2 * hk * d:3 * hk * d].view(n, hk, d), qd[:, 3 * hk * d:].view(n, hk, d), kd, vd,
                          slots.to(DEV))
    kv_store.store_kvcache(key, value, kc, vc, slots)
    assert torch.equal(kd.cpu(), kc) and torch.equal(vd.cpu(), vc)


@pytest.mark.parametrize("hk,scaled", [(8, False), (8, True), (2, True)])
def test_store_fp8_bit_exact(hk, scaled):
    g = torch.Generator().manual_seed(hk + scaled)
    n, d, nb, bs = 300, 128, 8, 256
    key = (torch.randn(n, hk, d, generator=g) * torch.logspace(-4, 3, n).view(n, 1, 1)).bfloat16()
    value = (torch.randn(n, hk, d, generator=g) * 3).bfloat16()
    key[0, 0, :4] = torch.tensor([1e6, -1e6, 448.0, 2 ** -10]).bfloat16()
    ks = (torch.rand(hk, generator=g) * 4 + 0.1) if scaled else None
    vs = (torch.rand(hk, generator=g) * 0.5 + 0.05) if scaled else None
    slots = torch.randperm(nb * bs, generator=g)[:n].to(torch.int32)
    slots[5] = -1
    kc = torch.zeros(nb, bs, hk, d, dtype=torch.uint8)
    vc = torch.zeros_like(kc)
    kv_store.store_kvcache_fp8(key, value, kc, vc, slots, ks, vs)
    kd = torch.zeros(nb, bs, hk, d, dtype=torch.float8_e4m3fn, device=DEV)
    vd = torch.zeros_like(kd)
    kernels.store_kvcache_fp8(key.to(DEV), value.to(DEV), kd, vd, slots.to(DEV),
                              None if ks is None else ks.to(DEV), None if vs is None else vs.to(DEV))
    assert torch.equal(kd.view(torch.uint8).cpu(), kc)
    assert torch.equal(vd.view(torch.uint8).cpu(), vc)


def test_copy_bf16_to_fp8_all_layers_bit_exact():
    g = torch.Generator().manual_seed(9)
    layers, nb, bs, hk, d = 3, 6, 256, 8, 128
    src = (torch.randn(2, layers, nb, bs, hk, d, generator=g) * 20).bfloat16()
    scales = torch.rand(2, layers, hk, generator=g) + 0.2
    slots = torch.randperm(nb * bs, generator=g)[:700].to(torch.int32)
    dst = torch.zeros(2, layers, nb, bs, hk, d, dtype=torch.float8_e4m3fn, device=DEV)
    kernels.copy_kvcache_fp8_layers(src[0].to(DEV), src[1].to(DEV), dst[0], dst[1], slots.to(DEV),
                                    scales[0].contiguous().to(DEV), scales[1].contiguous().to(DEV))
    for layer in range(layers):
        want_k = torch.zeros(nb, bs, hk, d, dtype=torch.uint8)
        want_v = torch.zeros_like(want_k)
        kv_store.copy_kvcache_fp8(src[0, layer], src[1, layer], want_k, want_v, slots, scales[0, layer],
                                  scales[1, layer])
        assert torch.equal(dst[0, layer].view(torch.uint8).cpu(), want_k)
        assert torch.equal(dst[1, layer].view(torch.uint8).cpu(), want_v)


# ----------------------------------------------------------------------------- decode
def run_decode(q, k, v, bt, lens, scale, fp8=False, ks=None, vs=None, ws=None, tensor_cores=False):
    if fp8:
        kd = k.to(DEV).view(torch.float8_e4m3fn)
        vd = v.to(DEV).view(torch.float8_e4m3fn)
    else:
        kd, vd = k.to(DEV), v.to(DEV)
    return kernels.paged_decode(q.to(DEV), kd, vd, bt.to(DEV), lens.to(DEV), scale, workspace=ws,
                                k_scale=None if ks is None else ks.to(DEV),
                                v_scale=None if vs is None else vs.to(DEV), tensor_cores=tensor_cores)


def test_decode_config1_shapes():
    """8 sequences, lens ~ U[16,1024], 16 Q / 8 KV heads, 64 blocks of 256."""
    g = torch.Generator().manual_seed(1)
    lens = torch.randint(16, 1025, (8,), generator=g).tolist()
    k, v, bt, ln = make_paged(g, 8, 8, 128, 64, 256, lens)
    q = torch.randn(8, 16, 128, generator=g).bfloat16()
    out = run_decode(q, k, v, bt, ln, 128 ** -0.5)
    want = oattn.paged_decode(q, k, v, bt, ln, 128 ** -0.5)
    assert_close(out, want, **BF16_TOL, what="config1")


EDGE_LENS = [0, 1, 2, 127, 128, 129, 255, 256, 257, 511, 512, 1000, 1024, 1025, 2047, 3000, 4096]


@pytest.mark.parametrize("hq,hk", [(16, 8), (32, 8), (8, 8), (16, 4), (8, 2), (8, 1), (64, 8), (4, 4), (2, 1)])
def test_decode_gqa_layouts_and_edge_lengths(hq, hk):
    g = torch.Generator().manual_seed(hq * 10 + hk)
    lens = EDGE_LENS
    k, v, bt, ln = make_paged(g, len(lens), hk, 128, 96, 256, lens)
    q = torch.randn(len(lens), hq, 128, generator=g).bfloat16()
    out = run_decode(q, k, v, bt, ln, 128 ** -0.5)
    want = oattn.paged_decode(q, k, v, bt, ln, 128 ** -0.5)
    assert torch.all(out[0] == 0)
    assert torch.isfinite(out).all()
    assert_close(out, want, **BF16_TOL, what=f"hq={hq} hk={hk}")


def test_decode_workspace_reuse_and_padding_rows():
    """Two launches sharing one workspace (tickets must be reset), with padding rows
    (context 0, block table -1) as the CUDA graph buckets produce."""
    g = torch.Generator().manual_seed(3)
    lens = [700, 0, 300, 0, 1]
    k, v, bt, ln = make_paged(g, 5, 8, 128, 16, 256, lens)
    ws = kernels.make_decode_workspace(5, 16, 128, bt.shape[1], 256, DEV)
    for trial in range(3):
        q = torch.randn(5, 16, 128, generator=g).bfloat16()
        out = run_decode(q, k, v, bt, ln, 0.1, ws=ws)
        want = oattn.paged_decode(q, k, v, bt, ln, 0.1)
        assert_close(out, want, **BF16_TOL, what=f"trial {trial}")
    assert kernels.decode_errors(ws) == 0


def test_decode_large_batch():
    g = torch.Generator().manual_seed(4)
    lens = torch.randint(65, 1089, (256,), generator=g).tolist()
    k, v, bt, ln = make_paged(g, 256, 8, 128, 1400, 256, lens)
    q = torch.randn(256, 16, 128, generator=g).bfloat16()
    out = run_decode(q, k, v, bt, ln, 128 ** -0.5)
    idx = list(range(0, 256, 9))
    want = oattn.paged_decode(q[idx], k, v, bt[idx], ln[idx], 128 ** -0.5)
    assert_close(out[idx], want, **BF16_TOL, what="B=256")


def test_decode_inside_cuda_graph():
    g = torch.Generator().manual_seed(5)
    lens = [300, 17, 1024, 5]
    k, v, bt, ln = make_paged(g, 4, 8, 128, 32, 256, [1024] * 4)
    kd, vd, btd = k.to(DEV), v.to(DEV), bt.to(DEV)
    lnd = torch.zeros(4, dtype=torch.int32, device=DEV)
    qd = torch.zeros(4, 16, 128, dtype=torch.bfloat16, device=DEV)
    out = torch.zeros(4, 16, 128, dtype=torch.bfloat16, device=DEV)
    ws = kernels.make_decode_workspace(4, 16, 128, bt.shape[1], 256, DEV)
    kernels.paged_decode(qd, kd, vd, btd, lnd, 0.1, out=out, workspace=ws)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        kernels.paged_decode(qd, kd, vd, btd, lnd, 0.1, out=out, workspace=ws)
    for trial in range(3):
        q = torch.randn(4, 16, 128, generator=g).bfloat16()
        L = torch.tensor([(x * (trial + 1)) % 1025 for x in lens], dtype=torch.int32)
        qd.copy_(q)
        lnd.copy_(L)
        graph.replay()
        want = oattn.paged_decode(q, k, v, bt, L, 0.1)
        assert_close(out, want, **BF16_TOL, what=f"graph replay {trial}")


@pytest.mark.parametrize("hq,hk", [(32, 8), (64, 8)])
def test_decode_cuda_core_kernel_at_high_gqa_ratio(hq, hk):
    """hl_paged_decode runs the tensor-core kernel for BF16 caches with Hq/Hk >= 4 up to 2048
    sequences and the CUDA-core kernel beyond; a 2100-sequence batch (sequences share pages of a
    small pool) keeps the CUDA-core kernel's G = 4 / 8 instantiations covered."""
    g = torch.Generator().manual_seed(hq)
    b, nb, bs = 2100, 12, 256
    lens = torch.randint(0, 700, (b,), generator=g)
    lens[:4] = torch.tensor([0, 1, 256, 699])
    k = torch.randn(nb, bs, hk, 128, generator=g).bfloat16()
    v = torch.randn(nb, bs, hk, 128, generator=g).bfloat16()
    bt = torch.randint(0, nb, (b, 3), generator=g, dtype=torch.int32)
    q = torch.randn(b, hq, 128, generator=g).bfloat16()
    ws = kernels.make_decode_workspace(b, hq, 128, 3, bs, DEV)
    out = kernels.paged_decode(q.to(DEV), k.to(DEV), v.to(DEV), bt.to(DEV), lens.to(torch.int32).to(DEV),
                               128 ** -0.5, workspace=ws)
    torch.cuda.synchronize()
    assert kernels.decode_errors(ws) == 0
    idx = list(range(4)) + list(range(5, b, 97))
    want = oattn.paged_decode(q[idx], k, v, bt[idx], lens[idx].to(torch.int32), 128 ** -0.5)
    assert_close(out[idx], want, **BF16_TOL, what=f"CUDA-core decode hq={hq} hk={hk} B={b}")
    assert torch.all(out[0] == 0)


@pytest.mark.parametrize("case", ["one_long", "mixed_long", "many_short", "g16"])
def test_decode_tensor_core_against_oracle_and_cuda_core(case):
    """The tcgen05 decode kernel (hl_paged_decode_tc) against the fp32 oracle and the
    CUDA-core kernel: one 20k-token sequence (each KV head's tiles spread over ~18 CTAs, merged
    by the last one), long and short sequences mixed, many short ones, and G = 16."""
    g = torch.Generator().manual_seed({"one_long": 1, "mixed_long": 2, "many_short": 3, "g16": 4}[case])
    hq, hk = 16, 8
    if case == "one_long":
        lens = [20000]
    elif case == "mixed_long":
        lens = [9000, 1, 0, 300, 4097, 128, 129, 6000]
    elif case == "many_short":
        lens = torch.randint(0, 200, (300,), generator=g).tolist()
    else:
        hq, hk = 32, 2
        lens = [777, 2048, 5, 0]
    nblocks = sum(-(-n // 256) for n in lens) + 4
    k, v, bt, ln = make_paged(g, len(lens), hk, 128, nblocks, 256, lens)
    q = torch.randn(len(lens), hq, 128, generator=g).bfloat16()
    ws = kernels.make_decode_workspace(len(lens), hq, 128, bt.shape[1], 256, DEV)
    kd, vd, btd, lnd, qd = k.to(DEV), v.to(DEV), bt.to(DEV), ln.to(DEV), q.to(DEV)
    for trial in range(2):  # tickets must be back at zero for the second launch
        out = kernels.paged_decode(qd, kd, vd, btd, lnd, 128 ** -0.5, workspace=ws, tensor_cores=True)
        torch.cuda.synchronize()
        assert kernels.decode_errors(ws) == 0
        idx = list(range(len(lens))) if len(lens) <= 16 else list(range(0, len(lens), 7))
        want = oattn.paged_decode(q[idx], k, v, bt[idx], ln[idx], 128 ** -0.5)
        assert_close(out[idx], want, **BF16_TOL, what=f"tensor-core decode {case} trial {trial}")
    if hq // hk <= 8:  # the CUDA-core kernel covers GQA ratios 1, 2, 4, 8
        cc = kernels.paged_decode(qd, kd, vd, btd, lnd, 128 ** -0.5, workspace=ws)
        assert_close(out.float().cpu(), cc.float().cpu(), rtol=2e-2, atol=2e-3, what="tensor-core vs CUDA-core")
    for i, n in enumerate(lens):
        if n == 0:
            assert torch.all(out[i] == 0)


@pytest.mark.parametrize("hq,hk,scaled,tc", [(16, 8, False, False), (16, 8, True, False), (32, 8, True, False),
                                             (8, 1, True, False), (16, 8, True, True), (8, 8, True, True),
                                             (16, 2, False, True)])
def test_decode_fp8(hq, hk, scaled, tc):
    """e4m3 caches with per-head scales.  Hq/Hk >= 4 runs the tensor-core kernel by default;
    tc=True forces it for the smaller ratios."""
    g = torch.Generator().manual_seed(7 + hq)
    lens = [0, 1, 129, 256, 700, 1500]
    kb, vb, bt, ln = make_paged(g, len(lens), hk, 128, 24, 256, lens)
    ks = (torch.rand(hk, generator=g) + 0.5) if scaled else None
    vs = (torch.rand(hk, generator=g) + 0.5) if scaled else None
    kq = kv_store.quantize_e4m3(kb, ks)
    vq = kv_store.quantize_e4m3(vb, vs)
    q = torch.randn(len(lens), hq, 128, generator=g).bfloat16()
    out = run_decode(q, kq, vq, bt, ln, 128 ** -0.5, fp8=True, ks=ks, vs=vs, tensor_cores=tc)
    want = oattn.paged_decode(q, kq, vq, bt, ln, 128 ** -0.5, ks, vs, fp8=True)
    assert_close(out, want, rtol=2e-2, atol=6e-2, what="fp8")
    assert_close(out, want, **BF16_TOL, what="fp8 (tight)")


# ----------------------------------------------------------------------------- packing
@pytest.mark.parametrize("name", ["sched_trace_churn", "sched_trace_prefix", "sched_trace_complete"])
def test_pack_kernel_replays_reference_trace(golden_dir, seq_block_size, name):
    from tests.test_trace_parity import _load, _replay
    from hilda_vllm_b200.engine.decode_packer import DecodePacker, packet_capacity_bytes

    trace = _load(golden_dir, name)
    meta = trace["meta"]
    bs, max_bs = meta["block_size"], meta["max_bs"]
    mb = -(-meta["max_model_len"] // bs)
    cap = (packet_capacity_bytes(max_bs, mb) + 15) & ~15
    host = torch.zeros(cap, dtype=torch.uint8)
    packer = DecodePacker(max_bs, mb, host.numpy())
    pkt = torch.zeros(cap, dtype=torch.uint8, device=DEV)
    st = dict(input_ids=torch.zeros(max_bs, dtype=torch.int64, device=DEV),
              positions=torch.zeros(max_bs, dtype=torch.int64, device=DEV),
              slot_mapping=torch.full((max_bs,), -1, dtype=torch.int32, device=DEV),
              context_lens=torch.zeros(max_bs, dtype=torch.int32, device=DEV),
              block_tables=torch.full((max_bs, mb), -1, dtype=torch.int32, device=DEV))
    seq_ids = torch.full((max_bs,), -1, dtype=torch.int64, device=DEV)
    bt_lens = torch.zeros(max_bs, dtype=torch.int32, device=DEV)
    next_tokens = torch.zeros(max_bs, dtype=torch.int64, device=DEV)
    n = [0]

    def check(rec, scheduled, is_prefill):
        if is_prefill:
            return
        graph_bs = rec["graph_bs"]
        nbytes = packer.build(scheduled, graph_bs)
        pkt[:nbytes].copy_(host[:nbytes])
        kernels.pack_decode_batch(pkt, graph_bs, bs, seq_ids, bt_lens, next_tokens, st["input_ids"],
                                  st["positions"], st["slot_mapping"], st["context_lens"], st["block_tables"])
        for key, want in rec["decode"].items():
            got = st[key][:graph_bs].cpu().numpy()
            np.testing.assert_array_equal(got, np.asarray(want), err_msg=key)
        toks = [0 if t is None else t for t in rec["tokens"]]
        next_tokens[: len(toks)] = torch.tensor(toks, device=DEV)
        packer.note_sampled(len(toks), toks)
        n[0] += 1

    _replay(trace, seq_block_size, check)
    assert n[0] > 10


# ----------------------------------------------------------------------------- layer kernels
def ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    ai = a.view(torch.int16).to(torch.int32)
    bi = b.view(torch.int16).to(torch.int32)
    # map sign-magnitude to a monotonic integer line
    ai = torch.where(ai < 0, -(ai & 0x7FFF), ai)
    bi = torch.where(bi < 0, -(bi & 0x7FFF), bi)
    return (ai - bi).abs()


def assert_ulps(got, want_bits, what):
    d = ulp_diff(got.cpu().contiguous(), torch.from_numpy(want_bits).view(torch.bfloat16))
    assert int(d.max()) <= 1, f"{what}: max {int(d.max())} ulp"
    assert float((d > 0).float().mean()) < 0.02, f"{what}: {float((d > 0).float().mean()):.3%} differ"


def test_rmsnorm_kernels_match_reference_modules(golden_dir):
    g = np.load(golden_dir / "layers.npz")
    x, r, w = bf(g["rms_x"]).to(DEV), bf(g["rms_r"]).to(DEV), bf(g["rms_w"]).to(DEV)
    assert_ulps(kernels.rmsnorm(x, w, 1e-6), g["rms_y"], "rmsnorm")
    res = r.clone()
    y, res = kernels.rmsnorm(x, w, 1e-6, residual=res)
    assert_ulps(y, g["add_y"], "add_rmsnorm")
    assert torch.equal(res.cpu().view(torch.int16), torch.from_numpy(g["add_r"]))


def test_qk_norm_rope_matches_reference_modules(golden_dir):
    from hilda_vllm_b200.layers.rotary_embedding import RotaryEmbedding
    g = np.load(golden_dir / "layers.npz")
    q = bf(g["rope_q"])  # [T, 4, 128]: heads 0-1 act as q heads, head 2 as the k head (same weight)
    t = q.shape[0]
    w = bf(g["rope_w"]).to(DEV)
    qkv = torch.cat([q.reshape(t, -1)[:, :3 * 128], torch.zeros(t, 128, dtype=torch.bfloat16)], 1).to(DEV)
    rope = RotaryEmbedding(128, 128, 4096, 1000000.0)
    cos_sin = rope.cos_sin_cache.to(DEV).contiguous()
    kernels.qk_norm_rope(qkv, 2, 1, 128, w, w, cos_sin, torch.from_numpy(g["rope_pos"]).to(DEV), 1e-6)
    want = g["rope_out"].reshape(t, -1)
    assert_ulps(qkv[:, :3 * 128], want[:, :3 * 128], "qk_norm_rope")
    assert torch.all(qkv[:, 3 * 128:] == 0)  # v untouched


@pytest.mark.parametrize("kv,hq,hk,n", [("bf16", 16, 8, 300), ("fp8", 16, 8, 257), ("fp8s", 8, 2, 64),
                                        ("bf16", 4, 1, 1), ("fp8m", 16, 8, 129), ("fp8sm", 8, 2, 64)])
def test_fused_rope_store_equals_rope_then_store(kv, hq, hk, n):
    """hl_qk_norm_rope_store == hl_qk_norm_rope followed by the store kernel, byte for byte, in
    the qkv rows and in both caches (strided rows, skipped slots, untouched cache rows).  "m" cases:
    the FP8 store with bf16 mirror caches (hl_qk_norm_rope_store_mirrored), whose mirror rows must
    equal the BF16 store of the same rotated rows."""
    from hilda_vllm_b200.layers.rotary_embedding import RotaryEmbedding
    g = torch.Generator().manual_seed(n + hq)
    d, nb, bs = 128, 8, 256
    width = (hq + 2 * hk) * d
    qkv = (torch.randn(n, width, generator=g) * 2).bfloat16()
    qw = (torch.rand(d, generator=g) + 0.5).bfloat16().to(DEV)
    kw = (torch.rand(d, generator=g) + 0.5).bfloat16().to(DEV)
    pos = torch.randint(0, 4000, (n,), generator=g).to(DEV)
    slots = torch.randperm(nb * bs, generator=g)[:n].to(torch.int32)
    slots[::5] = -1
    slots = slots.to(DEV)
    cos_sin = RotaryEmbedding(d, d, 4096, 1000000.0).cos_sin_cache.to(DEV).contiguous()
    fp8 = kv != "bf16"
    mirrored = kv.endswith("m")
    ks = (torch.rand(hk, generator=g) + 0.3).to(DEV) if kv.startswith("fp8s") else None
    vs = (torch.rand(hk, generator=g) + 0.3).to(DEV) if kv.startswith("fp8s") else None
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    init = torch.randn(nb, bs, hk, d, generator=g).to(dt)
    caches = [[init.clone().to(DEV), init.clone().to(DEV)] for _ in range(2)]
    rows = []
    for _ in range(2):
        buf = torch.zeros(n, width + 64, dtype=torch.bfloat16, device=DEV)
        buf[:, :width] = qkv.to(DEV)
        rows.append(buf[:, :width])
    # separate: rotate, then store the strided k / v views
    kernels.qk_norm_rope(rows[0], hq, hk, d, qw, kw, cos_sin, pos, 1e-6)
    k = rows[0][:, hq * d:(hq + hk) * d].view(n, hk, d)
    v = rows[0][:, (hq + hk) * d:].view(n, hk, d)
    minit = torch.randn(nb, bs, hk, d, generator=g).bfloat16()
    mirrors = [[minit.clone().to(DEV), minit.clone().to(DEV)] for _ in range(2)] if mirrored else [[None, None]] * 2
    if fp8:
        kernels.store_kvcache_fp8(k, v, caches[0][0], caches[0][1], slots, ks, vs)
        if mirrored:
            kernels.store_kvcache(k, v, mirrors[0][0], mirrors[0][1], slots)
    else:
        kernels.store_kvcache(k, v, caches[0][0], caches[0][1], slots)
    kernels.qk_norm_rope_store(rows[1], hq, hk, d, qw, kw, cos_sin, pos, 1e-6, caches[1][0], caches[1][1], slots,
                               ks, vs, k_mirror=mirrors[1][0], v_mirror=mirrors[1][1])
    assert rows[1].stride(0) == width + 64
    assert torch.equal(rows[0].contiguous().view(torch.int16), rows[1].contiguous().view(torch.int16))
    for a, b in zip(caches[0], caches[1]):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    if mirrored:
        for a, b in zip(mirrors[0], mirrors[1]):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))
        assert not torch.equal(mirrors[1][0].cpu().view(torch.int16), minit.view(torch.int16))  # rows were written


def test_silu_mul_matches_reference_module(golden_dir):
    g = np.load(golden_dir / "layers.npz")
    a = bf(g["silu_in"]).to(DEV)
    assert_ulps(kernels.silu_mul(a), g["silu_out"], "silu_mul")


def test_argmax_lowest_index_on_ties():
    g = torch.Generator().manual_seed(13)
    logits = torch.randn(37, 151936, generator=g).bfloat16()
    logits[5, 100] = logits[5, 2000] = 50.0  # tie -> 100
    logits[6, :] = -1.0
    got = kernels.argmax(logits.to(DEV)).cpu()
    assert got[5] == 100 and got[6] == 0
    assert torch.equal(got, logits.float().argmax(-1))


# ----------------------------------------------------------------------------- device sampling
def test_sample_greedy_rows_equal_argmax_and_shards_merge():
    """hl_sample: temperature-0 rows are the argmax; with temperatures, sampling two vocabulary
    shards (index_offset) and keeping the larger perturbed value gives the same token as sampling
    the whole row (the noise is a function of the global index)."""
    g = torch.Generator().manual_seed(17)
    rows, vocab = 64, 151936
    logits = torch.randn(rows, vocab, generator=g).bfloat16().to(DEV)
    zero = torch.zeros(rows, dtype=torch.float32, device=DEV)
    assert torch.equal(kernels.sample(logits, zero, 5, None).cpu(), kernels.argmax(logits).cpu())
    temps = (torch.rand(rows, generator=g) + 0.3).to(DEV)
    full = kernels.sample(logits, temps, 5, None)
    half = vocab // 2
    vals, idxs = [], []
    for off in (0, half):
        v = torch.empty(rows, dtype=torch.float32, device=DEV)
        i = kernels.sample(logits[:, off:off + half].contiguous(), temps, 5, None, index_offset=off, out_values=v)
        vals.append(v)
        idxs.append(i)
    merged = torch.where(vals[1] > vals[0], idxs[1], idxs[0])
    assert torch.equal(merged.cpu(), full.cpu())


def test_sample_matches_softmax_distribution():
    """Empirical token frequencies of Gumbel-max sampling (the step counter advancing per launch)
    match softmax(logits / T) — the reference Sampler's distribution — within sampling error."""
    g = torch.Generator().manual_seed(23)
    rows, vocab, T = 512, 16, 0.7
    base = torch.randn(vocab, generator=g) * 1.5
    logits = base.bfloat16().repeat(rows, 1).to(DEV)
    temps = torch.full((rows,), T, dtype=torch.float32, device=DEV)
    state = torch.zeros(2, dtype=torch.int64, device=DEV)
    counts = torch.zeros(vocab, dtype=torch.float64)
    launches = 40
    for _ in range(launches):
        tok = kernels.sample(logits, temps, 1234, state)
        counts += torch.bincount(tok.cpu(), minlength=vocab).double()
    assert int(state[0].item()) == launches and int(state[1].item()) == 0
    freq = counts / counts.sum()
    want = torch.softmax(base.bfloat16().float() / T, -1).double()
    n = rows * launches
    assert float((freq - want).abs().max()) < 5 * float((want * (1 - want) / n).sqrt().max()) + 1e-4


# ----------------------------------------------------------------------------- flash-attn pin
def _flash_attn():
    try:
        from flash_attn import flash_attn_varlen_func, flash_attn_with_kvcache
    except Exception:  # pragma: no cover - depends on the installed wheel
        return None
    return flash_attn_varlen_func, flash_attn_with_kvcache


def test_oracle_and_kernels_agree_with_flash_attn_when_it_runs():
    """The reference calls flash-attn 2.x (attention.py:149-170).  Where the installed wheel runs
    on this GPU, the fp32 oracle and our kernels are compared with it on the reference's exact
    call signatures (this pins the oracle's restatement of flash-attn's semantics)."""
    fa = _flash_attn()
    if fa is None:
        pytest.skip("flash-attn not importable")
    varlen, with_kvcache = fa
    g = torch.Generator().manual_seed(21)
    lens = [1, 100, 256, 700, 1024]
    k, v, bt, ln = make_paged(g, len(lens), 8, 128, 24, 256, lens)
    q = torch.randn(len(lens), 16, 128, generator=g).bfloat16()
    try:
        ref = with_kvcache(q.to(DEV).unsqueeze(1), k.to(DEV), v.to(DEV), cache_seqlens=ln.to(DEV),
                           block_table=bt.to(DEV), softmax_scale=128 ** -0.5, causal=True).squeeze(1)
        torch.cuda.synchronize()
    except Exception as exc:  # the wheel may not carry sm_100 code
        pytest.skip(f"flash-attn does not run here: {type(exc).__name__}: {exc}")
    want = oattn.paged_decode(q, k, v, bt, ln, 128 ** -0.5)
    assert_close(ref, want, **BF16_TOL, what="flash-attn decode vs oracle")
    out = run_decode(q, k, v, bt, ln, 128 ** -0.5)
    assert_close(out, ref.float(), **BF16_TOL, what="ours vs flash-attn decode")
    # varlen prefill with prefix pages (the chunked-prefill call, attention.py:149-160)
    starts, chunks = [0, 256, 40], [64, 128, 300]
    kl = [s + c for s, c in zip(starts, chunks)]
    k2, v2, bt2, _ = make_paged(g, 3, 8, 128, 12, 256, kl)
    cuq = torch.tensor([0] + np.cumsum(chunks).tolist(), dtype=torch.int32)
    cuk = torch.tensor([0] + np.cumsum(kl).tolist(), dtype=torch.int32)
    q2 = torch.randn(int(cuq[-1]), 16, 128, generator=g).bfloat16()
    ref2 = varlen(q2.to(DEV), k2.to(DEV), v2.to(DEV), max_seqlen_q=max(chunks), cu_seqlens_q=cuq.to(DEV),
                  max_seqlen_k=max(kl), cu_seqlens_k=cuk.to(DEV), softmax_scale=128 ** -0.5, causal=True,
                  block_table=bt2.to(DEV))
    want2 = oattn.varlen_prefill(q2, k2, v2, cuq, cuk, 128 ** -0.5, block_table=bt2)
    assert_close(ref2, want2, **BF16_TOL, what="flash-attn varlen vs oracle")


# ----------------------------------------------------------------------------- tcgen05 prefill
@pytest.mark.parametrize("hq,hk,lens,one_head", [
    (16, 8, [1, 5, 64, 64, 130, 257, 31], False),
    (16, 8, [1, 5, 64, 64, 130, 257, 31], True),
    (16, 8, [128, 256, 1000], False),
    (32, 8, [300, 7], False),
    (8, 1, [513], False),
    (4, 4, [200, 129], False),  # Hq / Hk odd: the one-head kernel
])
def test_prefill_tensor_core_contiguous(hq, hk, lens, one_head):
    g = torch.Generator().manual_seed(31 + hq + len(lens))
    cu = torch.tensor([0] + np.cumsum(lens).tolist(), dtype=torch.int32)
    t = int(cu[-1])
    qkv = torch.randn(t, (hq + 2 * hk) * 128, generator=g).bfloat16()
    q = qkv[:, :hq * 128].view(t, hq, 128)
    k = qkv[:, hq * 128:(hq + hk) * 128].view(t, hk, 128)
    v = qkv[:, (hq + hk) * 128:].view(t, hk, 128)
    qd = qkv.to(DEV)
    out = kernels.varlen_prefill(qd[:, :hq * 128].view(t, hq, 128), qd[:, hq * 128:(hq + hk) * 128].view(t, hk, 128),
                                    qd[:, (hq + hk) * 128:].view(t, hk, 128), cu.to(DEV), cu.to(DEV), max(lens),
                                    max(lens), 128 ** -0.5, one_head_per_cta=one_head)
    torch.cuda.synchronize()
    assert kernels.prefill_errors() == 0
    want = oattn.varlen_prefill(q, k, v, cu, cu, 128 ** -0.5)
    assert_close(out, want, **BF16_TOL, what="tcgen05 prefill contiguous")


@pytest.mark.parametrize("precise,one_head", [(True, False), (True, True), (False, False)])
def test_prefill_tensor_core_large_scores_rescale(precise, one_head):
    """Scores with a spread of hundreds (q scaled by 8): the running max jumps by far more
    than the lazy-rescale threshold from tile to tile, so O is rescaled in TMEM often."""
    g = torch.Generator().manual_seed(77)
    hq, hk, lens = 16, 8, [700, 260, 1]
    cu = torch.tensor([0] + np.cumsum(lens).tolist(), dtype=torch.int32)
    t = int(cu[-1])
    q = (torch.randn(t, hq, 128, generator=g) * 8).bfloat16()
    k = torch.randn(t, hk, 128, generator=g).bfloat16()
    v = torch.randn(t, hk, 128, generator=g).bfloat16()
    out = kernels.varlen_prefill(q.to(DEV), k.to(DEV), v.to(DEV), cu.to(DEV), cu.to(DEV), max(lens), max(lens),
                                 128 ** -0.5, precise_p=precise, one_head_per_cta=one_head)
    torch.cuda.synchronize()
    assert kernels.prefill_errors() == 0
    want = oattn.varlen_prefill(q, k, v, cu, cu, 128 ** -0.5)
    if precise:
        assert_close(out, want, **BF16_TOL, what="tcgen05 prefill, large scores")
    else:
        # bf16-rounded P (flash-attn's own precision, the non-default mode): P carries 2^-9
        # relative rounding, so at this score spread ~4e-5 of the outputs miss atol 2e-3.  Check
        # against a 2x absolute floor, allowing 1e-5 of the outputs past it, and a hard bound.
        err = (out.float().cpu() - want.float()).abs()
        over = err > 2 * BF16_TOL["atol"] + BF16_TOL["rtol"] * want.float().abs()
        assert int(over.sum()) <= max(1, err.numel() // 100000) and float(err.max()) < 4e-2


def test_prefill_block_outside_the_pool_sets_error_bit():
    """A key tile whose block id lies outside the pool reads zeros (TMA fill, no fault) and sets
    bit 1 of the prefill error word; clearing the word restores zero."""
    from hilda_vllm_b200 import _lib
    g = torch.Generator().manual_seed(77)
    hq, hk, bs, nb = 16, 8, 256, 8
    k, v, bt, _ = make_paged(g, 1, hk, 128, nb, bs, [600])
    bad = bt.clone()
    bad[0, 1] = nb + 3
    cuq = torch.tensor([0, 88], dtype=torch.int32)
    cuk = torch.tensor([0, 600], dtype=torch.int32)
    q = torch.randn(88, hq, 128, generator=g).bfloat16()
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.hl_varlen_prefill_clear_errors(stream) == 0
    kernels.varlen_prefill(q.to(DEV), k.to(DEV), v.to(DEV), cuq.to(DEV), cuk.to(DEV), 88, 600, 128 ** -0.5,
                           block_table=bad.to(DEV))
    torch.cuda.synchronize()
    assert kernels.prefill_errors() & 2
    assert lib.hl_varlen_prefill_clear_errors(stream) == 0
    assert kernels.prefill_errors() == 0


@pytest.mark.parametrize("one_head", [False, True])
def test_prefill_tensor_core_paged_with_prefix_chunks(one_head):
    g = torch.Generator().manual_seed(41)
    hq, hk, bs, nb = 16, 8, 256, 40
    starts = [0, 256, 100, 512, 2048, 3]
    chunks = [64, 128, 1, 300, 512, 700]
    kl = [s + c for s, c in zip(starts, chunks)]
    k, v, bt, _ = make_paged(g, len(kl), hk, 128, nb, bs, kl)
    cuq = torch.tensor([0] + np.cumsum(chunks).tolist(), dtype=torch.int32)
    cuk = torch.tensor([0] + np.cumsum(kl).tolist(), dtype=torch.int32)
    q = torch.randn(int(cuq[-1]), hq, 128, generator=g).bfloat16()
    out = kernels.varlen_prefill(q.to(DEV), k.to(DEV), v.to(DEV), cuq.to(DEV), cuk.to(DEV), max(chunks), max(kl),
                                    128 ** -0.5, block_table=bt.to(DEV), one_head_per_cta=one_head)
    torch.cuda.synchronize()
    assert kernels.prefill_errors() == 0
    want = oattn.varlen_prefill(q, k, v, cuq, cuk, 128 ** -0.5, block_table=bt)
    assert_close(out, want, **BF16_TOL, what="tcgen05 prefill paged")


@pytest.mark.parametrize("case", ["one_long", "many_short", "q_range"])
def test_decode_fp8_tensor_core_splits_and_q_range(case):
    """The tcgen05 kernel on e4m3 caches: a 20k-token sequence split over many CTAs (partial
    merges), many short sequences, and query rows whose magnitudes span 2^-20 .. 2^20 (Q goes to
    f16 with a per-head power-of-two shift)."""
    g = torch.Generator().manual_seed({"one_long": 11, "many_short": 12, "q_range": 13}[case])
    hq, hk = 32, 8
    if case == "one_long":
        lens = [20000]
    elif case == "many_short":
        lens = torch.randint(0, 200, (300,), generator=g).tolist()
    else:
        lens = [300, 1000, 77, 2]
    nblocks = sum(-(-n // 256) for n in lens) + 4
    kb, vb, bt, ln = make_paged(g, len(lens), hk, 128, nblocks, 256, lens)
    ks = torch.rand(hk, generator=g) + 0.5
    vs = torch.rand(hk, generator=g) + 0.5
    kq = kv_store.quantize_e4m3(kb, ks)
    vq = kv_store.quantize_e4m3(vb, vs)
    q = torch.randn(len(lens), hq, 128, generator=g)
    if case == "q_range":
        exps = torch.tensor([-20.0, -6.0, 0.0, 20.0])
        q = q * (2.0 ** exps).view(-1, 1, 1)
    q = q.bfloat16()
    ws = kernels.make_decode_workspace(len(lens), hq, 128, bt.shape[1], 256, DEV)
    for trial in range(2):
        out = run_decode(q, kq, vq, bt, ln, 128 ** -0.5, fp8=True, ks=ks, vs=vs, ws=ws)
        torch.cuda.synchronize()
        assert kernels.decode_errors(ws) == 0
        idx = list(range(len(lens))) if len(lens) <= 16 else list(range(0, len(lens), 7))
        want = oattn.paged_decode(q[idx], kq, vq, bt[idx], ln[idx], 128 ** -0.5, ks, vs, fp8=True)
        assert_close(out[idx], want, **BF16_TOL, what=f"fp8 tensor-core {case} trial {trial}")


@pytest.mark.parametrize("fp8", [False, True])
def test_decode_tensor_core_ignores_nan_past_context(fp8):
    """Cache slots past a sequence's context may hold any bits (an uninitialised cache); the
    tcgen05 kernel loads whole 128-token tiles, so it must keep NaN there out of P.V."""
    g = torch.Generator().manual_seed(21 + fp8)
    hq, hk = 32, 8
    lens = [1, 100, 129, 255, 300]
    kb, vb, bt, ln = make_paged(g, len(lens), hk, 128, 8, 256, lens)
    q = torch.randn(len(lens), hq, 128, generator=g).bfloat16()
    if fp8:
        kc, vc = kv_store.quantize_e4m3(kb, None), kv_store.quantize_e4m3(vb, None)
        nan_byte = 0x7F
    else:
        kc, vc = kb.clone(), vb.clone()
    for i, n in enumerate(lens):
        for j in range(n, -(-n // 256) * 256):
            blk = int(bt[i, j // 256])
            if fp8:
                kc[blk, j % 256] = nan_byte
                vc[blk, j % 256] = nan_byte
            else:
                kc[blk, j % 256] = float("nan")
                vc[blk, j % 256] = float("nan")
    out = run_decode(q, kc, vc, bt, ln, 128 ** -0.5, fp8=fp8)
    assert torch.isfinite(out.float()).all()
    want = oattn.paged_decode(q, kc, vc, bt, ln, 128 ** -0.5, fp8=fp8)
    assert_close(out, want, **BF16_TOL, what=f"NaN past context fp8={fp8}")


# ----------------------------------------------------------------------------- top-k / top-p sampling
def _filtered_rows(g, rows, vocab, scale=3.0, levels=0):
    x = torch.randn(rows, vocab, generator=g) * scale
    if levels:  # few distinct values: filter boundaries cut through groups of equal logits
        x = torch.randint(0, levels, (rows, vocab), generator=g).float()
    return x.bfloat16()


@pytest.mark.parametrize("vocab", [1000, 151936])
def test_sample_filtered_without_filters_equals_sample(vocab):
    """Rows without top-k / top-p (k in {-1, 0, >= V}, p = 1) get exactly hl_sample's token for
    the same seed and step, greedy rows included."""
    g = torch.Generator().manual_seed(vocab)
    rows = 64
    logits = _filtered_rows(g, rows, vocab).to(DEV)
    temps = torch.rand(rows, generator=g) + 0.2
    temps[::4] = 0.0
    temps = temps.to(DEV)
    ks = torch.tensor([[-1, 0, vocab, vocab + 5][i % 4] for i in range(rows)], dtype=torch.int32, device=DEV)
    ps = torch.ones(rows, dtype=torch.float32, device=DEV)
    for step in range(3):
        s1 = torch.tensor([step, 0], dtype=torch.int64, device=DEV)
        s2 = s1.clone()
        want = kernels.sample(logits, temps, 77, s1)
        got = kernels.sample_filtered(logits, temps, ks, ps, 77, s2)
        assert torch.equal(got, want)
        assert torch.equal(s1, s2)
    got = kernels.sample_filtered(logits, temps, None, None, 5, None)
    assert torch.equal(got, kernels.sample(logits, temps, 5, None))


@pytest.mark.parametrize("vocab,levels", [(151936, 0), (5000, 8), (3000, 0)])
def test_sample_filtered_draws_stay_in_the_kept_set(vocab, levels):
    """Every draw lies in the reference's kept set (oracle/sampler.kept_set, equal logits ordered
    by index): top-k alone, top-p alone, both, greedy rows with filters; levels > 0 makes the
    top-k boundary cut through groups of equal logits."""
    from oracle.sampler import kept_set

    g = torch.Generator().manual_seed(vocab + levels)
    rows = 48
    logits = _filtered_rows(g, rows, vocab, levels=levels)
    temps = torch.rand(rows, generator=g) + 0.3
    temps[::7] = 0.0
    ks = torch.randint(1, 300, (rows,), generator=g).to(torch.int32)
    ks[1::3] = -1
    ps = (torch.rand(rows, generator=g) * 0.95 + 0.04).to(torch.float32)
    ps[2::3] = 1.0
    ps[3] = 0.0  # keeps only the first token (the reference's forced first entry)
    state = torch.zeros(2, dtype=torch.int64, device=DEV)
    ld, td, kd, pd = logits.to(DEV), temps.to(DEV), ks.to(DEV), ps.to(DEV)
    keep = []
    for r in range(rows):
        t = float(temps[r])
        if t <= 0:
            keep.append(None)
            continue
        # top_p + 1e-4: a draw may sit exactly on the boundary that float sums in another order decide
        p_r = float(ps[r])
        keep.append(kept_set(logits[r], t, int(ks[r]), p_r if p_r <= 0.0 else (min(1.0, p_r + 1e-4)
                                                                                if p_r < 1.0 else 1.0)))
    for _ in range(8):
        tok = kernels.sample_filtered(ld, td, kd, pd, 99, state).cpu()
        for r in range(rows):
            if keep[r] is None:
                assert int(tok[r]) == int(torch.argmax(logits[r].float())), r
            else:
                assert bool(keep[r][int(tok[r])]), (r, int(tok[r]), int(ks[r]), float(ps[r]))
    assert int(state[0]) == 8


@pytest.mark.parametrize("k,p,levels", [(10, 1.0, 0), (-1, 0.8, 0), (12, 0.7, 0), (9, 1.0, 5)])
def test_sample_filtered_matches_reference_distribution(k, p, levels):
    """Empirical frequencies over many rows and launches match the reference's distribution
    (softmax over the kept set, oracle/sampler.filtered_distribution) within sampling error;
    with levels = 5 the top-k boundary splits a group of equal logits (lowest ids kept)."""
    from oracle.sampler import filtered_distribution

    g = torch.Generator().manual_seed(41 + k + levels)
    rows, vocab, T = 512, 40, 0.9
    base = (torch.randn(vocab, generator=g) * 1.5) if not levels else \
        torch.randint(0, levels, (vocab,), generator=g).float()
    base = base.bfloat16()
    logits = base.repeat(rows, 1).to(DEV)
    temps = torch.full((rows,), T, dtype=torch.float32, device=DEV)
    ks = torch.full((rows,), k, dtype=torch.int32, device=DEV)
    ps = torch.full((rows,), p, dtype=torch.float32, device=DEV)
    state = torch.zeros(2, dtype=torch.int64, device=DEV)
    counts = torch.zeros(vocab, dtype=torch.float64)
    launches = 40
    for _ in range(launches):
        tok = kernels.sample_filtered(logits, temps, ks, ps, 4321, state)
        counts += torch.bincount(tok.cpu(), minlength=vocab).double()
    freq = counts / counts.sum()
    want = filtered_distribution(base, T, k, p)
    assert float(freq[want == 0].sum()) == 0.0
    n = rows * launches
    assert float((freq - want).abs().max()) < 5 * float((want * (1 - want) / n).sqrt().max()) + 1e-4
