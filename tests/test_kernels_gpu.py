"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""

import pytest
import torch
import torch.nn.functional as F

from mimir_b200 import ops
from mimir_b200.data.prefixlm import compute_aux_seq_tensors_scalars

pytestmark = pytest.mark.gpu


def _close(a, b, atol, rtol=0.0, name=""):
    err = (a.float() - b.float()).abs()
    bound = atol + rtol * b.float().abs()
    assert bool((err <= bound).all()), f"{name}: max abs err {err.max().item():.3e}"


@pytest.mark.parametrize("d", [256, 2048, 1536])
def test_rmsnorm(d):
    x = torch.randn(300, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = ops.rms_norm(x, 1e-6)
    xr = x.detach().float().requires_grad_(True)
    yr = F.rms_norm(xr, (d,), eps=1e-6)
    _close(y, yr, 2e-2, 1e-2, "rmsnorm fwd")
    g = torch.randn_like(y)
    y.backward(g)
    yr.backward(g.float())
    _close(x.grad, xr.grad, 3e-2, 2e-2, "rmsnorm bwd")


def test_add_rmsnorm_matches_composite():
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(300, 2048, device="cuda", generator=g).to(torch.bfloat16).requires_grad_(True)
    a = torch.randn(300, 2048, device="cuda", generator=g).to(torch.bfloat16).requires_grad_(True)
    h, y = ops.add_rms_norm(x, a, 1e-6)
    hr = (x.float() + a.float()).to(torch.bfloat16)
    yr = torch.nn.functional.rms_norm(hr.float(), (2048,), eps=1e-6)
    assert torch.equal(h, hr)
    _close(y.float(), yr, 2e-2, 2e-2, "add_rmsnorm fwd")
    dh = torch.randn_like(h)
    dy = torch.randn_like(y)
    (h.float() * dh.float()).sum().add((y.float() * dy.float()).sum()).backward()
    xr = x.detach().float().requires_grad_(True)
    ar = a.detach().float().requires_grad_(True)
    hr2 = xr + ar
    yr2 = torch.nn.functional.rms_norm(hr2, (2048,), eps=1e-6)
    (hr2 * dh.float()).sum().add((yr2 * dy.float()).sum()).backward()
    _close(x.grad.float(), xr.grad, 3e-2, 3e-2, "add_rmsnorm bwd x")
    assert torch.equal(x.grad, a.grad)


def test_swiglu():
    gu = torch.randn(257, 2 * 5632, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    out = ops.swiglu(gu)
    ref_in = gu.detach().float().requires_grad_(True)
    ref = ops.swiglu_reference(ref_in)
    _close(out, ref, 2e-2, 1e-2, "swiglu fwd")
    g = torch.randn_like(out)
    out.backward(g)
    ref.backward(g.float())
    _close(gu.grad, ref_in.grad, 3e-2, 2e-2, "swiglu bwd")


def test_cross_entropy():
    torch.manual_seed(0)
    h = torch.randn(200, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(4096, 256, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_(True)
    labels = torch.randint(0, 4096, (200,), device="cuda")
    labels[:17] = -100
    loss, correct = ops.linear_cross_entropy(h, w, labels)
    hr, wr = h.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    logits = (hr.bfloat16() @ wr.bfloat16().t()).float()
    ref = F.cross_entropy(logits, labels, ignore_index=-100, reduction="sum")
    assert abs(loss.item() - ref.item()) <= 1e-3 * abs(ref.item()) + 1e-2
    assert torch.equal(correct, logits.argmax(-1) == labels)
    (loss * 0.5).backward()
    (ref * 0.5).backward()
    _close(h.grad, hr.grad, 2e-2, 2e-2, "ce dh")
    _close(w.grad, wr.grad, 2e-2, 2e-2, "ce dw")


def test_adam_atan2_fused_matches_reference():
    from mimir_b200.optim.adam_atan2 import AdamATan2
    torch.manual_seed(0)
    ps = [torch.randn(s, device="cuda", requires_grad=True) for s in [(100, 37), (5000,), (3, 3)]]
    ref = [p.detach().clone().requires_grad_(True) for p in ps]
    o1 = AdamATan2(ps, lr=1e-2, ema=0.99)
    o2 = AdamATan2(ref, lr=1e-2, ema=0.99, fused=False)
    for _ in range(3):
        for a, b in zip(ps, ref):
            g = torch.randn_like(a)
            a.grad, b.grad = g.clone(), g.clone()
        o1.step()
        o2.step()
    for a, b in zip(ps, ref):
        _close(a, b, 1e-5, 1e-5, "param")
        _close(o1.state[a]["param_ema"], o2.state[b]["param_ema"], 1e-5, 1e-5, "ema")
        _close(o1.state[a]["exp_avg_sq"], o2.state[b]["exp_avg_sq"], 1e-7, 1e-5, "v")


def test_ngram_kernel_matches_torch():
    from mimir_b200.models.ngram import NGramMemory
    torch.manual_seed(0)
    mem = NGramMemory(256, (2, 3), 1021, heads=2).cuda()
    for t in mem.tables:
        torch.nn.init.normal_(t)
    ids = torch.randint(0, 500, (1, 777), device="cuda")
    pos = torch.cat([torch.arange(300), torch.arange(477)]).cuda()[None]
    out = mem.lookup(ids, pos, torch.float32)
    import os
    os.environ["MIMIR_DISABLE_KERNELS"] = "1"
    try:
        ref = mem.lookup(ids, pos, torch.float32)
    finally:
        os.environ.pop("MIMIR_DISABLE_KERNELS")
    _close(out, ref, 1e-5, 1e-5, "ngram")


def _ngram_case():
    from mimir_b200.models.ngram import NGramMemory
    torch.manual_seed(0)
    mem = NGramMemory(256, (2, 3), 1021, heads=2).cuda()
    for t in mem.tables:
        torch.nn.init.normal_(t)
    ids = torch.randint(0, 40, (1, 777), device="cuda")  # few distinct ids: long runs of equal keys
    pos = torch.cat([torch.arange(300), torch.arange(477)]).cuda()[None]
    return mem, ids, pos


def test_ngram_backward_matches_torch_and_is_deterministic():
    import os
    mem, ids, pos = _ngram_case()
    g = torch.randn(1, 777, 256, device="cuda")
    runs = []
    for _ in range(2):
        mem.zero_grad(set_to_none=True)
        mem.lookup(ids, pos, torch.float32).backward(g)
        runs.append([t.grad.clone() for t in mem.tables])
    mem.zero_grad(set_to_none=True)
    os.environ["MIMIR_DISABLE_KERNELS"] = "1"
    try:
        mem.lookup(ids, pos, torch.float32).backward(g)
    finally:
        os.environ.pop("MIMIR_DISABLE_KERNELS")
    for a, b, t in zip(runs[0], runs[1], mem.tables):
        assert torch.equal(a, b)  # sorted run sums: no atomics, same bits every time
        _close(a, t.grad, 1e-5, 1e-5, "ngram grad")


def test_ngram_backward_accumulates_into_owned_bf16_gradients():
    """With a gradient sink (the replicated engine's flat buffer) only hashed rows change."""
    mem, ids, pos = _ngram_case()
    mem = mem.to(torch.bfloat16)
    g = torch.randn(1, 777, 256, device="cuda")
    ref = [torch.zeros_like(t, dtype=torch.float32) for t in mem.tables]
    import os
    os.environ["MIMIR_DISABLE_KERNELS"] = "1"
    try:
        fp32 = [t.detach().float().requires_grad_(True) for t in mem.tables]
        from mimir_b200.models.ngram import ngram_hashes
        for order, (hashes, valid) in ngram_hashes(ids, pos, mem.orders, mem.heads, mem.buckets).items():
            base = mem.orders.index(order) * mem.heads
            for h in range(mem.heads):
                rows = torch.nn.functional.embedding(hashes[h], fp32[base + h]) * valid[..., None]
                (rows * g[..., h * 128:(h + 1) * 128]).sum().backward()
    finally:
        os.environ.pop("MIMIR_DISABLE_KERNELS")
    sunk = []
    for t in mem.tables:
        t.grad = torch.full_like(t, 0.25)
        t._mimir_grad_sink = sunk.append
    mem.lookup(ids, pos, torch.bfloat16).backward(g.to(torch.bfloat16))
    assert len(sunk) == len(mem.tables)
    for t, f in zip(mem.tables, fp32):
        hit = f.grad.abs().sum(-1) > 0
        assert torch.equal(t.grad[~hit], torch.full_like(t.grad[~hit], 0.25))
        _close(t.grad.float()[hit], (0.25 + f.grad[hit]).to(torch.bfloat16).float(), 3e-2, 3e-2, "ngram in place")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("gain", [False, True])
def test_branch_mixes_match_torch(dtype, gain):
    """Fused residual-branch read/write (csrc/branches.cu) against the eager fp32 path: outputs
    and the gradients of streams, update, logits and gains; the broadcast initial streams too."""
    import os

    from mimir_b200.models.branches import ResidualConnection, _fanout
    torch.manual_seed(0)
    B, d = 3, 320
    conn = ResidualConnection(B, d, 1, 0.5, input_dependent=gain).cuda()
    with torch.no_grad():
        for prm in conn.parameters():
            prm.normal_(0, 0.5)
    alpha = torch.tensor(0.7, device="cuda")
    x0 = torch.randn(2, 33, d, device="cuda").to(dtype)
    upd = torch.randn(2, 33, d, device="cuda").to(dtype)
    g_read, g_write = torch.randn(2, 33, d, device="cuda"), torch.randn(2, 33, B, d, device="cuda")

    def run():
        xs = x0.clone().requires_grad_(True)
        us = upd.clone().requires_grad_(True)
        streams = _fanout(xs, B) * 1.5 + 0.1 * torch.arange(B, device="cuda", dtype=dtype)[:, None]
        read = conn.read(streams, alpha)
        wrote = conn.write(streams, us, alpha)
        read0 = conn.read(_fanout(xs, B), alpha)  # a broadcast view (branch stride 0), read in place
        conn.zero_grad()
        ((read.float() * g_read).sum() + (wrote.float() * g_write).sum() + (read0.float() * g_read).sum()).backward()
        grads = [xs.grad, us.grad] + [prm.grad.clone() for prm in conn.parameters()]
        return [read, wrote, read0] + grads

    fused = run()
    os.environ["MIMIR_DISABLE_KERNELS"] = "1"
    try:
        ref = run()
    finally:
        os.environ.pop("MIMIR_DISABLE_KERNELS")
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    names = ["read", "write", "read of the broadcast view", "d streams", "d update"] + [
        n for n, _ in conn.named_parameters()]
    for a, b, name in zip(fused, ref, names):
        _close(a, b, tol * max(1.0, float(b.float().abs().max())), tol, name)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_invocation_gate_matches_torch(dtype):
    """GEMM + fused bias/tanh/gate (ops/gate.py) against the eager path, outputs and gradients."""
    import os

    from mimir_b200.models.mimir2 import InvocationGate
    torch.manual_seed(0)
    d = 256
    gate = InvocationGate(d).cuda().to(dtype)
    with torch.no_grad():
        gate.weight.normal_(0, 0.05)
        gate.bias.normal_(0, 0.5)
    alpha = torch.tensor(0.6, device="cuda")
    h0 = torch.randn(2, 40, d, device="cuda").to(dtype)
    i0 = torch.randn(2, 40, d, device="cuda").to(dtype)
    g = torch.randn(2, 40, d, device="cuda")

    def run():
        h, i = h0.clone().requires_grad_(True), i0.clone().requires_grad_(True)
        gate.zero_grad()
        out = gate(h, i, alpha)
        (out.float() * g).sum().backward()
        return [out, h.grad, i.grad, gate.weight.grad.clone(), gate.bias.grad.clone()]

    fused = run()
    os.environ["MIMIR_DISABLE_KERNELS"] = "1"
    try:
        ref = run()
    finally:
        os.environ.pop("MIMIR_DISABLE_KERNELS")
    tol = 2e-3 if dtype == torch.float32 else 4e-2
    for a, b, name in zip(fused, ref, ["out", "d hidden", "d injection", "d weight", "d bias"]):
        _close(a, b, tol * max(1.0, float(b.float().abs().max())), tol, name)


@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_goldfish_kernel_matches_torch_bit_for_bit(dtype):
    from mimir_b200.models.goldfish import goldfish_drop_mask, goldfish_drop_mask_reference
    g = torch.Generator(device="cuda").manual_seed(7)
    T = 3000
    inputs = torch.randint(0, 65536, (T,), device="cuda", generator=g, dtype=dtype)
    supervised = torch.rand(T, device="cuda", generator=g) > 0.2
    cu = torch.tensor([0, 5, 5, 700, 701, 2100, 2999] + [0] * 9, device="cuda", dtype=torch.int32)  # padded bounds
    for k, w, seed in ((2, 50, 0), (3, 7, 12345), (50, 50, 2 ** 40 + 3)):
        ours = goldfish_drop_mask(inputs, supervised, cu, k, w, seed)
        ref = goldfish_drop_mask_reference(inputs, supervised, cu, k, w, seed)
        assert torch.equal(ours, ref), (k, w, seed)
        assert bool(ours.any()) and not bool(ours[2999:].any())


def _packed(lengths, prefixes, heads, kv_heads, seed=0, pad=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    T = sum(lengths) + pad
    q = torch.randn(T, heads, 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(T, kv_heads, 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(T, kv_heads, 128, device="cuda", generator=g).to(torch.bfloat16)
    p = torch.tensor(prefixes, dtype=torch.int32)
    c = torch.tensor(lengths, dtype=torch.int32) - p
    tensors, scalars = compute_aux_seq_tensors_scalars(p.numpy(), c.numpy(), T)
    meta = {k2: torch.from_numpy(v2).cuda() for k2, v2 in tensors.items()} | scalars
    return q, k, v, meta


CASES = [
    ([4096, 4096], [1000, 0], 16, 4),
    ([130, 1, 257, 513], [5, 1, 256, 0], 2, 2),
    ([128, 256], [128, 129], 4, 1),
    ([300], [299], 2, 1),
]


@pytest.mark.parametrize("lengths,prefixes,H,KV", CASES)
@pytest.mark.parametrize("causal", [False, True])
def test_fmha_forward(lengths, prefixes, H, KV, causal):
    q, k, v, meta = _packed(lengths, prefixes, H, KV, pad=37)
    out = ops.prefixlm_attention(q, k, v, causal, **meta)
    ref = ops.dense_prefixlm_attention(q.float(), k.float(), v.float(), causal, **meta)
    total = sum(lengths)
    assert ops.ext().fmha_status(q.device) == 0
    _close(out[:total], ref[:total], 2e-2, 2e-2, "fmha fwd")


@pytest.mark.parametrize("lengths,prefixes,H,KV", CASES)
def test_fmha_forward_kernels_agree(lengths, prefixes, H, KV, monkeypatch):
    """The two-query-tile forward (default) and the one-tile forward give the same rows and LSE."""
    q, k, v, meta = _packed(lengths, prefixes, H, KV, pad=37, seed=3)
    total = sum(lengths)
    outs = {}
    for version in ("1", "2"):
        monkeypatch.setenv("MIMIR_FMHA_FWD", version)
        outs[version] = ops.prefixlm_attention(q, k, v, False, **meta)
    assert ops.ext().fmha_status(q.device) == 0
    _close(outs["2"][:total], outs["1"][:total], 2e-2, 2e-2, "fmha fwd2 vs fwd1")


def test_gated_attention_block_matches_composite():
    from mimir_b200.models.layers import RotaryEmbedding
    torch.manual_seed(0)
    H, KV, hd = 4, 2, 128
    lengths, prefixes = [200, 333], [50, 1]
    _, _, _, meta = _packed(lengths, prefixes, H, KV)
    T = sum(lengths)
    gqkv = (torch.randn(T, (2 * H + 2 * KV) * hd, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    rope = RotaryEmbedding(hd, 4096, 10000.0).cuda()
    pos = torch.cat([torch.arange(n) for n in lengths]).cuda()
    tables = (rope.cos_cached, rope.sin_cached)
    y = ops.gated_prefixlm_attention(gqkv, tables, pos, H, KV, hd, False, meta)
    g32 = gqkv.detach().float().requires_grad_(True)
    ref = ops.gated_attention_composite(g32, tables, pos, H, KV, hd, False, meta)
    _close(y, ref, 3e-2, 3e-2, "gated fwd")
    dy = torch.randn_like(y)
    y.backward(dy)
    ref.backward(dy.float())
    _close(gqkv.grad, g32.grad, 6e-2, 5e-2, "gated bwd")


@pytest.mark.parametrize("lengths,prefixes,H,KV", CASES)
@pytest.mark.parametrize("causal", [False, True])
def test_fmha_backward(lengths, prefixes, H, KV, causal):
    q, k, v, meta = _packed(lengths, prefixes, H, KV, pad=37)
    total = sum(lengths)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    q, k, v = (t.detach().requires_grad_(True) for t in (q, k, v))
    out = ops.prefixlm_attention(q, k, v, causal, **meta)
    ref = ops.dense_prefixlm_attention(qr, kr, vr, causal, **meta)
    g = torch.randn_like(ref)
    g[total:] = 0
    out.backward(g.to(out.dtype))
    ref.backward(g)
    assert ops.ext().fmha_status(q.device) == 0
    for name, a, b in (("dq", q.grad, qr.grad), ("dk", k.grad, kr.grad), ("dv", v.grad, vr.grad)):
        scale = b[:total].abs().max().item() + 1e-6
        _close(a[:total] / scale, b[:total] / scale, 2e-2, 0.0, f"fmha bwd {name}")


def test_fmha_padding_rows_do_not_leak():
    """Sentinels in the padding rows after the last sequence (q, k, v and the output gradient):
    the outputs and gradients of the valid rows are finite and bit-identical to a run with zero
    padding, so masked keys and queries contribute exact zeros.  The sentinel is a large finite
    value, not NaN: the last sequence's 128-row tiles extend into the padding by design, and a
    NaN there would pass through a tile-wide MMA even with a probability of zero."""
    lengths, prefixes, H, KV = [300, 129, 513], [100, 129, 0], 4, 2
    total = sum(lengths)
    runs = []
    for poison in (False, True):
        q, k, v, meta = _packed(lengths, prefixes, H, KV, pad=70, seed=5)
        for t in (q, k, v):
            t[total:] = 1.0e4 if poison else 0.0
        q, k, v = (t.detach().requires_grad_(True) for t in (q, k, v))
        out = ops.prefixlm_attention(q, k, v, False, **meta)
        g = torch.randn(out.shape, device="cuda", generator=torch.Generator(device="cuda").manual_seed(6)).to(out.dtype)
        g[total:] = 1.0e4 if poison else 0.0
        out.backward(g)
        runs.append([out[:total], q.grad[:total], k.grad[:total], v.grad[:total]])
    assert ops.ext().fmha_status(torch.device("cuda", 0)) == 0
    for a, b, name in zip(runs[0], runs[1], ["out", "dq", "dk", "dv"]):
        assert bool(torch.isfinite(b.float()).all()), name
        assert torch.equal(a, b), name


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_scaled_embedding_matches_torch(dtype):
    """Fused gather + scale forward and the sorted, deterministic backward (repeated ids included)."""
    g = torch.Generator(device="cuda").manual_seed(11)
    V, d, T = 1000, 256, 4097
    w = torch.randn(V, d, device="cuda", generator=g).to(dtype).requires_grad_(True)
    ids = torch.randint(0, 50, (T,), device="cuda", generator=g, dtype=torch.int32)  # many repeats
    out = ops.scaled_embedding(ids, w, 2.5)
    wr = w.detach().float().requires_grad_(True)
    ref = 2.5 * torch.nn.functional.embedding(ids.long(), wr)
    _close(out, ref, 2e-2 if dtype == torch.bfloat16 else 1e-6, 1e-2, "embedding forward")
    dy = torch.randn(T, d, device="cuda", generator=g).to(dtype)
    out.backward(dy)
    ref.backward(dy.float())
    scale = wr.grad.abs().max().item()
    _close(w.grad.float() / scale, wr.grad / scale, 1e-2 if dtype == torch.bfloat16 else 1e-5, 0.0, "embedding backward")
    first = w.grad.clone()
    w.grad = None
    ops.scaled_embedding(ids, w, 2.5).backward(dy)
    assert torch.equal(first, w.grad), "the backward is deterministic"


@pytest.mark.parametrize("d", [2048, 3072])
def test_scaled_embedding_backward_skewed_ids(d):
    """Zipf-like ids: one id on thousands of positions, runs of exactly 32 and 33 rows, singletons
    (short runs summed by one warp, long runs by one CTA of eight warps), against fp32 index_add;
    bit-identical on a second run."""
    g = torch.Generator(device="cuda").manual_seed(5)
    V = 4096
    parts = [torch.full((3000,), 7), torch.full((32,), 11), torch.full((33,), 12), torch.full((200,), 13),
             torch.randint(100, V, (1500,), generator=torch.Generator().manual_seed(1))]
    ids = torch.cat(parts)[torch.randperm(4765, generator=torch.Generator().manual_seed(2))].cuda()
    T = ids.numel()
    w = (torch.randn(V, d, device="cuda", generator=g) * 0.1).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(T, d, device="cuda", generator=g).to(torch.bfloat16)
    ops.scaled_embedding(ids, w, 0.5).backward(dy)
    ref = torch.zeros(V, d, device="cuda").index_add_(0, ids.long(), 0.5 * dy.float())
    scale = ref.abs().max().item()
    _close(w.grad.float() / scale, ref / scale, 1e-2, 0.0, "skewed embedding backward")
    first = w.grad.clone()
    w.grad = None
    ops.scaled_embedding(ids, w, 0.5).backward(dy)
    assert torch.equal(first, w.grad)
