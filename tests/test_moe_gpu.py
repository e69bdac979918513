"""MoE token-exchange kernels (csrc/moe.cu) and expert parallelism on B200s.

* dispatch / combine / combine-backward kernels against PyTorch fp32 indexing arithmetic;
* the grouped MoE path on one GPU against the per-expert ``index_add`` path;
* expert parallelism over CUDA-IPC peer buffers on 2+ GPUs (spawned NCCL ranks) against one
  process running every expert on the concatenated batch.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

D, F, E, K = 256, 384, 8, 2


def test_exchange_kernels_match_torch():
    from mimir_b200.ops._ext import ext
    C = ext()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    T = 37
    x = torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16)
    topi = torch.stack([torch.randperm(E, device=dev, generator=g)[:K] for _ in range(T)])
    from mimir_b200.parallel.expert import expert_parallel
    ep = expert_parallel(E, dev, distributed=False)
    plan = ep.plan(topi)
    buf = torch.zeros(T * K, D, device=dev, dtype=torch.bfloat16)
    C.moe_dispatch(x, plan.rows, plan.dst, [buf.data_ptr()], K, T * K)
    rows = plan.rows.long()
    for j in range(K):
        assert torch.equal(buf[rows[:, j]], x)
    y = torch.randn(T * K, D, device=dev, generator=g).to(torch.bfloat16)
    w = torch.rand(T, K, device=dev, generator=g)
    ys = torch.empty(T * K, D, device=dev, dtype=torch.bfloat16)
    out = C.moe_combine([y.data_ptr()], plan.rows, plan.dst, w, T, K, D, ys, T * K)
    want = (y[rows].float() * w.unsqueeze(-1)).sum(1)
    torch.testing.assert_close(out.float(), want, rtol=1e-2, atol=1e-2)
    assert torch.equal(ys.view(T, K, D), y[rows])  # the loaded rows are kept for the backward
    dout = torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16)
    dy = torch.zeros_like(y)
    dw = C.moe_combine_bwd(dout, w, plan.rows, plan.dst, ys, [dy.data_ptr()], K, T * K)
    torch.testing.assert_close(dw, (dout.float().unsqueeze(1) * y[rows].float()).sum(-1), rtol=1e-4, atol=1e-3)
    for j in range(K):
        torch.testing.assert_close(dy[rows[:, j]].float(), (w[:, j:j + 1] * dout.float()), rtol=1e-2, atol=1e-2)


def test_exchange_skips_and_reports_routes_outside_the_buffers():
    """A route naming a rank or row outside the peer buffers is skipped and reported through the
    status word (read by ``check_kernel_status``) instead of becoming a peer access."""
    from mimir_b200.ops._ext import KernelTimeout, check_kernel_status, ext
    C = ext()
    dev = torch.device("cuda", 0)
    T, K, D = 8, 2, 64
    x = torch.randn(T, D, device=dev).to(torch.bfloat16)
    rows = torch.arange(T * K, device=dev, dtype=torch.int32).view(T, K).contiguous()
    dst = torch.zeros(T, K, device=dev, dtype=torch.int32)
    bad_rows, bad_dst = rows.clone(), dst.clone()
    bad_rows[3, 1] = T * K + 5  # past the buffer
    bad_dst[5, 0] = 1  # a rank that does not exist (one-rank group)
    buf = torch.zeros(T * K, D, device=dev, dtype=torch.bfloat16)
    C.moe_dispatch(x, bad_rows, bad_dst, [buf.data_ptr()], K, T * K)
    torch.cuda.synchronize()
    assert C.moe_route_status(0) == 1 and C.moe_route_status(0) == 0  # read clears it
    good = [t for t in range(T) if t not in (3, 5)]
    assert torch.equal(buf[rows[good, 0].long()], x[good])
    y = torch.randn(T * K, D, device=dev).to(torch.bfloat16)
    out = C.moe_combine([y.data_ptr()], bad_rows, bad_dst, None, T, K, D, None, T * K)
    torch.testing.assert_close(out[3].float(), y[rows[3, 0].long()].float())  # the bad slot adds zero
    with pytest.raises(KernelTimeout, match="moe_routes"):
        check_kernel_status(dev)
    C.moe_dispatch(x, rows, dst, [buf.data_ptr()], K, T * K)  # a good launch afterwards
    torch.cuda.synchronize()
    assert C.moe_route_status(0) == 0


def _mixture(grouped, ep=False, shared=1, seed=0):
    from mimir_b200.models.experts import MLPMixture
    from mimir_b200.models.layers import SwiGLU
    torch.manual_seed(seed)
    m = MLPMixture(SwiGLU(D, F), D, E, K, sparse=True, grouped=grouped, expert_parallel=ep, shared_experts=shared,
                   expert_intermediate_size=F)
    with torch.no_grad():
        for i, r in enumerate(m.router.rows):
            r.copy_(torch.randn(D, generator=torch.Generator().manual_seed(10 + i)) * 0.5)
    return m


def _run(m, x, g):
    x = x.clone().requires_grad_(True)
    y = m(x)
    (y.float() * g).sum().backward()
    return y.detach().float(), x.grad.float(), {n: p.grad.float() for n, p in m.named_parameters()}


def test_grouped_path_matches_index_path():
    dev = torch.device("cuda", 0)
    ref = _mixture(False).to(dev, torch.bfloat16)
    grp = _mixture(True).to(dev, torch.bfloat16)
    grp.load_state_dict(ref.state_dict())
    gen = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(300, D, device=dev, generator=gen).to(torch.bfloat16)
    g = torch.randn(300, D, device=dev, generator=gen)
    a, b = _run(ref, x, g), _run(grp, x, g)
    # bf16 sums in a different order (fp32 combine here, bf16 index_add there): compare against
    # the tensor's scale
    for name, u, v in (("y", b[0], a[0]), ("dx", b[1], a[1])):
        assert (u - v).abs().max() / v.abs().max() < 2e-2, name
    for n in a[2]:
        scale = a[2][n].abs().max().clamp_min(1e-6)
        assert (b[2][n] - a[2][n]).abs().max() / scale < 3e-2, n


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_rank(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        m = _mixture(True, ep=True).to(dev, torch.bfloat16)
        gen = torch.Generator(device=dev).manual_seed(100 + rank)
        x = torch.randn(200, D, device=dev, generator=gen).to(torch.bfloat16)
        g = torch.randn(200, D, device=dev, generator=gen)
        for _ in range(2):  # second pass reuses the pooled peer buffers
            for p in m.parameters():
                p.grad = None
            y, dx, grads = _run(m, x, g)
        torch.cuda.synchronize()
        torch.save({"x": x.cpu(), "g": g.cpu(), "y": y.cpu(), "dx": dx.cpu(),
                    "grads": {n: t.cpu() for n, t in grads.items()}}, f"{out}.{rank}.pt")
        from mimir_b200.parallel.expert import expert_parallel
        expert_parallel(E, dev).close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_matches_single_process(tmp_path):
    import torch.multiprocessing as mp
    world = 2 if E % min(torch.cuda.device_count(), 8) else min(torch.cuda.device_count(), 8)
    mp.spawn(_ep_rank, args=(world, _free_port(), str(tmp_path / "ep")), nprocs=world, join=True)
    res = [torch.load(tmp_path / f"ep.{r}.pt") for r in range(world)]
    dev = torch.device("cuda", 0)
    full = _mixture(True).to(dev, torch.bfloat16)
    x = torch.cat([r["x"] for r in res]).to(dev)
    g = torch.cat([r["g"] for r in res]).to(dev)
    y, dx, grads = _run(full, x, g)
    T = res[0]["x"].shape[0]
    for r in range(world):
        torch.testing.assert_close(res[r]["y"], y[r * T:(r + 1) * T].cpu(), rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(res[r]["dx"], dx[r * T:(r + 1) * T].cpu(), rtol=2e-2, atol=2e-2)
    local = E // world
    for n, want in grads.items():
        want = want.cpu()
        if n.startswith("experts."):
            got = res[int(n.split(".")[1]) // local]["grads"][n]
        else:
            got = sum(r["grads"][n] for r in res)
        scale = want.abs().max().clamp_min(1e-6)
        assert (got - want).abs().max() / scale < 3e-2, n


@pytest.mark.parametrize("b_kn", [False, True])
@pytest.mark.parametrize("N,K", [(256, 128), (384, 192), (2816, 2048), (1408, 2048), (2048, 2816)])
def test_grouped_gemm_matches_fp32(N, K, b_kn):
    from mimir_b200.ops._ext import ext
    C = ext()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(N + K)
    counts = [130, 0, 1, 257, 64, 0, 300, 5]
    R = sum(counts)
    a = torch.randn(R, K, device=dev, generator=g).to(torch.bfloat16)
    shape = (K, N) if b_kn else (N, K)
    bs = [(torch.randn(*shape, device=dev, generator=g) / K ** 0.5).to(torch.bfloat16) for _ in counts]
    out = torch.full((R, N), float("nan"), device=dev, dtype=torch.bfloat16)
    C.grouped_gemm(a, bs, torch.tensor(counts, dtype=torch.int32, device=dev), out, b_kn)
    torch.cuda.synchronize()
    assert C.grouped_gemm_status(0) == 0
    s = 0
    for n, b in zip(counts, bs):
        want = a[s:s + n].float() @ (b.float() if b_kn else b.float().t())
        torch.testing.assert_close(out[s:s + n].float(), want, rtol=2e-2, atol=2e-2)
        s += n


@pytest.mark.parametrize("M,N", [(256, 128), (2816, 2048), (2048, 1408)])
def test_grouped_wgrad_accumulates_fp32_products(M, N):
    from mimir_b200.ops._ext import ext
    C = ext()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + N)
    rows = [70, 0, 129, 1, 64, 200]
    R = sum(rows) + 17  # trailing rows that belong to no group
    a = torch.randn(R, M, device=dev, generator=g).to(torch.bfloat16)
    b = torch.randn(R, N, device=dev, generator=g).to(torch.bfloat16)
    grads = [torch.randn(M, N, device=dev, generator=g).to(torch.bfloat16) for _ in rows]
    before = [w.float().clone() for w in grads]
    C.grouped_wgrad(a, b, rows, grads)
    torch.cuda.synchronize()
    assert C.grouped_gemm_status(0) == 0
    s = 0
    for n, w, w0 in zip(rows, grads, before):
        want = w0 + a[s:s + n].float().t() @ b[s:s + n].float()
        assert (w.float() - want).abs().max() / want.abs().max() < 1e-2
        s += n


@pytest.mark.parametrize("E,k", [(8, 2), (64, 2), (64, 8), (256, 1)])
def test_router_topk_matches_stable_argsort_and_counts(E, k):
    from mimir_b200.ops._ext import ext
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(E * 10 + k)
    sel = torch.randn(1000, E, device=dev, generator=g)
    sel[::7, : E // 2] = 0.25  # exact ties: the lower expert index must win, as in a stable argsort
    load = torch.full((E,), 5, dtype=torch.int64, device=dev)
    chosen = ext().router_topk(sel, k, load)
    want = sel.argsort(dim=-1, descending=True, stable=True)[:, :k]
    assert torch.equal(chosen, want)
    assert torch.equal(load - 5, torch.bincount(want.reshape(-1), minlength=E))


def test_grouped_path_under_activation_checkpointing_returns_every_buffer():
    from torch.utils.checkpoint import checkpoint
    from mimir_b200.parallel.expert import expert_parallel
    dev = torch.device("cuda", 0)
    m = _mixture(True).to(dev, torch.bfloat16)
    ep = expert_parallel(E, dev, distributed=False)
    x = torch.randn(300, D, device=dev, dtype=torch.bfloat16, requires_grad=True)
    sizes = []
    for _ in range(3):
        checkpoint(m, x, use_reentrant=False).float().square().sum().backward()
        assert not ep._busy  # nothing held after the backward
        sizes.append(len(ep._pool))
    assert sizes[1] == sizes[2]  # the pool stops growing: buffers are reused


@pytest.mark.parametrize("tokens,n", [(16384, 64), (1000, 32), (7, 128)])
def test_router_logits_tensor_core_path_matches_fp32(tokens, n):
    """bf16 hidden states and router rows: the tcgen05 fp32-output path against the fp32 F.linear
    the reference runs (forward, input, row and bias gradients)."""
    import torch.nn.functional as F

    from mimir_b200.ops.router import router_logits, tensor_core_path
    g = torch.Generator(device="cuda").manual_seed(tokens + n)
    x = torch.randn(tokens, 2048, device="cuda", generator=g).to(torch.bfloat16).requires_grad_()
    w = (torch.randn(n, 2048, device="cuda", generator=g) * 0.02).to(torch.bfloat16).requires_grad_()
    b = (torch.randn(n, device="cuda", generator=g) * 0.1).to(torch.bfloat16).requires_grad_()
    assert tensor_core_path(x, w)
    s = router_logits(x, w, b)
    ref_leaves = [t.detach().float().requires_grad_() for t in (x, w, b)]
    ref = F.linear(*ref_leaves)
    assert s.dtype == torch.float32
    scale = ref.abs().max().item()
    assert (s - ref).abs().max().item() <= 1e-4 * scale
    ds = torch.randn(tokens, n, device="cuda", generator=g)
    s.backward(ds)
    ref.backward(ds)
    for got, want, name in ((x.grad, ref_leaves[0].grad, "x"), (w.grad, ref_leaves[1].grad, "w"),
                            (b.grad, ref_leaves[2].grad, "b")):
        err = ((got.float() - want).abs().max() / want.abs().max()).item()
        assert err <= 8e-3, (name, err)
    from mimir_b200.ops import gemm as G
    assert G.status(0) == 0
