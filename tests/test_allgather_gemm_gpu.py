"""The fused all-gather + GEMM (``gemm_allgather``, ``csrc/gemm.cu``) and ``ShardedLinear``.

One GPU: the kernel is given ``world`` shard pointers that all live on this GPU (the ranks are
emulated: nothing in the kernel waits on another rank, so one launch covers every code path but
the NVLink transfer).  The product is compared with a plain PyTorch fp32 matmul (error relative
to the largest reference magnitude, as in the other GEMM tests), the gathered copy with the
weight bit for bit, and a second call after the shards changed must see the new rows.

Two or more GPUs: ``ShardedLinear`` on spawned NCCL ranks against the full-weight fp32 reference
(forward, input gradient, reduce-scattered weight gradient), over two weight versions.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from mimir_b200 import ops
from mimir_b200.ops import gemm as G

pytestmark = pytest.mark.gpu


def _close(a, b, tol=1.5e-2, name=""):
    a, b = a.float(), b.float()
    scale = b.abs().max().item() + 1e-6
    err = ((a - b).abs() / scale).max().item()
    assert err <= tol, f"{name}: max error {err:.3e} of the largest magnitude {scale:.3e}"


def _rand(*shape, seed=0, device="cuda"):
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(*shape, device=device, generator=g).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K,world,rank", [(4096, 2048, 2048, 8, 3), (1000, 5120, 2048, 8, 0),
                                              (300, 1024, 136, 2, 1), (512, 512, 64, 1, 0), (0, 2048, 256, 4, 2)])
def test_emulated_ranks_gather_and_multiply(M, N, K, world, rank):
    C = ops.ext()
    S = N // world
    flags = torch.zeros(N // 128, dtype=torch.int32, device="cuda")
    g = torch.full((N, K), float("nan"), dtype=torch.bfloat16, device="cuda")
    for epoch in (1, 2):
        w = _rand(N, K, seed=10 + epoch)
        shards = [w[k * S:(k + 1) * S].clone() for k in range(world)]
        x = _rand(M, K, seed=20 + epoch)
        y = C.gemm_allgather(x, [s.data_ptr() for s in shards], rank, g, flags, epoch)
        torch.cuda.synchronize()
        assert G.status(0) == 0
        assert torch.equal(g, w), f"gathered copy differs (epoch {epoch})"
        if M:
            _close(y, x.float() @ w.float().t(), name=f"{M}x{N}x{K} world {world} epoch {epoch}")


def test_sharded_linear_one_gpu_forward_backward():
    from mimir_b200.parallel.sharded_linear import ShardedLinear
    w = _rand(1024, 512, seed=3)
    layer = ShardedLinear(w, device="cuda")
    x = _rand(700, 512, seed=4).requires_grad_()
    for _ in range(2):  # the second forward reuses the gathered copy
        y = layer(x)
        _close(y, x.float() @ w.float().t(), name="forward")
    dy = _rand(700, 1024, seed=5)
    y.backward(dy)
    _close(x.grad, dy.float() @ w.float(), name="input grad")
    _close(layer.shard.grad, dy.float().t() @ x.detach().float(), name="weight grad")
    assert layer.calls == 1 and G.status(0) == 0
    layer.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    from datetime import timedelta

    import torch.distributed as dist

    from mimir_b200.parallel.sharded_linear import ShardedLinear
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    try:
        N, K, M = 2048, 1024, 1500
        w = _rand(N, K, seed=7, device=dev)
        layer = ShardedLinear(w, device=dev)
        result = {}
        for version in range(2):
            x = _rand(M, K, seed=100 * version + rank, device=dev).requires_grad_()
            y = layer(x)
            dy = _rand(M, N, seed=200 * version + rank, device=dev)
            y.backward(dy)
            xs = [torch.empty_like(x) for _ in range(world)]
            dys = [torch.empty_like(dy) for _ in range(world)]
            dist.all_gather(xs, x.detach())
            dist.all_gather(dys, dy)
            wf = w.float()
            S = N // world
            full_grad = sum(d.float().t() @ a.float() for d, a in zip(dys, xs))
            result[version] = dict(
                y=((y.float() - x.detach().float() @ wf.t()).abs().max() / (x.detach().float() @ wf.t()).abs().max()).item(),
                dx=((x.grad.float() - dy.float() @ wf).abs().max() / (dy.float() @ wf).abs().max()).item(),
                dw=((layer.shard.grad.float() - full_grad[rank * S:(rank + 1) * S]).abs().max()
                    / full_grad.abs().max()).item(),
                gathered=bool(torch.equal(layer.gathered, w)))
            # a new weight version: every rank rewrites its rows, then publishes
            with torch.no_grad():
                w = _rand(N, K, seed=8 + version, device=dev)
                layer.shard.copy_(w[rank * S:(rank + 1) * S])
                layer.shard.grad = None
            layer.publish()
        torch.cuda.synchronize()
        result["status"] = G.status(rank)
        torch.save(result, f"{out}.{rank}.pt")
        layer.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_linear_multi_gpu_matches_full_weight(tmp_path):
    world = min(torch.cuda.device_count(), 8)
    mp.spawn(_rank, args=(world, _free_port(), str(tmp_path / "r")), nprocs=world, join=True)
    for rank in range(world):
        r = torch.load(f"{tmp_path / 'r'}.{rank}.pt")
        assert r["status"] == 0
        for version in range(2):
            v = r[version]
            assert v["gathered"], (rank, version)
            assert v["y"] < 1.5e-2 and v["dx"] < 1.5e-2 and v["dw"] < 1.5e-2, (rank, version, v)
