"""Fused reduce-scatter + AdamATan2 + all-gather kernel (csrc/dp_fused.cu) against PyTorch fp32.

One GPU: the kernel's update of the master shard, moments, EMA and the bf16 weight copy is
compared with the per-parameter AdamATan2 arithmetic in fp32.  Two or more GPUs (spawned
ranks, NCCL): every rank's replicated weights must equal the single-process result computed
from the summed gradients, and all ranks must hold bit-identical weights.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _reference_update(w, g, m, v, e, lr, wd, b1, b2, step, ema):
    w = w * (1 - lr * wd)
    v = b2 * v + (1 - b2) * g * g
    m = m + (1 - b1) * (g - m)
    bc1 = 1 - b1 ** step
    bc2 = (1 - b2 ** step) ** 0.5
    w = w - (lr / bc1) * torch.atan2(m, v.sqrt() / bc2)
    e = e + (1 - ema) * (w - e)
    return w, m, v, e


def _model(device):
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Linear(64, 96), torch.nn.Linear(96, 40, bias=True),
                               torch.nn.Linear(40, 8, bias=False)).to(device)


def test_single_gpu_step_matches_fp32_reference():
    from mimir_b200.parallel.replicated import ReplicatedAdamATan2, wrap_replicated
    dev = torch.device("cuda", 0)
    model = _model(dev)
    init = {n: p.detach().float().clone() for n, p in model.named_parameters()}
    engine = wrap_replicated(model, dev, torch.bfloat16)
    opt = ReplicatedAdamATan2(engine, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9)
    state = {n: (init[n], torch.zeros_like(init[n]), torch.zeros_like(init[n]), init[n].clone()) for n in init}
    gen = torch.Generator(device=dev).manual_seed(3)
    for step in (1, 2, 3):
        opt.zero_grad()
        x = torch.randn(33, 64, device=dev, dtype=torch.bfloat16, generator=gen)
        model(x).float().square().mean().backward()
        grads = {n: p.grad.float().clone() for n, p in model.named_parameters()}
        opt.step()
        torch.cuda.synchronize()
        for s in engine.slots:
            w, m, v, e = state[s.fqn]
            w, m, v, e = _reference_update(w, grads[s.fqn], m, v, e, 1e-2, 0.1, 0.9, 0.95, step, 0.9)
            state[s.fqn] = (w, m, v, e)
            sl = slice(s.shard, s.shard + s.shard_numel)
            torch.testing.assert_close(engine.master[sl].view(s.shape), w, rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(opt.exp_avg_sq[sl].view(s.shape), v, rtol=1e-5, atol=1e-9)
            torch.testing.assert_close(opt.ema[sl].view(s.shape), e, rtol=1e-5, atol=1e-6)
            assert torch.equal(s.param.detach(), engine.master[sl].view(s.shape).to(torch.bfloat16))


def test_clip_path_matches_unclipped_reference_with_coefficient():
    from mimir_b200.parallel.replicated import ReplicatedAdamATan2, wrap_replicated
    dev = torch.device("cuda", 0)
    model = _model(dev)
    engine = wrap_replicated(model, dev, torch.bfloat16)
    opt = ReplicatedAdamATan2(engine, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.0, ema=None)
    opt.zero_grad()
    model(torch.randn(9, 64, device=dev, dtype=torch.bfloat16)).float().sum().backward()
    want = torch.sqrt(sum(p.grad.float().square().sum() for p in model.parameters()).double())
    got = engine.reduce_for_clipping().sqrt()
    torch.testing.assert_close(got.cpu(), want.reshape(1).cpu(), rtol=1e-5, atol=0)
    opt.grad_scale = torch.tensor([0.5], device=dev)
    before = engine.master.clone()
    opt.step()
    assert not torch.equal(before, engine.master)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import torch.distributed as dist
    from mimir_b200.parallel.replicated import ReplicatedAdamATan2, wrap_replicated
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        model = _model(dev)
        engine = wrap_replicated(model, dev, torch.bfloat16)
        opt = ReplicatedAdamATan2(engine, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9)
        for step in range(3):
            opt.zero_grad()
            gen = torch.Generator(device=dev).manual_seed(100 * step + rank)
            x = torch.randn(17, 64, device=dev, dtype=torch.bfloat16, generator=gen)
            model(x).float().square().mean().backward()
            torch.save({n: p.grad.detach().float().cpu() for n, p in model.named_parameters()},
                       f"{out}.grad.{step}.{rank}.pt")
            opt.step()
        torch.cuda.synchronize()
        torch.save({n: p.detach().float().cpu() for n, p in model.named_parameters()}, f"{out}.w.{rank}.pt")
        engine.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_multi_gpu_fused_step_matches_summed_reference(tmp_path):
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    mp.spawn(_rank, args=(world, _free_port(), str(tmp_path / "r")), nprocs=world, join=True)
    weights = [torch.load(tmp_path / f"r.w.{r}.pt") for r in range(world)]
    for r in range(1, world):
        for n in weights[0]:
            assert torch.equal(weights[0][n], weights[r][n]), (r, n)
    model = _model("cpu")
    state = {n: (p.detach().float(), torch.zeros_like(p), torch.zeros_like(p), p.detach().float().clone())
             for n, p in model.named_parameters()}
    for step in range(3):
        grads = [torch.load(tmp_path / f"r.grad.{step}.{r}.pt") for r in range(world)]
        for n in state:
            g = sum(gr[n] for gr in grads)
            w, m, v, e = state[n]
            state[n] = _reference_update(w, g, m, v, e, 1e-2, 0.1, 0.9, 0.95, step + 1, 0.9)
    for n, (w, *_rest) in state.items():
        torch.testing.assert_close(weights[0][n], w.to(torch.bfloat16).float(), rtol=1e-2, atol=1e-3)


# ------------------------------------------------------------------ MuonAdamW on the fused engine
def _muon_net(device):
    from test_replicated_muon import _Net
    torch.manual_seed(0)
    return _Net().to(device)


MUON_HP = dict(lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9, momentum=0.95, ns_steps=5, muon_lr_scale=0.5)


def _muon_reference(model, grads_per_step):
    """Per-parameter MuonAdamW in fp32 fed with the given (summed) gradients."""
    from mimir_b200.optim.muon import MuonAdamW
    opt = MuonAdamW(model.named_parameters(), **MUON_HP)
    for grads in grads_per_step:
        for n, p in model.named_parameters():
            p.grad = grads[n].to(p.device)
        opt.step()
    return {n: p.detach().float().cpu() for n, p in model.named_parameters()}


def _muon_tokens(gen, dev):
    return torch.randint(0, 11, (6, 5), device=dev, generator=gen)


def test_single_gpu_muon_step_matches_fp32_reference():
    from mimir_b200.parallel.replicated import ReplicatedMuonAdamW, wrap_replicated
    dev = torch.device("cuda", 0)
    model = _muon_net(dev)
    shadow = _muon_net(dev)
    engine = wrap_replicated(model, dev, torch.bfloat16)
    opt = ReplicatedMuonAdamW(engine, **MUON_HP)
    gen = torch.Generator(device=dev).manual_seed(3)
    history = []
    for _ in range(3):
        opt.zero_grad()
        model(_muon_tokens(gen, dev)).float().square().mean().backward()
        history.append({n: p.grad.float().clone() for n, p in model.named_parameters()})
        opt.step()
    torch.cuda.synchronize()
    want = _muon_reference(shadow, history)
    for s in engine.slots:
        got = engine.master[s.shard:s.shard + s.shard_numel].view(s.shape).cpu()
        torch.testing.assert_close(got, want[s.fqn], rtol=1e-4, atol=1e-5, msg=lambda m, n=s.fqn: f"{n}: {m}")
        assert torch.equal(s.param.detach().cpu(), got.to(torch.bfloat16))


def _muon_rank(rank, world, port, out):
    import sys
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(__file__))
    from mimir_b200.parallel.replicated import ReplicatedMuonAdamW, wrap_replicated
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        model = _muon_net(dev)
        engine = wrap_replicated(model, dev, torch.bfloat16)
        opt = ReplicatedMuonAdamW(engine, **MUON_HP)
        for step in range(3):
            opt.zero_grad()
            gen = torch.Generator(device=dev).manual_seed(100 * step + rank)
            model(_muon_tokens(gen, dev)).float().square().mean().backward()
            torch.save({n: p.grad.detach().float().cpu() for n, p in model.named_parameters()},
                       f"{out}.grad.{step}.{rank}.pt")
            opt.step()
        torch.cuda.synchronize()
        torch.save({n: p.detach().float().cpu() for n, p in model.named_parameters()}, f"{out}.w.{rank}.pt")
        torch.save({s.fqn: engine.master[s.shard:s.shard + s.shard_numel].cpu() for s in engine.slots},
                   f"{out}.m.{rank}.pt")
        engine.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_multi_gpu_muon_step_matches_summed_reference(tmp_path):
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    mp.spawn(_muon_rank, args=(world, _free_port(), str(tmp_path / "r")), nprocs=world, join=True)
    weights = [torch.load(tmp_path / f"r.w.{r}.pt") for r in range(world)]
    for r in range(1, world):
        for n in weights[0]:
            assert torch.equal(weights[0][n], weights[r][n]), (r, n)
    history = []
    for step in range(3):
        grads = [torch.load(tmp_path / f"r.grad.{step}.{r}.pt") for r in range(world)]
        history.append({n: sum(gr[n] for gr in grads) for n in grads[0]})
    want = _muon_reference(_muon_net("cpu"), history)
    masters = [torch.load(tmp_path / f"r.m.{r}.pt") for r in range(world)]
    for n, w in want.items():
        rows = w.shape[0] if w.dim() else 1
        chunk = -(-rows // world)
        for r in range(world):
            piece = w.reshape(rows, -1)[r * chunk:(r + 1) * chunk].reshape(-1)
            torch.testing.assert_close(masters[r][n], piece, rtol=1e-4, atol=1e-5, msg=lambda m, n=n: f"{n}: {m}")


def test_lean_update_variant_is_bit_identical():
    """The update that runs beside the backward (128-thread CTAs, one per chunk, no gradient
    prefetch) computes exactly what the persistent variant computes."""
    from mimir_b200.parallel.replicated import ReplicatedAdamATan2, wrap_replicated
    dev = torch.device("cuda", 0)
    runs = []
    for lean in (False, True):
        model = _model(dev)
        engine = wrap_replicated(model, dev, torch.bfloat16)
        opt = ReplicatedAdamATan2(engine, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9)
        gen = torch.Generator(device=dev).manual_seed(3)
        for _ in range(3):
            opt.zero_grad()
            x = torch.randn(33, 64, device=dev, dtype=torch.bfloat16, generator=gen)
            model(x).float().square().mean().backward()
            slots = [s for s in engine.slots if s.fqn in engine.touched]
            opt.update_slots(slots[:1], lean=lean)  # two launches, as the overlapped step makes them
            opt.update_slots(slots[1:], lean=lean, closing=True)
        torch.cuda.synchronize()
        runs.append((engine.master.clone(), opt.exp_avg_sq.clone(), opt.ema.clone(), engine.weights.clone()))
        engine.close()
    for a, b in zip(*runs):
        assert torch.equal(a, b)


class _Blocks(torch.nn.Module):
    """A head, three blocks (block 1 used twice) and an input projection registered last."""

    def __init__(self):
        super().__init__()
        self.blocks = torch.nn.ModuleList(torch.nn.Sequential(torch.nn.Linear(64, 64), torch.nn.Tanh())
                                          for _ in range(3))
        self.head = torch.nn.Linear(64, 32, bias=False)
        self.embed = torch.nn.Linear(64, 64)

    def forward(self, x):
        h = self.embed(x)
        for i in (0, 1, 1, 2):
            h = h + self.blocks[i](h)
        return self.head(h)


def _overlap_rank(rank, world, port, out):
    """Trains the same model with the update overlapped with the backward and without; every rank
    sees its own data, so each bucket's update reads the peers' gradients."""
    from contextlib import nullcontext
    from datetime import timedelta

    import torch.distributed as dist
    from mimir_b200.parallel.replicated import ReplicatedAdamATan2, wrap_replicated
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    try:
        results = []
        for enabled in (False, True):
            torch.manual_seed(0)
            model = _Blocks().to(dev)
            engine = wrap_replicated(model, dev, torch.bfloat16)
            engine.overlap_enabled = enabled
            opt = ReplicatedAdamATan2(engine, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9)
            gen = torch.Generator(device=dev).manual_seed(100 + rank)
            armed_steps = 0
            for _ in range(6):
                opt.zero_grad()
                x = torch.randn(48, 64, device=dev, dtype=torch.bfloat16, generator=gen)
                armed = engine.arm_overlap(opt)
                armed_steps += armed
                with engine.compute_stream() if armed else nullcontext():
                    model(x).float().square().mean().backward()
                opt.step()
            torch.cuda.synchronize()
            results.append((engine.master.cpu(), opt.exp_avg_sq.cpu(), opt.ema.cpu(), engine.weights.cpu(),
                            armed_steps))
            dist.barrier()
            engine.close()
        torch.save(results, f"{out}.{rank}.pt")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_multi_gpu_overlapped_update_equals_closing_update(tmp_path):
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    mp.spawn(_overlap_rank, args=(world, _free_port(), str(tmp_path / "o")), nprocs=world, join=True)
    ranks = [torch.load(tmp_path / f"o.{r}.pt") for r in range(world)]
    for plain, over in ranks:
        assert plain[4] == 0 and over[4] == 4  # two learning steps, then four overlapped ones
        for a, b in zip(plain[:4], over[:4]):
            assert torch.equal(a, b)
    for r in range(1, world):
        assert torch.equal(ranks[r][1][3], ranks[0][1][3])  # every replica holds the same weights


@pytest.mark.parametrize("extra", [{}, dict(moe_num_experts=4, moe_top_k=2, moe_sparse=True, moe_dispatch="grouped",
                                             moe_aux_loss_free=True, moe_expert_intermediate_size=256)],
                         ids=["dense", "moe"])
def test_overlapped_update_is_bit_identical_in_the_training_step(extra):
    """The real model on the tcgen05 kernels (dense, and a routed MoE with grouped experts and
    routing balance), trained through ``train_accumulated_batches`` with the update overlapped
    with the backward and without, and overlapped a second time: the master weights, moments and
    EMA of all three runs must match bit for bit (any weight read racing its bucket's update, or
    any nondeterministic kernel, would show here)."""
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    from test_reference_losses_gpu import MODEL, OPTIM, SEQ, SEQS, _batches, _on

    from mimir_b200.config.schema import PretrainConfig
    from mimir_b200.models import LMHead, Mimir2
    from mimir_b200.models.common import wrap_tensor
    from mimir_b200.optim.schedules import update_lr
    from mimir_b200.parallel.replicated import ReplicatedAdamATan2, wrap_replicated
    from mimir_b200.train.setup import make_train_state
    from mimir_b200.train.steps import train_accumulated_batches
    dev = torch.device("cuda", 0)
    model_cfg = MODEL | extra
    arch = {k: v for k, v in model_cfg.items() if k not in ("vocab_size", "max_seq_len", "fwd_bwd_dtype")}
    config = PretrainConfig(arch=arch, data=dict(path="synthetic"), global_batch_size=SEQ * SEQS,
                            distributed_strategy="replicated", **OPTIM)
    batches = _batches()
    runs = []
    for enabled in (False, True, True):
        torch.manual_seed(0)
        model = LMHead(Mimir2(model_cfg), model_cfg).to(dev)
        engine = wrap_replicated(model, dev, torch.bfloat16)
        engine.overlap_enabled = enabled
        optim = ReplicatedAdamATan2(engine, lr=0.0, betas=(0.9, 0.95), weight_decay=0.1, ema=0.999,
                                    ema_dtype=torch.float32)
        state = make_train_state(config, model, None, optim, total_steps=10_000, device=dev)
        for i in range(6):
            state.step += 1
            update_lr(config, state)
            train_accumulated_batches(config, 0, state, [_on(dev, batches[i % 2], wrap_tensor)])
        torch.cuda.synchronize()
        assert engine.overlap_ready is (True if enabled else None)
        runs.append((engine.master.clone(), optim.exp_avg_sq.clone(), optim.ema.clone()))
        engine.close()
    for other in runs[1:]:
        for a, b in zip(runs[0], other):
            assert torch.equal(a, b)
