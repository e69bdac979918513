"""Replicated-weight MuonAdamW (owner-rank Newton-Schulz, fused gather/scatter) on CPU.

The CPU path runs the algorithm of the fused CUDA step with PyTorch ops (momentum on the
shard, gather of the Nesterov input to the matrix's owner, Newton-Schulz once on the owner,
scatter + decay + update on every shard).  It must equal the per-parameter MuonAdamW
(reference behaviour ``src/mimir/model/muon.py:62-108``) on one rank and on two Gloo ranks,
and its DCP state must carry MuonAdamW's slot names.
"""
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

from mimir_b200.optim.muon import MuonAdamW
from mimir_b200.parallel.replicated import ReplicatedMuonAdamW, wrap_replicated


class _Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.embed = nn.Embedding(11, 8)
        self.attn = nn.Module()
        self.attn.gqkv_proj = nn.Linear(8, 20, bias=False)  # 4 logical 5x8 pieces
        self.attn.o_proj = nn.Linear(5, 8, bias=False)
        self.mlp = nn.Module()
        self.mlp.gate_up_proj = nn.Linear(8, 26, bias=False)  # 2 logical 13x8 pieces (tall)
        self.mlp.down_proj = nn.Linear(13, 8, bias=False)
        self.norm = nn.Parameter(torch.ones(8))
        self.head = nn.Linear(8, 3)

    def forward(self, tok):
        x = self.embed(tok) * self.norm
        g, q, k, v = self.attn.gqkv_proj(x).chunk(4, -1)
        x = x + self.attn.o_proj(torch.sigmoid(g) * q * k + v)
        a, b = self.mlp.gate_up_proj(x).chunk(2, -1)
        x = x + self.mlp.down_proj(torch.nn.functional.silu(a) * b)
        return self.head(x)


def _model():
    torch.manual_seed(0)
    return _Net()


HP = dict(lr=0.0, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9, momentum=0.95, ns_steps=5, muon_lr_scale=0.5)


def _train(model, optim, steps=3, seed=1):
    gen = torch.Generator().manual_seed(seed)
    for i in range(steps):
        tok = torch.randint(0, 11, (6, 5), generator=gen)
        optim.zero_grad()
        model(tok).square().mean().backward()
        for g in optim.param_groups:
            g["lr"] = 1e-2 * (i + 1)
        optim.step()


def _reference():
    ref = _model()
    opt = MuonAdamW(ref.named_parameters(), **HP)
    _train(ref, opt)
    return ref, opt


def _replicated():
    model = _model()
    engine = wrap_replicated(model, torch.device("cpu"), torch.float32)
    return model, engine, ReplicatedMuonAdamW(engine, **HP)


def test_owner_assignment_balances_and_covers_every_matrix():
    model, engine, opt = _replicated()
    matrices = {n for n, _ in model.named_parameters() if n.endswith(("gqkv_proj.weight", "o_proj.weight",
                                                                          "gate_up_proj.weight", "down_proj.weight"))}
    assert set(opt.owner) == matrices and set(opt.owner.values()) == {0}
    offsets = sorted(opt.work_offset.values())
    assert offsets[0] == 0 and all(o % 8 == 0 for o in offsets)


def test_single_rank_matches_muon_adamw():
    ref, ref_opt = _reference()
    model, engine, opt = _replicated()
    _train(model, opt)
    for s, (name, p) in zip(engine.slots, ref.named_parameters()):
        assert s.fqn == name
        torch.testing.assert_close(engine.master[s.shard:s.shard + s.shard_numel].view(p.shape), p.detach(),
                                   rtol=1e-6, atol=1e-7, msg=name)
        st = ref_opt.state[p]
        for slot, buf in opt.slot_buffers(s).items():
            torch.testing.assert_close(buf[s.shard:s.shard + s.shard_numel].view(p.shape), st[slot],
                                       rtol=1e-6, atol=1e-7, msg=f"{name}.{slot}")
        assert set(opt.slot_buffers(s)) | {"step"} == set(st), name


def _worker(rank, world, init, out):
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        model, engine, opt = _replicated()
        assert set(opt.owner.values()) == {0, 1}  # the matrices are split between the two ranks
        _train(model, opt)  # identical data on every rank: the summed gradient is 2x
        torch.save({n: p.detach().clone() for n, p in model.named_parameters()}, f"{out}.{rank}.pt")
        state = opt.dcp_state()["state"]
        torch.save({k: sorted(v) for k, v in state.items()}, f"{out}.slots.{rank}.pt")
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_match_muon_adamw_on_doubled_gradients(tmp_path):
    ref = _model()
    opt = MuonAdamW(ref.named_parameters(), **HP)
    gen = torch.Generator().manual_seed(1)
    for i in range(3):  # two ranks with identical data sum to twice the gradient
        tok = torch.randint(0, 11, (6, 5), generator=gen)
        opt.zero_grad()
        (2 * ref(tok).square().mean()).backward()
        for g in opt.param_groups:
            g["lr"] = 1e-2 * (i + 1)
        opt.step()
    mp.spawn(_worker, args=(2, f"file://{tmp_path / 'rdv'}", str(tmp_path / "w")), nprocs=2, join=True)
    for r in range(2):
        got = torch.load(tmp_path / f"w.{r}.pt")
        for name, p in ref.named_parameters():
            torch.testing.assert_close(got[name], p.detach(), rtol=1e-5, atol=1e-6, msg=lambda m: f"{name}: {m}")
    slots = torch.load(tmp_path / "w.slots.0.pt")
    assert slots["attn.gqkv_proj.weight"] == ["momentum_buffer", "param_ema", "step"]
    assert slots["norm"] == ["exp_avg", "exp_avg_sq", "param_ema", "step"]


@pytest.mark.parametrize("bad", [dict(momentum=1.0), dict(ns_steps=0), dict(muon_lr_scale=0.0)])
def test_invalid_hyperparameters(bad):
    model = _model()
    engine = wrap_replicated(model, torch.device("cpu"), torch.float32)
    with pytest.raises(ValueError):
        ReplicatedMuonAdamW(engine, **(HP | bad))
