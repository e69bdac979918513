"""Grouped MoE dispatch and expert parallelism on CPU (Gloo ranks).

* The grouped token exchange (top-k slots permuted into per-expert row blocks, one GEMM pair
  per expert, weighted combine) equals the reference-style sparse path (per-expert
  ``index_select`` / ``index_add``, ``src/mimir/model/expert_mixtures.py:92-104``) in fp32,
  forward and backward.
* With expert parallelism on two Gloo ranks (each rank owns half of the experts; token rows
  travel with ``all_to_all_single``), outputs and gradients equal the one-process grouped
  path over the concatenated batch, and every expert's weights get their gradient on the rank
  that owns them.
* The replicated engine keeps expert-parallel parameters rank-local (no reduction): two ranks
  training an EP model match one process training the same model on both ranks' data.
"""
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mimir_b200.models.experts import MLPMixture
from mimir_b200.models.layers import SwiGLU

D, F, E, K = 16, 24, 4, 2


def _mixture(grouped=False, ep=False, shared=0, width=None, seed=0):
    torch.manual_seed(seed)
    return MLPMixture(SwiGLU(D, F), D, E, K, sparse=True, grouped=grouped, expert_parallel=ep, shared_experts=shared,
                      expert_intermediate_size=width)


def _inputs(seed, T=13):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(T, D, generator=g), torch.randn(T, D, generator=g)


@pytest.mark.parametrize("shared,width", [(0, None), (1, 32)])
def test_grouped_matches_index_dispatch(shared, width):
    ref, grp = _mixture(shared=shared, width=width), _mixture(grouped=True, shared=shared, width=width)
    with torch.no_grad():  # identical router rows so the selection differs between experts
        for i, r in enumerate(ref.router.rows):
            r.copy_(torch.randn(D, generator=torch.Generator().manual_seed(10 + i)))
    grp.load_state_dict(ref.state_dict())
    x, g = _inputs(1)
    outs = []
    for m in (ref, grp):
        xi = x.clone().requires_grad_(True)
        y = m(xi)
        (y * g).sum().backward()
        outs.append((y.detach(), xi.grad, {n: p.grad.clone() for n, p in m.named_parameters()}))
    torch.testing.assert_close(outs[1][0], outs[0][0], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(outs[1][1], outs[0][1], rtol=1e-5, atol=1e-6)
    for n in outs[0][2]:
        torch.testing.assert_close(outs[1][2][n], outs[0][2][n], rtol=1e-5, atol=1e-6, msg=n)


def _ep_worker(rank, world, init, out):
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        m = _mixture(grouped=True, ep=True, shared=1, width=32)
        assert sorted(m.experts.keys()) == [str(i) for i in range(rank * E // world, (rank + 1) * E // world)]
        assert all(getattr(p, "_mimir_rank_local", False) for p in m.experts.parameters())
        x, g = _inputs(100 + rank)
        x.requires_grad_(True)
        y = m(x)
        (y * g).sum().backward()
        torch.save({"y": y.detach(), "dx": x.grad, "grads": {n: p.grad for n, p in m.named_parameters()}},
                   f"{out}.{rank}.pt")
    finally:
        dist.destroy_process_group()


def test_expert_parallel_two_ranks_match_one_process(tmp_path):
    world = 2
    mp.spawn(_ep_worker, args=(world, f"file://{tmp_path / 'rdv'}", str(tmp_path / "ep")), nprocs=world, join=True)
    full = _mixture(grouped=True, shared=1, width=32)
    res = [torch.load(tmp_path / f"ep.{r}.pt") for r in range(world)]
    xs = [_inputs(100 + r) for r in range(world)]
    x = torch.cat([a for a, _ in xs]).requires_grad_(True)
    g = torch.cat([b for _, b in xs])
    y = full(x)
    (y * g).sum().backward()
    T = xs[0][0].shape[0]
    for r in range(world):
        torch.testing.assert_close(res[r]["y"], y[r * T:(r + 1) * T].detach(), rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(res[r]["dx"], x.grad[r * T:(r + 1) * T], rtol=1e-5, atol=1e-6)
    grads = {n: p.grad for n, p in full.named_parameters()}
    for n, want in grads.items():
        if n.startswith("experts."):
            owner = int(n.split(".")[1]) // (E // world)
            torch.testing.assert_close(res[owner]["grads"][n], want, rtol=1e-5, atol=1e-6, msg=n)
        else:  # replicated parameters: the data-parallel sum of the ranks' gradients
            torch.testing.assert_close(res[0]["grads"][n] + res[1]["grads"][n], want, rtol=1e-5, atol=1e-6, msg=n)


def test_route_plan_groups_rows_by_expert_in_token_order():
    from mimir_b200.parallel.expert import expert_parallel
    ep = expert_parallel(E, torch.device("cpu"), distributed=False)
    topi = torch.tensor([[2, 0], [0, 3], [2, 1], [3, 2], [0, 1]])
    plan = ep.plan(topi)
    rows = plan.rows.reshape(-1).tolist()
    assert sorted(rows) == list(range(topi.numel()))
    assert plan.expert_rows == [3, 2, 3, 2] and plan.capacity == 10
    by_row = sorted(zip(rows, topi.reshape(-1).tolist(), [i // 2 for i in range(10)]))
    assert [e for _, e, _ in by_row] == [0, 0, 0, 1, 1, 2, 2, 2, 3, 3]
    for e in range(E):  # token order inside an expert's block
        toks = [t for _, ee, t in by_row if ee == e]
        assert toks == sorted(toks)


class _Net(torch.nn.Module):
    def __init__(self, ep):
        super().__init__()
        torch.manual_seed(0)
        self.inp = torch.nn.Linear(D, D)
        self.mix = MLPMixture(SwiGLU(D, F), D, E, K, sparse=True, grouped=True, expert_parallel=ep, shared_experts=1,
                              expert_intermediate_size=32)

    def forward(self, x):
        return self.mix(self.inp(x))


def _train(net, opt, xs):
    for i, (x, g) in enumerate(xs):
        opt.zero_grad()
        (net(x) * g).sum().backward()
        for group in opt.param_groups:
            group["lr"] = 1e-2 * (i + 1)
        opt.step()


def _engine_worker(rank, world, init, out):
    from mimir_b200.parallel.replicated import ReplicatedAdamATan2, model_dcp_state, wrap_replicated
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        net = _Net(ep=True)
        engine = wrap_replicated(net, torch.device("cpu"), torch.float32)
        assert [s.local for s in engine.slots] == sorted(s.local for s in engine.slots)  # local slots last
        opt = ReplicatedAdamATan2(engine, lr=0.0, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9)
        _train(net, opt, [_inputs(10 * s + rank) for s in range(2)])
        torch.save({n: p.detach().clone() for n, p in net.named_parameters()}, f"{out}.{rank}.pt")
        import torch.distributed.checkpoint as dcp
        dcp.save({"model": model_dcp_state(engine), "optim": opt.dcp_state()}, checkpoint_id=f"{out}.dcp")
    finally:
        dist.destroy_process_group()


def test_replicated_engine_keeps_expert_parallel_parameters_local(tmp_path):
    from mimir_b200.parallel.replicated import ReplicatedAdamATan2, wrap_replicated
    world = 2
    mp.spawn(_engine_worker, args=(world, f"file://{tmp_path / 'rdv'}", str(tmp_path / "w")), nprocs=world, join=True)
    net = _Net(ep=False)
    engine = wrap_replicated(net, torch.device("cpu"), torch.float32)
    opt = ReplicatedAdamATan2(engine, lr=0.0, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9)
    batches = []
    for s in range(2):
        xs = [_inputs(10 * s + r) for r in range(world)]
        batches.append((torch.cat([a for a, _ in xs]), torch.cat([b for _, b in xs])))
    _train(net, opt, batches)
    want = {n: p.detach() for n, p in net.named_parameters()}
    got = [torch.load(tmp_path / f"w.{r}.pt") for r in range(world)]
    for n, w in want.items():
        if n.startswith("mix.experts."):
            owner = int(n.split(".")[2]) // (E // world)
            assert n in got[owner] and n not in got[1 - owner]
            torch.testing.assert_close(got[owner][n], w, rtol=1e-5, atol=1e-6, msg=n)
        else:
            for r in range(world):
                torch.testing.assert_close(got[r][n], w, rtol=1e-5, atol=1e-6, msg=n)
    import torch.distributed.checkpoint as dcp
    meta = dcp.FileSystemReader(str(tmp_path / "w.dcp")).read_metadata()
    keys = set(meta.state_dict_metadata)
    for e in range(E):
        assert f"model.mix.experts.{e}.gate_up_proj.weight" in keys
        assert f"optim.state.mix.experts.{e}.down_proj.weight.exp_avg" in keys
    full = {f"model.mix.experts.{e}.down_proj.weight": torch.empty(want[f"mix.experts.{e}.down_proj.weight"].shape)
            for e in range(E)}
    dcp.load(full, checkpoint_id=str(tmp_path / "w.dcp"), no_dist=True)
    for e in range(E):
        torch.testing.assert_close(full[f"model.mix.experts.{e}.down_proj.weight"],
                                   want[f"mix.experts.{e}.down_proj.weight"], rtol=1e-5, atol=1e-6)


# ------------------------------------------------------------------ EP training: checkpoint + exact resume
def _launch_worker(rank, world, port, overrides):
    import os
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), LOCAL_WORLD_SIZE=str(world),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from mimir_b200.config.schema import load_config
    from mimir_b200.train.loop import launch
    try:
        launch(load_config(overrides))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_parallel_training_resumes_exactly(tmp_path):
    from mimir_b200.data.synthetic import write_corpus
    from test_replicated_dp import BASE
    from test_train_resume import _same_state, _tensors
    data = write_corpus(str(tmp_path / "d"), rows=64, seq_len=32, vocab=64)
    common = BASE + [f"data.path={data}", "distributed_strategy=replicated", "arch.moe_num_experts=4",
                     "arch.moe_top_k=2", "arch.moe_sparse=true", "arch.moe_dispatch=grouped",
                     "arch.moe_expert_parallel=true", "arch.moe_expert_intermediate_size=32",
                     "arch.moe_shared_experts=1", "arch.moe_aux_loss_free=true", "arch.moe_router_init_std=0.1"]
    runs = [(tmp_path / "full", ["checkpoint_step_interval=3", "stop_after_step=6"]),
            (tmp_path / "resumed", ["stop_after_step=6", f"resume_checkpoint_path={tmp_path / 'full'}",
                                    "resume_checkpoint_tag=step_3"])]
    for run, extra in runs:
        mp.spawn(_launch_worker, args=(2, _free_port(), common + [f"checkpoint_path={run}", *extra]), nprocs=2,
                 join=True)
    _same_state(tmp_path / "full", tmp_path / "resumed", "step_6")
    keys = set(_tensors(tmp_path / "full" / "step_6", "step_6"))
    experts = {k for k in keys if ".mlp.experts." in k and k.startswith("model.")}
    assert {k.split(".mlp.experts.")[1].split(".")[0] for k in experts} == {"0", "1", "2", "3"}
    assert any(".mlp.shared_experts.0." in k for k in keys)
