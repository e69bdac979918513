"""Replicated-weight data parallelism (sharded fp32 master + optimizer, fused step) on CPU.

The CPU path runs the same algorithm as the fused CUDA kernel with PyTorch ops; these tests
pin it to the per-parameter AdamATan2 (bit-exact on one rank; on two Gloo ranks that see
identical data the summed gradient is exactly 2x and AdamATan2 is scale invariant, so only the
last bit of the vectorised CPU atan2 may differ with the shard layout) and check
that its DCP checkpoints resume exactly and load into a non-replicated model.
"""

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mimir_b200.optim.adam_atan2 import AdamATan2
from mimir_b200.parallel.replicated import ReplicatedAdamATan2, wrap_replicated


def _model():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Linear(16, 24), torch.nn.GELU(), torch.nn.Linear(24, 5, bias=False))


def _train(model, optim, steps=3, seed=1):
    gen = torch.Generator().manual_seed(seed)
    for i in range(steps):
        x = torch.randn(7, 16, generator=gen)
        optim.zero_grad()
        model(x).square().sum().backward()
        for g in optim.param_groups:
            g["lr"] = 1e-2 * (i + 1)
        optim.step()


def _reference():
    ref = _model()
    opt = AdamATan2(ref.parameters(), lr=0.0, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9, fused=False)
    _train(ref, opt)
    return ref, opt


def test_single_rank_matches_per_parameter_optimizer():
    ref, ref_opt = _reference()
    model = _model()
    engine = wrap_replicated(model, torch.device("cpu"), torch.float32)
    opt = ReplicatedAdamATan2(engine, lr=0.0, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9)
    _train(model, opt)
    for s, (name, p) in zip(engine.slots, ref.named_parameters()):
        assert s.fqn == name
        assert torch.equal(engine.master[s.shard:s.shard + s.shard_numel].view(p.shape), p.detach()), name
        assert torch.equal(s.param.detach(), p.detach()), name
        st = ref_opt.state[p]
        assert torch.equal(opt.ema[s.shard:s.shard + s.shard_numel].view(p.shape), st["param_ema"])
        assert torch.equal(opt.exp_avg_sq[s.shard:s.shard + s.shard_numel].view(p.shape), st["exp_avg_sq"])


def _worker(rank, world, init, out):
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        model = _model()
        engine = wrap_replicated(model, torch.device("cpu"), torch.float32)
        opt = ReplicatedAdamATan2(engine, lr=0.0, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9)
        _train(model, opt)  # identical data on every rank
        torch.save({n: p.detach().clone() for n, p in model.named_parameters()}, f"{out}.{rank}.pt")
        # sharded checkpoint written through DCP with Shard(0) placements
        from mimir_b200.parallel.replicated import model_dcp_state
        import torch.distributed.checkpoint as dcp
        dcp.save({"model": model_dcp_state(engine), "optim": opt.dcp_state()}, checkpoint_id=f"{out}.dcp")
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_equal_single_process(tmp_path):
    ref, _ = _reference()
    init = f"file://{tmp_path / 'rdv'}"
    mp.spawn(_worker, args=(2, init, str(tmp_path / "w")), nprocs=2, join=True)
    for r in range(2):
        got = torch.load(tmp_path / f"w.{r}.pt")
        for name, p in ref.named_parameters():
            # same arithmetic on a different shard layout: CPU atan2 vectorisation may differ in the last bit
            torch.testing.assert_close(got[name], p.detach(), rtol=1e-6, atol=1e-7)
    # the DCP checkpoint holds full fp32 tensors under FSDP-style keys; load it unsharded
    import torch.distributed.checkpoint as dcp
    from torch.distributed.checkpoint.metadata import TensorStorageMetadata
    meta = dcp.FileSystemReader(str(tmp_path / "w.dcp")).read_metadata()
    keys = {k for k, m in meta.state_dict_metadata.items() if isinstance(m, TensorStorageMetadata)}
    assert {"model.0.weight", "optim.state.0.weight.exp_avg", "optim.state.0.weight.param_ema"} <= keys
    full = {k: torch.empty(meta.state_dict_metadata[k].size) for k in ("model.0.weight", "model.2.weight")}
    dcp.load(full, checkpoint_id=str(tmp_path / "w.dcp"), no_dist=True)
    torch.testing.assert_close(full["model.0.weight"], ref[0].weight.detach(), rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(full["model.2.weight"], ref[2].weight.detach(), rtol=1e-6, atol=1e-7)


BASE = ["size@arch=XXS", "accelerator_type=cpu", "fwd_bwd_dtype=float32", "global_batch_size=128", "epochs=1",
        "lr_warmup_steps=2", "log_interval=2", "arch.hidden_size=64", "arch.n_layers=2", "arch.H_cycles=2",
        "arch.L_cycles=2", "dataloader_prefetch_factor=2"]


@pytest.mark.parametrize("optimizer", ["adam_atan2", "muon"])
def test_replicated_training_resumes_exactly_and_matches_plain(tmp_path, optimizer):
    from mimir_b200.config.schema import load_config
    from mimir_b200.data.synthetic import write_corpus
    from mimir_b200.train.loop import launch
    from test_train_resume import _same_state, _tensors
    data = write_corpus(str(tmp_path / "d"), rows=64, seq_len=32, vocab=64)
    common = BASE + [f"data.path={data}", f"optimizer={optimizer}"]
    launch(load_config(common + ["distributed_strategy=none", f"checkpoint_path={tmp_path / 'plain'}",
                                 "stop_after_step=6"]))
    launch(load_config(common + ["distributed_strategy=replicated", f"checkpoint_path={tmp_path / 'rep'}",
                                 "checkpoint_step_interval=3", "stop_after_step=6"]))
    if dist.is_initialized():
        dist.destroy_process_group()
    launch(load_config(common + ["distributed_strategy=replicated", f"checkpoint_path={tmp_path / 'resumed'}",
                                 "stop_after_step=6", f"resume_checkpoint_path={tmp_path / 'rep'}",
                                 "resume_checkpoint_tag=step_3"]))
    if dist.is_initialized():
        dist.destroy_process_group()
    _same_state(tmp_path / "rep", tmp_path / "resumed", "step_6")
    # plain vs replicated: same arithmetic, different memory layout (CPU atan2 vector/tail split)
    plain, rep = _tensors(tmp_path / "plain" / "step_6", "step_6"), _tensors(tmp_path / "rep" / "step_6", "step_6")
    assert plain.keys() == rep.keys()
    for k in plain:
        torch.testing.assert_close(plain[k], rep[k], rtol=1e-5, atol=1e-6, msg=k)


class _Blocks(torch.nn.Module):
    """Three blocks and a head; block 1 runs twice per forward (two gradient arrivals per weight).
    The input projection is registered last but used first, like a language model's embedding."""

    def __init__(self):
        super().__init__()
        torch.manual_seed(0)
        self.blocks = torch.nn.ModuleList(torch.nn.Sequential(torch.nn.Linear(24, 24), torch.nn.Tanh())
                                          for _ in range(3))
        self.head = torch.nn.Linear(24, 5, bias=False)
        self.embed = torch.nn.Linear(16, 24)

    def forward(self, x):
        h = self.embed(x)
        for i in (0, 1, 1, 2):
            h = h + self.blocks[i](h)
        return self.head(h)


def _train_overlapped(model, opt, engine, steps, seed=1):
    """Arms the engine before each backward, as the training step does; returns the number of
    bucket updates that ran inside a backward and, for the last step, the gradient arrival after
    which each of them ran."""
    gen = torch.Generator().manual_seed(seed)
    inside, when = [], []
    update = opt.update_slots

    def spy(slots, closing=False, lean=False):
        inside.append(engine.overlap_armed() and not closing)
        when.append(engine._arrival_seq)
        update(slots, closing, lean)
    opt.update_slots = spy
    for i in range(steps):
        x = torch.randn(7, 16, generator=gen)
        opt.zero_grad()
        for g in opt.param_groups:
            g["lr"] = 1e-2 * (i + 1)
        when.clear()
        engine.arm_overlap(opt)
        model(x).square().sum().backward()
        opt.step()
    return sum(inside), list(when)


def _overlap_worker(rank, world, init, out):
    if world > 1:
        dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        results = []
        for enabled in (False, True):
            model = _Blocks()
            engine = wrap_replicated(model, torch.device("cpu"), torch.float32)
            engine.overlap_enabled = enabled
            opt = ReplicatedAdamATan2(engine, lr=0.0, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9)
            fired, when = _train_overlapped(model, opt, engine, steps=5)
            results.append(({n: p.detach().clone() for n, p in model.named_parameters()},
                            opt.exp_avg_sq.clone(), opt.ema.clone(), fired, when))
        torch.save(results, f"{out}.{rank}.pt")
    finally:
        if world > 1:
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2])
def test_update_overlapped_with_backward_equals_closing_update(tmp_path, world):
    """Bucket-by-bucket updates inside the backward give the same weights, moments and EMA as
    the single update after it; two steps teach the arrival counts, the last three overlap."""
    init = f"file://{tmp_path / 'rdv'}"
    if world == 1:
        _overlap_worker(0, 1, init, str(tmp_path / "o"))
    else:
        mp.spawn(_overlap_worker, args=(world, init, str(tmp_path / "o")), nprocs=world, join=True)
    for rank in range(world):
        (plain, v0, e0, fired0, _), (over, v1, e1, fired1, when) = torch.load(f"{tmp_path / 'o'}.{rank}.pt")
        assert fired0 == 0 and fired1 == 3 * 6  # 3 overlapped steps x (head, 3 blocks, embed weight, bias)
        # head and blocks are updated while the backward still runs (after arrivals 1, 3, 7, 9 of 11)
        assert when == sorted(when) and len(set(when)) >= 5 and when[0] < when[-1] - 5, when
        for n in plain:
            assert torch.equal(plain[n], over[n]), n
        assert torch.equal(v0, v1) and torch.equal(e0, e1)


def test_gradient_after_its_bucket_update_raises():
    model = _Blocks()
    engine = wrap_replicated(model, torch.device("cpu"), torch.float32)
    opt = ReplicatedAdamATan2(engine, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9)
    _train_overlapped(model, opt, engine, steps=2)
    opt.zero_grad()
    assert engine.arm_overlap(opt)
    model(torch.randn(7, 16)).square().sum().backward()
    model.head(torch.randn(3, 24)).sum().backward()  # a second arrival for the already-updated head
    with pytest.raises(RuntimeError, match="arrived after its bucket was updated"):
        opt.step()


def test_stacked_router_rows_match_torch_stack():
    """Router rows under the engine are read as one strided matrix and their gradients written by
    one add: the gradients equal those of ``torch.stack`` and every parameter is announced."""
    from mimir_b200.models.experts import TopKRouter
    from mimir_b200.ops.stacked import _StackedFn, stacked

    def build(freeze_base=False):
        torch.manual_seed(0)
        return TopKRouter(16, 6, 2, init_std=0.02, freeze_base=freeze_base)

    x = torch.randn(10, 16)
    for freeze in (False, True):
        plain, wrapped = build(freeze), build(freeze)
        engine = wrap_replicated(wrapped, torch.device("cpu"), torch.float32)
        fast = stacked(wrapped.rows).grad_fn
        assert (type(fast).__name__ == _StackedFn.__name__ + "Backward") is not freeze
        for m in (plain, wrapped):
            for _ in range(2):  # two micro-batches accumulate
                m.scores(x).square().sum().backward()
        params = dict(plain.named_parameters())
        for s in engine.slots:
            if s.trainable:
                assert torch.allclose(s.param.grad, params[s.fqn].grad, rtol=1e-6, atol=1e-7), s.fqn
        # every trainable row and bias was announced, equally often (the counts the overlap learns)
        counts = {engine.arrivals.get(s.fqn, 0) for s in engine.slots if s.trainable}
        assert len(counts) == 1 and counts.pop() >= 2
        engine.close()


def _sharded_worker(rank, world, init, out):
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        from mimir_b200.parallel.sharded_linear import ShardedLinear
        torch.manual_seed(0)
        w = torch.randn(8, 6)
        layer = ShardedLinear(w, device="cpu")
        x = torch.randn(5, 6, generator=torch.Generator().manual_seed(rank), requires_grad=True)
        y = layer(x)
        y.square().sum().backward()
        torch.save({"y": y.detach(), "x": x.detach(), "dx": x.grad, "dshard": layer.shard.grad,
                    "full": layer.full_weight()}, f"{out}.{rank}.pt")
    finally:
        dist.destroy_process_group()


def test_sharded_linear_two_gloo_ranks(tmp_path):
    """Row-sharded projection on CPU ranks: forward, input gradient, summed weight gradient."""
    world = 2
    init = f"file://{tmp_path / 'init'}"
    mp.spawn(_sharded_worker, args=(world, init, str(tmp_path / "s")), nprocs=world, join=True)
    torch.manual_seed(0)
    w = torch.randn(8, 6)
    rs = [torch.load(f"{tmp_path / 's'}.{r}.pt") for r in range(world)]
    grad = sum((2 * r["y"]).t() @ r["x"] for r in rs)
    for rank, r in enumerate(rs):
        assert torch.allclose(r["y"], r["x"] @ w.t(), atol=1e-6)
        assert torch.allclose(r["dx"], (2 * r["y"]) @ w, atol=1e-5)
        assert torch.allclose(r["dshard"], grad[rank * 4:(rank + 1) * 4], atol=1e-5)
        assert torch.equal(r["full"], w)


def test_zero_grad_zeroes_once_per_arrival_window():
    """The engine zeroes its gradient buffer when something arrived since the last zeroing and
    skips the call otherwise (training zeroes after the step and again before the next)."""
    model = _model()
    engine = wrap_replicated(model, torch.device("cpu"), torch.float32)
    opt = ReplicatedAdamATan2(engine, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, ema=0.9)
    calls = []
    real = engine.grads.zero_
    engine.grads.zero_ = lambda: (calls.append(1), real())[1]
    model(torch.randn(3, 16)).square().sum().backward()
    assert engine.grads.abs().sum() > 0
    opt.zero_grad()
    assert torch.count_nonzero(engine.grads) == 0 and len(calls) == 1
    opt.zero_grad()  # nothing arrived: skipped
    assert len(calls) == 1
    model(torch.randn(3, 16)).square().sum().backward()
    opt.step()
    opt.zero_grad()
    assert torch.count_nonzero(engine.grads) == 0 and len(calls) == 2
    engine.close()


def test_bf16_gradient_accumulation_drift_is_bounded():
    """The engine accumulates micro-batch gradients in its bf16 buffer (FSDP2 sums in fp32): over
    four micro-batches the accumulated gradient stays within three bf16 roundings (2^-8 each,
    relative to the largest magnitude) of the fp32 sum of the same micro-batch gradients."""
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(64, 96), torch.nn.GELU(), torch.nn.Linear(96, 32)).to(torch.bfloat16)
    engine = wrap_replicated(model, torch.device("cpu"), torch.bfloat16)
    gen = torch.Generator().manual_seed(3)
    batches = [torch.randn(16, 64, generator=gen).to(torch.bfloat16) for _ in range(4)]
    exact = torch.zeros(engine.grads.numel())
    for x in batches:  # each micro-batch alone: its gradient is exact in bf16 storage
        engine.zero_grad()
        model(x).float().square().sum().backward()
        exact += engine.grads.float()
    engine.zero_grad()
    for x in batches:
        model(x).float().square().sum().backward()
    drift = (engine.grads.float() - exact).abs().max() / exact.abs().max()
    assert drift <= 3 * 2.0 ** -8, float(drift)
    engine.close()


def _sharded_ckpt_worker(rank, world, init, out):
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        from mimir_b200.parallel.sharded_linear import ShardedLinear
        torch.manual_seed(0)
        w = torch.randn(8, 6)
        layer = ShardedLinear(w, device="cpu")
        state = layer.state_dict()
        assert list(state) == ["weight"] and torch.equal(state["weight"], w)
        other = ShardedLinear(torch.zeros(8, 6), device="cpu")
        other.load_state_dict({"weight": w * 2})
        torch.save(other.shard.detach().clone(), f"{out}.{rank}.pt")
    finally:
        dist.destroy_process_group()


def test_sharded_linear_checkpoints_hold_the_whole_matrix(tmp_path):
    mp.spawn(_sharded_ckpt_worker, args=(2, f"file://{tmp_path / 'init'}", str(tmp_path / "c")), nprocs=2, join=True)
    torch.manual_seed(0)
    w = torch.randn(8, 6)
    for rank in range(2):
        assert torch.equal(torch.load(f"{tmp_path / 'c'}.{rank}.pt"), 2 * w[rank * 4:(rank + 1) * 4])


@pytest.mark.parametrize("N,K,world,rank,pairs", [(5120, 2048, 8, 3, 74), (11264, 2048, 8, 0, 74), (2048, 5632, 2, 1, 74),
                                                  (1024, 136, 4, 2, 7), (65536, 2048, 8, 7, 74), (256, 64, 1, 0, 3)])
def test_allgather_gemm_work_split_covers_every_block_once(N, K, world, rank, pairs):
    """The index arithmetic of ``gemm_gather_kernel`` (``csrc/gemm.cu``), restated on the host:
    the gatherers' items cover every (128-row block, k-block) of the weight exactly once, each
    row block's counter grows by ``parts`` per call, and the tile order visits every output tile
    once starting at this rank's own columns."""
    nkb, blocks = (K + 63) // 64, N // 128
    parts = max(1, min(nkb, (2 * pairs + blocks - 1) // blocks))
    shard_rows, per_rank = N // world, N // world // 128
    items = world * per_rank * parts
    seen, counters = {}, [0] * blocks
    for cid in range(pairs):
        for item in range(cid, items, pairs):
            owner = (rank + 1 + (item // parts) // per_rank) % world
            grow = owner * shard_rows + ((item // parts) % per_rank) * 128
            lo, hi = ((item % parts) * nkb) // parts, ((item % parts + 1) * nkb) // parts
            assert hi > lo
            for kb in range(lo, hi):
                assert (grow, kb) not in seen
                seen[(grow, kb)] = cid
            counters[grow // 128] += 1
    assert len(seen) == blocks * nkb and counters == [parts] * blocks
    tiles_m, tiles_n = 3, N // 256
    order = [((t % tiles_m), (t // tiles_m + (rank * shard_rows) // 256) % tiles_n) for t in range(tiles_m * tiles_n)]
    assert len(set(order)) == tiles_m * tiles_n
    first_rows = order[0][1] * 256
    assert first_rows <= rank * shard_rows < first_rows + 256  # the first column holds this rank's first row
