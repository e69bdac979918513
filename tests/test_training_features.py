"""Training-step features on CPU: GAS parity under DDP/FSDP2 (2 Gloo ranks), HSDP mesh shapes,
gradient skipping, per-module learning rates, routing-balance counts with idle ranks,
activation checkpointing and torch.compile equivalence.

Mirrors the reference's test strategy (``tests/test_distributed_gas.py``,
``tests/test_hrm_experts.py:183-240``, ``tests/test_fsdp_topology.py:84-114``,
``tests/test_gradient_skip.py``, ``tests/test_module_learning_rates.py``,
``tests/test_routing_balance.py:56-68``).
"""
import os
from unittest import mock

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mimir_b200.config.schema import PretrainConfig
from mimir_b200.models.common import wrap_tensor

ARCH = dict(n_layers=2, hidden_size=16, num_heads=2, H_cycles=2, L_cycles=2, half_layers=False, max_seq_len=64,
            rope_theta=10000.0, bp_min_steps=3, bp_max_steps=3)


def _config(**kw):
    base = dict(arch=ARCH, data=dict(path="unused"), global_batch_size=48, epochs=1, lr=1e-2, lr_warmup_steps=0,
                lr_min_ratio=1.0, weight_decay=0.1, beta1=0.9, beta2=0.95, ema=0.9, fwd_bwd_dtype="float32",
                accelerator_type="cpu", distributed_strategy="none", lr_auto=False)
    arch = dict(ARCH) | kw.pop("arch", {})
    return PretrainConfig(**(base | kw | {"arch": arch}))


def _batches(n, T=24, seed=0):
    from mimir_b200.data.prefixlm import compute_aux_seq_tensors_scalars
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        p, c = np.array([3, 5], np.int32), np.array([7, 9], np.int32)
        tensors, scalars = compute_aux_seq_tensors_scalars(p, c, T)
        inputs = torch.randint(0, 32, (T,), generator=g)
        labels = torch.randint(0, 32, (T,), generator=g)
        labels[:3] = -100
        pos = torch.cat([torch.arange(10), torch.arange(14), torch.zeros(T - 24, dtype=torch.long)])
        out.append(dict(inputs=inputs, labels=labels, position_ids=pos) | {k: torch.from_numpy(v) for k, v in tensors.items()}
                   | {k: wrap_tensor(torch.tensor(v)) for k, v in scalars.items()})
    return out


def _state(config, rank=0):
    from mimir_b200.train.setup import create_model_and_optimizer, make_train_state
    torch.manual_seed(0)
    model, carry, optim = create_model_and_optimizer(config, {"vocab_size": 32, "max_seq_len": 64}, torch.device("cpu"))
    return make_train_state(config, model, carry, optim, 10, torch.device("cpu"))


def _full(t):
    return t.full_tensor() if hasattr(t, "full_tensor") else t


def _run(config, batches, steps=2):
    from mimir_b200.optim.schedules import update_lr
    from mimir_b200.train.steps import train_accumulated_batches
    st = _state(config)
    rank = dist.get_rank() if dist.is_initialized() else 0
    for i in range(steps):
        st.step += 1
        update_lr(config, st)
        train_accumulated_batches(config, rank, st, batches[i], bp_steps=3)
    from mimir_b200.parallel.fsdp import unwrap_model
    return {n: _full(p).detach().clone() for n, p in unwrap_model(st.model).named_parameters()}


# ------------------------------------------------------------------ GAS parity, DDP and FSDP2
def _gas_worker(rank, world, init, strategy, out):
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        batches = _batches(8)
        # rank r takes microbatches r, r+2, ... of each 4-microbatch global step
        mine = [[batches[4 * s + 2 * m + rank] for m in range(2)] for s in range(2)]
        cfg = _config(distributed_strategy=strategy, gradient_accumulation_steps=2)
        result = _run(cfg, mine)
        if rank == 0:
            torch.save(result, out)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("strategy", ["ddp", "fsdp"])
def test_distributed_gas_matches_single_process(tmp_path, strategy):
    batches = _batches(8)
    single = _run(_config(gradient_accumulation_steps=4), [batches[0:4], batches[4:8]])
    mp.spawn(_gas_worker, args=(2, f"file://{tmp_path / 'rdv'}", strategy, str(tmp_path / "out.pt")), nprocs=2,
             join=True)
    dist_result = torch.load(tmp_path / "out.pt")
    assert single.keys() == dist_result.keys()
    for n in single:
        torch.testing.assert_close(dist_result[n], single[n], rtol=2e-5, atol=2e-6, msg=n)


# ------------------------------------------------------------------ HSDP mesh (mocked world)
def test_hsdp_mesh_shape_and_validation():
    from mimir_b200.parallel.fsdp import create_fsdp_mesh
    cfg = _config(fsdp_shard_degree=4)
    with mock.patch("torch.distributed.is_available", return_value=True), \
            mock.patch("torch.distributed.is_initialized", return_value=True), \
            mock.patch("torch.distributed.get_world_size", return_value=16), \
            mock.patch.dict(os.environ, {"LOCAL_WORLD_SIZE": "8"}), \
            mock.patch("mimir_b200.parallel.fsdp.init_device_mesh") as init:
        create_fsdp_mesh(cfg)
        args, kwargs = init.call_args
        assert args[1] == (4, 4) and kwargs["mesh_dim_names"] == ("replicate", "shard")
    with mock.patch("torch.distributed.is_available", return_value=True), \
            mock.patch("torch.distributed.is_initialized", return_value=True), \
            mock.patch("torch.distributed.get_world_size", return_value=12), \
            mock.patch.dict(os.environ, {"LOCAL_WORLD_SIZE": "8"}):
        with pytest.raises(ValueError, match="divisible"):
            create_fsdp_mesh(_config(fsdp_shard_degree=8))
        with pytest.raises(ValueError, match="exceeds LOCAL_WORLD_SIZE"):
            create_fsdp_mesh(_config(fsdp_shard_degree=16))


# ------------------------------------------------------------------ gradient skip
def test_gradient_skip_leaves_weights_and_counts():
    from mimir_b200.train.steps import train_accumulated_batches
    cfg = _config(gradient_skip_norm=1e-9)
    st = _state(cfg)
    before = {n: p.detach().clone() for n, p in st.model.named_parameters()}
    st.step = 1
    metrics, skipped = train_accumulated_batches(cfg, 0, st, _batches(1), bp_steps=3)
    assert skipped and metrics["optimizer_step_skipped"][0].item() == 1
    for n, p in st.model.named_parameters():
        assert torch.equal(p, before[n]), n
        assert p.grad is None or not p.grad.abs().sum()
    cfg2 = _config(gradient_skip_norm=1e9, gradient_clip_norm=1e-3)
    st2 = _state(cfg2)
    st2.step = 1
    metrics, skipped = train_accumulated_batches(cfg2, 0, st2, _batches(1), bp_steps=3)
    assert not skipped and metrics["grad_clipped"][0].item() == 1.0
    assert metrics["grad_clip_coefficient"][0].item() < 1.0


# ------------------------------------------------------------------ module learning rates
def test_auto_module_learning_rates_follow_bptt_window():
    from mimir_b200.optim.module_lr import configured_module_rates, module_lr_metrics
    cfg = _config(lr_auto=True, arch=dict(H_cycles=2, L_cycles=3, bp_min_steps=4, bp_max_steps=4))
    rates = configured_module_rates(cfg, bp_steps=4)
    # H gets min(H_cycles, bp-1)=2 backward invocations, L the remaining 2
    assert rates["h"] == pytest.approx(cfg.lr / 2) and rates["l"] == pytest.approx(cfg.lr / 2)
    assert rates["embeddings"] == rates["head"] == cfg.lr
    st = _state(cfg)
    scales = st.optim.parameter_lr_scales
    emb = next(p for n, p in st.model.named_parameters() if "embed_tokens" in n)
    hw = next(p for n, p in st.model.named_parameters() if "H_level" in n)
    assert scales[emb] == 1.0 and scales[hw] == pytest.approx(0.5)
    metrics = module_lr_metrics(cfg, 1e-3, 4)
    assert metrics["train/lr_H"] == pytest.approx(5e-4) and metrics["train/lr_embedding_head"] == 1e-3


# ------------------------------------------------------------------ routing balance with an idle rank
def _balance_worker(rank, world, init, out):
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        from mimir_b200.models.experts import TopKRouter
        from mimir_b200.optim.routing_balance import routing_balance
        torch.manual_seed(0)
        router = TopKRouter(8, 4, 1, balance_enabled=True, balance_update_rate=0.1)
        router.train()
        with routing_balance(router) as step:
            if rank == 0:  # rank 1 routes no tokens at all but still joins the reduction
                x = torch.randn(16, 8)
                with torch.no_grad():
                    router.rows[2].copy_(torch.ones(8) * 5)
                router(x.abs())
            step.commit()
        torch.save(router.selection_bias.clone(), f"{out}.{rank}")
    finally:
        dist.destroy_process_group()


def test_routing_counts_include_idle_ranks(tmp_path):
    mp.spawn(_balance_worker, args=(2, f"file://{tmp_path / 'rdv'}", str(tmp_path / "b")), nprocs=2, join=True)
    b0, b1 = torch.load(f"{tmp_path / 'b'}.0"), torch.load(f"{tmp_path / 'b'}.1")
    assert torch.equal(b0, b1)
    assert b0[2].item() == pytest.approx(-0.1) and all(b0[i].item() == pytest.approx(0.1) for i in (0, 1, 3))


# ------------------------------------------------------------------ recurrence / checkpointing / compile
def test_activation_checkpointing_is_numerically_identical():
    from mimir_b200.train.steps import train_accumulated_batches
    results = []
    for ac in ("none", "full"):
        cfg = _config(activation_checkpointing=ac)
        st = _state(cfg)
        st.step = 1
        train_accumulated_batches(cfg, 0, st, _batches(1), bp_steps=3, zero_grad_after_step=False)
        results.append({n: p.detach().clone() for n, p in st.model.named_parameters()})
    for n in results[0]:
        torch.testing.assert_close(results[0][n], results[1][n], rtol=0, atol=0, msg=n)


def test_compiled_step_matches_eager():
    pytest.importorskip("torch._dynamo")
    from mimir_b200.train import steps
    cfg_e = _config()
    cfg_c = _config(compile_train_batch=True)
    eager = _run(cfg_e, [_batches(1), _batches(1, seed=1)])
    with mock.patch.object(steps, "compiled_forward_backward",
                           lambda mode: torch.compile(steps.forward_backward_batch, backend="aot_eager",
                                                      dynamic=False)):
        st = _state(cfg_c)
        from mimir_b200.optim.schedules import update_lr
        for i, b in enumerate([_batches(1), _batches(1, seed=1)]):
            st.step += 1
            update_lr(cfg_c, st)
            steps.train_accumulated_batches(cfg_c, 0, st, b, use_compiled=True, bp_steps=3)
    for n, p in st.model.named_parameters():
        torch.testing.assert_close(p.detach(), eager[n], rtol=1e-5, atol=1e-6, msg=n)


def test_upcycling_reads_a_ddp_checkpoint(tmp_path):
    """A dense run under DDP checkpoints its wrapped model (``module.`` keys, as the reference
    does); ``initialize_from`` with upcycling must read it into the unwrapped expert model."""
    import os
    import subprocess
    import sys

    from mimir_b200.ckpt.importer import _load_model_tensors
    from mimir_b200.data.synthetic import write_corpus
    corpus = write_corpus(str(tmp_path / "data"), rows=32, seq_len=64, vocab=256, min_prefix=1, max_prefix=1)
    base = ["size@arch=XXS", "arch.hidden_size=64", "arch.n_layers=2", "accelerator_type=cpu",
            "fwd_bwd_dtype=float32", "compile_train_batch=false", f"data.path={corpus}", "global_batch_size=256",
            "epochs=1"]
    env = os.environ | {"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0", "MASTER_ADDR": "127.0.0.1",
                        "MASTER_PORT": "29961"}
    subprocess.run([sys.executable, "-m", "mimir_b200", "train", *base, "distributed_strategy=ddp",
                    f"checkpoint_path={tmp_path / 'dense'}", "stop_after_step=2", "checkpoint_step_interval=2"],
                   env=env, check=True)
    keys = list(_load_model_tensors(tmp_path / "dense" / "step_2", "step_2"))
    assert keys and not any(k.startswith("module.") for k in keys) and "model.zL_init" in keys
    from mimir_b200.config.schema import load_config
    from mimir_b200.train.loop import launch
    launch(load_config(base + ["distributed_strategy=none", f"checkpoint_path={tmp_path / 'moe'}",
                               f"initialize_from={tmp_path / 'dense' / 'step_2'}", "arch.upcycle_from_dense=true",
                               "arch.moe_num_experts=4", "arch.moe_top_k=2", "arch.residual_branches=2",
                               "stop_after_step=1"]))
