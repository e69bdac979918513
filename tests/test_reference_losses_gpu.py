"""Per-step training losses of this framework against the unmodified reference, on one GPU.

Both frameworks build the same small Mimir2 (KV heads = query heads, the only layout the
reference expresses: ``src/mimir/model/transformer.py:78``) from the same seed on the CPU, so
the initial weights are equal bit for bit, then train 10 steps on the same prefix-LM batches
through their own public step (``train_accumulated_batches``) and AdamATan2 + EMA:

* ours: the replicated engine (bf16 weights, fp32 master and moments, the fused update kernel),
  tcgen05 attention / GEMM / fused cross-entropy kernels;
* the reference: fp32 weights under CUDA autocast (``src/mimir/training/steps.py:15-24``) and its
  dense prefix-LM attention backend (FlashAttention-4 is not installable offline).

The step-0 losses differ only by bf16 rounding of the forward; later steps add bf16 weight
rounding on our side.  Tolerance: 2 % relative per step, and both runs must learn the two
alternated batches (loss falls by more than 1 nat).
"""
import os
import sys

import numpy as np
import pytest
import torch

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "mimir")), reason="reference not installed")]

SEQ, SEQS, VOCAB, STEPS = 256, 4, 512, 10
MODEL = dict(max_seq_len=SEQ, n_layers=2, hidden_size=256, num_heads=2, expansion=4, init_type="lecun_normal",
             norm_type="pre", norm_eps=1e-6, pos_emb_type="rope", rope_theta=10000.0, recurrence_mode="looped",
             half_layers=False, H_override={"n_layers": 0}, H_cycles=1, L_cycles=1, bp_min_steps=2, bp_max_steps=2,
             bp_warmup_ratio=0.0, fwd_bwd_dtype="bfloat16", vocab_size=VOCAB)
OPTIM = dict(epochs=1, lr=2e-3, lr_warmup_steps=0, lr_min_ratio=1.0, weight_decay=0.1, beta1=0.9, beta2=0.95,
             ema=0.999, lr_auto=False)


def _batches():
    from mimir_b200.data.prefixlm import compute_aux_seq_tensors_scalars
    out = []
    for i in range(2):
        rng = np.random.default_rng(17 + i)
        prefix = rng.integers(1, SEQ // 2, size=SEQS).astype(np.int32)
        tensors, scalars = compute_aux_seq_tensors_scalars(prefix, (SEQ - prefix).astype(np.int32), SEQ * SEQS)
        inputs = rng.integers(0, VOCAB, size=SEQ * SEQS)
        labels = rng.integers(0, VOCAB, size=SEQ * SEQS)
        for s in range(SEQS):
            labels[s * SEQ: s * SEQ + prefix[s] - 1] = -100
        tensors = {k: torch.from_numpy(v) for k, v in tensors.items()}
        tensors |= dict(inputs=torch.from_numpy(inputs), labels=torch.from_numpy(labels),
                        position_ids=torch.arange(SEQ).repeat(SEQS))
        out.append((tensors, scalars))
    return out


def _on(device, batch, wrap):
    tensors, scalars = batch
    return {k: v.to(device) for k, v in tensors.items()} | {k: wrap(torch.tensor(v)) for k, v in scalars.items()}


def _reference_losses(device, batches):
    if REF not in sys.path:
        sys.path.append(REF)
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from bench import _stub_missing_reference_deps
    _stub_missing_reference_deps()
    from mimir.model import Mimir2
    from mimir.model.accelerator import set_accelerator_type
    from mimir.model.adam_atan2 import AdamATan2
    from mimir.model.common import wrap_tensor
    from mimir.model.lm_head import LMHead
    from mimir.training.config import PretrainConfig
    from mimir.training.schedules import update_lr
    from mimir.training.state import TrainState
    from mimir.training.steps import train_accumulated_batches

    set_accelerator_type("none")
    arch = {k: v for k, v in MODEL.items() if k not in ("vocab_size", "max_seq_len", "fwd_bwd_dtype")}
    config = PretrainConfig(arch=arch, data=dict(path="synthetic"), global_batch_size=SEQ * SEQS,
                            distributed_strategy="none", compile_train_batch=False, **OPTIM)
    torch.manual_seed(0)
    model = LMHead(Mimir2(MODEL), MODEL).to(device)
    optim = AdamATan2(model.parameters(), lr=0.0, betas=(0.9, 0.95), weight_decay=0.1, ema=0.999)
    state = TrainState(model=model, carry=None, optim=optim, step=0, total_steps=10_000,
                       fwd_bwd_dtype=torch.bfloat16, use_cuda_autocast=True)
    losses = []
    for i in range(STEPS):
        state.step += 1
        update_lr(config, state)
        metrics, _ = train_accumulated_batches(config, 0, state, [_on(device, batches[i % 2], wrap_tensor)], False,
                                               bp_steps=2)
        losses.append(float(metrics["loss"][0] / metrics["loss"][1]))
    return losses


def _our_losses(device, batches):
    from mimir_b200.config.schema import PretrainConfig
    from mimir_b200.models import LMHead, Mimir2
    from mimir_b200.models.common import wrap_tensor
    from mimir_b200.ops._ext import check_kernel_status
    from mimir_b200.optim.schedules import update_lr
    from mimir_b200.parallel.replicated import ReplicatedAdamATan2, wrap_replicated
    from mimir_b200.train.setup import make_train_state
    from mimir_b200.train.steps import train_accumulated_batches

    arch = {k: v for k, v in MODEL.items() if k not in ("vocab_size", "max_seq_len", "fwd_bwd_dtype")}
    config = PretrainConfig(arch=arch, data=dict(path="synthetic"), global_batch_size=SEQ * SEQS,
                            distributed_strategy="replicated", **OPTIM)
    torch.manual_seed(0)
    model = LMHead(Mimir2(MODEL), MODEL).to(device)
    engine = wrap_replicated(model, device, torch.bfloat16)
    optim = ReplicatedAdamATan2(engine, lr=0.0, betas=(0.9, 0.95), weight_decay=0.1, ema=0.999,
                                ema_dtype=torch.float32)
    state = make_train_state(config, model, None, optim, total_steps=10_000, device=device)
    losses = []
    for i in range(STEPS):
        state.step += 1
        update_lr(config, state)
        metrics, _ = train_accumulated_batches(config, 0, state, [_on(device, batches[i % 2], wrap_tensor)])
        losses.append(float(metrics["loss"][0] / metrics["loss"][1]))
    check_kernel_status(device)
    engine.close()
    return losses


def test_per_step_losses_match_the_reference():
    device = torch.device("cuda", 0)
    batches = _batches()
    ref = _reference_losses(device, batches)
    ours = _our_losses(device, batches)
    rel = [abs(a - b) / b for a, b in zip(ours, ref)]
    print("reference", [round(x, 4) for x in ref], "\nours     ", [round(x, 4) for x in ours])
    assert max(rel) < 0.02, (ref, ours)
    assert ref[0] - ref[-1] > 1.0 and ours[0] - ours[-1] > 1.0, (ref, ours)
