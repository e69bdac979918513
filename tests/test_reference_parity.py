"""Bit-level parity of Mimir2 (all opt-in features) with the reference implementation on CPU.

The reference package is imported from ``baseline/_ref`` (installed offline, git-ignored); the
test is skipped when it is absent.  Same seed => identical initial weights (RNG consumption
order), identical loss, and gradients equal to fp32 round-off.
"""
import os
import sys

import numpy as np
import pytest
import torch

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "mimir")), reason="reference not installed")


def _ref():
    if REF not in sys.path:
        sys.path.append(REF)
    from mimir.model import Mimir2 as RM
    from mimir.model.accelerator import set_accelerator_type
    from mimir.model.common import wrap_tensor as rwrap
    from mimir.model.lm_head import LMHead as RH
    set_accelerator_type("cpu")
    return RM, RH, rwrap


def _cfg(**kw):
    base = dict(max_seq_len=64, n_layers=2, hidden_size=32, num_heads=2, expansion=4, init_type="lecun_normal",
                norm_type="pre", norm_eps=1e-6, pos_emb_type="rope", rope_theta=10000.0, H_cycles=2, L_cycles=2,
                half_layers=False, fwd_bwd_dtype="float32", vocab_size=64)
    base.update(kw)
    return base


def _batch(T=24):
    from mimir_b200.data.prefixlm import compute_aux_seq_tensors_scalars
    g = torch.Generator().manual_seed(0)
    p, c = np.array([3, 5, 2], np.int32), np.array([4, 6, 3], np.int32)
    tensors, scalars = compute_aux_seq_tensors_scalars(p, c, T)
    inputs = torch.randint(0, 64, (T,), generator=g)
    labels = torch.randint(0, 64, (T,), generator=g)
    labels[:2] = -100
    pos = torch.cat([torch.arange(int(a + b)) for a, b in zip(p, c)] + [torch.zeros(T - int((p + c).sum()), dtype=torch.long)])
    return dict(inputs=inputs, labels=labels, position_ids=pos) | {k: torch.from_numpy(v) for k, v in tensors.items()}, scalars


VARIANTS = [
    dict(),
    dict(recurrence_mode="looped", H_override=dict(n_layers=0), H_cycles=1, L_cycles=1),
    dict(recurrence_mode="looped", H_override=dict(n_layers=1), H_cycles=2, L_cycles=2),
    dict(gates_enabled=True),
    dict(moe_num_experts=4, moe_top_k=2),
    dict(moe_num_experts=3, moe_top_k=1, moe_sparse=True),
    dict(moe_num_experts=2, moe_top_k=1, moe_aux_loss_free=True),
    dict(mos_num_experts=2, mos_top_k=1),
    dict(mos_num_experts=2, mos_top_k=2, mos_sparse=True),
    dict(mos_num_experts=2, mos_state_mode="separate", gates_enabled=True),
    dict(residual_branches=2),
    dict(residual_branches=2, residual_levels="H", h_residual_persistence=True, h_branch_l_mixing=True,
         mos_num_experts=2, mos_top_k=2),
    dict(ngram_orders=[2, 3], ngram_buckets=97, ngram_heads=2, ngram_contextual_gate=True),
    dict(h_memory_branches=2, l_memory_branches=3),
    dict(goldfish_strategy="hash", goldfish_k=3),
    dict(norm_type="post", init_type="megatron"),
]


@pytest.mark.parametrize("variant", VARIANTS, ids=[str(i) for i in range(len(VARIANTS))])
def test_model_parity(variant):
    from mimir_b200.models import LMHead, Mimir2
    from mimir_b200.models.common import wrap_tensor
    RM, RH, rwrap = _ref()
    c = _cfg(**variant)
    torch.manual_seed(0)
    ref = RH(RM(c), c)
    torch.manual_seed(0)
    ours = LMHead(Mimir2(c), c)
    rs, ms = ref.state_dict(), ours.state_dict()
    assert list(rs) == list(ms)
    for k in rs:
        assert torch.equal(rs[k], ms[k]), k
    b, s = _batch()
    _, rl, rm = ref(None, b | {k: rwrap(torch.tensor(v)) for k, v in s.items()}, bp_steps=3)
    _, ml, mm = ours(None, b | {k: wrap_tensor(torch.tensor(v)) for k, v in s.items()}, bp_steps=3)
    assert torch.equal(rl, ml)
    rl.backward()
    ml.backward()
    for (n, p), (_, q) in zip(ref.named_parameters(), ours.named_parameters()):
        if p.grad is None:
            assert q.grad is None, n
        else:
            torch.testing.assert_close(q.grad, p.grad, atol=1e-6, rtol=1e-5, msg=n)
    for k in rm:
        assert torch.equal(rm[k][0], mm[k][0]) and torch.equal(rm[k][1], mm[k][1]), k


def test_optimizer_parity():
    if REF not in sys.path:
        sys.path.append(REF)
    from mimir.model.adam_atan2 import AdamATan2 as RefAdam
    from mimir.model.muon import MuonAdamW as RefMuon
    from mimir_b200.optim.adam_atan2 import AdamATan2
    from mimir_b200.optim.muon import MuonAdamW
    torch.manual_seed(0)
    shapes = {"layers.0.attn.gqkv_proj.weight": (16, 8), "layers.0.mlp.gate_up_proj.weight": (8, 8),
              "layers.0.mlp.down_proj.weight": (8, 4), "embed": (5, 8)}
    for ours_cls, ref_cls, kw in ((AdamATan2, RefAdam, {}), (MuonAdamW, RefMuon, dict(momentum=0.9))):
        a = {n: torch.randn(s, requires_grad=True) for n, s in shapes.items()}
        b = {n: t.detach().clone().requires_grad_(True) for n, t in a.items()}
        args_a = list(a.items()) if ours_cls is MuonAdamW else list(a.values())
        args_b = list(b.items()) if ours_cls is MuonAdamW else list(b.values())
        oa = ours_cls(args_a, lr=1e-2, ema=0.99, **kw)
        ob = ref_cls(args_b, lr=1e-2, ema=0.99, **kw)
        for _ in range(3):
            for n in a:
                g = torch.randn(shapes[n])
                a[n].grad, b[n].grad = g.clone(), g.clone()
            oa.step()
            ob.step()
        for n in a:
            assert torch.equal(a[n], b[n]), (ours_cls.__name__, n)
