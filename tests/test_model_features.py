"""Behaviour of individual Mimir2 features on CPU: invocation gates, n-gram memory, windowed
cosine module learning rates.

* Gates with ``alpha = 0`` are the identity on their injection, so a gated model trains exactly
  like the ungated one until alpha ramps up (the gates add no RNG draws); a gate is token-local
  and scales its injection by a factor within ``1 +- alpha``.
* N-gram memory is causal, restarts at packed-sequence boundaries (positions restart at 0), and
  token-by-token decoding with its history cache equals the full forward.
* The windowed cosine starts at the base rate, ends at ``base * min_ratio``, is clamped outside
  the window and rejects malformed windows.
"""
import math

import numpy as np
import pytest
import torch

from mimir_b200.models.common import wrap_tensor
from mimir_b200.models.mimir2 import InvocationGate
from mimir_b200.models.ngram import NGramMemory
from mimir_b200.optim.module_lr import windowed_cosine_lr


def _cfg(**kw):
    return dict(max_seq_len=64, n_layers=2, hidden_size=32, num_heads=2, expansion=4, init_type="lecun_normal",
                norm_type="pre", norm_eps=1e-6, pos_emb_type="rope", rope_theta=10000.0, H_cycles=2, L_cycles=2,
                half_layers=False, fwd_bwd_dtype="float32", vocab_size=64) | kw


def _batch(T=24):
    from mimir_b200.data.prefixlm import compute_aux_seq_tensors_scalars
    g = torch.Generator().manual_seed(4)
    p, c = np.array([3, 6], np.int32), np.array([5, 7], np.int32)
    tensors, scalars = compute_aux_seq_tensors_scalars(p, c, T)
    pos = torch.cat([torch.arange(int(a + b)) for a, b in zip(p, c)]
                    + [torch.zeros(T - int((p + c).sum()), dtype=torch.long)])
    b = dict(inputs=torch.randint(0, 64, (T,), generator=g), labels=torch.randint(0, 64, (T,), generator=g),
             position_ids=pos) | {k: torch.from_numpy(v) for k, v in tensors.items()}
    return b | {k: wrap_tensor(torch.tensor(v)) for k, v in scalars.items()}


def test_zero_alpha_gates_train_like_the_ungated_model():
    from mimir_b200.models import LMHead, Mimir2
    runs = {}
    for gated in (False, True):
        c = _cfg(gates_enabled=gated)
        torch.manual_seed(0)
        model = LMHead(Mimir2(c), c)
        _, loss, _ = model(None, _batch(), bp_steps=3)
        loss.backward()
        runs[gated] = (loss.detach(), {n: p.grad for n, p in model.named_parameters()})
    assert torch.equal(runs[False][0], runs[True][0])
    plain, gated = runs[False][1], runs[True][1]
    for name, grad in plain.items():
        torch.testing.assert_close(gated[name], grad, atol=0, rtol=0, msg=name)
    for name, grad in gated.items():
        if "invocation_gates" in name:  # d/dW carries alpha = 0 (None outside the BPTT window)
            assert grad is None or not bool(grad.any()), name


def test_gate_is_token_local_and_bounded():
    torch.manual_seed(1)
    gate = InvocationGate(16)
    with torch.no_grad():
        gate.weight.normal_(0, 1.0)
        gate.bias.normal_(0, 1.0)
    hidden, injection = torch.randn(7, 16), torch.randn(7, 16)
    alpha = torch.tensor(0.7)
    out = gate(hidden, injection, alpha)
    ratio = out / injection
    assert bool((ratio >= 1 - 0.7 - 1e-6).all() and (ratio <= 1 + 0.7 + 1e-6).all())
    hidden2 = hidden.clone()
    hidden2[3] += 5.0
    out2 = gate(hidden2, injection, alpha)
    changed = (out2 != out).any(-1)
    assert changed.tolist() == [i == 3 for i in range(7)]
    torch.testing.assert_close(gate(hidden, injection, torch.tensor(0.0)), injection, atol=0, rtol=0)


def _ngram():
    torch.manual_seed(2)
    mem = NGramMemory(16, orders=(2, 3), buckets=97, heads=2)
    with torch.no_grad():
        for t in mem.tables:
            t.normal_()
        mem.alpha.fill_(0.5)
    return mem


def test_ngram_is_causal_and_restarts_at_sequence_boundaries():
    mem = _ngram()
    tokens = torch.randint(0, 50, (1, 12), generator=torch.Generator().manual_seed(3))
    positions = torch.cat([torch.arange(5), torch.arange(7)])[None]  # two packed sequences
    x = torch.zeros(1, 12, 16)
    base = mem(x, tokens, positions)
    for t in range(11):  # changing a later token leaves every earlier output alone
        later = tokens.clone()
        later[0, t + 1] = (later[0, t + 1] + 7) % 50
        torch.testing.assert_close(mem(x, later, positions)[:, :t + 1], base[:, :t + 1], atol=0, rtol=0)
    first = tokens.clone()
    first[0, :5] = (first[0, :5] + 11) % 50  # the first sequence is invisible to the second
    torch.testing.assert_close(mem(x, first, positions)[:, 5:], base[:, 5:], atol=0, rtol=0)


def test_ngram_decode_with_history_equals_full_forward():
    mem = _ngram()
    tokens = torch.randint(0, 50, (2, 9), generator=torch.Generator().manual_seed(5))
    positions = torch.arange(9).expand(2, 9)
    x = torch.randn(2, 9, 16)
    full = mem(x, tokens, positions)
    history = {}
    prompt = mem(x[:, :4], tokens[:, :4], positions[:, :4], history)
    steps = [mem(x[:, t:t + 1], tokens[:, t:t + 1], positions[:, t:t + 1], history) for t in range(4, 9)]
    torch.testing.assert_close(torch.cat([prompt] + steps, dim=1), full, atol=1e-6, rtol=1e-6)


def test_windowed_cosine_endpoints_clamping_and_validation():
    base, low = 3e-4, 0.1
    assert windowed_cosine_lr(base, low, 10, 10, 30) == pytest.approx(base)
    assert windowed_cosine_lr(base, low, 30, 10, 30) == pytest.approx(base * low)
    assert windowed_cosine_lr(base, low, 20, 10, 30) == pytest.approx(base * (low + (1 - low) / 2))
    assert windowed_cosine_lr(base, low, 15, 10, 30) == pytest.approx(
        base * (low + (1 - low) * (1 + math.cos(math.pi / 4)) / 2))
    assert windowed_cosine_lr(base, low, 0, 10, 30) == pytest.approx(base)
    assert windowed_cosine_lr(base, low, 99, 10, 30) == pytest.approx(base * low)
    for start, end, ratio in ((None, 5, low), (5, 5, low), (-1, 3, low), (0, 10, 1.5), (0, 10, -0.1)):
        with pytest.raises(ValueError):
            windowed_cosine_lr(base, ratio, 3, start, end)


def test_sequence_routes_read_only_what_their_policy_allows():
    """Sparse MoS routing pools each packed sequence: ``prefix_mean`` reads its prompt only,
    ``first_token`` its first token only; other sequences never leak in."""
    from mimir_b200.models.experts import TopKRouter
    from mimir_b200.models.mimir2 import Mimir2
    from mimir_b200.models.sparse_stacks import sequence_routes
    torch.manual_seed(6)
    router = TopKRouter(8, 3, 2, init_std=0.5)
    info = dict(numseqs=torch.tensor(2), cu_seqlens=torch.tensor([0, 6, 11]), prefix_lens=torch.tensor([2, 4]))
    x = torch.randn(11, 8)
    for policy, visible in (("prefix_mean", [0, 1, 6, 7, 8, 9]), ("first_token", [0, 6])):
        base = sequence_routes(router, x, info, policy=policy)
        for row in range(11):
            moved = x.clone()
            moved[row] += 3.0
            same = torch.equal(sequence_routes(router, moved, info, policy=policy), base)
            assert same is (row not in visible), (policy, row)
    with pytest.raises(ValueError, match="PrefixLM"):
        Mimir2(_cfg(mos_num_experts=2, mos_top_k=1, mos_sparse=True, mos_sparse_routing="prefix_mean",
                    attn_type="causal"))


def test_metadata_routing_bias_schedule_and_training_only():
    """Category rows of the routing-logit bias decay linearly to zero over the configured step
    window and apply in training forwards only; warm-up ramps move alpha linearly from 0 to max."""
    from types import SimpleNamespace

    from mimir_b200.models.mimir2 import Mimir2
    model = Mimir2(_cfg(moe_num_experts=2, moe_top_k=1, moe_metadata_bias=[[0.0, 4.0], [2.0, 0.0]],
                        routing_bias_decay_start=10, routing_bias_decay_end=30, gates_enabled=True,
                        gate_warmup_start_step=5, gate_warmup_steps=10, gate_alpha_max=0.8))
    model.train()
    category = torch.tensor([1, 0, 1])
    for step, scale, alpha in ((0, 1.0, 0.0), (10, 1.0, 0.4), (20, 0.5, 0.8), (30, 0.0, 0.8), (99, 0.0, 0.8)):
        model.compute_train_extra_args(SimpleNamespace(step=step))
        expected = torch.tensor([[2.0, 0.0], [0.0, 4.0], [2.0, 0.0]]) * scale
        torch.testing.assert_close(model._metadata_bias(category, "moe"), expected)
        assert float(model.gate_alpha) == pytest.approx(alpha), step
    model.eval()
    assert model._metadata_bias(category, "moe") is None


@pytest.mark.parametrize("changes,message", [
    (dict(moe_aux_loss_free=True), "MoE balancing requires multiple MoE experts"),
    (dict(H_override={"n_layers": 0}), "Zero-layer H requires looped recurrence"),
    (dict(h_residual_persistence=True), "H stream options require hierarchical recurrence"),
    (dict(h_branch_l_mixing=True, residual_branches=2, residual_levels="H"), "Branch-specific L mixing requires MoS"),
    (dict(recurrence_mode="looped", gates_enabled=True), "Looped recurrence requires shared MoS state"),
    (dict(moe_num_experts=2, moe_metadata_bias=[[0.0]]), "Metadata bias rows must contain one finite logit"),
    (dict(routing_bias_decay_start=5, routing_bias_decay_end=5), "Routing bias decay end must follow start"),
    (dict(moe_num_experts=2, specialist_training=True), "Specialist training requires a frozen reference expert"),
    (dict(moe_num_experts=2, moe_dispatch="grouped"), "need moe_sparse with several experts"),
    (dict(moe_num_experts=2, moe_top_k=3), "Expert top_k must not exceed num_experts"),
    (dict(residual_branches=2, norm_type="post"), "Multiple residual branches currently require pre-norm"),
    (dict(expert_freeze_base=True), "expert_freeze_base requires an expert mixture"),
    (dict(gate_initialize_from_v1=True), "gate_initialize_from_v1 requires gates_enabled=true"),
])
def test_invalid_feature_combinations_are_rejected(changes, message):
    from mimir_b200.models.mimir2 import Mimir2
    with pytest.raises(ValueError, match=message):
        Mimir2(_cfg(**changes))


def test_frozen_base_expert_takes_no_gradient():
    """A frozen reference expert (``expert_freeze_base``) and its router row receive no parameter
    gradient while the other experts and the backbone train."""
    from mimir_b200.models import LMHead, Mimir2
    c = _cfg(moe_num_experts=3, moe_top_k=2, expert_freeze_base=True)
    torch.manual_seed(0)
    model = LMHead(Mimir2(c), c)
    _, loss, _ = model(None, _batch(), bp_steps=3)
    loss.backward()
    grads = {n: p.grad for n, p in model.named_parameters()}
    frozen = [n for n, p in model.named_parameters() if not p.requires_grad]
    assert frozen and all(grads[n] is None for n in frozen)
    assert any(".experts.0." in n for n in frozen) and any("rows.0" in n for n in frozen)
    trained = [n for n in grads if n not in frozen and grads[n] is not None]
    assert any(".experts.1." in n for n in trained)
    assert any("embed" in n for n in trained)


def test_residual_branches_add_no_sublayer_calls():
    """Residual branches mix the streams around each sublayer; the attention and MLP sublayers run
    as often as in the single-stream model."""
    from mimir_b200.models import LMHead, Mimir2
    from mimir_b200.models.transformer import Attention
    from mimir_b200.models.layers import SwiGLU

    def calls(**kw):
        c = _cfg(**kw)
        torch.manual_seed(0)
        model = LMHead(Mimir2(c), c)
        seen = {"attn": 0, "mlp": 0}
        for m in model.modules():
            if isinstance(m, (Attention, SwiGLU)):
                key = "attn" if isinstance(m, Attention) else "mlp"
                m.register_forward_hook(lambda *_, key=key: seen.__setitem__(key, seen[key] + 1))
        model(None, _batch(), bp_steps=3)
        return seen

    single = calls()
    assert single["attn"] > 0 and single["mlp"] > 0
    assert calls(residual_branches=2) == single
    assert calls(residual_branches=3, residual_levels="H") == single


@pytest.mark.parametrize("levels,branched", [("both", {"L", "H"}), ("H", {"H"}), ("L", {"L"})])
def test_residual_branch_levels_and_alpha_ramp(levels, branched):
    """``residual_levels`` picks which stacks get branched residual streams, and their mixing
    alpha ramps linearly from 0 to ``residual_alpha_max`` over the warm-up window."""
    from types import SimpleNamespace

    from mimir_b200.models.branches import BranchedTransformer
    from mimir_b200.models.mimir2 import Mimir2
    model = Mimir2(_cfg(residual_branches=2, residual_levels=levels, residual_alpha_max=0.6,
                        residual_warmup_start_step=4, residual_warmup_steps=8))
    found = {name for name in ("L", "H") if isinstance(getattr(model, f"{name}_level").core, BranchedTransformer)}
    assert found == branched
    for step, alpha in ((0, 0.0), (4, 0.0), (8, 0.3), (12, 0.6), (50, 0.6)):
        model.compute_train_extra_args(SimpleNamespace(step=step))
        values = [float(m.residual_alpha) for m in model.modules() if isinstance(m, BranchedTransformer)]
        assert values and all(v == pytest.approx(alpha) for v in values), (step, values)


def test_model_yaml_defaults_equal_the_schema_defaults():
    """Every feature key of ``conf/model/mimir2.yaml`` carries the schema's default value, so a run
    without overrides is the plain backbone whichever way it is configured."""
    from pathlib import Path

    import yaml

    import mimir_b200
    from mimir_b200.models.mimir2 import Mimir2Config
    conf = yaml.safe_load((Path(mimir_b200.__file__).parent / "conf" / "model" / "mimir2.yaml").read_text())
    fields = Mimir2Config.model_fields
    checked = 0
    for key, value in conf.items():
        if key in fields and not fields[key].is_required():
            default = fields[key].get_default(call_default_factory=True)
            if key in ("H_cycles", "L_cycles", "half_layers", "bp_min_steps", "bp_max_steps", "bp_warmup_ratio",
                       "recurrence_mode", "H_override"):
                continue  # architecture of the preset, not an opt-in feature
            assert value == default, (key, value, default)
            checked += 1
    assert checked > 20
