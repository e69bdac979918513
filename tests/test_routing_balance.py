"""Aux-loss-free routing balance (``mimir_b200.optim.routing_balance`` and ``TopKRouter``), CPU.

The selection bias only changes which experts are chosen, never the mixing weights; a step's
ledger counts each real routing decision once (not eval forwards, not activation-checkpoint
replays, nothing outside an open step); the commit moves each bias by ``rate * sign(mean - load)``;
the bias stays fp32 when the model changes precision.
"""
import torch
import torch.utils.checkpoint as cp

from mimir_b200.models.experts import TopKRouter
from mimir_b200.optim.routing_balance import routing_balance


def _router(n=4, k=2, rate=0.25):
    torch.manual_seed(0)
    r = TopKRouter(8, n, k, balance_enabled=True, balance_update_rate=rate, init_std=0.5)
    r.train()
    return r


def test_bias_changes_selection_but_not_weights():
    r = _router()
    x = torch.randn(6, 8)
    weights, chosen = r(x, return_indices=True)
    r.selection_bias[3] = 100.0  # expert 3 now always wins a slot
    weights_b, chosen_b = r(x, return_indices=True)
    assert bool((chosen_b == 3).any(-1).all())
    affinity = r.scores(x).sigmoid()
    mask = torch.zeros_like(affinity, dtype=torch.bool).scatter(-1, chosen_b, True)
    expected = affinity * mask
    expected = expected / expected.sum(-1, keepdim=True)
    torch.testing.assert_close(weights_b, expected)  # the bias is absent from the weights
    assert torch.allclose(weights.sum(-1), torch.ones(6))


def test_commit_moves_bias_by_sign_of_mean_minus_load():
    r = _router(rate=0.25)
    with routing_balance(r) as ledger:
        ledger.counts(r).copy_(torch.tensor([5, 1, 0, 2]))
        ledger.commit()
    torch.testing.assert_close(r.selection_bias, torch.tensor([-0.25, 0.25, 0.25, 0.0]))


def test_only_real_training_forwards_are_counted():
    r = _router()
    x = torch.randn(5, 8)
    r(x)  # no open step: nothing to record into
    with routing_balance(r) as ledger:
        r.eval()
        r(x)
        assert int(ledger.counts(r).sum()) == 0  # eval forwards do not count
        r.train()
        r(x)
        assert int(ledger.counts(r).sum()) == 5 * r.k  # one forward: k selections per token
        ledger.counts(r).zero_()
        y = cp.checkpoint(lambda t: r(t), x.requires_grad_(), use_reentrant=False)
        y.sum().backward()  # the backward replays the forward: not a new routing decision
        assert int(ledger.counts(r).sum()) == 5 * r.k


def test_bias_stays_fp32_under_precision_changes():
    r = _router()
    r.selection_bias.fill_(0.125)
    r.to(torch.bfloat16)
    assert r.selection_bias.dtype == torch.float32
    assert r.rows[0].dtype == torch.bfloat16
    assert torch.equal(r.selection_bias, torch.full((4,), 0.125))


def test_top1_router_gradient_comes_only_from_the_straight_through_surrogate():
    """With one expert per token the mixing weight is exactly 1: the router learns only through
    the straight-through surrogate (on by default) and gets a zero gradient without it."""
    x = torch.randn(9, 8)
    for straight_through in (True, False):
        torch.manual_seed(0)
        r = TopKRouter(8, 4, 1, top1_straight_through=straight_through, init_std=0.5)
        w = r(x)
        assert torch.equal(w.detach().sum(-1), torch.ones(9))
        (w * torch.randn(9, 4, generator=torch.Generator().manual_seed(1))).sum().backward()
        moved = any(bool(p.grad.any()) for p in r.rows if p.grad is not None)
        assert moved is straight_through


def test_selection_bias_is_checkpointed():
    r = _router()
    r.selection_bias.copy_(torch.tensor([0.5, -0.25, 0.0, 1.0]))
    state = r.state_dict()
    assert torch.equal(state["selection_bias"], r.selection_bias)
    fresh = _router()
    fresh.load_state_dict(state)
    assert torch.equal(fresh.selection_bias, r.selection_bias)
