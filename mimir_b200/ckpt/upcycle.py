"""Strict DCP/unsharded migrations: dense -> expert upcycling and v1 -> v2 gate migration.

Reference behaviour: ``src/mimir/model/v2_checkpoint.py:8-123``.

* Upcycling maps each destination key to its dense origin (``dense_source_key``); new v2
  tensors (routers, gates, residual branches, memories, n-gram) keep their initial values,
  every other key must exist with the same shape, and every source key must be used.  Expert
  copies are independent clones; optimizer slots (step, moments, EMA) follow their weights.
* A same-architecture source (identical key sets) is loaded as a plain resume.
* v1 -> v2 migration loads everything except the new gate tensors and refuses sources that
  already carry gate state (those use the normal strict loader).
"""
from __future__ import annotations

import copy

import torch.distributed.checkpoint as dcp
from torch.distributed.checkpoint.state_dict import get_optimizer_state_dict, set_state_dict

from mimir_b200.models.experts import dense_source_key, is_new_v2_key


def _stored_model_keys(checkpoint_id) -> set[str]:
    meta = dcp.FileSystemReader(str(checkpoint_id)).read_metadata()
    return {k.removeprefix("model.") for k in meta.state_dict_metadata if k.startswith("model.")}


def _key_map(target_keys, source_keys) -> dict[str, str]:
    """destination key -> source key; raises on a missing or unused source key."""
    same = set(target_keys) == set(source_keys)
    mapping = {}
    for name in target_keys:
        src = name if same else dense_source_key(name)
        if src in source_keys:
            mapping[name] = src
        elif not is_new_v2_key(name):
            raise ValueError(f"Missing upcycling source key: {src}")
    unused = set(source_keys) - set(mapping.values())
    if unused:
        raise ValueError(f"Unexpected upcycling source keys: {sorted(unused)}")
    return mapping


def expand_unsharded_state(target: dict, optim: dict, checkpoint: dict):
    """Expand a full CPU ``{'model', 'optim'}`` checkpoint into ``target``/``optim`` (full dicts).

    Optimizer slots may be keyed by name or, for old single-group checkpoints, by integer id
    in source-parameter order.
    """
    source, src_optim = checkpoint["model"], checkpoint["optim"]
    slots = src_optim["state"]
    if slots and all(isinstance(k, int) for k in slots):
        if len(src_optim["param_groups"]) != 1:
            raise ValueError("Numeric optimizer ids can only be mapped with a single parameter group")
        trained = {dense_source_key(n) for n in optim["state"]}
        ordered = [n for n in source if n in trained]
        ids = src_optim["param_groups"][0]["params"]
        if len(ids) != len(ordered):
            raise ValueError("Cannot map numeric optimizer ids to parameter names unambiguously")
        slots = dict(zip(ordered, (slots[i] for i in ids)))
    mapping = _key_map(list(target), set(source))
    for name, src in mapping.items():
        if source[src].shape != target[name].shape:
            raise ValueError(f"Upcycling shape mismatch for {name}: {tuple(source[src].shape)} vs "
                             f"{tuple(target[name].shape)}")
        target[name] = source[src].clone()
        if name in optim["state"]:
            if src not in slots or set(slots[src]) != set(optim["state"][name]):
                raise ValueError(f"Optimizer/EMA slot mismatch for {name}")
            optim["state"][name] = copy.deepcopy(slots[src])
    return target, optim


def _unwrap(model):
    from torch.nn.parallel import DistributedDataParallel
    return model.module if isinstance(model, DistributedDataParallel) else model


def load_upcycled_checkpoint(model, optimizer, checkpoint_id) -> None:
    """Load a dense DCP checkpoint into an expert model (sharded templates, independent clones)."""
    model = _unwrap(model)
    stored = _stored_model_keys(checkpoint_id)
    by_plain = {k.removeprefix("module."): k for k in stored}
    target = model.state_dict()
    mapping = _key_map(list(target), set(by_plain))
    request = {by_plain[src]: target[name].clone() for name, src in mapping.items()}
    optim = get_optimizer_state_dict(model, optimizer)
    stray = [n for n in optim["state"] if n not in mapping and not is_new_v2_key(n)]
    if stray:
        raise ValueError(f"Optimizer parameter names do not match the migration: {stray}")
    slots = {mapping[n]: copy.deepcopy(s) for n, s in optim["state"].items() if n in mapping}
    # Only slots are requested: the destination config owns param-group hyper-parameters.
    dcp.load({"model": request, "optim": {"state": slots}}, checkpoint_id=str(checkpoint_id))
    for name, src in mapping.items():
        target[name] = request[by_plain[src]].clone()
        if name in optim["state"]:
            optim["state"][name] = copy.deepcopy(slots[src])
    set_state_dict(model, optimizer, model_state_dict=target, optim_state_dict=optim)


def is_gate_key(name: str) -> bool:
    parts = name.split(".")
    return "invocation_gates" in parts or parts[-1] == "gate_alpha"


def load_v1_checkpoint(model, optimizer, checkpoint_id) -> bool:
    """Load a gate-free v1 DCP checkpoint into a gated v2 model; False if the source is v2."""
    stored = _stored_model_keys(checkpoint_id)
    if any(is_gate_key(k) for k in stored):
        return False
    full = model.state_dict()
    backbone = {k for k in full if not is_gate_key(k)}
    if stored != backbone:
        raise ValueError(f"v1 migration backbone mismatch: missing={sorted(backbone - stored)} "
                         f"unexpected={sorted(stored - backbone)}")
    if backbone == set(full):
        raise ValueError("v1 migration needs a v2 destination with gates")
    optim = get_optimizer_state_dict(model, optimizer)
    params = [list(g["params"]) for g in optim["param_groups"]]
    request_optim = {"state": {k: v for k, v in optim["state"].items() if not is_gate_key(k)},
                     "param_groups": [dict(g, params=[k for k in g["params"] if not is_gate_key(k)])
                                      for g in optim["param_groups"]]}
    request_model = {k: v for k, v in full.items() if not is_gate_key(k)}
    dcp.load({"model": request_model, "optim": request_optim}, checkpoint_id=str(checkpoint_id))
    full.update(request_model)
    optim["state"].update(request_optim["state"])
    optim["param_groups"] = [dict(g, params=p) for g, p in zip(request_optim["param_groups"], params)]
    set_state_dict(model, optimizer, model_state_dict=full, optim_state_dict=optim)
    return True


__all__ = ["expand_unsharded_state", "load_upcycled_checkpoint", "load_v1_checkpoint", "is_gate_key"]
