"""``mimir_b200 export``: published checkpoint -> verified HF Mimir2 directory.

Reference behaviour: ``src/mimir/export/convert.py:11-66``.

1. ``validate`` the checkpoint (full hashes); never overwrite ``output``.
2. Only hierarchical Mimir2 without persistent-H streams or branch-specific L mixing
   (the inference integrations do not implement them).
3. Weights come from the DCP ``model.*`` tensors or, with ``ema`` (default), from the
   ``optim.state.<name>.param_ema`` slots; a ``.weight`` without an EMA slot is an error.
4. The tokenizer directory must carry an explicit chat template; its special-token ids go
   into the model and generation configs and its size must fit the model vocabulary.
5. Everything is written to a sibling ``.partial`` directory, reloaded, the reloaded logits
   must equal the in-memory logits exactly and the chat template must survive serialization;
   then ``export_receipt.json`` is written and the directory is renamed into place.
"""
from __future__ import annotations

import json
import shutil
import uuid
from pathlib import Path

import torch
import yaml

from mimir_b200.ckpt.contract import validate
from mimir_b200.export.hf import Mimir2ForCausalLM

_PROBE = [{"role": "user", "content": "Test"}]


def read_weights(checkpoint: Path, tag: str, checkpoint_format: str, ema: bool) -> dict:
    if checkpoint_format == "sharded":
        import torch.distributed.checkpoint as dcp
        reader = dcp.FileSystemReader(str(checkpoint / f"fsdp2_{tag}"))
        entries = reader.read_metadata().state_dict_metadata
        sources = {}
        for key in entries:
            if not key.startswith("model."):
                continue
            name = key.removeprefix("model.")
            slot = f"optim.state.{name}.param_ema"
            if ema and name.endswith(".weight") and slot not in entries:
                raise ValueError(f"Missing EMA: {name}")
            sources[name] = slot if ema and slot in entries else key
        tensors = {k: torch.empty(entries[k].size, dtype=entries[k].properties.dtype) for k in sources.values()}
        dcp.load(tensors, storage_reader=reader, no_dist=True)
        return {name: tensors[k] for name, k in sources.items()}
    data = torch.load(checkpoint / f"unsharded_{tag}.pt", map_location="cpu", weights_only=False)
    state = dict(data["model"])
    if ema:
        slots = data.get("optim", {}).get("state", {})
        if any(not isinstance(k, str) for k in slots):
            raise ValueError("EMA export requires named optimizer state")
        for name in state:
            slot = slots.get(name, {})
            if "param_ema" in slot:
                state[name] = slot["param_ema"]
            elif name.endswith(".weight"):
                raise ValueError(f"Missing EMA: {name}")
    return state


def export(checkpoint, output, tokenizer, *, ema: bool = True) -> Path:
    from transformers import AutoTokenizer
    checkpoint, output = Path(checkpoint), Path(output)
    manifest = validate(checkpoint)
    if output.exists():
        raise FileExistsError(output)
    cfg = yaml.safe_load((checkpoint / "all_config.yaml").read_text())
    meta = yaml.safe_load((checkpoint / "train_metadata.yaml").read_text())
    arch = cfg["arch"]
    if arch["name"] != "mimir2":
        raise ValueError("Only Mimir2 exports are supported")
    if arch.get("recurrence_mode", "hierarchical") != "hierarchical":
        raise ValueError("Looped recurrence export is not supported by the inference integrations")
    if arch.get("h_residual_persistence") or arch.get("h_branch_l_mixing"):
        raise ValueError("Persistent H streams and branch-specific L mixing require inference support")
    state = read_weights(checkpoint, manifest["tag"], cfg["checkpoint_format"], ema)
    # The exported model runs in fp32 regardless of the training compute dtype.
    state = {k: v.float() if v.is_floating_point() else v for k, v in state.items()}
    native = arch | {k: meta[k] for k in ("vocab_size", "max_seq_len")}
    model = Mimir2ForCausalLM.from_native(native, state)
    tok = AutoTokenizer.from_pretrained(str(tokenizer), local_files_only=True)
    if not tok.chat_template:
        raise ValueError("Tokenizer must own an explicit chat template")
    ids = {k: getattr(tok, k) for k in ("bos_token_id", "eos_token_id", "pad_token_id")}
    model.config.update(ids)
    model.generation_config = dict(ids)
    if len(tok) > model.config["vocab_size"]:
        raise ValueError("Tokenizer exceeds model vocabulary")
    template = tok.apply_chat_template(_PROBE, tokenize=True, add_generation_prompt=True)
    stage = output.with_name(f".{output.name}.{uuid.uuid4().hex}.partial")
    stage.mkdir(parents=True)
    try:
        model.save_pretrained(stage)
        tok.save_pretrained(str(stage))
        again = AutoTokenizer.from_pretrained(str(stage), local_files_only=True)
        if again.apply_chat_template(_PROBE, tokenize=True, add_generation_prompt=True) != template:
            raise ValueError("Chat template changed during serialization")
        restored = Mimir2ForCausalLM.from_pretrained(stage)
        probe = torch.tensor([[1, 2, 3]])
        torch.testing.assert_close(model(probe), restored(probe), rtol=0, atol=0)
        (stage / "export_receipt.json").write_text(json.dumps({"schema": 1, "architecture": "mimir2",
                                                               "checkpoint_manifest": manifest, "ema": ema},
                                                              indent=2))
        stage.rename(output)
    except BaseException:
        shutil.rmtree(stage, ignore_errors=True)
        raise
    return output
