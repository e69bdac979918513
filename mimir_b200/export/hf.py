"""Hugging Face file format for Mimir2: config, weight names and a loadable inference model.

The on-disk layout matches the Mimir2 Transformers integration the reference targets
(``patches/transformers.patch:545-625``): ``config.json`` with ``model_type = "mimir2"`` and
its fields, and ``model.safetensors`` in HF names:

* the packed ``attn.gqkv_proj`` splits into ``self_attn.{gate,q,k,v}_proj`` (in that order;
  with GQA the K/V pieces hold ``num_key_value_heads`` heads), ``mlp[.experts.N].gate_up_proj``
  into ``gate_proj``/``up_proj``, ``attn.o_proj`` becomes ``self_attn.o_proj``;
* ``model.{L,H}_level[.core].`` becomes ``model.{L,H}_module.``, ``model.zL_init`` becomes
  ``model.z_L_init``, ``embed_tokens.embedding_weight`` becomes ``model.embed_tokens.weight``;
* non-persistent rotary tables and the training-only ``model.routing_bias_scale`` are dropped.

``Mimir2ForCausalLM`` reads and writes that format and runs the native model for inference
(``forward(input_ids) -> logits``), so an export can be verified bit-exactly here without the
patched Transformers; any loader that understands the format (the patched Transformers or the
vLLM fork) reads the same files.
"""
from __future__ import annotations

import json
import math
import re
from pathlib import Path
from typing import Optional

import numpy as np
import torch
from torch import nn

FEATURE_FIELDS = (
    "gates_enabled", "moe_num_experts", "moe_top_k", "moe_levels", "moe_sparse", "mos_num_experts", "mos_top_k",
    "mos_state_mode", "mos_sparse", "mos_sparse_routing", "residual_branches", "residual_levels",
    "residual_input_dependent", "residual_write_init_scale", "h_memory_branches", "l_memory_branches",
    "ngram_orders", "ngram_buckets", "ngram_heads", "ngram_contextual_gate", "router_top1_straight_through",
    "moe_aux_loss_free", "mos_aux_loss_free", "routing_bias_update_rate", "expert_freeze_base",
)
NATIVE_CONFIG_KEY = "mimir_native_config"


def _init_std(native: dict) -> float:
    size, kind = native["hidden_size"], native.get("init_type", "lecun_normal")
    if kind == "lecun_normal":
        return 1 / math.sqrt(size)
    if kind == "fixed_normal":
        return native.get("init_std") or 0.02
    if kind == "megatron":
        return native.get("init_std") or 1 / math.sqrt(size)
    raise ValueError(f"Unsupported initialization: {kind}")


def hf_config(native: dict) -> dict:
    """HF ``config.json`` for a native architecture dict (plus ``vocab_size``/``max_seq_len``)."""
    if native.get("norm_type", "pre") != "pre" or native.get("pos_emb_type", "rope") != "rope":
        raise ValueError("Mimir2 export supports pre-norm RoPE checkpoints only")
    if native.get("H_override"):
        raise ValueError("Asymmetric H_override requires a dedicated conversion")
    if native.get("attn_type", "prefixlm") not in ("prefixlm", "causal"):
        raise ValueError("Unsupported attention type")
    size, heads = native["hidden_size"], native["num_heads"]
    layers = native["n_layers"]
    if native.get("half_layers", False):
        if layers % 2:
            raise ValueError("half_layers requires an even n_layers")
        layers //= 2
    std = _init_std(native)
    mos = native.get("mos_num_experts", 1)
    cfg = {
        "model_type": "mimir2", "architectures": ["Mimir2ForCausalLM"], "vocab_size": native["vocab_size"],
        "hidden_size": size, "intermediate_size": ((round(native.get("expansion", 4.0) * size * 2 / 3) + 255) // 256) * 256,
        "num_layers_per_stack": layers, "num_hidden_layers": layers * native["H_cycles"] * (native["L_cycles"] * mos + 1),
        "num_attention_heads": heads, "num_key_value_heads": native.get("num_key_value_heads") or heads,
        "head_dim": size // heads, "max_position_embeddings": native["max_seq_len"], "H_cycles": native["H_cycles"],
        "L_cycles": native["L_cycles"], "bp_steps": native.get("bp_max_steps", 5),
        "rms_norm_eps": native.get("norm_eps", 1e-6), "hidden_act": "silu",
        "rope_parameters": {"rope_type": "default", "rope_theta": float(native.get("rope_theta", 10000))},
        "initializer_range": std, "embedding_scale": 1 / std, "tie_word_embeddings": False,
        "prefix_lm": native.get("attn_type", "prefixlm") == "prefixlm", "torch_dtype": "float32",
    }
    cfg.update({k: native[k] for k in FEATURE_FIELDS if k in native})
    cfg[NATIVE_CONFIG_KEY] = native
    return cfg


_LEVEL = re.compile(r"model\.(L|H)_level\.(?:core\.)?")
_GATE_UP = re.compile(r"\.mlp(?:\.experts\.\d+)?\.gate_up_proj\.weight$")


def to_hf_state(state: dict, num_heads: int, num_kv_heads: int) -> dict:
    out = {}
    for key, value in state.items():
        if ".rotary_emb." in key or key == "model.routing_bias_scale":
            continue
        key = key.replace("embed_tokens.embedding_weight", "model.embed_tokens.weight")
        key = key.replace("model.zL_init", "model.z_L_init")
        key = _LEVEL.sub(lambda m: f"model.{m.group(1)}_module.", key)
        if key.endswith(".attn.gqkv_proj.weight"):
            hd = value.shape[0] // (2 * num_heads + 2 * num_kv_heads)
            sizes = [num_heads * hd, num_heads * hd, num_kv_heads * hd, num_kv_heads * hd]
            prefix = key.removesuffix(".attn.gqkv_proj.weight")
            for name, piece in zip(("gate_proj", "q_proj", "k_proj", "v_proj"), value.split(sizes, dim=0)):
                out[f"{prefix}.self_attn.{name}.weight"] = piece.contiguous()
        elif _GATE_UP.search(key):
            prefix = key.removesuffix(".gate_up_proj.weight")
            for name, piece in zip(("gate_proj", "up_proj"), value.chunk(2, dim=0)):
                out[f"{prefix}.{name}.weight"] = piece.contiguous()
        else:
            out[key.replace(".attn.o_proj.", ".self_attn.o_proj.")] = value.contiguous()
    return out


def from_hf_state(hf: dict, native_keys) -> dict:
    """Inverse of ``to_hf_state`` for the key set of a freshly built native model."""
    out = {}
    for key in native_keys:
        if ".rotary_emb." in key or key == "model.routing_bias_scale":
            continue
        hf_key = key.replace("embed_tokens.embedding_weight", "model.embed_tokens.weight")
        hf_key = hf_key.replace("model.zL_init", "model.z_L_init")
        hf_key = _LEVEL.sub(lambda m: f"model.{m.group(1)}_module.", hf_key)
        if hf_key.endswith(".attn.gqkv_proj.weight"):
            prefix = hf_key.removesuffix(".attn.gqkv_proj.weight")
            out[key] = torch.cat([hf[f"{prefix}.self_attn.{n}.weight"] for n in ("gate_proj", "q_proj", "k_proj",
                                                                                  "v_proj")])
        elif _GATE_UP.search(hf_key):
            prefix = hf_key.removesuffix(".gate_up_proj.weight")
            out[key] = torch.cat([hf[f"{prefix}.gate_proj.weight"], hf[f"{prefix}.up_proj.weight"]])
        else:
            out[key] = hf[hf_key.replace(".attn.o_proj.", ".self_attn.o_proj.")]
    return out


def build_native(native: dict, dtype=torch.float32):
    from mimir_b200.models import LMHead, Mimir2
    cfg = dict(native) | {"fwd_bwd_dtype": "float32" if dtype == torch.float32 else str(dtype).split(".")[-1]}
    return LMHead(Mimir2(cfg), cfg)


class Mimir2ForCausalLM(nn.Module):
    """Inference wrapper over the native model that reads/writes the HF Mimir2 format."""

    def __init__(self, config: dict, native_model: Optional[nn.Module] = None):
        super().__init__()
        self.config = dict(config)
        self.native_config = dict(config[NATIVE_CONFIG_KEY])
        self.model = native_model if native_model is not None else build_native(self.native_config)
        self.generation_config: dict = {}

    @classmethod
    def from_native(cls, native: dict, state: dict) -> "Mimir2ForCausalLM":
        model = cls(hf_config(native))
        missing, unexpected = model.model.load_state_dict(state, strict=False)
        stray = [k for k in missing if ".rotary_emb." not in k and k != "model.routing_bias_scale"]
        if stray or unexpected:
            raise ValueError(f"Native state mismatch: missing={stray} unexpected={list(unexpected)}")
        return model.eval()

    def hf_state_dict(self) -> dict:
        return to_hf_state(self.model.state_dict(), self.config["num_attention_heads"],
                           self.config["num_key_value_heads"])

    def save_pretrained(self, directory) -> None:
        from safetensors.torch import save_file
        directory = Path(directory)
        directory.mkdir(parents=True, exist_ok=True)
        save_file(self.hf_state_dict(), str(directory / "model.safetensors"), metadata={"format": "pt"})
        (directory / "config.json").write_text(json.dumps(self.config, indent=2, sort_keys=True))
        if self.generation_config:
            (directory / "generation_config.json").write_text(json.dumps(self.generation_config, indent=2))

    @classmethod
    def from_pretrained(cls, directory) -> "Mimir2ForCausalLM":
        from safetensors.torch import load_file
        directory = Path(directory)
        config = json.loads((directory / "config.json").read_text())
        if config.get("model_type") != "mimir2":
            raise ValueError(f"{directory} is not a Mimir2 export")
        model = cls(config)
        tensors = load_file(str(directory / "model.safetensors"))
        native_keys = list(model.model.state_dict())
        state = from_hf_state(tensors, native_keys)
        used = set(to_hf_state(state, config["num_attention_heads"], config["num_key_value_heads"]))
        if used != set(tensors):
            raise ValueError(f"Unexpected tensors in {directory}: {sorted(set(tensors) - used)}")
        model.model.load_state_dict(state, strict=False)
        if (directory / "generation_config.json").exists():
            model.generation_config = json.loads((directory / "generation_config.json").read_text())
        return model.eval()

    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, prefix_lengths: Optional[list[int]] = None) -> torch.Tensor:
        """Logits ``[batch, seq, vocab]``; each row is one sequence (prefix-LM over its first
        ``prefix_lengths[i]`` tokens when the model was trained as a prefix LM, else causal)."""
        from mimir_b200.data.prefixlm import compute_aux_seq_tensors_scalars
        from mimir_b200.models.common import wrap_tensor
        b, s = input_ids.shape
        prefix = np.asarray(prefix_lengths if prefix_lengths is not None else [0] * b, dtype=np.int32)
        causal = s - prefix
        tensors, scalars = compute_aux_seq_tensors_scalars(prefix, causal, b * s)
        batch = {"inputs": input_ids.reshape(-1), "position_ids": torch.arange(s).repeat(b).to(input_ids.device)}
        batch.update({k: torch.from_numpy(v).to(input_ids.device) for k, v in tensors.items()})
        batch.update({k: wrap_tensor(torch.tensor(v)) for k, v in scalars.items()})
        _, logits = self.model(None, batch)
        return logits.view(b, s, -1)
