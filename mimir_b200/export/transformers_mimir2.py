"""Mimir2 as a Hugging Face Transformers model: reads the files ``mimir_b200 export`` writes.

Behavioural reference: the Mimir2 Transformers integration (``patches/transformers.patch``:
``Mimir2Config`` ``:278-545``, the modelling code ``:714-1500``), re-implemented here as a plain
``PreTrainedModel`` so that ``AutoModelForCausalLM.from_pretrained(<export dir>)`` works with the
stock Transformers package once :func:`register` has run (no patch, no remote code).

Layout (the export's HF names):

* ``model.embed_tokens`` (multiplied by ``embedding_scale``), optional ``model.ngram`` (hashed
  n-gram memory, the same module as the training model), ``model.z_L_init``;
* ``model.L_module`` / ``model.H_module``: pre-norm stacks of blocks with a weightless RMSNorm,
  gated attention (``self_attn.{gate,q,k,v,o}_proj``: ``o_proj(sigmoid(gate) * attention)``,
  RoPE on q/k in fp32, grouped KV heads) and a SwiGLU MLP (``mlp.{gate,up,down}_proj``), and a
  weightless final norm; optional ``invocation_gates``;
* ``lm_head``.

The recurrence is the training model's: per H cycle, ``L_cycles`` L-stack calls on ``z_L +
injection(z_H)`` then one H-stack call on ``z_H + injection(z_L)`` (looped recurrence: L restarts
from z_H with no injection and H follows L directly).  Attention is prefix-LM: the first
``prefix_length`` tokens of a sequence see each other, every later token sees all earlier ones.
For generation every stack invocation keeps its own KV cache (virtual layer ``invocation *
layers + layer``) and the prompt is the prefix.

Mixtures of experts or stacks, residual branches and recurrent memories are not implemented by
this model (the export's own :class:`mimir_b200.export.hf.Mimir2ForCausalLM` runs those).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F
from torch import nn
from transformers import AutoConfig, AutoModelForCausalLM, GenerationMixin, PretrainedConfig, PreTrainedModel
from transformers.cache_utils import DynamicCache
from transformers.modeling_outputs import CausalLMOutputWithPast

_UNSUPPORTED = {"moe_num_experts": 1, "mos_num_experts": 1, "residual_branches": 1, "h_memory_branches": 1,
                "l_memory_branches": 1}


class Mimir2Config(PretrainedConfig):
    model_type = "mimir2"

    def __init__(self, vocab_size=32000, hidden_size=512, intermediate_size=1536, num_layers_per_stack=2,
                 num_hidden_layers=None, num_attention_heads=8, num_key_value_heads=None, head_dim=None,
                 max_position_embeddings=2048, H_cycles=2, L_cycles=2, rms_norm_eps=1e-6, rope_parameters=None,
                 embedding_scale=1.0, prefix_lm=True, gates_enabled=False, ngram_orders=None, ngram_buckets=4096,
                 ngram_heads=1, ngram_contextual_gate=False, tie_word_embeddings=False, **kwargs):
        native = kwargs.get("mimir_native_config") or {}
        self.vocab_size, self.hidden_size, self.intermediate_size = vocab_size, hidden_size, intermediate_size
        self.num_layers_per_stack = num_layers_per_stack
        self.num_attention_heads = num_attention_heads
        self.num_key_value_heads = num_key_value_heads or num_attention_heads
        self.head_dim = head_dim or hidden_size // num_attention_heads
        self.max_position_embeddings = max_position_embeddings
        self.H_cycles, self.L_cycles = H_cycles, L_cycles
        self.num_hidden_layers = num_hidden_layers or num_layers_per_stack * H_cycles * (L_cycles + 1)
        self.rms_norm_eps = rms_norm_eps
        self.rope_parameters = rope_parameters or {"rope_type": "default", "rope_theta": 10000.0}
        self.embedding_scale = embedding_scale
        self.prefix_lm = prefix_lm
        self.gates_enabled = gates_enabled
        self.recurrence_mode = kwargs.pop("recurrence_mode", native.get("recurrence_mode", "hierarchical"))
        self.ngram_orders = list(ngram_orders or [])
        self.ngram_buckets, self.ngram_heads = ngram_buckets, ngram_heads
        self.ngram_contextual_gate = ngram_contextual_gate
        super().__init__(tie_word_embeddings=tie_word_embeddings, **kwargs)

    def check_supported(self) -> None:
        for name, plain in _UNSUPPORTED.items():
            if getattr(self, name, plain) != plain:
                raise NotImplementedError(f"{name}={getattr(self, name)} is not implemented by the Transformers "
                                          "Mimir2 model; use mimir_b200.export.hf.Mimir2ForCausalLM")


def _rms(x: torch.Tensor, eps: float) -> torch.Tensor:
    return F.rms_norm(x, (x.shape[-1],), eps=eps)


def _rotate(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


class _Rope(nn.Module):
    """cos/sin tables for positions (computed on the fly: nothing here is loaded from a checkpoint,
    and a model built on the meta device by ``from_pretrained`` holds no initialised buffer)."""

    def __init__(self, dim: int, theta: float):
        super().__init__()
        self.dim, self.theta = dim, theta

    def forward(self, positions: torch.Tensor):
        inv_freq = 1.0 / (self.theta ** (torch.arange(0, self.dim, 2, dtype=torch.float32,
                                                      device=positions.device) / self.dim))
        angles = positions.float()[..., None] * inv_freq
        table = torch.cat((angles, angles), dim=-1)
        return table.cos(), table.sin()


def _apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """fp32 rotary embedding of ``x [b, s, heads, d]`` with tables ``[b, s, d]``."""
    return (x * cos.unsqueeze(-2) + _rotate(x) * sin.unsqueeze(-2)).to(x.dtype)


class Mimir2Attention(nn.Module):
    def __init__(self, config: Mimir2Config):
        super().__init__()
        d, h, kv, hd = config.hidden_size, config.num_attention_heads, config.num_key_value_heads, config.head_dim
        self.heads, self.kv_heads, self.head_dim = h, kv, hd
        self.gate_proj = nn.Linear(d, h * hd, bias=False)
        self.q_proj = nn.Linear(d, h * hd, bias=False)
        self.k_proj = nn.Linear(d, kv * hd, bias=False)
        self.v_proj = nn.Linear(d, kv * hd, bias=False)
        self.o_proj = nn.Linear(h * hd, d, bias=False)

    def forward(self, x, rope, mask, cache: Optional[DynamicCache], layer_idx: int):
        b, s, _ = x.shape
        shape = (b, s, -1, self.head_dim)
        gate = self.gate_proj(x).view(shape)
        q = _apply_rope(self.q_proj(x).view(shape), *rope)
        k = _apply_rope(self.k_proj(x).view(shape), *rope)
        v = self.v_proj(x).view(shape)
        k, v = k.transpose(1, 2), v.transpose(1, 2)
        if cache is not None:
            k, v = cache.update(k, v, layer_idx)
        if self.kv_heads != self.heads:
            rep = self.heads // self.kv_heads
            k, v = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
        attn = F.scaled_dot_product_attention(q.transpose(1, 2), k, v, attn_mask=mask).transpose(1, 2)
        return self.o_proj((torch.sigmoid(gate) * attn).flatten(-2))


class Mimir2MLP(nn.Module):
    def __init__(self, config: Mimir2Config):
        super().__init__()
        d, f = config.hidden_size, config.intermediate_size
        self.gate_proj = nn.Linear(d, f, bias=False)
        self.up_proj = nn.Linear(d, f, bias=False)
        self.down_proj = nn.Linear(f, d, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class Mimir2Block(nn.Module):
    def __init__(self, config: Mimir2Config):
        super().__init__()
        self.eps = config.rms_norm_eps
        self.self_attn = Mimir2Attention(config)
        self.mlp = Mimir2MLP(config)

    def forward(self, x, rope, mask, cache, layer_idx):
        x = x + self.self_attn(_rms(x, self.eps), rope, mask, cache, layer_idx)
        return x + self.mlp(_rms(x, self.eps))


class Mimir2InvocationGate(nn.Module):
    """``injection * (1 + alpha * tanh(W [hidden; injection] + b))``."""

    def __init__(self, hidden_size: int):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(hidden_size, 2 * hidden_size))
        self.bias = nn.Parameter(torch.zeros(hidden_size))

    def forward(self, hidden, injection, alpha):
        hidden, injection = torch.broadcast_tensors(hidden, injection)
        x = torch.cat((hidden, injection), dim=-1)
        return injection * (1 + alpha.to(x.dtype) * torch.tanh(F.linear(x, self.weight.to(x.dtype),
                                                                        self.bias.to(x.dtype))))


class Mimir2Stack(nn.Module):
    def __init__(self, config: Mimir2Config, invocations: int):
        super().__init__()
        self.eps = config.rms_norm_eps
        self.layers = nn.ModuleList(Mimir2Block(config) for _ in range(config.num_layers_per_stack))
        if config.gates_enabled:
            self.invocation_gates = nn.ModuleList(Mimir2InvocationGate(config.hidden_size) for _ in range(invocations))

    def forward(self, x, rope, mask, cache, first_layer_idx: int):
        for i, block in enumerate(self.layers):
            x = block(x, rope, mask, cache, first_layer_idx + i)
        return _rms(x, self.eps)


class Mimir2PreTrainedModel(PreTrainedModel):
    config_class = Mimir2Config
    base_model_prefix = "model"
    _no_split_modules = ["Mimir2Block"]

    def _init_weights(self, module):  # weights always come from an export
        return


class Mimir2Model(Mimir2PreTrainedModel):
    def __init__(self, config: Mimir2Config):
        super().__init__(config)
        config.check_supported()
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        if config.ngram_orders:
            from mimir_b200.models.ngram import NGramMemory
            self.ngram = NGramMemory(config.hidden_size, config.ngram_orders, config.ngram_buckets, config.ngram_heads,
                                     config.ngram_contextual_gate)
        self.L_module = Mimir2Stack(config, config.H_cycles * config.L_cycles)
        self.H_module = Mimir2Stack(config, config.H_cycles)
        self.register_buffer("z_L_init", torch.zeros(config.hidden_size))
        if config.gates_enabled:
            self.register_buffer("gate_alpha", torch.tensor(0.0))
        self.rope = _Rope(config.head_dim, float(config.rope_parameters.get("rope_theta", 10000.0)))
        self.post_init()

    def _mask(self, b, s, past, prefix_lengths, device, dtype, key_valid=None):
        """Additive mask ``[b, 1, s, past + s]``: keys before the new tokens are all visible; among
        the new ones, a query sees every key up to its own position and, inside the prefix, all of
        the prefix.  ``key_valid`` ([b, past + s] bool) hides padding keys of a left-padded batch."""
        q = torch.arange(s, device=device)[:, None] + past
        k = torch.arange(past + s, device=device)[None, :]
        allowed = (k <= q).expand(b, s, past + s)
        if prefix_lengths is not None:
            p = prefix_lengths.to(device)[:, None, None]
            allowed = allowed | ((q[None] < p) & (k[None] < p))
        if key_valid is not None:
            allowed = allowed & key_valid.to(device)[:, None, :]
        mask = torch.zeros(b, 1, s, past + s, device=device, dtype=dtype)
        return mask.masked_fill(~allowed[:, None], torch.finfo(dtype).min)

    def forward(self, input_ids, prefix_lengths=None, past_key_values: Optional[DynamicCache] = None,
                position_ids=None, key_valid=None):
        cfg = self.config
        b, s = input_ids.shape
        past = past_key_values.get_seq_length() if past_key_values is not None else 0
        if position_ids is None:
            position_ids = torch.arange(past, past + s, device=input_ids.device).expand(b, s)
        x = self.embed_tokens(input_ids) * cfg.embedding_scale
        if cfg.ngram_orders:
            history = None
            if past_key_values is not None:
                history = getattr(past_key_values, "mimir_ngram_history", None)
                if history is None:
                    history = past_key_values.mimir_ngram_history = {}
            x = self.ngram(x, input_ids, position_ids, history)
        rope = self.rope(position_ids)
        mask = self._mask(b, s, past, prefix_lengths if cfg.prefix_lm else None, x.device, x.dtype, key_valid)
        layers = cfg.num_layers_per_stack
        looped = cfg.recurrence_mode == "looped"
        z_h, z_l = x, self.z_L_init.to(x.dtype)
        call = 0
        for i in range(cfg.H_cycles):
            if looped:
                z_l = z_h
            for k in range(i * cfg.L_cycles, (i + 1) * cfg.L_cycles):
                if looped:
                    stack_in = z_l
                elif cfg.gates_enabled:
                    stack_in = z_l + self.L_module.invocation_gates[k](z_l, z_h, self.gate_alpha)
                else:
                    stack_in = z_l + z_h
                z_l = self.L_module(stack_in, rope, mask, past_key_values, call * layers)
                call += 1
            if looped:
                stack_in = z_l
            elif cfg.gates_enabled:
                stack_in = z_h + self.H_module.invocation_gates[i](z_h, z_l, self.gate_alpha)
            else:
                stack_in = z_h + z_l
            z_h = self.H_module(stack_in, rope, mask, past_key_values, call * layers)
            call += 1
        return z_h


class Mimir2ForCausalLM(Mimir2PreTrainedModel, GenerationMixin):
    def __init__(self, config: Mimir2Config):
        super().__init__(config)
        self.model = Mimir2Model(config)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        self.post_init()

    def forward(self, input_ids=None, attention_mask=None, past_key_values=None, use_cache=None, labels=None,
                prefix_lengths=None, position_ids=None, cache_position=None, **kwargs):
        if use_cache and past_key_values is None:
            past_key_values = DynamicCache()
        if prefix_lengths is None and self.config.prefix_lm and (past_key_values is None
                                                                 or past_key_values.get_seq_length() == 0):
            # A prompt is the prefix: every prompt token sees the whole prompt.
            prefix_lengths = torch.full((input_ids.shape[0],), input_ids.shape[1], dtype=torch.long)
        positions, key_valid = None, None
        if attention_mask is not None and not bool(attention_mask.all()):
            # A left-padded batch (batched serving): positions count real tokens only (padding
            # sits at position 0, so no n-gram or rotary phase reaches across it) and padding keys
            # are hidden from every query.
            past = past_key_values.get_seq_length() if past_key_values is not None else 0
            am = attention_mask.to(device=input_ids.device, dtype=torch.long)[:, :past + input_ids.shape[1]]
            positions = (am.cumsum(-1) - 1).clamp_min(0)[:, past:]
            key_valid = am.bool()
        hidden = self.model(input_ids, prefix_lengths=prefix_lengths,
                            past_key_values=past_key_values if use_cache or past_key_values is not None else None,
                            position_ids=positions, key_valid=key_valid)
        logits = self.lm_head(hidden)
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), labels[:, 1:].reshape(-1),
                                   ignore_index=-100)
        return CausalLMOutputWithPast(loss=loss, logits=logits, past_key_values=past_key_values)


def register() -> None:
    """Make ``AutoConfig`` / ``AutoModelForCausalLM`` resolve ``model_type = "mimir2"``."""
    try:
        AutoConfig.register("mimir2", Mimir2Config)
    except ValueError:
        pass  # already registered
    try:
        AutoModelForCausalLM.register(Mimir2Config, Mimir2ForCausalLM)
    except ValueError:
        pass
