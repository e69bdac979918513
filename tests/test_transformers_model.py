"""The Transformers Mimir2 model (``mimir_b200.export.transformers_mimir2``) loads an export made
by ``mimir_b200.export.hf`` through ``AutoModelForCausalLM`` and reproduces the training model's
logits; cached greedy generation equals recomputing the whole sequence at every step (CPU)."""
import pytest
import torch

pytest.importorskip("transformers")

BASE = dict(max_seq_len=64, n_layers=2, hidden_size=64, num_heads=4, num_key_value_heads=2, expansion=4,
            init_type="lecun_normal", norm_type="pre", norm_eps=1e-6, pos_emb_type="rope", rope_theta=10000.0,
            H_cycles=2, L_cycles=2, half_layers=False, fwd_bwd_dtype="float32", vocab_size=96)
VARIANTS = [dict(), dict(gates_enabled=True), dict(ngram_orders=[2, 3], ngram_buckets=97, ngram_heads=2,
                                                   ngram_contextual_gate=True),
            dict(recurrence_mode="looped", H_cycles=2, L_cycles=2)]


def _export(tmp_path, extra):
    from mimir_b200.export.hf import Mimir2ForCausalLM as NativeExport, build_native
    native = BASE | extra
    torch.manual_seed(0)
    model = build_native(native)
    with torch.no_grad():  # move every parameter and alpha away from its initial value
        for p in model.parameters():
            p.add_(torch.randn_like(p) * 0.05)
        for name, buf in model.named_buffers():
            if name.endswith("alpha"):
                buf.fill_(0.6)
    wrapper = NativeExport.from_native(native, model.state_dict())
    wrapper.save_pretrained(tmp_path)
    return wrapper


@pytest.mark.parametrize("extra", VARIANTS, ids=["plain", "gates", "ngram", "looped"])
def test_auto_model_logits_equal_training_model(tmp_path, extra):
    from transformers import AutoModelForCausalLM
    from mimir_b200.export.transformers_mimir2 import Mimir2ForCausalLM, register
    register()
    native = _export(tmp_path, extra)
    model, info = AutoModelForCausalLM.from_pretrained(tmp_path, output_loading_info=True)
    assert isinstance(model, Mimir2ForCausalLM)
    assert not info["missing_keys"] and not info["unexpected_keys"]
    ids = torch.randint(0, 96, (2, 17), generator=torch.Generator().manual_seed(1))
    for prefix in ([5, 9], [0, 0], [17, 1]):
        ref = native(ids, prefix_lengths=prefix)
        out = model(ids, prefix_lengths=torch.tensor(prefix)).logits
        torch.testing.assert_close(out, ref, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("extra", VARIANTS[:3], ids=["plain", "gates", "ngram"])
def test_cached_generation_equals_full_recomputation(tmp_path, extra):
    from transformers import AutoModelForCausalLM
    from mimir_b200.export.transformers_mimir2 import register
    register()
    native = _export(tmp_path, extra)
    model = AutoModelForCausalLM.from_pretrained(tmp_path)
    prompt = torch.randint(0, 96, (1, 6), generator=torch.Generator().manual_seed(2))
    out = model.generate(prompt, max_new_tokens=5, do_sample=False, pad_token_id=0)
    seq = prompt
    for _ in range(5):  # the prompt is the prefix; generated tokens are causal
        logits = native(seq, prefix_lengths=[prompt.shape[1]])
        seq = torch.cat([seq, logits[:, -1].argmax(-1, keepdim=True)], dim=1)
    assert torch.equal(out, seq)


@pytest.mark.parametrize("extra", VARIANTS, ids=["plain", "gates", "ngram", "looped"])
def test_left_padded_batch_generates_like_single_prompts(tmp_path, extra):
    """Prompts of different lengths, left-padded into one batch (what batched serving does), give
    each prompt's own greedy continuation and the same first-step logits."""
    from transformers import AutoModelForCausalLM
    from mimir_b200.export.transformers_mimir2 import register
    register()
    _export(tmp_path, extra)
    model = AutoModelForCausalLM.from_pretrained(tmp_path)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(1, 96, (n,), generator=g) for n in (9, 4, 6)]
    width = max(len(p) for p in prompts)
    batch = torch.zeros(len(prompts), width, dtype=torch.long)
    mask = torch.zeros_like(batch)
    for i, p in enumerate(prompts):
        batch[i, width - len(p):] = p
        mask[i, width - len(p):] = 1
    with torch.no_grad():
        padded_logits = model(batch, attention_mask=mask).logits[:, -1]
    out = model.generate(batch, attention_mask=mask, max_new_tokens=5, do_sample=False, pad_token_id=0)
    for i, p in enumerate(prompts):
        with torch.no_grad():
            alone_logits = model(p[None]).logits[:, -1]
        torch.testing.assert_close(padded_logits[i:i + 1], alone_logits, atol=1e-5, rtol=1e-5)
        alone = model.generate(p[None], max_new_tokens=5, do_sample=False, pad_token_id=0)
        assert torch.equal(out[i, width:], alone[0, len(p):]), (i, out[i, width:], alone[0, len(p):])
