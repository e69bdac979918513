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
