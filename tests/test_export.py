"""Export to the HF Mimir2 format: key mapping, EMA selection, bit-exact reload, refusals."""
import json

import pytest
import torch

from mimir_b200.config.schema import load_config
from mimir_b200.data.synthetic import write_corpus
from mimir_b200.export.convert import export
from mimir_b200.export.hf import Mimir2ForCausalLM, from_hf_state, to_hf_state

BASE = ["size@arch=XXS", "accelerator_type=cpu", "distributed_strategy=none", "fwd_bwd_dtype=float32",
        "global_batch_size=128", "epochs=1", "lr_warmup_steps=1", "arch.hidden_size=64", "arch.n_layers=2",
        "arch.H_cycles=2", "arch.L_cycles=2", "dataloader_prefetch_factor=2", "ema=0.9"]


def _tokenizer(path):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    vocab = {w: i for i, w in enumerate(["<unk>", "<s>", "</s>", "<pad>", "user", "assistant", "Test", ":"])}
    core = Tokenizer(models.WordLevel(vocab, unk_token="<unk>"))
    core.pre_tokenizer = pre_tokenizers.Whitespace()
    tok = PreTrainedTokenizerFast(tokenizer_object=core, bos_token="<s>", eos_token="</s>", pad_token="<pad>",
                                  unk_token="<unk>")
    tok.chat_template = "{% for m in messages %}{{ m['role'] }} : {{ m['content'] }} {% endfor %}" \
                        "{% if add_generation_prompt %}assistant :{% endif %}"
    tok.save_pretrained(str(path))
    return path


@pytest.fixture(scope="module")
def trained(tmp_path_factory):
    from mimir_b200.train.loop import launch
    root = tmp_path_factory.mktemp("export")
    data = write_corpus(str(root / "data"), rows=32, seq_len=32, vocab=64)
    launch(load_config(BASE + [f"data.path={data}", f"checkpoint_path={root / 'run'}", "stop_after_step=3"]))
    return root / "run" / "step_3", _tokenizer(root / "tok")


def test_key_mapping_roundtrip_with_gqa():
    state = {"model.L_level.core.layers.0.attn.gqkv_proj.weight": torch.randn(6 * 4, 8),
             "model.H_level.core.layers.0.mlp.gate_up_proj.weight": torch.randn(10, 8),
             "model.L_level.core.layers.0.attn.o_proj.weight": torch.randn(8, 8),
             "model.zL_init": torch.randn(8), "embed_tokens.embedding_weight": torch.randn(5, 8),
             "model.routing_bias_scale": torch.tensor(1.0)}
    hf = to_hf_state(state, num_heads=2, num_kv_heads=1)
    assert hf["model.L_module.layers.0.self_attn.q_proj.weight"].shape == (8, 8)
    assert hf["model.L_module.layers.0.self_attn.k_proj.weight"].shape == (4, 8)
    assert {"model.H_module.layers.0.mlp.gate_proj.weight", "model.z_L_init", "model.embed_tokens.weight",
            "model.L_module.layers.0.self_attn.o_proj.weight"} <= set(hf)
    assert "model.routing_bias_scale" not in hf
    back = from_hf_state(hf, [k for k in state if k != "model.routing_bias_scale"])
    for k, v in back.items():
        assert torch.equal(v, state[k])


def test_export_ema_roundtrip(trained, tmp_path):
    ckpt, tok = trained
    out = export(ckpt, tmp_path / "hf", tok, ema=True)
    cfg = json.loads((out / "config.json").read_text())
    assert cfg["model_type"] == "mimir2" and cfg["eos_token_id"] == 2 and cfg["num_layers_per_stack"] == 1
    receipt = json.loads((out / "export_receipt.json").read_text())
    assert receipt["ema"] and receipt["checkpoint_manifest"]["tag"] == "step_3"
    model = Mimir2ForCausalLM.from_pretrained(out)
    logits = model(torch.tensor([[1, 2, 3, 4]]), prefix_lengths=[2])
    assert logits.shape == (1, 4, cfg["vocab_size"]) and torch.isfinite(logits).all()
    live = export(ckpt, tmp_path / "live", tok, ema=False)
    assert not torch.equal(Mimir2ForCausalLM.from_pretrained(live)(torch.tensor([[1, 2]])),
                           model(torch.tensor([[1, 2]])))
    with pytest.raises(FileExistsError):
        export(ckpt, out, tok)


def test_export_refuses_corrupt_checkpoint(trained, tmp_path):
    import shutil
    ckpt, tok = trained
    copy = tmp_path / "copy"
    shutil.copytree(ckpt, copy)
    (copy / "rng.0.pt").write_bytes(b"x" * (copy / "rng.0.pt").stat().st_size)
    with pytest.raises(ValueError, match="Corrupt"):
        export(copy, tmp_path / "out", tok)
    assert not (tmp_path / "out").exists()


def test_cpu_qualification_campaign(tmp_path):
    """Train / split+resume / EMA export + smoke eval / disk suspension, all bit-exact."""
    from mimir_b200.qualify import main
    result = json.loads(main(tmp_path / "campaign").read_text())
    assert result["status"] == "passed"
    assert (tmp_path / "campaign" / "evaluation" / "receipt.json").is_file()
