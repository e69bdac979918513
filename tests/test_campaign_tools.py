"""Campaign preparation / extension, the OKF bundle validator and protocol recovery (CPU).

Reference behaviour: ``tools/prepare_xxs_ablation.py``, ``tools/extend_xxs_ablation.py``,
``scripts/validate_okf.py``, ``tools/recover_protocols.py``.
"""
import json
import zipfile

import pytest

from mimir_b200.data.synthetic import write_corpus


def _tokenizer(path):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    vocab = {f"t{i}": i for i in range(60)} | {"<unk>": 60, "<s>": 61, "</s>": 62}
    tok = Tokenizer(models.WordLevel(vocab, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="<unk>", bos_token="<s>", eos_token="</s>").save_pretrained(path)
    template = path / "template.jinja"
    template.write_text("{% for m in messages %}{{ m['role'] }}: {{ m['content'] }}\n{% endfor %}"
                        "{% if add_generation_prompt %}assistant:{% if enable_thinking is defined and enable_thinking %}"
                        " <think>{% endif %}{% endif %}")
    return path, template


def _recipe(tmp_path, steps=4000):
    recipe = {"schema": 1, "id": "tiny", "steps": steps, "batch_tokens": 1, "eval_step_multiple": 2000,
              "capacity_target": {"baseline": "default", "ratio": 2.0, "tolerance_percent": 2.0},
              "common_overrides": ["size@arch=XXS", "arch.hidden_size=64", "arch.n_layers=2", "epochs=1"],
              "variants": {"default": [], "wider": ["arch.n_layers=4"]},
              "suites": ["cpu-smoke-v1"], "default_eval_steps": [steps]}
    path = tmp_path / "recipe.json"
    path.write_text(json.dumps(recipe))
    return path


def test_prepare_writes_a_held_queue_and_extend_appends(tmp_path):
    from mimir_b200.campaigns.prepare import extend, prepare
    from mimir_b200.scheduling.store import Store
    data = write_corpus(str(tmp_path / "data"), rows=400, seq_len=32, vocab=64)
    tok, template = _tokenizer(tmp_path / "tok")
    out = prepare(tmp_path / "campaign", data, tok, template, recipe=_recipe(tmp_path), gpus="0,1",
                  eval_steps=[2000, 4000], database=tmp_path / "q" / "queue.sqlite")
    plan = json.loads((out / "plan.json").read_text())
    ids = [j["id"] for j in plan["jobs"]]
    assert ids[:4] == ["default.step_2000.train", "default.step_2000.checkpoint", "default.step_2000.export",
                       "default.step_2000.cpu-smoke-v1.next-token"]
    second = next(j for j in plan["jobs"] if j["id"] == "default.step_4000.train")
    assert "resume_checkpoint_tag=step_2000" in second["config"]["command"]
    assert {"id": "default.step_2000.train", "policy": "success"} in second["depends"]
    wider = next(j for j in plan["jobs"] if j["id"] == "wider.step_2000.train")
    assert {d["id"] for d in wider["depends"]} == {"default.step_4000.cpu-smoke-v1.next-token"}  # after its evals
    rows = Store(tmp_path / "q" / "queue.sqlite").rows()
    assert len(rows) == len(ids) and all(r["held"] and r["state"] == "pending" for r in rows)
    counts = json.loads((out / "parameters.json").read_text())
    assert counts["wider"]["capacity"] > counts["default"]["capacity"]
    receipt = json.loads((out / "preparation.json").read_text())
    assert receipt["status"] == "prepared_not_started" and receipt["jobs"] == len(ids)
    with pytest.raises(FileExistsError):  # a preparation directory is never reused
        prepare(out, data, tok, template, recipe=_recipe(tmp_path))

    # extension: final-step-only preparations are required
    with pytest.raises(ValueError, match="final-step-only"):
        extend(out, extensions=_extensions(tmp_path))
    out2 = prepare(tmp_path / "campaign2", data, tok, template, recipe=_recipe(tmp_path),
                   database=tmp_path / "q2" / "queue.sqlite")
    added = extend(out2, extensions=_extensions(tmp_path))
    plan2 = json.loads((out2 / "scheduled-plan.json").read_text())
    muon = next(j for j in plan2["jobs"] if j["id"] == "muon.step_4000.train")
    assert "optimizer=muon" in muon["config"]["command"] and "/runs/muon/" in json.dumps(muon["config"])
    assert {d["id"] for d in muon["depends"]} == {"wider.step_4000.cpu-smoke-v1.next-token"}
    assert added == 4 and len(Store(tmp_path / "q2" / "queue.sqlite").rows()) == len(plan2["jobs"])


def _extensions(tmp_path):
    path = tmp_path / "ext.json"
    path.write_text(json.dumps({"schema": 1, "after": "wider",
                                "variants": {"muon": {"source": "default", "overrides": ["optimizer=muon"]}}}))
    return path


def test_recipe_rejects_bad_eval_steps(tmp_path):
    from mimir_b200.campaigns.prepare import Recipe
    recipe = Recipe.load(_recipe(tmp_path))
    assert recipe.eval_steps([4000, 2000]) == [2000, 4000]
    for bad in ([3000, 4000], [2000]):
        with pytest.raises(ValueError):
            recipe.eval_steps(bad)


def test_shipped_recipes_compose():
    from mimir_b200.campaigns.prepare import RECIPES, Recipe
    from mimir_b200.config.schema import load_config
    recipe = Recipe.load(RECIPES / "xxs-dfm15-20k.json")
    ext = json.loads((RECIPES / "xxs-dfm15-20k.extensions.json").read_text())
    for extra in list(recipe.variants.values()) + [recipe.variants[v["source"]] + v["overrides"]
                                                   for v in ext["variants"].values()]:
        load_config(recipe.common_overrides + extra + ["data.path=x", "checkpoint_path=y"])


def _page(path, text):
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(text)


def test_okf_bundle_validation(tmp_path):
    from mimir_b200.utils.okf import validate
    b = tmp_path / "wiki"
    _page(b / "index.md", '---\nokf_version: "0.2"\n---\n# Wiki\n[a](a.md) [g](group/)\n')
    _page(b / "a.md", "---\ntype: concept\nstatus: stable\nsources:\n  - resource: paper\n---\nSee [b](group/b.md).\n")
    _page(b / "group" / "index.md", "# Group\n[b](b.md)\n")
    _page(b / "group" / "b.md", "---\ntype: note\nconfidence: high\n---\nBack to [a](../a.md).\n")
    _page(b / "group" / "log.md", "## 2026-01-02\nstarted\n")
    report = validate(b)
    assert report.ok and not report.warnings, report
    _page(b / "group" / "c.md", "---\nstatus: shaky\n---\n[[old]] [gone](missing.md)\n")
    _page(b / "group" / "log.md", "---\nx: 1\n---\nno dates\n")
    report = validate(b)
    text = "\n".join(report.errors)
    for expected in ("missing immediate child link 'c.md'", "concept requires a non-empty type",
                     "invalid status 'shaky'", "legacy wiki-link syntax", "log files must not have frontmatter",
                     "log must contain ISO"):
        assert expected in text, (expected, text)
    assert any("missing.md" in w for w in report.warnings)


def test_protocol_recovery_keeps_only_allowlisted_fields(tmp_path):
    from mimir_b200.evaluation.protocols import recover
    header = {"status": "success",
              "eval": {"task": "piqa", "dataset": {"name": "piqa", "samples": 108, "location": "/secret/path"},
                       "config": {"limit": 10, "epochs": 1, "api_key": "sk-123"},
                       "model_args": {"token": "hf_xyz"}},
              "plan": {"config": {"max_tokens": 16, "temperature": 0.0, "api_base": "http://internal"}},
              "results": {"scores": [{"name": "choice"}]}}
    logs = tmp_path / "logs" / "run1"
    logs.mkdir(parents=True)
    with zipfile.ZipFile(logs / "a.eval", "w", compression=zipfile.ZIP_DEFLATED) as z:
        z.writestr("header.json", json.dumps(header))
    with zipfile.ZipFile(logs / "b.eval", "w") as z:
        z.writestr("samples/1.json", "{}")  # no header: ignored
    (logs / "c.eval").write_bytes(b"not a zip")
    result = recover(tmp_path / "logs", tmp_path / "out.json")
    (record,) = result["records"]
    assert record["task"] == "piqa" and record["dataset"] == {"name": "piqa", "samples": 108}
    assert record["selection"] == {"limit": 10, "epochs": 1} and record["scorers"] == ["choice"]
    assert record["generation"] == {"max_tokens": 16, "temperature": 0.0}
    dumped = (tmp_path / "out.json").read_text()
    assert "secret" not in dumped and "sk-123" not in dumped and "hf_xyz" not in dumped and "internal" not in dumped
    assert result["skipped"] == [{"source": "run1/c.eval", "reason": "unreadable log"}]
