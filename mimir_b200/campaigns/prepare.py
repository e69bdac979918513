"""Campaign preparation: a recipe of model variants, each trained to a fixed token budget, then
checkpointed, exported and evaluated at chosen steps, turned into HELD jobs of the scheduler
queue.  Preparation runs nothing (no training, no GPU); an operator releases the jobs.

Reference behaviour: ``tools/prepare_xxs_ablation.py`` (prepare) and
``tools/extend_xxs_ablation.py`` (append variants derived from prepared ones).  The recipe and
extension JSON formats and the queue's job configs are interfaces shared with the scheduler
(``mimir_b200/scheduling``), so they keep the reference's keys.

Per variant and evaluation step ``s`` the plan holds, in dependency order:

    <variant>.step_<s>.train             train to s (resumed from the previous step's checkpoint)
    <variant>.step_<s>.checkpoint        wait until checkpoint step_<s> is complete (manifest)
    <variant>.step_<s>.export            Hugging Face export of that checkpoint
    <variant>.step_<s>.<suite>.<task>    one evaluation per task of every suite
    <variant>.step_<s>.<suite>.merge     per-task metric records of the suite's Inspect tasks

Variants train one after another: a variant's first training job waits (terminal policy) for
the previous variant's evaluations, so evaluation servers never share GPUs with training.
"""
from __future__ import annotations

import hashlib
import json
import shutil
import sys
import tempfile
from dataclasses import dataclass, field, fields
from pathlib import Path
from typing import Optional

RECIPES = Path(__file__).resolve().parent / "recipes"
SUITES = Path(__file__).resolve().parents[1] / "evaluation" / "suites"


def _write(path: Path, value) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(value, indent=2, allow_nan=False) + "\n")


def _sha256(path: Path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


@dataclass
class Recipe:
    id: str
    steps: int
    common_overrides: list
    variants: dict
    suites: list
    default_eval_steps: list
    batch_tokens: int = 196608
    eval_step_multiple: int = 5000
    capacity_target: Optional[dict] = None
    path: Optional[Path] = None

    @classmethod
    def load(cls, path) -> "Recipe":
        path = Path(path)
        raw = json.loads(path.read_text())
        if raw.get("schema") != 1:
            raise ValueError(f"{path}: unsupported recipe schema {raw.get('schema')!r}")
        known = {f.name for f in fields(cls)} - {"path"}
        return cls(**{k: v for k, v in raw.items() if k in known}, path=path)

    def eval_steps(self, requested=None) -> list:
        steps = sorted(set(requested or self.default_eval_steps))
        if (not steps or steps[-1] != self.steps
                or any(s < 1 or s > self.steps or s % self.eval_step_multiple for s in steps)):
            raise ValueError(f"Evaluation steps must be multiples of {self.eval_step_multiple} and include the "
                             f"final step {self.steps}")
        return steps


def inspect_corpus(path) -> dict:
    """Receipt of a prepared corpus: header files, array shapes and a bounded validation of three
    index windows (start, middle, end).  The token stream itself is not scanned."""
    import numpy as np

    from mimir_b200.data.corpus import V1DatasetIndices, validate_arrays
    path = Path(path).resolve()
    metadata = json.loads((path / "metadata.json").read_text())
    tokens = np.load(path / "tokens.npy", mmap_mode="r")
    names = [f.name for f in fields(V1DatasetIndices)]
    index = {n: np.load(path / "epoch_0" / f"{n}.npy", mmap_mode="r") for n in names}
    rows = len(index[names[0]])
    if rows == 0 or any(a.ndim != 1 or len(a) != rows for a in index.values()):
        raise ValueError(f"{path}: empty or misaligned index arrays")
    window = 1024
    for start in sorted({0, rows // 2, max(0, rows - window)}):
        validate_arrays(tokens, V1DatasetIndices(**{n: a[start:start + window] for n, a in index.items()}))
    receipt = {"path": str(path), "metadata_sha256": _sha256(path / "metadata.json"), "metadata": metadata,
               "epoch_0_rows": rows, "stored_tokens": int(len(tokens)),
               "validation_scope": f"headers and up to {3 * window} index rows; no token scan",
               "arrays": {n: {"shape": list(a.shape), "dtype": str(a.dtype)} for n, a in index.items()}}
    for name in ("ready.json", "validated.json"):
        if (path / name).exists():
            receipt[name] = {"sha256": _sha256(path / name), "content": json.loads((path / name).read_text())}
    return receipt


def count_parameters(arch: dict) -> dict:
    """Trainable capacity of a model config, counted on the meta device (no memory, no GPU)."""
    import torch

    from mimir_b200.models import LMHead, Mimir2
    with torch.device("meta"):
        model = LMHead(Mimir2(arch), arch)
    io = sum(p.numel() for n, p in model.named_parameters() if n.startswith(("embed_tokens.", "lm_head.")))
    total = sum(p.numel() for p in model.parameters())
    return {"capacity": total - io, "token_embedding_and_lm_head": io, "total": total}


def _copy_tokenizer(tokenizer: Path, template: Path, out: Path, vocab: int) -> dict:
    """Copy the tokenizer files and the dataset's chat template (never weights or code) and check
    that the template's default is the non-thinking generation prompt."""
    out.mkdir(parents=True)
    for name in ("tokenizer.json", "tokenizer_config.json", "special_tokens_map.json", "added_tokens.json"):
        if (tokenizer / name).exists():
            shutil.copyfile(tokenizer / name, out / name)
    shutil.copyfile(template, out / "chat_template.jinja")
    from transformers import AutoTokenizer
    tok = AutoTokenizer.from_pretrained(out, local_files_only=True)
    if len(tok) > vocab:
        raise ValueError(f"Tokenizer ({len(tok)} entries) exceeds the corpus vocabulary ({vocab})")
    probe = [{"role": "user", "content": "Test"}]
    plain = tok.apply_chat_template(probe, tokenize=False, add_generation_prompt=True)
    if plain != tok.apply_chat_template(probe, tokenize=False, add_generation_prompt=True, enable_thinking=False):
        raise ValueError("The chat template must default to the non-thinking generation prompt")
    return {"source": str(tokenizer), "tokenizer_sha256": _sha256(out / "tokenizer.json"),
            "template_source": str(template), "template_sha256": _sha256(template), "vocab_size": len(tok)}


@dataclass
class _Plan:
    jobs: list = field(default_factory=list)

    def add(self, identity: str, kind: str, config: dict, depends=()) -> str:
        self.jobs.append({"id": identity, "kind": kind, "config": config, "held": True,
                          "max_attempts": 1 if kind == "train" else 3,
                          "depends": [{"id": d, "policy": p} for d, p in depends]})
        return identity


def _suite_tasks(name: str) -> tuple[Path, list]:
    source = SUITES / f"{name}.json"
    return source, json.loads(source.read_text())["tasks"]


def prepare(output, data, tokenizer, template, *, recipe=RECIPES / "xxs-dfm15-20k.json", gpus: Optional[str] = None,
            eval_steps=None, database=None, python: str = sys.executable) -> Path:
    """Write the campaign directory ``output`` and a held queue; return ``output``."""
    from mimir_b200.config.schema import load_config
    from mimir_b200.scheduling.store import Store
    from mimir_b200.train.setup import model_config_dict

    output, data, tokenizer, template = (Path(p).absolute() for p in (output, data, tokenizer, template))
    if output.exists():
        raise FileExistsError(f"{output}: use a fresh preparation directory")
    recipe = Recipe.load(recipe)
    steps = recipe.eval_steps(eval_steps)
    gpu_ids = [] if gpus is None else gpus.split(",")
    if gpus is not None and (not gpu_ids or not all(g.isdigit() for g in gpu_ids) or len(set(gpu_ids)) != len(gpu_ids)):
        raise ValueError("GPU assignment must be distinct numeric indices")
    corpus = inspect_corpus(data)
    meta = corpus["metadata"]
    if meta["total_length"] < recipe.steps * recipe.batch_tokens:
        raise ValueError("One epoch holds fewer tokens than the training budget")
    output.mkdir(parents=True)
    tok_dir = output / "tokenizer"
    corpus["tokenizer"] = _copy_tokenizer(tokenizer, template, tok_dir, meta["tokenizer_info"]["vocab_size"])
    _write(output / "data.json", corpus)

    resources = [f"gpu:{g}" for g in gpu_ids] or ["gpu:UNASSIGNED"]
    env = {"CUDA_VISIBLE_DEVICES": ",".join(gpu_ids), "MIMIR_WANDB": "0", "HF_HOME": str(output / "cache" / "huggingface")}
    plan, counts, before = _Plan(), {}, []
    for variant, extra in recipe.variants.items():
        run = output / "runs" / variant
        ckpts = run / "checkpoints"
        common = recipe.common_overrides + extra + [f"data.path={data}", f"checkpoint_path={ckpts}",
                                                    f"run_name={recipe.id}-{variant}"]
        config = load_config(common)
        metadata = {"vocab_size": meta["tokenizer_info"]["vocab_size"], "max_seq_len": meta["max_seq_len"] - 1}
        counts[variant] = count_parameters(model_config_dict(config, metadata))
        _write(output / "configs" / f"{variant}.json", config.model_dump(mode="json"))
        _write(output / "configs" / f"{variant}.overrides.json", common)
        previous_step, previous_train, evals = 0, None, []
        for step in steps:
            base = f"{variant}.step_{step}"
            overrides = common + [f"stop_after_step={step}"]
            depends = [(e, "terminal") for e in (evals if previous_step else before)]
            if previous_step:
                overrides += [f"resume_checkpoint_path={ckpts}", f"resume_checkpoint_tag=step_{previous_step}"]
                depends.append((previous_train, "success"))
            command = [python, "-m", "torch.distributed.run", "--standalone", f"--nproc_per_node={len(gpu_ids) or 1}",
                       "--module", "mimir_b200", "train", *overrides]
            train = plan.add(base + ".train", "train", {"command": command, "env": env, "resources": resources,
                                                         "progress_file": str(ckpts / "progress.json")}, depends)
            ckpt = plan.add(base + ".checkpoint", "checkpoint_wait", {"path": str(ckpts / f"step_{step}"), "timeout": 60},
                            [(train, "success")])
            exported = run / "exports" / f"step_{step}"
            export = plan.add(base + ".export", "export",
                              {"command": [python, "-m", "mimir_b200", "export", str(ckpts / f"step_{step}"),
                                           str(exported), "--tokenizer", str(tok_dir)],
                               "env": env | {"CUDA_VISIBLE_DEVICES": ""}}, [(ckpt, "success")])
            evals = []
            for suite in recipe.suites:
                source, tasks = _suite_tasks(suite)
                inputs, expected, suite_evals = [], {}, []
                for task in tasks:
                    tid = task["id"]
                    task_suite = output / "suites" / f"{suite}.{tid}.json"
                    _write(task_suite, {"schema": 1, "id": f"{suite}.{tid}", "source_sha256": _sha256(source),
                                        "tasks": [task]})
                    result = run / "eval" / f"step_{step}" / suite / tid
                    gpu = gpu_ids[len(evals) % len(gpu_ids)] if gpu_ids else ""
                    e = plan.add(f"{base}.{suite}.{tid}", "eval",
                                 {"evaluation": {"suite": str(task_suite), "model": str(exported), "output": str(result)},
                                  "server": {"model": str(exported), "gpus": gpu, "port": 8100 + int(gpu or 0),
                                             "eager": False, "max_model_len": meta["max_seq_len"] - 1},
                                  "controls": {"max_connections": 4},
                                  "resources": [f"gpu:{gpu}"] if gpu else resources}, [(export, "success")])
                    evals.append(e)
                    suite_evals.append(e)
                    if task.get("backend") == "inspect":
                        inputs.append(str(result / f"{tid}.samples.jsonl"))
                        expected[task.get("aggregate_task", tid)] = {
                            "samples": len(task.get("sample_ids", [])) or task["samples"], "passes": task["passes"]}
                if inputs:  # per-task records; no scalar mean across unlike benchmarks
                    plan.add(f"{base}.{suite}.merge", "merge",
                             {"inputs": inputs, "expected": expected,
                              "output": str(run / "metrics" / f"step_{step}.{suite}.json")},
                             [(e, "success") for e in suite_evals])
            previous_step, previous_train = step, train
        before = evals
    _check_capacity(recipe, counts)

    database = Path(database or Path(tempfile.mkdtemp(prefix=f"mimir-{recipe.id}-")) / "queue.sqlite").absolute()
    if database.exists():
        raise FileExistsError(database)
    store = Store(database)
    for job in plan.jobs:
        store.add(job["id"], job["kind"], job["config"], [(d["id"], d["policy"]) for d in job["depends"]],
                  job["max_attempts"], held=True)
    store.backup(output / "queue.backup.sqlite")
    rows = store.rows()
    if not all(r["state"] == "pending" and r["held"] and r["attempt"] == 0 for r in rows):
        raise RuntimeError("A prepared job is not pending and held")
    _write(output / "plan.json", {"schema": 1, "id": recipe.id, "jobs": plan.jobs})
    _write(output / "scheduled-plan.json", {"schema": 1, "id": recipe.id, "jobs": plan.jobs})
    _write(output / "parameters.json", counts)
    _write(output / "preparation.json", {
        "status": "prepared_not_started", "recipe": str(recipe.path), "recipe_sha256": _sha256(recipe.path),
        "database": str(database), "jobs": len(plan.jobs), "held_jobs": len(rows), "attempts": 0,
        "gpu_assignment": gpu_ids, "eval_steps": steps, "steps_per_variant": recipe.steps,
        "global_batch_tokens": recipe.batch_tokens, "token_budget_per_variant": recipe.steps * recipe.batch_tokens,
        "training_order": list(recipe.variants), "python": python,
        "notes": ["capacity-matched, not FLOP-matched", "the live queue must be on local disk; "
                  "queue.backup.sqlite is a snapshot"]})
    return output


def _check_capacity(recipe: Recipe, counts: dict) -> None:
    """Every variant's capacity relative to the baseline; with a target, the non-baseline variants
    must lie within the tolerance of ``ratio`` x the baseline."""
    target = recipe.capacity_target or {}
    base_name = target.get("baseline", next(iter(counts)))
    base = counts[base_name]["capacity"]
    for name, c in counts.items():
        c["ratio_to_baseline"] = c["capacity"] / base
        if target and name != base_name:
            c["difference_from_target_percent"] = (c["capacity"] / (target["ratio"] * base) - 1) * 100
            if abs(c["difference_from_target_percent"]) > target["tolerance_percent"]:
                raise ValueError(f"{name}: capacity {c['capacity']} is not within {target['tolerance_percent']}% of "
                                 f"{target['ratio']} x {base_name}")


def extend(output, *, extensions=RECIPES / "xxs-dfm15-20k.extensions.json", release: bool = False) -> int:
    """Append the variants of ``extensions`` to a prepared campaign.  Each new variant copies the
    jobs of its source variant (final-step-only preparations), with its own run directory, run
    name and extra overrides; it trains after the previous variant's evaluations.  Returns the
    number of jobs added (held unless ``release``)."""
    from mimir_b200.config.schema import load_config
    from mimir_b200.scheduling.store import Store
    output = Path(output).absolute()
    spec = json.loads(Path(extensions).read_text())
    if spec.get("schema") != 1:
        raise ValueError("unsupported extension schema")
    plan = json.loads((output / "scheduled-plan.json").read_text())
    receipt = json.loads((output / "preparation.json").read_text())
    store = Store(receipt["database"])
    queued = {r["id"] for r in store.rows()}
    added, previous = [], spec["after"]
    for name, variant in spec["variants"].items():
        source = variant["source"]
        templates = [j for j in plan["jobs"] if j["id"].startswith(source + ".")]
        if not templates:
            raise ValueError(f"no prepared jobs for source variant {source!r}")
        if sum(j["kind"] == "train" for j in templates) != 1:
            raise ValueError("extensions need final-step-only preparations (one training job per variant)")
        if any(q.startswith(name + ".") for q in queued):
            raise ValueError(f"{name!r} is already queued")

        def rename(text: str) -> str:
            return (text.replace(f"/runs/{source}/", f"/runs/{name}/")
                    .replace(f"run_name={plan["id"]}-{source}", f"run_name={plan["id"]}-{name}"))
        base_overrides = json.loads((output / "configs" / f"{source}.overrides.json").read_text())
        overrides = [rename(o) for o in base_overrides] + variant["overrides"]
        _write(output / "configs" / f"{name}.json", load_config(overrides).model_dump(mode="json"))
        _write(output / "configs" / f"{name}.overrides.json", overrides)
        for template in templates:
            job = json.loads(rename(json.dumps(template)))
            job["id"] = name + template["id"][len(source):]
            job["held"] = True
            for d in job["depends"]:
                if d["id"].startswith(source + "."):
                    d["id"] = name + d["id"][len(source):]
            if job["kind"] == "train":
                job["config"]["command"] += variant["overrides"]
                job["depends"] = [{"id": j["id"], "policy": "terminal"} for j in plan["jobs"] + added
                                  if j["id"].startswith(previous + ".") and j["kind"] == "eval"]
            added.append(job)
        previous = name
    for job in added:  # every config validated above before the first insertion
        store.add(job["id"], job["kind"], job["config"], [(d["id"], d["policy"]) for d in job["depends"]],
                  job["max_attempts"], held=True)
    if release:
        for job in added:
            store.hold(job["id"], False)
            job["held"] = False
    plan["jobs"] += added
    _write(output / "scheduled-plan.json", plan)
    _write(output / "extension-plan.json", {"jobs": added})
    store.backup(output / f"queue.extended.{len(plan['jobs'])}.backup.sqlite")
    receipt["training_order"] = receipt.get("training_order", []) + list(spec["variants"])
    rows = store.rows()
    receipt["jobs"], receipt["held_jobs"] = len(rows), sum(bool(r["held"]) for r in rows)
    _write(output / "preparation.json", receipt)
    return len(added)
