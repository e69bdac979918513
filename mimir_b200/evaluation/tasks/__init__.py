"""Evaluation task registry: dataset loader + prompt + scorer per task, runnable without Inspect AI.

The reference defines its tasks as Inspect AI modules (``src/mimir/evaluation/tasks/*.py``).
Here a task is a plain :class:`TaskSpec`; the direct runner (``evaluation/runner.py``) drives
any OpenAI-compatible endpoint with it, and ``inspect_task()`` adapts a spec to Inspect AI
when that package is installed.  Datasets are local files (no network): each task reads the
path given by its ``dataset_path`` argument or its environment variable.

Families:

* multiple choice (letter answer, optional partial credit ``1/choices`` for unparseable
  answers): ``hellaswag_da``, ``piqa``, ``mmlu``, ``winogrande``, ``boolq_5shot``;
* classification (label words, macro-F1/MCC through ``target_class``/``predicted_class``):
  ``angry_tweets``, ``dala``;
* generation scored by chrF3++: ``wmt24pp``, ``andersen_modernize``, ``gec_dala``,
  ``nordjylland_news_summarization``;
* extractive QA (exact match + token F1): ``multi_wiki_qa``;
* ``smoke``: one fixed sample for wiring tests;
* the comparison suites' tasks (``tasks/comparison.py``): ``arc_25shot``, ``mmlu_5shot`` and
  ``hellaswag_ie_fmt`` / ``math_ie`` in chunks, ``drop``, ``gsm8k``, ``winogrande_ie``,
  ``govreport_summarization``, ``humaneval_ie`` (execution), ``daisy``, ``ifeval_da``
  (``tasks/ifeval.py``), ``wmt24pp_en_da``.
"""
from __future__ import annotations

import json
import os
import random
import re
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Optional

REGISTRY: dict[str, Callable[..., "TaskSpec"]] = {}


@dataclass
class TaskSpec:
    name: str
    samples: list[dict]                       # {"id", "messages", "target", "metadata"}
    score: Callable[[str, dict], dict]        # (completion, sample) -> row fields ("scores", ...)
    generation: dict = field(default_factory=lambda: {"temperature": 0.0, "max_tokens": 16})


def register(name: str):
    def wrap(fn):
        REGISTRY[name] = fn
        return fn
    return wrap


def build(name: str, **kwargs) -> TaskSpec:
    if name not in REGISTRY:
        raise ValueError(f"Unknown task {name!r}; registered: {sorted(REGISTRY)}")
    return REGISTRY[name](**kwargs)


# ------------------------------------------------------------------------------ loading
def load_records(dataset_path, env: str) -> list[dict]:
    path = Path(dataset_path or os.environ.get(env, ""))
    if not str(path) or not path.is_file():
        raise FileNotFoundError(f"Dataset not found; pass dataset_path or set {env}")
    if path.suffix == ".parquet":
        import pyarrow.parquet as pq
        return pq.read_table(path).to_pylist()
    if path.suffix == ".jsonl":
        return [json.loads(line) for line in path.read_text().splitlines() if line.strip()]
    data = json.loads(path.read_text())
    return data if isinstance(data, list) else data["records"]


def _select(records: list, shuffle_seed: Optional[int], limit: Optional[int]) -> list:
    records = list(records)
    if shuffle_seed is not None:
        random.Random(shuffle_seed).shuffle(records)
    return records[:limit] if limit is not None else records


def _user(text: str) -> list[dict]:
    return [{"role": "user", "content": text}]


# ------------------------------------------------------------------------------ scorers
def letter_scorer(letters: str, partial_credit: bool):
    pattern = re.compile(rf"^\s*\(?([{letters}{letters.lower()}])\b")

    def score(completion: str, sample: dict) -> dict:
        m = pattern.search(completion)
        pred = m.group(1).upper() if m else None
        if pred is None:
            value = 1.0 / len(letters) if partial_credit else 0.0
        else:
            value = float(pred == sample["target"].upper())
        return {"scores": {"accuracy": value}, "answer": pred}
    return score


def label_scorer(labels: list[str]):
    def score(completion: str, sample: dict) -> dict:
        text = completion.strip().lower()
        pred = next((lab for lab in labels if text.startswith(lab)), None)
        if pred is None:
            pred = next((lab for lab in labels if lab in text), "<invalid>")
        return {"scores": {"accuracy": float(pred == sample["target"])}, "target_class": sample["target"],
                "predicted_class": pred}
    return score


def chrf_scorer(completion: str, sample: dict) -> dict:
    from mimir_b200.evaluation.scorers.chrf import compute_chrf3pp
    refs = sample["target"] if isinstance(sample["target"], list) else [sample["target"]]
    return {"scores": {"chrf3pp": compute_chrf3pp(completion.strip(), refs)}}


def _norm_tokens(text: str) -> list[str]:
    return re.sub(r"[^\w\s]", " ", text.lower()).split()


def qa_scorer(completion: str, sample: dict) -> dict:
    pred = _norm_tokens(completion)
    best_em, best_f1 = 0.0, 0.0
    for ans in (sample["target"] if isinstance(sample["target"], list) else [sample["target"]]):
        gold = _norm_tokens(ans)
        best_em = max(best_em, float(pred == gold))
        common = sum((__import__("collections").Counter(pred) & __import__("collections").Counter(gold)).values())
        if common:
            p, r = common / len(pred), common / len(gold)
            best_f1 = max(best_f1, 2 * p * r / (p + r))
    return {"scores": {"exact_match": best_em, "f1": best_f1}}


# ------------------------------------------------------------------------------ tasks
@register("smoke")
def smoke(**_):
    return TaskSpec("smoke", [{"id": "a", "messages": _user("Return the test response."),
                               "target": "Default output from mockllm/model", "metadata": {}}],
                    lambda c, s: {"scores": {"exact": float(c.strip() == s["target"])}})


def _mcq(name, env, prompt_fn, letters, partial, *, dataset_path=None, shuffle_seed=None, limit=None,
         max_tokens=8):
    recs = _select(load_records(dataset_path, env), shuffle_seed, limit)
    samples = [{"id": r.get("id", i), "messages": _user(prompt_fn(r)), "target": _mcq_target(r, letters),
                "metadata": {}} for i, r in enumerate(recs)]
    return TaskSpec(name, samples, letter_scorer(letters, partial), {"temperature": 0.0, "max_tokens": max_tokens})


def _mcq_target(record: dict, letters: str) -> str:
    label = record.get("label", record.get("answer"))
    if isinstance(label, int) or (isinstance(label, str) and label.isdigit()):
        return letters[int(label)]
    return str(label).upper()


@register("hellaswag_da")
def hellaswag_da(**kw):
    return _mcq("hellaswag_da", "HELLASWAG_DA_PATH",
                lambda r: f"{r['text']}\n\nSvar kun med ét bogstav: a, b, c eller d.\nSvar:", "ABCD", True, **kw)


@register("piqa")
def piqa(**kw):
    def prompt(r):
        return ("Vælg den løsning, der bedst opnår målet.\n\n"
                f"Mål: {r['prompt']}\nA: {r['solution0']}\nB: {r['solution1']}\n\nSvar kun med A eller B.")
    return _mcq("piqa", "PIQA_DA_PATH", prompt, "AB", False, **kw)


@register("mmlu")
def mmlu(**kw):
    def prompt(r):
        opts = "\n".join(f"{'ABCD'[i]}. {c}" for i, c in enumerate(r["choices"]))
        return f"{r['question']}\n{opts}\n\nAnswer with the letter of the correct option only."
    return _mcq("mmlu", "MMLU_PATH", prompt, "ABCD", False, **kw)


@register("winogrande")
def winogrande(**kw):
    def prompt(r):
        return (f"Fill in the blank (_) in the sentence.\n\n{r['sentence']}\nA: {r['option1']}\nB: {r['option2']}"
                "\n\nAnswer with A or B only.")
    return _mcq("winogrande", "WINOGRANDE_PATH", prompt, "AB", False, **kw)


@register("boolq_5shot")
def boolq_5shot(**kw):
    def prompt(r):
        return f"{r['passage']}\nQuestion: {r['question']}?\nA: yes\nB: no\nAnswer with A or B only."
    spec = _mcq("boolq_5shot", "BOOLQ_PATH", prompt, "AB", False, max_tokens=1, **kw)
    for s in spec.samples:  # boolean labels: True -> A (yes), False -> B (no)
        s["target"] = "A" if s["target"] in ("TRUE", "1", "A") else "B"
    return spec


def _classification(name, env, prompt_fn, labels, *, dataset_path=None, shuffle_seed=None, limit=None):
    recs = _select(load_records(dataset_path, env), shuffle_seed, limit)
    samples = [{"id": r.get("id", i), "messages": _user(prompt_fn(r)), "target": str(r["label"]).lower(),
                "metadata": {}} for i, r in enumerate(recs)]
    return TaskSpec(name, samples, label_scorer(labels), {"temperature": 0.0, "max_tokens": 8})


@register("angry_tweets")
def angry_tweets(**kw):
    return _classification("angry_tweets", "ANGRY_TWEETS_PATH",
                           lambda r: f"Tweet: {r['text']}\n\nEr stemningen positiv, neutral eller negativ? "
                                     "Svar med ét ord.", ["positiv", "neutral", "negativ"], **kw)


@register("dala")
def dala(**kw):
    return _classification("dala", "DALA_PATH",
                           lambda r: f"Sætning: {r['text']}\n\nEr sætningen grammatisk korrekt? Svar ja eller nej.",
                           ["ja", "nej"], **kw)


def _generation(name, env, prompt_fn, target_key, scorer, *, dataset_path=None, shuffle_seed=None, limit=None,
                max_tokens=512):
    recs = _select(load_records(dataset_path, env), shuffle_seed, limit)
    samples = [{"id": r.get("id", i), "messages": _user(prompt_fn(r)), "target": r[target_key], "metadata": {}}
               for i, r in enumerate(recs)]
    return TaskSpec(name, samples, scorer, {"temperature": 0.0, "max_tokens": max_tokens})


@register("wmt24pp")
def wmt24pp(source_language="English", target_language="Danish", **kw):
    return _generation("wmt24pp", "WMT24PP_PATH",
                       lambda r: f"Translate the following {source_language} text into {target_language}. "
                                 f"Reply with the translation only.\n\n{r['source']}", "target", chrf_scorer, **kw)


@register("andersen_modernize")
def andersen_modernize(**kw):
    return _generation("andersen_modernize", "ANDERSEN_PATH",
                       lambda r: f"Omskriv teksten til moderne dansk. Svar kun med den omskrevne tekst.\n\n{r['source']}",
                       "target", chrf_scorer, **kw)


@register("gec_dala")
def gec_dala(**kw):
    return _generation("gec_dala", "GEC_DALA_PATH",
                       lambda r: f"Ret eventuelle grammatiske fejl. Svar kun med den rettede sætning.\n\n{r['text']}",
                       "corrected", chrf_scorer, max_tokens=256, **kw)


@register("nordjylland_news_summarization")
def nordjylland_news_summarization(**kw):
    return _generation("nordjylland_news_summarization", "NORDJYLLAND_NEWS_PATH",
                       lambda r: f"Skriv et kort resumé af artiklen.\n\n{r['text']}", "summary", chrf_scorer,
                       max_tokens=256, **kw)


@register("multi_wiki_qa")
def multi_wiki_qa(**kw):
    return _generation("multi_wiki_qa", "MULTI_WIKI_QA_PATH",
                       lambda r: f"Tekst: {r['context']}\n\nSpørgsmål: {r['question']}\n"
                                 "Svar med et kort uddrag fra teksten.", "answers", qa_scorer, max_tokens=64, **kw)


def inspect_task(spec: TaskSpec):
    """Adapt a spec to an Inspect AI ``Task`` (requires ``inspect_ai``)."""
    from inspect_ai import Task
    from inspect_ai.dataset import MemoryDataset, Sample
    from inspect_ai.scorer import Score, mean, scorer
    from inspect_ai.solver import generate

    @scorer(metrics=[mean()])
    def spec_scorer():
        async def score(state, target):
            sample = {"target": state.metadata["target"]}
            out = spec.score(state.output.completion, sample)
            return Score(value=next(iter(out["scores"].values())), answer=state.output.completion)
        return score

    samples = [Sample(id=s["id"], input=s["messages"][-1]["content"],
                      target=s["target"] if isinstance(s["target"], str) else s["target"][0],
                      metadata={"target": s["target"]}) for s in spec.samples]
    return Task(dataset=MemoryDataset(samples, name=spec.name), solver=generate(), scorer=spec_scorer())


from mimir_b200.evaluation.tasks import comparison  # noqa: E402,F401  (registers the comparison-suite tasks)
