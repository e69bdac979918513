"""Tasks of the comparison suites (``comparison-inspect-v1``, ``comparison-danish-v1``): few-shot
and chunked English benchmarks, maths and code with answer extraction, Danish QA and
instruction following.

Reference behaviour (task sets, answer formats, metrics): ``src/mimir/evaluation/tasks/``
``custom_english_tasks.py`` (ARC 25-shot, GovReport), ``mmlu_winogrande_tasks.py`` (MMLU 5-shot
in chunks, "nothink"), ``hellaswag_ie_fmt_task.py`` (HellaSwag with an "ANSWER: X" format, in
chunks), ``math_humaneval_tasks.py`` (MATH with "ANSWER:" / ``\\boxed{}`` extraction in chunks,
HumanEval with execution), ``daisy.py`` (exact match, token F1, sentence BLEU), ``ifeval_da.py``
and the Inspect ``drop`` / ``gsm8k`` / ``winogrande`` evals.  Prompts, extraction and scoring
here are this framework's own; datasets are local files (records listed per task below).

Chunking: ``chunk`` / ``chunks`` select the ``chunk``-th of ``chunks`` contiguous slices of the
dataset (the suites split the long benchmarks so that one job stays short).  Few-shot: exemplars
come from ``fewshot_path`` (or the task's ``*_FEWSHOT_PATH`` variable), the first ``shots``
records, rendered as earlier user/assistant turns.
"""
from __future__ import annotations

import math
import os
import re
import subprocess
import sys
import tempfile
from collections import Counter
from fractions import Fraction
from typing import Optional

from mimir_b200.evaluation.tasks import (TaskSpec, _mcq_target, _select, _user, chrf_scorer, load_records,
                                         register)
from mimir_b200.evaluation.tasks.ifeval import ifeval_scorer, normalise_kwargs


# ------------------------------------------------------------------------------ selection helpers
def _chunk(records: list, chunk: Optional[int], chunks: Optional[int]) -> list:
    if chunks is None:
        return records
    if not 0 <= (chunk or 0) < chunks:
        raise ValueError(f"chunk must be in [0, {chunks})")
    size = math.ceil(len(records) / chunks)
    return records[(chunk or 0) * size:((chunk or 0) + 1) * size]


def _records(env, dataset_path, shuffle_seed, limit, chunk=None, chunks=None) -> list:
    return _select(_chunk(load_records(dataset_path, env), chunk, chunks), shuffle_seed, limit)


def _shots(env: str, fewshot_path, shots: int) -> list:
    if shots <= 0:
        return []
    pool = load_records(fewshot_path, env)
    if len(pool) < shots:
        raise ValueError(f"{shots}-shot prompt needs {shots} exemplars, found {len(pool)}")
    return pool[:shots]


def _dialogue(exemplars: list[tuple[str, str]], question: str) -> list[dict]:
    turns = []
    for q, a in exemplars:
        turns += [{"role": "user", "content": q}, {"role": "assistant", "content": a}]
    return turns + [{"role": "user", "content": question}]


# ------------------------------------------------------------------------------ answer extraction
_ANSWER_TAG = re.compile(r"ANSWER\s*:\s*(.+)", re.I)


def answer_tag(text: str) -> Optional[str]:
    """The text after the last ``ANSWER:`` tag, up to the end of its line."""
    found = _ANSWER_TAG.findall(text)
    return found[-1].strip().split("\n")[0].strip() if found else None


def last_boxed(text: str) -> Optional[str]:
    """Content of the last ``\\boxed{...}`` (balanced braces), or None."""
    start = text.rfind("\\boxed")
    if start < 0:
        return None
    i = text.find("{", start)
    if i < 0:
        return None
    depth = 0
    for j in range(i, len(text)):
        depth += {"{": 1, "}": -1}.get(text[j], 0)
        if depth == 0:
            return text[i + 1:j]
    return None


def _letter_after_tag(letters: str):
    def score(completion: str, sample: dict) -> dict:
        tagged = answer_tag(completion)
        source = tagged if tagged is not None else completion
        m = re.search(rf"\b([{letters}])\b", source.upper())
        pred = m.group(1) if m else None
        return {"scores": {"accuracy": float(pred == sample["target"])}, "answer": pred}
    return score


# ------------------------------------------------------------------------------ maths
def _strip_math(s: str) -> str:
    s = s.strip().strip("$").strip()
    for a, b in (("\\left", ""), ("\\right", ""), ("\\!", ""), ("\\,", ""), ("\\;", ""), ("\\ ", ""),
                 ("dfrac", "frac"), ("tfrac", "frac"), ("^\\circ", ""), ("^{\\circ}", ""), ("\\%", ""), ("%", ""),
                 ("\\$", ""), ("\\text{", "{"), ("\\mbox{", "{")):
        s = s.replace(a, b)
    s = re.sub(r"\s+", "", s).rstrip(".")
    s = re.sub(r"\\frac(\d)(\d)", r"\\frac{\1}{\2}", s)
    s = re.sub(r"^\{(.*)\}$", r"\1", s)
    if re.fullmatch(r"-?\d+\.0+", s):
        s = s.split(".")[0]
    return s


def _as_number(s: str) -> Optional[Fraction]:
    s = s.replace(",", "")
    m = re.fullmatch(r"\\frac\{(-?\d+)\}\{(-?\d+)\}", s) or re.fullmatch(r"(-?\d+)/(-?\d+)", s)
    try:
        if m:
            return Fraction(int(m.group(1)), int(m.group(2)))
        return Fraction(s) if re.fullmatch(r"-?\d+(\.\d+)?", s) else None
    except (ValueError, ZeroDivisionError):
        return None


def math_equal(prediction: str, target: str) -> bool:
    """Normalised string equality, or equality as exact rationals when both read as numbers."""
    p, t = _strip_math(prediction), _strip_math(target)
    if p == t:
        return True
    a, b = _as_number(p), _as_number(t)
    return a is not None and a == b


def math_scorer(completion: str, sample: dict) -> dict:
    pred = answer_tag(completion)
    if pred is None:
        pred = last_boxed(completion)
    if pred is not None and "\\boxed" in pred:
        pred = last_boxed(pred) or pred
    return {"scores": {"accuracy": float(pred is not None and math_equal(pred, sample["target"]))}, "answer": pred}


_NUMBER = re.compile(r"-?\d[\d,]*(?:\.\d+)?")


def gsm8k_scorer(completion: str, sample: dict) -> dict:
    tagged = answer_tag(completion)
    numbers = _NUMBER.findall(tagged if tagged is not None else completion)
    pred = numbers[-1].replace(",", "").rstrip(".") if numbers else None
    target = str(sample["target"]).split("####")[-1].strip().replace(",", "")
    ok = pred is not None and _as_number(pred) is not None and _as_number(pred) == _as_number(target)
    return {"scores": {"accuracy": float(ok)}, "answer": pred}


# ------------------------------------------------------------------------------ text overlap metrics
def _normalise(text: str) -> str:
    text = text.lower()
    text = re.sub(r"\b(a|an|the)\b", " ", text)
    return " ".join(re.sub(r"[^\w\s]", " ", text).split())


def token_f1(prediction: str, gold: str) -> float:
    p, g = _normalise(prediction).split(), _normalise(gold).split()
    if not p or not g:
        return float(p == g)
    common = sum((Counter(p) & Counter(g)).values())
    if not common:
        return 0.0
    precision, recall = common / len(p), common / len(g)
    return 2 * precision * recall / (precision + recall)


def sentence_bleu(prediction: str, references: list[str], max_order: int = 4) -> float:
    """BLEU of one hypothesis (Papineni et al. 2002) with add-one smoothing of the n-gram
    precisions above unigrams and the closest-reference brevity penalty."""
    hyp = _normalise(prediction).split()
    refs = [_normalise(r).split() for r in references]
    if not hyp or not any(refs):
        return 0.0
    log_p = 0.0
    for n in range(1, max_order + 1):
        grams = Counter(tuple(hyp[i:i + n]) for i in range(len(hyp) - n + 1))
        best: Counter = Counter()
        for r in refs:
            best |= Counter(tuple(r[i:i + n]) for i in range(len(r) - n + 1))
        matched = sum(min(c, best[g]) for g, c in grams.items())
        total = max(len(hyp) - n + 1, 0)
        num, den = (matched, total) if n == 1 else (matched + 1, total + 1)
        if num == 0 or den == 0:
            return 0.0
        log_p += math.log(num / den) / max_order
    closest = min((abs(len(r) - len(hyp)), len(r)) for r in refs)[1]
    bp = 1.0 if len(hyp) > closest else math.exp(1 - closest / len(hyp))
    return bp * math.exp(log_p)


def rouge_l(prediction: str, reference: str) -> float:
    """ROUGE-L F1 over normalised tokens (longest common subsequence)."""
    a, b = _normalise(prediction).split(), _normalise(reference).split()
    if not a or not b:
        return 0.0
    prev = [0] * (len(b) + 1)
    for x in a:
        cur = [0]
        for j, y in enumerate(b):
            cur.append(prev[j] + 1 if x == y else max(prev[j + 1], cur[j]))
        prev = cur
    lcs = prev[-1]
    if not lcs:
        return 0.0
    p, r = lcs / len(a), lcs / len(b)
    return 2 * p * r / (p + r)


def qa_overlap_scorer(completion: str, sample: dict) -> dict:
    refs = sample["target"] if isinstance(sample["target"], list) else [sample["target"]]
    pred = completion.strip().split("\n")[0]
    return {"scores": {"exact_match": max(float(_normalise(pred) == _normalise(r)) for r in refs),
                       "f1": max(token_f1(pred, r) for r in refs), "bleu": sentence_bleu(pred, refs)}}


def _drop_numbers(text: str) -> str:
    """DROP-style normalisation: numbers written the same way compare equal (1,000 == 1000.0)."""
    out = []
    for tok in _normalise(text.replace(",", "")).split():
        try:
            out.append(str(float(tok)))
        except ValueError:
            out.append(tok)
    return " ".join(out)


def drop_scorer(completion: str, sample: dict) -> dict:
    tagged = answer_tag(completion)
    pred = (tagged if tagged is not None else completion.strip().split("\n")[0]).strip()
    refs = sample["target"] if isinstance(sample["target"], list) else [sample["target"]]
    em = max(float(_drop_numbers(pred) == _drop_numbers(r)) for r in refs)
    f1 = max(token_f1(_drop_numbers(pred), _drop_numbers(r)) for r in refs)
    return {"scores": {"exact_match": em, "f1": f1}, "answer": pred}


# ------------------------------------------------------------------------------ code
def extract_code(completion: str) -> str:
    fenced = re.findall(r"```(?:python|py)?\n(.*?)```", completion, re.S)
    return fenced[0] if fenced else completion


def run_humaneval(program: str, timeout: float = 10.0) -> bool:
    """Run ``program`` in a separate isolated Python process with a time limit, in an empty
    temporary directory and without inherited environment secrets; True when it exits 0."""
    with tempfile.TemporaryDirectory() as work:
        path = os.path.join(work, "candidate.py")
        with open(path, "w") as f:
            f.write(program)
        env = {"PATH": os.environ.get("PATH", ""), "PYTHONHASHSEED": "0", "HOME": work}
        try:
            done = subprocess.run([sys.executable, "-I", path], cwd=work, env=env, stdin=subprocess.DEVNULL,
                                  stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL, timeout=timeout)
        except subprocess.TimeoutExpired:
            return False
        return done.returncode == 0


def humaneval_scorer(completion: str, sample: dict) -> dict:
    meta = sample["metadata"]
    code = extract_code(completion)
    body = code if re.search(rf"def\s+{re.escape(meta['entry_point'])}\s*\(", code) else meta["prompt"] + code
    program = f"{body}\n\n{meta['test']}\n\ncheck({meta['entry_point']})\n"
    return {"scores": {"pass": float(run_humaneval(program))}}


# ------------------------------------------------------------------------------ English tasks
def _mc_question(r: dict, letters: str) -> str:
    choices = r["choices"]
    texts = choices["text"] if isinstance(choices, dict) else choices
    return r["question"] + "\n" + "\n".join(f"{letters[i]}. {t}" for i, t in enumerate(texts))


def _arc_target(r: dict) -> str:
    key = str(r.get("answerKey", r.get("label")))
    labels = r["choices"].get("label") if isinstance(r["choices"], dict) else None
    if labels and key in labels:
        return "ABCDE"[labels.index(key)]
    return "ABCDE"[int(key) - 1] if key.isdigit() else key.upper()


@register("arc_25shot")
def arc_25shot(*, dataset_path=None, fewshot_path=None, shots=25, shuffle_seed=None, limit=None, **_):
    """ARC-Challenge with 25 exemplars; records ``question``, ``choices{text,label}``, ``answerKey``."""
    tail = "\n\nAnswer with the letter of the correct option only."
    ex = [(_mc_question(r, "ABCDE") + tail, _arc_target(r)) for r in _shots("ARC_FEWSHOT_PATH", fewshot_path, shots)]
    recs = _records("ARC_PATH", dataset_path, shuffle_seed, limit)
    samples = [{"id": r.get("id", i), "messages": _dialogue(ex, _mc_question(r, "ABCDE") + tail),
                "target": _arc_target(r), "metadata": {}} for i, r in enumerate(recs)]
    return TaskSpec("arc_25shot", samples, _letter_after_tag("ABCDE"), {"temperature": 0.0, "max_tokens": 4})


@register("mmlu_5shot")
def mmlu_5shot(*, dataset_path=None, fewshot_path=None, shots=5, chunk=None, chunks=None, shuffle_seed=None,
               limit=None, **_):
    """MMLU with 5 exemplars of the same subject, answer after ``ANSWER:``, thinking disabled in
    the chat template; records ``question``, ``choices``, ``answer``, ``subject``."""
    pool = load_records(fewshot_path, "MMLU_FEWSHOT_PATH") if shots > 0 else []
    tail = "\n\nThink briefly if needed, then finish with 'ANSWER: $LETTER'."
    recs = _records("MMLU_PATH", dataset_path, shuffle_seed, limit, chunk, chunks)
    samples = []
    for i, r in enumerate(recs):
        same = [p for p in pool if p.get("subject") == r.get("subject")][:shots]
        ex = [(_mc_question(p, "ABCD") + tail, f"ANSWER: {_mcq_target(p, 'ABCD')}") for p in same]
        samples.append({"id": r.get("id", i), "messages": _dialogue(ex, _mc_question(r, "ABCD") + tail),
                        "target": _mcq_target(r, "ABCD"), "metadata": {"subject": r.get("subject")}})
    name = "mmlu_5shot" if chunks is None else f"mmlu_5shot_chunk{chunk}_nothink"
    return TaskSpec(name, samples, _letter_after_tag("ABCD"),
                    {"temperature": 0.0, "max_tokens": 64, "chat_template_kwargs": {"enable_thinking": False}})


@register("hellaswag_ie_fmt")
def hellaswag_ie_fmt(*, dataset_path=None, chunk=None, chunks=None, shuffle_seed=None, limit=None, **_):
    """HellaSwag (English) with the answer after ``ANSWER:``; records ``ctx``, ``endings``, ``label``."""
    def prompt(r):
        opts = "\n".join(f"{'ABCD'[i]}. {e}" for i, e in enumerate(r["endings"]))
        return (f"Choose the most plausible continuation.\n\n{r['ctx']}\n{opts}\n\n"
                "Finish with 'ANSWER: $LETTER'.")
    recs = _records("HELLASWAG_PATH", dataset_path, shuffle_seed, limit, chunk, chunks)
    samples = [{"id": r.get("id", i), "messages": _user(prompt(r)), "target": "ABCD"[int(r["label"])],
                "metadata": {}} for i, r in enumerate(recs)]
    name = "hellaswag_ie_fmt" if chunks is None else f"hellaswag_ie_fmt_chunk{chunk}"
    return TaskSpec(name, samples, _letter_after_tag("ABCD"), {"temperature": 0.0, "max_tokens": 32})


@register("drop")
def drop(*, dataset_path=None, shuffle_seed=None, limit=None, **_):
    """DROP reading comprehension; records ``passage``, ``question``, ``answers`` (spans or numbers)."""
    recs = _records("DROP_PATH", dataset_path, shuffle_seed, limit)
    samples = [{"id": r.get("id", i),
                "messages": _user(f"{r['passage']}\n\nQuestion: {r['question']}\n"
                                  "Finish with 'ANSWER: $ANSWER' (a number, a date or a short span)."),
                "target": r["answers"] if isinstance(r["answers"], list) else [r["answers"]], "metadata": {}}
               for i, r in enumerate(recs)]
    return TaskSpec("drop", samples, drop_scorer, {"temperature": 0.0, "max_tokens": 128})


@register("gsm8k")
def gsm8k(*, dataset_path=None, shuffle_seed=None, limit=None, **_):
    """GSM8K; records ``question`` and ``answer`` (worked solution ending in ``#### N``)."""
    recs = _records("GSM8K_PATH", dataset_path, shuffle_seed, limit)
    samples = [{"id": r.get("id", i),
                "messages": _user(f"{r['question']}\n\nSolve step by step, then finish with 'ANSWER: $NUMBER'."),
                "target": r["answer"], "metadata": {}} for i, r in enumerate(recs)]
    return TaskSpec("gsm8k", samples, gsm8k_scorer, {"temperature": 0.0, "max_tokens": 512})


@register("winogrande_ie")
def winogrande_ie(*, dataset_path=None, shuffle_seed=None, limit=None, **_):
    """WinoGrande with the answer after ``ANSWER:``; records ``sentence``, ``option1/2``, ``answer``."""
    recs = _records("WINOGRANDE_PATH", dataset_path, shuffle_seed, limit)
    samples = [{"id": r.get("id", i),
                "messages": _user(f"Fill in the blank (_).\n\n{r['sentence']}\nA. {r['option1']}\nB. {r['option2']}"
                                  "\n\nFinish with 'ANSWER: $LETTER'."),
                "target": "AB"[int(r["answer"]) - 1], "metadata": {}} for i, r in enumerate(recs)]
    return TaskSpec("winogrande_ie", samples, _letter_after_tag("AB"), {"temperature": 0.0, "max_tokens": 32})


@register("govreport_summarization")
def govreport_summarization(*, dataset_path=None, shuffle_seed=None, limit=None, **_):
    """GovReport; records ``report`` and ``summary``; ROUGE-L and chrF3++."""
    recs = _records("GOVREPORT_PATH", dataset_path, shuffle_seed, limit)
    samples = [{"id": r.get("id", i), "messages": _user(f"Summarise the report.\n\n{r['report']}"),
                "target": r["summary"], "metadata": {}} for i, r in enumerate(recs)]

    def score(completion, sample):
        return {"scores": {"rouge_l": rouge_l(completion, sample["target"])} | chrf_scorer(completion, sample)["scores"]}
    return TaskSpec("govreport_summarization", samples, score, {"temperature": 0.0, "max_tokens": 1024})


@register("math_ie")
def math_ie(*, dataset_path=None, chunk=None, chunks=None, shuffle_seed=None, limit=None, **_):
    """MATH; records ``problem`` and ``answer`` (or ``solution`` with a ``\\boxed{}`` answer)."""
    recs = _records("MATH_PATH", dataset_path, shuffle_seed, limit, chunk, chunks)
    samples = []
    for i, r in enumerate(recs):
        target = r.get("answer") or last_boxed(r["solution"])
        samples.append({"id": r.get("id", i), "messages": _user(
            f"{r['problem']}\n\nSolve the problem, then finish with 'ANSWER: $ANSWER' (LaTeX allowed)."),
            "target": target, "metadata": {}})
    name = "math_ie" if chunks is None else f"math_ie_chunk{chunk}"
    return TaskSpec(name, samples, math_scorer, {"temperature": 0.0, "max_tokens": 2048})


@register("humaneval_ie")
def humaneval_ie(*, dataset_path=None, shuffle_seed=None, limit=None, **_):
    """HumanEval; records ``task_id``, ``prompt``, ``test``, ``entry_point``; pass@1 by execution."""
    recs = _records("HUMANEVAL_PATH", dataset_path, shuffle_seed, limit)
    samples = [{"id": r.get("task_id", i),
                "messages": _user("Complete the Python function. Reply with the code in one ```python block.\n\n"
                                  + r["prompt"]),
                "target": "", "metadata": {"prompt": r["prompt"], "test": r["test"], "entry_point": r["entry_point"]}}
               for i, r in enumerate(recs)]
    return TaskSpec("humaneval_ie", samples, humaneval_scorer, {"temperature": 0.0, "max_tokens": 768})


# ------------------------------------------------------------------------------ Danish tasks
@register("daisy")
def daisy(*, dataset_path=None, shuffle_seed=None, limit=None, **_):
    """Danish factual QA; records ``Question`` and ``Answer`` (or a list); exact match, F1, BLEU."""
    rules = ("Besvar spørgsmålet kort og direkte på dansk, uden forklaring. Højder i meter, vægt i kilogram, "
             "størrelser i centimeter; personer som de normalt nævnes i danske tekster.")
    recs = _records("DAISY_PATH", dataset_path, shuffle_seed, limit)
    samples = [{"id": r.get("id", i), "messages": _user(f"{rules}\n\nSpørgsmål: {r['Question']}\nSvar:"),
                "target": r["Answer"] if isinstance(r["Answer"], list) else [r["Answer"]], "metadata": {}}
               for i, r in enumerate(recs)]
    return TaskSpec("daisy", samples, qa_overlap_scorer, {"temperature": 0.0, "max_tokens": 100})


@register("ifeval_da")
def ifeval_da(*, dataset_path=None, shuffle_seed=None, limit=None, **_):
    """Danish IFEval; records ``prompt``, ``instruction_id_list``, ``kwargs``."""
    recs = _records("IFEVAL_DA_PATH", dataset_path, shuffle_seed, limit)
    samples = [{"id": r.get("key", r.get("id", i)), "messages": _user(r["prompt"]), "target": "",
                "metadata": {"instruction_id_list": list(r["instruction_id_list"]), "kwargs": normalise_kwargs(r)}}
               for i, r in enumerate(recs)]
    return TaskSpec("ifeval_da", samples, ifeval_scorer, {"temperature": 0.0, "max_tokens": 1280})


@register("wmt24pp_en_da")
def wmt24pp_en_da(**kw):
    from mimir_b200.evaluation.tasks import REGISTRY
    spec = REGISTRY["wmt24pp"](source_language="English", target_language="Danish", **kw)
    spec.name = "wmt24pp_en_da"
    return spec
