"""Comparison-suite evaluation tasks: answer extraction, scoring, execution, instruction checks,
chunking, and that every suite entry resolves to a registered task (CPU, no network)."""
import json
from pathlib import Path

import pytest

from mimir_b200.evaluation.tasks import REGISTRY, build
from mimir_b200.evaluation.tasks import comparison as C
from mimir_b200.evaluation.tasks.ifeval import follows, ifeval_scorer

SUITES = Path(__file__).resolve().parents[1] / "mimir_b200" / "evaluation" / "suites"


def _jsonl(path, rows):
    path.write_text("".join(json.dumps(r) + "\n" for r in rows))
    return str(path)


def test_every_suite_task_is_registered():
    for name in ("comparison-inspect-v1", "comparison-danish-v1"):
        suite = json.loads((SUITES / f"{name}.json").read_text())
        for item in suite["tasks"]:
            assert item["task"] in REGISTRY, item
    euro = json.loads((SUITES / "comparison-euroeval-v1.json").read_text())
    assert all(t["backend"] == "euroeval" and t["version"] for t in euro["tasks"])


@pytest.mark.parametrize("pred,target,ok", [
    ("\\frac{1}{2}", "0.5", True), ("\\dfrac12", "\\frac{1}{2}", True), ("$42$", "42", True),
    ("42.0", "42", True), ("\\left(3, 4\\right)", "(3,4)", True), ("7", "8", False), ("x^2", "x^{2}", False)])
def test_math_equality(pred, target, ok):
    assert C.math_equal(pred, target) is ok


def test_math_and_gsm8k_extraction():
    s = {"target": "\\frac{3}{4}"}
    assert C.math_scorer("so the result is \\boxed{\\frac{3}{4}}.", s)["scores"]["accuracy"] == 1.0
    assert C.math_scorer("work...\nANSWER: 0.75", s)["scores"]["accuracy"] == 1.0
    assert C.math_scorer("no answer here", s)["scores"]["accuracy"] == 0.0
    g = {"target": "Natalia sold 48/2 = 24 clips... #### 1,234"}
    assert C.gsm8k_scorer("She has 1234 in total.", g)["scores"]["accuracy"] == 1.0
    assert C.gsm8k_scorer("12 + 3 = 15\nANSWER: 1,234", g)["scores"]["accuracy"] == 1.0
    assert C.gsm8k_scorer("ANSWER: 1233", g)["scores"]["accuracy"] == 0.0


def test_overlap_metrics():
    assert C.token_f1("the Eiffel Tower", "Eiffel tower") == 1.0
    assert C.sentence_bleu("the cat sat on the mat", ["the cat sat on the mat"]) == pytest.approx(1.0)
    assert 0 < C.sentence_bleu("the cat sat on the rug", ["the cat sat on the mat"]) < 1
    assert C.rouge_l("w x y z", "w y z v") == pytest.approx(0.75)
    d = C.drop_scorer("Counting the games gives\nANSWER: 1,000", {"target": ["1000", "one thousand"]})
    assert d["scores"] == {"exact_match": 1.0, "f1": 1.0}
    q = C.qa_overlap_scorer("København\nmore text", {"target": ["København"]})
    assert q["scores"]["exact_match"] == 1.0 and q["scores"]["bleu"] > 0


def test_humaneval_execution_with_time_limit():
    meta = {"prompt": "def add(a, b):\n", "test": "def check(f):\n    assert f(2, 3) == 5\n", "entry_point": "add"}
    sample = {"metadata": meta}
    assert C.humaneval_scorer("```python\n    return a + b\n```", sample)["scores"]["pass"] == 1.0
    assert C.humaneval_scorer("    return a - b\n", sample)["scores"]["pass"] == 0.0
    full = "```python\ndef add(a, b):\n    return b + a\n```"
    assert C.humaneval_scorer(full, sample)["scores"]["pass"] == 1.0
    assert C.run_humaneval("while True:\n    pass\n", timeout=1.0) is False


def test_ifeval_checks():
    kw = {}
    assert follows("punctuation:no_comma", "no commas here", kw, "")
    assert not follows("punctuation:no_comma", "one, two", kw, "")
    assert follows("length_constraints:number_words", "one two three four", {"relation": "at least", "num_words": 4}, "")
    assert follows("detectable_format:json_format", '```json\n{"a": 1}\n```', kw, "")
    assert follows("detectable_format:title", "<<Titel>>\ntekst", kw, "")
    assert follows("startend:end_checker", "Slut. Har du flere spørgsmål?", {"end_phrase": "Har du flere spørgsmål?"}, "")
    assert follows("change_case:lowercase_letters", "kun små bogstaver", kw, "")
    assert follows("language:response_language", "Det er en god dag, og jeg har det fint i dag.", {"language": "da"}, "")
    assert not follows("language:response_language", "This is the answer and it is in English.", {"language": "da"}, "")
    assert follows("detectable_format:number_bullet_lists", "* a\n* b\n", {"num_bullets": 2}, "")
    # loose variants: a leading line dropped
    assert not follows("startend:quotation", 'Her er svaret:\n"citat"', kw, "")
    assert follows("startend:quotation", 'Her er svaret:\n"citat"', kw, "", loose=True)
    sample = {"messages": [{"role": "user", "content": "p"}],
              "metadata": {"instruction_id_list": ["punctuation:no_comma", "change_case:capital_letters"],
                           "kwargs": [{}, {}]}}
    scores = ifeval_scorer("HELLO THERE", sample)["scores"]
    assert scores["prompt_strict"] == 1.0 and scores["instruction_strict"] == 1.0
    assert ifeval_scorer("Hello, there", sample)["scores"]["instruction_strict"] == 0.0


def test_chunked_and_fewshot_tasks(tmp_path):
    rows = [{"ctx": f"c{i}", "endings": ["a", "b", "c", "d"], "label": i % 4} for i in range(10)]
    path = _jsonl(tmp_path / "hs.jsonl", rows)
    chunks = [build("hellaswag_ie_fmt", dataset_path=path, chunk=c, chunks=3) for c in range(3)]
    assert [len(s.samples) for s in chunks] == [4, 4, 2] and chunks[1].name == "hellaswag_ie_fmt_chunk1"
    assert chunks[0].samples[1]["target"] == "B"
    assert chunks[0].score("reasoning...\nANSWER: B", chunks[0].samples[1])["scores"]["accuracy"] == 1.0
    mmlu = [{"question": f"q{i}", "choices": ["w", "x", "y", "z"], "answer": i % 4, "subject": "s" + str(i % 2)}
            for i in range(6)]
    dev = [{"question": f"d{i}", "choices": ["w", "x", "y", "z"], "answer": 0, "subject": "s0"} for i in range(7)]
    spec = build("mmlu_5shot", dataset_path=_jsonl(tmp_path / "m.jsonl", mmlu),
                 fewshot_path=_jsonl(tmp_path / "d.jsonl", dev), chunk=0, chunks=2)
    assert spec.name == "mmlu_5shot_chunk0_nothink" and len(spec.samples) == 3
    assert len(spec.samples[0]["messages"]) == 11  # 5 exemplars of subject s0 + the question
    assert len(spec.samples[1]["messages"]) == 1  # no exemplars of subject s1
    assert spec.generation["chat_template_kwargs"] == {"enable_thinking": False}
    arc = [{"question": "q", "choices": {"text": ["a", "b", "c"], "label": ["A", "B", "C"]}, "answerKey": "C"}] * 30
    a = build("arc_25shot", dataset_path=_jsonl(tmp_path / "a.jsonl", arc[:3]),
              fewshot_path=_jsonl(tmp_path / "af.jsonl", arc))
    assert len(a.samples[0]["messages"]) == 51 and a.samples[0]["target"] == "C"
    with pytest.raises(ValueError):
        build("arc_25shot", dataset_path=_jsonl(tmp_path / "a2.jsonl", arc[:3]),
              fewshot_path=_jsonl(tmp_path / "af2.jsonl", arc[:5]))


def test_registered_tasks_run_through_the_direct_runner(tmp_path):
    from mimir_b200.evaluation.runner import run_task
    data = _jsonl(tmp_path / "g.jsonl", [{"question": "1+1?", "answer": "... #### 2"}])
    spec = build("gsm8k", dataset_path=data)
    rows = run_task(spec, {"id": "inspect_evals-gsm8k", "provider": "mockllm"}, "m", "http://unused")
    assert rows[0]["task"] == "inspect_evals-gsm8k" and rows[0]["scores"] == {"accuracy": 0.0}
    ifeval = _jsonl(tmp_path / "i.jsonl", [{"key": 7, "prompt": "Skriv uden komma.",
                                            "instruction_id_list": ["punctuation:no_comma"], "kwargs": [{"x": None}]}])
    spec = build("ifeval_da", dataset_path=ifeval)
    assert spec.samples[0]["metadata"]["kwargs"] == [{}]
    rows = run_task(spec, {"id": "ifeval_da", "provider": "mockllm"}, "m", "http://unused")
    assert set(rows[0]["scores"]) == {"prompt_strict", "instruction_strict", "prompt_loose", "instruction_loose"}
