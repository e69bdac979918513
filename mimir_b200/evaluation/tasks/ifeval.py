"""Verifiable-instruction checks (IFEval instruction ids) for ``ifeval_da``.

Reference behaviour: ``src/mimir/evaluation/tasks/ifeval_da.py``, which scores the Danish IFEval
set with the external ``instruction_following_eval`` package plus checkers of its own (all
lowercase / all capitals, one of given options, response language).  Here every checker is
written from the public instruction definitions (Zhou et al. 2023, "Instruction-Following
Evaluation for Large Language Models"), keyed by the same instruction ids, so no optional package
is needed.  ``language:response_language`` uses a stop-word vote over the languages the campaign
evaluates (Danish, English, Swedish, Norwegian, German) instead of a statistical detector.

Scores per sample: ``prompt_strict`` (every instruction followed), ``instruction_strict`` (share
followed), and the ``loose`` pair, where an instruction counts as followed if it holds for one of
the response variants IFEval defines (first line dropped, last line dropped, both, ``*`` removed).
"""
from __future__ import annotations

import json
import re

_WORD = re.compile(r"\b\w+\b", re.U)
_SENTENCE_END = re.compile(r"[.!?]+(?:\s|$)")
_COMPARE = {"less than": lambda n, k: n < k, "at least": lambda n, k: n >= k,
            "at most": lambda n, k: n <= k, "more than": lambda n, k: n > k, "exactly": lambda n, k: n == k}
_STOPWORDS = {
    "da": {"og", "i", "det", "at", "en", "den", "til", "er", "som", "på", "de", "med", "af", "for", "ikke", "der",
           "var", "jeg", "har", "et", "men", "om", "vi", "fra", "skal", "kan", "også", "efter", "eller", "hvor"},
    "en": {"the", "and", "of", "to", "a", "in", "is", "that", "it", "for", "on", "with", "as", "was", "are", "be",
           "this", "by", "not", "or", "have", "from", "but", "they", "you", "which", "an", "at", "we", "their"},
    "sv": {"och", "att", "det", "som", "en", "på", "är", "av", "för", "med", "till", "den", "har", "de", "inte",
           "om", "ett", "jag", "men", "var", "så", "vi", "från", "kan", "också", "eller", "när", "hur", "där"},
    "no": {"og", "i", "det", "at", "en", "er", "som", "på", "til", "med", "av", "for", "ikke", "den", "har", "de",
           "jeg", "et", "men", "om", "vi", "fra", "skal", "kan", "også", "eller", "hvor", "ble", "etter", "være"},
    "de": {"der", "die", "und", "in", "den", "von", "zu", "das", "mit", "sich", "des", "auf", "für", "ist", "im",
           "nicht", "ein", "eine", "als", "auch", "es", "an", "werden", "aus", "er", "hat", "dass", "sie", "nach"},
}


def _words(text: str) -> list[str]:
    return _WORD.findall(text)


def _count_ok(n: int, relation: str, k: int) -> bool:
    return _COMPARE.get(relation, _COMPARE["at least"])(n, k)


def _paragraphs(text: str, sep: str = r"\s?\*\*\*\s?") -> list[str]:
    parts = [p for p in re.split(sep, text) if p.strip()]
    return parts


def _language(text: str) -> str:
    words = [w.lower() for w in _words(text)]
    votes = {lang: sum(w in stop for w in words) for lang, stop in _STOPWORDS.items()}
    return max(votes, key=votes.get) if any(votes.values()) else ""


def _check(instruction: str, response: str, kw: dict, prompt: str) -> bool:  # noqa: C901 - one table of rules
    r = response
    if instruction == "keywords:existence":
        return all(re.search(re.escape(k), r, re.I) for k in kw.get("keywords") or [])
    if instruction == "keywords:frequency":
        n = len(re.findall(re.escape(kw["keyword"]), r, re.I))
        return _count_ok(n, kw.get("relation", "at least"), int(kw["frequency"]))
    if instruction == "keywords:forbidden_words":
        return not any(re.search(r"\b" + re.escape(k) + r"\b", r, re.I) for k in kw.get("forbidden_words") or [])
    if instruction == "keywords:letter_frequency":
        n = r.lower().count(str(kw["letter"]).lower())
        return _count_ok(n, kw.get("let_relation", "at least"), int(kw["let_frequency"]))
    if instruction == "language:response_language":
        return _language(r) == (kw.get("language") or "en")
    if instruction == "length_constraints:number_sentences":
        return _count_ok(len(_SENTENCE_END.findall(r.strip() + " ")), kw.get("relation", "at least"),
                         int(kw["num_sentences"]))
    if instruction == "length_constraints:number_paragraphs":
        return len(_paragraphs(r)) == int(kw["num_paragraphs"])
    if instruction == "length_constraints:number_words":
        return _count_ok(len(_words(r)), kw.get("relation", "at least"), int(kw["num_words"]))
    if instruction == "length_constraints:nth_paragraph_first_word":
        paras = [p for p in re.split(r"\n\s*\n", r) if p.strip()]
        n = int(kw["nth_paragraph"])
        if len(paras) != int(kw["num_paragraphs"]) or n > len(paras):
            return False
        first = _words(paras[n - 1])
        return bool(first) and first[0].lower() == str(kw["first_word"]).lower()
    if instruction == "detectable_content:number_placeholders":
        return len(re.findall(r"\[[^\]]+\]", r)) >= int(kw["num_placeholders"])
    if instruction == "detectable_content:postscript":
        marker = str(kw.get("postscript_marker") or "P.S.")
        return re.search(r"\s*" + re.escape(marker).replace(r"\ ", r"\s*"), r, re.I | re.M) is not None
    if instruction == "detectable_format:number_bullet_lists":
        bullets = re.findall(r"^\s*[\*\-]\s", r, re.M)
        return len(bullets) == int(kw["num_bullets"])
    if instruction == "detectable_format:constrained_response":
        return any(o in r.strip() for o in ("My answer is yes.", "My answer is no.", "My answer is maybe."))
    if instruction == "detectable_format:constrained_response_with_argument":
        options = [str(o) for o in (kw.get("options") or []) if str(o).strip()] or [
            "My answer is yes.", "My answer is no.", "My answer is maybe."]
        return any(o in r.strip() for o in options)
    if instruction == "detectable_format:number_highlighted_sections":
        marked = [m for m in re.findall(r"\*[^\n\*]+\*", r) if m.strip("*").strip()]
        marked += [m for m in re.findall(r"\*\*[^\n\*]+\*\*", r) if m.strip("*").strip()]
        return len(marked) >= int(kw["num_highlights"])
    if instruction == "detectable_format:multiple_sections":
        splitter = str(kw.get("section_spliter") or "Section").strip()
        sections = re.split(r"\s?" + re.escape(splitter) + r"\s?\d+\s?", r)
        return len(sections) - 1 >= int(kw["num_sections"])
    if instruction == "detectable_format:json_format":
        body = r.strip()
        for fence in ("```json", "```Json", "```JSON", "```"):
            body = body.removeprefix(fence)
        body = body.removesuffix("```").strip()
        try:
            json.loads(body)
            return True
        except ValueError:
            return False
    if instruction == "detectable_format:title":
        return any(t.strip() for t in re.findall(r"<<([^\n]+)>>", r))
    if instruction == "combination:two_responses":
        parts = [p.strip() for p in r.split("******")]
        return len(parts) == 2 and all(parts) and parts[0] != parts[1]
    if instruction == "combination:repeat_prompt":
        return r.strip().lower().startswith(str(kw.get("prompt_to_repeat") or prompt).strip().lower())
    if instruction == "startend:end_checker":
        return r.strip().lower().endswith(str(kw["end_phrase"]).strip().lower())
    if instruction == "startend:quotation":
        s = r.strip()
        return len(s) > 1 and s[0] == '"' and s[-1] == '"'
    if instruction in ("change_case:english_capital", "change_case:capital_letters"):
        return r.isupper()
    if instruction in ("change_case:english_lowercase", "change_case:lowercase_letters"):
        return r.islower()
    if instruction == "change_case:capital_word_frequency":
        n = sum(1 for w in _words(r) if w.isupper())
        return _count_ok(n, kw.get("capital_relation", "at least"), int(kw["capital_frequency"]))
    if instruction == "punctuation:no_comma":
        return "," not in r
    raise KeyError(f"unknown instruction id {instruction!r}")


def _variants(response: str) -> list[str]:
    lines = response.split("\n")
    dropped = ["\n".join(lines[1:]).strip(), "\n".join(lines[:-1]).strip(), "\n".join(lines[1:-1]).strip()]
    bases = [response, *dropped]
    return bases + [b.replace("*", "") for b in bases]


def follows(instruction: str, response: str, kwargs: dict, prompt: str, loose: bool = False) -> bool:
    candidates = _variants(response) if loose else [response]
    return any(c.strip() and _check(instruction, c, kwargs, prompt) for c in candidates)


def ifeval_scorer(completion: str, sample: dict) -> dict:
    meta = sample["metadata"]
    ids, kwargs = meta["instruction_id_list"], meta["kwargs"]
    prompt = sample["messages"][-1]["content"]
    strict = [follows(i, completion, k, prompt) for i, k in zip(ids, kwargs)]
    loose = [follows(i, completion, k, prompt, loose=True) for i, k in zip(ids, kwargs)]
    n = max(len(ids), 1)
    return {"scores": {"prompt_strict": float(all(strict)), "instruction_strict": sum(strict) / n,
                       "prompt_loose": float(all(loose)), "instruction_loose": sum(loose) / n}}


def normalise_kwargs(record: dict) -> list[dict]:
    """One kwargs mapping per instruction id (missing entries are empty; ``None`` values dropped)."""
    ids = record["instruction_id_list"]
    given = list(record.get("kwargs") or [])
    if len(given) > len(ids):
        raise ValueError("more kwargs than instruction ids")
    given += [{} for _ in range(len(ids) - len(given))]
    return [{k: v for k, v in (kw or {}).items() if v is not None} for kw in given]
