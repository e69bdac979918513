"""Validation of an Open Knowledge Format (OKF 0.2) Markdown bundle, the layout of a project wiki.

Reference behaviour: ``scripts/validate_okf.py``.  The rules are the format's, so they match:

* every directory that holds Markdown has an ``index.md`` linking each immediate child concept
  (``name.md``, except ``index.md`` / ``log.md``) and each child group (``dir/``);
* the root ``index.md`` has YAML frontmatter with ``okf_version: "0.2"``; other indexes have none;
* ``log.md`` files have no frontmatter and at least one ``## YYYY-MM-DD`` heading;
* a concept file is smaller than 50 000 bytes and has frontmatter with a non-empty ``type``, an
  optional ``status`` (draft / stable / deprecated), an optional ``confidence``
  (high / medium / low) and optional ``sources`` (a list of mappings, each with ``resource``);
* no ``[[wiki-link]]`` syntax remains;
* a relative link to a ``.md`` file or a ``dir/`` that does not exist is a warning.

Usage: ``python -m mimir_b200.utils.okf [bundle]`` (default ``wiki``); exit code 1 on errors.
"""
from __future__ import annotations

import argparse
import re
import sys
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional

import yaml

OKF_VERSION = "0.2"
CONCEPT_LIMIT = 50_000
STATUSES = frozenset({"draft", "stable", "deprecated"})
CONFIDENCES = frozenset({"high", "medium", "low"})
_FRONT = re.compile(r"\A---[ \t]*\n(.*?)\n---[ \t]*\n", re.S)
_LINK = re.compile(r"(?<!!)\[[^\]]+\]\(([^)]+)\)")
_LOG_DAY = re.compile(r"^## \d{4}-\d{2}-\d{2}$", re.M)
_RESERVED = ("index.md", "log.md")


@dataclass
class Report:
    errors: list = field(default_factory=list)
    warnings: list = field(default_factory=list)

    @property
    def ok(self) -> bool:
        return not self.errors


def _frontmatter(text: str) -> tuple[Optional[dict], str]:
    """(metadata or None, body); ValueError on malformed YAML or a non-mapping."""
    m = _FRONT.match(text)
    if m is None:
        return None, text
    try:
        meta = yaml.safe_load(m.group(1))
    except yaml.YAMLError as exc:
        raise ValueError(f"invalid YAML frontmatter: {exc}") from exc
    if not isinstance(meta, dict):
        raise ValueError("frontmatter must be a YAML mapping")
    return meta, text[m.end():]


def _link_target(raw: str) -> str:
    return raw.strip().split(maxsplit=1)[0].strip("<>")


def _local_file(bundle: Path, page: Path, target: str) -> Optional[Path]:
    """The file a relative Markdown link points at, or None for anything that is not a local page."""
    target = target.split("#", 1)[0].split("?", 1)[0]
    if not target or "://" in target or target.startswith("mailto:") or not target.endswith((".md", "/")):
        return None
    base = bundle / target.lstrip("/") if target.startswith("/") else page.parent / target
    return (base / "index.md" if target.endswith("/") else base).resolve()


def _check_index_links(bundle: Path, directory: Path, report: Report) -> None:
    index = directory / "index.md"
    where = directory.relative_to(bundle) if directory != bundle else Path(".")
    if not index.is_file():
        report.errors.append(f"{where}: directory requires index.md")
        return
    linked = {_link_target(t).split("#", 1)[0] for t in _LINK.findall(index.read_text(encoding="utf-8"))}
    children = [p.name for p in directory.glob("*.md") if p.name not in _RESERVED]
    children += [f"{p.name}/" for p in directory.iterdir() if p.is_dir() and any(p.rglob("*.md"))]
    for child in sorted(children):
        if child not in linked:
            report.errors.append(f"{index.relative_to(bundle)}: missing immediate child link {child!r}")


def _check_concept(rel: Path, size: int, meta: Optional[dict], report: Report) -> None:
    if size >= CONCEPT_LIMIT:
        report.errors.append(f"{rel}: concept is {size} bytes; split concepts below {CONCEPT_LIMIT} bytes")
    if meta is None:
        report.errors.append(f"{rel}: concept is missing YAML frontmatter")
        return
    kind = meta.get("type")
    if not (isinstance(kind, str) and kind.strip()):
        report.errors.append(f"{rel}: concept requires a non-empty type")
    if meta.get("status") is not None and meta["status"] not in STATUSES:
        report.errors.append(f"{rel}: invalid status {meta['status']!r}")
    if meta.get("confidence") is not None and meta["confidence"] not in CONFIDENCES:
        report.errors.append(f"{rel}: invalid confidence {meta['confidence']!r}")
    sources = meta.get("sources", [])
    if sources and not isinstance(sources, list):
        report.errors.append(f"{rel}: sources must be a list")
    elif isinstance(sources, list):
        for i, src in enumerate(sources):
            if not (isinstance(src, dict) and src.get("resource")):
                report.errors.append(f"{rel}: sources[{i}] requires resource")


def validate(bundle) -> Report:
    bundle = Path(bundle).resolve()
    report = Report()
    pages = sorted(bundle.rglob("*.md"))
    for directory in sorted({bundle, *(p.parent for p in pages)}):
        _check_index_links(bundle, directory, report)
    for page in pages:
        rel = page.relative_to(bundle)
        text = page.read_text(encoding="utf-8")
        try:
            meta, body = _frontmatter(text)
        except ValueError as exc:
            report.errors.append(f"{rel}: {exc}")
            continue
        if page.name == "index.md":
            if rel == Path("index.md"):
                if meta is None or str(meta.get("okf_version")) != OKF_VERSION:
                    report.errors.append(f'{rel}: root index must declare okf_version: "{OKF_VERSION}"')
            elif meta is not None:
                report.errors.append(f"{rel}: subdirectory indexes must not have frontmatter")
        elif page.name == "log.md":
            if meta is not None:
                report.errors.append(f"{rel}: log files must not have frontmatter")
            if not _LOG_DAY.search(body):
                report.errors.append(f"{rel}: log must contain ISO YYYY-MM-DD headings")
        else:
            _check_concept(rel, page.stat().st_size, meta, report)
            if meta is None:
                continue
        if "[[" in body or "]]" in body:
            report.errors.append(f"{rel}: legacy wiki-link syntax remains")
        for raw in _LINK.findall(body):
            target = _local_file(bundle, page, _link_target(raw))
            if target is not None and not target.exists():
                report.warnings.append(f"{rel}: unresolved local link {raw!r}")
    return report


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Validate an OKF 0.2 Markdown bundle")
    ap.add_argument("bundle", nargs="?", type=Path, default=Path("wiki"))
    args = ap.parse_args(argv)
    report = validate(args.bundle)
    for w in report.warnings:
        print(f"warning: {w}")
    for e in report.errors:
        print(f"error: {e}", file=sys.stderr)
    print(f"OKF validation: {len(report.errors)} error(s), {len(report.warnings)} warning(s)",
          file=sys.stderr if report.errors else sys.stdout)
    return 0 if report.ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
