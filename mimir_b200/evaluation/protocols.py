"""Recover the evaluation protocol of past Inspect runs from their ``.eval`` logs.

Reference behaviour: ``tools/recover_protocols.py``.  An Inspect ``.eval`` log is a zip archive
whose ``header.json`` describes the run.  Only an allowlist of protocol fields is kept (task,
dataset identity and size, sample selection, generation settings, scorer names, status and the
header's SHA-256), never credentials, model arguments or the dataset location, so the result can
be published beside the scores it explains.

Archive members compressed with Zstandard need the ``zstandard`` package; without it such a log
is listed under ``skipped`` with the reason instead of stopping the scan.

Usage: ``python -m mimir_b200.evaluation.protocols SOURCE OUTPUT.json [FOLDER ...]`` scans the
given folders under SOURCE (default: all of SOURCE) recursively.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import struct
import zipfile
from pathlib import Path
from typing import Iterable, Optional

SELECTION_KEYS = ("limit", "sample_id", "sample_shuffle", "epochs", "epochs_reducer", "max_samples")
GENERATION_KEYS = ("max_tokens", "temperature", "top_p", "stop_seqs", "seed")
DATASET_KEYS = ("name", "samples", "shuffled", "sample_ids")  # never "location"
_ZSTD = 93  # zip compression method id


def _pick(mapping: dict, keys: Iterable[str]) -> dict:
    return {k: mapping[k] for k in keys if k in mapping}


def _member(archive: zipfile.ZipFile, name: str) -> bytes:
    info = archive.getinfo(name)
    if info.compress_type != _ZSTD:
        return archive.read(name)
    try:
        import zstandard
    except ImportError as exc:
        raise LookupError("Zstandard-compressed member and no zstandard package") from exc
    with open(archive.filename, "rb") as f:  # raw member bytes after the local file header
        f.seek(info.header_offset)
        header = f.read(30)
        name_len, extra_len = struct.unpack_from("<HH", header, 26)
        f.seek(name_len + extra_len, 1)
        raw = f.read(info.compress_size)
    return zstandard.ZstdDecompressor().decompress(raw, max_output_size=info.file_size)


def protocol_of(path: Path, base: Path) -> Optional[dict]:
    """The allowlisted protocol record of one ``.eval`` log, or None if it has no header."""
    with zipfile.ZipFile(path) as archive:
        if "header.json" not in archive.namelist():
            return None
        raw = _member(archive, "header.json")
    header = json.loads(raw)
    ev = header.get("eval", {})
    results = header.get("results") or {}
    return {"source": str(path.relative_to(base)), "header_sha256": hashlib.sha256(raw).hexdigest(),
            "status": header.get("status"), "task": ev.get("task"),
            "dataset": _pick(ev.get("dataset", {}), DATASET_KEYS),
            "selection": _pick(ev.get("config", {}), SELECTION_KEYS),
            "generation": _pick(header.get("plan", {}).get("config", {}), GENERATION_KEYS),
            "scorers": [s.get("name") for s in results.get("scores", [])]}


def recover(source, output, folders: Optional[list] = None) -> dict:
    source = Path(source)
    roots = [source / f for f in folders] if folders else [source]
    records, skipped = [], []
    for root in roots:
        for path in sorted(root.rglob("*.eval")):
            try:
                record = protocol_of(path, source)
            except LookupError as exc:
                skipped.append({"source": str(path.relative_to(source)), "reason": str(exc)})
                continue
            except (zipfile.BadZipFile, ValueError, KeyError):
                skipped.append({"source": str(path.relative_to(source)), "reason": "unreadable log"})
                continue
            if record is not None:
                records.append(record)
    out = {"records": records, "skipped": skipped}
    Path(output).write_text(json.dumps(records, indent=2) + "\n")
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Recover allowlisted protocol fields from Inspect .eval logs")
    ap.add_argument("source", type=Path)
    ap.add_argument("output", type=Path)
    ap.add_argument("folders", nargs="*")
    args = ap.parse_args(argv)
    result = recover(args.source, args.output, args.folders or None)
    print(f"Recovered {len(result['records'])} allowlisted log headers; skipped {len(result['skipped'])}")
    for item in result["skipped"]:
        print(f"skipped {item['source']}: {item['reason']}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
