"""BERTScore rescoring of saved final answers (no generation), with a pinned encoder identity.

Reference behaviour: ``src/mimir/evaluation/bertscore.py:8-28``: layer 17 of a materialised
``xlm-roberta-large`` at a fixed revision, no IDF, no baseline rescaling, fp32 on CPU; empty
predictions score 0; records note whether either side was truncated.  Requires the
``bert_score`` package (not bundled).
"""
from __future__ import annotations

import json
from pathlib import Path

REVISION = "c23d21b0620b635a76227c604d44e43a9f0ee389"
ENCODER = {"model": "xlm-roberta-large", "revision": REVISION}


def score_saved(input_path, output_path, encoder_path, *, language: str, batch_size: int = 8) -> None:
    import torch
    from bert_score import BERTScorer
    identity = json.loads((Path(encoder_path) / "mimir_encoder_revision.json").read_text())
    if identity != ENCODER:
        raise ValueError("Unqualified BERTScore encoder")
    scorer = BERTScorer(model_type=str(encoder_path), num_layers=17, lang=language, device="cpu", idf=False,
                        rescale_with_baseline=False)
    scorer._model.float()
    rows = [json.loads(s) for s in Path(input_path).read_text().splitlines()]
    with Path(output_path).open("x") as out:
        for start in range(0, len(rows), batch_size):
            batch = rows[start:start + batch_size]
            keep = [i for i, r in enumerate(batch) if r["prediction"].strip()]
            values = [0.0] * len(batch)
            if keep:
                with torch.no_grad():
                    _, _, f1 = scorer.score([batch[i]["prediction"] for i in keep],
                                            [batch[i]["reference"] for i in keep], batch_size=batch_size)
                for i, v in zip(keep, f1.tolist()):
                    values[i] = v
            for row, value in zip(batch, values):
                lengths = {k: len(scorer._tokenizer.encode(row[k], truncation=False)) for k in ("prediction", "reference")}
                out.write(json.dumps(row | {"scores": {"bertscore_f1": value}, "encoder": identity,
                                            "truncated": {k: n > scorer._tokenizer.model_max_length
                                                          for k, n in lengths.items()}}, ensure_ascii=False) + "\n")
