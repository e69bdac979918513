"""Rich table of the queue with progress and ETA from recorded progress files.

Reference behaviour: ``src/mimir/scheduling/monitor.py:7-38``.
"""
from __future__ import annotations

import json
import time
from pathlib import Path


def _progress(cfg: dict) -> tuple[str, str]:
    path = cfg.get("progress_file")
    if not path:
        return "unknown", "unknown"
    try:
        data = json.loads(Path(path).read_text())
        done, total = data["completed"], data["total"]
        text = f"{done}/{total}" + (f"; passes {data['passes']}" if "passes" in data else "")
        elapsed = data.get("elapsed_seconds", 0)
        eta = f"{max(0, total - done) * elapsed / done:.0f}s" if done > 0 and elapsed > 0 else "unknown"
        return text, eta
    except (OSError, ValueError, KeyError):
        return "unknown", "unknown"


def render(store):
    from rich.table import Table
    rows, counts = store.rows(), {}
    table = Table(caption="ETAs use recorded progress rates; absent evidence is shown as unknown.")
    for label in ("Job / task", "State", "Attempt", "GPU / judge resources", "Progress", "ETA"):
        table.add_column(label)
    for row in rows:
        counts[row["state"]] = counts.get(row["state"], 0) + 1
        cfg = json.loads(row["config"])
        progress, eta = _progress(cfg)
        table.add_row(row["id"], row["state"] + (" (held)" if row["held"] else ""), str(row["attempt"]),
                      ", ".join(cfg.get("resources", [])), progress, eta)
    table.title = "Mimir queue — " + ", ".join(f"{n} {s}" for s, n in sorted(counts.items()))
    try:
        status = json.loads((store.path.parent / "idle-status.json").read_text())
        table.caption = (f"Scheduler: {status['state']} ({max(0, time.time() - status['time']):.0f}s ago). "
                         f"{status.get('reason', '')}")
    except (OSError, ValueError, KeyError):
        pass
    return table


def monitor(store, watch: bool = False) -> None:
    from rich.console import Console
    if not watch:
        Console().print(render(store))
        return
    from rich.live import Live
    with Live(render(store), refresh_per_second=1) as live:
        while True:
            time.sleep(1)
            live.update(render(store))
