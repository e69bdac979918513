"""Command line: ``python -m mimir_b200 <command>``.

Commands mirror the reference CLI (``src/mimir/cli.py:11-98``): ``train`` (Hydra-style
overrides passed through unchanged, ``--suspendable``), ``checkpoint import``, ``export``,
``serve``, ``eval``, ``schedule``, ``monitor`` and ``doctor``, plus ``qualify-cpu`` (the reference's
``tools/qualify_cpu.py`` campaign).  Built on argparse.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path


def _train(args, rest):
    from mimir_b200.train.entry import run
    run(rest, suspendable=args.suspendable)


def _import(args, _rest):
    from mimir_b200.ckpt.importer import import_legacy
    import_legacy(args.source, args.output, tag=args.tag, mode=args.mode)


def _export(args, _rest):
    from mimir_b200.export.convert import export
    export(args.checkpoint, args.output, args.tokenizer, ema=args.ema)


def _serve(args, _rest):
    from mimir_b200.serving.server import serve
    serve(args.model, args.port, args.gpus, eager=args.eager, backend=args.backend)


def _eval(args, _rest):
    from mimir_b200.evaluation.clients import evaluate
    print(json.dumps(evaluate(str(args.suite), args.model, str(args.output), args.base_url)))


def _schedule(args, _rest):
    from mimir_b200.scheduling.store import Store
    store = Store(args.database)
    if args.hold_job:
        store.hold(args.hold_job, True)
    if args.release_job:
        store.hold(args.release_job, False)
    if args.backup:
        store.backup(args.backup)
    if args.edit_job:
        if args.config_file is None:
            raise SystemExit("--edit-job requires --config-file")
        store.edit(args.edit_job, json.loads(args.config_file.read_text()))
    if args.plan:
        for row in json.loads(args.plan.read_text())["jobs"]:
            store.add(row["id"], row["kind"], row["config"],
                      [(d["id"], d.get("policy", "success")) for d in row.get("depends", [])],
                      row.get("max_attempts", 3), held=row.get("held", False))
    if args.run:
        from mimir_b200.scheduling.worker import recover_abandoned, run_one
        from mimir_b200.serving.server import ServerPool
        from mimir_b200.train.suspension.protocol import exclusive
        with exclusive(args.database.with_suffix(".runner.lock")):
            pool = ServerPool(args.database.parent / "servers")
            try:
                recover_abandoned(store, args.database.parent / "attempts")
                while run_one(store, args.database.parent / "attempts", pool):
                    pass
            finally:
                pool.close()
    print(json.dumps(store.rows(), indent=2))


def _monitor(args, _rest):
    from mimir_b200.scheduling.monitor import monitor
    from mimir_b200.scheduling.store import Store
    monitor(Store(args.database), args.watch)


def _qualify(args, _rest):
    from mimir_b200.qualify import main as qualify
    print(qualify(args.output))


def _doctor(_args, _rest):
    """Read-only dependency and capability report; never allocates a GPU."""
    from importlib.metadata import PackageNotFoundError, version
    out = {}
    for name in ("torch", "transformers", "vllm", "numpy", "pydantic"):
        try:
            out[name] = version(name)
        except PackageNotFoundError:
            out[name] = "not installed"
    from mimir_b200.ops import _ext
    out["mimir_b200._C"] = "built" if _ext.available() else "missing"
    try:
        from mimir_b200 import _host  # noqa: F401
        out["mimir_b200._host"] = "built"
    except ImportError:
        out["mimir_b200._host"] = "missing"
    out["gpus"] = _nvml_gpus()
    print(json.dumps(out, indent=2))


def _nvml_gpus():
    """GPUs as NVML reports them (read-only queries; no CUDA context): name, memory, compute
    capability and whether it is the sm_100 part the kernels are built for."""
    try:
        import pynvml
        pynvml.nvmlInit()
    except Exception as exc:  # no driver here (a CPU box) or no NVML bindings
        return f"unavailable ({type(exc).__name__})"
    try:
        gpus = []
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            name = pynvml.nvmlDeviceGetName(h)
            major, minor = pynvml.nvmlDeviceGetCudaComputeCapability(h)
            gpus.append({"index": i, "name": name.decode() if isinstance(name, bytes) else name,
                         "memory_mib": pynvml.nvmlDeviceGetMemoryInfo(h).total // (1 << 20),
                         "compute_capability": f"{major}.{minor}", "kernels_supported": (major, minor) == (10, 0)})
        return gpus
    finally:
        pynvml.nvmlShutdown()


def _campaign(args, _rest) -> None:
    from mimir_b200.campaigns.prepare import RECIPES, extend, prepare
    if args.action == "prepare":
        print(prepare(args.output, args.data, args.tokenizer, args.template,
                      recipe=args.recipe or RECIPES / "xxs-dfm15-20k.json", gpus=args.gpus,
                      eval_steps=args.eval_steps, database=args.database))
    else:
        print(f"Added {extend(args.output, extensions=args.extensions or RECIPES / 'xxs-dfm15-20k.extensions.json', release=args.release)} jobs")


def _okf(args, _rest) -> None:
    from mimir_b200.utils.okf import main as okf_main
    raise SystemExit(okf_main([str(args.bundle)]))


def _protocols(args, _rest) -> None:
    from mimir_b200.evaluation.protocols import main as protocols_main
    raise SystemExit(protocols_main([str(args.source), str(args.output), *args.folders]))


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="mimir_b200")
    sub = p.add_subparsers(dest="command", required=True)
    t = sub.add_parser("train", help="train with config overrides, e.g. size@arch=XXS")
    t.add_argument("--suspendable", action="store_true")
    t.set_defaults(fn=_train)
    ck = sub.add_parser("checkpoint").add_subparsers(dest="action", required=True)
    im = ck.add_parser("import", help="explicit one-way legacy checkpoint import")
    im.add_argument("source", type=Path)
    im.add_argument("output", type=Path)
    im.add_argument("--mode", required=True, choices=("exact", "weights"))
    im.add_argument("--tag", required=True)
    im.set_defaults(fn=_import)
    ex = sub.add_parser("export", help="convert a checkpoint to a Hugging Face directory")
    ex.add_argument("checkpoint", type=Path)
    ex.add_argument("output", type=Path)
    ex.add_argument("--tokenizer", type=Path, required=True)
    ex.add_argument("--ema", action=argparse.BooleanOptionalAction, default=True)
    ex.set_defaults(fn=_export)
    sv = sub.add_parser("serve")
    sv.add_argument("model", type=Path)
    sv.add_argument("--port", type=int, default=8000)
    sv.add_argument("--gpus", required=True)
    sv.add_argument("--eager", action="store_true")
    sv.add_argument("--backend", choices=("auto", "vllm", "native"), default="auto",
                    help="auto: vLLM when it registers Mimir2, else the native server")
    sv.set_defaults(fn=_serve)
    ev = sub.add_parser("eval")
    ev.add_argument("suite", type=Path)
    ev.add_argument("model")
    ev.add_argument("output", type=Path)
    ev.add_argument("--base-url", default="http://127.0.0.1:8000/v1")
    ev.set_defaults(fn=_eval)
    sc = sub.add_parser("schedule")
    sc.add_argument("database", type=Path)
    sc.add_argument("--plan", type=Path)
    sc.add_argument("--run", action="store_true")
    sc.add_argument("--hold-job")
    sc.add_argument("--release-job")
    sc.add_argument("--backup", type=Path)
    sc.add_argument("--edit-job")
    sc.add_argument("--config-file", type=Path)
    sc.set_defaults(fn=_schedule)
    mo = sub.add_parser("monitor")
    mo.add_argument("database", type=Path)
    mo.add_argument("--watch", action="store_true")
    mo.set_defaults(fn=_monitor)
    sub.add_parser("doctor").set_defaults(fn=_doctor)
    qc = sub.add_parser("qualify-cpu", help="isolated CPU campaign: train, export, eval, resume, suspend (bit-exact)")
    qc.add_argument("output", type=Path)
    qc.set_defaults(fn=_qualify)
    cp = sub.add_parser("campaign", help="prepare or extend a held training/evaluation campaign").add_subparsers(
        dest="action", required=True)
    pr = cp.add_parser("prepare", help="recipe -> held scheduler jobs (runs nothing)")
    pr.add_argument("output", type=Path)
    pr.add_argument("--data", type=Path, required=True)
    pr.add_argument("--tokenizer", type=Path, required=True)
    pr.add_argument("--template", type=Path, required=True)
    pr.add_argument("--recipe", type=Path)
    pr.add_argument("--gpus")
    pr.add_argument("--eval-steps", type=int, nargs="+")
    pr.add_argument("--database", type=Path)
    pr.set_defaults(fn=_campaign)
    xt = cp.add_parser("extend", help="append derived variants to a prepared campaign")
    xt.add_argument("output", type=Path)
    xt.add_argument("--extensions", type=Path)
    xt.add_argument("--release", action="store_true")
    xt.set_defaults(fn=_campaign)
    ok = sub.add_parser("okf", help="validate an OKF 0.2 Markdown bundle")
    ok.add_argument("bundle", type=Path, nargs="?", default=Path("wiki"))
    ok.set_defaults(fn=_okf)
    rp = sub.add_parser("recover-protocols", help="allowlisted protocol fields of Inspect .eval logs")
    rp.add_argument("source", type=Path)
    rp.add_argument("output", type=Path)
    rp.add_argument("folders", nargs="*")
    rp.set_defaults(fn=_protocols)
    return p


def main(argv=None) -> None:
    argv = sys.argv[1:] if argv is None else list(argv)
    args, rest = parser().parse_known_args(argv)
    if rest and args.command != "train":
        parser().error(f"unrecognized arguments: {' '.join(rest)}")
    args.fn(args, rest)


if __name__ == "__main__":
    main()
