"""Direct vLLM serving of exported Mimir2 models, and a pool that reuses compatible servers.

Reference behaviour: ``src/mimir/serving/server.py:12-75``.

* ``command(spec)`` validates the export (``model_type == "mimir2"``, hierarchical recurrence,
  no persistent-H / branch-specific L mixing; sparse MoS only in eager mode; explicit numeric
  GPU indices) and builds the OpenAI server argv: loopback host, tensor parallel = #GPUs.
  ``backend="native"`` launches :mod:`mimir_b200.serving.native` instead (this framework's
  Transformers model behind an OpenAI-compatible endpoint, one GPU): it serves every exported
  configuration, looped recurrence included, with the prompt as the prefix-LM prefix.
  ``backend="auto"`` (the default) takes vLLM when the installed vLLM registers the Mimir2
  architecture (the reference's patched fork does; stock vLLM does not) and the native server
  otherwise.
* ``ServerPool`` keys servers by SHA-256 of the export receipt, the chat template and the
  spec, so a server is reused only for an identical model/template/launch; it owns each
  server's process group and tears it down (TERM, then KILL after 30 s).
"""
from __future__ import annotations

import hashlib
import json
import os
import signal
import subprocess
import sys
import time
import urllib.request
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Optional


@dataclass(frozen=True)
class ServerSpec:
    model: str
    gpus: str
    port: int = 8000
    eager: bool = False
    max_model_len: Optional[int] = None
    template: Optional[str] = None
    backend: str = "auto"  # "vllm", "native", or "auto": vLLM when it knows Mimir2

    def key(self) -> str:
        receipt = (Path(self.model) / "export_receipt.json").read_bytes()
        template = Path(self.template).read_bytes() if self.template else b""
        return hashlib.sha256(receipt + template + json.dumps(asdict(self), sort_keys=True).encode()).hexdigest()


def vllm_knows_mimir2() -> bool:
    """True when the installed vLLM registers ``Mimir2ForCausalLM``."""
    try:
        from vllm import ModelRegistry
        return "Mimir2ForCausalLM" in ModelRegistry.get_supported_archs()
    except Exception:  # vLLM missing or unusable here
        return False


def command(spec: ServerSpec) -> list[str]:
    cfg = json.loads((Path(spec.model) / "config.json").read_text())
    if cfg.get("model_type") != "mimir2":
        raise ValueError("Only Mimir2 can be served")
    backend = spec.backend
    if backend == "auto":
        backend = "vllm" if vllm_knows_mimir2() else "native"
    if backend == "native":
        if not spec.gpus or len(spec.gpus.split(",")) != 1 or not spec.gpus.isdigit():
            raise ValueError("The native server runs on exactly one explicit GPU index")
        # CUDA_VISIBLE_DEVICES (set by the launcher) makes the chosen GPU cuda:0.
        return [sys.executable, "-m", "mimir_b200.serving.native", spec.model, "--host", "127.0.0.1",
                "--port", str(spec.port), "--device", "cuda:0", "--dtype", "bfloat16"]
    if backend != "vllm":
        raise ValueError(f"unknown serving backend {backend!r}")
    if cfg.get("recurrence_mode", "hierarchical") != "hierarchical":
        raise ValueError("Looped recurrence is not supported by the inference integrations")
    if cfg.get("h_residual_persistence") or cfg.get("h_branch_l_mixing"):
        raise ValueError("Persistent H streams and branch-specific L mixing require inference support")
    if cfg.get("mos_sparse") and not spec.eager:
        raise ValueError("Sparse MoS requires explicitly selected eager execution")
    if not spec.gpus or any(not g.isdigit() for g in spec.gpus.split(",")):
        raise ValueError("Explicit GPU indices required")
    args = [sys.executable, "-m", "vllm.entrypoints.openai.api_server", "--model", spec.model, "--host", "127.0.0.1",
            "--port", str(spec.port), "--tensor-parallel-size", str(len(spec.gpus.split(",")))]
    if spec.eager:
        args.append("--enforce-eager")
    if spec.max_model_len:
        args += ["--max-model-len", str(spec.max_model_len)]
    if spec.template:
        args += ["--chat-template", spec.template]
    return args


def serve(model, port: int, gpus: str, *, eager: bool = False, backend: str = "auto") -> None:
    spec = ServerSpec(str(model), gpus, port, eager, backend=backend)
    subprocess.run(command(spec), env=os.environ | {"CUDA_VISIBLE_DEVICES": gpus}, check=True)


class ServerPool:
    def __init__(self, root):
        self.root = Path(root)
        self.root.mkdir(parents=True, exist_ok=True)
        self.entries: dict[str, tuple] = {}

    def acquire(self, spec: ServerSpec, timeout: float = 300, launch=None) -> str:
        """Base URL of a ready server for ``spec`` (starting one if needed)."""
        key = spec.key()
        url = f"http://127.0.0.1:{spec.port}/v1"
        if key in self.entries:
            proc, log = self.entries[key]
            if proc.poll() is None:
                return url
            log.close()
            del self.entries[key]
        log = (self.root / f"{key}.log").open("ab")
        argv = launch(spec) if launch is not None else command(spec)
        proc = subprocess.Popen(argv, env=os.environ | {"CUDA_VISIBLE_DEVICES": spec.gpus}, stdout=log,
                                stderr=subprocess.STDOUT, start_new_session=True)
        self.entries[key] = (proc, log)
        deadline = time.monotonic() + timeout
        while time.monotonic() < deadline:
            if proc.poll() is not None:
                raise RuntimeError("Owned inference server exited; inspect its log")
            try:
                with urllib.request.urlopen(f"http://127.0.0.1:{spec.port}/health", timeout=1):
                    return url
            except OSError:
                time.sleep(0.2)
        self.close()
        raise TimeoutError("Server readiness timeout")

    def close(self) -> None:
        for proc, log in self.entries.values():
            if proc.poll() is None:
                os.killpg(proc.pid, signal.SIGTERM)
                try:
                    proc.wait(timeout=30)
                except subprocess.TimeoutExpired:
                    os.killpg(proc.pid, signal.SIGKILL)
                    proc.wait()
            log.close()
        self.entries.clear()
