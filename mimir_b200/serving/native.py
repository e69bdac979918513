"""Native OpenAI-compatible serving of exported Mimir2 models (no vLLM).

The vLLM server that the reference launches (``src/mimir/serving/server.py:12-75``) needs its
patched vLLM fork (``patches/vllm.patch``) to know Mimir2.  This server instead loads the export
with this framework's Transformers model (:mod:`mimir_b200.export.transformers_mimir2`), which
serves every configuration the exporter writes, including looped recurrence, exactly as trained:
the prompt is the prefix-LM prefix (its tokens see each other), generation is causal with a
per-invocation KV cache.

Endpoints (the subset the evaluation runner and the serving pool use):

* ``GET  /health``, ``GET /v1/models``
* ``POST /v1/chat/completions`` (``messages``; the export's chat template; ``chat_template_kwargs``)
* ``POST /v1/completions`` (``prompt``)
* ``"stream": true`` on either POST: server-sent events (``chat.completion.chunk`` /
  ``text_completion`` chunks, then ``data: [DONE]``), decoded text sent as it is generated.

Request fields: ``max_tokens``, ``temperature`` (0 = greedy), ``top_p``, ``stop``, ``seed``.
The HTTP server accepts concurrent connections.  Requests without a seed are batched: a worker
thread takes what has queued up with the same decoding rule (greedy, or one temperature/top-p;
up to ``--max-batch`` requests, waiting at most ``--batch-wait-ms`` after the first), left-pads
the prompts into one batch (the model hides padding keys and counts positions from each prompt's
first token) and decodes them together, which gives each greedy request its own greedy
continuation and each sampled request independent samples.  Seeded or streamed requests run one
at a time.

Usage: ``python -m mimir_b200.serving.native MODEL_DIR [--port 8000] [--device cuda:0]
[--max-batch 8] [--batch-wait-ms 5]``.
"""
from __future__ import annotations

import argparse
import json
import threading
import time
import uuid
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path
from typing import Optional

import torch


class _Pending:
    """One queued greedy request and, once its batch ran, its result (or the batch's error)."""

    def __init__(self, ids: list[int], body: dict):
        self.ids, self.body = ids, body
        self.done = threading.Event()
        self.result = None
        self.error: Optional[BaseException] = None


class Engine:
    """Tokenizer + model + a lock; ``complete`` returns ``(text, prompt_tokens, completion_tokens,
    finish_reason)``."""

    def __init__(self, model_dir, device: str = "cpu", dtype: Optional[torch.dtype] = None, name: Optional[str] = None,
                 max_batch: int = 8, batch_wait_ms: float = 5.0):
        from transformers import AutoModelForCausalLM, AutoTokenizer

        from mimir_b200.export.transformers_mimir2 import register
        register()
        self.name = name or Path(model_dir).name
        self.device = torch.device(device)
        self.tokenizer = AutoTokenizer.from_pretrained(model_dir, local_files_only=True)
        kwargs = {"dtype": dtype} if dtype is not None else {}
        self.model = AutoModelForCausalLM.from_pretrained(model_dir, local_files_only=True, **kwargs).to(self.device)
        self.model.eval()
        self.lock = threading.Lock()
        self.max_batch = max(1, int(max_batch))
        self.batch_wait = max(0.0, float(batch_wait_ms)) / 1000.0
        self.pad_id = (self.tokenizer.pad_token_id if self.tokenizer.pad_token_id is not None
                       else self.tokenizer.eos_token_id if self.tokenizer.eos_token_id is not None else 0)
        self._queue: list[_Pending] = []
        self._ready = threading.Condition()
        if self.max_batch > 1:
            threading.Thread(target=self._serve_batches, name="mimir-batcher", daemon=True).start()

    def prompt_ids(self, body: dict, chat: bool) -> list[int]:
        if chat:
            kw = dict(body.get("chat_template_kwargs") or {})
            text = self.tokenizer.apply_chat_template(body["messages"], tokenize=False, add_generation_prompt=True, **kw)
            return self.tokenizer(text, add_special_tokens=False)["input_ids"]
        prompt = body["prompt"]
        if isinstance(prompt, list) and prompt and isinstance(prompt[0], int):
            return list(prompt)
        return self.tokenizer(prompt if isinstance(prompt, str) else prompt[0])["input_ids"]

    @staticmethod
    def _max_tokens(body: dict) -> int:
        return int(body.get("max_tokens") or body.get("max_completion_tokens") or 16)

    def _gen_args(self, max_new: int) -> dict:
        gen = dict(max_new_tokens=max_new, pad_token_id=self.pad_id)
        if self.tokenizer.eos_token_id is not None:
            gen["eos_token_id"] = self.tokenizer.eos_token_id
        return gen

    def _finish(self, ids: list[int], new: list[int], body: dict) -> tuple[str, int, int, str]:
        max_tokens = self._max_tokens(body)
        eos = self.tokenizer.eos_token_id
        if eos is not None and eos in new:  # a batch row keeps padding after its end
            new = new[:new.index(eos) + 1]
        new = new[:max_tokens]
        finish = "length" if len(new) >= max_tokens else "stop"
        text = self.tokenizer.decode(new, skip_special_tokens=True)
        stops = body.get("stop") or []
        for s in [stops] if isinstance(stops, str) else list(stops):
            cut = text.find(s)
            if s and cut >= 0:
                text, finish = text[:cut], "stop"
        return text, len(ids), len(new), finish

    def batchable(self, body: dict) -> bool:
        return self.max_batch > 1 and body.get("seed") is None

    @staticmethod
    def _sampling(body: dict) -> tuple:
        """Requests share a batch only with the same decoding rule (greedy, or one temperature/top-p)."""
        temperature = float(body.get("temperature") or 0.0)
        return (temperature, float(body.get("top_p") or 1.0)) if temperature > 0 else (0.0, 1.0)

    @torch.no_grad()
    def complete(self, ids: list[int], body: dict) -> tuple[str, int, int, str]:
        if self.batchable(body):
            item = _Pending(ids, body)
            with self._ready:
                self._queue.append(item)
                self._ready.notify()
            item.done.wait()
            if item.error is not None:
                raise item.error
            return item.result
        temperature = float(body.get("temperature") or 0.0)
        gen = self._gen_args(self._max_tokens(body)) | dict(do_sample=temperature > 0)
        if temperature > 0:
            gen.update(temperature=temperature, top_p=float(body.get("top_p") or 1.0))
        with self.lock:
            if body.get("seed") is not None:
                torch.manual_seed(int(body["seed"]))
            x = torch.tensor([ids], device=self.device)
            out = self.model.generate(x, attention_mask=torch.ones_like(x), **gen)
        return self._finish(ids, out[0, len(ids):].tolist(), body)

    def stream(self, ids: list[int], body: dict):
        """Yield decoded text pieces as they are generated, then ``(None, result)`` where result
        is what :meth:`complete` returns (stop strings cut the text and end the stream early)."""
        from transformers import TextIteratorStreamer
        temperature = float(body.get("temperature") or 0.0)
        gen = self._gen_args(self._max_tokens(body)) | dict(do_sample=temperature > 0)
        if temperature > 0:
            gen.update(temperature=temperature, top_p=float(body.get("top_p") or 1.0))
        streamer = TextIteratorStreamer(self.tokenizer, skip_prompt=True, skip_special_tokens=True)
        holder: dict = {}

        def run():
            try:
                with self.lock, torch.no_grad():
                    if body.get("seed") is not None:
                        torch.manual_seed(int(body["seed"]))
                    x = torch.tensor([ids], device=self.device)
                    holder["out"] = self.model.generate(x, attention_mask=torch.ones_like(x), streamer=streamer, **gen)
            except BaseException as exc:  # reported to the reader below
                holder["error"] = exc
                streamer.end()

        worker = threading.Thread(target=run, daemon=True)
        worker.start()
        stops = body.get("stop") or []
        stops = [stops] if isinstance(stops, str) else [x for x in stops if x]
        sent, stopped = "", False
        for piece in streamer:
            if stopped:
                continue  # drain until generation ends
            text = sent + piece
            cut = min((text.find(x) for x in stops if x in text), default=-1)
            if cut >= 0:
                piece, stopped = text[len(sent):cut], True
            if piece:
                sent += piece
                yield piece, None
        worker.join()
        if "error" in holder:
            raise holder["error"]
        result = self._finish(ids, holder["out"][0, len(ids):].tolist(), body)
        yield None, (sent, result[1], result[2], "stop" if stopped else result[3])

    # ------------------------------------------------------------------ batched greedy decoding
    def _serve_batches(self) -> None:
        while True:
            with self._ready:
                while not self._queue:
                    self._ready.wait()
                rule = self._sampling(self._queue[0].body)

                def same():
                    return [item for item in self._queue if self._sampling(item.body) == rule][:self.max_batch]

                deadline = time.monotonic() + self.batch_wait
                while len(same()) < self.max_batch and time.monotonic() < deadline:
                    self._ready.wait(max(0.0, deadline - time.monotonic()))
                batch = same()
                taken = {id(item) for item in batch}
                self._queue = [item for item in self._queue if id(item) not in taken]
            try:
                for item, result in zip(batch, self._generate_batch(batch)):
                    item.result = result
            except BaseException as exc:  # the requests of a failed batch all report it
                for item in batch:
                    item.error = exc
            finally:
                for item in batch:
                    item.done.set()

    @torch.no_grad()
    def _generate_batch(self, batch: list[_Pending]) -> list:
        width = max(len(item.ids) for item in batch)
        x = torch.full((len(batch), width), self.pad_id, dtype=torch.long)
        mask = torch.zeros_like(x)
        for i, item in enumerate(batch):
            x[i, width - len(item.ids):] = torch.tensor(item.ids)
            mask[i, width - len(item.ids):] = 1
        temperature, top_p = self._sampling(batch[0].body)
        gen = self._gen_args(max(self._max_tokens(item.body) for item in batch)) | dict(do_sample=temperature > 0)
        if temperature > 0:
            gen.update(temperature=temperature, top_p=top_p)
        with self.lock:
            out = self.model.generate(x.to(self.device), attention_mask=mask.to(self.device), **gen)
        return [self._finish(item.ids, out[i, width:].tolist(), item.body) for i, item in enumerate(batch)]


def _handler(engine: Engine):
    class Handler(BaseHTTPRequestHandler):
        protocol_version = "HTTP/1.1"

        def log_message(self, fmt, *args):  # quiet by default
            pass

        def _send(self, code: int, payload: dict) -> None:
            data = json.dumps(payload).encode()
            self.send_response(code)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def do_GET(self):
            if self.path == "/health":
                self._send(200, {"status": "ok"})
            elif self.path == "/v1/models":
                self._send(200, {"object": "list", "data": [{"id": engine.name, "object": "model",
                                                             "owned_by": "mimir_b200"}]})
            else:
                self._send(404, {"error": {"message": f"unknown path {self.path}"}})

        def do_POST(self):
            try:
                body = json.loads(self.rfile.read(int(self.headers.get("Content-Length", 0))) or b"{}")
                chat = self.path == "/v1/chat/completions"
                if not chat and self.path != "/v1/completions":
                    return self._send(404, {"error": {"message": f"unknown path {self.path}"}})
                ids = engine.prompt_ids(body, chat)
                if body.get("stream"):
                    return self._stream(engine.stream(ids, body), chat)
                text, n_in, n_out, finish = engine.complete(ids, body)
            except (KeyError, ValueError, TypeError) as exc:
                return self._send(400, {"error": {"message": str(exc)}})
            usage = {"prompt_tokens": n_in, "completion_tokens": n_out, "total_tokens": n_in + n_out}
            base = {"id": f"cmpl-{uuid.uuid4().hex}", "created": int(time.time()), "model": engine.name,
                    "usage": usage}
            if chat:
                self._send(200, base | {"object": "chat.completion", "choices": [
                    {"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": finish}]})
            else:
                self._send(200, base | {"object": "text_completion", "choices": [
                    {"index": 0, "text": text, "finish_reason": finish}]})
        def _stream(self, pieces, chat: bool) -> None:
            cid, created = f"cmpl-{uuid.uuid4().hex}", int(time.time())
            kind = "chat.completion.chunk" if chat else "text_completion"
            self.send_response(200)
            self.send_header("Content-Type", "text/event-stream")
            self.send_header("Cache-Control", "no-cache")
            self.send_header("Connection", "close")
            self.end_headers()
            self.close_connection = True

            def event(payload) -> None:
                data = payload if isinstance(payload, str) else json.dumps(payload)
                self.wfile.write(f"data: {data}\n\n".encode())
                self.wfile.flush()

            def chunk(text, finish=None, usage=None):
                choice = ({"index": 0, "delta": {"content": text} if text else {}, "finish_reason": finish} if chat
                          else {"index": 0, "text": text or "", "finish_reason": finish})
                out = {"id": cid, "object": kind, "created": created, "model": engine.name, "choices": [choice]}
                return out | ({"usage": usage} if usage else {})

            if chat:
                event({"id": cid, "object": kind, "created": created, "model": engine.name,
                       "choices": [{"index": 0, "delta": {"role": "assistant"}, "finish_reason": None}]})
            for piece, result in pieces:
                if piece is not None:
                    event(chunk(piece))
                else:
                    _, n_in, n_out, finish = result
                    event(chunk(None, finish, {"prompt_tokens": n_in, "completion_tokens": n_out,
                                               "total_tokens": n_in + n_out}))
            event("[DONE]")
    return Handler


def make_server(engine: Engine, host: str = "127.0.0.1", port: int = 8000) -> ThreadingHTTPServer:
    return ThreadingHTTPServer((host, port), _handler(engine))


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="OpenAI-compatible server for an exported Mimir2 model")
    ap.add_argument("model", type=Path)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--dtype", choices=["float32", "bfloat16"], default=None)
    ap.add_argument("--max-batch", type=int, default=8, help="greedy requests decoded together (1: one at a time)")
    ap.add_argument("--batch-wait-ms", type=float, default=5.0, help="how long a batch waits for more requests")
    args = ap.parse_args(argv)
    engine = Engine(args.model, args.device, getattr(torch, args.dtype) if args.dtype else None,
                    max_batch=args.max_batch, batch_wait_ms=args.batch_wait_ms)
    server = make_server(engine, args.host, args.port)
    print(f"serving {engine.name} on http://{args.host}:{args.port}/v1", flush=True)
    server.serve_forever()


if __name__ == "__main__":
    main()
