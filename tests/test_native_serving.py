"""Native OpenAI-compatible serving of an export (``mimir_b200.serving.native``), CPU: the HTTP
endpoints answer in the OpenAI schema and the greedy completion equals the Transformers model's
own ``generate`` on the same prompt (prompt = prefix-LM prefix)."""
import json
import threading
import urllib.request

import pytest
import torch

pytest.importorskip("transformers")


def _tokenizer(path):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    vocab = {f"w{i}": i for i in range(90)} | {"<unk>": 90, "<s>": 91, "</s>": 92, "user": 93, "assistant": 94, ":": 95}
    tok = Tokenizer(models.WordLevel(vocab, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="<unk>", bos_token="<s>", eos_token="</s>")
    fast.chat_template = ("{% for m in messages %}{{ m['role'] }} : {{ m['content'] }} {% endfor %}"
                          "{% if add_generation_prompt %}assistant : {% endif %}")
    fast.save_pretrained(path)


def _post(url, body):
    req = urllib.request.Request(url, data=json.dumps(body).encode(), headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=60) as r:
        return json.loads(r.read())


def _stream(url, body):
    """POST with ``stream``: the server-sent events' payloads (JSON objects, then ``[DONE]``)."""
    req = urllib.request.Request(url, data=json.dumps(body).encode(), headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=60) as r:
        assert r.headers["Content-Type"] == "text/event-stream"
        lines = [line.decode().strip() for line in r.read().splitlines()]
    data = [line[len("data: "):] for line in lines if line.startswith("data: ")]
    return [d if d == "[DONE]" else json.loads(d) for d in data]


def test_native_server_answers_like_generate(tmp_path):
    from test_transformers_model import _export

    from mimir_b200.serving.native import Engine, make_server
    _export(tmp_path, {})
    _tokenizer(tmp_path)
    engine = Engine(tmp_path, "cpu", name="tiny")
    server = make_server(engine, "127.0.0.1", 0)
    thread = threading.Thread(target=server.serve_forever, daemon=True)
    thread.start()
    base = f"http://127.0.0.1:{server.server_address[1]}"
    try:
        with urllib.request.urlopen(base + "/health", timeout=10) as r:
            assert json.loads(r.read()) == {"status": "ok"}
        with urllib.request.urlopen(base + "/v1/models", timeout=10) as r:
            assert json.loads(r.read())["data"][0]["id"] == "tiny"
        chat = _post(base + "/v1/chat/completions", {"model": "tiny", "max_tokens": 4, "temperature": 0,
                                                     "messages": [{"role": "user", "content": "w1 w2 w3"}]})
        assert chat["object"] == "chat.completion" and chat["choices"][0]["message"]["role"] == "assistant"
        assert chat["usage"]["completion_tokens"] <= 4
        ids = engine.prompt_ids({"messages": [{"role": "user", "content": "w1 w2 w3"}]}, chat=True)
        out = engine.model.generate(torch.tensor([ids]), max_new_tokens=4, do_sample=False, pad_token_id=92,
                                    eos_token_id=92)
        expected = engine.tokenizer.decode(out[0, len(ids):].tolist(), skip_special_tokens=True)
        assert chat["choices"][0]["message"]["content"] == expected
        text = _post(base + "/v1/completions", {"prompt": "w5 w6", "max_tokens": 3})
        assert text["object"] == "text_completion" and isinstance(text["choices"][0]["text"], str)
        streamed = _stream(base + "/v1/chat/completions", {"model": "tiny", "max_tokens": 4, "temperature": 0,
                                                           "stream": True,
                                                           "messages": [{"role": "user", "content": "w1 w2 w3"}]})
        assert streamed[-1] == "[DONE]" and streamed[0]["choices"][0]["delta"] == {"role": "assistant"}
        chunks = streamed[1:-1]
        assert all(c["object"] == "chat.completion.chunk" for c in chunks)
        assert "".join(c["choices"][0]["delta"].get("content", "") for c in chunks) == expected
        assert chunks[-1]["choices"][0]["finish_reason"] == chat["choices"][0]["finish_reason"]
        assert chunks[-1]["usage"] == chat["usage"]
        plain = _stream(base + "/v1/completions", {"prompt": "w5 w6", "max_tokens": 3, "stream": True})
        assert "".join(c["choices"][0]["text"] for c in plain[:-1]) == text["choices"][0]["text"]
        full = text["choices"][0]["text"]
        if len(full.split()) > 1:  # a stop string cuts the stream where it cuts the plain answer
            stop = full.split()[1]
            cut = _post(base + "/v1/completions", {"prompt": "w5 w6", "max_tokens": 3, "stop": [stop]})
            streamed_cut = _stream(base + "/v1/completions", {"prompt": "w5 w6", "max_tokens": 3, "stop": [stop],
                                                              "stream": True})
            assert "".join(c["choices"][0]["text"] for c in streamed_cut[:-1]) == cut["choices"][0]["text"]
            assert streamed_cut[-2]["choices"][0]["finish_reason"] == "stop"
    finally:
        server.shutdown()
        server.server_close()


def test_native_backend_command(tmp_path):
    from mimir_b200.serving.server import ServerSpec, command
    (tmp_path / "config.json").write_text(json.dumps({"model_type": "mimir2", "recurrence_mode": "looped"}))
    argv = command(ServerSpec(str(tmp_path), "3", 8123, backend="native"))
    assert argv[1:4] == ["-m", "mimir_b200.serving.native", str(tmp_path)] and "8123" in argv
    with pytest.raises(ValueError, match="exactly one"):
        command(ServerSpec(str(tmp_path), "0,1", backend="native"))
    with pytest.raises(ValueError, match="Looped"):  # the vLLM command keeps its own limits
        command(ServerSpec(str(tmp_path), "0", backend="vllm"))
    import mimir_b200.serving.server as server
    original = server.vllm_knows_mimir2
    try:  # auto: native unless vLLM registers the architecture
        server.vllm_knows_mimir2 = lambda: False
        assert command(ServerSpec(str(tmp_path), "2"))[1:3] == ["-m", "mimir_b200.serving.native"]
        server.vllm_knows_mimir2 = lambda: True
        with pytest.raises(ValueError, match="Looped"):
            command(ServerSpec(str(tmp_path), "2"))
    finally:
        server.vllm_knows_mimir2 = original


def test_concurrent_greedy_requests_are_batched_and_match_single_requests(tmp_path):
    from test_transformers_model import _export

    from mimir_b200.serving.native import Engine
    _export(tmp_path, {})
    _tokenizer(tmp_path)
    engine = Engine(tmp_path, "cpu", name="tiny", max_batch=4, batch_wait_ms=200)
    single = Engine(tmp_path, "cpu", name="tiny", max_batch=1)
    bodies = [{"messages": [{"role": "user", "content": c}], "max_tokens": m}
              for c, m in (("w1 w2 w3 w4 w5 w6", 5), ("w7", 3), ("w8 w9 w10", 6))]
    sizes = []
    real = engine._generate_batch
    engine._generate_batch = lambda batch: (sizes.append(len(batch)), real(batch))[1]
    results = [None] * len(bodies)

    def ask(i):
        results[i] = engine.complete(engine.prompt_ids(bodies[i], chat=True), bodies[i])

    threads = [threading.Thread(target=ask, args=(i,)) for i in range(len(bodies))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert sizes and max(sizes) > 1, sizes  # at least two requests shared a batch
    for body, got in zip(bodies, results):
        assert got == single.complete(single.prompt_ids(body, chat=True), body), (body, got)
        assert got[2] <= body["max_tokens"]


def test_batches_never_mix_decoding_rules(tmp_path):
    from test_transformers_model import _export

    from mimir_b200.serving.native import Engine
    _export(tmp_path, {})
    _tokenizer(tmp_path)
    engine = Engine(tmp_path, "cpu", name="tiny", max_batch=4, batch_wait_ms=200)
    single = Engine(tmp_path, "cpu", name="tiny", max_batch=1)
    rules = []
    real = engine._generate_batch
    engine._generate_batch = lambda batch: (rules.append({engine._sampling(i.body) for i in batch}), real(batch))[1]
    bodies = [{"prompt": f"w{i} w{i + 1}", "max_tokens": 4, "temperature": t}
              for i, t in enumerate((0, 0.8, 0, 0.8, 0))]
    results = [None] * len(bodies)

    def ask(i):
        results[i] = engine.complete(engine.prompt_ids(bodies[i], chat=False), bodies[i])

    threads = [threading.Thread(target=ask, args=(i,)) for i in range(len(bodies))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert rules and all(len(r) == 1 for r in rules) and len(rules) < len(bodies), rules
    for body, got in zip(bodies, results):
        assert got is not None and got[2] <= body["max_tokens"]
        if body["temperature"] == 0:
            assert got == single.complete(single.prompt_ids(body, chat=False), body)
