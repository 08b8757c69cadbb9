"""The serving shell (qwen35_b200.serve) against the reference's protocols, with a stand-in engine (no GPU):
the daemon line protocol of models/qwen35_27b/test/test_dflash.cpp:902-946, 1874-1879 and the two HTTP routes of
models/qwen35_27b/scripts/server.py:79-199."""
import io
import json
import os
import struct

import pytest

from qwen35_b200 import serve


class CountingEngine(serve.Engine):
    """Generates prompt[-1] + 1, + 2, ...; records every call."""
    max_ctx = 64
    block = 4

    def __init__(self):
        self.calls = []

    def generate(self, prompt_ids, n_gen):
        self.calls.append((list(prompt_ids), n_gen))
        for i in range(n_gen):
            yield prompt_ids[-1] + 1 + i


def _write_prompt(path, ids):
    with open(path, "wb") as f:
        f.write(struct.pack("<%di" % len(ids), *ids))


def _read_stream(fd):
    out = []
    while True:
        b = os.read(fd, 4)
        if len(b) < 4:
            break
        out.append(struct.unpack("<i", b)[0])
    return out


def test_daemon_protocol_frames_tokens_and_terminates_every_request(tmp_path):
    eng = CountingEngine()
    p1, p2, p3 = str(tmp_path / "a.bin"), str(tmp_path / "b.bin"), str(tmp_path / "empty.bin")
    _write_prompt(p1, [5, 6, 7])
    _write_prompt(p2, list(range(60)))           # 60 + 8 + block 4 > max_ctx 64: rejected
    _write_prompt(p3, [])
    r, w = os.pipe()
    lines = io.StringIO(f"{p1} 4\nnot a request line with three fields\n{p2} 8\n{p3} 3\n{tmp_path / 'missing.bin'} 2\n{p1} 2\n")
    log = io.StringIO()
    served = serve.run_daemon(eng, stdin=lines, stream_fd=w, stdout=log)
    os.close(w)
    got = _read_stream(r)
    os.close(r)
    assert log.getvalue().startswith("[daemon] ready\n")
    # request 1: four tokens then -1; the over-long, the empty and the missing prompt: -1 alone each; request 6: two tokens, -1
    assert got == [8, 9, 10, 11, -1, -1, -1, -1, 8, 9, -1]
    assert served == 4 and eng.calls == [([5, 6, 7], 4), ([5, 6, 7], 2)]


def test_daemon_stops_at_the_end_of_sequence_id_and_survives_engine_errors(tmp_path):
    class Eos(serve.Engine):
        max_ctx, block = 64, 0

        def generate(self, prompt_ids, n_gen):
            yield 1
            yield serve.EOS_TOKEN_ID
            yield 2

    class Broken(serve.Engine):
        max_ctx, block = 64, 0

        def generate(self, prompt_ids, n_gen):
            yield 3
            raise RuntimeError("device status 1")

    out = []
    assert serve.run_request(Eos(), [1], 5, out.append) == 2
    assert out == [1, serve.EOS_TOKEN_ID, -1]
    out = []
    assert serve.run_request(Broken(), [1], 5, out.append) == 0
    assert out == [3, -1]                          # the stream is terminated whatever happened


def test_spec_engine_emits_exactly_n_tokens_from_multi_token_rounds():
    class FakeSpec:
        def __init__(self):
            self.k = 100

        def prefill(self, ids):
            return 100

        def step(self):
            self.k += 3
            return [self.k - 2, self.k - 1, self.k]          # three tokens per round

    eng = serve.SpecEngine(FakeSpec, max_ctx=64, block=16)
    assert list(eng.generate([1, 2], 5)) == [100, 101, 102, 103, 104]
    assert list(eng.generate([1, 2], 1)) == [100]


def test_http_routes():
    pytest.importorskip("httpx")
    from fastapi.testclient import TestClient
    eng = CountingEngine()
    app = serve.build_app(eng, stop_ids={13})
    c = TestClient(app)
    assert c.get("/v1/models").json()["data"][0]["id"] == serve.MODEL_NAME
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "7 8 9"}], "max_tokens": 6})
    body = r.json()
    assert r.status_code == 200 and body["object"] == "chat.completion"
    assert body["choices"][0]["message"]["content"].split() == ["10", "11", "12"]          # 13 is a stop id: dropped, generation ends
    assert body["usage"] == {"prompt_tokens": 3, "completion_tokens": 3, "total_tokens": 6}
    # ids instead of text; max_tokens clamped to max_ctx - prompt - block = 64 - 50 - 4
    r = c.post("/v1/chat/completions", json={"prompt_token_ids": list(range(100, 150)), "max_tokens": 500})
    assert r.status_code == 200 and eng.calls[-1][1] == 10
    r = c.post("/v1/chat/completions", json={"prompt_token_ids": list(range(70)), "max_tokens": 5})
    assert r.status_code == 400 and "exceeds max_ctx" in r.json()["detail"]
    # streaming: role chunk, one chunk per token, a stop chunk, [DONE]
    with c.stream("POST", "/v1/chat/completions", json={"prompt_token_ids": [20], "max_tokens": 3, "stream": True}) as s:
        events = [l[6:] for l in s.iter_lines() if l.startswith("data: ")]
    assert events[-1] == "[DONE]"
    chunks = [json.loads(e) for e in events[:-1]]
    assert chunks[0]["choices"][0]["delta"] == {"role": "assistant"}
    assert [ch["choices"][0]["delta"].get("content", "").strip() for ch in chunks[1:-1]] == ["21", "22", "23"]
    assert chunks[-1]["choices"][0]["finish_reason"] == "stop"
