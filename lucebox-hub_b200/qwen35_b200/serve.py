"""Serving shell around the decode engines: the reference's daemon line protocol and its OpenAI-compatible HTTP front.

Reference behaviour restated here:
  * daemon loop (models/qwen35_27b/test/test_dflash.cpp:902-946, 1345, 1874-1879): print "[daemon] ready", then per
    request read one line "<prompt file> <n_gen>" from stdin, start from a fresh cache (weights stay resident), read
    the prompt as little-endian int32 ids, generate, write every generated token as a little-endian int32 to the
    stream file descriptor and finish the request with -1; a bad request (unreadable or empty prompt, prompt + n_gen
    beyond the context) is answered with -1 alone; generation stops at the end-of-sequence id;
  * HTTP front (models/qwen35_27b/scripts/server.py:64-199): GET /v1/models, POST /v1/chat/completions with and
    without server-sent-event streaming, one request at a time, max_tokens clamped to the context that is left, stop
    ids filtered from the output.

Differences.  The reference spawns its C++ binary and talks to it over a pipe; here the engine lives in the same
process behind a small protocol (`reset()`, `generate(prompt_ids, n_gen)` yielding token ids), so the HTTP front
can call it directly, and `run_daemon` offers the pipe protocol for hosts that want the reference's process boundary.
No tokenizer ships with this repository (none can be downloaded where it is built): the front takes any object with
`encode` / `decode` / optionally `apply_chat_template` (a HuggingFace tokenizer fits), and a request may carry
`prompt_token_ids` instead of text.
"""
from __future__ import annotations

import json
import os
import struct
import sys
import threading
import time
import uuid
from typing import Iterable, Iterator, List, Optional, Sequence

EOS_TOKEN_ID = 248045          # test_dflash.cpp:1346
MODEL_NAME = "qwen35-b200"


class Engine:
    """What the shell needs from a decode engine.  `generate` starts from a fresh cache and yields generated ids."""

    max_ctx: int = 0
    block: int = 0             # positions the engine needs beyond prompt + n_gen (the draft block of the speculative loop)

    def generate(self, prompt_ids: Sequence[int], n_gen: int) -> Iterator[int]:
        raise NotImplementedError


class DecoderEngine(Engine):
    """Batch-1 greedy decoding on qwen35_b200.model.Decoder (prefill, then one token per step)."""

    def __init__(self, decoder):
        self.dec = decoder
        self.max_ctx = decoder.max_seq_len

    def generate(self, prompt_ids, n_gen):
        import torch
        ids = torch.tensor(list(prompt_ids), dtype=torch.int32, device=self.dec.device)
        tok = self.dec.prefill_tokens(ids)          # resets the state first
        for i in range(n_gen):
            yield int(tok)
            if i + 1 < n_gen:
                tok = self.dec.step(int(tok))


class SpecEngine(Engine):
    """Speculative decoding on qwen35_b200.spec_decode.SpecDecoder (draft -> tree -> verify -> commit rounds)."""

    def __init__(self, spec_decoder_factory, max_ctx: int, block: int = 16):
        self.factory = spec_decoder_factory      # builds a SpecDecoder on a fresh target cache; weights stay resident
        self.max_ctx, self.block = int(max_ctx), int(block)

    def generate(self, prompt_ids, n_gen):
        sd = self.factory()
        out = [sd.prefill(list(prompt_ids))]
        sent = 0
        while sent < n_gen:
            while sent < len(out) and sent < n_gen:
                yield int(out[sent])
                sent += 1
            if sent < n_gen:
                out.extend(sd.step())


def read_int32_file(path: str) -> List[int]:
    with open(path, "rb") as f:
        raw = f.read()
    n = len(raw) // 4
    return list(struct.unpack("<%di" % n, raw[:4 * n]))


def run_request(engine: Engine, prompt_ids: Sequence[int], n_gen: int, emit, eos_id: Optional[int] = EOS_TOKEN_ID) -> int:
    """One request of the daemon protocol: emit(token) per generated token, emit(-1) at the end.  Returns the number of
    tokens generated.  A request that cannot run is answered with -1 alone."""
    try:
        if not prompt_ids or n_gen <= 0 or len(prompt_ids) + n_gen + engine.block > engine.max_ctx:
            print(f"[daemon] rejected: prompt {len(prompt_ids)} + gen {n_gen} + block {engine.block} vs max_ctx {engine.max_ctx}", file=sys.stderr)
            emit(-1)
            return 0
        n = 0
        for tok in engine.generate(prompt_ids, n_gen):
            emit(int(tok))
            n += 1
            if eos_id is not None and int(tok) == eos_id:
                break
        emit(-1)
        return n
    except Exception as exc:                      # the stream must always be terminated, whatever the engine raised
        print(f"[daemon] request failed: {exc!r}", file=sys.stderr)
        emit(-1)
        return 0


def run_daemon(engine: Engine, stdin=None, stream_fd: int = -1, stdout=None, eos_id: Optional[int] = EOS_TOKEN_ID) -> int:
    """The reference's daemon loop.  Reads request lines until end of input; returns the number of requests served."""
    stdin = stdin if stdin is not None else sys.stdin
    stdout = stdout if stdout is not None else sys.stdout

    def emit(tok: int):
        if stream_fd >= 0:
            os.write(stream_fd, struct.pack("<i", int(tok)))

    print("[daemon] ready", file=stdout, flush=True)
    served = 0
    for line in stdin:
        parts = line.split()
        if len(parts) != 2:
            continue                               # the reference skips lines it cannot parse
        try:
            n_gen = int(parts[1])
            prompt = read_int32_file(parts[0])
        except (OSError, ValueError):
            print("[daemon] unreadable request:", line.strip(), file=sys.stderr)
            emit(-1)
            continue
        print(f"[prompt] {len(prompt)} tokens", file=stdout, flush=True)
        n = run_request(engine, prompt, n_gen, emit, eos_id)
        print(f"[daemon] generated {n} tokens", file=stdout, flush=True)
        served += 1
    return served


class IdTokenizer:
    """Stand-in tokenizer for hosts without a vocabulary: text is a whitespace-separated list of token ids."""

    def encode(self, text: str, add_special_tokens: bool = False) -> List[int]:
        return [int(t) for t in text.split()]

    def decode(self, ids: Iterable[int], skip_special_tokens: bool = True) -> str:
        return "".join(f"{int(i)} " for i in ids)


_MODELS = None


def _request_models():
    """The request schema (pydantic), built on first use so that the daemon path needs neither pydantic nor fastapi."""
    global _MODELS
    if _MODELS is None:
        from pydantic import BaseModel

        class ChatMessage(BaseModel):
            role: str
            content: str

        class ChatRequest(BaseModel):
            model: str = MODEL_NAME
            messages: List[ChatMessage] = []
            prompt_token_ids: Optional[List[int]] = None      # extension: ids instead of text
            stream: bool = False
            max_tokens: int = 512
            temperature: Optional[float] = None                # accepted and ignored: greedy only, like the reference
            top_p: Optional[float] = None

        _MODELS = (ChatMessage, ChatRequest)
    return _MODELS


def build_app(engine: Engine, tokenizer=None, stop_ids: Optional[set] = None, model_name: str = MODEL_NAME):
    """FastAPI application with the reference's two routes.  One generation at a time (a lock serialises requests, as the
    reference's single daemon does)."""
    from fastapi import FastAPI
    from fastapi.responses import JSONResponse, StreamingResponse

    ChatRequest = _request_models()[1]
    tokenizer = tokenizer or IdTokenizer()
    stop = set(stop_ids) if stop_ids is not None else {EOS_TOKEN_ID}
    lock = threading.Lock()
    app = FastAPI(title="qwen35_b200 OpenAI-compatible server")

    def prompt_ids_of(req) -> List[int]:
        if req.prompt_token_ids is not None:
            return [int(t) for t in req.prompt_token_ids]
        msgs = [m.model_dump() for m in req.messages]
        if hasattr(tokenizer, "apply_chat_template"):
            text = tokenizer.apply_chat_template(msgs, tokenize=False, add_generation_prompt=True)
        else:
            text = " ".join(m["content"] for m in msgs)
        return list(tokenizer.encode(text, add_special_tokens=False))

    def tokens_of(ids: List[int], n_gen: int) -> Iterator[int]:
        for tok in engine.generate(ids, n_gen):
            if tok in stop:
                return
            yield int(tok)

    @app.get("/v1/models")
    def list_models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "qwen35_b200"}]}

    def chat_completions(req):
        try:
            ids = prompt_ids_of(req)
        except ValueError as exc:
            return JSONResponse({"detail": f"cannot tokenise the prompt: {exc}"}, status_code=400)
        available = engine.max_ctx - len(ids) - engine.block
        n_gen = min(int(req.max_tokens), available)
        if not ids or n_gen <= 0:
            return JSONResponse({"detail": f"Prompt length ({len(ids)}) exceeds max_ctx ({engine.max_ctx})"}, status_code=400)
        cid = "chatcmpl-" + uuid.uuid4().hex[:24]
        created = int(time.time())

        def chunk(delta, finish=None):
            return "data: " + json.dumps({"id": cid, "object": "chat.completion.chunk", "created": created, "model": model_name,
                                          "choices": [{"index": 0, "delta": delta, "finish_reason": finish}]}) + "\n\n"

        if req.stream:
            def sse():
                with lock:
                    yield chunk({"role": "assistant"})
                    for tok in tokens_of(ids, n_gen):
                        yield chunk({"content": tokenizer.decode([tok])})
                    yield chunk({}, "stop")
                    yield "data: [DONE]\n\n"
            return StreamingResponse(sse(), media_type="text/event-stream")
        with lock:
            toks = list(tokens_of(ids, n_gen))
        return JSONResponse({"id": cid, "object": "chat.completion", "created": created, "model": model_name,
                             "choices": [{"index": 0, "message": {"role": "assistant", "content": tokenizer.decode(toks, skip_special_tokens=True)},
                                          "finish_reason": "stop"}],
                             "usage": {"prompt_tokens": len(ids), "completion_tokens": len(toks), "total_tokens": len(ids) + len(toks)}})

    chat_completions.__annotations__ = {"req": ChatRequest}        # the body model, resolved (annotations here are strings otherwise)
    app.post("/v1/chat/completions")(chat_completions)
    return app


def main(argv=None):
    """python -m qwen35_b200.serve --daemon [--stream-fd N] | --port P   (random-init 0.8B weights unless --weights PATH)"""
    import argparse
    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("--weights", default="random:1234", help="'random:<seed>' or a local HuggingFace checkpoint directory / .safetensors file")
    ap.add_argument("--max-ctx", type=int, default=4096)
    ap.add_argument("--daemon", action="store_true", help="serve the line protocol on stdin / --stream-fd")
    ap.add_argument("--stream-fd", type=int, default=-1)
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--host", default="127.0.0.1")
    args = ap.parse_args(argv)
    from .model import Decoder, load_weights
    weights, _ = load_weights(args.weights)
    engine = DecoderEngine(Decoder(weights=weights, max_seq_len=args.max_ctx))
    if args.daemon:
        run_daemon(engine, stream_fd=args.stream_fd)
        return 0
    import uvicorn
    uvicorn.run(build_app(engine), host=args.host, port=args.port)
    return 0


if __name__ == "__main__":
    sys.exit(main())
