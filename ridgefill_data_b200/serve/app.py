"""HTTP server over the scheduler (FastAPI + uvicorn): the llama.cpp server's request and stream layout for
`/completion` (kept alike so the 27B kit's clients and schedules run unchanged), plus `/health`, `/props` and a
Prometheus `/metrics`.

POST /completion  {"prompt": [ids] | "text", "n_predict": 16, "stream": false, "ridgefill_mode": "on" | "off"
                   (or "ridgefill": bool), "ignore_eos": false, ...}; other llama.cpp sampling fields (temperature 0,
                   top_k 1, seed, cache_prompt false, id_slot) are accepted and must mean greedy decoding.
  stream=false -> one JSON object: the final event with "tokens" = every generated id and "content" the text.
  stream=true  -> text/event-stream, one `data: {event}` per token and the final event (see serve/engine.py).
"""
from __future__ import annotations

import asyncio
import json

import torch

from .engine import Request


class BadRequest(ValueError):
    pass


def parse_body(body, arms, tokenizer=None):
    """(ids tensor, n_predict, arm, ignore_eos) from a request body; raises BadRequest."""
    prompt = body.get("prompt")
    if isinstance(prompt, str):
        if tokenizer is None:
            raise BadRequest("a text prompt needs the server's --tokenizer; send token ids instead")
        from ..eval.text import bos_ids, encode
        ids = bos_ids(tokenizer) + encode(tokenizer, prompt)
        if not ids:
            raise BadRequest("the text prompt encodes to no tokens")
    elif isinstance(prompt, list) and prompt and all(isinstance(t, int) for t in prompt):
        ids = prompt
    else:
        raise BadRequest("prompt: a non-empty list of token ids or a string")
    try:
        n_predict = int(body.get("n_predict", 16))
    except (TypeError, ValueError):
        raise BadRequest("n_predict must be an integer")
    if n_predict < 1:
        raise BadRequest("n_predict must be at least 1 (this server does not run prompt-only requests)")
    if float(body.get("temperature", 0) or 0) != 0 or int(body.get("top_k", 1) or 1) != 1:
        raise BadRequest("only greedy decoding (temperature 0, top_k 1) is served")
    if body.get("cache_prompt"):
        raise BadRequest("cache_prompt is not supported: every request prefills its whole prompt")
    mode = body.get("ridgefill_mode")
    if mode is None:
        mode = "on" if body.get("ridgefill", True) else "off"
    if mode not in arms:
        raise BadRequest(f"ridgefill_mode {mode!r}: one of {sorted(arms)}")
    return torch.tensor(ids, dtype=torch.long), n_predict, arms[mode], bool(body.get("ignore_eos", False))


def create_app(scheduler, arms, tokenizer=None, props=None):
    from fastapi import FastAPI
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    app = FastAPI(title="ridgefill-b200")
    detok = (lambda toks: tokenizer.decode(toks)) if tokenizer is not None else None

    @app.get("/health")
    def health():
        return {"status": "ok", **scheduler.load}

    @app.get("/props")
    def get_props():
        return dict(props or {}, modes=sorted(arms))

    @app.get("/metrics")
    def metrics():
        return PlainTextResponse(scheduler.metrics_text(), media_type="text/plain; version=0.0.4")

    @app.post("/completion")
    async def completion(body: dict):
        try:
            ids, n_predict, arm, ignore_eos = parse_body(body, arms, tokenizer)
        except BadRequest as e:
            return JSONResponse({"error": {"code": 400, "message": str(e)}}, status_code=400)
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        req = Request(ids=ids, n_predict=n_predict, arm=arm, ignore_eos=ignore_eos, detok=detok,
                      emit=lambda ev: loop.call_soon_threadsafe(q.put_nowait, ev))
        try:
            scheduler.submit(req)
        except ValueError as e:
            return JSONResponse({"error": {"code": 400, "message": str(e)}}, status_code=400)
        if body.get("stream"):
            async def events():
                while True:
                    ev = await q.get()
                    yield "data: " + json.dumps(ev) + "\n\n"
                    if ev.get("stop"):
                        break
            return StreamingResponse(events(), media_type="text/event-stream")
        toks, text = [], []
        while True:
            ev = await q.get()
            if "error" in ev:
                return JSONResponse({"error": {"code": 500, "message": ev["error"]}}, status_code=500)
            if ev.get("stop"):
                return dict(ev, tokens=toks, content="".join(text))
            toks += ev["tokens"]
            text.append(ev.get("content", ""))

    return app


class Server:
    """uvicorn in a background thread (tests, notebooks) or in the foreground (the CLI)."""

    def __init__(self, app, host="127.0.0.1", port=8080, log_level="warning"):
        import uvicorn
        self.config = uvicorn.Config(app, host=host, port=port, log_level=log_level, lifespan="off")
        self.server = uvicorn.Server(self.config)
        self.thread = None

    def start(self, timeout=30):
        import threading
        import time
        self.thread = threading.Thread(target=self.server.run, daemon=True)
        self.thread.start()
        t0 = time.monotonic()
        while not self.server.started:
            if time.monotonic() - t0 > timeout or not self.thread.is_alive():
                raise RuntimeError("the HTTP server did not start")
            time.sleep(0.02)
        return self

    @property
    def port(self):
        for s in self.server.servers:
            for sock in s.sockets:
                return sock.getsockname()[1]
        return self.config.port

    def stop(self):
        self.server.should_exit = True
        if self.thread is not None:
            self.thread.join(10)

    def run(self):
        self.server.run()
