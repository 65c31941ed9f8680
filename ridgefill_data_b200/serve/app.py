"""HTTP server over the scheduler (FastAPI + uvicorn): the llama.cpp server's request and stream layout for
`/completion` (kept alike so the 27B kit's clients and schedules run unchanged), plus `/health`, `/props` and a
Prometheus `/metrics`.

POST /tokenize, /detokenize  text <-> ids with the server's tokenizer (llama.cpp's and vLLM's field names)
POST /completion  {"prompt": [ids] | "text", "n_predict": 16, "stream": false, "ridgefill_mode": "on" | "off"
                   (or "ridgefill": bool), "ignore_eos": false, ...}; other llama.cpp sampling fields (temperature 0,
                   top_k 1, seed, cache_prompt false, id_slot) are accepted and must mean greedy decoding.
  stream=false -> one JSON object: the final event with "tokens" = every generated id and "content" the text.
  stream=true  -> text/event-stream, one `data: {event}` per token and the final event (see serve/engine.py).
OpenAI-compatible (the API the c5 kit's client and the LongBench v2 runner speak):
  GET  /v1/models
  POST /v1/completions       {"prompt": "text" | [ids] | a list of those (one choice each, non-streamed),
                              "max_tokens", "stream", "stop", "ridgefill_mode",
                              "prompt_logprobs": k (vLLM's field: the log-prob and rank of every prompt token given
                              its prefix, plus the k most likely tokens), "vllm_xargs": {"dyluhn_kva": "0" | "1",
                              "dyluhn_kva_tail": T} (the c5 kit's per-request RidgeFill switch: off / on),
                              "echo" + "logprobs": k (OpenAI's legacy log-probs of the echoed prompt; with
                              max_tokens 0 a scoring request, as evaluation harnesses send for log-likelihoods)}
  POST /v1/chat/completions  {"messages": [...], "max_tokens", "stream", "stop", "ridgefill_mode"} (the tokenizer's
                             chat template renders the prompt)
  Responses carry choices[0].text / .message.content, finish_reason ("stop" | "length") and usage token counts
  (plus prompt_filled_tokens, the prompt rows approximated from the maps: the request's real tail is the rest);
  streams are chunk objects ending with `data: [DONE]`. Greedy decoding only. Text is detokenized incrementally
  (the decoded prefix grows; a trailing partial character is held back), so multi-byte pieces stream correctly.
  prompt_logprobs: choices[0].prompt_logprobs holds one entry per prompt token, the first None, the others
  {str(id): {"logprob", "rank", "decoded_token"}} (and the k alternatives). Only rows that run through every layer
  have logits: under RidgeFill those are the exact tail, so the entries of the filled prefix carry "logprob": null
  (as do positions before the last MAX_SCORED_ROWS); an exact request scores every position.
"""

import asyncio
import json

import torch

from .engine import Request, ServerBusy


class BadRequest(ValueError):
    pass


class ClientGone(Exception):
    """The HTTP client disconnected while its non-streamed request was running."""


async def _next_event(q, http_req=None, poll_s=0.5):
    """The request's next event; with the HTTP request, at least every poll_s (also while events keep arriving)
    checks that its client is still connected."""
    if http_req is None:
        return await q.get()
    loop = asyncio.get_running_loop()
    last = getattr(http_req.state, "rf_checked", None)
    if last is None:
        last = http_req.state.rf_checked = loop.time()
    while True:
        if loop.time() - last >= poll_s:
            last = http_req.state.rf_checked = loop.time()
            if await http_req.is_disconnected():
                raise ClientGone()
        try:
            return await asyncio.wait_for(q.get(), max(1e-3, poll_s - (loop.time() - last)))
        except asyncio.TimeoutError:
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


class Detok:
    """Incremental detokenizer: the text of all ids so far, emitted as deltas (a trailing U+FFFD, an unfinished
    multi-byte character, is held back until the next token completes it)."""

    def __init__(self, tokenizer):
        self.tok = tokenizer
        self.ids, self.sent = [], ""

    def push(self, ids):
        if self.tok is None:
            return ""
        self.ids += list(ids)
        # JSON-safe text: a lone surrogate (a tokenizer that maps ids to raw code points) becomes "?"
        text = self.tok.decode(self.ids, skip_special_tokens=True).encode("utf-8", "replace").decode("utf-8")
        if text.endswith("\ufffd"):
            return ""
        delta = text[len(self.sent):] if text.startswith(self.sent) else text
        self.sent = text
        return delta


def _greedy_only(body):
    if float(body.get("temperature", 0) or 0) != 0 or int(body.get("top_k", 1) or 1) not in (1, -1) \
            or float(body.get("top_p", 1) or 1) != 1:
        raise BadRequest("only greedy decoding (temperature 0) is served")
    if int(body.get("n", 1) or 1) != 1 or int(body.get("best_of", 1) or 1) != 1:
        raise BadRequest("n / best_of: one greedy completion per request")
    if float(body.get("presence_penalty", 0) or 0) != 0 or float(body.get("frequency_penalty", 0) or 0) != 0 \
            or body.get("logit_bias"):
        raise BadRequest("presence / frequency penalties and logit_bias are not served (greedy decoding)")


def _mode(body, arms):
    xargs = body.get("vllm_xargs") or {}
    if not isinstance(xargs, dict):
        raise BadRequest("vllm_xargs: an object")
    default = "on" if body.get("ridgefill", True) else "off"
    if "dyluhn_kva" in xargs:                           # the c5 kit's switch: "1" RidgeFill, "0" exact
        default = "on" if str(xargs["dyluhn_kva"]) == "1" else "off"
    mode = body.get("ridgefill_mode", default)
    if mode not in arms:
        raise BadRequest(f"ridgefill_mode {mode!r}: one of {sorted(arms)}")
    if "dyluhn_kva_tail" in xargs and mode != "off":
        tail = getattr(arms[mode], "tail", None)
        if tail is None or int(xargs["dyluhn_kva_tail"]) != int(tail):
            raise BadRequest(f"dyluhn_kva_tail {xargs['dyluhn_kva_tail']}: this server's RidgeFill tail is {tail}")
    if float(body.get("repetition_penalty", 1.0) or 1.0) != 1.0:
        raise BadRequest("repetition_penalty: only 1.0 (greedy decoding) is served")
    return arms[mode]


def _prompt_logprobs(body):
    """-1 when the request asks for no prompt log-probs, else the number of alternatives per position (<= 20)."""
    v = body.get("prompt_logprobs")
    if v is None or v is False:
        return -1
    try:
        k = int(v)
    except (TypeError, ValueError):
        raise BadRequest("prompt_logprobs: an integer")
    if not 0 <= k <= 20:
        raise BadRequest("prompt_logprobs: 0 to 20 alternatives")
    return k


def _legacy_logprobs(body):
    """OpenAI's completions `logprobs` (alternatives per position, 0-5 there; up to 20 here), or None."""
    v = body.get("logprobs")
    if v is None or v is False:
        return None
    if v is True:
        return 0
    try:
        k = int(v)
    except (TypeError, ValueError):
        raise BadRequest("logprobs: an integer")
    if not 0 <= k <= 20:
        raise BadRequest("logprobs: 0 to 20 alternatives")
    return k


def legacy_logprobs(ids, scores, top, tokenizer=None, next_score=None):
    """OpenAI's legacy completions logprobs of the echoed prompt (and of the generated token, next_score, when there
    is one): tokens, token_logprobs (None for the first position and for positions without logits), top_logprobs and
    text_offset."""
    ids = [int(t) for t in ids]
    first, vals = scores

    def piece(t):
        if tokenizer is None:
            return str(t)
        return tokenizer.decode([t]).encode("utf-8", "replace").decode("utf-8")
    tokens = [piece(t) for t in ids]
    lps, tops, offsets, at = [None], [None], [], 0
    for tok in tokens:
        offsets.append(at)
        at += len(tok)
    for i in range(1, len(ids)):
        if i < first:
            lps.append(None)
            tops.append(None)
            continue
        lp, _, alts = vals[i - first]
        lps.append(float(lp))
        d = {piece(a): float(alp) for a, alp in alts[:top]}
        d[tokens[i]] = float(lp)
        tops.append(d)
    if next_score is not None:
        tok, lp, alts = next_score
        offsets.append(at)
        tokens.append(piece(tok))
        lps.append(float(lp))
        d = {piece(a): float(alp) for a, alp in alts[:top]}
        d[tokens[-1]] = float(lp)
        tops.append(d)
    return dict(tokens=tokens, token_logprobs=lps, top_logprobs=tops, text_offset=offsets)


def prompt_logprob_entries(ids, scores, tokenizer=None):
    """vLLM's prompt_logprobs list from the scheduler's (first scored position, [(logprob, rank, alternatives)])."""
    ids = [int(t) for t in ids]
    first, vals = scores

    def piece(t):                                       # JSON-safe text (a lone surrogate becomes U+FFFD)
        if tokenizer is None:
            return None
        return tokenizer.decode([t]).encode("utf-8", "replace").decode("utf-8")
    out = [None]
    for i in range(1, len(ids)):
        t = ids[i]
        if i < first:
            out.append({str(t): dict(logprob=None, rank=None, decoded_token=piece(t))})
            continue
        lp, rank, alts = vals[i - first]
        e = {str(a): dict(logprob=float(alp), rank=r + 1, decoded_token=piece(a)) for r, (a, alp) in enumerate(alts)}
        e[str(t)] = dict(logprob=float(lp), rank=int(rank), decoded_token=piece(t))
        out.append(e)
    return out


def _stops(body):
    st = body.get("stop")
    if st is None:
        return []
    st = [st] if isinstance(st, str) else list(st)
    if not all(isinstance(x, str) and x for x in st):
        raise BadRequest("stop: a string or a list of non-empty strings")
    return st


def create_app(scheduler, arms, tokenizer=None, props=None, api_key=None):
    """The FastAPI app. api_key: every endpoint but /health and /metrics then needs `Authorization: Bearer <key>`
    (or `x-api-key: <key>`), as vLLM's and llama.cpp's servers do with their --api-key."""
    import hmac
    import time
    import uuid

    from fastapi import FastAPI
    from fastapi import Request as HTTPRequest
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    app = FastAPI(title="ridgefill-b200")

    if api_key:
        @app.middleware("http")
        async def check_key(request, call_next):
            if request.url.path not in ("/health", "/metrics"):
                auth = request.headers.get("authorization", "")
                given = auth[7:] if auth.lower().startswith("bearer ") else request.headers.get("x-api-key", "")
                if not hmac.compare_digest(given.encode(), str(api_key).encode()):
                    return JSONResponse({"error": {"code": 401, "message": "invalid or missing API key",
                                                   "type": "invalid_request_error"}}, status_code=401)
            return await call_next(request)
    model_name = str((props or {}).get("model", "ridgefill"))

    def bad(msg, code=400):
        return JSONResponse({"error": {"code": code, "message": msg, "type": "invalid_request_error"}},
                            status_code=code)

    def submit(ids, n_predict, arm, ignore_eos=False, prompt_logprobs=-1, stop_ids=()):
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        req = Request(ids=ids, n_predict=n_predict, arm=arm, ignore_eos=ignore_eos, prompt_logprobs=prompt_logprobs,
                      stop_ids=frozenset(int(t) for t in stop_ids),
                      emit=lambda ev: loop.call_soon_threadsafe(q.put_nowait, ev))
        scheduler.submit(req)
        return req, q

    async def openai_run(ids, body, arm, kind, http_req=None):
        """Shared core of /v1/completions and /v1/chat/completions."""
        mt = body.get("max_tokens", body.get("max_completion_tokens"))
        n_predict = 16 if mt is None else int(mt)
        stops = _stops(body)
        plp = _prompt_logprobs(body) if kind == "text" else -1
        echo = bool(body.get("echo")) and kind == "text"
        legacy = _legacy_logprobs(body) if kind == "text" else None
        if echo and body.get("stream"):
            raise BadRequest("echo is served on non-streamed requests only")
        if echo and legacy is not None:                # OpenAI's echo + logprobs: score the prompt as well
            plp = max(plp, legacy)
        if n_predict < 1 and not (n_predict == 0 and plp >= 0):
            raise BadRequest("max_tokens must be at least 1 (0 only with echo + logprobs or prompt_logprobs)")
        if echo and legacy is not None and n_predict > 1:
            raise BadRequest("echo + logprobs: max_tokens 0 or 1 (log-probs of the prompt and the first token)")
        stop_ids = body.get("stop_token_ids") or []
        if not isinstance(stop_ids, list) or not all(isinstance(t, int) for t in stop_ids):
            raise BadRequest("stop_token_ids: a list of token ids")
        try:
            req, q = submit(ids, n_predict, arm, prompt_logprobs=plp, stop_ids=stop_ids)
        except ServerBusy as e:
            return bad(str(e), 503)
        except ValueError as e:
            raise BadRequest(str(e))
        rid = ("chatcmpl-" if kind == "chat" else "cmpl-") + uuid.uuid4().hex[:24]
        created = int(time.time())
        obj = "chat.completion" if kind == "chat" else "text_completion"
        dt = Detok(tokenizer)

        def chunk(text, finish=None, first=False):
            if kind == "chat":
                delta = ({"role": "assistant"} if first else {})
                if text:
                    delta["content"] = text
                choice = dict(index=0, delta=delta, finish_reason=finish)
            else:
                choice = dict(index=0, text=text, finish_reason=finish, logprobs=None)
            return dict(id=rid, object=obj + ".chunk" if kind == "chat" else obj, created=created,
                        model=model_name, choices=[choice])

        async def pieces():
            """(text delta, finish_reason or None, final event or None) as tokens arrive; applies stop strings."""
            text, emitted = "", 0
            while True:
                ev = await _next_event(q, None if body.get("stream") else http_req)
                if "error" in ev:
                    raise RuntimeError(ev["error"])
                if ev.get("stop"):
                    rest = text[emitted:]
                    yield rest, ("stop" if ev.get("stop_type") == "eos" else "length"), ev
                    return
                text += dt.push(ev["tokens"])
                hit = min((text.find(s_) for s_ in stops if s_ in text), default=-1)
                if hit >= 0:
                    req.cancelled = True
                    text = text[:hit]
                    ev2 = await _drain(q)
                    yield text[emitted:], "stop", ev2
                    return
                hold = max((len(s_) - 1 for s_ in stops), default=0)
                safe = max(emitted, len(text) - hold)
                if safe > emitted:
                    yield text[emitted:safe], None, None
                    emitted = safe

        def usage(final):
            n_out = final.get("tokens_predicted", 0) if final else 0
            filled = int(final.get("timings", {}).get("prompt_filled_n", 0)) if final else 0
            # prompt_filled_tokens: prompt rows approximated from the maps (the real tail is prompt_tokens minus it)
            return dict(prompt_tokens=int(ids.numel()), completion_tokens=n_out, total_tokens=int(ids.numel()) + n_out,
                        prompt_filled_tokens=filled)

        def add_prompt_logprobs(choice, final):
            if plp < 0 or final is None or "prompt_scores" not in final:
                return
            if _prompt_logprobs(body) >= 0:
                choice["prompt_logprobs"] = prompt_logprob_entries(ids, final["prompt_scores"], tokenizer)
            if echo and legacy is not None:
                choice["logprobs"] = legacy_logprobs(ids, final["prompt_scores"], legacy, tokenizer,
                                                     final.get("next_score"))

        if body.get("stream"):
            async def events():
                first, done = True, False
                try:
                    async for delta, finish, final in pieces():
                        if delta or first or finish:
                            c = chunk(delta, finish, first)
                            if finish:
                                c["usage"] = usage(final)
                                add_prompt_logprobs(c["choices"][0], final)
                            yield "data: " + json.dumps(c) + "\n\n"
                            first = False
                    done = True
                except RuntimeError as e:
                    done = True
                    yield "data: " + json.dumps({"error": {"message": str(e)}}) + "\n\n"
                finally:              # the client went away mid-stream: the scheduler ends the request next round
                    if not done:
                        req.cancelled = True
                yield "data: [DONE]\n\n"
            return StreamingResponse(events(), media_type="text/event-stream")
        out, finish, final = [], None, None
        try:
            async for delta, f, fin in pieces():
                out.append(delta)
                finish, final = f or finish, fin or final
        except RuntimeError as e:
            return bad(str(e), 500)
        except ClientGone:                  # nobody reads the reply: end the request at the next decode round
            req.cancelled = True
            return bad("client disconnected", 499)
        text = "".join(out)
        if echo:
            prompt_text = tokenizer.decode(ids.tolist(), skip_special_tokens=False) if tokenizer is not None else ""
            text = prompt_text.encode("utf-8", "replace").decode("utf-8") + text
        choice = (dict(index=0, message=dict(role="assistant", content=text), finish_reason=finish)
                  if kind == "chat" else dict(index=0, text=text, finish_reason=finish, logprobs=None))
        add_prompt_logprobs(choice, final)
        return dict(id=rid, object=obj, created=created, model=model_name, choices=[choice], usage=usage(final))

    async def batch_run(prompts, body, arm, http_req):
        """A list of prompts (texts or id lists): one request each, all submitted at once (the scheduler batches
        their decode rounds), answered as one reply with choices in prompt order and summed usage."""
        if body.get("stream"):
            raise BadRequest("a list of prompts is served without stream")
        all_ids = [parse_body(dict(prompt=p, n_predict=1, ridgefill_mode="x"), {"x": arm}, tokenizer)[0]
                   for p in prompts]
        results = await asyncio.gather(*(openai_run(ids, body, arm, "text", http_req) for ids in all_ids))
        for r in results:
            if not isinstance(r, dict):                 # an error reply of one prompt answers for the batch
                return r
        choices = []
        for i, r in enumerate(results):
            c = r["choices"][0]
            c["index"] = i
            choices.append(c)
        usage = {k: sum(r["usage"][k] for r in results) for k in results[0]["usage"]}
        return dict(results[0], choices=choices, usage=usage)

    @app.get("/v1/models")
    def models():
        return dict(object="list", data=[dict(id=model_name, object="model", owned_by="ridgefill-b200")])

    @app.post("/v1/completions")
    async def v1_completions(body: dict, http_req: HTTPRequest):
        try:
            _greedy_only(body)
            arm = _mode(body, arms)
            prompt = body.get("prompt")
            if isinstance(prompt, list) and len(prompt) == 1 and isinstance(prompt[0], (str, list)):
                prompt = prompt[0]
            if isinstance(prompt, list) and prompt and all(isinstance(p, (str, list)) for p in prompt):
                return await batch_run(prompt, body, arm, http_req)
            ids, _, _, _ = parse_body(dict(prompt=prompt, n_predict=1, ridgefill_mode="x"), {"x": arm}, tokenizer)
            return await openai_run(ids, body, arm, "text", http_req)
        except BadRequest as e:
            return bad(str(e))

    @app.post("/v1/chat/completions")
    async def v1_chat(body: dict, http_req: HTTPRequest):
        try:
            _greedy_only(body)
            arm = _mode(body, arms)
            msgs = body.get("messages")
            if tokenizer is None:
                raise BadRequest("chat needs the server's --tokenizer (its chat template)")
            if not isinstance(msgs, list) or not msgs or not all(isinstance(m, dict) and "content" in m for m in msgs):
                raise BadRequest("messages: a non-empty list of {role, content}")
            from ..eval.text import encode
            rendered = tokenizer.apply_chat_template(msgs, tokenize=False, add_generation_prompt=True)
            ids = torch.tensor(encode(tokenizer, rendered), dtype=torch.long)
            if ids.numel() == 0:
                raise BadRequest("the rendered chat prompt encodes to no tokens")
            return await openai_run(ids, body, arm, "chat", http_req)
        except BadRequest as e:
            return bad(str(e))

    @app.post("/tokenize")
    def tokenize(body: dict):
        """llama.cpp's {"content": text} or vLLM's {"prompt": text} -> {"tokens": [ids], "count": n}."""
        text = body.get("content", body.get("prompt"))
        if tokenizer is None:
            return bad("tokenizing needs the server's --tokenizer")
        if not isinstance(text, str):
            return bad("content: a string")
        from ..eval.text import encode
        ids = encode(tokenizer, text)
        if body.get("add_special", body.get("add_special_tokens", False)):
            from ..eval.text import bos_ids
            ids = bos_ids(tokenizer) + ids
        return dict(tokens=ids, count=len(ids))

    @app.post("/detokenize")
    def detokenize(body: dict):
        """{"tokens": [ids]} -> {"content": text, "prompt": text}."""
        ids = body.get("tokens")
        if tokenizer is None:
            return bad("detokenizing needs the server's --tokenizer")
        if not isinstance(ids, list) or not all(isinstance(t, int) for t in ids):
            return bad("tokens: a list of token ids")
        text = tokenizer.decode(ids, skip_special_tokens=False).encode("utf-8", "replace").decode("utf-8")
        return dict(content=text, prompt=text)

    @app.get("/health")
    def health():
        if getattr(scheduler, "failed", None):            # out of service: a load balancer should drop us
            return JSONResponse({"status": "error", "error": scheduler.failed, **scheduler.load}, status_code=503)
        return {"status": "ok", **scheduler.load}

    @app.get("/props")
    def get_props():
        return dict(props or {}, modes=sorted(arms))

    @app.get("/metrics")
    def metrics():
        return PlainTextResponse(scheduler.metrics_text(), media_type="text/plain; version=0.0.4")

    @app.post("/completion")
    async def completion(body: dict, http_req: HTTPRequest):
        try:
            ids, n_predict, arm, ignore_eos = parse_body(body, arms, tokenizer)
        except BadRequest as e:
            return JSONResponse({"error": {"code": 400, "message": str(e)}}, status_code=400)
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        req = Request(ids=ids, n_predict=n_predict, arm=arm, ignore_eos=ignore_eos,
                      detok=Detok(tokenizer).push if tokenizer is not None else None,
                      emit=lambda ev: loop.call_soon_threadsafe(q.put_nowait, ev))
        try:
            scheduler.submit(req)
        except ServerBusy as e:
            return JSONResponse({"error": {"code": 503, "message": str(e)}}, status_code=503)
        except ValueError as e:
            return JSONResponse({"error": {"code": 400, "message": str(e)}}, status_code=400)
        if body.get("stream"):
            async def events():
                done = False
                try:
                    while True:
                        ev = await q.get()
                        yield "data: " + json.dumps(ev) + "\n\n"
                        if ev.get("stop"):
                            done = True
                            break
                finally:              # the client went away mid-stream: the scheduler ends the request next round
                    if not done:
                        req.cancelled = True
            return StreamingResponse(events(), media_type="text/event-stream")
        toks, text = [], []
        while True:
            try:
                ev = await _next_event(q, http_req)
            except ClientGone:              # nobody reads the reply: end the request at the next decode round
                req.cancelled = True
                return JSONResponse({"error": {"code": 499, "message": "client disconnected"}}, status_code=499)
            if "error" in ev:
                return JSONResponse({"error": {"code": 500, "message": ev["error"]}}, status_code=500)
            if ev.get("stop"):
                return dict(ev, tokens=toks, content="".join(text))
            toks += ev["tokens"]
            text.append(ev.get("content", ""))

    return app


async def _drain(q):
    """The final event of a request that was cancelled mid-stream (the scheduler ends it at its next round)."""
    while True:
        ev = await q.get()
        if ev.get("stop"):
            return ev


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
