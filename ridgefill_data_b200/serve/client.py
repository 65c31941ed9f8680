"""Measurement clients for the `/completion` server (the roles of code/qwen38-27b-kit/timing.py and mix.py):

* `timing`: TTFT of distinct prompts on a warm server: one short warm-up request, then each prompt once, with the
  client-side TTFT (send -> first token event) next to the server's own prompt time.
* `load`: an open-loop load test: requests arrive as a Poisson process at a given rate for a given time, each with
  a prompt length drawn from a range; the summary gives request and token throughput, TTFT and inter-token gaps
  (p50 / p90 / p99), and the requests the server refused as busy (HTTP 503) or failed.
* `mix`: a fixed-arrival concurrency mix. Background requests start decoding; at a planned time an injector sends a
  long prompt; every request's stream is recorded with arrival-relative timestamps. The summary gives the injector's
  TTFT and the background streams' inter-token gaps before, during and after the injector's prefill: what a long
  RidgeFill prefill costs the requests already being served.

    python -m ridgefill_data_b200.serve.client timing --url http://127.0.0.1:8080 --length 16384 --prompts 3
    python -m ridgefill_data_b200.serve.client mix --url http://127.0.0.1:8080 --concurrency 4 --injector-len 16384

Only the standard library is used on the client side (urllib + threads), so it runs anywhere.
"""
from __future__ import annotations

import json
import os
import threading
import time
import urllib.request

import numpy as np


# ------------------------------------------------------------------------------------------------ transport
def headers():
    """JSON content type, plus `Authorization: Bearer $RF_API_KEY` when the server was started with a key."""
    h = {"Content-Type": "application/json"}
    key = os.environ.get("RF_API_KEY")
    if key:
        h["Authorization"] = f"Bearer {key}"
    return h


def post_json(url, path, body, timeout=600):
    req = urllib.request.Request(url + path, data=json.dumps(body).encode(), headers=headers())
    with urllib.request.urlopen(req, timeout=timeout) as r:
        return json.load(r)


def get_json(url, path, timeout=30):
    with urllib.request.urlopen(url + path, timeout=timeout) as r:
        return json.load(r)


def stream(url, body, epoch=None, timeout=600):
    """[{'t': seconds since epoch, 'data': event}] of one streamed completion, and the send time."""
    epoch = time.monotonic() if epoch is None else epoch
    body = dict(body, stream=True)
    req = urllib.request.Request(url + "/completion", data=json.dumps(body).encode(), headers=headers())
    sent = time.monotonic() - epoch
    events = []
    with urllib.request.urlopen(req, timeout=timeout) as r:
        for raw in r:
            raw = raw.strip()
            if not raw.startswith(b"data:"):
                continue
            raw = raw[5:].strip()
            if raw == b"[DONE]":
                break
            ev = json.loads(raw)
            events.append(dict(t=time.monotonic() - epoch, data=ev))
            if ev.get("stop"):
                break
    return events, sent


# ------------------------------------------------------------------------------------------------ metrics
def distribution(xs):
    xs = [float(x) for x in xs]
    if not xs:
        return dict(n=0)
    a = np.asarray(xs)
    return dict(n=len(xs), mean=float(a.mean()), p50=float(np.percentile(a, 50)), p90=float(np.percentile(a, 90)),
                p99=float(np.percentile(a, 99)), max=float(a.max()))


class StreamError(RuntimeError):
    pass


def token_metrics(events, expected):
    """Per-token arrival times of one stream (a token counted once, at the event that delivered it), the gaps
    between consecutive tokens, and the final event. Checks: no error event, monotone token counts, exactly one
    final event, `expected` tokens delivered."""
    delivered, times, final, coalesced = 0, [], None, 0
    for ev in events:
        d, t = ev["data"], ev["t"]
        if "error" in d:
            raise StreamError(f"server error: {d['error']}")
        if d.get("stop"):
            if final is not None:
                raise StreamError("two final events")
            final = d
            continue
        count = d.get("tokens_predicted", delivered + len(d.get("tokens", [])))
        if count < delivered:
            raise StreamError("token count went backwards")
        if count > delivered:
            coalesced += count - delivered - 1
            times += [t] * (count - delivered)
            delivered = count
    if final is None:
        raise StreamError("no final event")
    if delivered != expected or final.get("tokens_predicted") != expected:
        raise StreamError(f"{delivered} tokens delivered, {expected} expected")
    gaps = [dict(begin=a, end=b, ms=1e3 * (b - a)) for a, b in zip(times, times[1:])]
    return dict(first=times[0], last=times[-1], token_times=times, gaps=gaps, coalesced_tokens=coalesced,
                itl_ms=distribution([g["ms"] for g in gaps]),
                decode_tps=(expected - 1) / (times[-1] - times[0]) if expected > 1 and times[-1] > times[0] else None,
                final=final)


# ------------------------------------------------------------------------------------------------ timing
def timing(url, prompts, mode="on", warmup_len=32):
    """TTFT of each prompt (lists of ids) on a warm server, one at a time."""
    post_json(url, "/completion", dict(prompt=prompts[0][:warmup_len], n_predict=2, ridgefill_mode=mode,
                                       ignore_eos=True))
    rows = []
    for j, ids in enumerate(prompts):
        events, sent = stream(url, dict(prompt=list(ids), n_predict=1, ridgefill_mode=mode, ignore_eos=True,
                                        temperature=0, top_k=1, cache_prompt=False))
        m = token_metrics(events, 1)
        t = m["final"]["timings"]
        if t["prompt_n"] != len(ids) or t["cache_n"] != 0:
            raise StreamError(f"prompt {j}: the server evaluated {t['prompt_n']} of {len(ids)} tokens")
        rows.append(dict(prompt=j, n=len(ids), client_ttft_ms=1e3 * (m["first"] - sent),
                         server_prompt_ms=t["prompt_ms"], filled=t.get("prompt_filled_n", 0)))
    return dict(mode=mode, rows=rows, client_ttft_ms=distribution([r["client_ttft_ms"] for r in rows]),
                server_prompt_ms=distribution([r["server_prompt_ms"] for r in rows]))


# ------------------------------------------------------------------------------------------------ mix
def make_schedule(concurrency, vocab, background_len=1024, background_predict=64, injector_len=16384,
                  injector_predict=8, inject_at_s=1.0, stagger_s=0.05, seed=0):
    """A fixed-arrival plan: concurrency - 1 background requests arriving stagger_s apart from t = 0, then one
    injector (a long prompt) at inject_at_s. Seeded uniform ids."""
    if concurrency < 2:
        raise ValueError("a mix needs at least one background request and the injector")
    g = np.random.default_rng(seed)
    plan = [dict(id=f"bg{j}", role="background", arrival_s=j * stagger_s, predict=background_predict,
                 ids=g.integers(0, vocab, background_len).tolist()) for j in range(concurrency - 1)]
    plan.append(dict(id="inj", role="injector", arrival_s=inject_at_s, predict=injector_predict,
                     ids=g.integers(0, vocab, injector_len).tolist()))
    return plan


def run_mix(url, plan, mode="on", background_mode="off", timeout=900):
    """Send every planned request at its arrival time (the injector with `mode`, the background with
    `background_mode`), record the streams, return (results, summary)."""
    out, errors, threads = [], [], []
    epoch = time.monotonic() + 0.5

    def one(item):
        try:
            body = dict(prompt=item["ids"], n_predict=item["predict"], ignore_eos=True, temperature=0, top_k=1,
                        ridgefill_mode=mode if item["role"] == "injector" else background_mode)
            time.sleep(max(0.0, epoch + item["arrival_s"] - time.monotonic()))
            events, sent = stream(url, body, epoch, timeout)
            m = token_metrics(events, item["predict"])
            m.update(id=item["id"], role=item["role"], n_prompt=len(item["ids"]), predict=item["predict"], sent=sent,
                     planned=item["arrival_s"], lateness_ms=1e3 * (sent - item["arrival_s"]),
                     ttft_s=m["first"] - sent)
            out.append(m)
        except Exception as e:
            errors.append(dict(id=item["id"], error=repr(e)))

    for item in plan:
        th = threading.Thread(target=one, args=(item,), daemon=True)
        threads.append(th)
        th.start()
    for th in threads:
        th.join(timeout)
    if errors:
        raise StreamError(f"mix requests failed: {errors}")
    return out, summarize(out)


def summarize(results):
    inj = next(r for r in results if r["role"] == "injector")
    bg = [r for r in results if r["role"] == "background"]
    gaps = [g for r in bg for g in r["gaps"]]
    during = [g for g in gaps if g["end"] >= inj["sent"] and g["begin"] <= inj["first"]]
    before = [g for g in gaps if g["end"] <= inj["sent"]]
    after = [g for g in gaps if g["begin"] >= inj["first"]]
    wall = max(r["last"] for r in results) - min(r["sent"] for r in results)
    busy = inj["first"] - inj["sent"]
    return dict(
        injector_ttft_s=inj["ttft_s"], injector_server_prompt_ms=inj["final"]["timings"]["prompt_ms"],
        injector_filled=inj["final"]["timings"].get("prompt_filled_n", 0),
        background_ttft_s=distribution([r["ttft_s"] for r in bg]),
        background_itl_ms=distribution([g["ms"] for g in gaps]),
        background_itl_before_ms=distribution([g["ms"] for g in before]),
        background_itl_during_prefill_ms=distribution([g["ms"] for g in during]),
        background_itl_after_ms=distribution([g["ms"] for g in after]),
        background_tokens_during_prefill=sum(inj["sent"] <= t <= inj["first"] for r in bg for t in r["token_times"]),
        background_active_at_injection=sum(r["first"] < inj["sent"] < r["last"] for r in bg),
        background_tps_during_prefill=(sum(inj["sent"] <= t <= inj["first"] for r in bg for t in r["token_times"])
                                       / busy if busy > 0 else None),
        aggregate_tps=sum(r["predict"] for r in results) / wall if wall > 0 else None,
        lateness_ms=distribution([r["lateness_ms"] for r in results]), workload_s=wall,
        coalesced_tokens=sum(r["coalesced_tokens"] for r in results))


# ------------------------------------------------------------------------------------------------ load
def make_load(rate, duration_s, vocab, min_len=512, max_len=4096, predict=32, seed=0):
    """Poisson arrivals at `rate` requests per second over duration_s, prompt lengths uniform in [min_len,
    max_len], seeded uniform ids."""
    g = np.random.default_rng(seed)
    plan, t = [], float(g.exponential(1.0 / rate))
    while t < duration_s:
        n = int(g.integers(min_len, max_len + 1))
        plan.append(dict(id=f"r{len(plan)}", arrival_s=t, predict=predict, ids=g.integers(0, vocab, n).tolist()))
        t += float(g.exponential(1.0 / rate))
    return plan


def run_load(url, plan, mode="on", timeout=900):
    """Send every planned request at its arrival time (streamed), return (per-request results, summary)."""
    import urllib.error
    out, refused, failed, threads = [], [], [], []
    lock = threading.Lock()
    epoch = time.monotonic() + 0.5

    def one(item):
        body = dict(prompt=item["ids"], n_predict=item["predict"], ignore_eos=True, temperature=0, top_k=1,
                    ridgefill_mode=mode)
        time.sleep(max(0.0, epoch + item["arrival_s"] - time.monotonic()))
        try:
            events, sent = stream(url, body, epoch, timeout)
            m = token_metrics(events, item["predict"])
            m.update(id=item["id"], n_prompt=len(item["ids"]), predict=item["predict"], sent=sent,
                     ttft_s=m["first"] - sent)
            with lock:
                out.append(m)
        except urllib.error.HTTPError as e:
            with lock:
                (refused if e.code == 503 else failed).append(dict(id=item["id"], code=e.code))
        except Exception as e:
            with lock:
                failed.append(dict(id=item["id"], error=repr(e)))

    for item in plan:
        th = threading.Thread(target=one, args=(item,), daemon=True)
        threads.append(th)
        th.start()
    for th in threads:
        th.join(timeout)
    return out, summarize_load(out, plan, refused, failed)


def summarize_load(results, plan, refused=(), failed=()):
    if results:
        wall = max(r["last"] for r in results) - min(r["sent"] for r in results)
    else:
        wall = 0.0
    tokens = sum(r["predict"] for r in results)
    return dict(requests=len(plan), completed=len(results), refused_busy=len(refused), failed=len(failed),
                offered_rate_rps=len(plan) / max(1e-9, plan[-1]["arrival_s"]) if plan else 0.0,
                throughput_rps=len(results) / wall if wall > 0 else None,
                throughput_tokens_per_s=tokens / wall if wall > 0 else None,
                prompt_tokens_per_s=sum(r["n_prompt"] for r in results) / wall if wall > 0 else None,
                ttft_s=distribution([r["ttft_s"] for r in results]),
                itl_ms=distribution([g["ms"] for r in results for g in r["gaps"]]), workload_s=wall)


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="timing and concurrency-mix clients of the completion server")
    sub = ap.add_subparsers(dest="cmd", required=True)
    for name in ("timing", "mix", "load"):
        p = sub.add_parser(name)
        p.add_argument("--url", default="http://127.0.0.1:8080")
        p.add_argument("--mode", default="on", help="the prompt's (injector's) ridgefill_mode")
        p.add_argument("--seed", type=int, default=0)
        p.add_argument("--out")
    t = sub.choices["timing"]
    t.add_argument("--length", type=int, default=16384)
    t.add_argument("--prompts", type=int, default=3)
    m = sub.choices["mix"]
    m.add_argument("--concurrency", type=int, default=4)
    m.add_argument("--background-len", type=int, default=1024)
    m.add_argument("--background-predict", type=int, default=64)
    m.add_argument("--injector-len", type=int, default=16384)
    m.add_argument("--injector-predict", type=int, default=8)
    m.add_argument("--inject-at", type=float, default=1.0)
    m.add_argument("--background-mode", default="off")
    ld = sub.choices["load"]
    ld.add_argument("--rate", type=float, default=1.0, help="requests per second (Poisson arrivals)")
    ld.add_argument("--duration", type=float, default=60.0, help="seconds of arrivals")
    ld.add_argument("--min-len", type=int, default=512)
    ld.add_argument("--max-len", type=int, default=16384)
    ld.add_argument("--predict", type=int, default=32)
    a = ap.parse_args(argv)
    vocab = int(get_json(a.url, "/props").get("vocab", 32000))
    g = np.random.default_rng(a.seed)
    if a.cmd == "timing":
        res = timing(a.url, [g.integers(0, vocab, a.length).tolist() for _ in range(a.prompts)], a.mode)
    elif a.cmd == "load":
        plan = make_load(a.rate, a.duration, vocab, a.min_len, a.max_len, a.predict, seed=a.seed)
        _, res = run_load(a.url, plan, a.mode)
    else:
        plan = make_schedule(a.concurrency, vocab, a.background_len, a.background_predict, a.injector_len,
                             a.injector_predict, a.inject_at, seed=a.seed)
        _, res = run_mix(a.url, plan, a.mode, a.background_mode)
    if a.out:
        from ..utils.atomic import write_result
        write_result(a.out, res)
    print(json.dumps(res, indent=1))
    return 0


if __name__ == "__main__":
    import sys
    sys.exit(main())
