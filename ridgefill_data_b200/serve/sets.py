"""Locked-set tests of one arm against an OpenAI-API completion server (the role of code/c5/client.py).

    python -m ridgefill_data_b200.serve.sets --url http://127.0.0.1:8080 --kva 1 --tail 4096 \\
        --tokenizer DIR --model qwen3.8-27b --sets ppl,ruler,speed --out results/on

Sets (prompts from eval/locked.py, sent as token ids):
  ppl    every locked long-prompt document (up to --ppl-max-len tokens): one request with prompt_logprobs=0 over the
         whole document; scored = the continuation (the document's last cont_len tokens), all tokens and the novel
         ones (eval/text.py novel_mask), as negative log-likelihoods.
  ruler  the locked RULER prompts at --ruler-lengths, greedy, max_tokens = the task's cap, scored by
         eval/locked.py score.
  speed  time to the first streamed token (max_tokens 1) of prefixes of one document at --speed-lengths: one warm-up,
         then --speed-runs rounds; with --kva 1 each round runs the arm and the same server's exact path
         (dyluhn_kva 0) back to back.
  control  the positive control of a RidgeFill run: the first --control-docs ppl documents with dyluhn_kva 0 (no
         row approximated, the same server), to compare with an exact run.
The per-request switch is the c5 kit's `vllm_xargs` {"dyluhn_kva": "0" | "1", "dyluhn_kva_tail": T}, which this
framework's server reads too, so the same client drives either server. Each sample is one JSON file
<out>/<set>/<name>.json with a sha256 sidecar, written atomically; a sample whose file and sidecar agree is skipped
when the run is resumed.
"""
from __future__ import annotations

import json
import time
import urllib.request
from pathlib import Path

from .client import headers, post_json


class Endpoint:
    """Request bodies and transport for one server and arm. kva: None sends no switch (the server's default mode);
    0 / 1 asks for the exact path / RidgeFill with `tail`."""

    def __init__(self, url, model="ridgefill", kva=None, tail=None, timeout=3600):
        self.url, self.model, self.kva, self.tail, self.timeout = url.rstrip("/"), model, kva, tail, timeout

    def body(self, ids, max_tokens, kva=None, **more):
        b = {"model": self.model, "prompt": [int(t) for t in ids], "max_tokens": int(max_tokens), "temperature": 0,
             "repetition_penalty": 1.0, "skip_special_tokens": True}
        on = self.kva if kva is None else kva
        if on is not None:
            b["vllm_xargs"] = {"dyluhn_kva": "1" if on else "0"}
            if on and self.tail is not None:
                b["vllm_xargs"]["dyluhn_kva_tail"] = int(self.tail)
        b.update(more)
        return b

    def post(self, body):
        return post_json(self.url, "/v1/completions", body, timeout=self.timeout)

    def first_token_s(self, body):
        """Seconds from sending a streamed request to its first chunk with text (the whole reply drained)."""
        req = urllib.request.Request(self.url + "/v1/completions", data=json.dumps(dict(body, stream=True)).encode(),
                                     headers=headers())
        t0 = time.perf_counter()
        first = None
        with urllib.request.urlopen(req, timeout=self.timeout) as r:
            for raw in r:
                raw = raw.strip()
                if not raw.startswith(b"data:"):
                    continue
                data = raw[5:].strip()
                if data == b"[DONE]":
                    break
                ev = json.loads(data)
                if "error" in ev:
                    raise RuntimeError(f"server error: {ev['error']}")
                if first is None and ev["choices"][0].get("text") is not None:
                    first = time.perf_counter() - t0
        if first is None:
            raise RuntimeError("the stream ended without a text chunk")
        return first


def parse_prompt_logprobs(reply, ids):
    """Log-prob of every prompt position after the first (None where the server computed none); each entry must
    hold the prompt's own token."""
    entries = reply["choices"][0].get("prompt_logprobs")
    n = reply["usage"]["prompt_tokens"]
    if entries is None or n != len(ids) or len(entries) != n or entries[0] is not None:
        got = None if entries is None else len(entries)
        raise ValueError(f"prompt_logprobs: {got} entries, usage {n}, sent {len(ids)}")
    out = []
    for i, e in enumerate(entries[1:], 1):
        key = str(int(ids[i]))
        if key not in e:
            raise ValueError(f"prompt_logprobs position {i}: token {key} not in the entry")
        out.append(e[key]["logprob"])
    return out


def run_ppl(ep, doc, kva=None):
    """One ppl document ({"name", "ids", "cont_len", "novel"}): NLL of its continuation, all and novel tokens."""
    ids = doc["ids"]
    t0 = time.perf_counter()
    reply = ep.post(ep.body(ids, 1, kva=kva, prompt_logprobs=0))
    wall = time.perf_counter() - t0
    lp = parse_prompt_logprobs(reply, ids)[-doc["cont_len"]:]
    if any(x is None for x in lp):
        raise ValueError(f"{doc['name']}: the server gave no log-prob for part of the continuation (a RidgeFill "
                         f"tail shorter than {doc['cont_len'] + 1} rows)")
    nll = [-x for x in lp]
    novel = [x for x, m in zip(nll, doc.get("novel") or [True] * len(nll)) if m]
    return {"name": doc["name"], "set": "ppl", "n_prompt": len(ids), "cont_len": doc["cont_len"],
            "nll": sum(nll) / len(nll), "nll_novel": sum(novel) / len(novel) if novel else None,
            "n_novel": len(novel), "token_nll": nll, "wall_s": wall, **_tail(reply, len(ids))}


def _tail(reply, n):
    """The request's real tail, as the server reports it (usage.prompt_filled_tokens; None when it does not)."""
    filled = reply.get("usage", {}).get("prompt_filled_tokens")
    return {"filled": filled, "tail": None if filled is None else n - int(filled)}


def run_ruler(ep, q, kva=None, score=None):
    """One generation prompt ({"name", "ids", "max_new", ...}): the completion and its score."""
    if score is None:
        from ..eval.locked import score
    t0 = time.perf_counter()
    reply = ep.post(ep.body(q["ids"], q["max_new"], kva=kva))
    text = reply["choices"][0]["text"]
    rec = {"name": q["name"], "set": "ruler", "n_prompt": len(q["ids"]), "text": text,
           "finish_reason": reply["choices"][0].get("finish_reason"), "wall_s": time.perf_counter() - t0,
           **_tail(reply, len(q["ids"]))}
    rec.update(score(q, text))
    return rec


def run_speed(ep, ids, lengths, runs=3):
    """TTFT of prefixes of `ids` at each length: one warm-up, then `runs` rounds; with the arm on, each round times
    the arm and the exact path back to back (the order alternating by round)."""
    arms = ("arm", "exact") if ep.kva else ("arm",)
    out = []
    ep.first_token_s(ep.body(ids[:min(64, len(ids))], 1))
    for L in lengths:
        if L > len(ids):
            raise ValueError(f"speed length {L}: the document has {len(ids)} tokens")
        times = {a: [] for a in arms}
        for r in range(runs):
            order = arms if r % 2 == 0 else arms[::-1]
            for a in order:
                times[a].append(ep.first_token_s(ep.body(ids[:L], 1, kva=(0 if a == "exact" else None))))
        rec = {"length": L, "runs": runs, "ttft_s": times}
        if "exact" in times:
            med = {a: sorted(v)[len(v) // 2] for a, v in times.items()}
            rec["speedup_median"] = med["exact"] / med["arm"]
        out.append(rec)
    return out


def save(out, set_name, name, rec):
    """Write one sample (atomic JSON + sha256 sidecar); False when a finished sample is already there."""
    from ..utils.atomic import finished, write_result
    path = Path(out) / set_name / f"{name}.json"
    if finished(path):
        return False
    path.parent.mkdir(parents=True, exist_ok=True)
    write_result(path, rec)
    return True


def done(out, set_name, name):
    from ..utils.atomic import finished
    return out is not None and finished(Path(out) / set_name / f"{name}.json")


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="locked-set tests of one arm over the OpenAI API")
    ap.add_argument("--url", default="http://127.0.0.1:8080")
    ap.add_argument("--served-model", default="ridgefill", help="the `model` field of each request")
    ap.add_argument("--kva", type=int, choices=(0, 1), help="1: RidgeFill with --tail, 0: exact (unset: no switch)")
    ap.add_argument("--tail", type=int)
    ap.add_argument("--sets", default="ppl,ruler,speed")
    ap.add_argument("--tokenizer", required=True)
    ap.add_argument("--model", required=True, help="the model key of the locked sets' token counts")
    ap.add_argument("--locked-root")
    ap.add_argument("--ppl-max-len", type=int, default=32768)
    ap.add_argument("--ruler-lengths", default="8192,16384,32768")
    ap.add_argument("--ruler-tasks", default="", help="comma-separated RULER tasks (default: every locked task)")
    ap.add_argument("--speed-lengths", default="9216,16384,32768")
    ap.add_argument("--speed-runs", type=int, default=3)
    ap.add_argument("--control-docs", type=int, default=4)
    ap.add_argument("--out", required=True)
    a = ap.parse_args(argv)
    from ..eval import locked as LK
    from ..eval.text import tokenizer as load_tokenizer
    tok = load_tokenizer(a.tokenizer)
    man = LK.manifest(a.locked_root)
    ep = Endpoint(a.url, a.served_model, a.kva, a.tail)
    sets = [s for s in a.sets.split(",") if s]
    summary = {}
    if "ppl" in sets or "speed" in sets or "control" in sets:
        docs, _ = LK.longppl_docs(tok, man, a.model, max_len=a.ppl_max_len, root=a.locked_root)
    if "ppl" in sets:
        recs = []
        for d in docs:
            if done(a.out, "ppl", d["name"]):
                continue
            rec = run_ppl(ep, d)
            save(a.out, "ppl", d["name"], rec)
            recs.append(rec)
        summary["ppl"] = {"documents": len(recs), "nll_mean": sum(r["nll"] for r in recs) / max(1, len(recs))}
    if "control" in sets:
        recs = []
        for d in docs[:a.control_docs]:
            if done(a.out, "control", d["name"]):
                continue
            rec = run_ppl(ep, d, kva=0)
            save(a.out, "control", d["name"], rec)
            recs.append(rec)
        summary["control"] = {"documents": len(recs), "nll_mean": sum(r["nll"] for r in recs) / max(1, len(recs))}
    if "ruler" in sets:
        lengths = [int(x) for x in a.ruler_lengths.split(",") if x]
        tasks = [t for t in a.ruler_tasks.split(",") if t] or None
        prompts_, _ = LK.ruler_prompts(tok, "raw", man, tasks=tasks, lengths=lengths, root=a.locked_root)
        recs = []
        for q in prompts_:
            if done(a.out, "ruler", q["name"]):
                continue
            rec = run_ruler(ep, q)
            save(a.out, "ruler", q["name"], rec)
            recs.append(rec)
        summary["ruler"] = {"prompts": len(recs), "score_mean": sum(r["score"] for r in recs) / max(1, len(recs))}
    if "speed" in sets:
        lengths = [int(x) for x in a.speed_lengths.split(",") if x]
        longest = max(docs, key=lambda d: len(d["ids"]))
        recs = run_speed(ep, longest["ids"], lengths, a.speed_runs)
        save(a.out, "speed", "speed-" + longest["name"], {"document": longest["name"], "rows": recs})
        summary["speed"] = recs
    print(json.dumps(summary, indent=1))
    return 0


if __name__ == "__main__":
    import sys
    sys.exit(main())
