"""Serving on the CPU (tiny hybrid on the torch backend): the scheduler's streams equal the engine's greedy decode
for both modes, decode rounds interleave with a long prefill, the HTTP server speaks the /completion layout
(non-streamed, SSE, errors), and the timing and concurrency-mix clients run against it end to end."""
import json
import threading
import urllib.error
import urllib.request

import pytest
import torch

pytest.importorskip("fastapi")
pytest.importorskip("uvicorn")

from ridgefill_data_b200.engine.arm import Arm  # noqa: E402
from ridgefill_data_b200.engine.decode import greedy  # noqa: E402
from ridgefill_data_b200.engine.prefill import prefill  # noqa: E402
from ridgefill_data_b200.eval.data import synthetic_maps, uniform_prompt  # noqa: E402
from ridgefill_data_b200.models.base import from_config  # noqa: E402
from ridgefill_data_b200.models.tiny import tiny_configs  # noqa: E402
from ridgefill_data_b200.ridge.projector import Projector  # noqa: E402
from ridgefill_data_b200.serve import client as C  # noqa: E402
from ridgefill_data_b200.serve.app import Server, create_app  # noqa: E402
from ridgefill_data_b200.serve.engine import Request, Scheduler  # noqa: E402

CFG = tiny_configs(8, 64)["qwen3.5-9b"]
SPLIT, TAIL = 4, 16


@pytest.fixture(scope="module")
def setup():
    model = from_config(CFG, seed=0, device="cpu", dtype=torch.float32)
    W, B = synthetic_maps(CFG.hidden, SPLIT, CFG.n_layers, "cpu", dtype=torch.float32)
    arms = {"off": Arm("exact"), "on": Arm("ridgefill", split=SPLIT, tail=TAIL, fill="proj",
                                            projector=Projector(SPLIT, W, B))}
    return model, arms


def _expected(model, arm, ids, n):
    logits, cache, _ = prefill(model, ids, arm, keep=1)
    toks, _ = greedy(model, ids, cache, logits, n, arm)
    return toks


def _collect(sched, ids, n, arm):
    evs, done = [], threading.Event()

    def emit(ev):
        evs.append(ev)
        if ev.get("stop"):
            done.set()
    sched.submit(Request(ids=ids, n_predict=n, arm=arm, emit=emit, ignore_eos=True))
    return evs, done


def test_decode_gap_sets_the_interleave_period_from_measured_prefill_cost(setup):
    """With gap_ms, a prefill's decode-round period follows its size: the first prefill (nothing decoding) is a
    clean cost sample; afterwards period_for(rows) ~ gap / (rows x ms per row-layer), at least 1."""
    model, arms = setup
    sched = Scheduler(model, interleave=3, gap_ms=50.0, sample_rows=1)
    assert sched.period_for(100) == 3                       # no measurement yet: the fixed period
    ev, done = _collect(sched, uniform_prompt(64, CFG.vocab, seed=8), 2, arms["off"])
    sched.start()
    try:
        assert done.wait(60)
    finally:
        sched.stop()
    assert sched._row_layer_ms is not None and sched._row_layer_ms > 0
    sched._row_layer_ms = 0.01                              # 0.01 ms per row and layer
    assert sched.period_for(1000) == 5
    assert sched.period_for(10) == 500
    assert sched.period_for(10 ** 6) == 1
    assert Scheduler(model, interleave=3).period_for(1000) == 3   # gap_ms 0: always the fixed period
    big = Scheduler(model, interleave=3, gap_ms=50.0)             # default: only prefills of 4096+ rows are samples
    ev, done = _collect(big, uniform_prompt(64, CFG.vocab, seed=9), 2, arms["off"])
    big.start()
    try:
        assert done.wait(60)
    finally:
        big.stop()
    assert big._row_layer_ms is None and big.period_for(1000) == 3


def test_scheduler_matches_greedy_and_interleaves(setup):
    model, arms = setup
    sched = Scheduler(model, interleave=1)
    short = uniform_prompt(40, CFG.vocab, seed=5)
    long = uniform_prompt(96, CFG.vocab, seed=6)
    ev_a, done_a = _collect(sched, short, 12, arms["off"])      # queued before the worker starts: A prefills
    ev_b, done_b = _collect(sched, long, 5, arms["on"])         # first, then B's prefill interleaves A's decode
    sched.start()
    try:
        assert done_a.wait(60) and done_b.wait(60)
    finally:
        sched.stop()
    assert sched.stats["interleaved_rounds"] > 0
    toks_a = [t for e in ev_a if not e.get("stop") for t in e["tokens"]]
    toks_b = [t for e in ev_b if not e.get("stop") for t in e["tokens"]]
    assert toks_a == _expected(model, arms["off"], short, 12)
    assert toks_b == _expected(model, arms["on"], long, 5)
    fa, fb = ev_a[-1], ev_b[-1]
    assert fa["stop"] and fa["tokens_predicted"] == 12 and fa["timings"]["prompt_filled_n"] == 0
    assert fb["timings"]["prompt_filled_n"] == 96 - TAIL and fb["timings"]["ridgefill"]["split"] == SPLIT
    assert fb["tokens_evaluated"] == 96 and fb["stop_type"] == "limit"
    assert sched.stats["completed"] == 2 and sched.stats["errors"] == 0
    assert "ridgefill_completed_total 2" in sched.metrics_text()


def test_eos_and_bad_requests(setup):
    model, arms = setup
    ids = uniform_prompt(30, CFG.vocab, seed=7)
    first = _expected(model, arms["off"], ids, 1)[0]
    sched = Scheduler(model, eos=[first]).start()
    try:
        evs, done = [], threading.Event()
        sched.submit(Request(ids=ids, n_predict=9, arm=arms["off"],
                             emit=lambda e: (evs.append(e), e.get("stop") and done.set())))
        assert done.wait(60)
        assert evs[-1]["stop_type"] == "eos" and evs[-1]["tokens_predicted"] == 1
        with pytest.raises(ValueError):
            sched.submit(Request(ids=ids, n_predict=0, arm=arms["off"], emit=print))
        with pytest.raises(ValueError, match="vocabulary"):
            sched.submit(Request(ids=torch.tensor([CFG.vocab]), n_predict=1, arm=arms["off"], emit=print))
        if model.max_positions:
            with pytest.raises(ValueError, match="positions"):
                sched.submit(Request(ids=ids, n_predict=model.max_positions, arm=arms["off"], emit=print))
    finally:
        sched.stop()


def test_a_full_waiting_queue_refuses_with_busy(setup):
    """max_waiting: with that many requests waiting for a prefill, submit refuses (ServerBusy, HTTP 503 in the app);
    a stopped scheduler's queue stays full, so the refusal is deterministic here."""
    from ridgefill_data_b200.serve.engine import ServerBusy
    model, arms = setup
    sched = Scheduler(model, max_waiting=2)              # not started: nothing leaves the queue
    ids = uniform_prompt(20, CFG.vocab, seed=9)
    for _ in range(2):
        sched.submit(Request(ids=ids, n_predict=1, arm=arms["off"], emit=print))
    with pytest.raises(ServerBusy):
        sched.submit(Request(ids=ids, n_predict=1, arm=arms["off"], emit=print))
    assert sched.stats["refused_busy"] == 1 and sched.load["waiting"] == 2
    assert "ridgefill_refused_busy_total 1" in sched.metrics_text()


@pytest.fixture(scope="module")
def server(setup):
    model, arms = setup
    sched = Scheduler(model, interleave=2).start()
    srv = Server(create_app(sched, arms, props=dict(vocab=CFG.vocab)), port=0).start()
    yield f"http://127.0.0.1:{srv.port}", model, arms
    srv.stop()
    sched.stop()


def test_http_completion(server):
    url, model, arms = server
    assert C.get_json(url, "/health")["status"] == "ok"
    ids = uniform_prompt(64, CFG.vocab, seed=8)
    r = C.post_json(url, "/completion", dict(prompt=ids.tolist(), n_predict=6, ridgefill_mode="on", ignore_eos=True))
    assert r["tokens"] == _expected(model, arms["on"], ids, 6) and r["stop"] and r["tokens_evaluated"] == 64
    events, sent = C.stream(url, dict(prompt=ids.tolist(), n_predict=6, ridgefill=False, ignore_eos=True))
    m = C.token_metrics(events, 6)
    assert [e["data"]["tokens"][0] for e in events[:-1]] == _expected(model, arms["off"], ids, 6)
    assert m["final"]["timings"]["prompt_filled_n"] == 0 and m["itl_ms"]["n"] == 5
    for bad in (dict(prompt=[], n_predict=2), dict(prompt=[1, 2], n_predict=2, temperature=0.7),
                dict(prompt=[1, 2], ridgefill_mode="half"), dict(prompt="text without a tokenizer")):
        with pytest.raises(urllib.error.HTTPError) as e:
            C.post_json(url, "/completion", bad)
        assert e.value.code == 400
    text = urllib.request.urlopen(url + "/metrics").read().decode()
    assert "ridgefill_requests_total" in text and 'ridgefill_ttft_ms{quantile="0.5"}' in text
    assert "ridgefill_decode_round_ms_count" in text


def test_timing_and_mix_clients(server):
    url, _, _ = server
    res = C.timing(url, [uniform_prompt(80, CFG.vocab, seed=s).tolist() for s in (1, 2)], mode="on")
    assert len(res["rows"]) == 2 and all(r["filled"] == 80 - TAIL for r in res["rows"])
    plan = C.make_schedule(3, CFG.vocab, background_len=24, background_predict=40, injector_len=128,
                           injector_predict=3, inject_at_s=0.3, seed=1)
    results, summary = C.run_mix(url, plan, mode="on")
    assert len(results) == 3 and summary["injector_filled"] == 128 - TAIL
    assert summary["background_itl_ms"]["n"] == 2 * 39
    json.dumps(summary)


def test_open_loop_load_client(server):
    """The Poisson load client: every planned request completes with its tokens, the summary's counts add up, and a
    plan is the same for the same seed."""
    url, _, _ = server
    plan = C.make_load(rate=20.0, duration_s=0.5, vocab=CFG.vocab, min_len=16, max_len=48, predict=4, seed=3)
    assert plan == C.make_load(rate=20.0, duration_s=0.5, vocab=CFG.vocab, min_len=16, max_len=48, predict=4, seed=3)
    assert len(plan) >= 2 and all(16 <= len(p["ids"]) <= 48 for p in plan)
    results, summary = C.run_load(url, plan, mode="on")
    assert summary["completed"] == len(results) == len(plan) and summary["failed"] == summary["refused_busy"] == 0
    assert summary["itl_ms"]["n"] == 3 * len(plan) and summary["throughput_tokens_per_s"] > 0
    json.dumps(summary)


def test_token_metrics_checks():
    ev = [dict(t=0.1, data=dict(tokens=[5], tokens_predicted=1)), dict(t=0.3, data=dict(tokens=[6, 7],
                                                                                          tokens_predicted=3)),
          dict(t=0.4, data=dict(stop=True, tokens_predicted=3, timings={}))]
    m = C.token_metrics(ev, 3)
    assert m["coalesced_tokens"] == 1 and m["token_times"] == [0.1, 0.3, 0.3]
    with pytest.raises(C.StreamError):
        C.token_metrics(ev, 4)
    with pytest.raises(C.StreamError):
        C.token_metrics(ev[:2], 3)
    with pytest.raises(C.StreamError):
        C.token_metrics([dict(t=0, data=dict(error="x"))], 1)


def test_decode_batch_matches_single_steps(setup):
    """The model's batched decode (R sequences, one token each) equals R single steps."""
    from ridgefill_data_b200.engine.decode import fork_cache, step
    model, arms = setup
    seqs = []
    for s, n in ((11, 33), (12, 50), (13, 70)):
        ids = uniform_prompt(n, CFG.vocab, seed=s)
        logits, cache, _ = prefill(model, ids, arms["on"] if n > TAIL else arms["off"], keep=1)
        seqs.append((int(logits[-1].argmax()), n, cache))
    single = [step(model, t, p, fork_cache(c), None) for t, p, c in seqs]
    batched = model.decode_batch([t for t, _, _ in seqs], [p for _, p, _ in seqs], [fork_cache(c) for _, _, c in seqs])
    assert batched.shape == (3, CFG.vocab)
    for r in range(3):
        assert torch.equal(batched[r], single[r][-1])


@pytest.fixture(scope="module")
def text_server(setup):
    from ridgefill_data_b200.eval.text import CharTokenizer
    model, arms = setup
    tok = CharTokenizer()
    sched = Scheduler(model, interleave=2).start()
    srv = Server(create_app(sched, arms, tokenizer=tok, props=dict(vocab=CFG.vocab, model="tiny")), port=0).start()
    yield f"http://127.0.0.1:{srv.port}", model, arms, tok
    srv.stop()
    sched.stop()


def _sse(url, path, body):
    req = urllib.request.Request(url + path, data=json.dumps(dict(body, stream=True)).encode(),
                                 headers={"Content-Type": "application/json"})
    out = []
    with urllib.request.urlopen(req, timeout=120) as r:
        for raw in r:
            raw = raw.strip()
            if raw.startswith(b"data:"):
                out.append(raw[5:].strip().decode())
    return out


def test_openai_endpoints(text_server):
    url, model, arms, tok = text_server
    assert C.get_json(url, "/v1/models")["data"][0]["id"] == "tiny"
    prompt = "the river stone and the amber cloud " * 3
    ids = torch.tensor([1] + [ord(c) + 10 for c in prompt])
    want = tok.decode(_expected(model, arms["on"], ids, 8), skip_special_tokens=True)
    r = C.post_json(url, "/v1/completions", dict(model="tiny", prompt=prompt, max_tokens=8, temperature=0))
    assert r["object"] == "text_completion" and r["choices"][0]["text"] == want
    assert r["usage"] == dict(prompt_tokens=ids.numel(), completion_tokens=8, total_tokens=ids.numel() + 8,
                              prompt_filled_tokens=arms["on"].prefix_len(ids.numel()))
    assert r["choices"][0]["finish_reason"] == "length"
    chunks = _sse(url, "/v1/completions", dict(prompt=prompt, max_tokens=8))
    assert chunks[-1] == "[DONE]"
    assert "".join(json.loads(c)["choices"][0]["text"] for c in chunks[:-1]) == want
    chat = C.post_json(url, "/v1/chat/completions", dict(messages=[dict(role="user", content=prompt)], max_tokens=5,
                                                           ridgefill_mode="off"))
    msg = chat["choices"][0]["message"]
    assert chat["object"] == "chat.completion" and msg["role"] == "assistant" and isinstance(msg["content"], str)
    cchunks = _sse(url, "/v1/chat/completions", dict(messages=[dict(role="user", content=prompt)], max_tokens=5,
                                                      ridgefill_mode="off"))
    parts = [json.loads(c) for c in cchunks[:-1]]
    assert parts[0]["choices"][0]["delta"].get("role") == "assistant"
    assert "".join(p["choices"][0]["delta"].get("content", "") for p in parts) == msg["content"]
    if len(want) > 3:                                # a stop string cuts the text where it starts
        stop = want[2:4]
        r = C.post_json(url, "/v1/completions", dict(prompt=prompt, max_tokens=8, stop=[stop]))
        assert r["choices"][0]["text"] == want[:want.find(stop)] and r["choices"][0]["finish_reason"] == "stop"
    for bad in (dict(prompt=prompt, temperature=0.8), dict(prompt=prompt, ridgefill_mode="half")):
        with pytest.raises(urllib.error.HTTPError) as e:
            C.post_json(url, "/v1/completions", bad)
        assert e.value.code == 400


def test_server_cli_build():
    """The server CLI's model / maps / arms / tokenizer assembly (no socket)."""
    import argparse
    from ridgefill_data_b200.serve.__main__ import build
    a = argparse.Namespace(model="tiny-llama", checkpoint=None, backend="torch", device="cpu", maps=None,
                           synthetic_maps=True, split=4, tail=64, tokenizer="char", interleave=4)
    model, arms, tok, eos, props = build(a)
    assert set(arms) == {"on", "off", "quality"} and arms["on"].split == 4 and arms["on"].tail == 64
    assert arms["quality"].meta["quality"].min_prompt == 8192 and arms["quality"].split == 4
    assert props["vocab"] == model.cfg.vocab and eos == (tok.eos_token_id,)
    with pytest.raises(SystemExit):
        build(argparse.Namespace(**dict(vars(a), synthetic_maps=False)))


def test_scheduler_graph_policy_with_a_stand_in_graph(setup, monkeypatch):
    """The decode-graph policy of the scheduler, with a stand-in graph (CUDA graphs need a GPU): a set of running
    requests is captured only after it repeats for a round, the capture is reused while the set holds, dropped when
    one of its requests ends, and the tokens equal eager rounds; a capture that raises turns graphs off for good."""
    from ridgefill_data_b200.engine import decode_graph as DGM
    model, arms = setup
    made = []

    class StandIn:
        def __init__(self, model, caches, headroom, pool=None):
            self.model, self.caches = model, list(caches)
            att = next(i for i, t in enumerate(model.layer_types) if t == "attn")
            self.lengths = [int(c[att]["n"]) for c in caches]
            self.limit = [n + headroom for n in self.lengths]
            self.steps = 0
            made.append(self)

        def room(self):
            return min(lim - n for lim, n in zip(self.limit, self.lengths))

        def step(self, toks):
            out = self.model.decode_batch(list(toks), list(self.lengths), self.caches)
            self.lengths = [n + 1 for n in self.lengths]
            self.steps += 1
            return out

    monkeypatch.setattr(DGM, "DecodeGraph", StandIn)

    def run(graphs):
        sched = Scheduler(model, interleave=0, graphs=False, graph_min_tokens=3)
        sched.graphs = graphs                    # the CPU model: switch the policy on by hand
        evs = {}
        for name, n, seed, pred in (("a", 24, 31, 9), ("b", 30, 32, 6)):
            evs[name] = _collect(sched, uniform_prompt(n, CFG.vocab, seed=seed), pred, arms["off"])
        sched.start()
        try:
            assert all(done.wait(60) for _, done in evs.values())
        finally:
            sched.stop()
        toks = {k: [t for e in ev if not e.get("stop") for t in e["tokens"]] for k, (ev, _) in evs.items()}
        return sched, toks

    sched_e, toks_e = run(False)
    sched_g, toks_g = run(True)
    assert toks_g == toks_e
    assert sched_g.stats["graph_captures"] == len(made) >= 1
    assert sched_g.stats["graph_steps"] == sum(g.steps for g in made) > 0
    assert sched_g.stats["graph_steps"] < sched_g.stats["decode_batches"]   # the first round of a set runs eager
    assert sched_g._graph is None                                             # dropped when its requests ended

    class Broken(StandIn):
        def __init__(self, *a, **k):
            raise RuntimeError("capture failed")

    monkeypatch.setattr(DGM, "DecodeGraph", Broken)
    sched_b, toks_b = run(True)
    assert toks_b == toks_e and sched_b.graphs is False and sched_b.stats["graph_captures"] == 0


def test_prompt_logprobs_and_the_c5_switch(text_server):
    """vLLM's prompt_logprobs on /v1/completions: an exact request scores every position (against the model's own
    teacher-forced log-softmax), a RidgeFill request scores its exact tail and leaves the filled prefix null; the
    c5 kit's vllm_xargs switch picks the mode, and a tail other than the server's is refused."""
    url, model, arms, tok = text_server
    g = torch.Generator().manual_seed(21)
    ids = torch.randint(20, CFG.vocab, (48,), generator=g)
    body = dict(prompt=ids.tolist(), max_tokens=2, temperature=0, prompt_logprobs=2, cache_salt="x",
                repetition_penalty=1.0, skip_special_tokens=True)
    for kva, arm in (("0", arms["off"]), ("1", arms["on"])):
        r = C.post_json(url, "/v1/completions", dict(body, vllm_xargs=dict(dyluhn_kva=kva, dyluhn_kva_tail=TAIL)))
        entries = r["choices"][0]["prompt_logprobs"]
        assert len(entries) == ids.numel() == r["usage"]["prompt_tokens"] and entries[0] is None
        n = ids.numel()
        k = n if arm is arms["off"] else n - arm.prefix_len(n)
        logits, _, _ = prefill(model, ids, arm, keep=k)
        lp = logits[:-1].double().log_softmax(-1)
        lp32 = logits[:-1].float().log_softmax(-1)            # the server ranks in fp32
        first = n - (k - 1)
        for i in range(1, n):
            e = entries[i][str(int(ids[i]))]
            if i < first:
                assert e["logprob"] is None
                continue
            row = lp[i - first]
            assert abs(e["logprob"] - float(row[ids[i]])) < 1e-4
            r32 = lp32[i - first]
            assert e["rank"] == int((r32 > r32[ids[i]]).sum()) + 1
            assert len(entries[i]) >= 2 and len(entries[i]) <= 3           # the prompt token and 2 alternatives
        assert (first == 1) == (arm is arms["off"])
    with pytest.raises(Exception, match="400"):
        C.post_json(url, "/v1/completions", dict(body, vllm_xargs=dict(dyluhn_kva="1", dyluhn_kva_tail=TAIL + 1)))
    with pytest.raises(Exception, match="400"):
        C.post_json(url, "/v1/completions", dict(body, prompt_logprobs=99))


def test_locked_set_client_over_the_openai_api(text_server, tmp_path):
    """serve/sets.py (the c5 kit client's role) against the server: the ppl continuation NLL equals the model's own
    teacher-forced NLL for RidgeFill and exact requests, a RULER-style prompt gets the greedy completion and its
    score, speed rounds time the arm and the exact path, and samples resume from their sidecars."""
    from ridgefill_data_b200.serve import sets as SE
    url, model, arms, tok = text_server
    g = torch.Generator().manual_seed(23)
    ids = torch.randint(20, CFG.vocab, (48,), generator=g)
    doc = dict(name="d0", ids=ids.tolist(), cont_len=10, novel=[j % 3 != 0 for j in range(10)])
    for kva, arm in ((1, arms["on"]), (0, arms["off"])):
        rec = SE.run_ppl(SE.Endpoint(url, kva=kva, tail=TAIL), doc)
        logits, _, _ = prefill(model, ids, arm, keep=11)
        lp = logits[:-1].double().log_softmax(-1)
        want = [-float(lp[j, ids[38 + j]]) for j in range(10)]
        assert rec["cont_len"] == 10 and rec["n_novel"] == 6
        assert rec["tail"] == (48 - arm.prefix_len(48) if kva else 48)
        assert max(abs(a - b) for a, b in zip(rec["token_nll"], want)) < 1e-4
        assert abs(rec["nll"] - sum(want) / 10) < 1e-4
    ep = SE.Endpoint(url, kva=1, tail=TAIL)
    q = dict(name="r0", set="ruler", ids=ids[:30].tolist(), max_new=4, metric="string_match_all", refs=["zz"])
    rec = SE.run_ruler(ep, q)
    assert rec["text"] == tok.decode(_expected(model, arms["on"], ids[:30], 4), skip_special_tokens=True)
    assert rec["score"] in (0.0, 1.0) and rec["metric"] == "string_match_all"
    rows = SE.run_speed(ep, ids.tolist(), [20, 40], runs=2)
    assert [r["length"] for r in rows] == [20, 40]
    assert all(len(r["ttft_s"]["arm"]) == len(r["ttft_s"]["exact"]) == 2 and r["speedup_median"] > 0 for r in rows)
    assert SE.save(tmp_path, "ppl", "d0", dict(x=1)) and SE.done(tmp_path, "ppl", "d0")
    assert not SE.save(tmp_path, "ppl", "d0", dict(x=2))


def test_locked_set_client_cli_writes_and_resumes(text_server, tmp_path, monkeypatch):
    """`python -m ridgefill_data_b200.serve.sets` on a small locked set (the fixture of tests/test_eval_sets.py):
    ppl, RULER and control samples written with sidecars; a second run finds them finished and writes nothing."""
    from test_eval_sets import _write_set
    from ridgefill_data_b200.serve import sets as SE
    url, model, arms, tok = text_server
    root = tmp_path / "locked"
    _write_set(root)
    monkeypatch.setenv("RF_LOCKED_DIR", str(root))
    monkeypatch.setenv("RF_DERIVED_DIR", str(tmp_path / "derived"))
    out = tmp_path / "out"
    argv = ["--url", url, "--kva", "0", "--tokenizer", "char", "--model", "m", "--sets", "ppl,ruler,control",
            "--ruler-lengths", "8192", "--ruler-tasks", "niah_single_1", "--control-docs", "1", "--out", str(out)]
    assert SE.main(argv) == 0
    ppl = json.loads((out / "ppl" / "lp-doc_4096_0.json").read_text())
    assert ppl["cont_len"] == 200 and ppl["tail"] == ppl["n_prompt"] and ppl["nll"] > 0
    ruler = sorted((out / "ruler").glob("*.json"))
    assert len(ruler) == 3 and all(0.0 <= json.loads(f.read_text())["score"] <= 1.0 for f in ruler)
    assert (out / "control" / "lp-doc_4096_0.json.sha256").exists()
    stamps = {f: f.stat().st_mtime_ns for f in out.rglob("*.json")}
    assert SE.main(argv) == 0
    assert {f: f.stat().st_mtime_ns for f in out.rglob("*.json")} == stamps


def test_a_stream_whose_client_leaves_is_ended(server):
    """A streamed request whose client closes the connection after its first token is ended by the scheduler at
    its next decode round (its cache released, counted as cancelled) instead of decoding to its limit."""
    import http.client
    import time
    url, model, arms = server
    host, port = url.split("//")[1].split(":")
    before = _metric(url, "ridgefill_cancelled_total")
    ids = uniform_prompt(40, CFG.vocab, seed=31)
    conn = http.client.HTTPConnection(host, int(port), timeout=60)
    conn.request("POST", "/completion", body=json.dumps(dict(prompt=ids.tolist(), n_predict=100000, ignore_eos=True,
                                                             stream=True)),
                 headers={"Content-Type": "application/json"})
    r = conn.getresponse()
    line = b""
    while not line.startswith(b"data:"):
        line = r.fp.readline().strip()
    conn.sock.close()                                    # the client leaves after its first token
    conn.close()
    t0 = time.time()
    while time.time() - t0 < 30:
        if C.get_json(url, "/health")["active"] == 0 and _metric(url, "ridgefill_cancelled_total") > before:
            break
        time.sleep(0.05)
    assert C.get_json(url, "/health")["active"] == 0
    assert _metric(url, "ridgefill_cancelled_total") == before + 1


def test_a_non_streamed_request_whose_client_leaves_is_ended(server):
    """The same for a non-streamed request: the server notices the closed connection while it waits and ends it."""
    import http.client
    import time
    url, model, arms = server
    host, port = url.split("//")[1].split(":")
    before = _metric(url, "ridgefill_cancelled_total")
    ids = uniform_prompt(40, CFG.vocab, seed=32)
    conn = http.client.HTTPConnection(host, int(port), timeout=60)
    conn.request("POST", "/completion", body=json.dumps(dict(prompt=ids.tolist(), n_predict=100000,
                                                             ignore_eos=True)),
                 headers={"Content-Type": "application/json"})
    t0 = time.time()
    while C.get_json(url, "/health")["active"] == 0 and time.time() - t0 < 30:
        time.sleep(0.02)                                 # decoding has started
    conn.sock.close()
    conn.close()
    while time.time() - t0 < 30:
        if C.get_json(url, "/health")["active"] == 0 and _metric(url, "ridgefill_cancelled_total") > before:
            break
        time.sleep(0.05)
    assert C.get_json(url, "/health")["active"] == 0
    assert _metric(url, "ridgefill_cancelled_total") == before + 1


def _metric(url, name):
    for line in urllib.request.urlopen(url + "/metrics").read().decode().splitlines():
        if line.startswith(name + " "):
            return float(line.split()[1])
    return 0.0


def test_api_key_guards_every_endpoint_but_health(setup):
    """--api-key: requests without the key get 401, with it (Bearer or x-api-key) they are served; /health and
    /metrics stay open for probes."""
    model, arms = setup
    sched = Scheduler(model, interleave=2).start()
    srv = Server(create_app(sched, arms, props=dict(vocab=CFG.vocab), api_key="s3cret"), port=0).start()
    url = f"http://127.0.0.1:{srv.port}"
    try:
        body = json.dumps(dict(prompt=uniform_prompt(20, CFG.vocab, seed=3).tolist(), n_predict=2)).encode()

        def post(headers):
            req = urllib.request.Request(url + "/completion", data=body,
                                         headers=dict({"Content-Type": "application/json"}, **headers))
            with urllib.request.urlopen(req, timeout=60) as r:
                return json.load(r)
        for bad in ({}, {"Authorization": "Bearer wrong"}, {"x-api-key": "s3cre"}):
            with pytest.raises(urllib.error.HTTPError) as e:
                post(bad)
            assert e.value.code == 401
        assert post({"Authorization": "Bearer s3cret"})["tokens_predicted"] == 2
        assert post({"x-api-key": "s3cret"})["stop"]
        assert C.get_json(url, "/health")["status"] == "ok"
        assert "ridgefill_requests_total" in urllib.request.urlopen(url + "/metrics").read().decode()
    finally:
        srv.stop()
        sched.stop()


def test_echo_logprobs_scoring_request(text_server):
    """OpenAI's echo + logprobs with max_tokens 0 (what evaluation harnesses send for log-likelihoods): no token is
    generated, the text is the prompt, and the legacy logprobs block holds every prompt token's teacher-forced
    log-prob with its top alternatives."""
    url, model, arms, tok = text_server
    g = torch.Generator().manual_seed(41)
    ids = torch.randint(20, CFG.vocab, (40,), generator=g)
    r = C.post_json(url, "/v1/completions", dict(prompt=ids.tolist(), max_tokens=0, echo=True, logprobs=2,
                                                 ridgefill_mode="off"))
    ch = r["choices"][0]
    assert r["usage"]["completion_tokens"] == 0 and ch["finish_reason"] == "length"
    assert ch["text"] == tok.decode(ids.tolist(), skip_special_tokens=False).encode("utf-8", "replace").decode()
    lp = ch["logprobs"]
    assert len(lp["tokens"]) == len(lp["token_logprobs"]) == len(lp["top_logprobs"]) == 40
    assert lp["token_logprobs"][0] is None and lp["top_logprobs"][0] is None
    logits, _, _ = prefill(model, ids, arms["off"], keep=40)
    ref = logits[:-1].double().log_softmax(-1)
    for i in range(1, 40):
        assert abs(lp["token_logprobs"][i] - float(ref[i - 1, ids[i]])) < 1e-4
        assert lp["tokens"][i] in lp["top_logprobs"][i] and 1 <= len(lp["top_logprobs"][i]) <= 3
    for bad in (dict(max_tokens=0), dict(max_tokens=2, n=2), dict(max_tokens=2, presence_penalty=0.5),
                dict(max_tokens=2, logit_bias={"5": 1.0}), dict(max_tokens=0, echo=True, logprobs=1, stream=True)):
        with pytest.raises(urllib.error.HTTPError) as e:
            C.post_json(url, "/v1/completions", dict(bad, prompt=ids.tolist()))
        assert e.value.code == 400


def test_tokenize_and_detokenize(text_server):
    url, model, arms, tok = text_server
    r = C.post_json(url, "/tokenize", dict(content="amber cloud"))
    assert r["count"] == len(r["tokens"]) == len("amber cloud")
    assert C.post_json(url, "/detokenize", dict(tokens=r["tokens"]))["content"] == "amber cloud"
    assert C.post_json(url, "/tokenize", dict(prompt="ab", add_special=True))["tokens"][0] == tok.bos_token_id
    with pytest.raises(urllib.error.HTTPError) as e:
        C.post_json(url, "/detokenize", dict(tokens="x"))
    assert e.value.code == 400


def test_a_list_of_prompts_is_one_reply(text_server):
    """/v1/completions with several prompts (texts or id lists), as evaluation harnesses batch them: one choice per
    prompt in order, each equal to that prompt's own request, and the usage summed."""
    url, model, arms, tok = text_server
    g = torch.Generator().manual_seed(43)
    prompts = [torch.randint(20, CFG.vocab, (n,), generator=g).tolist() for n in (24, 31, 40)]
    r = C.post_json(url, "/v1/completions", dict(prompt=prompts, max_tokens=3, ridgefill_mode="off"))
    assert [c["index"] for c in r["choices"]] == [0, 1, 2]
    for p, c in zip(prompts, r["choices"]):
        one = C.post_json(url, "/v1/completions", dict(prompt=p, max_tokens=3, ridgefill_mode="off"))
        assert c["text"] == one["choices"][0]["text"]
    assert r["usage"]["prompt_tokens"] == 24 + 31 + 40 and r["usage"]["completion_tokens"] == 9
    scored = C.post_json(url, "/v1/completions", dict(prompt=prompts[:2], max_tokens=0, echo=True, logprobs=0,
                                                      ridgefill_mode="off"))
    assert [len(c["logprobs"]["token_logprobs"]) for c in scored["choices"]] == [24, 31]


def test_log_likelihood_request_as_evaluation_harnesses_send_it(text_server):
    """The log-likelihood request of OpenAI-API evaluation harnesses: echo, logprobs 1, max_tokens 1; the block
    covers the prompt and the one generated token, so summing token_logprobs[ctxlen:-1] gives the continuation's
    log-likelihood, and the continuation is greedy exactly when each token's log-prob is its row's largest."""
    url, model, arms, tok = text_server
    g = torch.Generator().manual_seed(47)
    ids = torch.randint(20, CFG.vocab, (36,), generator=g)
    ctxlen = 30
    r = C.post_json(url, "/v1/completions", dict(prompt=ids.tolist(), max_tokens=1, echo=True, logprobs=1,
                                                 temperature=0, seed=1234, ridgefill_mode="off"))
    lp = r["choices"][0]["logprobs"]
    assert len(lp["token_logprobs"]) == 37                       # the prompt and the generated token
    logits, _, _ = prefill(model, ids, arms["off"], keep=36)
    ref = logits.double().log_softmax(-1)
    want = sum(float(ref[i - 1, ids[i]]) for i in range(ctxlen, 36))
    assert abs(sum(lp["token_logprobs"][ctxlen:-1]) - want) < 1e-3
    greedy = all(int(ref[i - 1].argmax()) == int(ids[i]) for i in range(ctxlen, 36))
    is_greedy = all(t == max(top.values()) for t, top in zip(lp["token_logprobs"][ctxlen:-1],
                                                             lp["top_logprobs"][ctxlen:-1]))
    assert is_greedy == greedy
    assert lp["token_logprobs"][-1] == max(lp["top_logprobs"][-1].values())    # the generated token is greedy
    with pytest.raises(urllib.error.HTTPError):
        C.post_json(url, "/v1/completions", dict(prompt=ids.tolist(), max_tokens=2, echo=True, logprobs=1))


def test_a_broken_lockstep_group_fails_requests_and_health(setup):
    """When the lockstep group breaks (a collective raises: a rank is gone), the scheduler fails the running and
    waiting requests with an error, refuses new ones, and /health answers 503."""
    from ridgefill_data_b200.serve.engine import ServerBusy

    class Broken:
        arms = None

        def __init__(self, arms):
            self.arms = arms

        def key_of(self, arm):
            return next(k for k, a in self.arms.items() if a is arm)

        def command(self, *cmd):
            if cmd[0] == "decode":
                raise RuntimeError("gloo: connection closed by peer")

        def agree(self, ok):
            return ok
    model, arms = setup
    sched = Scheduler(model, lockstep=Broken(arms)).start()
    srv = Server(create_app(sched, arms, props=dict(vocab=CFG.vocab)), port=0).start()
    url = f"http://127.0.0.1:{srv.port}"
    try:
        evs, done = [], threading.Event()
        sched.submit(Request(ids=uniform_prompt(20, CFG.vocab, seed=5), n_predict=5, arm=arms["off"],
                             emit=lambda e: (evs.append(e), e.get("stop") and done.set())))
        assert done.wait(60) and "error" in evs[-1] and "gloo" in evs[-1]["error"]
        assert sched.failed is not None
        with pytest.raises(ServerBusy):
            sched.submit(Request(ids=uniform_prompt(20, CFG.vocab, seed=6), n_predict=1, arm=arms["off"], emit=print))
        with pytest.raises(urllib.error.HTTPError) as e:
            C.get_json(url, "/health")
        assert e.value.code == 503
    finally:
        srv.stop()
        sched.stop()


def test_kv_pool_admission_holds_a_request_until_pages_free(setup):
    """With a paged K/V pool, a request whose rows (prompt + tokens) would not fit beside the running requests'
    remaining growth waits at the head of the queue and starts once they end; one larger than the pool is refused.
    (A stand-in pool: the torch model keeps its own caches, so the free count stays what the pool reports.)"""
    from types import SimpleNamespace
    model, arms = setup
    pool = SimpleNamespace(page_size=16, pages=6, layers=[0], free_pages=lambda layer=None: 5, owner=None,
                           release=lambda cache: None, release_owner=lambda owner: None)
    model.kv_pool = pool
    try:
        sched = Scheduler(model, interleave=0).start()
        runs = []
        for j, (n, pred) in enumerate(((40, 8), (36, 8), (200, 4))):     # 3 pages, 3 pages, 13 pages
            evs, done = [], threading.Event()
            sched.submit(Request(ids=uniform_prompt(n, CFG.vocab, seed=50 + j), n_predict=pred, arm=arms["off"],
                                 ignore_eos=True, emit=lambda e, evs=evs, done=done: (evs.append(e),
                                                                                      e.get("stop") and done.set())))
            runs.append((evs, done))
        for _, done in runs:
            assert done.wait(60)
        first, second, big = (evs[-1] for evs, _ in runs)
        assert first["tokens_predicted"] == second["tokens_predicted"] == 8
        assert "pool" in big["error"]
        # the second waited for the whole first request (its prefill and its 8 tokens) before its own prefill
        lived = first["timings"]["prompt_ms"] + first["timings"]["predicted_ms"]
        assert second["timings"]["queue_ms"] >= 0.9 * lived
        sched.stop()
    finally:
        model.kv_pool = None


def test_stop_token_ids_end_a_completion(text_server):
    """vLLM's stop_token_ids: the completion ends at the first generated id in the list (finish_reason "stop")."""
    url, model, arms, tok = text_server
    ids = uniform_prompt(30, CFG.vocab, seed=61)
    want = _expected(model, arms["off"], ids, 6)
    r = C.post_json(url, "/v1/completions", dict(prompt=ids.tolist(), max_tokens=6, ridgefill_mode="off",
                                                 stop_token_ids=[want[2]]))
    assert r["usage"]["completion_tokens"] == want.index(want[2]) + 1
    assert r["choices"][0]["finish_reason"] == "stop"
