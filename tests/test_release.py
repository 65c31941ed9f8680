"""Release tooling: claims gate, recompute from evaluation records, hash-chained ledger, manifests, field stripping
and the secret scan, each with positive and negative controls. Planted secrets are assembled at run time so this
file holds none of the patterns it plants."""
import gzip
import hashlib
import json

import numpy as np
import pytest

from ridgefill_data_b200.release import claims as CL
from ridgefill_data_b200.release import ledger as LG
from ridgefill_data_b200.release import manifest as MF
from ridgefill_data_b200.release import recompute as RC
from ridgefill_data_b200.release import scrub as SC
from ridgefill_data_b200.release import strip as ST


def test_claim_formats_and_gate(tmp_path):
    assert CL.fixed(-0.0004, 3) == "0.000" and CL.fixed(1.23456, 2) == "1.23"
    assert CL.signed(0.0123, 3) == "+0.012" and CL.signed(-0.0041, 3) == "-0.004" and CL.signed(-1e-9, 3) == "0.000"
    with pytest.raises(CL.ClaimError):
        CL.line("a\tb", "1")
    c = CL.Claims()
    c.add("A.n", 30)
    c.interval("A.d", 0.01, -0.002, 0.021, 3)
    (tmp_path / "claims.csv").write_text("id,expected,note\nA.n,30,x\nA.d.delta,+0.010,x\nA.d.ci_lo,-0.002,x\n"
                                         "A.d.ci_hi,+0.021,x\n")
    (tmp_path / "out.txt").write_text("human line\n" + c.text())
    assert CL.main([str(tmp_path / "out.txt"), "--claims", str(tmp_path / "claims.csv")]) == 0
    rep = CL.gate(CL.read_expected(tmp_path / "claims.csv"),
                  [("A.n", "31"), ("A.d.delta", "+0.010"), ("A.d.delta", "+0.010"), ("B", "1")])
    assert not rep.passed
    assert rep.mismatched == {"A.n": ("30", "31")} and rep.missing == ["A.d.ci_lo", "A.d.ci_hi"]
    assert rep.twice == ["A.d.delta"] and rep.unlisted == {"B": "1"}
    assert "1 mismatched, 2 missing, 1 printed twice, 1 unlisted" in rep.lines()[-1]


def test_recompute_reproduces(tmp_path):
    rng = np.random.default_rng(3)
    res = tmp_path / "res" / "nll"
    res.mkdir(parents=True)
    for j in range(25):
        b = float(rng.normal(2.0, 0.2))
        runs = {"exact": {"nll": b, "ok": 1}, "ridgefill": {"nll": b + 0.02 + float(rng.normal(0, 0.01)), "ok": 1},
                "identity": {"nll": b + 0.3, "ok": 0}}
        (res / f"p{j}.json").write_text(json.dumps(dict(name=f"p{j}", runs=runs)))
    spec = {"claims": [
        dict(id="S.rf", results="res/nll", metric="nll", arm="ridgefill", ref="exact", kind="interval", digits=3),
        dict(id="S.n", results="res/nll", metric="nll", arm="ridgefill", kind="n"),
        dict(id="S.exact", results="res/nll", metric="nll", arm="exact", kind="mean", digits=4),
        dict(id="S.ok", results="res/nll", metric="ok", arm="identity", kind="share", digits=1),
        dict(id="S.p", results="res/nll", metric="nll", arm="identity", arms=["ridgefill", "identity"],
             kind="p_holm", digits=3)]}
    (tmp_path / "spec.json").write_text(json.dumps(spec))
    items = RC.load_spec(tmp_path / "spec.json")
    first = RC.Recompute(tmp_path).run(items).text()
    second = RC.Recompute(tmp_path).run(items).text()
    assert first == second                          # declared seed: the same strings every run
    got = dict(s.split("\t") for s in first.splitlines())
    assert got["S.n"] == "25" and got["S.ok"] == "0.0"
    assert float(got["S.rf.ci_lo"]) < 0.02 < float(got["S.rf.ci_hi"]) and got["S.rf.delta"].startswith("+")
    assert float(got["S.p"]) < 0.01
    (tmp_path / "bad.json").write_text(json.dumps({"claims": [dict(id="x", results="res/nll", metric="nll",
                                                                       kind="bogus")]}))
    with pytest.raises(ValueError, match="unknown kind"):
        RC.load_spec(tmp_path / "bad.json")
    with pytest.raises(FileNotFoundError):
        RC.Recompute(tmp_path).one(dict(id="y", results="res/none", metric="nll", arm="exact", kind="mean"))


def test_ledger_chain(tmp_path):
    led = LG.Ledger(tmp_path / "ledger")
    for i in range(4):
        led.append({"type": "hypothesis", "id": f"H{i}", "text": f"claim {i}"})
    assert LG.verify(tmp_path / "ledger") == (4, 4)
    from ridgefill_data_b200.engine.protocol import registered
    assert registered(tmp_path / "ledger" / "ledger.jsonl") == {"H0", "H1", "H2", "H3"}
    cited = led.cite([1, 3])
    assert LG.verify(tmp_path / "ledger", cited) == (4, 2)
    # tamper with an entry: its hash no longer matches the index
    lines = (tmp_path / "ledger" / "ledger.jsonl").read_text().splitlines()
    bad = json.loads(lines[2])
    bad["text"] = "changed"
    lines[2] = LG.canonical_line(bad)
    (tmp_path / "ledger" / "ledger.jsonl").write_text("\n".join(lines) + "\n")
    with pytest.raises(LG.LedgerError, match="seq 2"):
        LG.verify(tmp_path / "ledger")
    # break the chain in the index
    idx = (tmp_path / "ledger" / "index.tsv").read_text().splitlines()
    cols = idx[3].split("\t")
    cols[2] = "0" * 64
    idx[3] = "\t".join(cols)
    (tmp_path / "ledger" / "index.tsv").write_text("\n".join(idx) + "\n")
    assert LG.main(["verify", str(tmp_path / "ledger")]) == 1
    with pytest.raises(LG.LedgerError):
        led.append({"seq": 9})


def test_manifest_roundtrip(tmp_path):
    (tmp_path / "results").mkdir()
    (tmp_path / "results" / "a.json").write_text("{}")
    (tmp_path / "README.md").write_text("x")
    rows = MF.write(tmp_path)
    assert [r["path"] for r in rows] == ["README.md", "results/a.json"]
    assert rows[1]["kind"] == "result" and rows[1]["sha256"] == hashlib.sha256(b"{}").hexdigest()
    assert MF.verify(tmp_path) == ([], [], [])
    (tmp_path / "results" / "a.json").write_text("{ }")
    (tmp_path / "new.txt").write_text("n")
    (tmp_path / "README.md").unlink()
    assert MF.verify(tmp_path) == (["results/a.json"], ["README.md"], ["new.txt"])
    assert MF.main(["verify", str(tmp_path)]) == 1


def test_strip_tree(tmp_path):
    src = tmp_path / "src"
    (src / "run" / "skip").mkdir(parents=True)
    rec = {"name": "p1", "prompt": "secret prompt text", "answer": "42", "runs": {"exact": {"nll": 1.5}},
           "meta": {"host": "node-7", "messages": ["a", "b"]}}
    (src / "run" / "p1.json").write_text(json.dumps(rec, indent=1) + "\n")
    (src / "run" / "p1.json.sha256").write_text("x\n")
    (src / "run" / "rows.jsonl").write_text(json.dumps({"prompt": "q"}) + "\n" + json.dumps({"n": 1}) + "\n")
    (src / "run" / "log.txt").write_text("from node-7 and node-3 and node-7\n")
    (src / "run" / "skip" / "big.bin").write_bytes(b"\0" * 10)
    s = ST.Stripper(fields={"prompt", "messages"}, drop={"answer"},
                    redact=[("HOST", __import__("re").compile(r"node-\d+"))], gzip_globs=["*.txt"], exclude=["skip"])
    n, rows, labels = s.copy_tree(src, tmp_path / "dst", tmp_path / "log.tsv")
    assert n == 4 and labels["HOST"] == {"node-3": "HOST-1", "node-7": "HOST-2"}
    out = json.loads((tmp_path / "dst" / "run" / "p1.json").read_text())
    h = hashlib.sha256(json.dumps("secret prompt text", ensure_ascii=False).encode()).hexdigest()
    assert out["prompt"] == {"stripped": True, "sha256": h, "n": 18}
    assert out["answer"] == {"stripped": True, "n": 2} and out["meta"]["host"] == "HOST-2"
    assert out["meta"]["messages"]["n"] == 2 and out["runs"] == rec["runs"]
    assert not (tmp_path / "dst" / "run" / "p1.json.sha256").exists()
    assert gzip.decompress((tmp_path / "dst" / "run" / "log.txt.gz").read_bytes()) == \
        b"from HOST-2 and HOST-1 and HOST-2\n"
    assert not (tmp_path / "dst" / "run" / "skip").exists()
    log = (tmp_path / "log.tsv").read_text().splitlines()
    assert log[0].startswith("path\t") and any("withheld" in r and "drop:answer" in r for r in log)
    # stripping is idempotent: already-stripped values stay as they are
    s2 = ST.Stripper(fields={"prompt"})
    n2, rows2, _ = s2.copy_tree(tmp_path / "dst", tmp_path / "dst2")
    assert not any(r["path"].endswith("p1.json") for r in rows2)
    with pytest.raises(ValueError):
        s.copy_tree(src, src / "inside")


def test_scrub(tmp_path):
    root = tmp_path / "tree"
    (root / "results").mkdir(parents=True)
    (root / "results" / "r.json").write_text('{"prompt": "hello"}\n')
    tok = "hf" + "_" + "A" * 34
    (root / "notes.txt").write_text("ok line\nkey " + tok + "\n")
    (root / "prov.txt").write_text("bus 0000:" + "1b:00.0\n")
    (root / "x.pkl").write_bytes(b"\x80\x04")
    allow = tmp_path / "ALLOW.md"
    allow.write_text("| path glob | rule | reason |\n|---|---|---|\n"
                     "| prov.txt | PCI_ID | bus address of a rented GPU in a provenance block |\n")
    scan = SC.Scan()
    scan.load_allowlist(allow)
    rep = scan.run(root)
    hits = {(w, r) for w, r in rep.hits}
    assert ("notes.txt:2", "HF_TOKEN") in hits and ("results/r.json:1", "UNSTRIPPED_PROMPT") in hits
    assert ("x.pkl", "FORBIDDEN_FILE") in hits and rep.status == 1 and len(rep.allowed) == 1
    assert tok not in "\n".join(rep.lines())                       # never prints the matched value
    # a stale allowlist row fails the scan
    allow.write_text(allow.read_text() + "| gone/* | EMAIL | an address that was removed long ago |\n")
    scan = SC.Scan()
    scan.load_allowlist(allow)
    assert scan.run(root).status == 2
    # private rules, and a clean tree
    clean = tmp_path / "clean"
    clean.mkdir()
    (clean / "a.txt").write_text("nothing here but " + "proj" + "ect-zeta\n")
    pat = tmp_path / "private.tsv"
    pat.write_text("# local\nINTERNAL\tproject-zeta\n")
    assert SC.main([str(clean), "--allowlist", str(tmp_path / "none.md")]) == 2      # missing allowlist
    (tmp_path / "empty.md").write_text("")
    assert SC.main([str(clean), "--allowlist", str(tmp_path / "empty.md")]) == 0
    assert SC.main([str(clean), "--allowlist", str(tmp_path / "empty.md"), "--private", str(pat)]) == 1
    short = tmp_path / "short.md"
    short.write_text("| a | EMAIL | why |\n")
    assert SC.main([str(clean), "--allowlist", str(short)]) == 2
