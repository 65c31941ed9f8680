"""Text prompt sets on synthetic data with a character-level tokenizer: masks, graded prompts, the K20 NIAH
generator, the locked sets (manifest checks, RULER / LongBench / long-prompt builders), the derived RULER sets and
the non-numeric NIAH set with its scoring (the reference's synthetic-locked-set test strategy)."""
import hashlib
import json
import random

import pytest

from ridgefill_data_b200.eval import derived as DV
from ridgefill_data_b200.eval import locked as LK
from ridgefill_data_b200.eval import niahg as NG
from ridgefill_data_b200.eval import text as TX


class _Enc(dict):
    __getattr__ = dict.__getitem__


class CharTok:
    """One token per character (id = code point + 10); BOS 1 first by default; a tiny chat template."""
    bos_token_id, eos_token_id = 1, 2

    def __call__(self, text, add_special_tokens=True, return_offsets_mapping=False):
        ids = ([1] if add_special_tokens else []) + [ord(c) + 10 for c in text]
        enc = _Enc(input_ids=ids)
        if return_offsets_mapping:
            enc["offset_mapping"] = [(i, i + 1) for i in range(len(text))]
        return enc

    def decode(self, ids, skip_special_tokens=False):
        return "".join(chr(i - 10) for i in ids if i >= 10)

    def apply_chat_template(self, msgs, tokenize=False, add_generation_prompt=True, **_):
        return "<u>" + msgs[0]["content"] + "</u><a>"


TOK = CharTok()


def test_masks_and_cap():
    ids = list(range(10)) + list(range(10))
    m = TX.copy_mask(ids, span=8)
    assert m[:10] == [False] * 10 and all(m[10:18]) and m[18:] == [True, True]
    assert TX.novel_mask(ids, 5, span=8) == [False] * 5
    assert TX.cap([1, 5, 6, 7, 8], [1], max_len=3) == [1, 7, 8]
    assert TX.bos_ids(TOK) == [1]


def test_grade_prompts_raw_and_chat():
    body = "".join(random.Random(0).choice("abcdefgh ") for _ in range(700))
    plan = [dict(name="g0", kind="prose", text=body, short_start=100)]
    raw = TX.grade_prompts(TOK, "raw", plan=plan, helps={})[0]
    chat = TX.grade_prompts(TOK, "chat", plan=plan, helps={})[0]
    assert raw["ids"][0] == 1 and raw["ids"][-TX.SCORED:] == chat["ids"][-TX.SCORED:]
    assert raw["short_tail_match"] and len(raw["novel"]) == TX.SCORED
    dropped = TX.grade_prompts(TOK, "raw", drop_bos=True, plan=plan, helps={})[0]
    assert dropped["ids"] == raw["ids"][1:]


def _corpus(n=1200):
    r = random.Random(3)
    return {s: "".join(r.choice("abcdefghij klmnop\n") for _ in range(n * 7 + 30000)) for s in TX.NIAH_SOURCES}


@pytest.mark.parametrize("variant", [None, "mk4"])
def test_k20_niah(variant):
    text_of = _corpus()
    ps = TX.niah_prompts(TOK, "raw", variant=variant, text_of=text_of, lengths=(600, 1200))
    assert len(ps) == 2 * len(TX.NIAH_SOURCES) * len(TX.NIAH_DEPTHS)
    for p in ps:
        needle = TX.encode(TOK, TX.niah_needle(p["key"], p["value"]))
        assert p["ids"][p["needle_start"]:p["needle_end"]] == needle
        assert len(p["ids"]) == p["length"] + 1                    # BOS + L
        assert TX.niah_correct(f"<think>1111111</think> {p['value']}.", p["value"])
    again = TX.niah_prompts(TOK, "raw", variant=variant, text_of=text_of, lengths=(600, 1200))
    assert [p["ids"] for p in again] == [p["ids"] for p in ps]      # seeded draws


# ------------------------------------------------------------------------------------- synthetic locked set
INSTR = ("Some special magic numbers are hidden within the following text. Make sure to memorize it. "
         "I will quiz you about the numbers afterwards.")


def _ruler_row(r, idx):
    keys = [f"key-{r.randrange(10**6)}" for _ in range(4)]
    vals = [str(r.randrange(10**6, 10**7)) for _ in range(4)]
    filler = lambda: " ".join("w" + str(r.randrange(100)) for _ in range(20))  # noqa: E731
    ctx = " ".join(filler() + f" One of the special magic numbers for {k} is: {v}. " for k, v in zip(keys, vals))
    t = r.randrange(4)
    return dict(index=idx, input=f"{INSTR}\n{ctx}\nWhat is the special magic number for {keys[t]} mentioned in the "
                                 f"provided text?",
                answer_prefix=f" The special magic number for {keys[t]} mentioned in the provided text is",
                outputs=[vals[t]], length=8192)


def _write_set(root):
    r = random.Random(7)
    files = {}
    for task in ("niah_multikey_1", "niah_single_1"):
        files[f"ruler/{task}_8192.jsonl"] = "\n".join(json.dumps(_ruler_row(r, i)) for i in range(3)) + "\n"
    lb = [dict(context="c" * 400, input="what?", answers=["x"], all_classes=None, length=400, dataset="hotpotqa",
               _id=f"id{i}") for i in range(2)]
    files["longbench/hotpotqa.jsonl"] = "\n".join(json.dumps(x) for x in lb) + "\n"
    files["long-prompts/doc_4096_0.txt"] = "abc " * 300
    for rel, body in files.items():
        (root / rel).parent.mkdir(parents=True, exist_ok=True)
        (root / rel).write_text(body)
    (root / "longbench/dataset2prompt.json").write_text(json.dumps({"hotpotqa": "Passages:\n{context}\nQ: {input}\nA:"}))
    (root / "longbench/dataset2maxlen.json").write_text(json.dumps({"hotpotqa": 32}))
    (root / "long-prompts/SPLITS.tsv").write_text("path\tsplit_char\nlong-prompts/doc_4096_0.txt\t1000\n")
    lines = ["path\tsha256\tdomain/task"] + [f"{rel}\t{hashlib.sha256((root / rel).read_bytes()).hexdigest()}\t"
                                             f"{rel.split('/')[0]}/x" for rel in files]
    (root / "MANIFEST.tsv").write_text("\n".join(lines) + "\n")
    sha = hashlib.sha256((root / "MANIFEST.tsv").read_bytes()).hexdigest()
    (root / "FROZEN.json").write_text(json.dumps(dict(manifest_sha256=sha)))


@pytest.fixture()
def locked_root(tmp_path, monkeypatch):
    root = tmp_path / "locked"
    _write_set(root)
    monkeypatch.setenv("RF_LOCKED_DIR", str(root))
    monkeypatch.setenv("RF_DERIVED_DIR", str(tmp_path / "derived"))
    return root


def test_locked_sets(locked_root):
    man = LK.manifest()
    ps, skipped = LK.ruler_prompts(TOK, "raw", man, tasks=["niah_multikey_1", "niah_single_1"], lengths=[8192])
    assert len(ps) == 6 and not skipped
    for p in ps:
        (s, e), = p["needles"]
        assert TOK.decode(p["ids"][s:e]).startswith("One of the special magic numbers")
        assert p["refs"][0] in TOK.decode(p["ids"][s:e])
    sc = LK.score(ps[0], ps[0]["refs"][0] + " is the number")
    assert sc["score"] == 1.0
    lb, _ = LK.longbench_prompts(TOK, "chat", man, max_len=100)
    assert len(lb) == 2 and lb[0]["truncated"] and lb[0]["max_new"] == 32
    assert len(lb[0]["ids"]) <= 100 + 20
    lp, _ = LK.longppl_docs(TOK, man, "m")
    assert lp[0]["cont_len"] == 200 and len(lp[0]["ids"]) == 1201
    with pytest.raises(SystemExit):
        LK.ruler_selection(["nope"], None)
    (locked_root / "ruler/niah_single_1_8192.jsonl").write_text("{}\n")
    with pytest.raises(SystemExit):
        LK.ruler_prompts(TOK, "raw", man, tasks=["niah_single_1"], lengths=[8192])
    (locked_root / "MANIFEST.tsv").write_text("tampered")
    with pytest.raises(SystemExit):
        LK.manifest()


@pytest.mark.parametrize("which", DV.SETS)
def test_derived_sets(locked_root, which):
    m = DV.build_manifest(which)
    path = DV.manifest_path(which)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(DV.dumps(m))
    man = LK.manifest()
    ps, _ = DV.prompts(which, TOK, "raw", man, tasks=["niah_multikey_1", "niah_single_1"], lengths=[8192])
    want = 3 if which == "twokey" else 6
    assert len(ps) == want and m["count"] == want
    for p in ps:
        if which == "twokey":
            t1, t2 = p["turn_plan"]
            assert t1["key"] != t2["key"] and t2["value"] in TOK.decode(p["ids"][t2["needle_start"]:t2["needle_end"]])
            assert t2["key"] in p["asks"][0]["question"]
        else:
            text = TOK.decode(p["ids"])
            assert text.index("What is the special magic") < text.index("One of the special")
    m["samples"][0]["text_sha256"] = "0" * 64
    path.write_text(DV.dumps(m))
    with pytest.raises(SystemExit):
        DV.prompts(which, TOK, "raw", man, tasks=["niah_multikey_1", "niah_single_1"], lengths=[8192])


def test_pick_decode_docs():
    paths = [f"long-prompts/d{i}_{L}_0.txt" for i, L in enumerate([4096, 4096, 8192, 8192, 65536])]
    got = DV.pick_decode_docs(paths, n=4, max_len=32768)
    assert len(got) == 4 and all(g.startswith("lp-") for g in got)
    assert DV.pick_decode_docs(paths, n=4, max_len=32768) == got
    with pytest.raises(ValueError):
        DV.pick_decode_docs(paths, n=5, max_len=32768)


def test_niahg_prompts_and_scoring():
    text_of = _corpus()
    plan = [dict(name="g1", type="name", subtype="person", length=600, source="prose", depth=0.5, key="the project",
                 value="Ada Quill", needle_text="\nThe contact person for the project is Ada Quill.\n",
                 question="Who is the contact person for the project? Answer with the name only.")]
    p, = NG.prompts(TOK, "raw", plan=plan, text_of=text_of, lengths=(600, 1200))
    assert TOK.decode(p["ids"][p["value_start"]:p["value_end"]]) == "Ada Quill"
    assert TOK.decode(p["ids"]).endswith("Who is the contact person for the project? The contact person for the "
                                          "project is")
    assert NG.score(" Ada Quill, who runs it.", "Ada Quill", "name", "raw")["correct"]
    assert not NG.score(" Ada Quillson", "Ada Quill", "name", "raw")["correct"]
    assert NG.score("The contact person is Ada Quil", "Ada Quill", "name", "chat")["form"] == "truncated"
    assert NG.score("Ada Quiel", "Ada Quill", "name", "chat")["form"] == "near"
    assert NG.score("<think>x</think>\n\"3F9A 77\"", "3f9a77", "hexid", "chat")["correct"]
    assert NG.score("", "x", "name", "chat")["form"] == "none"
    assert NG.edit_distance("kitten", "sitting") == 3


def test_evaluate_cli_on_locked_sets(tmp_path, locked_root, tiny_llama):
    """The evaluation CLI on the synthetic locked set with the dry-run character tokenizer: RULER generation
    scored by RULER's metric and long-prompt NLL over the continuation, per arm, one result file per prompt."""
    from ridgefill_data_b200 import evaluate
    path, _ = tiny_llama
    arms = [dict(name="exact"), dict(name="identity", split=2, tail=64, fill="identity")]
    base = dict(model=str(path), tokenizer="char", device="cpu", backend="torch", dtype="fp32", arms=arms,
                format="raw", ruler_tasks=["niah_multikey_1"], ruler_lengths=[8192],
                ruler_max_new={"niah_multikey_1": 3})
    cfg = dict(base, prompts=dict(kind="ruler"), out=str(tmp_path / "ruler"))
    (tmp_path / "ruler.json").write_text(json.dumps(cfg))
    assert evaluate.main([str(tmp_path / "ruler.json"), "generate"]) == 0
    recs = sorted((tmp_path / "ruler" / "generate").glob("*.json"))
    assert len(recs) == 3
    r = json.loads(recs[0].read_text())
    for arm in ("exact", "identity"):
        run = r["runs"][arm]
        assert len(run["gen"]) == 3 and run["metric"] == "string_match_all" and 0.0 <= run["score"] <= 1.0
    cfg = dict(base, prompts=dict(kind="longppl"), out=str(tmp_path / "lp"))
    (tmp_path / "lp.json").write_text(json.dumps(cfg))
    with pytest.raises(SystemExit, match="exact tail"):        # tail 64 < continuation 200 + 1
        evaluate.main([str(tmp_path / "lp.json"), "ppl"])
    cfg["arms"] = [dict(name="exact"), dict(name="identity", split=2, tail=256, fill="identity")]
    (tmp_path / "lp.json").write_text(json.dumps(cfg))
    assert evaluate.main([str(tmp_path / "lp.json"), "ppl"]) == 0
    r = json.loads(next((tmp_path / "lp" / "ppl").glob("*.json")).read_text())
    assert all(r["runs"][a]["nll"] > 0 for a in ("exact", "identity"))


def test_alternate_frozen_dataset(locked_root, tmp_path):
    """Config 'dataset': another frozen set beside the locked one replaces it for longppl only, with its manifest
    sha256 pinned; unknown names, other sets and an unpinned or wrong pin are refused."""
    fresh = locked_root.parent / "fresh-long-20261008"
    _write_set(fresh)
    pin = hashlib.sha256((fresh / "MANIFEST.tsv").read_bytes()).hexdigest()
    cfg = dict(dataset="fresh-long-20261008", dataset_manifest_sha256=pin)
    lp, _ = LK.prompts("longppl", TOK, cfg, "m", {})
    assert lp and lp[0]["source"].startswith("long-prompts/")
    for bad in (dict(cfg, dataset="nope"), dict(cfg, dataset_manifest_sha256=None),
                dict(cfg, dataset_manifest_sha256="0" * 64)):
        with pytest.raises(SystemExit):
            LK.prompts("longppl", TOK, bad, "m", {})
    with pytest.raises(SystemExit):
        LK.prompts("ruler", TOK, cfg, "m", {})
