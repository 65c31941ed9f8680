"""The int8 map release: a synthetic release (quantised maps, a GDN correction, a rarity table) read, loaded as a
Projector (also through Projector.load of the directory), converted to the engine's files deterministically, and
refused when a file or the checksums list disagree with the manifest."""
import hashlib
import json

import pytest
import torch
from safetensors.torch import save

from ridgefill_data_b200.engine.pred import load_freq
from ridgefill_data_b200.ridge import release as R
from ridgefill_data_b200.ridge.projector import Projector, dequant_i8, load_st, quant_i8


def _release(root, split=2, layers=(2, 3), d=256):
    root.mkdir(parents=True, exist_ok=True)
    g = torch.Generator().manual_seed(0)
    files, proj = {}, {}
    ref = {}
    for L in layers:
        w = 0.05 * torch.randn(d, d, generator=g)
        b = 0.01 * torch.randn(d, generator=g)
        codes, scale, bias = quant_i8(w, b)
        name = f"proj8.L{L}.safetensors"
        data = save({f"proj.{L}.codes": codes, f"proj.{L}.scale": scale, f"proj.{L}.bias": bias})
        (root / name).write_bytes(data)
        files[name] = hashlib.sha256(data).hexdigest()
        proj[str(L)] = name
        ref[L] = dequant_i8(codes, scale, bias)
    st = {"st.3": torch.randn(4, 8, 8, generator=g)}
    data = save(st)
    (root / "correction.safetensors").write_bytes(data)
    files["correction.safetensors"] = hashlib.sha256(data).hexdigest()
    score = torch.rand(100, generator=g) * 10
    score[::3] = float("-inf")
    data = save({"score": score})
    (root / "rowsel.safetensors").write_bytes(data)
    files["rowsel.safetensors"] = hashlib.sha256(data).hexdigest()
    man = dict(split=split, projector=dict(layout="i8_row128", files=proj), files=files,
               correction=dict(layers=[3]), stream_width=d)
    (root / "ridgefill.json").write_text(json.dumps(man))
    return ref, st, score


def test_release_load_and_convert(tmp_path):
    ref, st, score = _release(tmp_path / "rel")
    p = Projector.load(tmp_path / "rel")
    assert p.split == 2 and sorted(p.W) == [2, 3]
    for L, (w, b) in ref.items():
        assert torch.equal(p.W[L], w.to(torch.bfloat16)) and torch.equal(p.b[L], b.to(torch.bfloat16))
    names = R.convert(tmp_path / "rel", tmp_path / "out")
    assert set(names) == {"ridgefill-s2.safetensors", "st.safetensors", "freq.safetensors", "CONVERSION.json",
                          "SHA256SUMS"}
    q = Projector.load(tmp_path / "out" / "ridgefill-s2.safetensors")
    assert q.split == 2 and all(torch.equal(q.W[L], p.W[L]) and torch.equal(q.b[L], p.b[L]) for L in (2, 3))
    lf = load_freq(tmp_path / "out" / "freq.safetensors")
    ok = torch.isfinite(score)
    assert torch.equal(lf[ok], -score[ok]) and (lf[~ok] == 0).all()
    s = load_st(tmp_path / "out" / "st.safetensors")
    assert torch.equal(s[3], st["st.3"].transpose(1, 2))              # release [heads, V, K] -> state [heads, K, V]
    conv = json.loads((tmp_path / "out" / "CONVERSION.json").read_text())
    assert conv["maps"] == 2 and conv["corrections"] == [3]
    assert R.convert(tmp_path / "rel", tmp_path / "out2") and \
        (tmp_path / "out2" / "ridgefill-s2.safetensors").read_bytes() == \
        (tmp_path / "out" / "ridgefill-s2.safetensors").read_bytes()


def test_release_refusals(tmp_path):
    _release(tmp_path / "rel")
    f = tmp_path / "rel" / "proj8.L2.safetensors"
    data = bytearray(f.read_bytes())
    data[-1] ^= 1
    f.write_bytes(bytes(data))
    with pytest.raises(R.ReleaseError, match="sha256"):
        R.read_release(tmp_path / "rel")
    _release(tmp_path / "rel2")
    (tmp_path / "rel2" / "SHA256SUMS").write_text("0" * 64 + "  rowsel.safetensors\n")
    with pytest.raises(R.ReleaseError, match="SHA256SUMS"):
        R.read_release(tmp_path / "rel2")


def test_map_files_are_reproducible(tmp_path):
    """Equal maps and metadata give identical file bytes (canonical safetensors header)."""
    w = {4: torch.randn(8, 8)}
    b = {4: torch.zeros(8)}
    meta = dict(model="m", lam=0.1, rows=10, docs=2, note="")
    Projector(4, w, b).save(tmp_path / "a.safetensors", meta)
    Projector(4, w, b).save(tmp_path / "b.safetensors", dict(reversed(list(meta.items()))))
    assert (tmp_path / "a.safetensors").read_bytes() == (tmp_path / "b.safetensors").read_bytes()
    assert Projector.load(tmp_path / "a.safetensors").meta["lam"] == "0.1"
