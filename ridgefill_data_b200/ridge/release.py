"""Published map releases (the int8 `i8_row128` layout) read and converted for this engine (the role of
code/c5/convert.py, which converted the same release for another engine).

A release directory holds ridgefill.json (the manifest: {"split", "projector": {"layout": "i8_row128", "files":
{layer: file}}, "files": {name: sha256}, optional "correction": {"layers": [...]}}), the per-layer map files
(proj.L.codes int8 [rows, width], proj.L.scale bf16 [rows, width / 128], proj.L.bias bf16 [rows]),
correction.safetensors (st.L fp32 [heads, V, K]: mean terminal-state errors of the late GDN layers) and
rowsel.safetensors (score fp32 [vocab]: -log unigram frequency on the selectable tokens, -inf elsewhere), with an
optional SHA256SUMS that must agree with the manifest.

Every file is checked against the manifest's sha256 before use. Maps are dequantised exactly in fp32 (an 8-bit code
times a bf16 scale fits fp32), the bias appended, then cast once to bf16: the engine's only rounding.
convert() writes the engine's files (ridgefill-s<split>.safetensors in the map-file format, st.safetensors,
freq.safetensors with logfreq = -score and 0.0 where the release masks the id, SHA256SUMS, CONVERSION.json), builds
them twice from two reads and requires identical bytes, and reads every output back to compare.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import torch

from .projector import I8_GROUP, Projector, check_weights, dequant_i8, stable_safetensors


class ReleaseError(ValueError):
    pass


def _sha(b):
    return hashlib.sha256(b).hexdigest()


def read_release(src):
    """(manifest, {file name: bytes}), every file checked against the manifest (and SHA256SUMS when present)."""
    src = Path(src)
    man = json.loads((src / "ridgefill.json").read_bytes())
    sums = {}
    if (src / "SHA256SUMS").is_file():
        for line in (src / "SHA256SUMS").read_text().splitlines():
            if line.strip():
                h, name = line.split(None, 1)
                sums[name.lstrip("*")] = h
    files = {}
    for name, h in man["files"].items():
        if name in sums and sums[name] != h:
            raise ReleaseError(f"{name}: SHA256SUMS {sums[name][:16]} disagrees with ridgefill.json {h[:16]}")
        data = (src / name).read_bytes()
        if _sha(data) != h:
            raise ReleaseError(f"{name}: sha256 {_sha(data)[:16]}, the manifest says {h[:16]}")
        files[name] = data
    if man.get("projector", {}).get("layout") != "i8_row128":
        raise ReleaseError(f"map layout {man.get('projector', {}).get('layout')!r}: only i8_row128 is known")
    return man, files


def _load(data):
    from safetensors.torch import load
    return load(data)


def maps(man, files):
    """{layer: bf16 [rows, width + 1]} (map | bias), dequantised exactly and cast once."""
    out = {}
    for L, name in sorted(man["projector"]["files"].items(), key=lambda kv: int(kv[0])):
        t = _load(files[name])
        w, b = dequant_i8(t[f"proj.{L}.codes"], t[f"proj.{L}.scale"], t[f"proj.{L}.bias"])
        m = torch.cat((w, b[:, None]), 1)
        check_weights({f"layer.{L}": m}, f"release map {name}")
        out[int(L)] = m.to(torch.bfloat16).contiguous()
    widths = {m.shape for m in out.values()}
    if len(widths) != 1:
        raise ReleaseError(f"the release's maps differ in shape: {sorted(widths)}")
    return out


def corrections(man, files):
    """{layer: fp32 [heads, V, K]} (the release layout) or {} when the release has none."""
    if "correction.safetensors" not in files:
        return {}
    t = _load(files["correction.safetensors"])
    layers = sorted(int(x) for x in man.get("correction", {}).get("layers", []))
    got = sorted(int(k.split(".")[1]) for k in t)
    if layers and got != layers:
        raise ReleaseError(f"correction layers {got} differ from the manifest's {layers}")
    return {int(k.split(".")[1]): v.float().contiguous() for k, v in t.items()}


def freq(files):
    """(logfreq fp32 [vocab] = -score, 0.0 where masked; selectable mask bool [vocab]) from rowsel.safetensors."""
    if "rowsel.safetensors" not in files:
        return None, None
    score = _load(files["rowsel.safetensors"])["score"].float()
    ok = torch.isfinite(score)
    return torch.where(ok, -score, torch.zeros_like(score)), ok


def load(src, device="cpu", dtype=torch.bfloat16):
    """A Projector (split from the manifest) straight from a release directory."""
    man, files = read_release(src)
    m = maps(man, files)
    W = {L: t[:, :-1].to(device, dtype).contiguous() for L, t in m.items()}
    B = {L: t[:, -1].to(device, dtype).contiguous() for L, t in m.items()}
    p = Projector(int(man["split"]), W, B, dict(layout="i8_row128", release=_sha(
        (Path(src) / "ridgefill.json").read_bytes())))
    p.sha256 = p.meta["release"]
    return p


def build(src):
    """{file name: bytes} of the engine files for a release (deterministic)."""
    save = stable_safetensors
    man, files = read_release(src)
    S = int(man["split"])
    m = maps(man, files)
    blobs = {f"ridgefill-s{S}.safetensors": save({f"layer.{L}": t for L, t in sorted(m.items())},
                                                 metadata=dict(split=str(S), source="release i8_row128",
                                                               release_manifest_sha256=_sha(
                                                                   (Path(src) / "ridgefill.json").read_bytes())))}
    st = corrections(man, files)
    if st:
        blobs["st.safetensors"] = save({f"st.{L}": v for L, v in sorted(st.items())})
    lf, _ = freq(files)
    if lf is not None:
        blobs["freq.safetensors"] = save({"logfreq": lf.contiguous()}, metadata=dict(source="rowsel: -score"))
    conv = dict(split=S, layout="i8_row128", group=I8_GROUP, maps=len(m), corrections=sorted(st),
                inputs={k: _sha(v) for k, v in sorted(files.items())},
                outputs={k: _sha(v) for k, v in sorted(blobs.items())})
    blobs["CONVERSION.json"] = (json.dumps(conv, indent=1, sort_keys=True) + "\n").encode()
    return blobs


def convert(src, out):
    """Write the engine files of a release to `out`; returns the written names. Two builds must agree byte for
    byte, and every file is read back and compared after writing."""
    a, b = build(src), build(src)
    if a != b:
        raise ReleaseError("two conversions of the same release differ")
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    for name, data in a.items():
        (out / name).write_bytes(data)
    (out / "SHA256SUMS").write_text("".join(f"{_sha(d)}  {n}\n" for n, d in sorted(a.items())))
    for name, data in a.items():
        if (out / name).read_bytes() != data:
            raise ReleaseError(f"{out / name} reads back different bytes")
    return sorted(a) + ["SHA256SUMS"]


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="convert an i8_row128 map release to this engine's files")
    ap.add_argument("--src", required=True)
    ap.add_argument("--out", required=True)
    a = ap.parse_args(argv)
    for n in convert(a.src, a.out):
        print(n)
    return 0


if __name__ == "__main__":
    import sys
    sys.exit(main())
