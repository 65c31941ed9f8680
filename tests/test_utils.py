"""Utilities: uncached reads with the plain-read fallback, model manifests, atomic result files, the shifted
ridge-statistics merge, needle splicing and the Arm helpers."""
import errno
import fcntl
import hashlib
import json
import os

import pytest
import torch

from ridgefill_data_b200.engine import arm as A
from ridgefill_data_b200.eval import text as TX
from ridgefill_data_b200.ridge import stats as RS
from ridgefill_data_b200.utils import atomic, integrity as I


def test_uncached_read_falls_back_after_a_refused_read(tmp_path, monkeypatch):
    data = os.urandom((1 << 24) + 4097)
    f = tmp_path / "blob.bin"
    f.write_bytes(data)
    real = os.readv
    calls = {"n": 0}

    def flaky(fd, bufs):                        # the second O_DIRECT read is refused, as some filesystems do
        calls["n"] += 1
        if calls["n"] == 2 and fcntl.fcntl(fd, fcntl.F_GETFL) & os.O_DIRECT:
            raise OSError(errno.EINVAL, "refused")
        return real(fd, bufs)

    monkeypatch.setattr(I.os, "readv", flaky)
    assert I.read_direct(f) == data               # the fallback resumes where the refused read stopped
    assert I.file_sha256(f, direct=True) == hashlib.sha256(data).hexdigest()


def test_model_manifest_and_verify(tmp_path):
    (tmp_path / "config.json").write_text("{}")
    (tmp_path / "model.safetensors").write_bytes(b"weights")
    sums = I.model_manifest(tmp_path)
    assert set(sums) == {"config.json", "model.safetensors"}
    assert I.verify_model(tmp_path) == []
    (tmp_path / "model.safetensors").write_bytes(b"changed")
    with pytest.raises(I.IntegrityError):
        I.verify_model(tmp_path)
    (tmp_path / "extra.json").write_text("{}")
    with pytest.raises(I.IntegrityError, match="exactly"):
        I.model_manifest(tmp_path)


def test_recorded_sha256(tmp_path):
    (tmp_path / "a.json").write_text(json.dumps({"runs": [{"projector": "/x/m.safetensors",
                                                           "projector_sha256": "ab" * 32}]}))
    assert I.recorded_sha256("m.safetensors", tmp_path) == "ab" * 32
    (tmp_path / "b.json").write_text(json.dumps({"path": "/y/m.safetensors", "sha256": "cd" * 32}))
    assert I.recorded_sha256("m.safetensors", tmp_path) is None       # records disagree: none is trusted


def test_atomic_result_and_treehash(tmp_path):
    digest = atomic.write_result(tmp_path / "r.json", {"b": 1, "a": [1, 2]})
    assert atomic.finished(tmp_path / "r.json") and atomic.read_sidecar(tmp_path / "r.json") == digest
    before = atomic.treehash(tmp_path)
    (tmp_path / "r.json").write_text("{}")
    assert not atomic.finished(tmp_path / "r.json") and atomic.treehash(tmp_path) != before
    assert atomic.main(["check", str(tmp_path / "r.json")]) == 2


def _stats(x, ys, layers):
    st = RS.RidgeStats(0, layers, x.shape[1], out_dim=ys[layers[0]].shape[1])
    st.add(x, ys, block=7)
    return st.state()


def test_combine_equals_one_pass():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(40, 5, generator=g) * 3 + 1
    ys = {1: torch.randn(40, 4, generator=g) - 2}
    whole = _stats(x, ys, [1])
    merged = RS.combine(_stats(x[:17], {1: ys[1][:17]}, [1]), _stats(x[17:], {1: ys[1][17:]}, [1]))
    assert merged["n"] == whole["n"] == 40
    for got, want in zip(RS.raw_moments(merged, 1), RS.raw_moments(whole, 1)):   # products are fp32 per block
        torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-4)
    xx, xy = RS.raw_moments(whole, 1)
    torch.testing.assert_close(xx, x.double().T @ x.double(), rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(xy, x.double().T @ ys[1].double(), rtol=1e-5, atol=1e-4)


def test_needle_splice_positions():
    body = list(range(100, 120))
    ids, span = TX._splice([1], body, [(0.25, [7, 7], False), (0.5, [8, 8, 8], True)])
    assert ids[:1] == [1] and len(ids) == 1 + 20 + 5
    assert ids[span[0]:span[1]] == [8, 8, 8] and span == (1 + 5 + 2 + 5, 1 + 5 + 2 + 5 + 3)


def test_arm_helpers():
    a = A.Arm("x", split=2, tail=16, fill="by_type", fill_by_type={"attention": "proj", "gdn": "identity"})
    assert a.fill_of("attn") == "proj" and a.fill_of("gdn") == "identity" and a.uses("identity")
    with pytest.raises(ValueError, match="no fill"):
        A.Arm("y", split=2, fill="by_type", fill_by_type={"attention": "proj"}).fill_of("gdn")
    assert A.rounded_tail(1000, 300, 128) == 1000 - 640 and A.rounded_tail(200, 300, 128) == 200
    r = A.Arm("r", split=2, tail=64, fill="proj", rescale="ktail", rescale_skip_last=3)
    assert A.exclude_scored(r, 10).rescale_skip_last == 10 and A.exclude_scored(r, 2) == r
    assert A.exclude_scored(r, 0) is r
