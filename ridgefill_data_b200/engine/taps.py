"""Debug tap on the fill inputs (the role of code/qwen38-27b-kit/identity_hidden.cpp:19-93): capture the first
`rows` rows of every late layer's fill input x_l during a prefill and check them against the split state h_S
(identity fill: bit for bit) or against an fp32 CPU restatement of the ridge map (x_l = h_S W_l^T + c_l, within
bf16 rounding).

    tap = FillTap(rows=112)
    with attached(model, tap):
        prefill(model, ids, arm)
    tap.check_identity(h_split)                 # {layer: mismatching values}
    tap.check_maps(h_split, projector)          # {layer: max relative error}
"""
from __future__ import annotations

from contextlib import contextmanager

import torch


class FillTap:
    def __init__(self, rows=112):
        self.rows = rows
        self.got = {}

    def __call__(self, i, x):
        self.got[i] = x[:self.rows].detach().to("cpu", copy=True)

    def check_identity(self, h_split):
        """{layer: number of values that differ bitwise from h_S's rows}."""
        ref = h_split[:self.rows].detach().cpu()
        return {i: int((x.view(torch.int16) != ref.to(x.dtype).view(torch.int16)).sum()) if x.dtype == torch.bfloat16
                else int((x != ref.to(x.dtype)).sum()) for i, x in self.got.items()}

    def check_maps(self, h_split, projector):
        """{layer: max |x_l - oracle| / max |oracle|} with the oracle in fp32 on the CPU."""
        b = h_split[:self.rows].detach().cpu().float()
        out = {}
        for i, x in self.got.items():
            w, c = projector.W[i], projector.b[i]
            want = b @ w.float().cpu().T + c.float().cpu()
            out[i] = float((x.float() - want).abs().max() / want.abs().max().clamp_min(1e-12))
        return out


@contextmanager
def attached(model, tap):
    """Route every model.fill(i, x, ...) call (the batched B200 fill included) through the tap first."""
    inner = model.fill

    def fill(i, x, pos, cache, **kw):
        tap(i, x)
        return inner(i, x, pos, cache, **kw)
    model.fill = fill
    try:
        yield tap
    finally:
        del model.fill
