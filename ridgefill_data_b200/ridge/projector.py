"""Ridge-map files and the projector that applies them.

File format (safetensors, code/kva/kva.py:188-193): key `layer.{i}` = bf16 [d_out, d_in + 1], the map
with the bias as the last column; string metadata split, model, model_commit, lam, rows, taps, sweep,
calib_exclude_sha256, code_commit, code_dirty, docs, note. save() and load() refuse a non-finite weight
or |w| > 1e4 (code/kva/kva.py:121-134); load() checks the file's sha256 against a recorded one (or the
disk copy read around the page cache).

Also read here: the int8 release layout `i8_row128` (proj.L.codes int8 [d, W], proj.L.scale bf16 [d, W/128],
proj.L.bias bf16 [d]; row i's 128-column group g is codes[i, 128g:128g+128] * scale[i, g],
code/c5/convert.py:96-104) and the Gated DeltaNet terminal-state correction `st.L` fp32 [heads, dv, dk]
(code/c5/convert.py:120-136), which this engine stores transposed as its state layout [heads, dk, dv].
"""
from __future__ import annotations

import json
from pathlib import Path

import torch
import torch.nn.functional as F

MAX_ABS_WEIGHT = 1e4
I8_GROUP = 128


def check_weights(tensors, where):
    """Refuse any map holding a NaN / inf or a weight beyond MAX_ABS_WEIGHT in magnitude."""
    for name, t in tensors.items():
        vals = t.float()
        ok = torch.isfinite(vals) & (vals.abs() <= MAX_ABS_WEIGHT)
        if bool(ok.all()):
            continue
        where_bad = (~ok).nonzero()
        r, c = where_bad[0].tolist()
        raise ValueError(f"{where}: refusing {name}: {where_bad.shape[0]} weights are NaN, infinite or above "
                         f"{MAX_ABS_WEIGHT:g} in magnitude (first at row {r}, col {c}: {vals[r, c].item():.4g})")


def _header_meta(data):
    """The __metadata__ map of safetensors bytes (empty when absent)."""
    size = int.from_bytes(data[:8], "little")
    return json.loads(data[8:8 + size]).get("__metadata__") or {}


def stable_safetensors(tensors, metadata=None):
    """safetensors bytes with a canonical header (keys sorted, compact JSON, padded to 8 bytes): the library writes
    its metadata map in hash order, so equal content could otherwise serialise to different bytes. The data
    section and its offsets are the library's (tensors in a fixed order)."""
    from safetensors.torch import save
    blob = save(tensors, metadata=metadata)
    n = int.from_bytes(blob[:8], "little")
    header = json.dumps(json.loads(blob[8:8 + n]), sort_keys=True, separators=(",", ":")).encode()
    header += b" " * (-len(header) % 8)
    return len(header).to_bytes(8, "little") + header + blob[8 + n:]


def meta_of(path):
    """A map file's metadata (strings) from its safetensors header alone."""
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        return json.loads(f.read(n)).get("__metadata__") or {}


class Projector:
    """Per late layer i: x_i = b W_i^T + c_i in the activation dtype. Maps may live on the host; the first
    call on a device copies them there (release() drops the device copy)."""

    def __init__(self, split, weights, biases, meta=None):
        self.split = split
        self.W = weights
        self.b = biases
        self.meta = dict(meta or {})
        self._dev = None
        self.sha256 = None

    @property
    def layers(self):
        return sorted(self.W)

    def to(self, device, dtype=None):
        """A projector whose maps are resident on `device` (the B200 engine keeps them in HBM)."""
        dt = dtype or next(iter(self.W.values())).dtype
        p = type(self)(self.split, {i: w.to(device, dt).contiguous() for i, w in self.W.items()},
                       {i: c.to(device, dt).contiguous() for i, c in self.b.items()}, self.meta)
        p.sha256 = self.sha256
        for k in ("n_kv", "eps"):
            if hasattr(self, k):
                setattr(p, k, getattr(self, k))
        return p

    def device_maps(self, device):
        if self.W[self.layers[0]].device == torch.device(device):
            return self.W, self.b
        if self._dev is None or self._dev[0] != torch.device(device):
            self._dev = (torch.device(device), {k: w.to(device) for k, w in self.W.items()},
                         {k: x.to(device) for k, x in self.b.items()})
        return self._dev[1], self._dev[2]

    def __call__(self, i, b):
        W, B = self.device_maps(b.device)
        return F.linear(b, W[i].to(b.dtype), B[i].to(b.dtype))

    def device_map(self, i, device):
        """(W_i, c_i) on `device` for a consumer that calls done_with(i) once its kernels reading them are queued."""
        W, B = self.device_maps(device)
        return W[i], B[i]

    def done_with(self, i):
        """The consumer of layer i's map has queued every kernel that reads it (resident maps: nothing to do)."""

    def begin(self, device):
        """A prompt's prefill starts (resident maps: nothing to do)."""

    def release(self):
        self._dev = None


    def tensors(self):
        return {f"layer.{i}": torch.cat((self.W[i], self.b[i][:, None]), 1).to(torch.bfloat16).cpu().contiguous()
                for i in self.layers}

    def save(self, path, meta):
        """The map file (bytes reproducible: a canonical header)."""
        t = self.tensors()
        check_weights(t, f"Projector.save {path}")
        Path(path).write_bytes(stable_safetensors(t, {k: str(v) for k, v in dict(meta, split=self.split).items()}))

    @classmethod
    def load(cls, path, device="cpu", dtype=torch.bfloat16, sha256=None):
        """A map file, or a release directory (ridgefill.json + int8 maps: ridge/release.py)."""
        if Path(path).is_dir():
            from . import release
            return release.load(path, device, dtype)
        from safetensors.torch import load as from_bytes

        from ..utils import integrity
        data, sha = integrity.read_verified(path, sha256)
        meta = _header_meta(data)
        W, B = {}, {}
        for name, packed in from_bytes(data).items():
            check_weights({name: packed}, f"Projector.load {path}")
            layer = int(name.split(".")[1])
            weight, bias = packed.split([packed.shape[1] - 1, 1], dim=1)
            W[layer] = weight.to(device, dtype).contiguous()
            B[layer] = bias.squeeze(1).to(device, dtype).contiguous()
        p = cls(int(meta["split"]), W, B, meta)
        p.sha256 = sha
        return p

    @classmethod
    def load_i8(cls, files, split, device="cpu", dtype=torch.bfloat16):
        """The int8 release layout: files {layer: path of a safetensors file holding proj.L.codes / scale /
        bias}. Dequantised exactly in fp32 (8-bit code x bf16 scale fits fp32), then one cast to dtype."""
        from safetensors.torch import load_file
        W, B = {}, {}
        for L, path in files.items():
            t = load_file(str(path))
            w, b = dequant_i8(t[f"proj.{L}.codes"], t[f"proj.{L}.scale"], t[f"proj.{L}.bias"])
            check_weights({f"layer.{L}": torch.cat((w, b[:, None]), 1)}, f"Projector.load_i8 {path}")
            W[int(L)] = w.to(device, dtype).contiguous()
            B[int(L)] = b.to(device, dtype).contiguous()
        return cls(split, W, B, dict(layout="i8_row128"))


class StreamedProjector(Projector):
    """Maps kept in pinned host memory and streamed to the GPU per prompt, for HBM budgets that cannot hold every late
    layer's map (the E3 engine's --ridgefill-stream-projector option, code/qwen38-27b-kit/common.py:27).

    A ring of `slots` device buffers holds the maps in flight. begin() (called as the prompt's lower layers start)
    queues the host-to-device copies of the first `slots` maps on a copy stream, so they overlap the lower layers;
    device_map(i) makes the compute stream wait for layer i's copy; done_with(i) records when the compute stream is
    finished with the slot and queues the copy of map i + slots into it. HBM held: slots x (d_out x (d_in + 1)) bf16
    instead of every late layer's map. Maps are consumed in layer order."""

    def __init__(self, split, weights, biases, meta=None, slots=4):
        host_w = {i: w.detach().to("cpu").contiguous().pin_memory() for i, w in weights.items()}
        host_b = {i: c.detach().to("cpu").contiguous().pin_memory() for i, c in biases.items()}
        super().__init__(split, host_w, host_b, meta)
        self.slots = max(1, int(slots))
        self._ring = None
        self._order = []
        self._ready = {}

    def _setup(self, device):
        device = torch.device(device)
        if self._ring is not None and self._ring["device"] == device:
            return self._ring
        first = self.layers[0]
        W0, B0 = self.W[first], self.b[first]
        k = min(self.slots, len(self.layers))
        self._ring = dict(device=device, stream=torch.cuda.Stream(device=device),
                          w=[torch.empty_like(W0, device=device) for _ in range(k)],
                          b=[torch.empty_like(B0, device=device) for _ in range(k)],
                          free=[None] * k, slot_of={})
        return self._ring

    def _issue(self, pos):
        r = self._ring
        layer = self._order[pos]
        slot = pos % len(r["w"])
        with torch.cuda.stream(r["stream"]):
            if r["free"][slot] is not None:
                r["stream"].wait_event(r["free"][slot])     # the kernels that read this slot last have finished
            r["w"][slot].copy_(self.W[layer], non_blocking=True)
            r["b"][slot].copy_(self.b[layer], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(r["stream"])
        self._ready[layer] = (slot, ev, pos)

    def begin(self, device):
        r = self._setup(device)
        self._order = list(self.layers)
        self._ready = {}
        for pos in range(min(len(r["w"]), len(self._order))):
            self._issue(pos)

    def device_map(self, i, device):
        if self._ring is None or self._ring["device"] != torch.device(device) or i not in self._ready:
            self.begin(device)                                  # a consumer that did not call begin()
            while self._ready and i not in self._ready:
                self.done_with(next(iter(self._ready)))
        slot, ev, _ = self._ready[i]
        torch.cuda.current_stream(self._ring["device"]).wait_event(ev)
        return self._ring["w"][slot], self._ring["b"][slot]

    def done_with(self, i):
        if i not in self._ready:
            return
        slot, _, pos = self._ready.pop(i)
        r = self._ring
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(r["device"]))
        r["free"][slot] = ev
        nxt = pos + len(r["w"])
        if nxt < len(self._order):
            self._issue(nxt)

    def device_maps(self, device):
        raise RuntimeError("streamed maps are read one layer at a time (device_map / done_with)")

    def __call__(self, i, b):
        if b.device.type != "cuda":
            return F.linear(b, self.W[i].to(b.device, b.dtype), self.b[i].to(b.device, b.dtype))
        w, c = self.device_map(i, b.device)
        out = F.linear(b, w.to(b.dtype), c.to(b.dtype))
        self.done_with(i)
        return out

    def resident_bytes(self):
        r = self._ring
        return 0 if r is None else sum(t.numel() * t.element_size() for t in r["w"] + r["b"])

    def release(self):
        torch.cuda.synchronize() if self._ring is not None else None
        self._ring, self._ready = None, {}


def dequant_i8(codes, scale, bias):
    rows, width = codes.shape
    if codes.dtype != torch.int8 or width % I8_GROUP or scale.shape != (rows, width // I8_GROUP) or \
            bias.shape != (rows,):
        raise ValueError(f"i8_row128 shapes {tuple(codes.shape)} {tuple(scale.shape)} {tuple(bias.shape)}")
    w = codes.float().view(rows, width // I8_GROUP, I8_GROUP) * scale.float()[:, :, None]
    return w.view(rows, width), bias.float()


def quant_i8(w, bias):
    """The i8_row128 encoding of an fp32 map (per row and 128-column group: scale = max|w| / 127)."""
    rows, width = w.shape
    g = w.float().view(rows, width // I8_GROUP, I8_GROUP)
    scale = (g.abs().amax(-1) / 127.0).clamp(min=1e-30).to(torch.bfloat16)
    codes = torch.round(g / scale.float()[:, :, None]).clamp(-127, 127).to(torch.int8).view(rows, width)
    return codes, scale, bias.to(torch.bfloat16)


class KVFold(Projector):
    """Per late attention layer: pre-RoPE [k | v] = u W_i^T + c_i with u = b / rms(b) (eps of the model's
    input norm; fp32, cast back) (code/kva/kva.py:196-219). Metadata n_kv and eps."""

    def __init__(self, split, weights, biases, n_kv, eps, meta=None):
        super().__init__(split, weights, biases, meta)
        self.n_kv, self.eps = n_kv, eps

    def kv(self, i, b):
        xf = b.float()
        u = (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + self.eps)).to(b.dtype)
        return self(i, u).unflatten(-1, (2, self.n_kv, -1)).unbind(1)

    @classmethod
    def load(cls, path, device="cpu", dtype=torch.bfloat16, sha256=None):
        p = Projector.load(path, device, dtype, sha256)
        f = cls(p.split, p.W, p.b, int(p.meta["n_kv"]), float(p.meta["eps"]), p.meta)
        f.sha256 = p.sha256
        return f

    def save(self, path, meta):
        super().save(path, dict(meta, n_kv=self.n_kv, eps=self.eps))


def save_st(path, st):
    """Terminal-state corrections {layer: [heads, dk, dv] fp32} as st.L [heads, dv, dk] (release layout)."""
    from safetensors.torch import save_file
    save_file({f"st.{i}": v.float().transpose(1, 2).contiguous().cpu() for i, v in st.items()}, str(path))


def load_st(path, device="cpu"):
    """{layer: [heads, dk, dv] fp32} from a release-layout correction file (or a torch .pt {layer: tensor}
    already in the state layout)."""
    path = str(path)
    if path.endswith(".pt"):
        return {int(k): v.float().to(device) for k, v in torch.load(path, map_location="cpu").items()}
    from safetensors.torch import load_file
    return {int(k.split(".")[1]): v.float().transpose(1, 2).contiguous().to(device)
            for k, v in load_file(path).items()}
