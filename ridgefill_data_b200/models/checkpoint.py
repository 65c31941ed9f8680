"""Weights: lazy access to (sharded) safetensors checkpoints and seeded random initialisation.

Checkpoint mirrors the reference's lazy reader (code/kva/model.py:46-68): tensors are read one at a
time straight onto the target device. `random_weights` builds a full Hugging Face-named state dict
of a ModelConfig from a seed (N(0, std) matrices, norm weights near their neutral value), which is
what the benchmark and the tests run: there are no real checkpoints on the GPU boxes.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch
from safetensors import safe_open

from .config import ModelConfig


class Checkpoint:
    """Lazy tensor access over model.safetensors or a model.safetensors.index.json shard set."""

    def __init__(self, path):
        self.path = Path(path)
        index = self.path / "model.safetensors.index.json"
        if index.exists():
            self.map = json.loads(index.read_text())["weight_map"]
        else:
            with safe_open(self.path / "model.safetensors", "pt") as f:
                self.map = {k: "model.safetensors" for k in f.keys()}
        self.files = {}

    def __contains__(self, key):
        return key in self.map

    def keys(self):
        return self.map.keys()

    def get(self, key, device="cpu", dtype=None):
        name = self.map[key]
        handle = (name, str(device))
        if handle not in self.files:
            self.files[handle] = safe_open(self.path / name, "pt", device=str(device))
        t = self.files[handle].get_tensor(key)
        return t.to(dtype) if dtype is not None and t.is_floating_point() else t


class DictSource:
    """The Checkpoint interface over an in-memory state dict (random init, tests)."""

    def __init__(self, tensors):
        self.tensors = tensors

    def __contains__(self, key):
        return key in self.tensors

    def keys(self):
        return self.tensors.keys()

    def get(self, key, device="cpu", dtype=None):
        t = self.tensors[key].to(device)
        return t.to(dtype) if dtype is not None and t.is_floating_point() else t


def hf_names(cfg: ModelConfig, prefix="model."):
    """{name: shape} of every weight of cfg in Hugging Face naming."""
    d = cfg.hidden
    names = {f"{prefix}embed_tokens.weight": (cfg.vocab, d), f"{prefix}norm.weight": (d,)}
    if not cfg.tie_embeddings:
        names["lm_head.weight"] = (cfg.vocab, d)
    for i, t in enumerate(cfg.layer_types):
        p = f"{prefix}layers.{i}."
        names[p + "input_layernorm.weight"] = (d,)
        names[p + "post_attention_layernorm.weight"] = (d,)
        if t == "attn":
            a = p + "self_attn."
            qw = cfg.n_heads * cfg.head_dim * (2 if cfg.gated_attn else 1)
            names[a + "q_proj.weight"] = (qw, d)
            names[a + "k_proj.weight"] = (cfg.n_kv * cfg.head_dim, d)
            names[a + "v_proj.weight"] = (cfg.n_kv * cfg.head_dim, d)
            names[a + "o_proj.weight"] = (d, cfg.n_heads * cfg.head_dim)
            if cfg.qk_norm:
                names[a + "q_norm.weight"] = (cfg.head_dim,)
                names[a + "k_norm.weight"] = (cfg.head_dim,)
        else:
            a = p + "linear_attn."
            vd = cfg.gdn_nv * cfg.gdn_dv
            names[a + "in_proj_qkv.weight"] = (cfg.gdn_conv_dim, d)
            names[a + "in_proj_z.weight"] = (vd, d)
            names[a + "in_proj_b.weight"] = (cfg.gdn_nv, d)
            names[a + "in_proj_a.weight"] = (cfg.gdn_nv, d)
            names[a + "conv1d.weight"] = (cfg.gdn_conv_dim, 1, cfg.conv_k)
            names[a + "A_log"] = (cfg.gdn_nv,)
            names[a + "dt_bias"] = (cfg.gdn_nv,)
            names[a + "norm.weight"] = (cfg.gdn_dv,)
            names[a + "out_proj.weight"] = (d, vd)
        if cfg.moe:
            m = p + "mlp."
            names[m + "gate.weight"] = (cfg.n_experts, d)
            names[m + "experts.gate_up_proj"] = (cfg.n_experts, 2 * cfg.moe_intermediate, d)
            names[m + "experts.down_proj"] = (cfg.n_experts, d, cfg.moe_intermediate)
            names[m + "shared_expert.gate_proj.weight"] = (cfg.shared_intermediate, d)
            names[m + "shared_expert.up_proj.weight"] = (cfg.shared_intermediate, d)
            names[m + "shared_expert.down_proj.weight"] = (d, cfg.shared_intermediate)
            names[m + "shared_expert_gate.weight"] = (1, d)
        else:
            m = p + "mlp."
            names[m + "gate_proj.weight"] = (cfg.intermediate, d)
            names[m + "up_proj.weight"] = (cfg.intermediate, d)
            names[m + "down_proj.weight"] = (d, cfg.intermediate)
    if cfg.swift_layers is not None:
        names[f"{prefix}norm_swiftkv.weight"] = (d,)
        for i in range(cfg.swift_layers, cfg.n_layers):
            a = f"{prefix}layers.{i}.self_attn."
            names[a + "q_proj_swiftkv.weight"] = (cfg.n_heads * cfg.head_dim, d)
            names[a + "k_proj_swiftkv.weight"] = (cfg.n_kv * cfg.head_dim, d)
            names[a + "v_proj_swiftkv.weight"] = (cfg.n_kv * cfg.head_dim, d)
    return names


def random_tensor(name, shape, cfg: ModelConfig, gen, std=0.02, dtype=torch.float32, device="cpu"):
    """Seeded init of one weight: N(0, std) matrices; norm weights 1 + N(0, 0.1) (zero-centred norms:
    N(0, 0.1)); GDN A_log ~ log U(1, 16), dt_bias ~ N(0, 0.1) (softplus-positive decay rates)."""
    if name.endswith("A_log"):
        t = torch.empty(shape).uniform_(1.0, 16.0, generator=gen).log()
    elif name.endswith("dt_bias"):
        t = 0.1 * torch.randn(shape, generator=gen)
    elif name.endswith("conv1d.weight"):
        t = torch.randn(shape, generator=gen) / cfg.conv_k ** 0.5
    elif len(shape) == 1:
        base = 0.0 if (cfg.zero_centred_norm and "linear_attn.norm" not in name) else 1.0
        t = base + 0.1 * torch.randn(shape, generator=gen)
    else:
        t = std * torch.randn(shape, generator=gen)
    return t.to(device=device, dtype=dtype)


def random_weights(cfg: ModelConfig, seed=0, std=0.02, dtype=torch.float32, device="cpu"):
    """A full Hugging Face-named state dict of cfg from `seed` (deterministic across machines: the
    generator runs on the CPU in a fixed name order)."""
    gen = torch.Generator().manual_seed(seed)
    return {n: random_tensor(n, s, cfg, gen, std, dtype, device) for n, s in hf_names(cfg).items()}


def save_checkpoint(path, cfg: ModelConfig, tensors, shard_bytes=None):
    """Write config.json + model.safetensors (or shards with an index when shard_bytes is given)."""
    from safetensors.torch import save_file
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    (path / "config.json").write_text(json.dumps(cfg.to_hf(), indent=1))
    tensors = {k: v.contiguous().cpu() for k, v in tensors.items()}
    if shard_bytes is None:
        save_file(tensors, str(path / "model.safetensors"))
        return path
    shards, cur, size = [], {}, 0
    for k in sorted(tensors):
        nb = tensors[k].numel() * tensors[k].element_size()
        if cur and size + nb > shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = tensors[k]
        size += nb
    if cur:
        shards.append(cur)
    wmap = {}
    for j, sh in enumerate(shards):
        fn = f"model-{j + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, str(path / fn))
        wmap.update({k: fn for k in sh})
    (path / "model.safetensors.index.json").write_text(json.dumps(dict(metadata={}, weight_map=wmap)))
    return path


class RandomSource:
    """Lazily generated seeded random weights (the Checkpoint interface), each tensor drawn on the target
    device from its own generator seeded by (seed, name): no host copy of the whole model is ever built,
    which is what lets a 27B-shaped model initialise straight into HBM."""

    def __init__(self, cfg: ModelConfig, seed=0, std=0.02):
        import zlib
        self.cfg = cfg
        self.seed = seed
        self.std = std
        self.shapes = hf_names(cfg)
        self._crc = zlib.crc32

    def __contains__(self, key):
        return key in self.shapes

    def keys(self):
        return self.shapes.keys()

    def get(self, key, device="cpu", dtype=None):
        dev = torch.device(device)
        s = (self.seed * 1000003 + self._crc(key.encode())) % (2**62)
        gen = torch.Generator(device=dev).manual_seed(s)
        shape = self.shapes[key]
        cfg = self.cfg
        if key.endswith("A_log"):
            t = torch.empty(shape, device=dev).uniform_(1.0, 16.0, generator=gen).log()
        elif key.endswith("dt_bias"):
            t = 0.1 * torch.randn(shape, generator=gen, device=dev)
        elif key.endswith("conv1d.weight"):
            t = torch.randn(shape, generator=gen, device=dev) / cfg.conv_k ** 0.5
        elif len(shape) == 1:
            base = 0.0 if (cfg.zero_centred_norm and "linear_attn.norm" not in key) else 1.0
            t = base + 0.1 * torch.randn(shape, generator=gen, device=dev)
        else:
            t = self.std * torch.randn(shape, generator=gen, device=dev)
        if dtype is not None and not key.endswith(("A_log", "dt_bias")):
            t = t.to(dtype)
        return t
