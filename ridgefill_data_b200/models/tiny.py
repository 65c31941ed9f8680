"""Tiny random checkpoints for dry runs (code/scripts/make_tiny.py): the layer patterns and vocabulary sizes of the
real models at toy width, saved in Hugging Face layout (config.json + model.safetensors) so every loader, fit and
evaluation path runs end to end on a CPU in seconds.

    python -m ridgefill_data_b200.models.tiny OUT [--tokenizers DIR]

writes OUT/llama-3.1-8b-instruct (32 layers, llama3 RoPE scaling), OUT/llama-3.1-swiftkv-8b-instruct (the same plus
SwiftKV extras from layer 16: norm_swiftkv and *_proj_swiftkv), OUT/qwen3.5-9b (3:1 GDN : attention, partial RoPE
0.25) and OUT/qwen3-8b (q/k norm). With --tokenizers, DIR/<name>/ tokenizer files are copied beside each.
"""
from __future__ import annotations

import argparse
import shutil
from pathlib import Path

import torch

from .checkpoint import random_weights, save_checkpoint
from .config import ModelConfig, _hybrid_types

TOKENIZER_FILES = ("tokenizer.json", "tokenizer_config.json", "special_tokens_map.json", "vocab.json", "merges.txt",
                   "chat_template.jinja", "generation_config.json")


def tiny_configs(layers=32, width=64):
    llama = ModelConfig(arch="llama", n_layers=layers, hidden=width, vocab=128256, n_heads=4, n_kv=2, head_dim=16,
                        intermediate=2 * width, eps=1e-5, rope_theta=5e5, rope_type="llama3",
                        rope_llama3=dict(factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                                         original_max_position_embeddings=8192), max_positions=131072,
                        name="llama-3.1-8b-instruct")
    return {
        "llama-3.1-8b-instruct": llama,
        "llama-3.1-swiftkv-8b-instruct": llama.replace(swift_layers=layers // 2, name="llama-3.1-swiftkv-8b-instruct"),
        "qwen3.5-9b": ModelConfig(arch="qwen3_5", n_layers=layers, hidden=width, vocab=248320, n_heads=4, n_kv=2,
                                  head_dim=32, intermediate=2 * width, eps=1e-6, rope_theta=1e7, partial_rotary=0.25,
                                  layer_types=_hybrid_types(layers), gdn_nk=2, gdn_nv=4, gdn_dk=16, gdn_dv=16,
                                  max_positions=262144, name="qwen3.5-9b"),
        "qwen3-8b": ModelConfig(arch="qwen3", n_layers=layers, hidden=width, vocab=151936, n_heads=4, n_kv=2,
                                head_dim=16, intermediate=2 * width, eps=1e-6, rope_theta=1e6, max_positions=40960,
                                name="qwen3-8b"),
    }


def swiftkv_extras(cfg: ModelConfig, tensors, seed=1):
    """norm_swiftkv and the late layers' *_proj_swiftkv (q and v copied, k scaled by 1.1)."""
    tensors["model.norm_swiftkv.weight"] = torch.ones(cfg.hidden)
    for i in range(cfg.swift_layers, cfg.n_layers):
        p = f"model.layers.{i}.self_attn."
        tensors[p + "q_proj_swiftkv.weight"] = tensors[p + "q_proj.weight"].clone()
        tensors[p + "k_proj_swiftkv.weight"] = tensors[p + "k_proj.weight"] * 1.1
        tensors[p + "v_proj_swiftkv.weight"] = tensors[p + "v_proj.weight"].clone()
    return tensors


def make_tiny(out, names=None, tokenizers=None, layers=32, width=64, seed=0, dtype=torch.bfloat16):
    out = Path(out)
    paths = {}
    for name, cfg in tiny_configs(layers, width).items():
        if names is not None and name not in names:
            continue
        tensors = random_weights(cfg, seed=seed)
        if cfg.swift_layers is not None:
            swiftkv_extras(cfg, tensors)
        tensors = {k: v.to(dtype) if v.is_floating_point() and "A_log" not in k and "dt_bias" not in k else v
                   for k, v in tensors.items()}
        path = out / name
        save_checkpoint(path, cfg, tensors)
        if tokenizers is not None:
            for f in TOKENIZER_FILES:
                src = Path(tokenizers) / name / f
                if src.exists():
                    shutil.copy(src, path / f)
        paths[name] = path
    return paths


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("out")
    ap.add_argument("--tokenizers")
    ap.add_argument("--layers", type=int, default=32)
    a = ap.parse_args(argv)
    for name, p in make_tiny(a.out, tokenizers=a.tokenizers, layers=a.layers).items():
        print(name, p)


if __name__ == "__main__":
    main()
