"""Typed model configuration.

One dataclass covers every architecture the engine runs: Llama-3.1 (with the optional SwiftKV
extras), dense Qwen3 (per-head q/k RMSNorm), the Qwen3.5 hybrid (Gated DeltaNet + gated attention)
and its mixture-of-experts variant. `from_hf` reads a Hugging Face config.json (the `text_config`
of a multimodal wrapper when present) and refuses features the forward pass does not implement
(code/kva/model.py:313-330, :574-586: attention bias, sliding window, YaRN-style RoPE scaling).

PRESETS holds the five shapes named by the benchmark plan (random-init weights of these shapes are
what bench.py and the tests run).
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from pathlib import Path


class UnsupportedArchitecture(ValueError):
    """config.json describes a model (or a feature) this forward pass does not implement."""


ARCHS = ("llama", "qwen3", "qwen3_5", "qwen3_5_moe")


@dataclass
class ModelConfig:
    arch: str
    n_layers: int
    hidden: int
    vocab: int
    n_heads: int
    n_kv: int
    head_dim: int
    intermediate: int
    eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_type: str = "default"                       # default | llama3
    rope_llama3: dict = field(default_factory=dict)  # factor, low_freq_factor, high_freq_factor, original_max_position_embeddings
    partial_rotary: float = 1.0
    layer_types: list = field(default_factory=list)  # per layer: 'attn' | 'gdn'
    # Gated DeltaNet
    gdn_nk: int = 0
    gdn_nv: int = 0
    gdn_dk: int = 0
    gdn_dv: int = 0
    conv_k: int = 4
    # mixture of experts (qwen3_5_moe)
    n_experts: int = 0
    top_k: int = 0
    moe_intermediate: int = 0
    shared_intermediate: int = 0
    # SwiftKV extras (llama): layers >= swift_layers have *_proj_swiftkv weights
    swift_layers: int | None = None
    tie_embeddings: bool = False
    max_positions: int | None = None
    name: str = ""

    def __post_init__(self):
        if self.arch not in ARCHS:
            raise UnsupportedArchitecture(f"arch {self.arch!r} (known: {', '.join(ARCHS)})")
        if not self.layer_types:
            self.layer_types = ["attn"] * self.n_layers
        if self.n_heads % self.n_kv:
            raise UnsupportedArchitecture(f"{self.n_heads} query heads not a multiple of {self.n_kv} KV heads")

    # ---- derived shapes
    @property
    def rot_dim(self):
        return int(self.head_dim * self.partial_rotary)

    @property
    def gated_attn(self):
        return self.arch in ("qwen3_5", "qwen3_5_moe")

    @property
    def zero_centred_norm(self):
        return self.arch in ("qwen3_5", "qwen3_5_moe")

    @property
    def qk_norm(self):
        return self.arch in ("qwen3", "qwen3_5", "qwen3_5_moe")

    @property
    def moe(self):
        return self.arch == "qwen3_5_moe"

    @property
    def gdn_conv_dim(self):
        return 2 * self.gdn_nk * self.gdn_dk + self.gdn_nv * self.gdn_dv

    def attn_layers(self):
        return [i for i, t in enumerate(self.layer_types) if t == "attn"]

    def gdn_layers(self):
        return [i for i, t in enumerate(self.layer_types) if t == "gdn"]

    def param_count(self, embeddings=True):
        """Weight count of the forward pass (for FLOP and memory estimates)."""
        d = self.hidden
        tot = 0
        for t in self.layer_types:
            if t == "attn":
                q = self.n_heads * self.head_dim * (2 if self.gated_attn else 1)
                tot += d * (q + 2 * self.n_kv * self.head_dim) + self.n_heads * self.head_dim * d
            else:
                vd = self.gdn_nv * self.gdn_dv
                tot += d * (self.gdn_conv_dim + vd + 2 * self.gdn_nv) + vd * d
            if self.moe:
                tot += d * self.n_experts + 3 * d * self.moe_intermediate * self.n_experts
                tot += 3 * d * self.shared_intermediate + d
            else:
                tot += 3 * d * self.intermediate
        if embeddings:
            tot += self.vocab * d * (1 if self.tie_embeddings else 2)
        return tot

    def active_param_count(self):
        """Weights one token touches (MoE: top_k routed experts + the shared expert), without embeddings."""
        if not self.moe:
            return self.param_count(embeddings=False)
        full = self.param_count(embeddings=False)
        routed_all = 3 * self.hidden * self.moe_intermediate * self.n_experts * self.n_layers
        routed_act = 3 * self.hidden * self.moe_intermediate * self.top_k * self.n_layers
        return full - routed_all + routed_act

    def replace(self, **kw):
        return dataclasses.replace(self, **kw)

    # ---- Hugging Face config.json
    @classmethod
    def from_hf(cls, raw: dict, name: str = "") -> "ModelConfig":
        c = raw.get("text_config", raw)
        mt = str(c.get("model_type", raw.get("model_type")))
        rs = c.get("rope_parameters") or c.get("rope_scaling") or {}
        theta = rs.get("rope_theta", c.get("rope_theta", 10000.0))
        common = dict(n_layers=c["num_hidden_layers"], hidden=c["hidden_size"], vocab=c["vocab_size"],
                      n_heads=c["num_attention_heads"], n_kv=c["num_key_value_heads"],
                      eps=c["rms_norm_eps"], rope_theta=float(theta),
                      tie_embeddings=bool(c.get("tie_word_embeddings", False)),
                      max_positions=c.get("max_position_embeddings"), name=name)
        if mt in ("llama", "llama_swiftkv"):
            rt = rs.get("rope_type", "default")
            if rt not in ("default", "llama3"):
                raise UnsupportedArchitecture(f"llama rope_type {rt!r}")
            if c.get("attention_bias") or c.get("mlp_bias"):
                raise UnsupportedArchitecture("llama with biases")
            hd = c.get("head_dim") or c["hidden_size"] // c["num_attention_heads"]
            l3 = {k: rs[k] for k in ("factor", "low_freq_factor", "high_freq_factor",
                                     "original_max_position_embeddings")} if rt == "llama3" else {}
            return cls(arch="llama", head_dim=hd, intermediate=c["intermediate_size"], rope_type=rt, rope_llama3=l3,
                       swift_layers=c.get("num_key_value_layers") if c.get("swiftkv") else None, **common)
        if mt == "qwen3":
            problems = [k for k in ("attention_bias", "use_sliding_window") if c.get(k)]
            if rs.get("rope_type", "default") != "default":
                problems.append(f"rope_type {rs.get('rope_type')}")
            if problems:
                raise UnsupportedArchitecture(f"qwen3 with {', '.join(map(str, problems))}")
            hd = c.get("head_dim") or c["hidden_size"] // c["num_attention_heads"]
            return cls(arch="qwen3", head_dim=hd, intermediate=c["intermediate_size"], **common)
        if mt.startswith("qwen3_5"):
            types = ["gdn" if t == "linear_attention" else "attn" for t in c["layer_types"]]
            prf = rs.get("partial_rotary_factor", c.get("partial_rotary_factor", 1.0))
            kw = dict(head_dim=c["head_dim"], partial_rotary=float(prf), layer_types=types,
                      gdn_nk=c["linear_num_key_heads"], gdn_nv=c["linear_num_value_heads"],
                      gdn_dk=c["linear_key_head_dim"], gdn_dv=c["linear_value_head_dim"],
                      conv_k=c["linear_conv_kernel_dim"])
            if "moe" in mt:
                return cls(arch="qwen3_5_moe", intermediate=c.get("intermediate_size") or 0,
                           n_experts=c["num_experts"], top_k=c["num_experts_per_tok"],
                           moe_intermediate=c["moe_intermediate_size"],
                           shared_intermediate=c["shared_expert_intermediate_size"], **kw, **common)
            return cls(arch="qwen3_5", intermediate=c["intermediate_size"], **kw, **common)
        raise UnsupportedArchitecture(f"model_type {mt!r} has no forward pass here (llama, llama_swiftkv, qwen3, "
                                      f"qwen3_5*)")

    @classmethod
    def from_dir(cls, path) -> "ModelConfig":
        path = Path(path)
        return cls.from_hf(json.loads((path / "config.json").read_text()), name=path.name)

    def to_hf(self) -> dict:
        """A config.json that from_hf reads back to this config (and transformers can load)."""
        c = dict(num_hidden_layers=self.n_layers, hidden_size=self.hidden, vocab_size=self.vocab,
                 num_attention_heads=self.n_heads, num_key_value_heads=self.n_kv, head_dim=self.head_dim,
                 rms_norm_eps=self.eps, tie_word_embeddings=self.tie_embeddings,
                 max_position_embeddings=self.max_positions or 131072, hidden_act="silu")
        if self.arch == "llama":
            c.update(model_type="llama", architectures=["LlamaForCausalLM"], intermediate_size=self.intermediate,
                     attention_bias=False, mlp_bias=False)
            if self.rope_type == "llama3":
                c["rope_scaling"] = dict(rope_type="llama3", rope_theta=self.rope_theta, **self.rope_llama3)
            c["rope_theta"] = self.rope_theta
            if self.swift_layers is not None:
                c.update(swiftkv=True, num_key_value_layers=self.swift_layers, key_value_group_size=1)
        elif self.arch == "qwen3":
            c.update(model_type="qwen3", architectures=["Qwen3ForCausalLM"], intermediate_size=self.intermediate,
                     rope_theta=self.rope_theta, attention_bias=False, use_sliding_window=False)
        else:
            c.update(layer_types=["linear_attention" if t == "gdn" else "full_attention" for t in self.layer_types],
                     linear_num_key_heads=self.gdn_nk, linear_num_value_heads=self.gdn_nv,
                     linear_key_head_dim=self.gdn_dk, linear_value_head_dim=self.gdn_dv,
                     linear_conv_kernel_dim=self.conv_k, attn_output_gate=self.gated_attn,
                     rope_parameters=dict(rope_type="default", rope_theta=self.rope_theta,
                                          partial_rotary_factor=self.partial_rotary))
            if self.arch == "qwen3_5_moe":
                c.update(model_type="qwen3_5_moe_text", architectures=["Qwen3_5MoeForCausalLM"],
                         num_experts=self.n_experts, num_experts_per_tok=self.top_k,
                         moe_intermediate_size=self.moe_intermediate,
                         shared_expert_intermediate_size=self.shared_intermediate)
            else:
                c.update(model_type="qwen3_5_text", architectures=["Qwen3_5ForCausalLM"],
                         intermediate_size=self.intermediate)
        return c


def _hybrid_types(n, period=4):
    """Every `period`-th layer full attention, the rest Gated DeltaNet (3:1 for period 4)."""
    return ["attn" if (i + 1) % period == 0 else "gdn" for i in range(n)]


PRESETS = {
    # Benchmark plan config 1: tiny Llama-style decoder on CPU in fp32.
    "tiny-llama": ModelConfig(arch="llama", n_layers=8, hidden=256, vocab=4096, n_heads=4, n_kv=2, head_dim=64,
                              intermediate=704, eps=1e-6, rope_theta=1e4, name="tiny-llama"),
    # Llama-3.1-8B shape.
    "llama-3.1-8b": ModelConfig(arch="llama", n_layers=32, hidden=4096, vocab=128256, n_heads=32, n_kv=8,
                                head_dim=128, intermediate=14336, eps=1e-5, rope_theta=5e5, rope_type="llama3",
                                rope_llama3=dict(factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                                                 original_max_position_embeddings=8192),
                                max_positions=131072, name="llama-3.1-8b"),
    # Qwen3-8B shape.
    "qwen3-8b": ModelConfig(arch="qwen3", n_layers=36, hidden=4096, vocab=151936, n_heads=32, n_kv=8, head_dim=128,
                            intermediate=12288, eps=1e-6, rope_theta=1e6, max_positions=40960, name="qwen3-8b"),
    # 27B-class hybrid (Qwen3.8-27B-shaped).
    "qwen3.8-27b": ModelConfig(arch="qwen3_5", n_layers=64, hidden=5120, vocab=248320, n_heads=24, n_kv=4,
                               head_dim=256, intermediate=17408, eps=1e-6, rope_theta=1e7, partial_rotary=0.25,
                               layer_types=_hybrid_types(64), gdn_nk=16, gdn_nv=48, gdn_dk=128, gdn_dv=128,
                               conv_k=4, max_positions=262144, name="qwen3.8-27b"),
    # MoE hybrid (Flash-Next-shaped, 80B total / 3B active).
    "flash-next": ModelConfig(arch="qwen3_5_moe", n_layers=48, hidden=2048, vocab=151936, n_heads=16, n_kv=2,
                              head_dim=256, intermediate=0, eps=1e-6, rope_theta=1e7, partial_rotary=0.25,
                              layer_types=_hybrid_types(48), gdn_nk=16, gdn_nv=32, gdn_dk=128, gdn_dv=128,
                              conv_k=4, n_experts=512, top_k=10, moe_intermediate=512, shared_intermediate=512,
                              max_positions=262144, name="flash-next"),
}
