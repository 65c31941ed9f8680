"""Shared fixtures: tiny random Hugging Face checkpoints of every supported family (written once per session), and
the `gpu` marker (skipped without a CUDA device)."""
import os

import pytest
import torch

for _k in ("HF_HUB_OFFLINE", "HF_HUB_DISABLE_IMPLICIT_TOKEN"):
    os.environ.setdefault(_k, "1")

# under pytest-xdist, share the cores among the workers instead of every worker starting one thread per core
if os.environ.get("PYTEST_XDIST_WORKER_COUNT"):
    torch.set_num_threads(max(1, (os.cpu_count() or 1) // int(os.environ["PYTEST_XDIST_WORKER_COUNT"])))

VOCAB = 300          # ids drawn by the tests stay below this


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device and the built extension")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    no_gpu = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(no_gpu)


def _jitter(model):
    """Move every 1-D gain / bias off its initial constant so that norms and biases are exercised (the GDN decay
    parameters keep their initialisation)."""
    keep = ("A_log", "dt_bias")
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.ndim == 1 and not any(k in name for k in keep):
                p.add_(torch.randn_like(p), alpha=0.1)


def _hybrid_layout():
    # two blocks of three Gated DeltaNet layers and one gated full-attention layer
    kinds = []
    for _ in range(2):
        kinds += ["linear_attention", "linear_attention", "linear_attention", "full_attention"]
    return dict(vocab_size=VOCAB, hidden_size=80, num_hidden_layers=len(kinds), layer_types=kinds,
                num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=16, linear_value_head_dim=16,
                linear_conv_kernel_dim=4, rms_norm_eps=1e-6, max_position_embeddings=4096,
                tie_word_embeddings=False,
                rope_parameters={"rope_type": "default", "rope_theta": 10000000, "partial_rotary_factor": 0.25,
                                 "mrope_interleaved": True, "mrope_section": [2, 1, 1]})


def _build(family):
    import transformers as T
    if family == "llama":
        rope = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                "original_max_position_embeddings": 64}
        cfg = T.LlamaConfig(vocab_size=VOCAB, hidden_size=80, intermediate_size=176, num_hidden_layers=6,
                            num_attention_heads=4, num_key_value_heads=2, head_dim=16, rms_norm_eps=1e-5,
                            rope_theta=500000.0, rope_scaling=rope, max_position_embeddings=4096,
                            tie_word_embeddings=False)
        return T.LlamaForCausalLM(cfg)
    if family == "qwen3":
        cfg = T.Qwen3Config(vocab_size=VOCAB, hidden_size=80, intermediate_size=176, num_hidden_layers=4,
                            num_attention_heads=4, num_key_value_heads=2, head_dim=16, rms_norm_eps=1e-6,
                            rope_theta=1000000.0, max_position_embeddings=4096, tie_word_embeddings=False)
        return T.Qwen3ForCausalLM(cfg)
    if family == "qwen35":
        return T.Qwen3_5ForCausalLM(T.Qwen3_5TextConfig(intermediate_size=176, **_hybrid_layout()))
    if family == "qwen35_moe":
        cfg = T.Qwen3_5MoeTextConfig(num_experts=8, num_experts_per_tok=3, moe_intermediate_size=40,
                                     shared_expert_intermediate_size=56, **_hybrid_layout())
        return T.Qwen3_5MoeForCausalLM(cfg)
    raise KeyError(family)


def _checkpoint(tmp_path_factory, family):
    torch.manual_seed(0)
    model = _build(family).float().eval()
    _jitter(model)
    if family == "qwen35_moe":
        with torch.no_grad():            # router and experts far enough from zero that routing is not a tie
            for name, p in model.named_parameters():
                if "experts" in name or "mlp.gate" in name:
                    p.normal_(0, 0.1)
    out = tmp_path_factory.mktemp(family)
    model.save_pretrained(str(out), safe_serialization=True)
    return out, model


@pytest.fixture(scope="session")
def tiny_llama(tmp_path_factory):
    return _checkpoint(tmp_path_factory, "llama")


@pytest.fixture(scope="session")
def tiny_qwen3(tmp_path_factory):
    return _checkpoint(tmp_path_factory, "qwen3")


@pytest.fixture(scope="session")
def tiny_qwen35(tmp_path_factory):
    return _checkpoint(tmp_path_factory, "qwen35")


@pytest.fixture(scope="session")
def tiny_qwen35_moe(tmp_path_factory):
    return _checkpoint(tmp_path_factory, "qwen35_moe")
