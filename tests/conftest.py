import os

import pytest
import torch

os.environ.setdefault("HF_HUB_OFFLINE", "1")
os.environ.setdefault("HF_HUB_DISABLE_IMPLICIT_TOKEN", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device and the built extension")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def _perturb_norms(m):
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() == 1 and "A_log" not in n and "dt_bias" not in n:
                p.add_(0.1 * torch.randn_like(p))


@pytest.fixture(scope="session")
def tiny_llama(tmp_path_factory):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=300, hidden_size=64, intermediate_size=160, num_hidden_layers=6,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=16, rms_norm_eps=1e-5,
                      rope_theta=500000.0, max_position_embeddings=4096, tie_word_embeddings=False,
                      rope_scaling=dict(rope_type="llama3", factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                                        original_max_position_embeddings=64))
    m = LlamaForCausalLM(cfg).float().eval()
    _perturb_norms(m)
    path = tmp_path_factory.mktemp("llama")
    m.save_pretrained(str(path), safe_serialization=True)
    return path, m


@pytest.fixture(scope="session")
def tiny_qwen3(tmp_path_factory):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=300, hidden_size=64, intermediate_size=160, num_hidden_layers=4,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=16, rms_norm_eps=1e-6,
                      rope_theta=1000000.0, max_position_embeddings=4096, tie_word_embeddings=False)
    m = Qwen3ForCausalLM(cfg).float().eval()
    _perturb_norms(m)
    path = tmp_path_factory.mktemp("qwen3")
    m.save_pretrained(str(path), safe_serialization=True)
    return path, m


def _qwen35_kw():
    types = (["linear_attention"] * 3 + ["full_attention"]) * 2
    return dict(vocab_size=300, hidden_size=64, num_hidden_layers=8, num_attention_heads=4, num_key_value_heads=2,
                head_dim=32, layer_types=types, linear_num_key_heads=2, linear_num_value_heads=4,
                linear_key_head_dim=16, linear_value_head_dim=16, linear_conv_kernel_dim=4, rms_norm_eps=1e-6,
                max_position_embeddings=4096, tie_word_embeddings=False,
                rope_parameters=dict(rope_type="default", rope_theta=10000000, partial_rotary_factor=0.25,
                                     mrope_interleaved=True, mrope_section=[2, 1, 1]))


@pytest.fixture(scope="session")
def tiny_qwen35(tmp_path_factory):
    from transformers import Qwen3_5ForCausalLM, Qwen3_5TextConfig
    torch.manual_seed(0)
    m = Qwen3_5ForCausalLM(Qwen3_5TextConfig(intermediate_size=160, **_qwen35_kw())).float().eval()
    _perturb_norms(m)
    path = tmp_path_factory.mktemp("qwen35")
    m.save_pretrained(str(path), safe_serialization=True)
    return path, m


@pytest.fixture(scope="session")
def tiny_qwen35_moe(tmp_path_factory):
    from transformers import Qwen3_5MoeForCausalLM, Qwen3_5MoeTextConfig
    torch.manual_seed(0)
    cfg = Qwen3_5MoeTextConfig(num_experts=8, num_experts_per_tok=3, moe_intermediate_size=32,
                               shared_expert_intermediate_size=48, **_qwen35_kw())
    m = Qwen3_5MoeForCausalLM(cfg).float().eval()
    _perturb_norms(m)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if "experts" in n or "mlp.gate" in n:
                p.normal_(0, 0.1)
    path = tmp_path_factory.mktemp("qwen35moe")
    m.save_pretrained(str(path), safe_serialization=True)
    return path, m
