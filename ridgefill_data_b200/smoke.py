"""One tiny forward of the flagship hybrid on cuda:0 through the sm_100a kernels: a RidgeFill prefill
(exact lower layers, ridge-map fill of the late layers, exact tail) plus one decode step."""
import torch


def run_smoke():
    from .engine.arm import Arm
    from .engine.prefill import finish, run_lower
    from .models.base import from_config
    from .models.config import ModelConfig, _hybrid_types
    from .ops._ext import check_errors
    from .ridge.projector import Projector

    cfg = ModelConfig(arch="qwen3_5", n_layers=8, hidden=512, vocab=1024, n_heads=4, n_kv=1, head_dim=256,
                      intermediate=1024, eps=1e-6, rope_theta=1e7, partial_rotary=0.25,
                      layer_types=_hybrid_types(8), gdn_nk=2, gdn_nv=4, gdn_dk=128, gdn_dv=128, conv_k=4,
                      name="smoke-hybrid")
    dev = torch.device("cuda", 0)
    model = from_config(cfg, seed=0, device=dev, backend="b200")
    split = 4
    W = {i: torch.eye(cfg.hidden, device=dev, dtype=torch.bfloat16) for i in range(split, cfg.n_layers)}
    B = {i: torch.zeros(cfg.hidden, device=dev, dtype=torch.bfloat16) for i in range(split, cfg.n_layers)}
    arm = Arm("ridgefill", split=split, tail=64, fill="proj", projector=Projector(split, W, B))
    ids = torch.randint(0, cfg.vocab, (256,), generator=torch.Generator().manual_seed(0)).to(dev)
    with torch.no_grad():
        hs, lower = run_lower(model, ids, [split])
        logits, cache, P = finish(model, ids, hs[split], lower, arm, keep=1)
        tok = logits[-1].argmax().view(1)
        h = model.embed(tok)
        pos = torch.tensor([ids.shape[0]], device=dev)
        for i in range(cfg.n_layers):
            h = model.layer(i, h, pos, cache)
        nxt = model.logits(h)
    torch.cuda.synchronize()
    check_errors(dev)
    assert torch.isfinite(logits).all() and torch.isfinite(nxt).all() and P == 192
    print(f"smoke ok: prefix {P} rows filled, first token {int(tok)}, next logits {tuple(nxt.shape)}")


if __name__ == "__main__":
    run_smoke()
