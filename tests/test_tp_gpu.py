"""Tensor parallelism on 2 GPUs (spawned NCCL ranks): the sharded B200 model reproduces the unsharded one's
logits for exact forward and RidgeFill prefill (map fill by column slices, or by row blocks and an
all-to-all). Skipped with fewer than 2 visible GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, q, fill="columns"):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from ridgefill_data_b200.engine.arm import Arm
        from ridgefill_data_b200.engine.prefill import finish, run_lower
        from ridgefill_data_b200.models.base import from_config
        from ridgefill_data_b200.parallel.tp import TensorParallel, shard
        from ridgefill_data_b200.ridge.projector import Projector
        from test_b200_model_gpu import HYB, MOE, QWEN3
        out = {}
        for cfg in (HYB, QWEN3, MOE):
            dev = torch.device("cuda", rank)
            m = from_config(cfg, seed=0, device=dev, std=0.05, backend="b200")
            ids = torch.randint(0, cfg.vocab, (300,), generator=torch.Generator().manual_seed(1)).to(dev)
            keep = torch.arange(290, 300, device=dev)
            split = cfg.n_layers // 2
            W = {i: torch.eye(cfg.hidden, device=dev, dtype=torch.bfloat16) for i in range(split, cfg.n_layers)}
            B = {i: torch.zeros(cfg.hidden, device=dev, dtype=torch.bfloat16) for i in range(split, cfg.n_layers)}
            arm = Arm("rf", split=split, tail=64, fill="proj", projector=Projector(split, W, B))
            with torch.no_grad():
                f32 = from_config(cfg, seed=0, device=dev, std=0.05, dtype=torch.float32)
                ref32, _ = f32.forward_exact(ids, keep=keep)
                hs32, lower32 = run_lower(f32, ids, [split])
                arm32 = Arm("rf", split=split, tail=64, fill="proj", projector=Projector(
                    split, {i: t.float() for i, t in W.items()}, {i: t.float() for i, t in B.items()}))
                rf32, _, _ = finish(f32, ids, hs32[split], lower32, arm32, 4)
                del f32, hs32, lower32
                ref, _ = m.forward_exact(ids, keep=keep)
                hs, lower = run_lower(m, ids, [split])
                ref_rf, _, _ = finish(m, ids, hs[split], lower, arm, 4)
                if mode == "nvls+overlap":     # row chunks of 128: GEMM of one beside the all-reduce of another
                    tp = TensorParallel(mode="nvls", fill=fill, overlap=4, overlap_min_rows=64)
                else:
                    tp = TensorParallel(mode=mode, fill=fill)
                shard(m, tp)
                got, _ = m.forward_exact(ids, keep=keep)
                hs, lower = run_lower(m, ids, [split])
                got_rf, _, _ = finish(m, ids, hs[split], lower, arm, 4)
                torch.cuda.synchronize()
                from ridgefill_data_b200.ops._ext import check_errors
                check_errors(dev)
                tp.close()
            rel = lambda a, b: float((a - b).norm() / b.norm())  # noqa: E731
            out[cfg.name] = (rel(got, ref32), rel(ref, ref32), rel(got_rf, rf32), rel(ref_rf, rf32))
        q.put((rank, out))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode,fill", [("nccl", "columns"), ("fused", "columns"), ("nvls", "columns"),
                                       ("nvls+overlap", "columns"), ("nccl", "rows")])
def test_tp2_matches_single_gpu(mode, fill):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q, fill)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, out in res.items():
        assert isinstance(out, dict), out
        for name, (e_tp, e_single, e_rf, e_rf_single) in out.items():
            # the sharded run is no further from fp32 than the unsharded bf16 run (plus a margin), for the exact
            # forward and for the RidgeFill prefill
            assert e_tp < 1.5 * e_single + 5e-3, (r, name, e_tp, e_single)
            assert e_rf < 1.5 * e_rf_single + 5e-3, (r, name, e_rf, e_rf_single)


def _fit_worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from ridgefill_data_b200.eval.data import zipf_docs
        from ridgefill_data_b200.models.base import from_config
        from ridgefill_data_b200.ridge import sweep
        from test_b200_model_gpu import HYB
        m = from_config(HYB, seed=0, device=torch.device("cuda", rank), std=0.05, backend="b200")
        docs = zipf_docs(6, 256, HYB.vocab, seed=1)
        dp = sweep.fit(m, docs, [4], lambdas=(0.03,), log=None, group=dist.group.WORLD)
        single = sweep.fit(m, docs, [4], lambdas=(0.03,), log=None)
        errs = []
        for i in range(4, HYB.n_layers):
            a, b = dp[4]["maps"][0.03][i][0], single[4]["maps"][0.03][i][0]
            errs.append(float((a.cpu() - b.cpu()).norm() / b.cpu().norm()))
        q.put((rank, max(errs)))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_data_parallel_fit_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fit_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, err in res.items():
        assert isinstance(err, float) and err < 1e-3, (r, err)


def _f64_worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from ridgefill_data_b200.parallel.nvls import NvlsF64Reducer, NvlsUnavailable
        try:
            red = NvlsF64Reducer(chunk=1000)          # small chunks: several per tensor, a ragged last one
        except NvlsUnavailable as e:
            q.put((rank, f"skip: {e}"))
            return
        dev = torch.device("cuda", rank)
        mine = [torch.randn(2500, generator=torch.Generator().manual_seed(10 * rank + j), dtype=torch.float64)
                .to(dev).view(50, 50) for j in range(2)] + [torch.full((3,), float(rank + 1), dtype=torch.float64,
                                                                       device=dev)]
        want = [sum(torch.randn(2500, generator=torch.Generator().manual_seed(10 * r + j), dtype=torch.float64)
                    for r in range(world)).view(50, 50) for j in range(2)]
        want.append(torch.full((3,), float(sum(range(1, world + 1))), dtype=torch.float64))
        red.allreduce_(mine)
        torch.cuda.synchronize()
        from ridgefill_data_b200.ops._ext import check_errors
        check_errors(dev)
        red.close()
        q.put((rank, all(torch.equal(a.cpu(), b) for a, b in zip(mine, want))))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_nvls_fp64_allreduce_is_exact():
    """The fit's fp64 sums reduced in the NVSwitch (two ranks: one exact fp64 add per element) equal the host sum
    bitwise, across chunk boundaries."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_f64_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    if any(isinstance(v, str) and v.startswith("skip") for v in res.values()):
        pytest.skip(str(res))
    assert all(v is True for v in res.values()), res
