"""Device guard (code/kva/gpu.py:38-104): one named B200 per process unless a multi-GPU launcher
owns the process group, deterministic library settings, an optional memory cap, and a CPU dry-run.

Environment:
  RF_CPU_DRYRUN=1     everything on the CPU (tiny models, tests)
  RF_GPU_NAME         substring the visible device's name must contain (default "B200")
  RF_VRAM_CAP_GIB     cap the caching allocator
  RF_DETERMINISTIC    1 (default): torch deterministic algorithms (warn only), TF32 off
setup() refuses by message (SystemExit) before any allocation when the device does not match.
Under torchrun (WORLD_SIZE > 1) each process takes cuda:LOCAL_RANK and the one-device check applies
to the device count being at least the local world size.
"""
from __future__ import annotations

import os


def setup(env=None, torch=None):
    env = os.environ if env is None else env
    if torch is None:
        import torch
    if env.get("RF_CPU_DRYRUN") == "1":
        return torch.device("cpu"), dict(cpu_dryrun=True)
    if getattr(torch.version, "hip", None):
        raise SystemExit(f"refusing: this torch is a ROCm build (hip {torch.version.hip}); sm_100a needs CUDA")
    if not torch.version.cuda:
        raise SystemExit("refusing: this torch has no CUDA (a CPU-only build); set RF_CPU_DRYRUN=1 for the CPU")
    world = int(env.get("WORLD_SIZE", "1"))
    local = int(env.get("LOCAL_RANK", "0"))
    n = torch.cuda.device_count()
    if world == 1 and n < 1:
        raise SystemExit("refusing: no visible CUDA device")
    if world > 1 and n < min(world, 8) and n != 1:
        raise SystemExit(f"refusing: {n} visible devices for {world} local ranks")
    dev_index = local if n > 1 else 0
    p = torch.cuda.get_device_properties(dev_index)
    want = env.get("RF_GPU_NAME", "B200").strip()
    if want and want.lower() not in p.name.lower():
        raise SystemExit(f"refusing: device {dev_index} is {p.name!r}, not a {want!r} (RF_GPU_NAME)")
    if (p.major, p.minor) != (10, 0):
        raise SystemExit(f"refusing: device {dev_index} is sm_{p.major}{p.minor}; the kernels are built for sm_100a")
    deterministic = env.get("RF_DETERMINISTIC", "1") == "1"
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    if deterministic:
        torch.use_deterministic_algorithms(True, warn_only=True)
    cap = float(env.get("RF_VRAM_CAP_GIB", 0)) * 2**30 or p.total_memory
    torch.cuda.set_device(dev_index)
    torch.cuda.set_per_process_memory_fraction(min(1.0, cap / p.total_memory), dev_index)
    return torch.device(f"cuda:{dev_index}"), dict(
        deterministic=deterministic, vendor="nvidia", name=p.name, arch=f"sm_{p.major}{p.minor}",
        sms=p.multi_processor_count, total_gib=round(p.total_memory / 2**30, 2), cap_gib=cap / 2**30,
        runtime=f"cuda {torch.version.cuda}", local_rank=local, world=world)


def peak_gib(device):
    import torch
    return torch.cuda.max_memory_allocated(device) / 2**30 if device.type == "cuda" else 0.0


def used_gib(device):
    import torch
    return torch.cuda.memory_allocated(device) / 2**30 if device.type == "cuda" else 0.0
