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
    gib = 2 ** 30
    total = p.total_memory
    cap = float(env.get("RF_VRAM_CAP_GIB", 0)) * gib or total
    torch.cuda.set_device(dev_index)
    torch.cuda.set_per_process_memory_fraction(min(1.0, cap / total), dev_index)
    info = {"deterministic": deterministic, "vendor": "nvidia", "name": p.name,
            "arch": f"sm_{p.major}{p.minor}", "sms": p.multi_processor_count}
    info.update(total_gib=round(total / gib, 2), cap_gib=cap / gib, runtime="cuda " + str(torch.version.cuda),
                local_rank=local, world=world)
    return torch.device("cuda", dev_index), info


def _gib(device, counter):
    if device.type != "cuda":
        return 0.0
    return counter(device) / 2 ** 30


def peak_gib(device):
    import torch
    return _gib(device, torch.cuda.max_memory_allocated)


def used_gib(device):
    import torch
    return _gib(device, torch.cuda.memory_allocated)
