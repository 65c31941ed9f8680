"""Loads the in-tree sm_100a extension (ridgefill_data_b200/_C*.so, built by `python setup.py
build_ext --inplace` or __graft_entry__.build()).

There is no fallback: on a machine with a CUDA device, a missing or stale extension raises at
first use, so a GPU run can never silently take a slower PyTorch path."""
import importlib

_mod = None
_err = None


class ExtensionMissing(RuntimeError):
    pass


def ext():
    global _mod, _err
    if _mod is not None:
        return _mod
    import torch  # noqa: F401  (loads libc10 / libtorch, which the extension links against)
    try:
        _mod = importlib.import_module("ridgefill_data_b200._C")
    except ImportError as e:  # pragma: no cover - depends on the build
        _err = e
        raise ExtensionMissing(
            "the sm_100a extension ridgefill_data_b200._C is not built; run `python setup.py build_ext --inplace`"
        ) from e
    return _mod


def available():
    try:
        ext()
        return True
    except ExtensionMissing:
        return False


ERROR_CODES = {1: "TMA producer wait timed out", 2: "MMA issuer wait timed out", 3: "epilogue wait timed out",
               4: "peer flag wait timed out (a rank did not arrive)", 5: "drain wait timed out",
               6: "unsupported shape", 7: "gather index outside its table"}


def check_errors(device=None):
    """Raise if any kernel recorded an error (a bounded wait that timed out, a bad shape or index) in the device
    error word; clears it."""
    import torch
    dev = torch.cuda.current_device() if device is None else torch.device(device).index or 0
    w = ext().error_word(dev)
    code = int(w.item())
    if code:
        w.zero_()
        raise RuntimeError(f"sm_100a kernel reported error code {code}: {ERROR_CODES.get(code, 'unknown')}")
