"""Loads the in-tree sm_100a extension (ridgefill_data_b200/_C*.so, built by `python setup.py
build_ext --inplace` or __graft_entry__.build()).

There is no fallback: on a machine with a CUDA device, a missing or stale extension raises at
first use, so a GPU run can never silently take a slower PyTorch path."""
import importlib

_mod = None
_err = None


class ExtensionMissing(RuntimeError):
    pass


class KernelError(RuntimeError):
    def __init__(self, op, code):
        super().__init__(f"{op}: sm_100a kernel reported error code {code}: {ERROR_CODES.get(code, 'unknown')}")
        self.op, self.code = op, code


class Checked:
    """Debug proxy over the extension (RF_CHECK_EACH=1 in the environment): after every call it synchronizes the
    device and reads the error word, so the first op whose kernel recorded an error (a timed-out bounded wait, a bad
    shape or index) is named in the exception instead of surfacing at a later check. Slow: for debugging only."""

    PASS = frozenset(("error_word", "launch_count"))

    def __init__(self, mod, sync=None, device=None):
        self._mod = mod
        self._sync = sync
        self._device = device

    def __getattr__(self, name):
        f = getattr(self._mod, name)
        if not callable(f) or name in self.PASS:
            return f

        def call(*a, **k):
            import torch
            out = f(*a, **k)
            (self._sync or torch.cuda.synchronize)()
            dev = self._device() if self._device else torch.cuda.current_device()
            w = self._mod.error_word(dev)
            code = int(w.item())
            if code:
                w.zero_()
                raise KernelError(name, code)
            return out
        call.__name__ = name
        return call


def ext():
    global _mod, _err
    if _mod is not None:
        return _mod
    import os

    import torch  # noqa: F401  (loads libc10 / libtorch, which the extension links against)
    try:
        mod = importlib.import_module("ridgefill_data_b200._C")
    except ImportError as e:  # pragma: no cover - depends on the build
        _err = e
        raise ExtensionMissing(
            "the sm_100a extension ridgefill_data_b200._C is not built; run `python setup.py build_ext --inplace`"
        ) from e
    _mod = Checked(mod) if os.environ.get("RF_CHECK_EACH") == "1" else mod
    if os.environ.get("RF_GEMM_2SM") == "0":     # A/B switch: every product on the one-SM GEMM kernel
        mod.set_gemm_2sm(False)
    if os.environ.get("RF_GEMV") == "0":         # A/B switch: 1-16 row products on the tile GEMMs instead of GEMVs
        mod.set_gemv(False)
    if os.environ.get("RF_GEMV_MMA") == "0":     # A/B switch: the CUDA-core GEMV for 1-2 rows, tile GEMMs above
        mod.set_gemv_mma(False)
        mod.set_gemv_max_rows(2)
    if os.environ.get("RF_GDN_TC") == "1":       # A/B switch: output-mode GDN state pass on tcgen05 (state in TMEM)
        mod.set_gdn_state_tc(1)
    if os.environ.get("RF_GDN_FUSED") == "0":    # A/B switch: GDN output in a separate pass after the state pass
        mod.set_gdn_fused_output(0)
    if os.environ.get("RF_ATTN_SWG") == "2":     # A/B switch: two softmax warpgroups in the tcgen05 attention
        mod.set_attn_softmax_groups(2)
    if os.environ.get("RF_ATTN_QT") == "1":      # A/B switch: Q read from TMEM by the S product
        mod.set_attn_q_tmem(1)
    if os.environ.get("RF_ATTN_ROT") == "1":     # A/B switch: per-CTA rotation of the key-tile order
        mod.set_attn_rotate(1)
    if os.environ.get("RF_ATTN_SBUF") in ("2", "3"):   # A/B switch: TMEM S buffers (default per head dim)
        mod.set_attn_s_buffers(int(os.environ["RF_ATTN_SBUF"]))
    if os.environ.get("RF_ATTN_PBUF") == "1":    # A/B switch: one P buffer in the tcgen05 attention
        mod.set_attn_p_buffers(1)
    if os.environ.get("RF_ATTN_POLY") in ("2", "4"):   # A/B switch: softmax exponentials partly on the FMA pipe
        mod.set_attn_poly(int(os.environ["RF_ATTN_POLY"]))
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
    dev = torch.device(device).index if device is not None else None
    if dev is None:                      # None or a bare "cuda": the current device
        dev = torch.cuda.current_device()
    w = ext().error_word(dev)
    code = int(w.item())
    if code:
        w.zero_()
        raise KernelError("check_errors", code)
