"""The built extension loads (every symbol resolves) on a machine without a GPU, as the build check does."""
import glob
import os

import pytest


def test_extension_imports_when_built():
    here = os.path.join(os.path.dirname(__file__), "..", "ridgefill_data_b200")
    if not glob.glob(os.path.join(here, "_C*.so")):
        pytest.skip("extension not built")
    import torch  # noqa: F401  (the extension links against libtorch)
    from ridgefill_data_b200.ops._ext import ext
    m = ext()
    for name in ("gemm", "flash_attention", "gdn_chunk_scan", "nvls_allreduce", "gemm_nvls_ar", "gemm_nvls_ag", "score_rows",
                 "window_mass", "row_cosine", "embed_gather", "cholesky_solve", "grouped_gemm"):
        assert hasattr(m, name), name


def test_checked_proxy_names_the_failing_op():
    """The RF_CHECK_EACH debug proxy: passes results through, and raises naming the op whose kernel set the error
    word (here a fake extension and a fake device sync on the CPU)."""
    import torch
    from ridgefill_data_b200.ops._ext import Checked, KernelError

    class Fake:
        def __init__(self):
            self.word = torch.zeros((), dtype=torch.int32)

        def error_word(self, dev):
            return self.word

        def good(self, x):
            return x + 1

        def bad(self):
            self.word.fill_(4)

        launch_count = staticmethod(lambda: 7)

    f = Fake()
    c = Checked(f, sync=lambda: None, device=lambda: 0)
    assert c.good(1) == 2 and c.launch_count() == 7
    with pytest.raises(KernelError, match="bad: .*code 4: peer flag wait timed out"):
        c.bad()
    assert int(f.word) == 0 and c.good(2) == 3          # the word is cleared after the report
