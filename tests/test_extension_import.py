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
