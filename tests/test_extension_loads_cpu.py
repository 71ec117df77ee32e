"""The built extension loads on a host without a GPU driver (the driver library must not be
a link dependency: build hosts and CPU test runs have none), and exposes its entry points."""
import glob
import os

import pytest

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_extension_imports_without_driver():
    if not glob.glob(os.path.join(HERE, "sigma0_b200", "_C*.so")):
        pytest.skip("extension not built")
    import torch  # noqa: F401
    from sigma0_b200 import _C
    for name in ("m3_fwd", "m3_bwd", "tp_gemm_allreduce", "attn_fwd", "attn_bwd", "gdn_scan_fwd", "s5_scan_fwd",
                 "kda_intra_fwd"):
        assert hasattr(_C, name), name
