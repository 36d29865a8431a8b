"""The built extension loads with every symbol resolved (no GPU needed)."""

import glob
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_extension_loads_if_built():
    built = glob.glob(os.path.join(ROOT, "zeroq_b200", "_C*.so"))
    if not built:
        pytest.skip("extension not built in-tree")
    from zeroq_b200.ops import _ext

    assert _ext.available(), f"extension failed to load: {_ext._EXT_ERR!r}"
    for name in ("gemm_bf16_tn", "gemm_bf16_nn", "add_rmsnorm_fwd", "rmsnorm_bwd", "attn_fwd_tc",
                 "nf4_quantize", "rs_adamw", "plan_gather_dequant"):
        assert hasattr(_ext.ext(), name), name
