"""Helpers shared by the -m gpu parity tests."""
from __future__ import annotations

import torch

# Parity bars: FP32 within 1e-5 relative (with a 1e-6 absolute floor for
# values that cancel to ~0); FP16 within 2e-3 absolute.
FP32_RTOL, FP32_ATOL = 1e-5, 1e-6
FP16_ATOL = 2e-3


def assert_parity(actual: torch.Tensor, expected: torch.Tensor, what: str = "") -> None:
    actual = actual.detach().cpu()
    expected = expected.detach().cpu()
    assert actual.dtype == expected.dtype, (actual.dtype, expected.dtype)
    if actual.dtype == torch.float32:
        torch.testing.assert_close(actual, expected, rtol=FP32_RTOL, atol=FP32_ATOL, msg=what or None)
    else:
        err = (actual.float() - expected.float()).abs()
        assert torch.isfinite(actual.float()).all(), what
        assert err.max().item() <= FP16_ATOL, f"{what}: max abs err {err.max().item():.3e}"


def subset_pool(tables, lengths, pools, block_size):
    """The used pages of some sequences, copied to the CPU with renumbered tables."""
    from conftest import import_module
    return import_module("workloads").compact_pages(tables, lengths, pools, block_size)
