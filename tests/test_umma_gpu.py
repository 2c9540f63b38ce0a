"""tcgen05 operand layouts: every (A major or A in TMEM, B major, N, K)
combination the prefill kernels use, in bf16 and fp16, against a float64 matmul of the same rounded
operands (fp32 accumulation: relative error ~1e-6)."""

from __future__ import annotations

import itertools

import pytest
import torch

from ria_b200 import _ext

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("a_mn,b_mn,n,k", list(itertools.product([0, 1, 2], [False, True], [64, 128], [64, 128])))
@pytest.mark.parametrize("f16", [False, True])
def test_umma_layouts(cuda_device, a_mn, b_mn, n, k, f16):
    """fp16 operands (the chunked prefill's internal type) use the same
    layouts with the descriptor's format fields set to F16."""
    g = torch.Generator().manual_seed(n * 7 + k + 100 * a_mn + 10 * b_mn)
    a = torch.randn(128, k, generator=g)
    b = torch.randn(k, n, generator=g)
    d = _ext.umma_selftest(a.to(cuda_device), b.to(cuda_device), a_mn, b_mn, f16=f16).cpu()
    t = torch.float16 if f16 else torch.bfloat16
    ref = a.to(t).double() @ b.to(t).double()
    err = (d.double() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, err
    assert _ext.device_error() == 0
