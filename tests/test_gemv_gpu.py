"""The small-batch projection kernels against a plain torch fp32 reference of
the same ops: fp16(rmsnorm(x) * (1 + w)) . W^T (W fp16) rounded to bf16, and
x0 + bf16(a . W^T) (a, W bf16).  The GEMV accumulates in fp32 in its own
order, so the bf16 results may differ from the reference by one bf16 rounding
(2^-8 relative) on isolated elements; relative RMS stays far below 1e-3."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import attention_oracle as O
from ria_b200 import _ext

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch", [1, 3, 8])
@pytest.mark.parametrize("n,k", [(12352, 2048), (9216, 2048), (100, 2048)])
def test_rmsnorm_gemv(cuda_device, batch, n, k):
    g = torch.Generator(device=cuda_device).manual_seed(n + batch)
    x = torch.randn(batch, k, device=cuda_device, generator=g) * 3
    nw = 0.1 * torch.randn(k, device=cuda_device, generator=g)
    w = (0.02 * torch.randn(n, k, device=cuda_device, generator=g)).to(torch.float16)
    out = torch.empty(batch, n, dtype=torch.bfloat16, device=cuda_device)
    _ext.rmsnorm_gemv(x, nw, w, out)
    h = torch.empty(batch, k, dtype=torch.float16, device=cuda_device)
    _ext.rmsnorm_rows(x, nw, h)  # the unfused norm kernel: the same fp16 activations
    ref_h = (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + nw)).to(torch.float16)
    assert O.max_abs(h.float(), ref_h.float()) <= 2 ** -10 * ref_h.float().abs().max().item()
    ref = F.linear(h.float(), w.float()).to(torch.bfloat16)
    assert O.rel_rms(out.float(), ref.float()) < 1e-3
    assert O.max_err_bf16(out.float(), ref.float()) < 1e-2


@pytest.mark.parametrize("batch", [1, 2, 8])
@pytest.mark.parametrize("n,k", [(2048, 4096), (48, 4096)])
def test_gemv_residual(cuda_device, batch, n, k):
    g = torch.Generator(device=cuda_device).manual_seed(n * 3 + batch)
    wide = torch.randn(batch, k + 64, device=cuda_device, generator=g).to(torch.bfloat16)
    a = wide[:, 8:8 + k]  # strided rows, 16-byte aligned
    x0 = torch.randn(batch, n, device=cuda_device, generator=g)
    w = (0.02 * torch.randn(n, k, device=cuda_device, generator=g)).to(torch.bfloat16)
    out = torch.empty(batch, n, device=cuda_device)
    _ext.gemv_residual(a, w, x0, out)
    ref = x0 + F.linear(a.float(), w.float()).to(torch.bfloat16).float()
    assert O.rel_rms(out - x0, ref - x0) < 1e-3
    assert O.max_abs(out, ref) <= 2 ** -7 * (ref - x0).abs().max().item() + 1e-6


def test_gemv_rejects_large_batch(cuda_device):
    x = torch.randn(9, 2048, device=cuda_device)
    w = torch.zeros(64, 2048, dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError, match="batch"):
        _ext.rmsnorm_gemv(x, torch.zeros(2048, device=cuda_device), w,
                          torch.empty(9, 64, dtype=torch.bfloat16, device=cuda_device))


def test_rmsnorm_rows_bf16_and_fp16(cuda_device):
    """The norm kernel's two output types against torch in fp32."""
    g = torch.Generator(device=cuda_device).manual_seed(4)
    x = torch.randn(5, 2048, device=cuda_device, generator=g) * 2
    nw = 0.1 * torch.randn(2048, device=cuda_device, generator=g)
    ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + nw)
    for dt, ulp in ((torch.bfloat16, 2 ** -8), (torch.float16, 2 ** -11)):
        h = torch.empty(5, 2048, dtype=dt, device=cuda_device)
        _ext.rmsnorm_rows(x, nw, h)
        assert ((h.float() - ref).abs() <= ulp * ref.abs() + 1e-6).all()
