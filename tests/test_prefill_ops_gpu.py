"""The prefill row kernels against the oracle's one-token arithmetic:
ria_conv1d_prefill == T conv steps (qwen36_attention_cache.py:176-221) from
the same rolling state, ria_gdn_gates == the gate lines (:242-250),
ria_gated_rmsnorm == gated_rmsnorm (qwen36_gated_norm_probe.py:19-36).

Outputs are bf16 like the reference's conv / norm outputs: within one bf16
rounding (2^-7 relative); the new conv state is the last four inputs, exact;
the fp32 gates within 1e-5 relative of torch's fp32 functions."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [1, 2, 5, 70, 300])
@pytest.mark.parametrize("offset", [16, 17])  # channel pairs aligned (pair kernel) or not (per-channel kernel)
def test_conv1d_prefill_equals_steps(cuda_device, T, offset):
    B, Cc = 2, 512
    g = torch.Generator().manual_seed(T)
    wide = torch.randn(B, T, Cc + 64, generator=g).to(torch.bfloat16)  # a strided view, like the projection
    x = wide[:, :, offset:offset + Cc]
    state0 = torch.randn(B, Cc, 4, generator=g).to(torch.bfloat16)
    weight = (torch.rand(Cc, 1, 4, generator=g) - 0.5).to(torch.bfloat16)
    xd, st = x.to(cuda_device), state0.to(cuda_device).contiguous()
    out = torch.empty(B, T, Cc, dtype=torch.bfloat16, device=cuda_device)
    _ext.conv1d_prefill(xd, st, weight.reshape(Cc, 4).to(cuda_device).contiguous(), out)
    assert _ext.device_error() == 0
    out, st = out.cpu(), st.cpu()
    for b in range(B):
        state = state0[b:b + 1]
        for t in range(T):
            ref, state = O.conv1d_step(state, x[b:b + 1, t], weight)
            got = out[b, t].float()
            err = ((got - ref[0].float()).abs() / ref[0].float().abs().clamp_min(1e-2)).max().item()
            assert err <= 2 ** -7, (b, t, err)
        assert torch.equal(st[b], state[0]), b


def test_conv1d_prefill_vector_form_equals_pair_form(cuda_device):
    """At sizes that fill the GPU, 16-byte aligned rows take the vector form
    (eight channels x sixteen tokens per thread); the same values in rows
    that are only 4-byte aligned take the pair form.  Same per-channel
    arithmetic and order: bit-identical outputs and states; sequence 0 is
    also checked against the oracle's steps."""
    dev = cuda_device
    B, T, Cc = 4, 1024, 8192
    g = torch.Generator(device=dev).manual_seed(99)
    vals = torch.randn(B, T, Cc, device=dev, generator=g).to(torch.bfloat16)
    wide_v = torch.zeros(B, T, Cc + 64, dtype=torch.bfloat16, device=dev)
    wide_p = torch.zeros_like(wide_v)
    wide_v[:, :, 16:16 + Cc] = vals  # 32-byte offset: the vector form
    wide_p[:, :, 18:18 + Cc] = vals  # 36-byte offset: the pair form
    state0 = (torch.randn(B, Cc, 4, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    weight = (torch.rand(Cc, 4, device=dev, generator=g) - 0.5).to(torch.bfloat16)
    outs, states = [], []
    for wide, off in ((wide_v, 16), (wide_p, 18)):
        st = state0.clone()
        out = torch.empty(B, T, Cc, dtype=torch.bfloat16, device=dev)
        _ext.conv1d_prefill(wide[:, :, off:off + Cc], st, weight, out)
        outs.append(out)
        states.append(st)
    torch.cuda.synchronize(dev)
    assert torch.equal(outs[0], outs[1]) and torch.equal(states[0], states[1])
    assert _ext.device_error() == 0
    x0 = vals[0].cpu()
    w3 = weight.cpu().reshape(Cc, 1, 4)
    got = outs[0][0].float().cpu()
    state = state0[0:1].cpu()  # every 37th token against the oracle's steps
    for t in range(T):
        ref, state = O.conv1d_step(state, x0[t:t + 1], w3)
        if t % 37 == 0 or t == T - 1:
            err = ((got[t] - ref[0].float()).abs() / ref[0].float().abs().clamp_min(1e-2)).max().item()
            assert err <= 2 ** -7, (t, err)
    assert torch.equal(states[0][0].cpu(), state[0])


def test_gdn_gates(cuda_device):
    rows, heads = 300, 32
    g = torch.Generator().manual_seed(3)
    proj = (torch.randn(rows, 100, generator=g) * 8).to(torch.bfloat16)  # a and b as strided columns
    a, b = proj[:, 0:heads], proj[:, 40:40 + heads]
    a_log = torch.rand(heads, generator=g) * 2.7
    dt_bias = torch.rand(heads, generator=g) * 30 - 10  # a + dt_bias crosses the softplus threshold (20)
    gg = torch.empty(rows, heads, device=cuda_device)
    bb = torch.empty(rows, heads, device=cuda_device)
    pd = proj.to(cuda_device)
    _ext.gdn_gates(pd[:, 0:heads], pd[:, 40:40 + heads], a_log.to(cuda_device), dt_bias.to(cuda_device), gg, bb)
    beta_ref, g_ref = O.deltanet_gates(a, b, a_log, dt_bias)
    assert torch.allclose(bb.cpu(), beta_ref, rtol=1e-5, atol=1e-7)
    assert torch.allclose(gg.cpu(), g_ref, rtol=1e-5, atol=1e-6)


def test_gated_rmsnorm(cuda_device):
    rows, heads = 77, 32
    g = torch.Generator().manual_seed(4)
    o = (torch.randn(rows, heads * 128 + 32, generator=g) * 3).to(torch.bfloat16)[:, :heads * 128]
    z = torch.randn(rows, heads * 128, generator=g).to(torch.bfloat16)
    w = 1 + 0.1 * torch.randn(128, generator=g)
    out = torch.empty(rows, heads * 128, dtype=torch.bfloat16, device=cuda_device)
    _ext.gated_rmsnorm(o.to(cuda_device), z.to(cuda_device), w.to(cuda_device), out)
    ref = O.gated_rmsnorm(o.reshape(rows, heads, 128), z.reshape(rows, heads, 128), w).reshape(rows, -1)
    assert O.max_err_bf16(out.cpu().float(), ref.float()) <= 2e-2
    assert O.rel_rms(out.cpu().float(), ref.float()) < 4e-3
