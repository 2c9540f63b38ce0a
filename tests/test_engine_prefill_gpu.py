"""Prompt prefill through the batched engine (K2 + K4 + conv/gates/norm row
kernels) equals the token-by-token decode path it replaces (router-ia's prompt
loop), starting from the same non-trivial state: outputs of every prompt token
and the final DeltaNet, conv and KV state.

The two paths differ only in the form of the recurrence (chunked bf16-operand
WY/UT vs exact per-token fp32) and in the bf16 rounding points, so the bound
is the chained-layer one: max-abs 6e-2 and relative RMS 1e-2 on the residual
stream after the 4-layer stack, 2e-2 relative RMS on the final fp32 state,
1e-2 relative RMS on the bf16 conv state and K/V rows."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from ria_b200 import constants as C
from ria_b200.engine import BatchedAttentionState
from ria_b200.weights import DeltaNetWeights, GqaWeights

pytestmark = pytest.mark.gpu


def _engines(dev, lengths):
    layers = [0, 1, 2, 3]
    w = {l: (GqaWeights if C.is_full_attention_layer(l) else DeltaNetWeights).from_tensors(
        synthetic.layer_weights(l, 4), dev) for l in layers}
    B = len(lengths)
    engines = [BatchedAttentionState(w, batch=B, pool_blocks=64, max_blocks_per_seq=16, device=dev) for _ in range(2)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    a, b = engines
    for l in a.rec:
        a.rec[l].normal_(0, 0.1, generator=gen)
        a.conv[l].normal_(0, 0.1, generator=gen)
        b.rec[l].copy_(a.rec[l])
        b.conv[l].copy_(a.conv[l])
    for i, n in enumerate(lengths):
        for e in engines:
            e.set_length(i, n, position=n + 3)
    for e in engines:
        e.sync_tables()
    for l in a.k_pool:
        for i, n in enumerate(lengths):
            rows = a.physical_rows(i, n).to(dev)
            kk = torch.randn(2, n, 256, device=dev, generator=gen).to(torch.bfloat16)
            vv = torch.randn(2, n, 256, device=dev, generator=gen).to(torch.bfloat16)
            for e in engines:
                e.k_pool[l][:, rows] = kk
                e.v_pool[l][:, rows] = vv
    return a, b


@pytest.mark.parametrize("T", [1, 70, 200])
def test_prefill_equals_token_by_token(cuda_device, T):
    lengths = [0, 65, 130]
    a, b = _engines(cuda_device, lengths)
    x = synthetic.hidden_stream(T, 11, rows=len(lengths)).transpose(0, 1).contiguous().to(cuda_device)  # [B, T, 2048]
    got = a.prefill(x)
    ref = torch.stack([b.step(x[:, t].contiguous()) for t in range(T)], dim=1)
    assert _ext.device_error() == 0
    err = (O.max_abs(got, ref), O.rel_rms(got, ref))
    print(f"T={T}: out max_abs={err[0]:.2e} rel_rms={err[1]:.2e}")
    assert err[0] < 6e-2 and err[1] < 1e-2, err
    for l in a.rec:
        e_s = O.rel_rms(a.rec[l], b.rec[l])
        assert e_s < 2e-2, (l, e_s)
        # conv state holds bf16 projections of the layer input, which already
        # differs by the chained-layer error above: bf16-ulp agreement
        assert O.rel_rms(a.conv[l].float(), b.conv[l].float()) < 1e-2, l
    assert a.lengths == b.lengths and a.positions_host == b.positions_host
    for l in a.k_pool:
        for i, n in enumerate(a.lengths):
            # the two engines allocate pages in a different order
            ra, rb = a.physical_rows(i, n).to(cuda_device), b.physical_rows(i, n).to(cuda_device)
            e_k = O.rel_rms(a.k_pool[l][:, ra].float(), b.k_pool[l][:, rb].float())
            e_v = O.rel_rms(a.v_pool[l][:, ra].float(), b.v_pool[l][:, rb].float())
            print(f"  layer {l} seq {i}: K rel_rms={e_k:.2e} V rel_rms={e_v:.2e}")
            assert e_k < 1e-2 and e_v < 1e-2, (l, i, e_k, e_v)
