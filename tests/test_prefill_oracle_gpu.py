"""Prompt prefill, one layer at a time, against the oracle's token-by-token
layer steps (the reference's CPU path, qwen36_attention_cache.py:224-324),
teacher-forced: every layer sees the same input on both sides.

This is what router-ia's prompt loop computes (qwen36_chat_batch.py:255-258:
one ``run_forward_token`` per prompt token, each calling ``step_attention``
per layer); the batched engine replaces it with one call per layer over the
whole prompt -- K2 (chunked DeltaNet) and K4 (causal GQA prefill) plus the
conv / gate / norm kernels and the projections.

Bars, per layer: every prompt token's fp32 residual within 2e-2 max-abs and
its attention contribution (residual minus input) within 1e-2 relative RMS.
The state after the prompt: DeltaNet fp32 state within 1e-2 relative RMS
(at the layer boundary the state's inputs are the bf16 projection outputs,
which already differ from the fp32 projections of the CPU path by a bf16
rounding; the K2 kernel alone holds 1e-3 against the float64 recurrence, see
test_gdn_prefill_gpu.py), conv state and appended K/V within 1e-2 relative
RMS.  Prompts of 64 (configuration 0), 200 and 1000 tokens, from zero and
non-zero states, over ragged prefixes for the GQA layer."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from ria_b200.engine import BatchedAttentionState, deltanet_prefill
from ria_b200.weights import DeltaNetWeights, GqaWeights

pytestmark = pytest.mark.gpu

OUT_MAX, OUT_REL, STATE_REL = 2e-2, 1e-2, 1e-2
_PROJ = ("in_proj_qkv", "in_proj_z", "in_proj_a", "in_proj_b", "out_proj", "q_proj", "k_proj", "v_proj", "o_proj")


def _oracle_weights(wt: dict) -> dict:
    """Projection matrices converted to fp32 once (the oracle would convert
    them on every call, as the reference does); everything else unchanged."""
    return {k: (v.float() if any(p in k for p in _PROJ) else v) for k, v in wt.items()}


def _compare_tokens(got, x, refs, tag):
    worst = [0.0, 0.0]
    for t, ref in enumerate(refs):
        xin = x[t:t + 1]
        out = got[t:t + 1]
        err = (O.max_abs(out, ref), O.rel_rms(out - xin, ref - xin))
        worst = [max(worst[0], err[0]), max(worst[1], err[1])]
        assert err[0] < OUT_MAX and err[1] < OUT_REL, (tag, t, err)
    return worst


@pytest.mark.parametrize("T,B,with_state", [(64, 2, False), (200, 2, True), (1000, 1, True)])
def test_deltanet_prefill_matches_oracle(cuda_device, T, B, with_state):
    dev = cuda_device
    layer = 0
    wt = synthetic.layer_weights(layer, 21)
    w = DeltaNetWeights.from_tensors(wt, dev)
    ow = _oracle_weights(wt)
    gen = torch.Generator().manual_seed(T)
    if with_state:
        rec0 = torch.randn(B, 32, 128, 128, generator=gen) * 0.1
        conv0 = (torch.randn(B, 8192, 4, generator=gen) * 0.1).to(torch.bfloat16)
    else:
        rec0 = torch.zeros(B, 32, 128, 128)
        conv0 = torch.zeros(B, 8192, 4, dtype=torch.bfloat16)
    rec, conv = rec0.to(dev), conv0.to(dev)
    x = synthetic.hidden_stream(T, 31, rows=B).transpose(0, 1).contiguous()  # [B, T, 2048]
    got = deltanet_prefill(x.to(dev), w, rec, conv).cpu()
    torch.cuda.synchronize()
    assert _ext.device_error() == 0
    for b in range(B):
        conv_s, rec_s = conv0[b:b + 1].clone(), rec0[b:b + 1].clone()
        refs = []
        for t in range(T):
            ref, conv_s, rec_s = O.deltanet_step(ow, x[b, t:t + 1], conv_s, rec_s)
            refs.append(ref)
        worst = _compare_tokens(got[b], x[b], refs, f"seq {b}")
        e_s = O.rel_rms(rec[b:b + 1].cpu(), rec_s)
        e_c = O.rel_rms(conv[b:b + 1].cpu().float(), conv_s.float())
        print(f"DeltaNet T={T} state0={with_state} seq {b}: out max_abs={worst[0]:.2e} "
              f"rel_rms={worst[1]:.2e} state rel_rms={e_s:.2e} conv rel_rms={e_c:.2e}")
        assert e_s < STATE_REL and e_c < STATE_REL, (b, e_s, e_c)


@pytest.mark.parametrize("T,prefixes", [(64, [0, 0]), (200, [0, 130]), (1000, [70])])
def test_gqa_prefill_matches_oracle(cuda_device, T, prefixes):
    dev = cuda_device
    layer = 3
    wt = synthetic.layer_weights(layer, 22)
    ow = _oracle_weights(wt)
    B = len(prefixes)
    eng = BatchedAttentionState({layer: GqaWeights.from_tensors(wt, dev)}, batch=B, pool_blocks=64,
                                max_blocks_per_seq=24, device=dev)
    gen = torch.Generator().manual_seed(T + 1)
    caches = []
    for i, n in enumerate(prefixes):
        eng.set_length(i, n, position=n + 5)
        kk = torch.randn(2, n, 256, generator=gen).to(torch.bfloat16)
        vv = torch.randn(2, n, 256, generator=gen).to(torch.bfloat16)
        rows = eng.physical_rows(i, n).to(dev)
        eng.k_pool[layer][:, rows] = kk.to(dev)
        eng.v_pool[layer][:, rows] = vv.to(dev)
        caches.append((kk.float().unsqueeze(0), vv.float().unsqueeze(0)))
    eng.sync_tables()
    x = synthetic.hidden_stream(T, 32, rows=B).transpose(0, 1).contiguous()
    got = eng.prefill(x.to(dev)).cpu()
    torch.cuda.synchronize()
    assert _ext.device_error() == 0
    for b, n in enumerate(prefixes):
        kc, vc = None if n == 0 else caches[b][0], None if n == 0 else caches[b][1]
        refs = []
        for t in range(T):
            ref, kc, vc = O.gqa_step(ow, x[b, t:t + 1], kc, vc, n + 5 + t)
            refs.append(ref)
        worst = _compare_tokens(got[b], x[b], refs, f"seq {b}")
        rows = eng.physical_rows(b, n + T)[n:].to(dev)
        e_k = O.rel_rms(eng.k_pool[layer][:, rows].float().cpu(), kc[0, :, n:])
        e_v = O.rel_rms(eng.v_pool[layer][:, rows].float().cpu(), vc[0, :, n:])
        print(f"GQA T={T} prefix={n}: out max_abs={worst[0]:.2e} rel_rms={worst[1]:.2e} "
              f"K rel_rms={e_k:.2e} V rel_rms={e_v:.2e}")
        assert e_k < STATE_REL and e_v < STATE_REL, (b, e_k, e_v)
