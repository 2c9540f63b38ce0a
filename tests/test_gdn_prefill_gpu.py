"""K2 (chunked Gated DeltaNet prefill on tcgen05) against the token-by-token
rule in float64 on the CPU (the oracle's restatement of
qwen36_attention_cache.py:256-266 with in-kernel L2 norms).

Tolerances: the kernel uses bf16 tensor-core operands (q, k, v, the chunk's
T-inverse, W, U, the per-chunk bf16 copy of the state) with fp32
accumulation and an fp32 state; outputs within 1e-2 relative RMS and 2e-2 in
the scale-aware max form (max |d| / max(1, |ref|)), the final fp32 state within
1e-2 relative RMS of the float64 recurrence."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import attention_oracle as O
from ria_b200 import _ext
from ria_b200.prefill import chunk_gated_delta_rule

pytestmark = pytest.mark.gpu

OUT_REL = 1e-2
OUT_MAX = 2e-2
STATE_REL = 1e-2


def make_inputs(B, T, Hk, Hv, seed):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, Hk, 128, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, T, Hk, 128, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, T, Hv, 128, generator=gen).to(torch.bfloat16)
    a_log = torch.rand(Hv, generator=gen) * 2.7
    dt_bias = torch.rand(Hv, generator=gen) * 2 - 1
    a = torch.randn(B, T, Hv, generator=gen)
    g = -torch.exp(a_log) * F.softplus(a + dt_bias)
    beta = torch.sigmoid(torch.randn(B, T, Hv, generator=gen))
    return q, k, v, g.float(), beta.float()


def run_case(dev, B, T, Hk, Hv, seed, with_state=False, ws_chunks=None):
    q, k, v, g, beta = make_inputs(B, T, Hk, Hv, seed)
    s0 = (torch.randn(B, Hv, 128, 128, generator=torch.Generator().manual_seed(seed + 1)) * 0.1) if with_state else None
    ws = None
    if ws_chunks is not None:  # a workspace of ws_chunks chunks: the prompt runs in blocks
        ws = torch.empty(_ext.gdn_chunk_prefill_workspace_bytes(B, 64 * ws_chunks, Hv), dtype=torch.uint8, device=dev)
    out, sf = chunk_gated_delta_rule(q.to(dev), k.to(dev), v.to(dev), g.to(dev), beta.to(dev),
                                     None if s0 is None else s0.to(dev), workspace=ws)
    grp = Hv // Hk
    ref_o, ref_s = O.recurrent_gated_delta_rule(q.float().repeat_interleave(grp, 2), k.float().repeat_interleave(grp, 2),
                                                v.float(), g, beta, s0, dtype=torch.float64)
    got_o, got_s = out.float().cpu(), sf.cpu()
    errs = (O.rel_rms(got_o, ref_o), O.max_err_bf16(got_o, ref_o), O.rel_rms(got_s, ref_s))
    print(f"B={B} T={T} Hk={Hk} Hv={Hv} state0={with_state}: out rel_rms={errs[0]:.2e} "
          f"max={errs[1]:.2e} state rel_rms={errs[2]:.2e}")
    assert _ext.device_error() == 0
    return errs


@pytest.mark.parametrize("T", [1, 63, 64, 65, 200])
def test_ragged_lengths(cuda_device, T):
    errs = run_case(cuda_device, 2, T, 2, 4, seed=T)
    assert errs[0] < OUT_REL and errs[1] < OUT_MAX and errs[2] < STATE_REL, errs


def test_initial_state(cuda_device):
    errs = run_case(cuda_device, 2, 130, 1, 2, seed=7, with_state=True)
    assert errs[0] < OUT_REL and errs[1] < OUT_MAX and errs[2] < STATE_REL, errs


def test_long_sequence_state(cuda_device):
    errs = run_case(cuda_device, 1, 1024, 1, 2, seed=9)
    assert errs[0] < OUT_REL and errs[1] < OUT_MAX and errs[2] < STATE_REL, errs


@pytest.mark.parametrize("ws_chunks", [1, 3])
def test_blocked_workspace(cuda_device, ws_chunks):
    """A workspace smaller than the prompt: blocks of chunks with the state
    carried through final_state give the same result."""
    errs = run_case(cuda_device, 2, 450, 1, 2, seed=11, with_state=True, ws_chunks=ws_chunks)
    assert errs[0] < OUT_REL and errs[1] < OUT_MAX and errs[2] < STATE_REL, errs


def test_workspace_too_small(cuda_device):
    q, k, v, g, beta = (t.to(cuda_device) for t in make_inputs(1, 64, 1, 2, 0))
    ws = torch.empty(1024, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(ValueError, match="workspace"):
        chunk_gated_delta_rule(q, k, v, g, beta, workspace=ws)
