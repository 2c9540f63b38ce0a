"""K2 (chunked Gated DeltaNet prefill on tcgen05) against the token-by-token
rule in float64 on the CPU (the oracle's restatement of
qwen36_attention_cache.py:256-266 and qwen36_linear_attention_hf.py:108-137,
with in-kernel L2 norms).

Tolerances (the bars of the attention path): outputs, stored in bf16, within
1e-2 relative RMS and 2e-2 in the scale-aware max form (max |d| / max(1,
|ref|)); the final fp32 state within 1e-3 relative RMS of the float64
recurrence.  The kernel runs the products that feed the state on fp16
operands and the rest on bf16 (fp32 accumulation, fp32 state), which puts the
state about 4e-4 and the outputs about 2.4e-3 from the recurrence on these
inputs.

Configuration 2 (8 sequences x 8192 tokens, 16 key / 32 value heads) runs at
full size; four seeded (sequence, value head) pairs, the two value heads of
one key head among them, are checked against the float64 recurrence over all
8192 tokens, from a zero and from a non-zero initial state."""

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
STATE_REL = 1e-3


def make_inputs(B, T, Hk, Hv, seed, device="cpu"):
    """q, k, v ~ N(0, 1) bf16; log decay g = -exp(A_log) softplus(a + dt_bias)
    with A_log ~ U(0, 2.7), dt_bias ~ U(-1, 1), a ~ N(0, 1); beta = sigmoid(N(0, 1))
    -- configuration 0's gate distributions."""
    gen = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(B, T, Hk, 128, generator=gen, device=device).to(torch.bfloat16)
    k = torch.randn(B, T, Hk, 128, generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn(B, T, Hv, 128, generator=gen, device=device).to(torch.bfloat16)
    a_log = torch.rand(Hv, generator=gen, device=device) * 2.7
    dt_bias = torch.rand(Hv, generator=gen, device=device) * 2 - 1
    a = torch.randn(B, T, Hv, generator=gen, device=device)
    g = -torch.exp(a_log) * F.softplus(a + dt_bias)
    beta = torch.sigmoid(torch.randn(B, T, Hv, generator=gen, device=device))
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


def check(errs):
    assert errs[0] < OUT_REL and errs[1] < OUT_MAX and errs[2] < STATE_REL, errs


@pytest.mark.parametrize("T", [1, 63, 64, 65, 200])
def test_ragged_lengths(cuda_device, T):
    check(run_case(cuda_device, 2, T, 2, 4, seed=T))


def test_initial_state(cuda_device):
    check(run_case(cuda_device, 2, 130, 1, 2, seed=7, with_state=True))


def test_long_sequence_state(cuda_device):
    """1024 tokens: the north-star horizon for the fp32 state."""
    check(run_case(cuda_device, 1, 1024, 1, 2, seed=9))
    check(run_case(cuda_device, 1, 1024, 1, 2, seed=10, with_state=True))


@pytest.mark.parametrize("ws_chunks", [1, 3])
def test_blocked_workspace(cuda_device, ws_chunks):
    """A workspace smaller than the prompt: blocks of chunks with the state
    carried through final_state give the same result."""
    check(run_case(cuda_device, 2, 450, 1, 2, seed=11, with_state=True, ws_chunks=ws_chunks))


def test_workspace_too_small(cuda_device):
    q, k, v, g, beta = (t.to(cuda_device) for t in make_inputs(1, 64, 1, 2, 0))
    ws = torch.empty(1024, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(ValueError, match="workspace"):
        chunk_gated_delta_rule(q, k, v, g, beta, workspace=ws)


# (sequence, value head): heads 16 and 17 share key head 8
CONFIG2_PAIRS = [(0, 0), (3, 16), (3, 17), (7, 31)]


@pytest.mark.parametrize("with_state", [False, True])
def test_configuration2_full_size(cuda_device, with_state):
    """Configuration 2 as benchmarked: 8 x 8192 tokens, Hk = 16, Hv = 32,
    chunk 64, one call.  Four (sequence, head) pairs against the float64
    recurrence over all 8192 tokens; every output finite."""
    B, T, Hk, Hv = 8, 8192, 16, 32
    dev = cuda_device
    q, k, v, g, beta = make_inputs(B, T, Hk, Hv, seed=2024, device=dev)
    s0 = None
    if with_state:
        s0 = torch.randn(B, Hv, 128, 128, generator=torch.Generator(device=dev).manual_seed(77), device=dev) * 0.1
    out, sf = chunk_gated_delta_rule(q, k, v, g, beta, s0)
    torch.cuda.synchronize()
    assert _ext.device_error() == 0
    assert O.finite(out) and O.finite(sf)
    grp = Hv // Hk
    worst = [0.0, 0.0, 0.0]
    for b, h in CONFIG2_PAIRS:
        hk = h // grp
        ref_o, ref_s = O.recurrent_gated_delta_rule(
            q[b:b + 1, :, hk:hk + 1].float().cpu(), k[b:b + 1, :, hk:hk + 1].float().cpu(),
            v[b:b + 1, :, h:h + 1].float().cpu(), g[b:b + 1, :, h:h + 1].cpu(), beta[b:b + 1, :, h:h + 1].cpu(),
            None if s0 is None else s0[b:b + 1, h:h + 1].cpu(), dtype=torch.float64)
        got_o = out[b:b + 1, :, h:h + 1].float().cpu()
        got_s = sf[b:b + 1, h:h + 1].cpu()
        errs = (O.rel_rms(got_o, ref_o), O.max_err_bf16(got_o, ref_o), O.rel_rms(got_s, ref_s))
        print(f"config 2 state0={with_state} seq {b} head {h}: out rel_rms={errs[0]:.2e} max={errs[1]:.2e} "
              f"state rel_rms={errs[2]:.2e}")
        worst = [max(w, e) for w, e in zip(worst, errs)]
        check(errs)
    print(f"config 2 state0={with_state} worst: out rel_rms={worst[0]:.2e} max={worst[1]:.2e} "
          f"state rel_rms={worst[2]:.2e}")
