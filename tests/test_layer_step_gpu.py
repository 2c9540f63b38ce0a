"""The one-call layer steps (ria_deltanet_layer_decode, ria_gqa_layer_decode)
launch the same kernels in the same order as the separate entry points, so a
layer stepped either way gives bit-identical outputs, recurrent and conv
states, and KV caches -- checked over several steps at batch 1 (the drop-in
module's case, scalar lengths for GQA) and batch 3 (device length arrays).
Argument checks: batches above the GEMV range and short scratch buffers are
rejected before any launch."""

from __future__ import annotations

import pytest
import torch

from ria_b200 import _ext, synthetic
from ria_b200 import constants as C
from ria_b200.engine import plan_gqa_split
from ria_b200.weights import DeltaNetWeights, GqaWeights, rope_inv_freq

pytestmark = pytest.mark.gpu


def _scratch(dev, nbytes):
    return torch.empty(nbytes, dtype=torch.uint8, device=dev)


def _dn_separate(x, w, rec, conv):
    """The DeltaNet layer step as three separate entry-point calls."""
    B = x.shape[0]
    proj = torch.empty(B, C.DN_PROJ_WIDTH, dtype=torch.bfloat16, device=x.device)
    _ext.rmsnorm_gemv(x, w.in_norm, w.w_in, proj)
    gated = torch.empty(B, C.LINEAR_VALUE_DIM, dtype=torch.bfloat16, device=x.device)
    _ext.gdn_decode_step(proj[:, C.DN_PROJ_QKV[0]:C.DN_PROJ_QKV[1]], proj[:, C.DN_PROJ_Z[0]:C.DN_PROJ_Z[1]],
                         proj[:, C.DN_PROJ_B[0]:C.DN_PROJ_B[1]], proj[:, C.DN_PROJ_A[0]:C.DN_PROJ_A[1]], w.conv_w,
                         w.a_log, w.dt_bias, w.norm_w, conv, rec, None, gated)
    out = torch.empty(B, C.HIDDEN, device=x.device)
    _ext.gemv_residual(gated, w.w_out, x, out)
    return out


def _gqa_separate(x, w, k_pool, v_pool, table, inv, launch, **lens):
    """The GQA layer step as three separate entry-point calls."""
    B = x.shape[0]
    proj = torch.empty(B, C.GQA_PROJ_WIDTH, dtype=torch.bfloat16, device=x.device)
    _ext.rmsnorm_gemv(x, w.in_norm, w.w_in, proj)
    attn = torch.empty(B, C.FULL_Q_DIM, dtype=torch.bfloat16, device=x.device)
    _ext.gqa_decode_paged(proj[:, C.GQA_PROJ_Q[0]:C.GQA_PROJ_Q[1]], proj[:, C.GQA_PROJ_K[0]:C.GQA_PROJ_K[1]],
                          proj[:, C.GQA_PROJ_V[0]:C.GQA_PROJ_V[1]], w.q_norm, w.k_norm, inv, k_pool, v_pool, table,
                          lens.get("seq_lens"), lens.get("positions"), attn, launch.workspace, launch.split_pages,
                          launch.max_splits, seq_len0=lens.get("seq_len0", 0), position0=lens.get("position0", 0))
    out = torch.empty(B, C.HIDDEN, device=x.device)
    _ext.gemv_residual(attn, w.w_out, x, out)
    return out


@pytest.mark.parametrize("batch", [1, 3])
def test_deltanet_layer_step_equals_separate_calls(cuda_device, batch):
    dev = cuda_device
    w = DeltaNetWeights.from_tensors(synthetic.deltanet_weights(9), dev)
    args = _ext.deltanet_layer_args(w)
    g = torch.Generator(device=dev).manual_seed(batch)
    rec_a = torch.randn(batch, 32, 128, 128, device=dev, generator=g) * 0.1
    conv_a = (torch.randn(batch, 8192, 4, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    rec_b, conv_b = rec_a.clone(), conv_a.clone()
    scratch = _scratch(dev, _ext.deltanet_layer_scratch_bytes(batch))
    for step in range(3):
        x = torch.randn(batch, C.HIDDEN, device=dev, generator=g)
        ref = _dn_separate(x, w, rec_a, conv_a)
        out = torch.empty(batch, C.HIDDEN, device=dev)
        _ext.deltanet_layer_decode(x, args, conv_b, rec_b, out, scratch)
        torch.cuda.synchronize(dev)
        assert torch.equal(out, ref), step
        assert torch.equal(rec_a, rec_b) and torch.equal(conv_a, conv_b), step
    assert _ext.device_error() == 0


@pytest.mark.parametrize("lengths", [[700], [0, 130, 4000]])
def test_gqa_layer_step_equals_separate_calls(cuda_device, lengths):
    dev = cuda_device
    w = GqaWeights.from_tensors(synthetic.gqa_weights(10), dev)
    args = _ext.gqa_layer_args(w)
    inv = rope_inv_freq(dev)
    B = len(lengths)
    steps = 3
    nb = max((n + steps + 63) // 64 for n in lengths) + 1
    table = torch.arange(B * nb, dtype=torch.int32, device=dev).reshape(B, nb)
    g = torch.Generator(device=dev).manual_seed(sum(lengths))
    k_a = torch.randn(2, B * nb * 64, 256, device=dev, generator=g).to(torch.bfloat16)
    v_a = torch.randn(2, B * nb * 64, 256, device=dev, generator=g).to(torch.bfloat16)
    k_b, v_b = k_a.clone(), v_a.clone()
    for step in range(steps):
        cur = [n + step for n in lengths]
        x = torch.randn(B, C.HIDDEN, device=dev, generator=g)
        launch = plan_gqa_split([n + 1 for n in cur], dev)
        out = torch.empty(B, C.HIDDEN, device=dev)
        scratch = _scratch(dev, _ext.gqa_layer_scratch_bytes(B, launch.max_splits))
        if B == 1:  # scalar length and position, as the drop-in module calls it
            ref = _gqa_separate(x, w, k_a, v_a, table, inv, launch, seq_len0=cur[0], position0=cur[0] + 11)
            _ext.gqa_layer_decode(x, args, inv, k_b, v_b, table, out, scratch, launch.split_pages, launch.max_splits,
                                  seq_len0=cur[0], position0=cur[0] + 11)
        else:
            seq_lens = torch.tensor(cur, dtype=torch.int32, device=dev)
            positions = seq_lens + 11
            ref = _gqa_separate(x, w, k_a, v_a, table, inv, launch, seq_lens=seq_lens, positions=positions)
            _ext.gqa_layer_decode(x, args, inv, k_b, v_b, table, out, scratch, launch.split_pages, launch.max_splits,
                                  seq_lens=seq_lens, positions=positions)
        torch.cuda.synchronize(dev)
        assert torch.equal(out, ref), step
        assert torch.equal(k_a, k_b) and torch.equal(v_a, v_b), step
    assert _ext.device_error() == 0


def test_layer_steps_reject_bad_arguments(cuda_device):
    dev = cuda_device
    w = DeltaNetWeights.from_tensors(synthetic.deltanet_weights(9), dev)
    args = _ext.deltanet_layer_args(w)
    rec = torch.zeros(9, 32, 128, 128, device=dev)
    conv = torch.zeros(9, 8192, 4, dtype=torch.bfloat16, device=dev)
    x = torch.zeros(9, C.HIDDEN, device=dev)
    out = torch.empty_like(x)
    with pytest.raises(ValueError, match="batch"):
        _ext.deltanet_layer_decode(x, args, conv, rec, out, _scratch(dev, 1 << 22))
    with pytest.raises(ValueError, match="scratch"):
        _ext.deltanet_layer_decode(x[:1], args, conv[:1], rec[:1], out[:1], _scratch(dev, 256))
