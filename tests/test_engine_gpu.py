"""Batched ragged hybrid decode (benchmark configuration 3 in miniature):
B sequences with different KV lengths through a 3:1 DeltaNet/GQA stack, each
sequence checked against the CPU oracle run one sequence at a time.

The residual stream goes through 8 layers here, each adding the bf16
projection rounding of its contribution, so the per-layer bound (2e-2 max-abs)
is widened to 6e-2 for the chain; the relative RMS bound stays 1e-2."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from ria_b200 import constants as C
from ria_b200.engine import BatchedAttentionState
from ria_b200.weights import DeltaNetWeights, GqaWeights

pytestmark = pytest.mark.gpu


def test_ragged_hybrid_stack_matches_per_sequence_oracle(cuda_device):
    layers = [0, 1, 2, 3, 4, 5, 6, 7]  # DN DN DN GQA DN DN DN GQA
    wt = {layer: synthetic.layer_weights(layer, 3) for layer in layers}
    dev_w = {layer: (GqaWeights if C.is_full_attention_layer(layer) else DeltaNetWeights).from_tensors(w, cuda_device)
             for layer, w in wt.items()}
    lengths = [0, 5, 64, 130, 257]
    B = len(lengths)
    steps = 3
    eng = BatchedAttentionState(dev_w, batch=B, pool_blocks=40, max_blocks_per_seq=8, device=cuda_device)
    gen = torch.Generator().manual_seed(5)
    # per-sequence initial state: random DN / conv state, random KV prefix
    ref_state = []
    for i, n in enumerate(lengths):
        eng.set_length(i, n, position=n + 2)
        seq = {}
        for layer in layers:
            if C.is_full_attention_layer(layer):
                k = torch.randn(2, n, 256, generator=gen).to(torch.bfloat16)
                v = torch.randn(2, n, 256, generator=gen).to(torch.bfloat16)
                rows = eng.physical_rows(i, n).to(cuda_device)
                eng.k_pool[layer][:, rows] = k.to(cuda_device)
                eng.v_pool[layer][:, rows] = v.to(cuda_device)
                seq[layer] = [k.float().unsqueeze(0), v.float().unsqueeze(0)]
            else:
                rec = torch.randn(1, 32, 128, 128, generator=gen) * 0.1
                conv = (torch.randn(1, 8192, 4, generator=gen) * 0.1).to(torch.bfloat16)
                eng.rec[layer][i] = rec[0].to(cuda_device)
                eng.conv[layer][i] = conv[0].to(cuda_device)
                seq[layer] = [conv, rec]
        ref_state.append(seq)
    eng.sync_tables()
    xs = synthetic.hidden_stream(steps, 6, rows=B)
    for t in range(steps):
        got = eng.step(xs[t].to(cuda_device)).cpu()
        for i in range(B):
            x = xs[t, i:i + 1]
            pos = lengths[i] + 2 + t
            for layer in layers:
                s = ref_state[i][layer]
                if C.is_full_attention_layer(layer):
                    x, s[0], s[1] = O.gqa_step(wt[layer], x, s[0], s[1], pos)
                else:
                    x, s[0], s[1] = O.deltanet_step(wt[layer], x, s[0], s[1])
            err = (O.max_abs(got[i:i + 1], x), O.rel_rms(got[i:i + 1], x))
            assert err[0] < 6e-2 and err[1] < 1e-2, (t, i, err)
    assert eng.lengths == [n + steps for n in lengths]
    assert eng.seq_lens.tolist() == eng.lengths
    assert _ext.device_error() == 0
