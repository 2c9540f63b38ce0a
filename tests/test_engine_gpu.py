"""Batched ragged hybrid decode (benchmark configuration 3 in miniature):
B sequences with different KV lengths through a 3:1 DeltaNet/GQA stack.

Two checks per step: (1) every layer of every sequence against the CPU
oracle on the same input (the GPU's own output of the layer below), at the
per-layer bound -- 2e-2 max-abs, 1e-2 relative RMS on the fp32 residual;
(2) ``BatchedAttentionState.step`` equal, bit for bit, to the same layers run
one at a time.  Checking each layer on its own input keeps the bound that of
one layer: compared end to end, the bf16 roundings of 8 layers compound.
Five sequences run the projections as the fused GEMVs, twenty-four as the
norm kernel plus library GEMMs."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from ria_b200 import constants as C
from ria_b200.engine import BatchedAttentionState
from ria_b200.weights import DeltaNetWeights, GqaWeights

pytestmark = pytest.mark.gpu


RAGGED_24 = [0, 1, 63, 64, 65, 127, 128, 129, 200, 255, 256, 257] + [(37 * i) % 300 for i in range(1, 13)]


@pytest.mark.parametrize("lengths,steps", [([0, 5, 64, 130, 257], 3), (RAGGED_24, 2)])
def test_ragged_hybrid_stack_matches_per_sequence_oracle(cuda_device, lengths, steps):
    from ria_b200.engine import deltanet_decode, gqa_decode

    layers = [0, 1, 2, 3, 4, 5, 6, 7]  # DN DN DN GQA DN DN DN GQA
    wt = {layer: synthetic.layer_weights(layer, 3) for layer in layers}
    dev_w = {layer: (GqaWeights if C.is_full_attention_layer(layer) else DeltaNetWeights).from_tensors(w, cuda_device)
             for layer, w in wt.items()}
    B = len(lengths)
    engines = [BatchedAttentionState(dev_w, batch=B, pool_blocks=8 * B, max_blocks_per_seq=8, device=cuda_device)
               for _ in range(2)]
    eng, twin = engines
    gen = torch.Generator().manual_seed(5)
    # per-sequence initial state: random DN / conv state, random KV prefix
    ref_state = []
    for i, n in enumerate(lengths):
        for e in engines:
            e.set_length(i, n, position=n + 2)
        seq = {}
        for layer in layers:
            if C.is_full_attention_layer(layer):
                k = torch.randn(2, n, 256, generator=gen).to(torch.bfloat16)
                v = torch.randn(2, n, 256, generator=gen).to(torch.bfloat16)
                for e in engines:
                    rows = e.physical_rows(i, n).to(cuda_device)
                    e.k_pool[layer][:, rows] = k.to(cuda_device)
                    e.v_pool[layer][:, rows] = v.to(cuda_device)
                seq[layer] = [k.float().unsqueeze(0), v.float().unsqueeze(0)]
            else:
                rec = torch.randn(1, 32, 128, 128, generator=gen) * 0.1
                conv = (torch.randn(1, 8192, 4, generator=gen) * 0.1).to(torch.bfloat16)
                for e in engines:
                    e.rec[layer][i] = rec[0].to(cuda_device)
                    e.conv[layer][i] = conv[0].to(cuda_device)
                seq[layer] = [conv, rec]
        ref_state.append(seq)
    for e in engines:
        e.sync_tables()
    xs = synthetic.hidden_stream(steps, 6, rows=B)
    worst = (0.0, 0.0)
    for t in range(steps):
        x = xs[t].to(cuda_device)
        got = eng.step(x)
        # the same step one layer at a time, keeping every layer's input
        twin.reserve_next()
        launch = twin.plan()
        ins, outs = [], []
        for layer in layers:
            ins.append(x)
            if C.is_full_attention_layer(layer):
                x = gqa_decode(x, dev_w[layer], twin.k_pool[layer], twin.v_pool[layer], twin.block_table,
                               twin.inv_freq, launch, twin.seq_lens, twin.positions)
            else:
                x = deltanet_decode(x, dev_w[layer], twin.rec[layer], twin.conv[layer])
            outs.append(x)
        _ext.advance_positions(twin.seq_lens, twin.positions)
        twin.lengths = [n + 1 for n in twin.lengths]
        assert torch.equal(got, x), "step() differs from its layers run one at a time"
        for i in range(B):
            pos = lengths[i] + 2 + t
            for li, layer in enumerate(layers):
                s = ref_state[i][layer]
                xin = ins[li][i:i + 1].cpu()
                if C.is_full_attention_layer(layer):
                    ref, s[0], s[1] = O.gqa_step(wt[layer], xin, s[0], s[1], pos)
                else:
                    ref, s[0], s[1] = O.deltanet_step(wt[layer], xin, s[0], s[1])
                out = outs[li][i:i + 1].cpu()
                err = (O.max_abs(out, ref), O.rel_rms(out - xin, ref - xin))
                worst = (max(worst[0], err[0]), max(worst[1], err[1]))
                assert err[0] < 2e-2 and err[1] < 1e-2, (t, i, layer, err)
    print(f"per-layer worst: max_abs={worst[0]:.2e} rel_rms(contribution)={worst[1]:.2e}")
    assert eng.lengths == [n + steps for n in lengths]
    assert eng.seq_lens.tolist() == eng.lengths
    assert _ext.device_error() == 0
