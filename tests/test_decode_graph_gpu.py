"""The decode step captured as one CUDA graph (DecodeGraph) equals the eager
step with the same split plan, token after token, across a page boundary
(the block table grows between replays) and for a sequence starting empty."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from ria_b200 import constants as C
from ria_b200.engine import BatchedAttentionState, DecodeGraph
from ria_b200.weights import DeltaNetWeights, GqaWeights

pytestmark = pytest.mark.gpu


def _twins(dev, lengths):
    layers = [0, 1, 2, 3]
    w = {l: (GqaWeights if C.is_full_attention_layer(l) else DeltaNetWeights).from_tensors(
        synthetic.layer_weights(l, 4), dev) for l in layers}
    engines = [BatchedAttentionState(w, batch=len(lengths), pool_blocks=64, max_blocks_per_seq=8, device=dev)
               for _ in range(2)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    a, b = engines
    for l in a.rec:
        a.rec[l].normal_(0, 0.1, generator=gen)
        a.conv[l].normal_(0, 0.1, generator=gen)
        b.rec[l].copy_(a.rec[l])
        b.conv[l].copy_(a.conv[l])
    for e in engines:
        for i, n in enumerate(lengths):
            e.set_length(i, n)
        e.sync_tables()
    for l in a.k_pool:
        a.k_pool[l].normal_(0, 1, generator=gen)
        a.v_pool[l].normal_(0, 1, generator=gen)
        b.k_pool[l].copy_(a.k_pool[l])
        b.v_pool[l].copy_(a.v_pool[l])
    return a, b


def test_graph_replay_equals_eager(cuda_device):
    lengths = [0, 62, 127]  # sequences 1 and 2 cross a 64-token page during the run
    a, b = _twins(cuda_device, lengths)
    xs = synthetic.hidden_stream(8, 21, rows=len(lengths)).to(cuda_device)  # [8, B, 2048]
    a.step(xs[0])  # eager warm-up on both (library and cuBLAS initialisation)
    b.step(xs[0])
    g = DecodeGraph(a)
    for t in range(1, 8):
        got = g.step(xs[t]).clone()
        ref = b.step(xs[t], launch=g.launch)
        err = O.max_abs(got, ref)
        assert err <= 1e-5 * max(1.0, ref.abs().max().item()), (t, err)
    assert a.lengths == b.lengths and a.positions_host == b.positions_host
    assert torch.equal(a.seq_lens, b.seq_lens) and torch.equal(a.positions, b.positions)
    for l in a.rec:
        assert O.rel_rms(a.rec[l], b.rec[l]) < 1e-6
    assert _ext.device_error() == 0
