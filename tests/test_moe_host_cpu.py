"""Host side of the MoE block (CPU): stacking the checkpoint's per-expert
tensors into the layout the kernels index, and the routing oracle's tie and
shape behaviour."""

from __future__ import annotations

import torch

from oracle import attention_oracle as O
from ria_b200 import synthetic
from ria_b200.weights import MoeWeights


def test_stacked_weights_follow_checkpoint_names():
    t = synthetic.moe_weights(5, num_experts=4)
    w = MoeWeights.from_tensors(t, "cpu")
    assert w.num_experts == 4
    assert w.experts_gate.shape == (4, 512, 2048) and w.experts_down.shape == (4, 2048, 512)
    for e in range(4):
        assert torch.equal(w.experts_gate[e], t[f"mlp.experts.{e}.gate_proj.weight"])
        assert torch.equal(w.experts_up[e], t[f"mlp.experts.{e}.up_proj.weight"])
        assert torch.equal(w.experts_down[e], t[f"mlp.experts.{e}.down_proj.weight"])
    assert torch.equal(w.shared_gate, t["mlp.shared_expert_gate.weight"].reshape(2048))
    assert w["router"] is w.router
    for f in w.__dataclass_fields__:
        assert getattr(w, f).dtype == torch.bfloat16
        assert getattr(w, f).is_contiguous()


def test_route_picks_largest_logits_and_normalises():
    g = torch.Generator().manual_seed(0)
    h = torch.randn(3, 16, generator=g)
    wr = torch.randn(10, 16, generator=g)
    ids, wts = O.route(h, wr, 4)
    logits = h @ wr.T
    for t in range(3):
        assert set(ids[t].tolist()) == set(logits[t].topk(4).indices.tolist())
        assert bool((logits[t, ids[t]][:-1] >= logits[t, ids[t]][1:]).all())
    assert torch.allclose(wts.sum(-1), torch.ones(3))
