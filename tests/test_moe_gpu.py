"""K5, the MoE block of a decode step, against the CPU oracle of router-ia's
batched_moe_step (qwen36_chat_batch.py:127-178), which the golden fixture
``reference_moe.npz`` pins to the reference itself.

The kernels compute in fp32 from the bf16 weights like the oracle, in their
own summation order, so the routing matches exactly except where two router
logits lie within rounding of each other (checked: such a token's logits at
the disagreement are within 1e-4), and the block's output agrees to fp32
rounding: the tolerances below (5e-5 max-abs on the output, 1e-4 relative
RMS of the MoE contribution) are far inside the attention path's 2e-2 /
1e-2 bar."""

from __future__ import annotations

from collections.abc import Mapping

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, engine, synthetic
from ria_b200.weights import MoeWeights

pytestmark = pytest.mark.gpu

TOP_K = 8


class _OnHost(Mapping):
    """Device weights seen by the CPU oracle: each tensor is copied on access,
    so only the experts it uses cross to the host."""

    def __init__(self, src):
        self.src = src

    def __getitem__(self, k):
        return self.src[k].cpu()

    def __iter__(self):
        return iter(self.src)

    def __len__(self):
        return len(self.src)


_CACHE: dict = {}


def _weights(num_experts: int, dev):
    key = (num_experts, str(dev))
    if key not in _CACHE:
        if num_experts <= 64:
            t = synthetic.moe_weights(31 + num_experts, num_experts=num_experts)
            host = t
        else:
            t = synthetic.moe_weights(31 + num_experts, num_experts=num_experts, device=dev)
            host = _OnHost(t)
        _CACHE.clear()
        _CACHE[key] = (host, MoeWeights.from_tensors(t, dev))
    return _CACHE[key]


def _residual(batch: int, seed: int, dev) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(batch, 2048, generator=g) * 2.0).to(dev)


def _oracle_logits(host, x_cpu: torch.Tensor) -> torch.Tensor:
    moe_in = O.rmsnorm(x_cpu, host["post_attention_layernorm.weight"])
    return moe_in @ host["mlp.gate.weight"].float().T


def _compare(host, x: torch.Tensor, out: torch.Tensor, plan: engine.MoePlan):
    x_cpu = x.cpu()
    ref_out, ref_ids, ref_wts, ref_sg = O.moe_step(host, x_cpu, top_k=TOP_K)
    ids = plan.expert_ids.cpu().long()
    wts = plan.expert_weights.cpu()
    same = (ids == ref_ids).all(dim=1)
    if not bool(same.all()):
        logits = _oracle_logits(host, x_cpu)
        for t in torch.nonzero(~same).flatten().tolist():
            a = logits[t, ids[t]].sort(descending=True).values
            b = logits[t, ref_ids[t]].sort(descending=True).values
            assert (a - b).abs().max().item() < 1e-4, f"token {t}: routing differs beyond a near tie"
    assert int(same.sum()) >= max(1, int(0.9 * same.numel()))
    keep = same.nonzero().flatten()
    assert O.max_abs(wts[keep], ref_wts[keep]) < 1e-5
    assert O.max_abs(plan.shared_gate.cpu(), ref_sg) < 1e-6
    got = out.cpu()[keep]
    ref = ref_out[keep]
    assert O.finite(got)
    assert O.max_abs(got, ref) < 5e-5
    assert O.rel_rms(got - x_cpu[keep], ref - x_cpu[keep]) < 1e-4


@pytest.mark.parametrize("batch", [1, 5, 16, 64])
def test_moe_matches_oracle_small_pool(cuda_device, batch):
    host, w = _weights(64, cuda_device)
    x = _residual(batch, 100 + batch, cuda_device)
    plan = engine.MoePlan.create(batch, w.num_experts, cuda_device, TOP_K)
    out = engine.moe_decode(x, w, plan)
    torch.cuda.synchronize()
    _compare(host, x, out, plan)


@pytest.mark.parametrize("batch", [8, 64])
def test_moe_matches_oracle_256_experts(cuda_device, batch):
    """The checkpoint's expert count (256, top-8)."""
    host, w = _weights(256, cuda_device)
    x = _residual(batch, 200 + batch, cuda_device)
    plan = engine.MoePlan.create(batch, w.num_experts, cuda_device, TOP_K)
    out = engine.moe_decode(x, w, plan)
    torch.cuda.synchronize()
    _compare(host, x, out, plan)


def test_moe_large_batch_many_tokens_per_expert(cuda_device):
    """256 tokens over 64 experts: about 32 tokens per expert, so every expert
    CTA stages several passes of 8 tokens, and the shared expert 32 passes."""
    host, w = _weights(64, cuda_device)
    x = _residual(256, 7, cuda_device)
    plan = engine.MoePlan.create(256, w.num_experts, cuda_device, TOP_K)
    out = engine.moe_decode(x, w, plan)
    torch.cuda.synchronize()
    _compare(host, x, out, plan)


def test_moe_unchosen_experts_are_not_read(cuda_device):
    """Experts no token chose are filled with NaN: the output stays finite and
    equal, so their weights were never read."""
    host, w = _weights(64, cuda_device)
    x = _residual(4, 11, cuda_device)
    plan = engine.MoePlan.create(4, w.num_experts, cuda_device, TOP_K)
    out = engine.moe_decode(x, w, plan).clone()
    used = set(plan.expert_ids.cpu().flatten().tolist())
    unused = [e for e in range(w.num_experts) if e not in used]
    assert unused
    poisoned = MoeWeights(**{f: getattr(w, f).clone() for f in w.__dataclass_fields__})
    for e in unused:
        poisoned.experts_gate[e].fill_(float("nan"))
        poisoned.experts_up[e].fill_(float("nan"))
        poisoned.experts_down[e].fill_(float("nan"))
    out2 = engine.moe_decode(x, poisoned, plan)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


def test_moe_deterministic_and_in_place(cuda_device):
    host, w = _weights(64, cuda_device)
    x = _residual(16, 3, cuda_device)
    plan = engine.MoePlan.create(16, w.num_experts, cuda_device, TOP_K)
    a = engine.moe_decode(x, w, plan).clone()
    b = engine.moe_decode(x, w, plan).clone()
    y = x.clone()
    engine.moe_decode(y, w, plan, out=y)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(a, y)


def test_moe_strided_rows(cuda_device):
    """Residual and output rows inside wider buffers (row strides > 2048)."""
    host, w = _weights(64, cuda_device)
    x = _residual(6, 5, cuda_device)
    xs = torch.zeros(6, 2048 + 64, device=cuda_device)
    xs[:, :2048] = x
    os_ = torch.zeros(6, 2048 + 128, device=cuda_device)
    plan = engine.MoePlan.create(6, w.num_experts, cuda_device, TOP_K)
    engine.moe_decode(xs[:, :2048], w, plan, out=os_[:, :2048])
    ref = engine.moe_decode(x, w, plan)
    torch.cuda.synchronize()
    assert torch.equal(os_[:, :2048], ref)
    assert bool((os_[:, 2048:] == 0).all())


def test_moe_graph_replay(cuda_device):
    """The block inside a captured CUDA graph gives the eager result."""
    host, w = _weights(64, cuda_device)
    x = _residual(8, 9, cuda_device)
    plan = engine.MoePlan.create(8, w.num_experts, cuda_device, TOP_K)
    eager = engine.moe_decode(x, w, plan).clone()
    out = torch.empty_like(x)
    engine.moe_decode(x, w, plan, out=out)  # warm-up outside capture
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            engine.moe_decode(x, w, plan, out=out)
    torch.cuda.current_stream().wait_stream(s)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    del g


def test_moe_argument_errors(cuda_device):
    host, w = _weights(64, cuda_device)
    x = _residual(4, 1, cuda_device)
    plan = engine.MoePlan.create(4, w.num_experts, cuda_device, TOP_K)
    small = engine.MoePlan(4, TOP_K, plan.expert_ids, plan.expert_weights, plan.shared_gate,
                           plan.workspace[:256])
    with pytest.raises(ValueError, match="workspace"):
        engine.moe_decode(x, w, small)
    too_many = engine.MoePlan.create(257, w.num_experts, cuda_device, TOP_K)
    with pytest.raises(ValueError, match="exceeds"):
        engine.moe_decode(_residual(257, 2, cuda_device), w, too_many)
    with pytest.raises(ValueError, match="plan is for batch"):
        engine.moe_decode(_residual(3, 2, cuda_device), w, plan)
    assert _ext.moe_workspace_bytes(0, 64, TOP_K) == 0
