"""Prompt prefill of the full model (attention prefill kernels K2 / K4 and
the MoE over all prompt tokens as grouped library GEMMs) against the decode
path, and the prompt MoE against the decode MoE kernels and the oracle.

The prompt MoE multiplies bf16 activations where the decode kernels keep
fp32-grade products (bf16 hi + lo), so the two agree to about 1e-3 relative
per block; over a 4-layer stack fed T tokens the hidden state and the
recurrent states stay within 2e-2 relative RMS of T teacher-forced decode
steps (the attention prefill's own bound, tests/test_engine_prefill_gpu.py).
"""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import synthetic
from ria_b200 import constants as C
from ria_b200.engine import MoePlan, moe_decode, moe_prefill
from ria_b200.weights import MoeWeights

from test_model_gpu import LAYERS, VOCAB, _model, _weights

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("num_experts,tokens", [(64, 300), (256, 256)])
def test_prompt_moe_matches_decode_kernels_and_oracle(cuda_device, num_experts, tokens):
    t = synthetic.moe_weights(70 + num_experts, num_experts=num_experts)
    w = MoeWeights.from_tensors(t, cuda_device)
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(tokens, 2048, generator=g) * 2.0).to(cuda_device)
    got = moe_prefill(x, w, chunk=128)  # several chunks
    ref = torch.empty_like(x)
    for s in range(0, tokens, 256):
        xc = x[s:s + 256]
        ref[s:s + 256] = moe_decode(xc, w, MoePlan.create(xc.shape[0], num_experts, cuda_device))
    torch.cuda.synchronize()
    assert O.finite(got)
    assert O.rel_rms(got - x, ref - x) < 5e-3
    assert O.max_abs(got, ref) < 1e-2
    # against the oracle on a few tokens, at the attention path's bar
    sel = torch.arange(0, tokens, 37)
    o_out, _, _, _ = O.moe_step(t, x.cpu()[sel], top_k=8)
    xs = x.cpu()[sel]
    assert O.max_abs(got.cpu()[sel], o_out) < 2e-2
    assert O.rel_rms(got.cpu()[sel] - xs, o_out - xs) < 1e-2
    # chunking does not change the result beyond GEMM rounding
    whole = moe_prefill(x, w)
    assert O.rel_rms(whole - x, got - x) < 1e-3


def test_model_prefill_matches_teacher_forced_decode(cuda_device):
    """8 experts, top-8: every token uses every expert, so the comparison is
    not at the mercy of a top-k boundary (two paths whose router logits differ
    by rounding may pick a different 8th expert out of 16, a discontinuity
    unrelated to the arithmetic under test)."""
    _, _, ht, attn, _, head = _weights(cuda_device)
    moe = {layer: MoeWeights.from_tensors(synthetic.moe_weights(80 + layer, num_experts=8), cuda_device)
           for layer in LAYERS}
    lengths = [0, 9, 70]
    a, _ = _model(attn, moe, head, lengths, cuda_device, 12)
    b, _ = _model(attn, moe, head, lengths, cuda_device, 12)
    T = 40
    g = torch.Generator().manual_seed(13)
    prompt = torch.randint(0, VOCAB, (len(lengths), T), generator=g, dtype=torch.int32).to(cuda_device)
    got = a.prefill(prompt).clone()
    # the prefill is its pieces: embedding rows, the layers with the prompt
    # MoE after each, the head on the last position
    c, _ = _model(attn, moe, head, lengths, cuda_device, 12)
    x = head.embedding.index_select(0, prompt.reshape(-1)).float().view(len(lengths), T, C.HIDDEN)
    x = c.state.prefill(x, after_layer=lambda layer, y: moe_prefill(y.reshape(-1, C.HIDDEN), moe[layer]).view(y.shape))
    assert torch.equal(x[:, -1], a.hidden)
    for i in range(T):
        b.ids.copy_(prompt[:, i])
        b.step()
    torch.cuda.synchronize()
    assert a.state.lengths == b.state.lengths == [n + T for n in lengths]
    assert torch.equal(a.state.seq_lens, b.state.seq_lens)
    assert O.rel_rms(a.hidden, b.hidden) < 2e-2
    for layer in LAYERS:
        if C.is_full_attention_layer(layer):
            for i, n in enumerate(lengths):
                rows_a = a.state.physical_rows(i, n + T).to(cuda_device)
                rows_b = b.state.physical_rows(i, n + T).to(cuda_device)
                assert O.rel_rms(a.state.v_pool[layer][:, rows_a].float(), b.state.v_pool[layer][:, rows_b].float()) < 2e-2
        else:
            assert O.rel_rms(a.state.rec[layer], b.state.rec[layer]) < 2e-2
    # the picked ids agree except where the decode path's two best logits are close
    ref_logits, _ = O.lm_head_greedy(b.hidden.cpu(), ht["model.language_model.norm.weight"], ht["lm_head.weight"])
    for i in range(len(lengths)):
        ia, ib = int(got[i]), int(b.ids[i])
        if ia != ib:
            assert ref_logits[i, ib] - ref_logits[i, ia] < 5e-2, (i, ia, ib)
