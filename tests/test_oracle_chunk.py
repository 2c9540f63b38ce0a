"""The oracle's chunked gated delta rule (the published WY/UT algorithm
router-ia calls for a prompt) equals its token-by-token recurrence and the
transformers implementation router-ia imports for it."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from tests.test_gdn_prefill_gpu import make_inputs


def test_chunk_oracle_equals_recurrence():
    """The oracle's chunked form (the published WY/UT algorithm the reference
    calls) equals its recurrence, so either pins K2."""
    q, k, v, g, beta = make_inputs(1, 150, 2, 2, 3)
    o1, s1 = O.chunk_gated_delta_rule(q.float(), k.float(), v.float(), g, beta)
    o2, s2 = O.recurrent_gated_delta_rule(q.float(), k.float(), v.float(), g, beta)
    assert O.rel_rms(o1, o2) < 1e-5 and O.rel_rms(s1, s2) < 1e-5


@pytest.mark.parametrize("T,with_state", [(64, False), (150, True), (257, False)])
def test_chunk_oracle_matches_transformers_chunk_rule(T, with_state):
    """Pin against the reference's dependency itself: transformers 5.5
    ``torch_chunk_gated_delta_rule`` called exactly as router-ia calls it
    (qwen36_linear_attention_hf.py:93-97: chunk 64, in-kernel L2 norm, final
    state returned), on seeded inputs including lengths that are not a
    multiple of 64 and a non-zero initial state (the rule's own argument)."""
    hf = pytest.importorskip("transformers.models.qwen3_5_moe.modeling_qwen3_5_moe")
    q, k, v, g, beta = make_inputs(2, T, 3, 3, 40 + T)
    s0 = torch.randn(2, 3, 128, 128, generator=torch.Generator().manual_seed(T)) * 0.1 if with_state else None
    q, k, v = q.float(), k.float(), v.float()
    ref_o, ref_s = hf.torch_chunk_gated_delta_rule(q, k, v, g=g, beta=beta, initial_state=s0,
                                                   output_final_state=True, use_qk_l2norm_in_kernel=True)
    o, s = O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0)
    assert O.rel_rms(o, ref_o.float()) < 1e-5 and O.rel_rms(s, ref_s.float()) < 1e-5
    # and the token-by-token rule, in float64, agrees with both
    o2, s2 = O.recurrent_gated_delta_rule(q, k, v, g, beta, s0, dtype=torch.float64)
    assert O.rel_rms(ref_o.float(), o2) < 1e-5 and O.rel_rms(ref_s.float(), s2) < 1e-5
