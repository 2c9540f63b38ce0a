"""The oracle's chunked gated delta rule (the published WY/UT algorithm
router-ia calls for a prompt) equals its token-by-token recurrence."""

from __future__ import annotations

from oracle import attention_oracle as O
from tests.test_gdn_prefill_gpu import make_inputs


def test_chunk_oracle_equals_recurrence():
    """The oracle's chunked form (the published WY/UT algorithm the reference
    calls) equals its recurrence, so either pins K2."""
    q, k, v, g, beta = make_inputs(1, 150, 2, 2, 3)
    o1, s1 = O.chunk_gated_delta_rule(q.float(), k.float(), v.float(), g, beta)
    o2, s2 = O.recurrent_gated_delta_rule(q.float(), k.float(), v.float(), g, beta)
    assert O.rel_rms(o1, o2) < 1e-5 and O.rel_rms(s1, s2) < 1e-5
