"""Pin the CPU oracle to router-ia's own outputs (tests/golden/make_golden.py)."""

from __future__ import annotations

import torch

from oracle import attention_oracle as O
from ria_b200 import synthetic


def _dn_run(meta):
    w = synthetic.layer_weights(meta["dn_layer"], meta["weight_seed"])
    xs = synthetic.hidden_stream(meta["dn_tokens"], meta["dn_input_seed"])
    conv = rec = None
    res = []
    for t in range(meta["dn_tokens"]):
        r, conv, rec = O.deltanet_step(w, xs[t], conv, rec)
        res.append(r.reshape(-1))
    return torch.stack(res), conv, rec


def test_deltanet_step_matches_reference(golden):
    meta = golden["meta"]
    res, conv, rec = _dn_run(meta)
    ref_res = torch.from_numpy(golden["dn_residual"])
    assert O.rel_rms(res, ref_res) < 1e-6
    assert O.max_abs(res, ref_res) < 1e-5
    assert torch.equal(conv[0].float(), torch.from_numpy(golden["dn_conv_state"]))
    heads = meta["rec_heads"]
    assert O.rel_rms(rec[0, heads], torch.from_numpy(golden["dn_rec_heads"])) < 1e-6
    norms = rec[0].double().flatten(1).norm(dim=1)
    assert O.rel_rms(norms, torch.from_numpy(golden["dn_rec_norms"])) < 1e-6


def test_gqa_step_matches_reference(golden):
    meta = golden["meta"]
    w = synthetic.layer_weights(meta["gqa_layer"], meta["weight_seed"])
    kp, vp = synthetic.kv_prefix(meta["gqa_prefix"], meta["gqa_cache_seed"])
    kc, vc = kp.float().unsqueeze(0), vp.float().unsqueeze(0)
    xs = synthetic.hidden_stream(meta["gqa_steps"], meta["gqa_input_seed"])
    res = []
    for t in range(meta["gqa_steps"]):
        r, kc, vc = O.gqa_step(w, xs[t], kc, vc, meta["gqa_prefix"] + t)
        res.append(r.reshape(-1))
    ref_res = torch.from_numpy(golden["gqa_residual"])
    assert O.rel_rms(torch.stack(res), ref_res) < 1e-6
    p = meta["gqa_prefix"]
    assert O.max_abs(kc[0, :, p:], torch.from_numpy(golden["gqa_k_new"])) < 1e-5
    assert O.max_abs(vc[0, :, p:], torch.from_numpy(golden["gqa_v_new"])) < 1e-6


def test_kernel_boundary_oracle_equals_layer_oracle():
    """deltanet_kernel_ref (projection outputs in) reproduces deltanet_step's
    state when fed the same fp32 projection outputs."""
    w = synthetic.layer_weights(0, 0)
    x = synthetic.hidden_stream(1, 5)[0]
    h = O.rmsnorm(x, w["input_layernorm.weight"])
    mixed = torch.nn.functional.linear(h, w["linear_attn.in_proj_qkv.weight"].float())
    z = torch.nn.functional.linear(h, w["linear_attn.in_proj_z.weight"].float())
    a = torch.nn.functional.linear(h, w["linear_attn.in_proj_a.weight"].float())
    b = torch.nn.functional.linear(h, w["linear_attn.in_proj_b.weight"].float())
    conv0 = torch.zeros(1, O.CONV_DIM, 4, dtype=torch.bfloat16)
    rec0 = torch.zeros(1, O.NV, O.DH, O.DH)
    _, conv1, rec1 = O.deltanet_step(w, x, conv0, rec0)
    gated, conv2, rec2 = O.deltanet_kernel_ref(mixed, z, b, a, w, conv0, rec0)
    assert torch.equal(conv1, conv2)
    assert O.rel_rms(rec2, rec1) < 1e-6


def test_moe_step_matches_reference():
    """The MoE block (router, routed experts, shared expert) against
    router-ia's own batched_moe_step (tests/golden/make_golden_moe.py)."""
    import json
    from pathlib import Path

    import numpy as np

    g = np.load(Path(__file__).resolve().parent / "golden" / "reference_moe.npz")
    meta = json.loads(str(g["meta"]))
    w = synthetic.moe_weights(meta["weight_seed"], num_experts=meta["num_experts"])
    xs = synthetic.hidden_stream(meta["tokens"], meta["input_seed"])
    out, ids, wts, sg = O.moe_step(w, xs.reshape(meta["tokens"], -1).float(), meta["top_k"])
    assert torch.equal(ids, torch.from_numpy(g["ids"]))
    assert O.max_abs(wts, torch.from_numpy(g["weights"])) < 1e-6
    assert O.max_abs(sg, torch.from_numpy(g["shared_gate"])) < 1e-6
    ref = torch.from_numpy(g["out"])
    x0 = xs.reshape(meta["tokens"], -1).float()
    assert O.rel_rms(out - x0, ref - x0) < 1e-5  # the MoE contribution
    assert O.max_abs(out, ref) < 1e-5


def test_greedy_head_matches_reference():
    """Final norm, lm_head and greedy pick against router-ia's own functions
    (tests/golden/make_golden_head.py)."""
    import json
    from pathlib import Path

    import numpy as np

    g = np.load(Path(__file__).resolve().parent / "golden" / "reference_head.npz")
    meta = json.loads(str(g["meta"]))
    w = synthetic.head_weights(meta["weight_seed"], vocab=meta["vocab"])
    xs = synthetic.hidden_stream(meta["tokens"], meta["input_seed"]).reshape(meta["tokens"], -1) * meta["input_scale"]
    logits, ids = O.lm_head_greedy(xs, w["model.language_model.norm.weight"], w["lm_head.weight"], fp16=False)
    assert torch.equal(ids, torch.from_numpy(g["ids"]))
    assert O.rel_rms(logits, torch.from_numpy(g["logits"])) < 1e-6
    # the CUDA path's fp16 rounding moves logits by at most a few fp16 steps
    l16, ids16 = O.lm_head_greedy(xs, w["model.language_model.norm.weight"], w["lm_head.weight"], fp16=True)
    assert O.max_abs(l16, torch.from_numpy(g["logits"])) < 1e-2
