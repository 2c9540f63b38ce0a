"""The drop-in ``step_attention`` on the GPU against router-ia's own outputs
(golden fixtures) and against the CPU oracle on benchmark configuration 0
(64 prompt + 64 decode tokens, token by token) and configuration 1 (GQA decode
with 4096 cached tokens).  Tolerance: 2e-2 max-abs and 1e-2 relative RMS on the
fp32 residual (bf16 projections and KV against the reference's fp32 CPU path)."""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from router_ia import qwen36_attention_cache as cache

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_RMS = 1e-2


def _root(tmp_path: Path, layers: dict[int, dict]) -> Path:
    root = tmp_path / "ckpt"
    root.mkdir(exist_ok=True)
    for layer, w in layers.items():
        cache.register_layer_weights(root, layer, w)
    return root


def test_deltanet_steps_match_reference_golden(golden, tmp_path, cuda_device):
    meta = golden["meta"]
    layer = meta["dn_layer"]
    root = _root(tmp_path, {layer: synthetic.layer_weights(layer, meta["weight_seed"])})
    state = cache.state_for(root, "cuda")
    state.reset()
    cache.activate(root, state)
    xs = synthetic.hidden_stream(meta["dn_tokens"], meta["dn_input_seed"])
    res = []
    for t in range(meta["dn_tokens"]):
        res.append(cache.step_attention(root, layer, xs[t].to(cuda_device), "cuda").reshape(-1).cpu())
        state.tokens_seen += 1
    cache.deactivate(root)
    got = torch.stack(res)
    ref = torch.from_numpy(golden["dn_residual"])
    assert O.max_abs(got, ref) < MAX_ABS and O.rel_rms(got, ref) < REL_RMS
    # attention contribution alone (residual minus input) is also close
    contrib_err = O.rel_rms(got - xs[:, 0], ref - xs[:, 0])
    assert contrib_err < 5e-2, contrib_err
    rec = state.linear_states[layer][0].cpu()
    assert O.rel_rms(rec[meta["rec_heads"]], torch.from_numpy(golden["dn_rec_heads"])) < 2e-2
    conv = state.linear_conv_states[layer][0].cpu().float()
    conv_ref = torch.from_numpy(golden["dn_conv_state"])
    assert O.max_abs(conv, conv_ref) < 0.05
    snap = cache.stats(root)
    assert snap["linear_bytes"] == 32 * 128 * 128 * 4 and snap["linear_conv_bytes"] == 8192 * 4 * 2


def test_gqa_steps_match_reference_golden(golden, tmp_path, cuda_device):
    meta = golden["meta"]
    layer = meta["gqa_layer"]
    root = _root(tmp_path, {layer: synthetic.layer_weights(layer, meta["weight_seed"])})
    state = cache.state_for(root, "cuda")
    state.reset()
    cache.activate(root, state)
    kp, vp = synthetic.kv_prefix(meta["gqa_prefix"], meta["gqa_cache_seed"])
    # seed the cache the way a probe would; the module adopts it into pages
    state.full_keys[layer] = kp.unsqueeze(0).to(cuda_device)
    state.full_values[layer] = vp.unsqueeze(0).to(cuda_device)
    state.tokens_seen = meta["gqa_prefix"]
    xs = synthetic.hidden_stream(meta["gqa_steps"], meta["gqa_input_seed"])
    res = []
    for t in range(meta["gqa_steps"]):
        res.append(cache.step_attention(root, layer, xs[t].to(cuda_device), "cuda").reshape(-1).cpu())
        state.tokens_seen += 1
    cache.deactivate(root)
    got = torch.stack(res)
    ref = torch.from_numpy(golden["gqa_residual"])
    assert O.max_abs(got, ref) < MAX_ABS and O.rel_rms(got, ref) < REL_RMS
    p = meta["gqa_prefix"]
    k_new = state.full_keys[layer][0, :, p:].float().cpu()
    v_new = state.full_values[layer][0, :, p:].float().cpu()
    assert O.max_abs(k_new, torch.from_numpy(golden["gqa_k_new"])) < 0.1
    assert O.rel_rms(v_new, torch.from_numpy(golden["gqa_v_new"])) < 1e-2
    snap = state.snapshot()
    n = p + meta["gqa_steps"]
    assert snap["full_tokens_resident"] == n
    assert snap["full_bytes"] == 2 * 2 * n * 256 * 2  # bf16 K and V actually resident


def test_config0_prompt_then_decode_vs_oracle(tmp_path, cuda_device):
    layer = 0
    w = synthetic.layer_weights(layer, 1)
    root = _root(tmp_path, {layer: w})
    state = cache.state_for(root, "cuda")
    state.reset()
    cache.activate(root, state)
    xs = synthetic.hidden_stream(128, 21)
    conv = rec = None
    worst_abs = worst_rel = 0.0
    for t in range(128):  # 64 prompt tokens then 64 decode steps, token by token
        got = cache.step_attention(root, layer, xs[t].to(cuda_device), "cuda").cpu()
        ref, conv, rec = O.deltanet_step(w, xs[t], conv, rec)
        worst_abs = max(worst_abs, O.max_abs(got, ref))
        worst_rel = max(worst_rel, O.rel_rms(got, ref))
        state.tokens_seen += 1
    cache.deactivate(root)
    assert worst_abs < MAX_ABS and worst_rel < REL_RMS, (worst_abs, worst_rel)
    assert O.rel_rms(state.linear_states[layer].cpu(), rec) < 2e-2


def test_config1_gqa_decode_vs_oracle(tmp_path, cuda_device):
    layer = 3
    w = synthetic.layer_weights(layer, 1)
    root = _root(tmp_path, {layer: w})
    state = cache.state_for(root, "cuda")
    state.reset()
    cache.activate(root, state)
    kp, vp = synthetic.kv_prefix(4096, 22)
    state.full_keys[layer] = kp.unsqueeze(0).to(cuda_device)
    state.full_values[layer] = vp.unsqueeze(0).to(cuda_device)
    state.tokens_seen = 4096
    x = synthetic.hidden_stream(1, 23)[0]
    got = cache.step_attention(root, layer, x.to(cuda_device), "cuda").cpu()
    ref, _, _ = O.gqa_step(w, x, kp.float().unsqueeze(0), vp.float().unsqueeze(0), 4096)
    cache.deactivate(root)
    assert O.max_abs(got, ref) < MAX_ABS and O.rel_rms(got, ref) < REL_RMS
    assert state.full_keys[layer].shape == (1, 2, 4097, 256)


def test_limits_raise_before_kernel_mutates(tmp_path, cuda_device):
    layer = 3
    root = _root(tmp_path, {layer: synthetic.layer_weights(layer, 2)})
    state = cache.state_for(root, "cuda")
    state.reset()
    state.configure(max_context_tokens=2)
    cache.activate(root, state)
    xs = synthetic.hidden_stream(3, 24)
    for t in range(2):
        cache.step_attention(root, layer, xs[t].to(cuda_device), "cuda")
        state.tokens_seen += 1
    before = state.full_keys[layer].clone()
    with pytest.raises(RuntimeError, match="max_context_tokens=2"):
        cache.step_attention(root, layer, xs[2].to(cuda_device), "cuda")
    assert torch.equal(state.full_keys[layer], before)
    state.configure(max_context_tokens=0, max_full_kv_bytes=state.snapshot()["full_bytes"])
    with pytest.raises(RuntimeError, match="max_full_kv_bytes"):
        cache.step_attention(root, layer, xs[2].to(cuda_device), "cuda")
    state.configure()
    cache.deactivate(root)


def test_private_helpers_on_gpu(cuda_device):
    q = torch.randn(1, 16, 1, 256, device=cuda_device)
    k = torch.randn(1, 2, 1, 256, device=cuda_device)
    qr, kr = cache._apply_rope(q, k, 1234)
    assert O.max_abs(qr.cpu(), O.apply_rope(q.cpu(), 1234)) < 1e-5
    assert O.max_abs(kr.cpu(), O.apply_rope(k.cpu(), 1234)) < 1e-5
    assert torch.equal(qr[..., 64:], q[..., 64:])
    state = cache.AttentionState()
    w = synthetic.deltanet_weights(0)["linear_attn.conv1d.weight"]
    st_ref = None
    for t in range(6):
        mixed = torch.randn(1, 8192)
        got = cache._causal_conv1d_step(state, 0, mixed.to(cuda_device), w.to(cuda_device))
        ref, st_ref = O.conv1d_step(st_ref, mixed, w)
        assert O.max_abs(got.cpu(), ref) < 2e-2
    assert O.max_abs(state.linear_conv_states[0].float().cpu(), st_ref.float()) == 0.0
    assert _ext.device_error() == 0
