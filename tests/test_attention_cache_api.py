"""The drop-in module keeps router-ia's public surface and bookkeeping
(v2/tests/test_qwen36_attention_cache.py semantics, snapshot keys, registry,
limits raised before mutation, no CPU compute path)."""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

from router_ia import qwen36_attention_cache as cache
from router_ia.qwen36_attention_cache import AttentionState, _append_full_kv

SNAPSHOT_KEYS = {
    "tokens_seen", "absolute_position", "kv_start_position", "full_layers_cached", "full_tokens",
    "full_tokens_resident", "full_token_entries", "full_bytes", "max_context_tokens", "max_full_kv_bytes",
    "linear_layers_cached", "linear_bytes", "linear_conv_layers_cached", "linear_conv_bytes", "bytes",
}


def _token():
    return torch.zeros((1, 1, 1, 2)), torch.zeros((1, 1, 1, 2))


def test_constants_match_reference():
    assert cache.ROPE_THETA == 10_000_000.0
    assert cache.ROPE_DIM == 64
    assert cache.LINEAR_CONV_KERNEL == 4
    assert cache.LINEAR_CONV_STATE == 4
    assert cache.LINEAR_CONV_DIM == 8192


def test_context_limit_raises_before_append():
    state = AttentionState(max_context_tokens=3)
    for pos in range(3):
        state.tokens_seen = pos
        _append_full_kv(state, 0, *_token())
        assert state.full_keys[0].shape[-2] <= 3
    state.tokens_seen = 3
    with pytest.raises(RuntimeError, match=r"max_context_tokens=3"):
        _append_full_kv(state, 0, *_token())
    snap = state.snapshot()
    assert state.full_keys[0].shape[-2] == 3
    assert snap["absolute_position"] == 3
    assert snap["full_tokens_resident"] == 3
    assert snap["kv_start_position"] == 0


def test_byte_budget_raises_before_append():
    key, value = _token()
    token_bytes = key.numel() * key.element_size() + value.numel() * value.element_size()
    state = AttentionState(max_full_kv_bytes=token_bytes * 2)
    for pos in range(2):
        state.tokens_seen = pos
        _append_full_kv(state, 0, key, value)
        assert state.snapshot()["full_bytes"] <= token_bytes * 2
    state.tokens_seen = 2
    with pytest.raises(RuntimeError, match=r"max_full_kv_bytes"):
        _append_full_kv(state, 0, key, value)
    assert state.full_keys[0].shape[-2] == 2
    assert state.snapshot()["full_bytes"] == token_bytes * 2


def test_snapshot_keys_and_accounting():
    state = AttentionState()
    assert set(state.snapshot()) == SNAPSHOT_KEYS
    state.linear_states[0] = torch.zeros(1, 32, 128, 128)
    state.linear_conv_states[0] = torch.zeros(1, 8192, 4, dtype=torch.bfloat16)
    state.full_keys[3] = torch.zeros(1, 2, 5, 256, dtype=torch.bfloat16)
    state.full_values[3] = torch.zeros(1, 2, 5, 256, dtype=torch.bfloat16)
    state.full_keys[7] = torch.zeros(1, 2, 4, 256, dtype=torch.bfloat16)
    state.full_values[7] = torch.zeros(1, 2, 4, 256, dtype=torch.bfloat16)
    state.tokens_seen = 9
    s = state.snapshot()
    assert s["linear_bytes"] == 32 * 128 * 128 * 4
    assert s["linear_conv_bytes"] == 8192 * 4 * 2
    assert s["full_bytes"] == 2 * (5 + 4) * 2 * 256 * 2
    assert s["full_tokens_resident"] == 5 and s["full_token_entries"] == 9
    assert s["kv_start_position"] == 4
    assert s["bytes"] == s["linear_bytes"] + s["linear_conv_bytes"] + s["full_bytes"]
    assert s["full_layers_cached"] == 2 and s["linear_layers_cached"] == 1


def test_configure_rejects_negative_limits():
    state = AttentionState()
    with pytest.raises(ValueError):
        state.configure(max_context_tokens=-1)
    with pytest.raises(ValueError):
        state.configure(max_full_kv_bytes=-1)
    state.configure(max_context_tokens=7, max_full_kv_bytes=9)
    assert (state.max_context_tokens, state.max_full_kv_bytes) == (7, 9)


def test_registry_reset_bind_activate(tmp_path: Path):
    root = tmp_path / "model"
    root.mkdir()
    st = cache.state_for(root, "cpu")
    assert cache.state_for(root, "cpu") is st
    st.tokens_seen = 5
    st.linear_states[0] = torch.zeros(1)
    assert cache.reset(root) is st and st.tokens_seen == 0 and not st.linear_states
    st.tokens_seen = 2
    st.bind("cpu")
    assert st.tokens_seen == 2
    st.bind("cuda:0")  # a device change drops everything
    assert st.tokens_seen == 0 and st.device == "cuda:0"
    cache.activate(root, st)
    assert cache.active(root, "cuda:0") is st
    cache.deactivate(root)
    assert cache.stats(tmp_path / "unknown")["bytes"] == 0
    assert set(cache.stats(root)) == SNAPSHOT_KEYS


def test_no_cpu_compute_path(tmp_path: Path):
    from ria_b200 import synthetic

    root = tmp_path / "m"
    cache.register_layer_weights(root, 0, synthetic.layer_weights(0, 0))
    st = cache.state_for(root, "cpu")
    cache.activate(root, st)
    with pytest.raises(RuntimeError, match="CUDA"):
        cache.step_attention(root, 0, torch.zeros(1, 2048), "cpu")
    cache.deactivate(root)


def test_attention_type_from_checkpoint(tmp_path: Path):
    from ria_b200 import synthetic
    from ria_b200.weights import CheckpointReader, write_checkpoint

    small_dn = {k: v for k, v in synthetic.layer_weights(0, 0).items() if "in_proj_qkv" in k}
    small_gqa = {k: v for k, v in synthetic.layer_weights(3, 0).items() if "q_proj" in k}
    write_checkpoint(tmp_path, {0: small_dn, 3: small_gqa})
    assert cache.attention_type(tmp_path, 0) == "linear_attention"
    assert cache.attention_type(tmp_path, 3) == "full_attention"
    with pytest.raises(KeyError):
        CheckpointReader(tmp_path).attention_type(5)


def test_conv_helper_validates_shapes():
    state = AttentionState()
    with pytest.raises(ValueError, match="mixed_qkv"):
        cache._causal_conv1d_step(state, 0, torch.zeros(1, 10), torch.zeros(8192, 1, 4))
    with pytest.raises(ValueError, match="conv weight"):
        cache._causal_conv1d_step(state, 0, torch.zeros(1, 8192), torch.zeros(8192, 4))


def test_rope_tables_match_reference_formula():
    cos, sin = cache._rope(17, torch.device("cpu"), torch.float32)
    inv = 1.0 / (1e7 ** (torch.arange(0, 64, 2, dtype=torch.float32) / 64))
    ang = 17.0 * inv
    assert torch.equal(cos, torch.cat((ang, ang)).cos())
    assert torch.equal(sin, torch.cat((ang, ang)).sin())
