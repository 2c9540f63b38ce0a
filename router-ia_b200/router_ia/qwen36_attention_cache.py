from __future__ import annotations

"""Persistent attention state for Qwen3.6 autoregressive decoding, on B200.

Drop-in replacement for router-ia's ``router_ia.qwen36_attention_cache``
(v2/src/router_ia/qwen36_attention_cache.py).  The public surface is the same:
constants, the ``AttentionState`` dataclass (fields, ``reset``/``bind``/
``configure``/``snapshot``), the per-checkpoint registry (``state_for``,
``reset``, ``activate``, ``deactivate``, ``active``), ``step_attention``,
``stats``, ``_append_full_kv`` and the private helpers probes use.  What
changed is underneath:

* the layer math runs in hand-written sm_100a kernels behind a C ABI
  (``ria_b200._ext``); there is no CPU path -- a non-CUDA device raises;
* DeltaNet state tensors are updated in place (one read and one write of the
  fp32 state per token) instead of being replaced by new tensors;
* the full-attention KV cache is bf16 in 64-token blocks with amortised
  growth instead of an fp32 ``torch.cat`` per token.  ``full_keys[layer]`` and
  ``full_values[layer]`` are views of shape (1, 2, L, 256) on that storage, so
  ``snapshot()`` reports the bytes actually resident (bf16) and the
  ``max_full_kv_bytes`` budget counts bf16 bytes.
"""

import sys
from dataclasses import dataclass, field
from pathlib import Path

import torch

_SRC_ROOT = Path(__file__).resolve().parents[1]
if str(_SRC_ROOT) not in sys.path:
    sys.path.insert(0, str(_SRC_ROOT))

from ria_b200 import _ext  # noqa: E402
from ria_b200 import constants as _C  # noqa: E402
from ria_b200.weights import CheckpointReader, DeltaNetWeights, GqaWeights, rope_inv_freq  # noqa: E402

ROPE_THETA = 10_000_000.0
ROPE_DIM = int(_C.FULL_HEAD_DIM * 0.25)
LINEAR_CONV_KERNEL = 4
# The rolling conv buffer keeps all four kernel positions; the current token
# is the last one after each update (Transformers' DynamicCache layout).
LINEAR_CONV_STATE = LINEAR_CONV_KERNEL
LINEAR_CONV_DIM = _C.LINEAR_KEY_DIM * 2 + _C.LINEAR_VALUE_DIM

# bf16 K and V of one token of one full-attention layer.
_KV_TOKEN_BYTES = 2 * _C.FULL_NUM_KV_HEADS * _C.FULL_HEAD_DIM * 2


class _PagedKV:
    """Single-sequence paged KV storage of one full-attention layer.

    K and V are [2, capacity, 256] bf16; blocks are 64 tokens and the block
    table is the identity, so the first L tokens are a plain strided view."""

    def __init__(self, device: torch.device, capacity_tokens: int = 256):
        self.device = device
        self.length = 0
        self.k = self.v = self.table = None
        self._alloc(max(_C.KV_BLOCK, capacity_tokens))

    def _alloc(self, capacity: int) -> None:
        capacity = ((capacity + _C.KV_BLOCK - 1) // _C.KV_BLOCK) * _C.KV_BLOCK
        shape = (_C.FULL_NUM_KV_HEADS, capacity, _C.FULL_HEAD_DIM)
        k = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        v = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        if self.k is not None and self.length:
            k[:, : self.length].copy_(self.k[:, : self.length])
            v[:, : self.length].copy_(self.v[:, : self.length])
        self.k, self.v = k, v
        self.table = torch.arange(capacity // _C.KV_BLOCK, dtype=torch.int32, device=self.device).reshape(1, -1)

    @property
    def capacity(self) -> int:
        return int(self.k.shape[1])

    def ensure(self, tokens: int) -> None:
        if tokens > self.capacity:
            cap = self.capacity
            while cap < tokens:
                cap *= 2
            self._alloc(cap)

    def views(self) -> tuple[torch.Tensor, torch.Tensor]:
        n = self.length
        return self.k[:, :n].unsqueeze(0), self.v[:, :n].unsqueeze(0)

    @classmethod
    def from_tensors(cls, keys: torch.Tensor, values: torch.Tensor, device: torch.device) -> "_PagedKV":
        """Adopt a (1, 2, L, 256) cache written by other code (any dtype)."""
        n = int(keys.shape[-2])
        kv = cls(device, capacity_tokens=max(256, 2 * n))
        kv.k[:, :n].copy_(keys.reshape(_C.FULL_NUM_KV_HEADS, n, _C.FULL_HEAD_DIM))
        kv.v[:, :n].copy_(values.reshape(_C.FULL_NUM_KV_HEADS, n, _C.FULL_HEAD_DIM))
        kv.length = n
        return kv


@dataclass
class AttentionState:
    full_keys: dict[int, torch.Tensor] = field(default_factory=dict)
    full_values: dict[int, torch.Tensor] = field(default_factory=dict)
    linear_states: dict[int, torch.Tensor] = field(default_factory=dict)
    linear_conv_states: dict[int, torch.Tensor] = field(default_factory=dict)
    # A value of zero disables the corresponding limit.  Limits fail before a
    # token is added; there is no sliding-window mode.
    max_context_tokens: int = 0
    max_full_kv_bytes: int = 0
    tokens_seen: int = 0
    device: str | None = None
    _paged: dict[int, _PagedKV] = field(default_factory=dict, repr=False, compare=False)

    def reset(self) -> None:
        self.full_keys.clear()
        self.full_values.clear()
        self.linear_states.clear()
        self.linear_conv_states.clear()
        self._paged.clear()
        self.tokens_seen = 0

    def bind(self, device: str) -> None:
        if self.device != device:
            self.reset()
            self.device = device

    def configure(self, *, max_context_tokens: int = 0, max_full_kv_bytes: int = 0) -> None:
        if max_context_tokens < 0:
            raise ValueError("max_context_tokens must be non-negative")
        if max_full_kv_bytes < 0:
            raise ValueError("max_full_kv_bytes must be non-negative")
        self.max_context_tokens = int(max_context_tokens)
        self.max_full_kv_bytes = int(max_full_kv_bytes)

    def snapshot(self) -> dict[str, int | float]:
        # KV layout is (batch, kv_heads, sequence, head_dim): length at dim -2.
        full_lengths = [int(value.shape[-2]) for value in self.full_keys.values()]
        full_tokens_resident = max(full_lengths, default=0)
        full_token_entries = sum(full_lengths)
        linear_bytes = sum(int(v.numel() * v.element_size()) for v in self.linear_states.values())
        conv_bytes = sum(int(v.numel() * v.element_size()) for v in self.linear_conv_states.values())
        full_bytes = _full_kv_bytes(self)
        return {
            "tokens_seen": int(self.tokens_seen),
            "absolute_position": int(self.tokens_seen),
            "kv_start_position": max(int(self.tokens_seen) - full_tokens_resident, 0),
            "full_layers_cached": len(self.full_keys),
            "full_tokens": full_tokens_resident,
            "full_tokens_resident": full_tokens_resident,
            "full_token_entries": full_token_entries,
            "full_bytes": full_bytes,
            "max_context_tokens": int(self.max_context_tokens),
            "max_full_kv_bytes": int(self.max_full_kv_bytes),
            "linear_layers_cached": len(self.linear_states),
            "linear_bytes": linear_bytes,
            "linear_conv_layers_cached": len(self.linear_conv_states),
            "linear_conv_bytes": conv_bytes,
            "bytes": full_bytes + linear_bytes + conv_bytes,
        }


_STATES: dict[Path, AttentionState] = {}
_ACTIVE_STATES: dict[Path, AttentionState] = {}
_ROOT_KEYS: dict = {}


def _rkey(root) -> Path:
    """``Path(root).resolve()``, the registry key, memoised per root object:
    resolving touches the filesystem (about 15 us), and step_attention needs
    the key three times per layer.  A root's resolution is fixed for the life
    of the process."""
    try:
        return _ROOT_KEYS[root]
    except (KeyError, TypeError):
        key = Path(root).resolve()
        try:
            _ROOT_KEYS[root] = key
        except TypeError:
            pass
        return key


def state_for(root: Path, device: str) -> AttentionState:
    key = _rkey(root)
    state = _STATES.get(key)
    if state is None:
        state = AttentionState()
        _STATES[key] = state
    state.bind(device)
    return state


def reset(root: Path) -> AttentionState:
    key = _rkey(root)
    state = _STATES.get(key)
    if state is None:
        state = AttentionState()
        _STATES[key] = state
    state.reset()
    return state


def activate(root: Path, state: AttentionState) -> None:
    _ACTIVE_STATES[_rkey(root)] = state


def deactivate(root: Path) -> None:
    _ACTIVE_STATES.pop(_rkey(root), None)


def active(root: Path, device: str) -> AttentionState:
    key = _rkey(root)
    state = _ACTIVE_STATES.get(key)
    if state is None:
        state = state_for(key, device)
        _ACTIVE_STATES[key] = state
    state.bind(device)
    return state


# --------------------------------------------------------------------------- weights
_REGISTERED: dict[tuple[Path, int], dict[str, torch.Tensor]] = {}
_READERS: dict[Path, CheckpointReader] = {}
_DEVICE_WEIGHTS: dict[tuple[Path, int, str], DeltaNetWeights | GqaWeights] = {}
# The same layers' weight arguments for the one-call layer steps (device
# pointers and strides): one foreign call per layer instead of three or four
# -- router-ia calls step_attention once per layer, and the host work of the
# separate calls exceeded a batch-1 layer's GPU time.
_LAYER_ARGS: dict[tuple[Path, int, str], tuple] = {}
_KINDS: dict[tuple[Path, int], str] = {}
_INV_FREQ: dict[str, torch.Tensor] = {}


def register_layer_weights(root: Path, layer: int, tensors: dict[str, torch.Tensor]) -> None:
    """Provide one layer's tensors (``{suffix: tensor}`` as in the checkpoint)
    without a checkpoint on disk, e.g. seeded synthetic weights."""
    key = (_rkey(root), int(layer))
    _REGISTERED[key] = dict(tensors)
    _KINDS.pop(key, None)
    for dkey in [k for k in _DEVICE_WEIGHTS if k[:2] == key]:
        del _DEVICE_WEIGHTS[dkey]
        _LAYER_ARGS.pop(dkey, None)


def _reader(root: Path) -> CheckpointReader:
    key = _rkey(root)
    reader = _READERS.get(key)
    if reader is None:
        reader = CheckpointReader(key)
        _READERS[key] = reader
    return reader


def attention_type(root: Path, layer: int) -> str:
    """``linear_attention`` or ``full_attention``, memoised per (root, layer)
    (qwen36_40layer_loop.py:68-78)."""
    key = (_rkey(root), int(layer))
    kind = _KINDS.get(key)
    if kind is None:
        tensors = _REGISTERED.get(key)
        if tensors is not None:
            if "linear_attn.in_proj_qkv.weight" in tensors:
                kind = "linear_attention"
            elif "self_attn.q_proj.weight" in tensors:
                kind = "full_attention"
            else:
                raise KeyError(f"Could not identify attention type for layer {layer}")
        else:
            kind = _reader(key[0]).attention_type(layer)
        _KINDS[key] = kind
    return kind


def _device_weights(root: Path, layer: int, device) -> DeltaNetWeights | GqaWeights:
    return _device_layer(root, layer, device)[0]


def _device_layer(root: Path, layer: int, device) -> tuple:
    """(weights, weight arguments of the one-call layer step) of one layer on
    ``device``, converted once and cached until the layer is re-registered."""
    rkey = _rkey(root)
    dev = torch.device(device)
    key = (rkey, int(layer), str(dev))
    w = _DEVICE_WEIGHTS.get(key)
    if w is None:
        kind = attention_type(rkey, layer)
        names = _C.DN_WEIGHT_NAMES if kind == "linear_attention" else _C.GQA_WEIGHT_NAMES
        tensors = _REGISTERED.get((rkey, int(layer)))
        if tensors is None:
            tensors = _reader(rkey).layer_tensors(layer, names)
        cls = DeltaNetWeights if kind == "linear_attention" else GqaWeights
        w = cls.from_tensors(tensors, dev)
        _DEVICE_WEIGHTS[key] = w
        _LAYER_ARGS[key] = _ext.deltanet_layer_args(w) if cls is DeltaNetWeights else _ext.gqa_layer_args(w)
    return w, _LAYER_ARGS[key]


def _projection(root: Path, prefix: str, device: str) -> torch.Tensor:
    """Projection weight ``prefix + '.weight'`` as a bf16 device tensor."""
    rkey = _rkey(root)
    name = prefix + ".weight"
    for (r, layer), tensors in _REGISTERED.items():
        lp = _C.layer_prefix(layer)
        if r == rkey and name.startswith(lp) and name[len(lp):] in tensors:
            return tensors[name[len(lp):]].to(device=device, dtype=torch.bfloat16)
    layer_tail = name.split("model.language_model.layers.", 1)[-1]
    layer = int(layer_tail.split(".", 1)[0])
    return _reader(rkey).layer_tensors(layer, [name[len(_C.layer_prefix(layer)):]])[
        name[len(_C.layer_prefix(layer)):]].to(device=device, dtype=torch.bfloat16)


def _cuda_device(device) -> torch.device:
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError(f"router-ia B200 attention runs on CUDA devices only (got {device!r}); no CPU path")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


def _inv_freq(device: torch.device) -> torch.Tensor:
    t = _INV_FREQ.get(str(device))
    if t is None:
        t = rope_inv_freq(device)
        _INV_FREQ[str(device)] = t
    return t


# --------------------------------------------------------------------------- RoPE helpers
def _rope(position: int, device: torch.device, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables of the partial RoPE at ``position`` (reference :137-146)."""
    if ROPE_DIM <= 0 or ROPE_DIM % 2:
        raise ValueError(f"Invalid rotary dimension: {ROPE_DIM}")
    inv_freq = 1.0 / (ROPE_THETA ** (torch.arange(0, ROPE_DIM, 2, device=device, dtype=torch.float32) / ROPE_DIM))
    angles = float(position) * inv_freq
    emb = torch.cat((angles, angles), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _apply_rope(q: torch.Tensor, k: torch.Tensor, position: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Rotate dims [0, ROPE_DIM) of q and k at ``position`` (reference
    :154-162) with the RoPE kernel; returns new tensors of the input dtype."""
    dev = _cuda_device(q.device)
    inv = _inv_freq(dev)
    outs = []
    for t in (q, k):
        rows = t.detach().to(device=dev, dtype=torch.float32).reshape(-1, t.shape[-1]).clone()
        _ext.rope_apply(rows, inv, ROPE_DIM, int(position))
        outs.append(rows.reshape(t.shape).to(dtype=t.dtype))
    return outs[0], outs[1]


# --------------------------------------------------------------------------- conv helper
def _causal_conv1d_step(
    state: AttentionState,
    layer: int,
    mixed_qkv: torch.Tensor,
    conv_weight: torch.Tensor,
) -> torch.Tensor:
    """One-token causal depthwise conv + SiLU with the rolling four-position
    state of ``layer`` (reference :176-221), on the conv kernel."""
    if mixed_qkv.ndim != 2 or mixed_qkv.shape != (1, LINEAR_CONV_DIM):
        raise ValueError(f"Unexpected mixed_qkv shape: {tuple(mixed_qkv.shape)}")
    if conv_weight.ndim != 3:
        raise ValueError(f"Unexpected conv weight shape: {tuple(conv_weight.shape)}")
    if (
        conv_weight.shape[0] != LINEAR_CONV_DIM
        or conv_weight.shape[1] != 1
        or conv_weight.shape[2] != LINEAR_CONV_KERNEL
    ):
        raise ValueError(f"Unexpected conv weight shape: {tuple(conv_weight.shape)}")
    dev = _cuda_device(mixed_qkv.device)
    conv_state = _conv_state(state, layer, dev)
    x = mixed_qkv.to(dtype=torch.bfloat16).contiguous()
    out = torch.empty(1, LINEAR_CONV_DIM, dtype=torch.bfloat16, device=dev)
    w = conv_weight.to(device=dev, dtype=torch.bfloat16).reshape(LINEAR_CONV_DIM, LINEAR_CONV_KERNEL).contiguous()
    _ext.conv1d_step(x, conv_state.reshape(1, LINEAR_CONV_DIM * LINEAR_CONV_STATE), w, out)
    return out.to(dtype=mixed_qkv.dtype)


def _conv_state(state: AttentionState, layer: int, dev: torch.device) -> torch.Tensor:
    expected = (1, LINEAR_CONV_DIM, LINEAR_CONV_STATE)
    conv = state.linear_conv_states.get(int(layer))
    if conv is None or conv.device != dev or tuple(conv.shape) != expected:
        conv = torch.zeros(expected, device=dev, dtype=torch.bfloat16)
    elif conv.dtype != torch.bfloat16 or not conv.is_contiguous():
        conv = conv.to(dtype=torch.bfloat16).contiguous()
    state.linear_conv_states[int(layer)] = conv
    return conv


def _linear_state(state: AttentionState, layer: int, dev: torch.device) -> torch.Tensor:
    expected = (1, _C.LINEAR_NUM_V_HEADS, _C.LINEAR_HEAD_DIM, _C.LINEAR_HEAD_DIM)
    rec = state.linear_states.get(int(layer))
    if rec is None or rec.device != dev or tuple(rec.shape) != expected:
        rec = torch.zeros(expected, device=dev, dtype=torch.float32)
    elif rec.dtype != torch.float32 or not rec.is_contiguous() or rec.data_ptr() % 16:
        rec = rec.to(dtype=torch.float32).contiguous()
    state.linear_states[int(layer)] = rec
    return rec


# --------------------------------------------------------------------------- layer steps
# Per device and stream, the scratch the one-call layer steps keep their
# intermediates in (grown on demand, never shared by concurrent streams).
_SCRATCH: dict = {}
_SCRATCH_OUTGROWN: list = []  # kept alive: work already queued may still use one


def _scratch(dev: torch.device, nbytes: int) -> torch.Tensor:
    key = (dev.index, torch._C._cuda_getCurrentRawStream(dev.index))
    buf = _SCRATCH.get(key)
    if buf is None or buf.numel() < nbytes:
        if buf is not None:
            _SCRATCH_OUTGROWN.append(buf)
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _SCRATCH[key] = buf
    return buf


def _linear_stateful(root: Path, layer: int, x0: torch.Tensor, device: str) -> torch.Tensor:
    """One Gated DeltaNet layer for one token: returns the residual (1, 2048)
    fp32 (reference :224-282), state updated in place."""
    state = active(root, device)
    dev = _cuda_device(device)
    _, wargs = _device_layer(root, layer, dev)
    x = x0.reshape(1, _C.HIDDEN).to(device=dev, dtype=torch.float32).contiguous()
    conv = _conv_state(state, layer, dev)
    rec = _linear_state(state, layer, dev)
    out = torch.empty(1, _C.HIDDEN, dtype=torch.float32, device=dev)
    _ext.deltanet_layer_decode(x, wargs, conv, rec, out, _scratch(dev, _ext.deltanet_layer_scratch_bytes(1)))
    return out


def _paged_kv(state: AttentionState, layer: int, dev: torch.device) -> _PagedKV:
    kv = state._paged.get(int(layer))
    keys = state.full_keys.get(int(layer))
    if kv is not None and kv.device == dev and keys is not None and int(keys.shape[-2]) == kv.length \
            and keys.data_ptr() == kv.k.data_ptr():
        return kv
    if keys is None:
        kv = _PagedKV(dev)
    else:  # adopt a cache that other code placed in full_keys/full_values
        kv = _PagedKV.from_tensors(keys.to(dev), state.full_values[int(layer)].to(dev), dev)
    state._paged[int(layer)] = kv
    return kv


def _check_full_kv_limits(state: AttentionState, resident_tokens: int, append_bytes: int) -> None:
    """Hard limits, raised before anything is appended (reference :344-363)."""
    if state.max_context_tokens and resident_tokens >= state.max_context_tokens:
        raise RuntimeError(
            "Full-attention KV context limit reached "
            f"at absolute position {state.tokens_seen}: "
            f"max_context_tokens={state.max_context_tokens}. "
            "This checkpoint runtime has no verified sliding-window policy; "
            "start a new context or raise --max-context-tokens."
        )
    projected_bytes = _full_kv_bytes(state) + append_bytes
    if state.max_full_kv_bytes and projected_bytes > state.max_full_kv_bytes:
        raise RuntimeError(
            "Full-attention KV byte budget reached "
            f"at absolute position {state.tokens_seen}: "
            f"projected={projected_bytes} bytes exceeds "
            f"max_full_kv_bytes={state.max_full_kv_bytes}. "
            "This checkpoint runtime has no verified sliding-window policy; "
            "start a new context or raise --max-full-kv-bytes."
        )


def _full_stateful(root: Path, layer: int, x0: torch.Tensor, device: str) -> torch.Tensor:
    """One GQA layer for one token at position ``tokens_seen``: returns the
    residual (1, 2048) fp32 (reference :285-324); K/V appended in-kernel."""
    state = active(root, device)
    dev = _cuda_device(device)
    position = int(state.tokens_seen)
    _, wargs = _device_layer(root, layer, dev)
    kv = _paged_kv(state, layer, dev)
    n = kv.length
    _check_full_kv_limits(state, n, _KV_TOKEN_BYTES)
    kv.ensure(n + 1)
    blocks = (n + 1 + _C.KV_BLOCK - 1) // _C.KV_BLOCK  # the split plan of plan_gqa_split for one sequence
    split_pages = _ext.gqa_split_pages(blocks, _C.FULL_NUM_KV_HEADS)
    max_splits = (blocks + split_pages - 1) // split_pages
    x = x0.reshape(1, _C.HIDDEN).to(device=dev, dtype=torch.float32).contiguous()
    out = torch.empty(1, _C.HIDDEN, dtype=torch.float32, device=dev)
    _ext.gqa_layer_decode(x, wargs, _inv_freq(dev), kv.k, kv.v, kv.table, out,
                          _scratch(dev, _ext.gqa_layer_scratch_bytes(1, max_splits)), split_pages, max_splits,
                          seq_len0=n, position0=position)
    kv.length = n + 1
    state.full_keys[int(layer)], state.full_values[int(layer)] = kv.views()
    return out


def _full_kv_bytes(state: AttentionState) -> int:
    return sum(
        int(tensor.numel() * tensor.element_size())
        for tensor in [*state.full_keys.values(), *state.full_values.values()]
    )


def _append_full_kv(
    state: AttentionState,
    layer: int,
    k_token: torch.Tensor,
    v_token: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Append one full-attention token after enforcing configured hard limits
    (reference :334-373).  On a layer backed by the paged cache the token is
    stored there (bf16); otherwise the layer's tensors are concatenated, which
    keeps the container semantics for caches built by other code."""
    full_k = state.full_keys.get(int(layer))
    full_v = state.full_values.get(int(layer))
    resident_tokens = int(full_k.shape[-2]) if full_k is not None else 0
    kv = state._paged.get(int(layer))
    paged = kv is not None and full_k is not None and full_k.data_ptr() == kv.k.data_ptr() and k_token.is_cuda
    if paged:
        append_bytes = _KV_TOKEN_BYTES
    else:
        append_bytes = int(k_token.numel() * k_token.element_size()) + int(v_token.numel() * v_token.element_size())
    _check_full_kv_limits(state, resident_tokens, append_bytes)
    if paged:
        n = kv.length
        kv.ensure(n + 1)
        row = _C.FULL_NUM_KV_HEADS * _C.FULL_HEAD_DIM
        dt = torch.float32 if k_token.dtype == torch.float32 else torch.bfloat16
        k_row = k_token.detach().to(device=kv.device, dtype=dt).reshape(1, row).contiguous()
        v_row = v_token.detach().to(device=kv.device, dtype=dt).reshape(1, row).contiguous()
        _ext.kv_append_paged(k_row, v_row, kv.k, kv.v, kv.table, seq_len0=n)
        kv.length = n + 1
        full_k, full_v = kv.views()
    elif full_k is None or full_v is None or full_k.device != k_token.device:
        full_k = k_token.detach()
        full_v = v_token.detach()
    else:
        full_k = torch.cat((full_k, k_token.detach()), dim=2)
        full_v = torch.cat((full_v, v_token.detach()), dim=2)
    state.full_keys[int(layer)] = full_k
    state.full_values[int(layer)] = full_v
    return full_k, full_v


def step_attention(root: Path, layer: int, x0: torch.Tensor, device: str) -> torch.Tensor:
    if attention_type(root, layer) == "linear_attention":
        return _linear_stateful(root, layer, x0, device)
    return _full_stateful(root, layer, x0, device)


def stats(root: Path) -> dict[str, int | float]:
    state = _STATES.get(_rkey(root))
    return (
        state.snapshot()
        if state is not None
        else {
            "tokens_seen": 0,
            "absolute_position": 0,
            "kv_start_position": 0,
            "full_layers_cached": 0,
            "full_tokens": 0,
            "full_tokens_resident": 0,
            "full_token_entries": 0,
            "full_bytes": 0,
            "max_context_tokens": 0,
            "max_full_kv_bytes": 0,
            "linear_layers_cached": 0,
            "linear_bytes": 0,
            "linear_conv_layers_cached": 0,
            "linear_conv_bytes": 0,
            "bytes": 0,
        }
    )
