"""CPU oracle for router-ia's stateful attention path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this module; only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use
it, as the checker.  It restates, in plain torch CPU code, the arithmetic of:

* ``rmsnorm``              router-ia v2/src/router_ia/qwen36_op_probe.py:55-67
* ``gated_rmsnorm``        v2/src/router_ia/qwen36_gated_norm_probe.py:19-36
* ``_l2norm``              v2/src/router_ia/qwen36_attention_cache.py:169-173
* ``_rope``/``_apply_rope``  qwen36_attention_cache.py:137-162
* ``_causal_conv1d_step``  qwen36_attention_cache.py:176-221
* ``_linear_stateful``     qwen36_attention_cache.py:224-282 (CPU path: fp32
  projections, conv in the conv weight dtype)
* ``_full_stateful``       qwen36_attention_cache.py:285-324 (CPU path: fp32)
* ``route``                v2/src/router_ia/qwen36_router.py:96-133 and the
  MoE block ``batched_moe_step`` qwen36_chat_batch.py:127-178 (CPU path: fp32
  router, experts, shared expert and its sigmoid gate)
* the greedy head: final ``rmsnorm``, ``F.linear(x, lm_head)`` and
  ``sample_next`` at temperature <= 0, qwen36_chat_batch.py:194-199 and
  qwen36_mini_chat.py:75-78 (CPU path fp32; CUDA path fp16 autocast)
* the gated delta rule, recurrent and chunked (C=64, WY/UT), as in
  transformers 5.5.0 ``models/qwen3_5_moe/modeling_qwen3_5_moe.py``
  ``torch_recurrent_gated_delta_rule`` (:315-354) and
  ``torch_chunk_gated_delta_rule`` (:235-312), which router-ia calls from
  qwen36_linear_attention_hf.py:91-137.

Parity pin: the layer steps are checked against outputs of the reference
itself (tests/golden/make_golden.py imports router-ia from a checkout and
records them; tests/test_oracle_golden.py compares).  The chunked rule is
pinned against the recurrent rule it must equal (the reference ships no
golden vectors for it).

Weights are dicts ``{suffix: tensor}`` with the checkpoint's tensor-name
suffixes and dtypes (bf16 projections / norms / conv, fp32 A_log / dt_bias).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

HIDDEN = 2048
EPS = 1e-6
NK, NV, DH = 16, 32, 128
KEY_DIM, VAL_DIM = NK * DH, NV * DH
CONV_DIM = 2 * KEY_DIM + VAL_DIM
CONV_K = 4
HQ, HKV, D = 16, 2, 256
GROUPS = HQ // HKV
ROPE_THETA = 10_000_000.0
ROPE_DIM = 64


def rmsnorm(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """fp32 RMSNorm with the (1 + w) weight, cast back to the input dtype."""
    input_dtype = x.dtype
    x32 = x.float()
    out = x32 * torch.rsqrt(x32.pow(2).mean(dim=-1, keepdim=True) + EPS)
    out = out * (1.0 + weight.float())
    return out.to(dtype=input_dtype)


def gated_rmsnorm(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """RMSNormGated: normalise in fp32, cast to the input dtype, times w, times silu(z)."""
    input_dtype = x.dtype
    x32 = x.float()
    var = x32.pow(2).mean(dim=-1, keepdim=True)
    normalized = (x32 * torch.rsqrt(var + EPS)).to(input_dtype)
    weighted = weight.reshape(1, 1, -1) * normalized
    return (weighted * F.silu(z.float())).to(input_dtype)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    x = x.float()
    return x * torch.rsqrt((x * x).sum(dim=-1, keepdim=True) + eps)


def rope_tables(position: int, dtype=torch.float32) -> tuple[torch.Tensor, torch.Tensor]:
    inv_freq = 1.0 / (ROPE_THETA ** (torch.arange(0, ROPE_DIM, 2, dtype=torch.float32) / ROPE_DIM))
    angles = float(position) * inv_freq
    emb = torch.cat((angles, angles), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rope(x: torch.Tensor, position: int) -> torch.Tensor:
    """Rotate dims [0, 64) of the last axis of ``x`` (any leading shape)."""
    cos, sin = rope_tables(position, x.dtype)
    rot, rest = x[..., :ROPE_DIM], x[..., ROPE_DIM:]
    rot = rot * cos + _rotate_half(rot) * sin
    return torch.cat((rot, rest), dim=-1)


def conv1d_step(conv_state: torch.Tensor | None, mixed: torch.Tensor, conv_weight: torch.Tensor):
    """mixed (1, C) -> (silu(conv) (1, C) in mixed's dtype, new state (1, C, 4))."""
    channels = mixed.shape[-1]
    conv_dtype = conv_weight.dtype
    x = mixed.to(dtype=conv_dtype).reshape(1, channels, 1)
    if conv_state is None:
        conv_state = torch.zeros(1, channels, CONV_K, dtype=conv_dtype)
    history = torch.cat((conv_state.to(conv_dtype), x), dim=-1)
    new_state = history[:, :, -CONV_K:].clone()
    out = F.conv1d(history, conv_weight, bias=None, groups=channels)
    out = F.silu(out[:, :, -1:])
    return out[:, :, 0].to(dtype=mixed.dtype), new_state


def deltanet_gates(a: torch.Tensor, b: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor):
    beta = torch.sigmoid(b.float())
    g = -torch.exp(a_log.float()) * F.softplus(a.float() + dt_bias.float())
    return beta, g


def delta_rule_step(state: torch.Tensor, q, k, v, decay, beta):
    """One token of the gated delta rule on (B, H, 128, 128) ``state`` [k][v].
    q, k, v: (B, H, 128); decay, beta: (B, H).  Returns (o, state)."""
    state = state * decay[..., None, None]
    retrieved = (state * k.unsqueeze(-1)).sum(dim=-2)
    delta = (v - retrieved) * beta.unsqueeze(-1)
    state = state + k.unsqueeze(-1) * delta.unsqueeze(-2)
    o = (state * q.unsqueeze(-1)).sum(dim=-2)
    return o, state


def deltanet_step(w: dict, x0: torch.Tensor, conv_state, rec_state):
    """One Gated DeltaNet layer for one token on the reference's CPU path.
    Returns (residual (1, 2048) fp32, conv_state, rec_state)."""
    h = rmsnorm(x0.reshape(1, HIDDEN).float(), w["input_layernorm.weight"])
    mixed = F.linear(h, w["linear_attn.in_proj_qkv.weight"].float()).reshape(1, CONV_DIM)
    mixed, conv_state = conv1d_step(conv_state, mixed, w["linear_attn.conv1d.weight"])
    q, k, v = torch.split(mixed, [KEY_DIM, KEY_DIM, VAL_DIM], dim=-1)
    q = q.reshape(1, NK, DH).repeat_interleave(2, dim=1)
    k = k.reshape(1, NK, DH).repeat_interleave(2, dim=1)
    v = v.reshape(1, NV, DH)
    a = F.linear(h, w["linear_attn.in_proj_a.weight"].float()).reshape(1, NV)
    b = F.linear(h, w["linear_attn.in_proj_b.weight"].float()).reshape(1, NV)
    beta, g = deltanet_gates(a, b, w["linear_attn.A_log"].reshape(1, NV), w["linear_attn.dt_bias"].reshape(1, NV))
    q = l2norm(q) * (128 ** -0.5)
    k = l2norm(k)
    if rec_state is None:
        rec_state = torch.zeros(1, NV, DH, DH, dtype=torch.float32)
    o, rec_state = delta_rule_step(rec_state, q, k, v.float(), torch.exp(g), beta)
    z = F.linear(h, w["linear_attn.in_proj_z.weight"].float()).reshape(1, NV, DH)
    gated = gated_rmsnorm(o, z, w["linear_attn.norm.weight"])
    proj = F.linear(gated.reshape(1, VAL_DIM), w["linear_attn.out_proj.weight"].float())
    return x0.reshape(1, HIDDEN).float() + proj, conv_state, rec_state


def deltanet_kernel_ref(mixed, z, b, a, w: dict, conv_state, rec_state, dtype=torch.float32):
    """The K1 boundary: projection outputs of B sequences (bf16 values) ->
    (gated output (B, 4096) fp32 before the bf16 store, conv_state, rec_state).

    Same arithmetic as ``deltanet_step`` from the conv onward, batched, with the
    recurrence in ``dtype`` (fp32 as the reference, or fp64 for drift checks)."""
    B = mixed.shape[0]
    conv_w = w["linear_attn.conv1d.weight"]
    outs, states = [], []
    for i in range(B):
        y, st = conv1d_step(conv_state[i:i + 1], mixed[i:i + 1].float(), conv_w)
        outs.append(y)
        states.append(st)
    y = torch.cat(outs, 0)
    conv_state = torch.cat(states, 0)
    q, k, v = torch.split(y, [KEY_DIM, KEY_DIM, VAL_DIM], dim=-1)
    q = l2norm(q.reshape(B, NK, DH).repeat_interleave(2, dim=1)) * (128 ** -0.5)
    k = l2norm(k.reshape(B, NK, DH).repeat_interleave(2, dim=1))
    v = v.reshape(B, NV, DH).float()
    beta, g = deltanet_gates(a.float(), b.float(), w["linear_attn.A_log"].reshape(1, NV),
                             w["linear_attn.dt_bias"].reshape(1, NV))
    o, rec_state = delta_rule_step(rec_state.to(dtype), q.to(dtype), k.to(dtype), v.to(dtype),
                                   torch.exp(g.to(dtype)), beta.to(dtype))
    gated = gated_rmsnorm(o.float(), z.float().reshape(B, NV, DH), w["linear_attn.norm.weight"])
    return gated.reshape(B, VAL_DIM), conv_state, rec_state


def gqa_step(w: dict, x0: torch.Tensor, k_cache, v_cache, position: int):
    """One GQA layer for one token on the reference's CPU path (fp32).
    k_cache/v_cache: (1, 2, L, 256) fp32 or None.  Returns
    (residual (1, 2048), k_cache, v_cache)."""
    h = rmsnorm(x0.reshape(1, HIDDEN).float(), w["input_layernorm.weight"])
    q_gate = F.linear(h, w["self_attn.q_proj.weight"].float()).reshape(1, HQ, 2 * D)
    q, gate = torch.chunk(q_gate, 2, dim=-1)
    k = F.linear(h, w["self_attn.k_proj.weight"].float()).reshape(1, HKV, D)
    v = F.linear(h, w["self_attn.v_proj.weight"].float()).reshape(1, HKV, D)
    q = rmsnorm(q, w["self_attn.q_norm.weight"]).float().unsqueeze(2)
    k = rmsnorm(k, w["self_attn.k_norm.weight"]).float().unsqueeze(2)
    q = apply_rope(q, position)
    k = apply_rope(k, position)
    v = v.float().unsqueeze(2)
    k_cache = k if k_cache is None else torch.cat((k_cache, k), dim=2)
    v_cache = v if v_cache is None else torch.cat((v_cache, v), dim=2)
    attn = attend(q.squeeze(2), k_cache, v_cache)
    attn = attn * torch.sigmoid(gate.float())
    proj = F.linear(attn.reshape(1, HQ * D), w["self_attn.o_proj.weight"].float())
    return x0.reshape(1, HIDDEN).float() + proj, k_cache, v_cache


def attend(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor) -> torch.Tensor:
    """softmax(q K^T / 16) V with query head h reading KV head h // 8.
    q (B, 16, 256); caches (B, 2, L, 256).  Returns (B, 16, 256) fp32."""
    k_exp = k_cache.repeat_interleave(GROUPS, dim=1).float()
    v_exp = v_cache.repeat_interleave(GROUPS, dim=1).float()
    scores = torch.einsum("bhd,bhld->bhl", q.float(), k_exp) * (D ** -0.5)
    return torch.einsum("bhl,bhld->bhd", torch.softmax(scores, dim=-1), v_exp)


def gqa_kernel_ref(q_gate, k, v, w: dict, k_cache, v_cache, position: int):
    """The K3 boundary for one sequence: projection outputs (bf16 values) q_gate
    (16*512,), k (512,), v (512,) and a cache (2, L, 256) -> (gated attention
    output (4096,) fp32, k_new (2, 256), v_new (2, 256)).  q/k norm and RoPE
    are kept in fp32 (no intermediate rounding), like the kernel."""
    qg = q_gate.float().reshape(HQ, 2 * D)
    q, gate = qg[:, :D], qg[:, D:]
    q = rmsnorm(q, w["self_attn.q_norm.weight"].float())
    kk = rmsnorm(k.float().reshape(HKV, D), w["self_attn.k_norm.weight"].float())
    q = apply_rope(q, position)
    kk = apply_rope(kk, position)
    vv = v.float().reshape(HKV, D)
    kc = torch.cat((k_cache.float(), kk.unsqueeze(1)), dim=1)
    vc = torch.cat((v_cache.float(), vv.unsqueeze(1)), dim=1)
    out = attend(q.unsqueeze(0), kc.unsqueeze(0), vc.unsqueeze(0))[0]
    out = out * torch.sigmoid(gate)
    return out.reshape(HQ * D), kk, vv


def gqa_prefill_ref(q_gate, k, v, w: dict, k_cache, v_cache, pos0: int):
    """T prompt tokens of one sequence through the GQA boundary at once: the
    result of T consecutive ``gqa_kernel_ref`` steps (token t at position
    pos0 + t sees the cache and the new tokens 0..t).  q_gate (T, 16*512),
    k, v (T, 512) bf16 values; caches (2, L0, 256).  Returns (out (T, 4096)
    fp32, k_new (2, T, 256), v_new (2, T, 256))."""
    T = q_gate.shape[0]
    qg = q_gate.float().reshape(T, HQ, 2 * D)
    q, gate = qg[..., :D], qg[..., D:]
    q = rmsnorm(q, w["self_attn.q_norm.weight"].float())
    kk = rmsnorm(k.float().reshape(T, HKV, D), w["self_attn.k_norm.weight"].float())
    q = torch.stack([apply_rope(q[t], pos0 + t) for t in range(T)])
    kk = torch.stack([apply_rope(kk[t], pos0 + t) for t in range(T)])
    vv = v.float().reshape(T, HKV, D)
    kc = torch.cat((k_cache.float(), kk.transpose(0, 1)), dim=1)  # (2, L0 + T, 256)
    vc = torch.cat((v_cache.float(), vv.transpose(0, 1)), dim=1)
    L0 = k_cache.shape[1]
    k_exp = kc.repeat_interleave(GROUPS, dim=0)  # (16, L, 256)
    v_exp = vc.repeat_interleave(GROUPS, dim=0)
    scores = torch.einsum("thd,hld->thl", q, k_exp) * (D ** -0.5)
    keypos = torch.arange(L0 + T)
    allowed = keypos[None, :] <= (L0 + torch.arange(T))[:, None]  # (T, L)
    scores = scores.masked_fill(~allowed[:, None, :], float("-inf"))
    out = torch.einsum("thl,hld->thd", torch.softmax(scores, dim=-1), v_exp) * torch.sigmoid(gate)
    return out.reshape(T, HQ * D), kk.transpose(0, 1), vv.transpose(0, 1)


# --------------------------------------------------------------------------- gated delta rule (core)
def recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=None, dtype=torch.float32, l2=True):
    """Token-by-token rule. q, k (B, T, H, Dk); v (B, T, H, Dv); g, beta (B, T, H).
    Returns (out (B, T, H, Dv) float32, final state (B, H, Dk, Dv) ``dtype``)."""
    if l2:
        q, k = l2norm(q), l2norm(k)
    q, k, v, g, beta = [x.transpose(1, 2).contiguous().to(dtype) for x in (q, k, v, g, beta)]
    B, H, T, Dk = k.shape
    Dv = v.shape[-1]
    q = q * (Dk ** -0.5)
    state = torch.zeros(B, H, Dk, Dv, dtype=dtype) if initial_state is None else initial_state.to(dtype)
    out = torch.zeros(B, H, T, Dv, dtype=dtype)
    for t in range(T):
        o, state = delta_rule_step(state, q[:, :, t], k[:, :, t], v[:, :, t], g[:, :, t].exp(), beta[:, :, t])
        out[:, :, t] = o
    return out.transpose(1, 2).contiguous().float(), state


def chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=64, initial_state=None, l2=True):
    """Chunked (WY/UT) form of the same rule, in fp32, chunk size 64.
    Same arguments and results as ``recurrent_gated_delta_rule``."""
    if l2:
        q, k = l2norm(q), l2norm(k)
    q, k, v, beta, g = [x.transpose(1, 2).contiguous().float() for x in (q, k, v, beta, g)]
    B, H, T, Dk = k.shape
    Dv = v.shape[-1]
    C = chunk_size
    pad = (C - T % C) % C
    q, k, v = (F.pad(x, (0, 0, 0, pad)) for x in (q, k, v))
    beta, g = F.pad(beta, (0, pad)), F.pad(g, (0, pad))
    n = (T + pad) // C
    q = q * (Dk ** -0.5)
    kb = k * beta[..., None]
    vb = v * beta[..., None]
    q, k, v, kb, vb = (x.reshape(B, H, n, C, x.shape[-1]) for x in (q, k, v, kb, vb))
    g = g.reshape(B, H, n, C).cumsum(dim=-1)
    tri_incl = torch.triu(torch.ones(C, C, dtype=torch.bool), diagonal=0)
    decay = (g[..., :, None] - g[..., None, :]).tril().exp().tril()
    # A = (I + strictly-lower(diag(beta) K K^T * decay))^-1 by forward substitution
    a = -((kb @ k.transpose(-1, -2)) * decay).masked_fill(tri_incl, 0)
    for i in range(1, C):
        row = a[..., i, :i].clone()
        sub = a[..., :i, :i].clone()
        a[..., i, :i] = row + (row.unsqueeze(-1) * sub).sum(-2)
    a = a + torch.eye(C)
    u = a @ vb
    wk = a @ (kb * g.exp()[..., None])
    state = torch.zeros(B, H, Dk, Dv) if initial_state is None else initial_state.float().clone()
    out = torch.zeros_like(u)
    strict = torch.triu(torch.ones(C, C, dtype=torch.bool), diagonal=1)
    for i in range(n):
        qi, ki = q[:, :, i], k[:, :, i]
        attn = (qi @ ki.transpose(-1, -2) * decay[:, :, i]).masked_fill(strict, 0)
        v_new = u[:, :, i] - wk[:, :, i] @ state
        out[:, :, i] = (qi * g[:, :, i, :, None].exp()) @ state + attn @ v_new
        g_last = g[:, :, i, -1]
        state = state * g_last[..., None, None].exp() + (
            ki * (g_last[..., None] - g[:, :, i]).exp()[..., None]).transpose(-1, -2) @ v_new
    out = out.reshape(B, H, n * C, Dv)[:, :, :T]
    return out.transpose(1, 2).contiguous(), state


def route(hidden: torch.Tensor, gate_weight: torch.Tensor, top_k: int):
    """Router (qwen36_router.py:96-133): logits = hidden @ W^T in the gate
    weight's dtype (fp32 here), the top_k largest, softmax over them.
    hidden [T, H]; returns (ids [T, k] int64, weights [T, k] fp32)."""
    x = hidden.to(gate_weight.dtype)
    logits = torch.matmul(x, gate_weight.transpose(0, 1))
    values, ids = torch.topk(logits, k=top_k, dim=-1)
    return ids, torch.softmax(values, dim=-1).float()


def moe_step(w: dict, residual: torch.Tensor, top_k: int = 8):
    """One MoE block for T tokens, each as the reference's CPU path runs one
    token (qwen36_chat_batch.py:127-178): post-attention RMSNorm (1 + w),
    router, the top_k experts' SwiGLU FFNs weighted by the router weights, the
    shared expert times sigmoid(shared gate), and the residual add.  Weights
    are the checkpoint's (bf16) tensors, used in fp32 as the CPU path loads
    them.  residual [T, H] fp32; returns (out [T, H], ids [T, k], weights
    [T, k], shared_gate [T])."""
    moe_in = rmsnorm(residual.float(), w["post_attention_layernorm.weight"])
    ids, wts = route(moe_in, w["mlp.gate.weight"].float(), top_k)
    routed = torch.zeros_like(moe_in)
    for t in range(moe_in.shape[0]):
        x = moe_in[t]
        acc = torch.zeros_like(x)
        outs = []
        for j in range(top_k):
            e = int(ids[t, j])
            gate = w[f"mlp.experts.{e}.gate_proj.weight"].float() @ x
            up = w[f"mlp.experts.{e}.up_proj.weight"].float() @ x
            outs.append(w[f"mlp.experts.{e}.down_proj.weight"].float() @ (F.silu(gate) * up))
        acc = (torch.stack(outs) * wts[t].reshape(-1, 1)).sum(dim=0)
        routed[t] = acc
    sg = torch.sigmoid(F.linear(moe_in, w["mlp.shared_expert_gate.weight"].float()))  # [T, 1]
    sh = F.silu(F.linear(moe_in, w["mlp.shared_expert.gate_proj.weight"].float())) * F.linear(
        moe_in, w["mlp.shared_expert.up_proj.weight"].float())
    shared = F.linear(sh, w["mlp.shared_expert.down_proj.weight"].float()) * sg
    return residual.float() + (routed + shared), ids, wts, sg[:, 0]


def lm_head_greedy(x: torch.Tensor, final_norm: torch.Tensor, lm_head: torch.Tensor, fp16: bool = True):
    """The end of run_forward_token (qwen36_chat_batch.py:194-199) and
    sample_next with temperature <= 0 (qwen36_mini_chat.py:75-78): fp32
    RMSNorm with the (1 + w) weight, then logits = x . lm_head^T and the
    argmax (first index among equal maxima).  fp16=True is the CUDA path
    (fp16 autocast: both operands rounded to fp16, fp32 sums, fp16 logits);
    fp16=False the CPU path (fp32 throughout).  x [T, H]; returns (logits
    [T, V] fp32 holding the path's values, ids [T] int64)."""
    h = rmsnorm(x.float(), final_norm.float())
    if fp16:
        logits = (h.half().float() @ lm_head.half().float().T).half().float()
    else:
        logits = h @ lm_head.float().T
    return logits, torch.argmax(logits, dim=-1)


def rel_rms(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b||_2 / ||b||_2 in float64."""
    a64, b64 = a.double(), b.double()
    den = b64.norm().item()
    return (a64 - b64).norm().item() / (den if den > 0 else 1.0)


def max_abs(a: torch.Tensor, b: torch.Tensor) -> float:
    return (a.double() - b.double()).abs().max().item()


def max_err_bf16(a: torch.Tensor, b: torch.Tensor) -> float:
    """max |a - b| / max(1, |b|): absolute error for |b| <= 1 and relative
    error above, the scale-aware form of a max-abs bound for values that are
    stored in bf16 (whose rounding step grows with magnitude)."""
    a64, b64 = a.double(), b.double()
    return ((a64 - b64).abs() / b64.abs().clamp(min=1.0)).max().item()


def finite(x: torch.Tensor) -> bool:
    return bool(torch.isfinite(x).all())


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("math", "torch", "F", "annotations")]
