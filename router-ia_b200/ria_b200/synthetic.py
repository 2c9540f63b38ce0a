"""Seeded synthetic weights and inputs for the benchmark configurations.

There is no checkpoint or dataset on the build or benchmark machines, so every
tensor is generated on the CPU from a fixed seed (``torch.Generator``) with the
shapes and distributions the benchmark configurations name:

* projections ~ N(0, 0.02), stored bf16 like the checkpoint;
* conv1d weight ~ U(-0.5, 0.5) (torch's default bound 1/sqrt(4)), bf16;
* A_log ~ U(0, 2.7), dt_bias ~ U(-1, 1), fp32;
* norm weights: the ``(1 + w)`` RMSNorms (input, q, k) use w ~ N(0, 0.1) and the
  gated norm uses 1 + N(0, 0.1), so parity tests exercise every weight;
* activations ~ N(0, 1) rounded to bf16 (the benchmark's "bf16 activations").

Generating on the CPU keeps the values identical across machines with the same
torch build, which is what lets committed golden fixtures store only outputs.
"""

from __future__ import annotations

import torch

from . import constants as C


def _gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    return g


def _normal(g: torch.Generator, shape, std: float, mean: float = 0.0) -> torch.Tensor:
    return torch.randn(*shape, generator=g, dtype=torch.float32) * std + mean


def _uniform(g: torch.Generator, shape, lo: float, hi: float) -> torch.Tensor:
    return torch.rand(*shape, generator=g, dtype=torch.float32) * (hi - lo) + lo


def deltanet_weights(seed: int) -> dict[str, torch.Tensor]:
    """One Gated DeltaNet layer in checkpoint dtypes, keyed by the tensor-name
    suffixes the reference reads (qwen36_attention_cache.py:227-272)."""
    g = _gen(seed)
    bf = torch.bfloat16
    return {
        "input_layernorm.weight": _normal(g, (C.HIDDEN,), 0.1).to(bf),
        "linear_attn.in_proj_qkv.weight": _normal(g, (C.LINEAR_CONV_DIM, C.HIDDEN), 0.02).to(bf),
        "linear_attn.in_proj_z.weight": _normal(g, (C.LINEAR_VALUE_DIM, C.HIDDEN), 0.02).to(bf),
        "linear_attn.in_proj_b.weight": _normal(g, (C.LINEAR_NUM_V_HEADS, C.HIDDEN), 0.02).to(bf),
        "linear_attn.in_proj_a.weight": _normal(g, (C.LINEAR_NUM_V_HEADS, C.HIDDEN), 0.02).to(bf),
        "linear_attn.conv1d.weight": _uniform(g, (C.LINEAR_CONV_DIM, 1, C.LINEAR_CONV_KERNEL), -0.5, 0.5).to(bf),
        "linear_attn.A_log": _uniform(g, (C.LINEAR_NUM_V_HEADS,), 0.0, 2.7),
        "linear_attn.dt_bias": _uniform(g, (C.LINEAR_NUM_V_HEADS,), -1.0, 1.0),
        "linear_attn.norm.weight": _normal(g, (C.LINEAR_HEAD_DIM,), 0.1, 1.0).to(bf),
        "linear_attn.out_proj.weight": _normal(g, (C.HIDDEN, C.LINEAR_VALUE_DIM), 0.02).to(bf),
    }


def gqa_weights(seed: int) -> dict[str, torch.Tensor]:
    """One GQA full-attention layer in checkpoint dtypes."""
    g = _gen(seed)
    bf = torch.bfloat16
    return {
        "input_layernorm.weight": _normal(g, (C.HIDDEN,), 0.1).to(bf),
        "self_attn.q_proj.weight": _normal(g, (C.FULL_Q_GATE_DIM, C.HIDDEN), 0.02).to(bf),
        "self_attn.k_proj.weight": _normal(g, (C.FULL_KV_DIM, C.HIDDEN), 0.02).to(bf),
        "self_attn.v_proj.weight": _normal(g, (C.FULL_KV_DIM, C.HIDDEN), 0.02).to(bf),
        "self_attn.q_norm.weight": _normal(g, (C.FULL_HEAD_DIM,), 0.1).to(bf),
        "self_attn.k_norm.weight": _normal(g, (C.FULL_HEAD_DIM,), 0.1).to(bf),
        "self_attn.o_proj.weight": _normal(g, (C.HIDDEN, C.FULL_Q_DIM), 0.02).to(bf),
    }


MOE_EXPERTS = 256
MOE_TOP_K = 8
MOE_INTERMEDIATE = 512
SHARED_INTERMEDIATE = 512


def moe_weights(seed: int, num_experts: int = MOE_EXPERTS, device="cpu") -> dict[str, torch.Tensor]:
    """The MoE block of one decoder layer (router, routed experts, shared
    expert and its gate, post-attention norm) in checkpoint dtypes, keyed by
    the tensor-name suffixes the reference reads (qwen36_chat_batch.py:127-178):
    projections N(0, 0.02) bf16, norm weight N(0, 0.1) bf16 (the (1 + w) form)."""
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    bf = torch.bfloat16

    def nrm(shape, std):
        return (torch.randn(*shape, generator=g, device=device) * std).to(bf)

    out = {
        "post_attention_layernorm.weight": nrm((C.HIDDEN,), 0.1),
        "mlp.gate.weight": nrm((num_experts, C.HIDDEN), 0.02),
        "mlp.shared_expert_gate.weight": nrm((1, C.HIDDEN), 0.02),
        "mlp.shared_expert.gate_proj.weight": nrm((SHARED_INTERMEDIATE, C.HIDDEN), 0.02),
        "mlp.shared_expert.up_proj.weight": nrm((SHARED_INTERMEDIATE, C.HIDDEN), 0.02),
        "mlp.shared_expert.down_proj.weight": nrm((C.HIDDEN, SHARED_INTERMEDIATE), 0.02),
    }
    for e in range(num_experts):
        out[f"mlp.experts.{e}.gate_proj.weight"] = nrm((MOE_INTERMEDIATE, C.HIDDEN), 0.02)
        out[f"mlp.experts.{e}.up_proj.weight"] = nrm((MOE_INTERMEDIATE, C.HIDDEN), 0.02)
        out[f"mlp.experts.{e}.down_proj.weight"] = nrm((C.HIDDEN, MOE_INTERMEDIATE), 0.02)
    return out


def layer_weights(layer: int, seed: int = 0) -> dict[str, torch.Tensor]:
    """Weights of decoder layer ``layer`` of the 3:1 hybrid stack."""
    s = seed * 1000 + layer
    return gqa_weights(s) if C.is_full_attention_layer(layer) else deltanet_weights(s)


def layer_weights_on_device(layer: int, device, seed: int = 0) -> dict[str, torch.Tensor]:
    """Same shapes and distributions as ``layer_weights``, drawn directly on
    ``device`` (fast, for benchmarks; values differ from the CPU stream)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1000 + layer)
    bf = torch.bfloat16
    shapes = {
        "input_layernorm.weight": ((C.HIDDEN,), "n", 0.1, 0.0),
    }
    if C.is_full_attention_layer(layer):
        shapes.update({
            "self_attn.q_proj.weight": ((C.FULL_Q_GATE_DIM, C.HIDDEN), "n", 0.02, 0.0),
            "self_attn.k_proj.weight": ((C.FULL_KV_DIM, C.HIDDEN), "n", 0.02, 0.0),
            "self_attn.v_proj.weight": ((C.FULL_KV_DIM, C.HIDDEN), "n", 0.02, 0.0),
            "self_attn.q_norm.weight": ((C.FULL_HEAD_DIM,), "n", 0.1, 0.0),
            "self_attn.k_norm.weight": ((C.FULL_HEAD_DIM,), "n", 0.1, 0.0),
            "self_attn.o_proj.weight": ((C.HIDDEN, C.FULL_Q_DIM), "n", 0.02, 0.0),
        })
    else:
        shapes.update({
            "linear_attn.in_proj_qkv.weight": ((C.LINEAR_CONV_DIM, C.HIDDEN), "n", 0.02, 0.0),
            "linear_attn.in_proj_z.weight": ((C.LINEAR_VALUE_DIM, C.HIDDEN), "n", 0.02, 0.0),
            "linear_attn.in_proj_b.weight": ((C.LINEAR_NUM_V_HEADS, C.HIDDEN), "n", 0.02, 0.0),
            "linear_attn.in_proj_a.weight": ((C.LINEAR_NUM_V_HEADS, C.HIDDEN), "n", 0.02, 0.0),
            "linear_attn.conv1d.weight": ((C.LINEAR_CONV_DIM, 1, C.LINEAR_CONV_KERNEL), "u", -0.5, 0.5),
            "linear_attn.A_log": ((C.LINEAR_NUM_V_HEADS,), "u32", 0.0, 2.7),
            "linear_attn.dt_bias": ((C.LINEAR_NUM_V_HEADS,), "u32", -1.0, 1.0),
            "linear_attn.norm.weight": ((C.LINEAR_HEAD_DIM,), "n", 0.1, 1.0),
            "linear_attn.out_proj.weight": ((C.HIDDEN, C.LINEAR_VALUE_DIM), "n", 0.02, 0.0),
        })
    out = {}
    for name, (shape, kind, a, b) in shapes.items():
        if kind == "n":
            t = torch.randn(*shape, generator=g, device=device) * a + b
            out[name] = t.to(bf)
        else:
            t = torch.rand(*shape, generator=g, device=device) * (b - a) + a
            out[name] = t if kind == "u32" else t.to(bf)
    return out


def moe_layer_on_device(seed: int, device, num_experts: int = MOE_EXPERTS):
    """A ``MoeWeights`` with ``moe_weights``' shapes and distributions, drawn
    stacked directly on ``device`` (fast, for benchmarks; values differ from
    the per-expert CPU stream)."""
    from .weights import MoeWeights

    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    bf = torch.bfloat16

    def nrm(shape, std):
        return (torch.randn(*shape, generator=g, device=device) * std).to(bf)

    return MoeWeights(
        post_norm=nrm((C.HIDDEN,), 0.1), router=nrm((num_experts, C.HIDDEN), 0.02),
        shared_gate=nrm((C.HIDDEN,), 0.02),
        experts_gate=nrm((num_experts, MOE_INTERMEDIATE, C.HIDDEN), 0.02),
        experts_up=nrm((num_experts, MOE_INTERMEDIATE, C.HIDDEN), 0.02),
        experts_down=nrm((num_experts, C.HIDDEN, MOE_INTERMEDIATE), 0.02),
        shared_gate_proj=nrm((SHARED_INTERMEDIATE, C.HIDDEN), 0.02),
        shared_up_proj=nrm((SHARED_INTERMEDIATE, C.HIDDEN), 0.02),
        shared_down_proj=nrm((C.HIDDEN, SHARED_INTERMEDIATE), 0.02))


def head_weights(seed: int, vocab: int = C.VOCAB, device="cpu") -> dict[str, torch.Tensor]:
    """Embedding, final norm and lm_head in checkpoint dtypes (bf16), keyed
    by the names the reference looks up (qwen36_mini_chat.py:52-61,
    qwen36_op_probe.py:46-52): embedding and lm_head N(0, 0.02), final norm
    weight N(0, 0.1) (the (1 + w) form)."""
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    bf = torch.bfloat16
    return {
        "model.language_model.embed_tokens.weight": (torch.randn(vocab, C.HIDDEN, generator=g, device=device)
                                                     * 0.02).to(bf),
        "model.language_model.norm.weight": (torch.randn(C.HIDDEN, generator=g, device=device) * 0.1).to(bf),
        "lm_head.weight": (torch.randn(vocab, C.HIDDEN, generator=g, device=device) * 0.02).to(bf),
    }


def hidden_stream(n: int, seed: int, rows: int = 1) -> torch.Tensor:
    """``n`` steps of layer inputs, (n, rows, 2048) fp32 holding bf16 values."""
    g = _gen(seed)
    return torch.randn(n, rows, C.HIDDEN, generator=g, dtype=torch.float32).to(torch.bfloat16).float()


def kv_prefix(length: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    """A pre-filled GQA cache of ``length`` tokens, K and V ~ N(0,1) in bf16,
    laid out (kv_heads, length, head_dim)."""
    g = _gen(seed)
    k = torch.randn(C.FULL_NUM_KV_HEADS, length, C.FULL_HEAD_DIM, generator=g).to(torch.bfloat16)
    v = torch.randn(C.FULL_NUM_KV_HEADS, length, C.FULL_HEAD_DIM, generator=g).to(torch.bfloat16)
    return k, v


def ragged_lengths(batch: int, lo: int, hi: int, seed: int) -> list[int]:
    """Per-sequence KV lengths uniform in [lo, hi] (independent draws)."""
    g = _gen(seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (batch,), generator=g)]


def stratified_lengths(batch: int, lo: int, hi: int, seed: int) -> list[int]:
    """``batch`` KV lengths of U[lo, hi] as a stratified sample -- one length
    from each of ``batch`` equal-probability strata, at a seeded offset inside
    its stratum -- in seeded order.  Benchmark configuration 3 gives every GPU
    such a set, so the work per GPU is the same at any GPU count."""
    g = _gen(seed)
    u = (torch.arange(batch, dtype=torch.float64) + torch.rand(batch, generator=g, dtype=torch.float64)) / batch
    vals = [int(lo + x * (hi - lo + 1)) for x in u.tolist()]
    vals = [min(max(v, lo), hi) for v in vals]
    order = torch.randperm(batch, generator=g).tolist()
    return [vals[i] for i in order]


def config4_decode_model(device, batch: int = 64, prompt: int = 2048, extra_tokens: int = 32, seed: int = 4,
                         empty: bool = False):
    """Benchmark configuration 4's decode-phase state on one GPU: a
    ``model.DecodeModel`` of the random-init 40-layer stack (every layer with
    its own attention and 256-expert MoE weights, ~63 GB), ``batch``
    sequences each holding a ``prompt``-token cache (KV ~ N(0, 1), DeltaNet
    and conv states ~ N(0, 0.1)), page room for ``extra_tokens`` more, and
    random current token ids.  ``empty``: the sequences start with no context
    instead (page room for ``prompt + extra_tokens`` tokens), for a run that
    prefills the prompt itself."""
    from .model import DecodeModel, HeadWeights
    from .weights import DeltaNetWeights, GqaWeights

    attn, moe = {}, {}
    for layer in range(C.NUM_LAYERS):
        t = layer_weights_on_device(layer, device, seed=seed)
        attn[layer] = (GqaWeights if C.is_full_attention_layer(layer) else DeltaNetWeights).from_tensors(t, device)
        del t
        moe[layer] = moe_layer_on_device(seed * 1000 + layer, device)
    head = HeadWeights.from_tensors(head_weights(seed, device=device), device)
    per_seq = (prompt + extra_tokens + C.KV_BLOCK - 1) // C.KV_BLOCK + 1
    model = DecodeModel(attn, moe, head, batch, pool_blocks=batch * per_seq, max_blocks_per_seq=per_seq,
                        device=device)
    st = model.state
    g = torch.Generator(device=device)
    g.manual_seed(seed * 11)
    if empty:
        st.sync_tables()
        return model
    for layer in st.rec:
        st.rec[layer].normal_(0.0, 0.1, generator=g)
        st.conv[layer].normal_(0.0, 0.1, generator=g)
    for layer in st.k_pool:
        st.k_pool[layer].normal_(0.0, 1.0, generator=g)
        st.v_pool[layer].normal_(0.0, 1.0, generator=g)
    for i in range(batch):
        st.set_length(i, prompt)
    st.sync_tables()
    model.ids.copy_(torch.randint(0, head.vocab, (batch,), device=device, generator=g, dtype=torch.int32))
    return model

