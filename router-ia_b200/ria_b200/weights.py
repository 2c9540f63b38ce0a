"""Attention weights resident on the device, prepared once per layer.

The reference fetches every projection through a RAM/VRAM/SSD cache on each
call and re-casts it (qwen36_cached_loop.py:527-560).  A B200 keeps the 40
layers' attention weights resident (about 2.6 GB in bf16), so this module
loads them once, fuses each layer's input projections into one matrix (one
GEMM per layer instead of four / three) and converts the small vectors to fp32.

The fused in-projection is kept in fp16 (checkpoint bf16 values convert
exactly inside fp16's range), as router-ia's CUDA path keeps every projection
(qwen36_cached_loop.py:552-557), so that the normalised layer input can enter
it in fp16: a bf16 input (2^-9 rounding) moved single tokens' attention
output by up to ~2e-2 against the fp32 CPU path, an fp16 one by ~6e-3.  The
out-projections stay bf16 (their input, the attention output, is bf16).

Sources: a dict of checkpoint tensors (``{suffix: tensor}``) or a checkpoint
directory laid out like the reference expects (``model.safetensors.index.json``
or ``*.safetensors`` with names ``model.language_model.layers.{L}.<suffix>``);
FP8 projections with ``weight_scale_inv`` are dequantised with 128x128 blocks
(qwen36_op_probe.py dequantize_fp8_blockwise).
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import torch

from . import constants as C

FP8_BLOCK = 128


def _fp16_projection(parts: list[torch.Tensor]) -> torch.Tensor:
    """Row-concatenated projection matrices in fp16; raises if a weight lies
    outside fp16's range."""
    w = torch.cat([p.to(torch.float16) for p in parts], dim=0).contiguous()
    if not bool(torch.isfinite(w).all()):
        raise ValueError("projection weights exceed the fp16 range (|w| > 65504)")
    return w


@dataclass
class DeltaNetWeights:
    in_norm: torch.Tensor  # [2048] f32, the (1+w) RMSNorm weight
    w_in: torch.Tensor  # [12352, 2048] fp16 = [qkv | z | b | a]
    conv_w: torch.Tensor  # [8192, 4] bf16
    a_log: torch.Tensor  # [32] f32
    dt_bias: torch.Tensor  # [32] f32
    norm_w: torch.Tensor  # [128] f32 gated-norm weight
    w_out: torch.Tensor  # [2048, 4096] bf16
    conv_dtype: torch.dtype = torch.bfloat16

    @classmethod
    def from_tensors(cls, t: dict[str, torch.Tensor], device) -> "DeltaNetWeights":
        bf = torch.bfloat16
        w_in = _fp16_projection(
            [t["linear_attn.in_proj_qkv.weight"], t["linear_attn.in_proj_z.weight"], t["linear_attn.in_proj_b.weight"],
             t["linear_attn.in_proj_a.weight"]])
        conv = t["linear_attn.conv1d.weight"]
        if tuple(conv.shape) != (C.LINEAR_CONV_DIM, 1, C.LINEAR_CONV_KERNEL):
            raise ValueError(f"Unexpected conv weight shape: {tuple(conv.shape)}")
        return cls(
            in_norm=t["input_layernorm.weight"].float().contiguous().to(device),
            w_in=w_in.to(device),
            conv_w=conv.reshape(C.LINEAR_CONV_DIM, C.LINEAR_CONV_KERNEL).to(bf).contiguous().to(device),
            a_log=t["linear_attn.A_log"].float().reshape(C.LINEAR_NUM_V_HEADS).contiguous().to(device),
            dt_bias=t["linear_attn.dt_bias"].float().reshape(C.LINEAR_NUM_V_HEADS).contiguous().to(device),
            norm_w=t["linear_attn.norm.weight"].float().reshape(C.LINEAR_HEAD_DIM).contiguous().to(device),
            w_out=t["linear_attn.out_proj.weight"].to(bf).contiguous().to(device),
            conv_dtype=conv.dtype,
        )


@dataclass
class GqaWeights:
    in_norm: torch.Tensor  # [2048] f32
    w_in: torch.Tensor  # [9216, 2048] fp16 = [q_gate | k | v]
    q_norm: torch.Tensor  # [256] f32
    k_norm: torch.Tensor  # [256] f32
    w_out: torch.Tensor  # [2048, 4096] bf16

    @classmethod
    def from_tensors(cls, t: dict[str, torch.Tensor], device) -> "GqaWeights":
        bf = torch.bfloat16
        w_in = _fp16_projection([t["self_attn.q_proj.weight"], t["self_attn.k_proj.weight"],
                                 t["self_attn.v_proj.weight"]])
        return cls(
            in_norm=t["input_layernorm.weight"].float().contiguous().to(device),
            w_in=w_in.to(device),
            q_norm=t["self_attn.q_norm.weight"].float().reshape(C.FULL_HEAD_DIM).contiguous().to(device),
            k_norm=t["self_attn.k_norm.weight"].float().reshape(C.FULL_HEAD_DIM).contiguous().to(device),
            w_out=t["self_attn.o_proj.weight"].to(bf).contiguous().to(device),
        )


@dataclass
class MoeWeights:
    """The MoE block of one layer (qwen36_chat_batch.py:127-178), bf16 as in
    the checkpoint, with each expert's three projections stacked so that the
    kernels index an expert by offset."""

    post_norm: torch.Tensor  # [2048] bf16, the (1+w) RMSNorm weight
    router: torch.Tensor  # [E, 2048] bf16
    shared_gate: torch.Tensor  # [2048] bf16
    experts_gate: torch.Tensor  # [E, 512, 2048] bf16
    experts_up: torch.Tensor  # [E, 512, 2048] bf16
    experts_down: torch.Tensor  # [E, 2048, 512] bf16
    shared_gate_proj: torch.Tensor  # [512, 2048] bf16
    shared_up_proj: torch.Tensor  # [512, 2048] bf16
    shared_down_proj: torch.Tensor  # [2048, 512] bf16

    @property
    def num_experts(self) -> int:
        return self.router.shape[0]

    def __getitem__(self, key: str) -> torch.Tensor:
        return getattr(self, key)

    @classmethod
    def from_tensors(cls, t: dict[str, torch.Tensor], device) -> "MoeWeights":
        bf = torch.bfloat16
        num_experts = t["mlp.gate.weight"].shape[0]

        def stack(proj: str) -> torch.Tensor:
            first = t[f"mlp.experts.0.{proj}.weight"]
            out = torch.empty((num_experts, *first.shape), dtype=bf, device=device)
            for e in range(num_experts):
                out[e].copy_(t[f"mlp.experts.{e}.{proj}.weight"].to(bf))
            return out

        def dev(name: str) -> torch.Tensor:
            return t[name].to(bf).contiguous().to(device)

        return cls(
            post_norm=dev("post_attention_layernorm.weight"),
            router=dev("mlp.gate.weight"),
            shared_gate=dev("mlp.shared_expert_gate.weight").reshape(C.HIDDEN),
            experts_gate=stack("gate_proj"),
            experts_up=stack("up_proj"),
            experts_down=stack("down_proj"),
            shared_gate_proj=dev("mlp.shared_expert.gate_proj.weight"),
            shared_up_proj=dev("mlp.shared_expert.up_proj.weight"),
            shared_down_proj=dev("mlp.shared_expert.down_proj.weight"),
        )


def rope_inv_freq(device) -> torch.Tensor:
    """Inverse RoPE frequencies exactly as the reference computes them
    (qwen36_attention_cache.py:140-143): fp32 on the CPU, then moved."""
    inv = 1.0 / (C.ROPE_THETA ** (torch.arange(0, C.ROPE_DIM, 2, dtype=torch.float32) / C.ROPE_DIM))
    return inv.to(device)


def dequantize_fp8_blockwise(weight: torch.Tensor, scale_inv: torch.Tensor) -> torch.Tensor:
    """FP8 e4m3 weight times its per-128x128-block inverse scale, in fp32."""
    out_f, in_f = weight.shape
    rows = (out_f + FP8_BLOCK - 1) // FP8_BLOCK
    cols = (in_f + FP8_BLOCK - 1) // FP8_BLOCK
    if tuple(scale_inv.shape) != (rows, cols):
        raise ValueError(f"Scale shape {tuple(scale_inv.shape)} does not match weight {tuple(weight.shape)}")
    scale = scale_inv.float().repeat_interleave(FP8_BLOCK, 0)[:out_f].repeat_interleave(FP8_BLOCK, 1)[:, :in_f]
    return weight.float() * scale


class CheckpointReader:
    """Minimal safetensors reader over a checkpoint directory."""

    def __init__(self, root: Path):
        self.root = Path(root).resolve()
        self.weight_map: dict[str, str] = {}
        index = self.root / "model.safetensors.index.json"
        if index.is_file():
            self.weight_map = dict(json.loads(index.read_text(encoding="utf-8")).get("weight_map", {}))
        self._keys: dict[Path, set[str]] = {}

    def _shards(self, name: str) -> list[Path]:
        shard = self.weight_map.get(name)
        return [self.root / shard] if shard else sorted(self.root.glob("*.safetensors"))

    def has(self, name: str) -> bool:
        from safetensors import safe_open

        if name in self.weight_map:
            return True
        for shard in self._shards(name):
            if shard not in self._keys:
                with safe_open(str(shard), framework="pt", device="cpu") as h:
                    self._keys[shard] = set(h.keys())
            if name in self._keys[shard]:
                return True
        return False

    def get(self, name: str) -> torch.Tensor:
        from safetensors import safe_open

        for shard in self._shards(name):
            if not shard.is_file():
                continue
            with safe_open(str(shard), framework="pt", device="cpu") as h:
                if name in h.keys():
                    return h.get_tensor(name)
        raise KeyError(f"Tensor not found: {name}")

    def layer_tensors(self, layer: int, names) -> dict[str, torch.Tensor]:
        prefix = C.layer_prefix(layer)
        out = {}
        for suffix in names:
            t = self.get(prefix + suffix)
            if t.dtype == torch.float8_e4m3fn:
                scale_name = prefix + suffix.replace(".weight", ".weight_scale_inv")
                t = dequantize_fp8_blockwise(t, self.get(scale_name)).to(torch.bfloat16)
            out[suffix] = t
        return out

    def attention_type(self, layer: int) -> str:
        """Layer kind from the tensors present (qwen36_40layer_loop.py:68-78)."""
        prefix = C.layer_prefix(layer)
        if self.has(prefix + "linear_attn.in_proj_qkv.weight"):
            return "linear_attention"
        if self.has(prefix + "self_attn.q_proj.weight"):
            return "full_attention"
        raise KeyError(f"Could not identify attention type for layer {layer}")


def write_checkpoint(root: Path, layers: dict[int, dict[str, torch.Tensor]]) -> Path:
    """Write ``{layer: {suffix: tensor}}`` as one safetensors file with the
    reference tensor names (used by tests and the golden-fixture script)."""
    from safetensors.torch import save_file

    root = Path(root)
    root.mkdir(parents=True, exist_ok=True)
    flat = {}
    for layer, tensors in layers.items():
        for suffix, t in tensors.items():
            flat[C.layer_prefix(layer) + suffix] = t.contiguous()
    path = root / "model.safetensors"
    save_file(flat, str(path))
    return path
