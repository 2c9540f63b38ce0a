"""Batched greedy decode of the whole Qwen3.6-35B-A3B stack on one GPU.

router-ia generates one sequence at a time: ``run_forward_token``
(qwen36_chat_batch.py:181-207) loads the token's embedding row, runs the 40
layers as ``step_attention`` then ``batched_moe_step``, applies the final
RMSNorm and the lm_head (fp16 autocast on CUDA), and ``run_generated_token``
(:210-213) picks the next id with ``sample_next`` (greedy at temperature 0).
``DecodeModel`` does the same for B sequences per launch on the device:
embedding gather, per layer the attention step (K1 / K3 with the projection
kernels) and the MoE block (K5), then the greedy head; the next ids are fed
back on the device, so a step needs no host data and ``ModelGraph`` replays
it as one CUDA graph.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _ext
from . import constants as C
from .engine import BatchedAttentionState, GqaLaunch, MoePlan, _cdiv, moe_decode, moe_prefill
from .weights import DeltaNetWeights, GqaWeights, MoeWeights


@dataclass
class HeadWeights:
    """Embedding table (bf16, rows read as fp32 like load_embedding_row,
    qwen36_op_probe.py:46-52), final norm weight (fp32, load_final_norm) and
    lm_head in fp16 (the dtype run_forward_token caches it in on CUDA,
    qwen36_chat_batch.py:190)."""

    embedding: torch.Tensor  # [V, 2048] bf16
    final_norm: torch.Tensor  # [2048] f32
    lm_head: torch.Tensor  # [V, 2048] fp16

    @property
    def vocab(self) -> int:
        return self.lm_head.shape[0]

    @classmethod
    def from_tensors(cls, t: dict[str, torch.Tensor], device) -> "HeadWeights":
        return cls(embedding=t["model.language_model.embed_tokens.weight"].to(torch.bfloat16).contiguous().to(device),
                   final_norm=t["model.language_model.norm.weight"].float().contiguous().to(device),
                   lm_head=t["lm_head.weight"].to(device).to(torch.float16).contiguous())


def greedy_head(x: torch.Tensor, head: HeadWeights, next_ids: torch.Tensor, workspace: torch.Tensor | None = None,
                logits: torch.Tensor | None = None) -> None:
    """next_ids [B] int32 <- argmax of fp16(rmsnorm(x) (1 + w)) . lm_head^T for
    x [B, 2048] fp32: one fused weight-streaming launch for B <= 8 (workspace:
    a zero-filled buffer of ``_ext.lm_head_workspace_bytes(B)`` bytes), else the
    fp16 norm kernel, a library GEMM and the row argmax kernel."""
    batch = x.shape[0]
    if batch <= _ext.LM_HEAD_MAX_BATCH:
        if workspace is None:
            workspace = torch.zeros(_ext.lm_head_workspace_bytes(batch), dtype=torch.uint8, device=x.device)
        _ext.lm_head_greedy(x, head.final_norm, head.lm_head, next_ids, workspace, logits)
        return
    h = torch.empty(batch, C.HIDDEN, dtype=torch.float16, device=x.device)
    _ext.final_norm_f16(x, head.final_norm, h)
    lg = F.linear(h, head.lm_head)
    if logits is not None:
        logits.copy_(lg)
    _ext.argmax_f16_rows(lg, next_ids)


class DecodeModel:
    """B sequences of the full stack on one device: attention state
    (``BatchedAttentionState``), per-layer MoE weights, the head, and the
    current token id of every sequence (``ids``, int32, on the device)."""

    def __init__(self, attn_layers: dict[int, DeltaNetWeights | GqaWeights], moe_layers: dict[int, MoeWeights],
                 head: HeadWeights, batch: int, pool_blocks: int, max_blocks_per_seq: int, device):
        self.state = BatchedAttentionState(attn_layers, batch, pool_blocks, max_blocks_per_seq, torch.device(device))
        self.moe = moe_layers
        self.head = head
        self.batch = batch
        num_experts = next(iter(moe_layers.values())).num_experts
        self.plan = MoePlan.create(batch, num_experts, device)
        self.head_ws = (torch.zeros(_ext.lm_head_workspace_bytes(batch), dtype=torch.uint8, device=device)
                        if batch <= _ext.LM_HEAD_MAX_BATCH else None)
        self.ids = torch.zeros(batch, dtype=torch.int32, device=device)
        self.hidden: torch.Tensor | None = None

    def _moe(self, layer: int, x: torch.Tensor) -> torch.Tensor:
        return moe_decode(x, self.moe[layer], self.plan, out=x)

    def _moe_prompt(self, layer: int, x: torch.Tensor) -> torch.Tensor:
        B, T, H = x.shape
        return moe_prefill(x.reshape(B * T, H), self.moe[layer]).view(B, T, H)

    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """A prompt of T tokens for every sequence (``prompt`` [B, T] int32 on
        the device): embedding rows -> 40 x (attention prefill + MoE over all
        B T tokens) -> the greedy head on each sequence's last position.  The
        state advances by T tokens and ``ids`` holds the first generated token
        of every sequence (router-ia's prompt loop, qwen36_chat_batch.py:
        255-268, with the whole prompt in one pass)."""
        B, T = prompt.shape
        if B != self.batch:
            raise ValueError(f"prefill expects all {self.batch} sequences, got {B}")
        x = self.head.embedding.index_select(0, prompt.reshape(-1)).float().view(B, T, C.HIDDEN)
        x = self.state.prefill(x, after_layer=self._moe_prompt)
        self.hidden = x[:, -1].contiguous()
        greedy_head(self.hidden, self.head, self.ids, self.head_ws)
        return self.ids

    def run(self, launch: GqaLaunch) -> None:
        """Device work of one step (what ``ModelGraph`` captures): embedding
        rows of ``ids`` -> 40 x (attention + MoE) -> greedy head -> ``ids``,
        then every sequence's position advances."""
        x = self.head.embedding.index_select(0, self.ids).float()
        x = self.state.run_layers(x, launch, after_layer=self._moe)
        self.hidden = x  # the last step's final hidden state (before the head)
        greedy_head(x, self.head, self.ids, self.head_ws)
        _ext.advance_positions(self.state.seq_lens, self.state.positions)

    def step(self, launch: GqaLaunch | None = None) -> torch.Tensor:
        """One eager decode step; returns ``ids`` (the new token of every
        sequence, also the next step's input).  ``launch``: a split-KV plan
        to use instead of the one planned for the current lengths."""
        st = self.state
        st.reserve_next()
        self.run(launch if launch is not None else st.plan())
        st.lengths = [n + 1 for n in st.lengths]
        st.positions_host = [p + 1 for p in st.positions_host]
        return self.ids


class ModelGraph:
    """``DecodeModel``'s step captured once as a CUDA graph and replayed per
    token (the split-KV plan fixed for the longest sequence the block table
    holds, as ``engine.DecodeGraph``).  Run one eager step first so that
    library initialisation happens outside capture."""

    def __init__(self, model: DecodeModel, split_pages: int | None = None):
        self.model = model
        st = model.state
        if split_pages is None:
            total = sum(_cdiv(n + 1, C.KV_BLOCK) for n in st.lengths)
            split_pages = _ext.gqa_split_pages(max(total, 1), C.FULL_NUM_KV_HEADS)
        max_splits = _cdiv(st.max_blocks_per_seq, split_pages)
        need = _ext.gqa_workspace_bytes(st.batch, max_splits) if max_splits > 1 else 0
        ws = torch.empty(_cdiv(need, 16) * 4, dtype=torch.float32, device=st.device) if need else None
        self.launch = GqaLaunch(split_pages, max_splits, ws)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            model.run(self.launch)

    def step(self) -> torch.Tensor:
        st = self.model.state
        st.reserve_next()
        self.graph.replay()
        st.lengths = [n + 1 for n in st.lengths]
        st.positions_host = [p + 1 for p in st.positions_host]
        return self.model.ids
