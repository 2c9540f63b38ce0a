"""Batched decode of the hybrid attention stack on one GPU.

One decode step of one layer for B sequences is:

    DeltaNet: h = rmsnorm(x) -> proj = h W_in^T (cuBLAS) -> K1 (conv, gates,
              norms, delta rule, gated norm) -> o = g W_out^T (cuBLAS) -> x + o
    GQA:      h = rmsnorm(x) -> proj = h W_in^T -> K3 (q/k norm, RoPE, KV append,
              split-KV attention, gate) -> o = a W_out^T -> x + o

which is router-ia's ``_linear_stateful`` / ``_full_stateful``
(qwen36_attention_cache.py:224-324) with the per-sequence Python loop replaced
by a batch dimension.  All state stays in HBM:

* DeltaNet: ``rec[layer]`` [slots, 32, 128, 128] fp32 and ``conv[layer]``
  [slots, 8192, 4] bf16, one slot per sequence;
* GQA: one paged bf16 pool per layer, K and V each [2, pool_tokens, 256], with
  64-token blocks; all GQA layers share one block table because every layer
  appends the same token positions.
"""

from __future__ import annotations

import weakref

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import _ext
from . import constants as C
from .weights import DeltaNetWeights, GqaWeights, MoeWeights, rope_inv_freq


def _cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def _in_projection(x: torch.Tensor, w: DeltaNetWeights | GqaWeights) -> torch.Tensor:
    """bf16(W_in . fp16(rmsnorm(x) * (1 + w))) through the layer's fused fp16
    in-projection: one weight-streaming GEMV kernel with the norm fused for
    small batches, the norm kernel plus a library fp16 GEMM with fp32 output
    otherwise (rounded once to bf16, the kernels' input type)."""
    batch = x.shape[0]
    if batch <= _ext.GEMV_MAX_BATCH:
        proj = torch.empty(batch, w.w_in.shape[0], dtype=torch.bfloat16, device=x.device)
        _ext.rmsnorm_gemv(x, w.in_norm, w.w_in, proj)
        return proj
    return _norm_gemm(x, w)


def _norm_gemm(x: torch.Tensor, w: DeltaNetWeights | GqaWeights) -> torch.Tensor:
    """Rows x [N, 2048] fp32 -> bf16(W_in . fp16(rmsnorm(x) * (1 + w))) [N, n].

    The library GEMM writes fp32 and the result is rounded to bf16 once: an
    fp16 GEMM output rounded again to bf16 lands on bf16 ties in about one
    element in sixteen (fp16 holds every bf16 midpoint) and moved the
    DeltaNet conv input, which both paths round to bf16, by a bf16 step
    there -- about 1e-2 on single tokens' attention output."""
    h = torch.empty(x.shape[0], C.HIDDEN, dtype=torch.float16, device=x.device)
    _ext.rmsnorm_rows(x, w.in_norm, h)
    return torch.mm(h, w.w_in.t(), out_dtype=torch.float32).to(torch.bfloat16)


def _out_projection(a: torch.Tensor, w: DeltaNetWeights | GqaWeights, x: torch.Tensor) -> torch.Tensor:
    """x + bf16(a . w_out^T): the out-projection and the residual add, fused
    into one GEMV kernel for small batches."""
    batch = a.shape[0]
    out = torch.empty(batch, C.HIDDEN, dtype=torch.float32, device=x.device)
    if batch <= _ext.GEMV_MAX_BATCH:
        _ext.gemv_residual(a, w.w_out, x, out)
        return out
    o = F.linear(a, w.w_out)
    _ext.residual_add(x, o, out)
    return out


# Batches up to 8 step a layer with one C call (ria_*_layer_decode: the same
# GEMV / attention / GEMV launches issued from C), its intermediates in a
# scratch buffer per device and stream (allocated from the capture pool when
# first used inside a CUDA-graph capture) and the weights' pointers cached per
# weights object: three or four Python-level calls per layer cost more host
# time than a small-batch layer's GPU time.
_LAYER_SCRATCH: dict = {}
_LAYER_SCRATCH_OUTGROWN: list = []  # kept alive: a captured graph may still point at one
_LAYER_ARGS: dict = {}


def _layer_scratch(dev: torch.device, nbytes: int) -> torch.Tensor:
    key = (dev.index, torch._C._cuda_getCurrentRawStream(dev.index))
    buf = _LAYER_SCRATCH.get(key)
    if buf is None or buf.numel() < nbytes:
        if buf is not None:
            _LAYER_SCRATCH_OUTGROWN.append(buf)
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _LAYER_SCRATCH[key] = buf
    return buf


def _layer_args(w: DeltaNetWeights | GqaWeights) -> tuple:
    entry = _LAYER_ARGS.get(id(w))
    if entry is None or entry[0]() is not w:
        args = _ext.deltanet_layer_args(w) if isinstance(w, DeltaNetWeights) else _ext.gqa_layer_args(w)
        entry = (weakref.ref(w), args)
        _LAYER_ARGS[id(w)] = entry
    return entry[1]


def deltanet_decode(x: torch.Tensor, w: DeltaNetWeights, rec: torch.Tensor, conv: torch.Tensor,
                    slots: torch.Tensor | None = None) -> torch.Tensor:
    """One DeltaNet layer step for ``x`` [B, 2048] fp32; returns the residual."""
    batch = x.shape[0]
    if batch <= _ext.GEMV_MAX_BATCH:
        out = torch.empty(batch, C.HIDDEN, dtype=torch.float32, device=x.device)
        _ext.deltanet_layer_decode(x, _layer_args(w), conv, rec, out,
                                   _layer_scratch(x.device, _ext.deltanet_layer_scratch_bytes(batch)), slots)
        return out
    proj = _in_projection(x, w)
    gated = torch.empty(batch, C.LINEAR_VALUE_DIM, dtype=torch.bfloat16, device=x.device)
    _ext.gdn_decode_step(
        proj[:, C.DN_PROJ_QKV[0]:C.DN_PROJ_QKV[1]], proj[:, C.DN_PROJ_Z[0]:C.DN_PROJ_Z[1]],
        proj[:, C.DN_PROJ_B[0]:C.DN_PROJ_B[1]], proj[:, C.DN_PROJ_A[0]:C.DN_PROJ_A[1]],
        w.conv_w, w.a_log, w.dt_bias, w.norm_w, conv, rec, slots, gated)
    return _out_projection(gated, w, x)


@dataclass
class GqaLaunch:
    """Split-KV launch shape for one decode step of a batch."""

    split_pages: int
    max_splits: int
    workspace: torch.Tensor | None


def plan_gqa_split(lengths_after: list[int], device, workspace: torch.Tensor | None = None) -> GqaLaunch:
    """Choose blocks-per-split for a batch whose KV lengths (after this step's
    append) are ``lengths_after`` and size the split workspace."""
    blocks = [_cdiv(n, C.KV_BLOCK) for n in lengths_after]
    split_pages = _ext.gqa_split_pages(sum(blocks), C.FULL_NUM_KV_HEADS)
    max_splits = max(_cdiv(b, split_pages) for b in blocks)
    need = _ext.gqa_workspace_bytes(len(blocks), max_splits) if max_splits > 1 else 0
    if need:
        if workspace is None or workspace.numel() * workspace.element_size() < need:
            workspace = torch.empty(_cdiv(need, 16) * 4, dtype=torch.float32, device=device)
    return GqaLaunch(split_pages, max_splits, workspace)


def gqa_decode(x: torch.Tensor, w: GqaWeights, k_pool: torch.Tensor, v_pool: torch.Tensor,
               block_table: torch.Tensor, inv_freq: torch.Tensor, launch: GqaLaunch,
               seq_lens: torch.Tensor | None = None, positions: torch.Tensor | None = None,
               seq_len0: int = 0, position0: int = 0) -> torch.Tensor:
    """One GQA layer step for ``x`` [B, 2048] fp32; returns the residual.  The
    new token of sequence i is appended to the pool at index seq_lens[i]."""
    batch = x.shape[0]
    if batch <= _ext.GEMV_MAX_BATCH:
        out = torch.empty(batch, C.HIDDEN, dtype=torch.float32, device=x.device)
        _ext.gqa_layer_decode(x, _layer_args(w), inv_freq, k_pool, v_pool, block_table, out,
                              _layer_scratch(x.device, _ext.gqa_layer_scratch_bytes(batch, launch.max_splits)),
                              launch.split_pages, launch.max_splits, seq_lens, positions, seq_len0, position0)
        return out
    proj = _in_projection(x, w)
    attn = torch.empty(batch, C.FULL_Q_DIM, dtype=torch.bfloat16, device=x.device)
    _ext.gqa_decode_paged(
        proj[:, C.GQA_PROJ_Q[0]:C.GQA_PROJ_Q[1]], proj[:, C.GQA_PROJ_K[0]:C.GQA_PROJ_K[1]],
        proj[:, C.GQA_PROJ_V[0]:C.GQA_PROJ_V[1]], w.q_norm, w.k_norm, inv_freq, k_pool, v_pool, block_table,
        seq_lens, positions, attn, launch.workspace, launch.split_pages, launch.max_splits,
        seq_len0=seq_len0, position0=position0)
    return _out_projection(attn, w, x)


def deltanet_prefill(x: torch.Tensor, w: DeltaNetWeights, rec: torch.Tensor, conv: torch.Tensor) -> torch.Tensor:
    """T prompt tokens of B sequences through one DeltaNet layer at once:
    x [B, T, 2048] fp32 -> residual [B, T, 2048] fp32; ``rec`` [B, 32, 128, 128]
    and ``conv`` [B, 8192, 4] continue from and end at the sequences' state.
    Same arithmetic as T decode steps, with the recurrence in chunked form
    (K2) instead of token by token."""
    B, T, _ = x.shape
    xf = x.reshape(B * T, C.HIDDEN)
    proj = _norm_gemm(xf, w)
    mixed = proj.view(B, T, C.DN_PROJ_WIDTH)[:, :, C.DN_PROJ_QKV[0]:C.DN_PROJ_QKV[1]]
    y = torch.empty(B, T, C.LINEAR_CONV_DIM, dtype=torch.bfloat16, device=x.device)
    _ext.conv1d_prefill(mixed, conv, w.conv_w, y)
    q = y[:, :, :C.LINEAR_KEY_DIM].unflatten(2, (C.LINEAR_NUM_K_HEADS, C.LINEAR_HEAD_DIM))
    k = y[:, :, C.LINEAR_KEY_DIM:2 * C.LINEAR_KEY_DIM].unflatten(2, (C.LINEAR_NUM_K_HEADS, C.LINEAR_HEAD_DIM))
    v = y[:, :, 2 * C.LINEAR_KEY_DIM:].unflatten(2, (C.LINEAR_NUM_V_HEADS, C.LINEAR_HEAD_DIM))
    g = torch.empty(B * T, C.LINEAR_NUM_V_HEADS, dtype=torch.float32, device=x.device)
    beta = torch.empty_like(g)
    _ext.gdn_gates(proj[:, C.DN_PROJ_A[0]:C.DN_PROJ_A[1]], proj[:, C.DN_PROJ_B[0]:C.DN_PROJ_B[1]], w.a_log,
                   w.dt_bias, g, beta)
    o = torch.empty(B, T, C.LINEAR_NUM_V_HEADS, C.LINEAR_HEAD_DIM, dtype=torch.bfloat16, device=x.device)
    _ext.gdn_chunk_prefill(q, k, v, g.view(B, T, -1), beta.view(B, T, -1), rec, rec, o)
    gated = torch.empty(B * T, C.LINEAR_VALUE_DIM, dtype=torch.bfloat16, device=x.device)
    _ext.gated_rmsnorm(o.view(B * T, C.LINEAR_VALUE_DIM), proj[:, C.DN_PROJ_Z[0]:C.DN_PROJ_Z[1]], w.norm_w, gated)
    out_p = F.linear(gated, w.w_out)
    out = torch.empty(B * T, C.HIDDEN, dtype=torch.float32, device=x.device)
    _ext.residual_add(xf, out_p, out)
    return out.view(B, T, C.HIDDEN)


def gqa_prefill(x: torch.Tensor, w: GqaWeights, k_pool: torch.Tensor, v_pool: torch.Tensor,
                block_table: torch.Tensor, inv_freq: torch.Tensor, seq_lens: torch.Tensor, positions: torch.Tensor,
                workspace: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """T prompt tokens of B sequences through one GQA layer (K4): x
    [B, T, 2048] fp32 -> (residual [B, T, 2048] fp32, workspace); K/V appended
    at seq_lens[b] + t, RoPE at positions[b] + t."""
    B, T, _ = x.shape
    xf = x.reshape(B * T, C.HIDDEN)
    proj = _norm_gemm(xf, w).view(B, T, C.GQA_PROJ_WIDTH)
    attn = torch.empty(B, T, C.FULL_Q_DIM, dtype=torch.bfloat16, device=x.device)
    workspace = _ext.gqa_prefill(proj[:, :, C.GQA_PROJ_Q[0]:C.GQA_PROJ_Q[1]], proj[:, :, C.GQA_PROJ_K[0]:C.GQA_PROJ_K[1]],
                                 proj[:, :, C.GQA_PROJ_V[0]:C.GQA_PROJ_V[1]], w.q_norm, w.k_norm, inv_freq, k_pool,
                                 v_pool, block_table, seq_lens, positions, attn, workspace)
    o = F.linear(attn.view(B * T, C.FULL_Q_DIM), w.w_out)
    out = torch.empty(B * T, C.HIDDEN, dtype=torch.float32, device=x.device)
    _ext.residual_add(xf, o, out)
    return out.view(B, T, C.HIDDEN), workspace


@dataclass
class MoePlan:
    """Buffers of one MoE launch for a fixed batch: the routing it writes
    (expert ids, router weights, shared gate) and the kernels' workspace
    (zero-filled once: its hand-off counters start at zero and every call
    leaves them there).  Allocated once so that a captured decode step
    reuses them."""

    batch: int
    top_k: int
    expert_ids: torch.Tensor  # [B, k] int32
    expert_weights: torch.Tensor  # [B, k] f32
    shared_gate: torch.Tensor  # [B] f32
    workspace: torch.Tensor  # uint8

    @classmethod
    def create(cls, batch: int, num_experts: int, device, top_k: int = 8) -> "MoePlan":
        ws = _ext.moe_workspace_bytes(batch, num_experts, top_k)
        return cls(batch, top_k,
                   torch.empty(batch, top_k, dtype=torch.int32, device=device),
                   torch.empty(batch, top_k, dtype=torch.float32, device=device),
                   torch.empty(batch, dtype=torch.float32, device=device),
                   torch.zeros(max(ws, 1), dtype=torch.uint8, device=device))


def moe_decode(x: torch.Tensor, w: MoeWeights, plan: MoePlan | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """The MoE block after a layer's attention (K5): x [B, 2048] fp32 residual
    -> x + routed experts + gated shared expert, as batched_moe_step
    (qwen36_chat_batch.py:127-178) computes it token by token.  ``out`` may
    be ``x`` (in place).  The routing lands in ``plan``."""
    if plan is None:
        plan = MoePlan.create(x.shape[0], w.num_experts, x.device)
    if plan.batch != x.shape[0]:
        raise ValueError(f"MoE plan is for batch {plan.batch}, got {x.shape[0]} tokens")
    if out is None:
        out = torch.empty_like(x)
    _ext.moe_decode(x, w, out, plan.expert_ids, plan.expert_weights, plan.shared_gate, plan.workspace, plan.top_k)
    return out


def moe_prefill(x: torch.Tensor, w: MoeWeights, top_k: int = 8, chunk: int = 16384) -> torch.Tensor:
    """The MoE block for many tokens at once (a prompt prefill): x [N, 2048]
    fp32 -> x + routed experts + gated shared expert, batched_moe_step's
    arithmetic (qwen36_chat_batch.py:127-178) for every token.

    With thousands of tokens per expert the block is a grouped GEMM, compute-
    rather than weight-bound, so this path runs its projections on library
    GEMMs instead of the decode kernels: the post-attention norm (one kernel,
    fp32 and bf16 copies), fp32 router logits (fp32 GEMM), top-k and softmax
    as in the decode path; the (token, slot) pairs sorted by expert (stable),
    their bf16 activations gathered and the expert projections run as grouped
    bf16 GEMMs over the sorted pairs (``torch._grouped_mm``, fp32
    accumulation) with silu(gate) * up in one kernel; the shared expert as
    plain GEMMs; one kernel then sums each token's k weighted expert rows (in
    slot order, read from their sorted positions), the gated shared row and
    the residual.  bf16 activations put the result within about 1e-3
    relative of the fp32-grade decode kernels.  Tokens go through in chunks
    of ``chunk`` to bound the temporaries (~1.5 GB at 16384)."""
    bf = torch.bfloat16
    n, hidden = x.shape
    out = torch.empty_like(x)
    router = w.router.float()
    sgw = w.shared_gate.float()
    for s in range(0, n, chunk):
        xc = x[s:s + chunk]
        c = xc.shape[0]
        h = torch.empty(c, hidden, dtype=torch.float32, device=x.device)
        hb = torch.empty(c, hidden, dtype=bf, device=x.device)
        _ext.moe_prompt_norm(xc, w.post_norm, h, hb)
        vals, ids = (h @ router.T).topk(top_k, dim=-1)
        wts = torch.softmax(vals, dim=-1)
        sg = torch.sigmoid(h @ sgw)
        flat = ids.reshape(-1)
        order = torch.argsort(flat, stable=True)
        pos = torch.empty_like(order, dtype=torch.int32)
        pos[order] = torch.arange(order.numel(), dtype=torch.int32, device=x.device)
        offs = torch.cumsum(torch.bincount(flat, minlength=w.num_experts), 0, dtype=torch.int32)
        xs = hb.index_select(0, order // top_k)
        g = torch._grouped_mm(xs, w.experts_gate.transpose(1, 2), offs=offs)
        u = torch._grouped_mm(xs, w.experts_up.transpose(1, 2), offs=offs)
        _ext.silu_mul_bf16(g, u, g)
        y = torch._grouped_mm(g, w.experts_down.transpose(1, 2), offs=offs)
        sh = F.linear(hb, w.shared_gate_proj)
        _ext.silu_mul_bf16(sh, F.linear(hb, w.shared_up_proj), sh)
        shared = F.linear(sh, w.shared_down_proj)
        _ext.moe_prompt_combine(xc, y, pos.view(c, top_k), wts, shared, sg, out[s:s + chunk])
    return out


class BlockAllocator:
    """Free list of physical KV blocks shared by every GQA layer's pool."""

    def __init__(self, num_blocks: int):
        self.num_blocks = int(num_blocks)
        self._free = list(range(self.num_blocks - 1, -1, -1))

    def alloc(self, n: int) -> list[int]:
        if n > len(self._free):
            raise RuntimeError(f"KV pool exhausted: need {n} blocks, {len(self._free)} free of {self.num_blocks}")
        return [self._free.pop() for _ in range(n)]

    def free(self, blocks: list[int]) -> None:
        self._free.extend(reversed(blocks))

    @property
    def free_blocks(self) -> int:
        return len(self._free)


@dataclass
class BatchedAttentionState:
    """Decode state of B sequences over the whole hybrid stack on one device.

    ``layers`` maps a layer index to DeltaNetWeights or GqaWeights.  Sequences
    occupy slots 0..B-1; their KV lengths and absolute positions live on the
    device (``seq_lens``, ``positions``) with a host mirror used for planning.
    """

    layers: dict[int, DeltaNetWeights | GqaWeights]
    batch: int
    pool_blocks: int
    max_blocks_per_seq: int
    device: torch.device
    rec: dict[int, torch.Tensor] = field(default_factory=dict)
    conv: dict[int, torch.Tensor] = field(default_factory=dict)
    k_pool: dict[int, torch.Tensor] = field(default_factory=dict)
    v_pool: dict[int, torch.Tensor] = field(default_factory=dict)

    def __post_init__(self):
        dev = self.device
        for layer, w in self.layers.items():
            if isinstance(w, DeltaNetWeights):
                self.rec[layer] = torch.zeros(self.batch, C.LINEAR_NUM_V_HEADS, C.LINEAR_HEAD_DIM,
                                              C.LINEAR_HEAD_DIM, dtype=torch.float32, device=dev)
                self.conv[layer] = torch.zeros(self.batch, C.LINEAR_CONV_DIM, C.LINEAR_CONV_STATE,
                                               dtype=torch.bfloat16, device=dev)
            else:
                shape = (C.FULL_NUM_KV_HEADS, self.pool_blocks * C.KV_BLOCK, C.FULL_HEAD_DIM)
                self.k_pool[layer] = torch.zeros(shape, dtype=torch.bfloat16, device=dev)
                self.v_pool[layer] = torch.zeros(shape, dtype=torch.bfloat16, device=dev)
        self.allocator = BlockAllocator(self.pool_blocks)
        self.block_table = torch.zeros(self.batch, self.max_blocks_per_seq, dtype=torch.int32, device=dev)
        self._table_host = torch.zeros(self.batch, self.max_blocks_per_seq, dtype=torch.int32)
        self._blocks: list[list[int]] = [[] for _ in range(self.batch)]
        self.lengths: list[int] = [0] * self.batch
        self.positions_host: list[int] = [0] * self.batch
        self.seq_lens = torch.zeros(self.batch, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(self.batch, dtype=torch.int32, device=dev)
        self.inv_freq = rope_inv_freq(dev)
        self._workspace: torch.Tensor | None = None

    # ---- bookkeeping
    def reserve(self, seq: int, total_tokens: int) -> None:
        """Make sure sequence ``seq`` owns blocks for ``total_tokens`` tokens."""
        need = _cdiv(total_tokens, C.KV_BLOCK)
        if need > self.max_blocks_per_seq:
            raise RuntimeError(f"sequence {seq} needs {need} blocks > max_blocks_per_seq={self.max_blocks_per_seq}")
        have = len(self._blocks[seq])
        if need > have:
            new = self.allocator.alloc(need - have)
            self._blocks[seq].extend(new)
            self._table_host[seq, have:need] = torch.tensor(new, dtype=torch.int32)

    def reset(self) -> None:
        """Every sequence back to an empty context (a fresh request per slot):
        zero recurrent and conv states, pages returned, lengths and positions 0."""
        for layer in self.rec:
            self.rec[layer].zero_()
            self.conv[layer].zero_()
        for blocks in self._blocks:
            self.allocator.free(blocks)
            blocks.clear()
        self._table_host.zero_()
        self.lengths = [0] * self.batch
        self.positions_host = [0] * self.batch
        self.sync_tables()

    def sync_tables(self) -> None:
        """Upload the block table and lengths (call after reserve/set_length)."""
        self.block_table.copy_(self._table_host)
        self.seq_lens.copy_(torch.tensor(self.lengths, dtype=torch.int32))
        self.positions.copy_(torch.tensor(self.positions_host, dtype=torch.int32))

    def set_length(self, seq: int, length: int, position: int | None = None) -> None:
        self.reserve(seq, length)
        self.lengths[seq] = int(length)
        self.positions_host[seq] = int(length if position is None else position)

    def physical_rows(self, seq: int, length: int) -> torch.Tensor:
        """Pool row indices (per KV head) of the first ``length`` tokens."""
        blocks = torch.tensor(self._blocks[seq][: _cdiv(length, C.KV_BLOCK)], dtype=torch.int64)
        rows = (blocks[:, None] * C.KV_BLOCK + torch.arange(C.KV_BLOCK)[None, :]).reshape(-1)
        return rows[:length]

    # ---- one decode step over all layers
    def plan(self) -> GqaLaunch:
        launch = plan_gqa_split([n + 1 for n in self.lengths], self.device, self._workspace)
        self._workspace = launch.workspace
        return launch

    def reserve_next(self) -> None:
        """Reserve the page of each sequence's next token (uploading the block
        table when one was added)."""
        grew = False
        for i, n in enumerate(self.lengths):
            if n % C.KV_BLOCK == 0 and len(self._blocks[i]) * C.KV_BLOCK <= n:
                self.reserve(i, n + 1)
                grew = True
        if grew:
            self.block_table.copy_(self._table_host)

    def prepare_step(self) -> GqaLaunch:
        """Reserve the page of each sequence's next token and plan the launch."""
        self.reserve_next()
        return self.plan()

    def prefill(self, x: torch.Tensor, after_layer=None) -> torch.Tensor:
        """T prompt tokens for every sequence at once: x [B, T, 2048] fp32 ->
        [B, T, 2048] fp32, every layer's state advanced by T tokens.  Equals T
        calls of ``step`` (router-ia's prompt loop, qwen36_chat_batch.py:
        255-258) with the DeltaNet recurrence in chunked form (K2) and the GQA
        layers through the causal prefill kernel (K4).  ``after_layer(layer,
        x) -> x`` runs after each layer's attention (the full model's MoE)."""
        B, T, _ = x.shape
        if B != self.batch:
            raise ValueError(f"prefill expects all {self.batch} sequences, got {B}")
        for i, n in enumerate(self.lengths):
            self.reserve(i, n + T)
        self.block_table.copy_(self._table_host)
        self.seq_lens.copy_(torch.tensor(self.lengths, dtype=torch.int32))
        self.positions.copy_(torch.tensor(self.positions_host, dtype=torch.int32))
        ws = None
        for layer in sorted(self.layers):
            w = self.layers[layer]
            if isinstance(w, DeltaNetWeights):
                x = deltanet_prefill(x, w, self.rec[layer], self.conv[layer])
            else:
                x, ws = gqa_prefill(x, w, self.k_pool[layer], self.v_pool[layer], self.block_table, self.inv_freq,
                                    self.seq_lens, self.positions, ws)
            if after_layer is not None:
                x = after_layer(layer, x)
        self.lengths = [n + T for n in self.lengths]
        self.positions_host = [p + T for p in self.positions_host]
        self.seq_lens.copy_(torch.tensor(self.lengths, dtype=torch.int32))
        self.positions.copy_(torch.tensor(self.positions_host, dtype=torch.int32))
        return x

    def run_layers(self, x: torch.Tensor, launch: GqaLaunch, after_layer=None) -> torch.Tensor:
        """The layer chain of one decode step, device work only (no host
        bookkeeping, no synchronisation): what a CUDA graph captures.
        ``after_layer(layer, x) -> x`` runs after each layer's attention (the
        full model's MoE block)."""
        for layer in sorted(self.layers):
            w = self.layers[layer]
            if isinstance(w, DeltaNetWeights):
                x = deltanet_decode(x, w, self.rec[layer], self.conv[layer])
            else:
                x = gqa_decode(x, w, self.k_pool[layer], self.v_pool[layer], self.block_table, self.inv_freq,
                               launch, self.seq_lens, self.positions)
            if after_layer is not None:
                x = after_layer(layer, x)
        return x

    def step(self, x: torch.Tensor, launch: GqaLaunch | None = None, advance: bool = True) -> torch.Tensor:
        """Run every layer once for the batch: x [B, 2048] fp32 -> [B, 2048] fp32.

        This is ``run_forward_token``'s attention chain (qwen36_chat_batch.py:
        184-187) without the MoE; ``advance`` then moves every sequence one
        position forward on the device (the caller's ``tokens_seen += 1``)."""
        self.reserve_next()
        if launch is None:
            launch = self.plan()
        x = self.run_layers(x, launch)
        if advance:
            _ext.advance_positions(self.seq_lens, self.positions)
            self.lengths = [n + 1 for n in self.lengths]
            self.positions_host = [p + 1 for p in self.positions_host]
        return x


class DecodeGraph:
    """The decode step of a ``BatchedAttentionState`` (every layer, plus the
    device-side position advance) captured once as a CUDA graph and replayed
    per token: the batched form of router-ia's per-token loop
    (qwen36_chat_batch.py:181-207) without its per-layer launches and host
    syncs.

    The split-KV plan is fixed at capture for the longest sequence the block
    table can hold (``max_blocks_per_seq`` pages), so the graph stays valid as
    sequences grow; per-sequence lengths, positions and the block table live
    on the device and are read by the kernels at replay.  The state must have
    run at least one eager step (or prefill) first, so that library and cuBLAS
    initialisation happens outside capture.
    """

    def __init__(self, state: BatchedAttentionState, split_pages: int | None = None):
        self.state = state
        dev = state.device
        cap_blocks = state.max_blocks_per_seq
        if split_pages is None:
            total = sum(_cdiv(n + 1, C.KV_BLOCK) for n in state.lengths)
            split_pages = _ext.gqa_split_pages(max(total, 1), C.FULL_NUM_KV_HEADS)
        max_splits = _cdiv(cap_blocks, split_pages)
        need = _ext.gqa_workspace_bytes(state.batch, max_splits) if max_splits > 1 else 0
        ws = torch.empty(_cdiv(need, 16) * 4, dtype=torch.float32, device=dev) if need else None
        self.launch = GqaLaunch(split_pages, max_splits, ws)
        self.x = torch.zeros(state.batch, C.HIDDEN, dtype=torch.float32, device=dev)
        self.graph = torch.cuda.CUDAGraph()
        # Capture records work without running it: the state is untouched.
        with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            self.out = state.run_layers(self.x, self.launch)
            _ext.advance_positions(state.seq_lens, state.positions)

    def step(self, x: torch.Tensor) -> torch.Tensor:
        """x [B, 2048] fp32 on the device -> the residual stream [B, 2048] fp32
        (a buffer owned by the graph, overwritten by the next step)."""
        st = self.state
        st.reserve_next()
        self.x.copy_(x)
        self.graph.replay()
        st.lengths = [n + 1 for n in st.lengths]
        st.positions_host = [p + 1 for p in st.positions_host]
        return self.out

