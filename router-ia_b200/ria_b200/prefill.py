"""Chunked Gated DeltaNet prefill (K2) host API.

``chunk_gated_delta_rule`` has the argument meaning of the rule router-ia
calls for a prompt (transformers ``torch_chunk_gated_delta_rule`` with
``use_qk_l2norm_in_kernel=True``, through qwen36_linear_attention_hf.py:91-100)
except that key heads are not repeated: value head h reads key head
h // (Hv // Hk), the 2:1 grouping of the Qwen3.6 layers.
"""

from __future__ import annotations

import torch

from . import _ext


def chunk_gated_delta_rule(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                           initial_state: torch.Tensor | None = None, final_state: torch.Tensor | None = None,
                           out: torch.Tensor | None = None,
                           workspace: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """q, k [B, T, Hk, 128] bf16; v [B, T, Hv, 128] bf16; g (log decay) and
    beta [B, T, Hv] fp32; initial_state [B, Hv, 128, 128] fp32 or None;
    workspace: uint8 scratch (see ``_ext.gdn_chunk_prefill_workspace_bytes``)
    or None.  Returns (out [B, T, Hv, 128] bf16, final_state [B, Hv, 128, 128]
    fp32)."""
    B, T, _, _ = q.shape
    Hv = v.shape[2]
    if out is None:
        out = torch.empty(B, T, Hv, 128, dtype=torch.bfloat16, device=v.device)
    if final_state is None:
        final_state = torch.empty(B, Hv, 128, 128, dtype=torch.float32, device=v.device)
    _ext.gdn_chunk_prefill(q, k, v, g.float(), beta.float(), initial_state, final_state, out, workspace)
    return out, final_state
