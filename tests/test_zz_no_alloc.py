"""The allocation-free GQA decode entry point (ria_gqa_decode_paged_static).

Some callers cannot allocate device memory where they decode (code captured
into a CUDA graph, runtimes that own all GPU memory, plugin interfaces without
a workspace); this entry point keeps its split scratch in a fixed array inside
the library instead.  The test calls it through the C ABI twice in a row, with
different inputs each time (the array still holds the first call's partials
when the second runs), and checks each output against the workspace entry
point ria_gqa_decode_paged on the same inputs, within the tolerance the GQA
kernel tests use (2e-2 in the scale-aware max form, 1e-2 relative RMS).

This file is named so that pytest collects it last.
"""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from ria_b200 import constants as C
from ria_b200.weights import GqaWeights, rope_inv_freq

pytestmark = pytest.mark.gpu


def _case(lengths, device, seed):
    gen = torch.Generator().manual_seed(seed)
    blocks = [(n + 1 + C.KV_BLOCK - 1) // C.KV_BLOCK for n in lengths]
    total = sum(blocks) + 2
    perm = torch.randperm(total, generator=gen)
    table = torch.zeros(len(lengths), max(blocks), dtype=torch.int32)
    cur = 0
    for i, nb in enumerate(blocks):
        table[i, :nb] = perm[cur:cur + nb].to(torch.int32)
        cur += nb
    k_pool = torch.randn(2, total * C.KV_BLOCK, 256, generator=gen).to(torch.bfloat16).to(device)
    v_pool = torch.randn(2, total * C.KV_BLOCK, 256, generator=gen).to(torch.bfloat16).to(device)
    proj = torch.randn(len(lengths), C.GQA_PROJ_WIDTH, generator=gen).to(torch.bfloat16).to(device)
    return k_pool, v_pool, table.to(device), proj


def test_static_scratch_entry_point_matches_workspace_entry_point(cuda_device):
    lib = _ext.lib()
    w = GqaWeights.from_tensors(synthetic.gqa_weights(77), cuda_device)
    inv = rope_inv_freq(cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    cases = [([300, 1000, 77, 64], 2, 1), ([4096, 5, 640], 3, 2)]
    for lengths, split_pages, seed in cases:  # two calls in a row, different inputs
        k_pool, v_pool, table, proj = _case(lengths, cuda_device, seed)
        B = len(lengths)
        q = proj[:, C.GQA_PROJ_Q[0]:C.GQA_PROJ_Q[1]]
        k = proj[:, C.GQA_PROJ_K[0]:C.GQA_PROJ_K[1]]
        v = proj[:, C.GQA_PROJ_V[0]:C.GQA_PROJ_V[1]]
        seq_lens = torch.tensor(lengths, dtype=torch.int32, device=cuda_device)
        positions = torch.tensor([n + 7 for n in lengths], dtype=torch.int32, device=cuda_device)
        max_splits = max(((n + 1 + 63) // 64 + split_pages - 1) // split_pages for n in lengths)
        assert max_splits > 1 and _ext.gqa_workspace_bytes(B, max_splits) <= _ext.GQA_STATIC_SCRATCH_BYTES

        out_static = torch.empty(B, 4096, dtype=torch.bfloat16, device=cuda_device)
        rc = lib.ria_gqa_decode_paged_static(
            q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), w.q_norm.data_ptr(),
            w.k_norm.data_ptr(), inv.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.shape[1],
            table.data_ptr(), table.stride(0), seq_lens.data_ptr(), positions.data_ptr(), 0, 0,
            out_static.data_ptr(), out_static.stride(0), B, split_pages, max_splits, stream)
        assert rc == 0, _ext.last_error()

        out_ws = torch.empty_like(out_static)
        ws = torch.empty(_ext.gqa_workspace_bytes(B, max_splits) // 4, dtype=torch.float32, device=cuda_device)
        _ext.gqa_decode_paged(q, k, v, w.q_norm, w.k_norm, inv, k_pool, v_pool, table, seq_lens, positions, out_ws,
                              ws, split_pages, max_splits)
        torch.cuda.synchronize(cuda_device)
        got, ref = out_static.float().cpu(), out_ws.float().cpu()
        assert O.finite(got)
        assert O.max_err_bf16(got, ref) < 2e-2 and O.rel_rms(got, ref) < 1e-2
    assert _ext.device_error() == 0


def test_static_scratch_rejects_sizes_past_the_array(cuda_device):
    lib = _ext.lib()
    too_many = _ext.GQA_STATIC_SCRATCH_BYTES // _ext.gqa_workspace_bytes(1, 1) + 1
    dummy = torch.zeros(16, dtype=torch.int32, device=cuda_device)
    p = dummy.data_ptr()
    rc = lib.ria_gqa_decode_paged_static(p, 8192, p, 512, p, 512, p, p, p, p, p, 64, p, 1, p, p, 0, 0, p, 4096, 1,
                                         1, too_many, None)
    assert rc == _ext.RIA_ERR_INVALID
    assert "fixed" in _ext.last_error() and "bytes" in _ext.last_error()
