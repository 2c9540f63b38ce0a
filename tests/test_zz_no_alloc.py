"""The allocation-free GQA decode entry point (ria_gqa_decode_paged_static).

Some callers of the decode step cannot allocate device memory where they
decode: a host runtime that carves all GPU memory into its own pools up
front, a process held to a hard VRAM budget (router-ia's own governors keep
the whole model inside a few GB), or a plugin interface that hands over
inputs and outputs but no workspace.  For them a cudaMalloc at decode time
would fail, exceed the budget or break the host's accounting, so this entry
point keeps its split scratch in a fixed array inside the library instead.

The test calls it through the C ABI twice in a row with different inputs
(the array still holds the first call's partials when the second runs) and
requires each output to equal, bit for bit, the workspace entry point
ria_gqa_decode_paged on the same inputs: both launch the same kernels with
the same split plan, only the scratch address differs.  One sequence of each
call is also checked against the CPU oracle at the GQA tolerance (2e-2 in
the scale-aware max form, 1e-2 relative RMS), and a batch-1 call with
scalar seq_len0 / position0 (no device length arrays) is covered too.

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
    """Random paged caches in shuffled blocks and random projection rows;
    also each sequence's cached prefix (2, n, 256) on the host."""
    gen = torch.Generator().manual_seed(seed)
    blocks = [(n + 1 + C.KV_BLOCK - 1) // C.KV_BLOCK for n in lengths]
    total = sum(blocks) + 2
    perm = torch.randperm(total, generator=gen)
    table = torch.zeros(len(lengths), max(blocks), dtype=torch.int32)
    k_pool = torch.randn(2, total * C.KV_BLOCK, 256, generator=gen).to(torch.bfloat16)
    v_pool = torch.randn(2, total * C.KV_BLOCK, 256, generator=gen).to(torch.bfloat16)
    prefixes = []
    cur = 0
    for i, nb in enumerate(blocks):
        ids = perm[cur:cur + nb]
        table[i, :nb] = ids.to(torch.int32)
        cur += nb
        rows = (ids[:, None] * C.KV_BLOCK + torch.arange(C.KV_BLOCK)[None]).reshape(-1)[:lengths[i]]
        prefixes.append((k_pool[:, rows].clone(), v_pool[:, rows].clone()))
    proj = torch.randn(len(lengths), C.GQA_PROJ_WIDTH, generator=gen).to(torch.bfloat16)
    return k_pool.to(device), v_pool.to(device), table.to(device), proj, prefixes


def _call_static(lib, q, k, v, w, inv, k_pool, v_pool, table, seq_lens, positions, seq_len0, position0, out,
                 batch, split_pages, max_splits, stream):
    return lib.ria_gqa_decode_paged_static(
        q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), w.q_norm.data_ptr(),
        w.k_norm.data_ptr(), inv.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.shape[1],
        table.data_ptr(), table.stride(0), 0 if seq_lens is None else seq_lens.data_ptr(),
        0 if positions is None else positions.data_ptr(), seq_len0, position0, out.data_ptr(), out.stride(0),
        batch, split_pages, max_splits, stream)


def test_static_scratch_entry_point_matches_workspace_entry_point(cuda_device):
    lib = _ext.lib()
    wt = synthetic.gqa_weights(77)
    w = GqaWeights.from_tensors(wt, cuda_device)
    inv = rope_inv_freq(cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    cases = [([300, 1000, 77, 64], 2, 1), ([4096, 5, 640], 3, 2)]
    for lengths, split_pages, seed in cases:  # two calls in a row, different inputs
        k_pool, v_pool, table, proj, prefixes = _case(lengths, cuda_device, seed)
        pd = proj.to(cuda_device)
        B = len(lengths)
        q = pd[:, C.GQA_PROJ_Q[0]:C.GQA_PROJ_Q[1]]
        k = pd[:, C.GQA_PROJ_K[0]:C.GQA_PROJ_K[1]]
        v = pd[:, C.GQA_PROJ_V[0]:C.GQA_PROJ_V[1]]
        seq_lens = torch.tensor(lengths, dtype=torch.int32, device=cuda_device)
        positions = torch.tensor([n + 7 for n in lengths], dtype=torch.int32, device=cuda_device)
        max_splits = max(((n + 1 + 63) // 64 + split_pages - 1) // split_pages for n in lengths)
        assert max_splits > 1 and _ext.gqa_workspace_bytes(B, max_splits) <= _ext.GQA_STATIC_SCRATCH_BYTES

        out_static = torch.empty(B, 4096, dtype=torch.bfloat16, device=cuda_device)
        rc = _call_static(lib, q, k, v, w, inv, k_pool, v_pool, table, seq_lens, positions, 0, 0, out_static, B,
                          split_pages, max_splits, stream)
        assert rc == 0, _ext.last_error()

        # the workspace entry point on the same inputs (the new token is
        # appended again into the same rows, with the same values)
        out_ws = torch.empty_like(out_static)
        ws = torch.empty(_ext.gqa_workspace_bytes(B, max_splits) // 4, dtype=torch.float32, device=cuda_device)
        _ext.gqa_decode_paged(q, k, v, w.q_norm, w.k_norm, inv, k_pool, v_pool, table, seq_lens, positions, out_ws,
                              ws, split_pages, max_splits)
        torch.cuda.synchronize(cuda_device)
        assert torch.equal(out_static, out_ws)

        i = 0  # one sequence against the CPU oracle
        kc, vc = prefixes[i]
        ref, _, _ = O.gqa_kernel_ref(proj[i, C.GQA_PROJ_Q[0]:C.GQA_PROJ_Q[1]], proj[i, C.GQA_PROJ_K[0]:C.GQA_PROJ_K[1]],
                                     proj[i, C.GQA_PROJ_V[0]:C.GQA_PROJ_V[1]], wt, kc, vc, lengths[i] + 7)
        got = out_static[i].float().cpu()
        assert O.finite(got)
        assert O.max_err_bf16(got, ref) < 2e-2 and O.rel_rms(got, ref) < 1e-2
    assert _ext.device_error() == 0


def test_static_scratch_batch1_scalar_lengths(cuda_device):
    """Batch 1 with seq_len0 / position0 instead of device arrays, split over
    the scratch array, equal to the workspace entry point."""
    lib = _ext.lib()
    wt = synthetic.gqa_weights(78)
    w = GqaWeights.from_tensors(wt, cuda_device)
    inv = rope_inv_freq(cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    n, split_pages = 700, 2
    k_pool, v_pool, table, proj, prefixes = _case([n], cuda_device, 3)
    pd = proj.to(cuda_device)
    q, k, v = (pd[:, a:b] for a, b in (C.GQA_PROJ_Q, C.GQA_PROJ_K, C.GQA_PROJ_V))
    max_splits = ((n + 1 + 63) // 64 + split_pages - 1) // split_pages
    out_static = torch.empty(1, 4096, dtype=torch.bfloat16, device=cuda_device)
    rc = _call_static(lib, q, k, v, w, inv, k_pool, v_pool, table, None, None, n, n + 3, out_static, 1, split_pages,
                      max_splits, stream)
    assert rc == 0, _ext.last_error()
    out_ws = torch.empty_like(out_static)
    ws = torch.empty(_ext.gqa_workspace_bytes(1, max_splits) // 4, dtype=torch.float32, device=cuda_device)
    seq_lens = torch.tensor([n], dtype=torch.int32, device=cuda_device)
    positions = torch.tensor([n + 3], dtype=torch.int32, device=cuda_device)
    _ext.gqa_decode_paged(q, k, v, w.q_norm, w.k_norm, inv, k_pool, v_pool, table, seq_lens, positions, out_ws, ws,
                          split_pages, max_splits)
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(out_static, out_ws)
    kc, vc = prefixes[0]
    ref, _, _ = O.gqa_kernel_ref(proj[0, C.GQA_PROJ_Q[0]:C.GQA_PROJ_Q[1]], proj[0, C.GQA_PROJ_K[0]:C.GQA_PROJ_K[1]],
                                 proj[0, C.GQA_PROJ_V[0]:C.GQA_PROJ_V[1]], wt, kc, vc, n + 3)
    got = out_static[0].float().cpu()
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
