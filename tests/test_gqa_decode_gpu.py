"""K3 (paged split-KV GQA decode with fused norm / RoPE / append / gate)
against the CPU oracle.  Outputs within 2e-2 in the scale-aware max form
(``max |d| / max(1, |ref|)``, since outputs are stored in bf16) and 1e-2
relative RMS;
appended K within one bf16 rounding of the oracle, appended V exact."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from ria_b200 import constants as C
from ria_b200.engine import plan_gqa_split
from ria_b200.weights import GqaWeights, rope_inv_freq

pytestmark = pytest.mark.gpu

OUT_MAX_ABS = 2e-2
OUT_REL_RMS = 1e-2


def _build_pool(lengths, extra_blocks, gen, device):
    """Random paged caches: returns pools, block table and per-sequence CPU
    caches (2, L, 256) bf16.  Blocks are assigned in a shuffled order."""
    blocks_per = [(n + 1 + C.KV_BLOCK - 1) // C.KV_BLOCK for n in lengths]
    total = sum(blocks_per) + extra_blocks
    perm = torch.randperm(total, generator=gen)
    k_pool = torch.randn(2, total * C.KV_BLOCK, 256, generator=gen).to(torch.bfloat16)
    v_pool = torch.randn(2, total * C.KV_BLOCK, 256, generator=gen).to(torch.bfloat16)
    max_blocks = max(blocks_per) + 1
    table = torch.zeros(len(lengths), max_blocks, dtype=torch.int32)
    caches = []
    cur = 0
    for i, n in enumerate(lengths):
        ids = perm[cur:cur + blocks_per[i]]
        cur += blocks_per[i]
        table[i, : len(ids)] = ids.to(torch.int32)
        rows = (ids[:, None] * C.KV_BLOCK + torch.arange(C.KV_BLOCK)[None]).reshape(-1)[:n]
        caches.append((k_pool[:, rows].clone(), v_pool[:, rows].clone(), ids))
    return k_pool.to(device), v_pool.to(device), table.to(device), caches


def _run(lengths, positions, cuda_device, split_pages=None, seed=0):
    gen = torch.Generator().manual_seed(seed)
    wt = synthetic.gqa_weights(seed + 100)
    w = GqaWeights.from_tensors(wt, cuda_device)
    B = len(lengths)
    k_pool, v_pool, table, caches = _build_pool(lengths, 3, gen, cuda_device)
    proj = (torch.randn(B, C.GQA_PROJ_WIDTH, generator=gen) * 2.0).to(torch.bfloat16)
    pd = proj.to(cuda_device)
    q = pd[:, C.GQA_PROJ_Q[0]:C.GQA_PROJ_Q[1]]
    k = pd[:, C.GQA_PROJ_K[0]:C.GQA_PROJ_K[1]]
    v = pd[:, C.GQA_PROJ_V[0]:C.GQA_PROJ_V[1]]
    seq_lens = torch.tensor(lengths, dtype=torch.int32, device=cuda_device)
    pos = torch.tensor(positions, dtype=torch.int32, device=cuda_device)
    launch = plan_gqa_split([n + 1 for n in lengths], cuda_device)
    if split_pages is not None:
        blocks = [(n + 1 + 63) // 64 for n in lengths]
        max_splits = max((b + split_pages - 1) // split_pages for b in blocks)
        ws = torch.empty(max(1, _ext.gqa_workspace_bytes(B, max_splits) // 4), device=cuda_device)
        launch.split_pages, launch.max_splits, launch.workspace = split_pages, max_splits, ws
    out = torch.empty(B, 4096, dtype=torch.bfloat16, device=cuda_device)
    _ext.gqa_decode_paged(q, k, v, w.q_norm, w.k_norm, rope_inv_freq(cuda_device), k_pool, v_pool, table, seq_lens,
                          pos, out, launch.workspace, launch.split_pages, launch.max_splits)
    assert _ext.device_error() == 0
    out = out.float().cpu()
    kp, vp = k_pool.cpu(), v_pool.cpu()
    for i, n in enumerate(lengths):
        kc, vc, ids = caches[i]
        ref, k_new, v_new = O.gqa_kernel_ref(proj[i, C.GQA_PROJ_Q[0]:C.GQA_PROJ_Q[1]],
                                             proj[i, C.GQA_PROJ_K[0]:C.GQA_PROJ_K[1]],
                                             proj[i, C.GQA_PROJ_V[0]:C.GQA_PROJ_V[1]], wt, kc, vc, positions[i])
        assert O.max_err_bf16(out[i], ref) < OUT_MAX_ABS, (i, n, O.max_err_bf16(out[i], ref))
        assert O.rel_rms(out[i], ref) < OUT_REL_RMS, (i, n, O.rel_rms(out[i], ref))
        row = int(ids[n // C.KV_BLOCK]) * C.KV_BLOCK + n % C.KV_BLOCK
        assert torch.allclose(kp[:, row].float(), k_new, rtol=2 ** -7, atol=1e-6)
        assert torch.equal(vp[:, row].float(), v_new)
        # the cached prefix is untouched
        rows = (ids[:, None] * C.KV_BLOCK + torch.arange(C.KV_BLOCK)[None]).reshape(-1)[:n]
        assert torch.equal(kp[:, rows], kc) and torch.equal(vp[:, rows], vc)


def test_ragged_lengths_block_edges(cuda_device):
    lengths = [0, 1, 63, 64, 65, 127, 128, 200, 1000]
    positions = [n + 3 for n in lengths]
    _run(lengths, positions, cuda_device)


@pytest.mark.parametrize("split_pages", [1, 2, 5])
def test_split_combine_paths(cuda_device, split_pages):
    lengths = [300, 64, 777, 5]
    _run(lengths, [n for n in lengths], cuda_device, split_pages=split_pages, seed=1)


def test_single_split_direct_output(cuda_device):
    lengths = [130, 10]
    _run(lengths, lengths, cuda_device, split_pages=64, seed=2)


def test_config1_shape_long_context_positions(cuda_device):
    """Benchmark configuration 1: one sequence, 4096 cached tokens; plus a
    far position to exercise RoPE argument reduction."""
    _run([4096], [4096], cuda_device, seed=3)
    _run([2000, 33], [32768, 20000], cuda_device, seed=4)


def test_scalar_length_path_batch1(cuda_device):
    """seq_lens / positions may be host scalars for a single sequence."""
    gen = torch.Generator().manual_seed(9)
    wt = synthetic.gqa_weights(9)
    w = GqaWeights.from_tensors(wt, cuda_device)
    n, pos = 70, 75
    k_pool, v_pool, table, caches = _build_pool([n], 0, gen, cuda_device)
    proj = torch.randn(1, C.GQA_PROJ_WIDTH, generator=gen).to(torch.bfloat16)
    pd = proj.to(cuda_device)
    out = torch.empty(1, 4096, dtype=torch.bfloat16, device=cuda_device)
    launch = plan_gqa_split([n + 1], cuda_device)
    _ext.gqa_decode_paged(pd[:, :8192], pd[:, 8192:8704], pd[:, 8704:], w.q_norm, w.k_norm,
                          rope_inv_freq(cuda_device), k_pool, v_pool, table, None, None, out, launch.workspace,
                          launch.split_pages, launch.max_splits, seq_len0=n, position0=pos)
    kc, vc, _ = caches[0]
    ref, _, _ = O.gqa_kernel_ref(proj[0, :8192], proj[0, 8192:8704], proj[0, 8704:], wt, kc, vc, pos)
    assert O.max_err_bf16(out[0].float().cpu(), ref) < OUT_MAX_ABS


def test_out_of_range_block_is_reported_not_faulted(cuda_device):
    """A block id past the pool is caught in-kernel: the error word is set and
    nothing is written out of bounds (no fault)."""
    gen = torch.Generator().manual_seed(10)
    wt = synthetic.gqa_weights(10)
    w = GqaWeights.from_tensors(wt, cuda_device)
    k_pool, v_pool, table, _ = _build_pool([100], 0, gen, cuda_device)
    table[0, 1] = 10_000  # the block holding token 100 is out of range
    pd = torch.randn(1, C.GQA_PROJ_WIDTH, generator=gen).to(torch.bfloat16).to(cuda_device)
    out = torch.empty(1, 4096, dtype=torch.bfloat16, device=cuda_device)
    launch = plan_gqa_split([101], cuda_device)
    _ext.device_error(clear=True)
    _ext.gqa_decode_paged(pd[:, :8192], pd[:, 8192:8704], pd[:, 8704:], w.q_norm, w.k_norm,
                          rope_inv_freq(cuda_device), k_pool, v_pool, table, None, None, out, launch.workspace,
                          launch.split_pages, launch.max_splits, seq_len0=100, position0=100)
    assert _ext.device_error(clear=True) != 0
    assert _ext.device_error() == 0


def test_undersized_split_plan_is_reported_and_skipped(cuda_device):
    """A split plan smaller than a sequence needs (max_splits x split_pages
    pages < its pages) is caught in-kernel: the device error word reads 7
    (RIA_DEVERR_SPLIT_PLAN), and that sequence's output, workspace partials
    and pool rows are left untouched; the other sequence is still served."""
    gen = torch.Generator().manual_seed(12)
    wt = synthetic.gqa_weights(12)
    w = GqaWeights.from_tensors(wt, cuda_device)
    lengths = [1000, 100]  # 16 and 2 pages; 3 splits of 2 pages cover only 6
    k_pool, v_pool, table, caches = _build_pool(lengths, 1, gen, cuda_device)
    proj = torch.randn(2, C.GQA_PROJ_WIDTH, generator=gen).to(torch.bfloat16)
    pd = proj.to(cuda_device)
    seq_lens = torch.tensor(lengths, dtype=torch.int32, device=cuda_device)
    pos = torch.tensor(lengths, dtype=torch.int32, device=cuda_device)
    split_pages, max_splits = 2, 3
    out = torch.full((2, 4096), 7.0, dtype=torch.bfloat16, device=cuda_device)
    ws = torch.full((_ext.gqa_workspace_bytes(2, max_splits) // 4,), -3.0, device=cuda_device)
    k_before, v_before = k_pool.clone(), v_pool.clone()
    _ext.device_error(clear=True)
    _ext.gqa_decode_paged(pd[:, :8192], pd[:, 8192:8704], pd[:, 8704:], w.q_norm, w.k_norm,
                          rope_inv_freq(cuda_device), k_pool, v_pool, table, seq_lens, pos, out, ws, split_pages,
                          max_splits)
    assert _ext.device_error(clear=True) == 7
    assert torch.all(out[0] == 7.0)
    per_seq = ws[: 2 * max_splits * 16 * 256].view(2, max_splits, 16, 256)
    assert torch.all(per_seq[0] == -3.0)
    lse = ws[2 * max_splits * 16 * 256:].view(2, max_splits, 16)
    assert torch.all(lse[0] == -3.0)
    ids0 = caches[0][2]
    rows0 = (ids0[:, None] * C.KV_BLOCK + torch.arange(C.KV_BLOCK)[None]).reshape(-1).to(cuda_device)
    assert torch.equal(k_pool[:, rows0], k_before[:, rows0]) and torch.equal(v_pool[:, rows0], v_before[:, rows0])
    # the second sequence (one split, direct output) is computed as usual
    kc, vc, _ = caches[1]
    ref, _, _ = O.gqa_kernel_ref(proj[1, :8192], proj[1, 8192:8704], proj[1, 8704:], wt, kc, vc, lengths[1])
    assert O.max_err_bf16(out[1].float().cpu(), ref) < OUT_MAX_ABS
    assert _ext.device_error() == 0


def test_undersized_split_plan_rejected_on_host_for_scalar_length(cuda_device):
    """With host scalars (batch 1) the same condition is an argument error."""
    gen = torch.Generator().manual_seed(13)
    w = GqaWeights.from_tensors(synthetic.gqa_weights(13), cuda_device)
    k_pool, v_pool, table, _ = _build_pool([1000], 0, gen, cuda_device)
    pd = torch.randn(1, C.GQA_PROJ_WIDTH, generator=gen).to(torch.bfloat16).to(cuda_device)
    out = torch.empty(1, 4096, dtype=torch.bfloat16, device=cuda_device)
    ws = torch.empty(_ext.gqa_workspace_bytes(1, 3) // 4, device=cuda_device)
    with pytest.raises(ValueError, match="pages"):
        _ext.gqa_decode_paged(pd[:, :8192], pd[:, 8192:8704], pd[:, 8704:], w.q_norm, w.k_norm,
                              rope_inv_freq(cuda_device), k_pool, v_pool, table, None, None, out, ws, 2, 3,
                              seq_len0=1000, position0=1000)
