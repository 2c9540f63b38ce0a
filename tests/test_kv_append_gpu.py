"""ria_kv_append_paged: the storage step of _append_full_kv
(qwen36_attention_cache.py:365-373) on the paged cache.  V (and bf16 K)
rows land bit for bit at the sequence's next row, through shuffled block
tables and across page edges; f32 rows are rounded once to bf16; nothing
else in the pools changes.  Appending the oracle's post-RoPE K (fp32) gives
the row the GQA decode kernel appends in-kernel, within one bf16 rounding."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from ria_b200 import constants as C
from ria_b200.engine import plan_gqa_split
from ria_b200.weights import GqaWeights, rope_inv_freq

pytestmark = pytest.mark.gpu


def _pool_and_table(lengths, gen, device, extra=2):
    blocks = [n // C.KV_BLOCK + 1 for n in lengths]
    total = sum(blocks) + extra
    perm = torch.randperm(total, generator=gen)
    table = torch.full((len(lengths), max(blocks) + 1), -1, dtype=torch.int32)
    cur = 0
    for i, nb in enumerate(blocks):
        table[i, :nb] = perm[cur:cur + nb].to(torch.int32)
        cur += nb
    k_pool = torch.randn(2, total * C.KV_BLOCK, 256, generator=gen).to(torch.bfloat16).to(device)
    v_pool = torch.randn(2, total * C.KV_BLOCK, 256, generator=gen).to(torch.bfloat16).to(device)
    return k_pool, v_pool, table.to(device)


def _row(table, i, n):
    return int(table[i, n // C.KV_BLOCK]) * C.KV_BLOCK + n % C.KV_BLOCK


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_append_rows_land_exactly(cuda_device, dtype):
    gen = torch.Generator().manual_seed(3)
    lengths = [0, 1, 63, 64, 65, 1000]
    k_pool, v_pool, table = _pool_and_table(lengths, gen, cuda_device)
    k_before, v_before = k_pool.clone(), v_pool.clone()
    wide_k = torch.randn(len(lengths), 512 + 64, generator=gen).to(dtype).to(cuda_device)
    k_new = wide_k[:, 32:544] if dtype == torch.bfloat16 else wide_k[:, 16:528]  # strided, aligned rows
    v_new = torch.randn(len(lengths), 512, generator=gen).to(dtype).to(cuda_device)
    seq_lens = torch.tensor(lengths, dtype=torch.int32, device=cuda_device)
    _ext.kv_append_paged(k_new, v_new, k_pool, v_pool, table, seq_lens)
    torch.cuda.synchronize()
    assert _ext.device_error() == 0
    touched = []
    for i, n in enumerate(lengths):
        r = _row(table.cpu(), i, n)
        touched.append(r)
        assert torch.equal(k_pool[:, r].reshape(512), k_new[i].to(torch.bfloat16))
        assert torch.equal(v_pool[:, r].reshape(512), v_new[i].to(torch.bfloat16))
    mask = torch.ones(k_pool.shape[1], dtype=torch.bool)
    mask[touched] = False
    assert torch.equal(k_pool[:, mask.to(cuda_device)], k_before[:, mask.to(cuda_device)])
    assert torch.equal(v_pool[:, mask.to(cuda_device)], v_before[:, mask.to(cuda_device)])


def test_append_batch1_scalar_length_and_bad_block(cuda_device):
    gen = torch.Generator().manual_seed(4)
    k_pool, v_pool, table = _pool_and_table([130], gen, cuda_device)
    k_new = torch.randn(1, 512, generator=gen).to(torch.bfloat16).to(cuda_device)
    v_new = torch.randn(1, 512, generator=gen).to(torch.bfloat16).to(cuda_device)
    _ext.kv_append_paged(k_new, v_new, k_pool, v_pool, table, None, seq_len0=130)
    r = _row(table.cpu(), 0, 130)
    assert torch.equal(k_pool[:, r].reshape(512), k_new[0]) and torch.equal(v_pool[:, r].reshape(512), v_new[0])
    # a block id outside the pool: device error 3, pools untouched
    bad = table.clone()
    bad[0, 2] = 10_000
    k_before, v_before = k_pool.clone(), v_pool.clone()
    _ext.device_error(clear=True)
    _ext.kv_append_paged(k_new, v_new, k_pool, v_pool, bad, None, seq_len0=131)
    assert _ext.device_error(clear=True) == 3
    assert torch.equal(k_pool, k_before) and torch.equal(v_pool, v_before)
    with pytest.raises(ValueError, match="block table"):
        _ext.kv_append_paged(k_new, v_new, k_pool, v_pool, table, None, seq_len0=64 * table.shape[1])


def test_append_of_oracle_rows_matches_the_decode_kernels_append(cuda_device):
    """The oracle's post-norm, post-RoPE K and raw V of a decode step
    (gqa_kernel_ref, the reference's _full_stateful arithmetic) appended in
    f32 equal the row K3 writes itself: V exactly, K within one bf16
    rounding (the two round an fp32 value computed in a different order)."""
    gen = torch.Generator().manual_seed(5)
    wt = synthetic.gqa_weights(5)
    w = GqaWeights.from_tensors(wt, cuda_device)
    lengths, positions = [70, 200], [75, 4096]
    k_pool, v_pool, table = _pool_and_table(lengths, gen, cuda_device)
    proj = torch.randn(2, C.GQA_PROJ_WIDTH, generator=gen).to(torch.bfloat16)
    pd = proj.to(cuda_device)
    seq_lens = torch.tensor(lengths, dtype=torch.int32, device=cuda_device)
    pos = torch.tensor(positions, dtype=torch.int32, device=cuda_device)
    launch = plan_gqa_split([n + 1 for n in lengths], cuda_device)
    out = torch.empty(2, 4096, dtype=torch.bfloat16, device=cuda_device)
    k2, v2 = k_pool.clone(), v_pool.clone()
    _ext.gqa_decode_paged(pd[:, :8192], pd[:, 8192:8704], pd[:, 8704:], w.q_norm, w.k_norm,
                          rope_inv_freq(cuda_device), k_pool, v_pool, table, seq_lens, pos, out, launch.workspace,
                          launch.split_pages, launch.max_splits)
    k_rows, v_rows = [], []
    for i, n in enumerate(lengths):
        empty = torch.zeros(2, 0, 256)
        _, k_new, v_new = O.gqa_kernel_ref(proj[i, :8192], proj[i, 8192:8704], proj[i, 8704:], wt, empty, empty,
                                           positions[i])
        k_rows.append(k_new.reshape(512))
        v_rows.append(v_new.reshape(512))
    _ext.kv_append_paged(torch.stack(k_rows).to(cuda_device), torch.stack(v_rows).to(cuda_device), k2, v2, table,
                         seq_lens)
    torch.cuda.synchronize()
    assert _ext.device_error() == 0
    for i, n in enumerate(lengths):
        r = _row(table.cpu(), i, n)
        assert torch.equal(v2[:, r], v_pool[:, r])
        assert torch.allclose(k2[:, r].float(), k_pool[:, r].float(), rtol=2 ** -7, atol=1e-6)
