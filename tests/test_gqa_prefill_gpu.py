"""K4 (GQA prefill on tcgen05) against the CPU oracle: T prompt tokens at
once must equal T token-by-token GQA steps.  Outputs within 2e-2 in the
scale-aware max form and 1e-2 relative RMS; appended K within one bf16
rounding of the oracle, appended V exact."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from ria_b200 import constants as C
from ria_b200.weights import GqaWeights, rope_inv_freq

pytestmark = pytest.mark.gpu


def _run(dev, prefixes, T, pos_offset=5, seed=0):
    gen = torch.Generator().manual_seed(seed)
    wt = synthetic.gqa_weights(seed + 50)
    w = GqaWeights.from_tensors(wt, dev)
    B = len(prefixes)
    nblk = [(L0 + T + 63) // 64 for L0 in prefixes]
    total_blocks = sum(nblk) + 2
    perm = torch.randperm(total_blocks, generator=gen)
    table = torch.zeros(B, max(nblk), dtype=torch.int32)
    k_pool = torch.randn(2, total_blocks * 64, 256, generator=gen).to(torch.bfloat16)
    v_pool = torch.full((2, total_blocks * 64, 256), float("nan")).to(torch.bfloat16)  # garbage past the end
    caches, cur = [], 0
    for i, L0 in enumerate(prefixes):
        ids = perm[cur:cur + nblk[i]]
        cur += nblk[i]
        table[i, :nblk[i]] = ids.to(torch.int32)
        rows = (ids[:, None] * 64 + torch.arange(64)[None]).reshape(-1)[:L0]
        v_pool[:, rows] = torch.randn(2, L0, 256, generator=gen).to(torch.bfloat16)
        caches.append((k_pool[:, rows].clone(), v_pool[:, rows].clone(), ids))
    q = torch.randn(B, T, C.FULL_Q_GATE_DIM, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, T, C.FULL_KV_DIM, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, T, C.FULL_KV_DIM, generator=gen).to(torch.bfloat16)
    kp, vp = k_pool.to(dev), v_pool.to(dev)
    out = torch.empty(B, T, 4096, dtype=torch.bfloat16, device=dev)
    lens = torch.tensor(prefixes, dtype=torch.int32, device=dev)
    pos = torch.tensor([L0 + pos_offset for L0 in prefixes], dtype=torch.int32, device=dev)
    _ext.gqa_prefill(q.to(dev), k.to(dev), v.to(dev), w.q_norm, w.k_norm, rope_inv_freq(dev), kp, vp,
                     table.to(dev), lens, pos, out)
    assert _ext.device_error() == 0
    out = out.float().cpu()
    kp, vp = kp.cpu(), vp.cpu()
    worst = (0.0, 0.0)
    for i, L0 in enumerate(prefixes):
        kc, vc, ids = caches[i]
        ref, k_new, v_new = O.gqa_prefill_ref(q[i], k[i], v[i], wt, kc, vc, L0 + pos_offset)
        e = (O.max_err_bf16(out[i], ref), O.rel_rms(out[i], ref))
        worst = (max(worst[0], e[0]), max(worst[1], e[1]))
        rows = (ids[:, None] * 64 + torch.arange(64)[None]).reshape(-1)[L0:L0 + T]
        assert torch.allclose(kp[:, rows].float(), k_new, rtol=2 ** -7, atol=1e-6)
        assert torch.equal(vp[:, rows].float(), v_new)
    print(f"prefixes={prefixes} T={T}: max={worst[0]:.2e} rel_rms={worst[1]:.2e}")
    assert worst[0] < 2e-2 and worst[1] < 1e-2, worst


@pytest.mark.parametrize("T", [1, 100, 128, 129, 300])
def test_prefill_lengths(cuda_device, T):
    _run(cuda_device, [0, 70], T, seed=T)


def test_prefill_long_prefix(cuda_device):
    _run(cuda_device, [1000], 257, seed=3)
