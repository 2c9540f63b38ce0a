"""Benchmark configuration 3 at full size, one layer of each kind: 256
sequences whose KV lengths are the benchmark's stratified sample of
U[512, 32768] (4.26M cached tokens, 8.7 GB of bf16 KV on the GQA layer),
DeltaNet and conv states ~ N(0, 0.1), KV ~ N(0, 1) -- the decode step the
headline times, checked against the oracle's restatement of router-ia's CPU
path (qwen36_attention_cache.py:224-324) on sampled sequences: the shortest,
the longest, the median and two seeded others.

Each layer gets the same input rows on both sides (teacher-forced, as in
tests/test_engine_gpu.py).  Bars, per sequence: the fp32 residual within
2e-2 max-abs and its attention contribution within 1e-2 relative RMS; the
DeltaNet state after the step within 1e-2 relative RMS (layer level: the
state's inputs are bf16 projection outputs); the appended K and V rows
within 1e-2 relative RMS of the oracle's (which come from fp32
projections)."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from ria_b200 import constants as C
from ria_b200.engine import BatchedAttentionState, deltanet_decode, gqa_decode
from ria_b200.weights import DeltaNetWeights, GqaWeights

pytestmark = pytest.mark.gpu

_PROJ = ("in_proj_qkv", "in_proj_z", "in_proj_a", "in_proj_b", "out_proj", "q_proj", "k_proj", "v_proj", "o_proj")


def _oracle_weights(wt: dict) -> dict:
    return {k: (v.float() if any(p in k for p in _PROJ) else v) for k, v in wt.items()}


def test_configuration3_full_size_sampled_sequences(cuda_device):
    dev = cuda_device
    B = 256
    lengths = synthetic.stratified_lengths(B, 512, 32768, seed=0)
    assert sum(lengths) > 4_000_000
    wt_dn, wt_gqa = synthetic.layer_weights(0, 0), synthetic.layer_weights(3, 0)
    w_dn, w_gqa = DeltaNetWeights.from_tensors(wt_dn, dev), GqaWeights.from_tensors(wt_gqa, dev)
    blocks = [(n + 2 + C.KV_BLOCK - 1) // C.KV_BLOCK for n in lengths]
    eng = BatchedAttentionState({0: w_dn, 3: w_gqa}, batch=B, pool_blocks=sum(blocks) + 8,
                                max_blocks_per_seq=max(blocks) + 1, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(33)
    eng.rec[0].normal_(0.0, 0.1, generator=g)
    eng.conv[0].normal_(0.0, 0.1, generator=g)
    eng.k_pool[3].normal_(0.0, 1.0, generator=g)
    eng.v_pool[3].normal_(0.0, 1.0, generator=g)
    for i, n in enumerate(lengths):
        eng.set_length(i, n, position=n + 9)
    eng.sync_tables()
    order = sorted(range(B), key=lambda i: lengths[i])
    picks = [order[0], order[-1], order[B // 2]] + torch.randperm(B, generator=torch.Generator().manual_seed(3))[:2].tolist()
    before = {}
    for i in picks:
        rows = eng.physical_rows(i, lengths[i]).to(dev)
        before[i] = (eng.rec[0][i:i + 1].cpu(), eng.conv[0][i:i + 1].cpu(),
                     eng.k_pool[3][:, rows].float().cpu().unsqueeze(0), eng.v_pool[3][:, rows].float().cpu().unsqueeze(0))
    x = torch.randn(B, C.HIDDEN, device=dev, generator=g).to(torch.bfloat16).float()

    eng.reserve_next()
    launch = eng.plan()
    out_dn = deltanet_decode(x, w_dn, eng.rec[0], eng.conv[0])
    out_gqa = gqa_decode(x, w_gqa, eng.k_pool[3], eng.v_pool[3], eng.block_table, eng.inv_freq, launch, eng.seq_lens,
                         eng.positions)
    torch.cuda.synchronize()
    assert _ext.device_error() == 0
    assert O.finite(out_dn) and O.finite(out_gqa)

    ow_dn, ow_gqa = _oracle_weights(wt_dn), _oracle_weights(wt_gqa)
    xc = x.cpu()
    for i in picks:
        n = lengths[i]
        rec0, conv0, kc, vc = before[i]
        xin = xc[i:i + 1]
        ref, conv1, rec1 = O.deltanet_step(ow_dn, xin, conv0, rec0)
        got = out_dn[i:i + 1].cpu()
        e_dn = (O.max_abs(got, ref), O.rel_rms(got - xin, ref - xin), O.rel_rms(eng.rec[0][i:i + 1].cpu(), rec1))
        ref_g, kc1, vc1 = O.gqa_step(ow_gqa, xin, kc, vc, n + 9)
        got_g = out_gqa[i:i + 1].cpu()
        e_g = (O.max_abs(got_g, ref_g), O.rel_rms(got_g - xin, ref_g - xin))
        print(f"seq {i} (KV {n}): DeltaNet max_abs={e_dn[0]:.2e} rel_rms={e_dn[1]:.2e} state={e_dn[2]:.2e}; "
              f"GQA max_abs={e_g[0]:.2e} rel_rms={e_g[1]:.2e}")
        assert e_dn[0] < 2e-2 and e_dn[1] < 1e-2 and e_dn[2] < 1e-2, (i, n, e_dn)
        assert e_g[0] < 2e-2 and e_g[1] < 1e-2, (i, n, e_g)
        row = int(eng.physical_rows(i, n + 1)[n])
        k_new = eng.k_pool[3][:, row].float().cpu()
        v_new = eng.v_pool[3][:, row].float().cpu()
        # the oracle appended fp32 K/V of its own fp32 projections: within
        # the bf16 projection rounding of this path
        assert O.rel_rms(k_new, kc1[0, :, n]) < 1e-2 and O.rel_rms(v_new, vc1[0, :, n]) < 1e-2
