"""The greedy head (final RMSNorm, fp16 lm_head, argmax) against the CPU
oracle of router-ia's CUDA path (fp16 autocast: operands rounded to fp16,
fp32 sums, fp16 logits; qwen36_chat_batch.py:194-199 and sample_next at
temperature 0, qwen36_mini_chat.py:75-78), which tests/test_oracle_golden.py
pins to the reference's own functions.

Both sides round the same fp32 sums to fp16 but add them in different
orders, so a logit may land one fp16 step away: logits are checked to 2e-3 of
max(1, |ref|) (one step at 1.0 is 9.8e-4).  The picked id equals the
oracle's unless the oracle's best two logits are that close, in which case
the pick must be one of them."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from ria_b200.model import HeadWeights, greedy_head

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _head(vocab: int, dev, seed: int = 51):
    t = synthetic.head_weights(seed, vocab=vocab, device=dev)
    return t, HeadWeights.from_tensors(t, dev)


def _inputs(batch: int, seed: int, dev) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(batch, 2048, generator=g) * 3.0).to(dev)


def _check(t, x, ids, logits=None):
    ref_logits, ref_ids = O.lm_head_greedy(x.cpu(), t["model.language_model.norm.weight"].cpu(),
                                           t["lm_head.weight"].cpu(), fp16=True)
    if logits is not None:
        assert O.max_err_bf16(logits.float().cpu(), ref_logits) < TOL
    got = ids.cpu().long()
    for b in range(x.shape[0]):
        if got[b] != ref_ids[b]:
            top = ref_logits[b].max()
            assert top - ref_logits[b, got[b]] <= TOL * max(1.0, abs(float(top))), (b, int(got[b]), int(ref_ids[b]))


@pytest.mark.parametrize("batch", [1, 3, 8])
@pytest.mark.parametrize("vocab", [1001, 151936])
def test_fused_head_matches_oracle(cuda_device, batch, vocab):
    t, head = _head(vocab, cuda_device)
    x = _inputs(batch, 7 + batch, cuda_device)
    ids = torch.empty(batch, dtype=torch.int32, device=cuda_device)
    logits = torch.empty(batch, vocab, dtype=torch.float16, device=cuda_device)
    greedy_head(x, head, ids, logits=logits)
    torch.cuda.synchronize()
    _check(t, x, ids, logits)
    # the logits the library GEMM path computes: same picks
    h = torch.empty(batch, 2048, dtype=torch.float16, device=cuda_device)
    _ext.final_norm_f16(x, head.final_norm, h)
    lib = F.linear(h, head.lm_head)
    assert O.max_err_bf16(logits.float(), lib.float()) < TOL


def test_large_batch_head_matches_oracle(cuda_device):
    """64 rows: fp16 norm kernel, library GEMM, row argmax kernel."""
    t, head = _head(151936, cuda_device)
    x = _inputs(64, 3, cuda_device)
    ids = torch.empty(64, dtype=torch.int32, device=cuda_device)
    logits = torch.empty(64, 151936, dtype=torch.float16, device=cuda_device)
    greedy_head(x, head, ids, logits=logits)
    torch.cuda.synchronize()
    _check(t, x, ids, logits)
    assert torch.equal(ids.long(), logits.float().argmax(dim=-1))


def test_equal_maxima_pick_the_first_row(cuda_device):
    """Two identical lm_head rows that give the largest logit: the lower index
    wins, as torch.argmax picks.  Both head paths."""
    vocab = 50000
    t, head = _head(vocab, cuda_device, seed=52)
    x = _inputs(1, 9, cuda_device)
    hrow = torch.empty(1, 2048, dtype=torch.float16, device=cuda_device)
    _ext.final_norm_f16(x, head.final_norm, hrow)
    row = (0.05 * torch.sign(hrow[0].float())).to(torch.float16)
    head.lm_head[7] = row
    head.lm_head[40000] = row
    ids = torch.empty(1, dtype=torch.int32, device=cuda_device)
    greedy_head(x, head, ids)
    torch.cuda.synchronize()
    assert int(ids[0]) == 7
    x10 = x.repeat(10, 1)
    ids10 = torch.empty(10, dtype=torch.int32, device=cuda_device)
    greedy_head(x10, head, ids10)
    torch.cuda.synchronize()
    assert ids10.tolist() == [7] * 10


def test_repeated_calls_reuse_the_workspace(cuda_device):
    """The hand-off counter returns to zero: consecutive calls on one
    workspace give the same picks, and different inputs their own."""
    t, head = _head(1001, cuda_device)
    ws = torch.zeros(_ext.lm_head_workspace_bytes(4), dtype=torch.uint8, device=cuda_device)
    ids = torch.empty(4, dtype=torch.int32, device=cuda_device)
    results = []
    for seed in (1, 2, 1):
        x = _inputs(4, seed, cuda_device)
        greedy_head(x, head, ids, ws)
        torch.cuda.synchronize()
        _check(t, x, ids)
        results.append(ids.clone())
    assert torch.equal(results[0], results[2])
    assert int(ws[:4].view(torch.int32)[0]) == 0


def test_head_argument_errors(cuda_device):
    t, head = _head(1001, cuda_device)
    x = _inputs(9, 1, cuda_device)
    ids = torch.empty(9, dtype=torch.int32, device=cuda_device)
    ws = torch.zeros(_ext.lm_head_workspace_bytes(8), dtype=torch.uint8, device=cuda_device)
    with pytest.raises(ValueError, match="batch"):
        _ext.lm_head_greedy(x, head.final_norm, head.lm_head, ids, ws)
    with pytest.raises(ValueError, match="workspace"):
        _ext.lm_head_greedy(x[:2], head.final_norm, head.lm_head, ids, ws[:64])
