"""Small, self-contained kernel cases for profiler captures and quick timing.

    python router-ia_b200/ria_b200/profile_cases.py --kernel gdn --batch 64 --iters 20
    python router-ia_b200/ria_b200/profile_cases.py --kernel gqa --batch 32 --len 4096 --iters 20
    python router-ia_b200/ria_b200/profile_cases.py --kernel moe --batch 64 --iters 3
    python router-ia_b200/ria_b200/profile_cases.py --kernel head --batch 8 --iters 3
    python router-ia_b200/ria_b200/profile_cases.py --kernel model_step --batch 64
    python router-ia_b200/ria_b200/profile_cases.py --kernel model_prefill --batch 64 --seq 2048
    python router-ia_b200/ria_b200/profile_cases.py --kernel stack --batch 1 --len 4096

Each case allocates only one layer's state (about 1 GB), so a multi-pass
``ncu`` capture of one launch stays small, while one launch still moves more
than the 126 MB L2 (DRAM counters stay meaningful).  Prints the mean CUDA-event
time per launch and the achieved algorithmic bandwidth.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch  # noqa: E402

from ria_b200 import _ext, synthetic  # noqa: E402
from ria_b200 import constants as C  # noqa: E402
from ria_b200.engine import plan_gqa_split  # noqa: E402
from ria_b200.weights import DeltaNetWeights, GqaWeights, rope_inv_freq  # noqa: E402

B_DN = 4_292_736


def gdn_case(batch: int, iters: int, device) -> dict:
    w = DeltaNetWeights.from_tensors(synthetic.layer_weights_on_device(0, device), device)
    g = torch.Generator(device=device)
    g.manual_seed(0)
    rec = torch.randn(batch, 32, 128, 128, device=device, generator=g) * 0.1
    conv = (torch.randn(batch, 8192, 4, device=device, generator=g) * 0.1).to(torch.bfloat16)
    proj = torch.randn(batch, C.DN_PROJ_WIDTH, device=device, generator=g).to(torch.bfloat16)
    out = torch.empty(batch, 4096, dtype=torch.bfloat16, device=device)
    parts = (proj[:, :8192], proj[:, 8192:12288], proj[:, 12288:12320], proj[:, 12320:12352])

    def run():
        _ext.gdn_decode_step(*parts, w.conv_w, w.a_log, w.dt_bias, w.norm_w, conv, rec, None, out)

    ms = _time(run, iters, device)
    return {"kernel": "gdn_decode", "batch": batch, "ms": ms, "gbs": batch * B_DN / (ms * 1e6)}


def gqa_case(batch: int, length: int, iters: int, device) -> dict:
    w = GqaWeights.from_tensors(synthetic.layer_weights_on_device(3, device), device)
    nb = (length + 1 + 63) // 64
    pool_tokens = batch * nb * 64
    g = torch.Generator(device=device)
    g.manual_seed(1)
    k_pool = torch.randn(2, pool_tokens, 256, device=device, generator=g).to(torch.bfloat16)
    v_pool = torch.randn(2, pool_tokens, 256, device=device, generator=g).to(torch.bfloat16)
    table = torch.arange(batch * nb, dtype=torch.int32, device=device).reshape(batch, nb)
    proj = torch.randn(batch, C.GQA_PROJ_WIDTH, device=device, generator=g).to(torch.bfloat16)
    lens = torch.full((batch,), length, dtype=torch.int32, device=device)
    pos = lens.clone()
    out = torch.empty(batch, 4096, dtype=torch.bfloat16, device=device)
    inv = rope_inv_freq(device)
    launch = plan_gqa_split([length + 1] * batch, device)

    def run():
        _ext.gqa_decode_paged(proj[:, :8192], proj[:, 8192:8704], proj[:, 8704:], w.q_norm, w.k_norm, inv, k_pool,
                              v_pool, table, lens, pos, out, launch.workspace, launch.split_pages, launch.max_splits)

    ms = _time(run, iters, device)
    nbytes = batch * (2048 * length + 2048 + 24576)
    return {"kernel": "gqa_decode", "batch": batch, "len": length, "ms": ms, "gbs": nbytes / (ms * 1e6),
            "split_pages": launch.split_pages, "max_splits": launch.max_splits}


PREFILL_FLOP_PER_CHUNK_HEAD = 11_534_336  # 2C^2(3d+2d) + 6 C d^2, C=64, d=128


def prefill_case(batch: int, seq: int, iters: int, device, hk: int = 16, hv: int = 32) -> dict:
    """Benchmark configuration 2 shape by default: 8 x 8192 tokens, 16 key / 32
    value heads, chunk 64, bf16 inputs, fp32 final state."""
    import torch.nn.functional as F

    from ria_b200.prefill import chunk_gated_delta_rule

    g0 = torch.Generator(device=device)
    g0.manual_seed(2)
    q = torch.randn(batch, seq, hk, 128, device=device, generator=g0).to(torch.bfloat16)
    k = torch.randn(batch, seq, hk, 128, device=device, generator=g0).to(torch.bfloat16)
    v = torch.randn(batch, seq, hv, 128, device=device, generator=g0).to(torch.bfloat16)
    a_log = torch.rand(hv, device=device, generator=g0) * 2.7
    dt_bias = torch.rand(hv, device=device, generator=g0) * 2 - 1
    g = (-torch.exp(a_log) * F.softplus(torch.randn(batch, seq, hv, device=device, generator=g0) + dt_bias)).float()
    beta = torch.sigmoid(torch.randn(batch, seq, hv, device=device, generator=g0)).float()
    out = torch.empty(batch, seq, hv, 128, dtype=torch.bfloat16, device=device)
    fs = torch.empty(batch, hv, 128, 128, dtype=torch.float32, device=device)
    ws = torch.empty(_ext.gdn_chunk_prefill_workspace_bytes(batch, seq, hv), dtype=torch.uint8, device=device)

    def run():
        chunk_gated_delta_rule(q, k, v, g, beta, None, fs, out, ws)

    ms = _time(run, iters, device)
    chunks = batch * hv * ((seq + 63) // 64)
    flops = chunks * PREFILL_FLOP_PER_CHUNK_HEAD
    return {"kernel": "gdn_prefill", "batch": batch, "seq": seq, "ms": ms, "tokens_per_s": batch * seq / (ms * 1e-3),
            "tflops": flops / (ms * 1e9)}


def gqa_prefill_case(batch: int, seq: int, iters: int, device) -> dict:
    """One GQA layer prefilling ``seq`` new tokens per sequence (empty cache):
    causal attention FLOPs = 16 heads x 2 x 2 x 256 x seq(seq+1)/2 per sequence."""
    w = GqaWeights.from_tensors(synthetic.layer_weights_on_device(3, device), device)
    nb = (seq + 63) // 64
    g0 = torch.Generator(device=device)
    g0.manual_seed(3)
    k_pool = torch.zeros(2, batch * nb * 64, 256, dtype=torch.bfloat16, device=device)
    v_pool = torch.zeros_like(k_pool)
    table = torch.arange(batch * nb, dtype=torch.int32, device=device).reshape(batch, nb)
    q = torch.randn(batch, seq, C.FULL_Q_GATE_DIM, device=device, generator=g0).to(torch.bfloat16)
    k = torch.randn(batch, seq, C.FULL_KV_DIM, device=device, generator=g0).to(torch.bfloat16)
    v = torch.randn(batch, seq, C.FULL_KV_DIM, device=device, generator=g0).to(torch.bfloat16)
    lens = torch.zeros(batch, dtype=torch.int32, device=device)
    out = torch.empty(batch, seq, 4096, dtype=torch.bfloat16, device=device)
    inv = rope_inv_freq(device)
    ws = [None]

    def run():
        ws[0] = _ext.gqa_prefill(q, k, v, w.q_norm, w.k_norm, inv, k_pool, v_pool, table, lens, lens, out, ws[0])

    ms = _time(run, iters, device)
    flops = batch * 16 * 2 * 2 * 256 * seq * (seq + 1) / 2
    return {"kernel": "gqa_prefill", "batch": batch, "seq": seq, "ms": ms, "tokens_per_s": batch * seq / (ms * 1e-3),
            "tflops": flops / (ms * 1e9)}


def moe_case(batch: int, iters: int, device) -> dict:
    """One layer's MoE block (256 experts top-8 + shared, 1.6 GB of weights)
    for ``batch`` tokens."""
    from ria_b200.engine import MoePlan, moe_decode

    w = synthetic.moe_layer_on_device(41, device)
    g = torch.Generator(device=device)
    g.manual_seed(5)
    x = torch.randn(batch, C.HIDDEN, device=device, generator=g) * 2.0
    plan = MoePlan.create(batch, w.num_experts, device)
    y = torch.empty_like(x)
    ms = _time(lambda: moe_decode(x, w, plan, out=y), iters, device)
    active = len(set(plan.expert_ids.flatten().tolist()))
    return {"kernel": "moe", "batch": batch, "ms": ms, "active_experts": active}


def head_case(batch: int, iters: int, device) -> dict:
    """The greedy head over the fp16 lm_head (151936 x 2048) for ``batch`` rows."""
    from ria_b200.model import HeadWeights, greedy_head

    head = HeadWeights.from_tensors(synthetic.head_weights(1, device=device), device)
    x = torch.randn(batch, C.HIDDEN, device=device)
    ids = torch.empty(batch, dtype=torch.int32, device=device)
    ws = (torch.zeros(_ext.lm_head_workspace_bytes(batch), dtype=torch.uint8, device=device)
          if batch <= _ext.LM_HEAD_MAX_BATCH else None)
    ms = _time(lambda: greedy_head(x, head, ids, ws), iters, device)
    return {"kernel": "head", "batch": batch, "ms": ms, "gb_per_s": head.lm_head.numel() * 2 / (ms * 1e6)}


def model_step_case(batch: int, device) -> dict:
    """Configuration 4's decode step (``batch`` sequences with 2048-token
    prompts, 40 layers with MoE, greedy head): two eager steps, then one in
    the NVTX range ``decode_step`` (for ``ncu --nvtx --nvtx-include``)."""
    model = synthetic.config4_decode_model(device, batch, 2048)
    for _ in range(2):
        model.step()
    torch.cuda.synchronize(device)
    torch.cuda.nvtx.range_push("decode_step")
    model.step()
    torch.cuda.synchronize(device)
    torch.cuda.nvtx.range_pop()
    return {"kernel": "model_step", "batch": batch, "ids": model.ids[:4].tolist()}


def model_prefill_case(batch: int, seq: int, device) -> dict:
    """Configuration 4's prompt prefill (``batch`` sequences x ``seq`` tokens
    through the 40 layers with MoE and the head), the timed pass inside the
    NVTX range ``prefill`` after a short warm-up prefill and a state reset."""
    model = synthetic.config4_decode_model(device, batch, seq, extra_tokens=64, empty=True)
    g = torch.Generator(device=device)
    g.manual_seed(404)
    model.prefill(torch.randint(0, model.head.vocab, (batch, 64), device=device, generator=g, dtype=torch.int32))
    torch.cuda.synchronize(device)
    model.state.reset()
    ids = torch.randint(0, model.head.vocab, (batch, seq), device=device, generator=g, dtype=torch.int32)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    torch.cuda.nvtx.range_push("prefill")
    s.record()
    model.prefill(ids)
    e.record()
    torch.cuda.synchronize(device)
    torch.cuda.nvtx.range_pop()
    return {"kernel": "model_prefill", "batch": batch, "seq": seq, "ms": s.elapsed_time(e)}


def stack_case(batch: int, length: int, iters: int, device) -> dict:
    """The 40-layer decode step without MoE (30 DeltaNet + 10 GQA layers,
    ``length`` cached tokens per sequence on every GQA layer): mean eager and
    CUDA-graph-replay times per token, then one eager step in the NVTX range
    ``stack_step`` (for ``ncu --nvtx --nvtx-include``)."""
    from ria_b200.engine import BatchedAttentionState, DecodeGraph

    layers = {}
    for layer in range(C.NUM_LAYERS):
        t = synthetic.layer_weights_on_device(layer, device, seed=0)
        cls = GqaWeights if C.is_full_attention_layer(layer) else DeltaNetWeights
        layers[layer] = cls.from_tensors(t, device)
        del t
    nb = (length + 2 * iters + 128) // C.KV_BLOCK + 2
    eng = BatchedAttentionState(layers, batch=batch, pool_blocks=nb * batch, max_blocks_per_seq=nb, device=device)
    g = torch.Generator(device=device)
    g.manual_seed(7)
    for layer in eng.rec:
        eng.rec[layer].normal_(0.0, 0.1, generator=g)
    for layer in eng.k_pool:
        eng.k_pool[layer].normal_(0.0, 1.0, generator=g)
        eng.v_pool[layer].normal_(0.0, 1.0, generator=g)
    for i in range(batch):
        eng.set_length(i, length)
    eng.sync_tables()
    x = torch.randn(batch, C.HIDDEN, device=device, generator=g)
    eager_ms = _time(lambda: eng.step(x), iters, device)
    graph = DecodeGraph(eng)
    graph_ms = _time(lambda: graph.step(x), iters, device)
    del graph
    torch.cuda.nvtx.range_push("stack_step")
    eng.step(x)
    torch.cuda.synchronize(device)
    torch.cuda.nvtx.range_pop()
    return {"kernel": "stack", "batch": batch, "len": length, "eager_ms": eager_ms, "graph_ms": graph_ms}


def _time(fn, iters, device):
    for _ in range(3):
        fn()
    torch.cuda.synchronize(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize(device)
    return s.elapsed_time(e) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", choices=("gdn", "gqa", "prefill", "gqa_prefill", "moe", "head", "model_step",
                                         "model_prefill", "stack", "all"),
                    default="all")
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--len", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.kernel in ("gdn", "all"):
        print(gdn_case(args.batch, args.iters, dev), flush=True)
    if args.kernel in ("gqa", "all"):
        print(gqa_case(args.batch if args.kernel == "gqa" else max(1, args.batch // 2), args.len, args.iters, dev),
              flush=True)
    if args.kernel == "gqa_prefill":
        print(gqa_prefill_case(args.batch, args.seq, args.iters, dev), flush=True)
    if args.kernel == "prefill":
        print(prefill_case(args.batch, args.seq, args.iters, dev), flush=True)
    if args.kernel == "moe":
        print(moe_case(args.batch, args.iters, dev), flush=True)
    if args.kernel == "head":
        print(head_case(args.batch, args.iters, dev), flush=True)
    if args.kernel == "model_step":
        print(model_step_case(args.batch, dev), flush=True)
    if args.kernel == "model_prefill":
        print(model_prefill_case(args.batch, args.seq, dev), flush=True)
    if args.kernel == "stack":
        print(stack_case(args.batch, args.len, args.iters, dev), flush=True)
    if _ext.device_error():
        raise SystemExit("device error word set")


if __name__ == "__main__":
    main()
