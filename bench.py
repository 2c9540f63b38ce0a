"""Benchmark of the stateful hybrid attention hot path on B200.

Workload (N=1): benchmark configuration 3, the batched ragged hybrid decode
step -- 256 sequences with KV lengths uniform in [512, 32768] (seeded), 64-token
paged bf16 KV, fp32 DeltaNet states and bf16 conv states ~ N(0, 0.1), KV ~ N(0, 1),
random-init weights of the 40-layer 3:1 stack (30 Gated DeltaNet + 10 GQA).
One step = every layer's attention (input norm, projections, fused kernel,
output projection, residual) for all 256 sequences: one decoded token per
sequence.  Metric: decode tokens/s (whole job) with the fraction of the HBM
roofline of the dominant kernel.

Multi-GPU (torchrun): each rank decodes its own 256 sequences (weak scaling, no
collective on the path); the elapsed time is the max over ranks.  Two more
multi-GPU lines ride along at N > 1: the fixed 256-sequence job split 256/N
per GPU (strong scaling) and benchmark configuration 4 with 64 requests per
GPU (512 at N = 8).

``--impl reference`` times router-ia itself: the unmodified reference package
installed under ``baseline/_ref`` (its ``qwen36_attention_cache.step_attention``
on the host cores, one sequence at a time as router-ia runs, through a
synthetic safetensors checkpoint) on a bounded sample of the same workload.
The ``cpu_baseline`` of this arm's own line is the CPU oracle port of the same
layer steps (weights converted to fp32 once).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (str(REPO / "router-ia_b200"), str(REPO)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "attn decode tokens/s/GPU + %HBM peak; DeltaNet chunked prefill tokens/s"
REF_DIR = REPO / "baseline" / "_ref"  # the unmodified reference, pip-installed here
UNIT = "tokens/s"
B_DN = 4_292_736  # algorithmic bytes of K1 per (sequence, layer)
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) over algorithmic
# bytes, from one ncu capture of each kernel on a small case (K3: 32
# sequences at 4096 cached tokens, 280.3 of 269.3 MB; K1: 64 sequences,
# 222.0 of 274.7 MB, the written state partly still in L2 at kernel end).
# Traffic of a full launch = ratio x its algorithmic bytes.
TRAFFIC_RATIO = {"gqa_decode": 280.3 / 269.3, "gdn_decode": 222.0 / 274.7}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--len-lo", type=int, default=512)
    ap.add_argument("--len-hi", type=int, default=32768)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--cpu-sample", type=int, default=4, help="sequences in the CPU baseline sample")
    ap.add_argument("--reference-gpu-anchor", action="store_true",
                    help="(internal) time the reference's own attention on cuda:0 and print one JSON line")
    return ap.parse_args()


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return dict(PEAKS_FALLBACK, source="fallback")


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.path = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.gpu = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            self.gpu = str(device.index or 0)

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        def num(x):
            try:
                return float(x)
            except ValueError:
                return float("nan")
        sm = [num(r[1]) for r in rows]
        power = [num(r[3]) for r in rows]
        pmax = max(p for p in power if not math.isnan(p)) if any(not math.isnan(p) for p in power) else 0
        loaded = [s for s, p in zip(sm, power) if p >= 0.5 * pmax] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in rows for j in range(4) if r[5 + j].lower().startswith("active")})
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(num(r[2]) for r in rows),
                "reasons": reasons, "samples": len(rows), "power_w_max": pmax}


# --------------------------------------------------------------------------- launch instrumentation
class EventHook:
    """CUDA events around each kernel-launching library call (on the current
    stream, which is the launch stream) plus a launch counter."""

    def __init__(self, timed=("gqa_decode", "gdn_decode")):
        self.timed = set(timed)
        self.events: dict[str, list] = {n: [] for n in timed}
        self.launches = 0
        self._open = None

    def before(self, name):
        if name in self.timed:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._open = e

    def after(self, name, kernels):
        self.launches += kernels
        if name in self.timed:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.events[name].append((self._open, e))

    def mean_ms(self, name):
        pairs = self.events[name]
        return sum(a.elapsed_time(b) for a, b in pairs) / max(1, len(pairs)), len(pairs)


# --------------------------------------------------------------------------- workload
def build_layers(device):
    """The 40-layer stack's attention weights, seeded random init on the device."""
    from ria_b200 import constants as C, synthetic
    from ria_b200.weights import DeltaNetWeights, GqaWeights

    layers = {}
    for layer in range(C.NUM_LAYERS):
        t = synthetic.layer_weights_on_device(layer, device, seed=0)
        cls = GqaWeights if C.is_full_attention_layer(layer) else DeltaNetWeights
        layers[layer] = cls.from_tensors(t, device)
        del t
    return layers


def weak_lengths(args, rank, world):
    """Each rank decodes args.batch sequences whose KV lengths are a stratified
    sample of U[len_lo, len_hi] (the same multiset on every rank and at every
    GPU count: weak scaling with fixed work per GPU).  The job's request list
    is the ranks' lists concatenated; the cost-balanced assignment keeps each
    rank's list."""
    from ria_b200 import synthetic
    from ria_b200.sharding import balanced_assignment

    per_rank = synthetic.stratified_lengths(args.batch, args.len_lo, args.len_hi, seed=0)
    requests = per_rank * world
    return [requests[i] for i in balanced_assignment(requests, world)[rank]]


def strong_lengths(args, rank, world):
    """The fixed job of args.batch sequences (the N = 1 workload) split over
    the ranks by the cost-balanced assignment: args.batch / world each."""
    from ria_b200 import synthetic
    from ria_b200.sharding import balanced_assignment

    requests = synthetic.stratified_lengths(args.batch, args.len_lo, args.len_hi, seed=0)
    return [requests[i] for i in balanced_assignment(requests, world)[rank]]


def build_engine(args, device, rank, world, headroom, layers, lengths):
    from ria_b200 import constants as C
    from ria_b200.engine import BatchedAttentionState

    blocks = [math.ceil((n + headroom) / C.KV_BLOCK) for n in lengths]
    eng = BatchedAttentionState(layers, batch=len(lengths), pool_blocks=sum(blocks) + 8,
                                max_blocks_per_seq=max(blocks) + 1, device=device)
    g = torch.Generator(device=device)
    g.manual_seed(1234 + rank)
    for layer in eng.rec:
        eng.rec[layer].normal_(0.0, 0.1, generator=g)
        eng.conv[layer].normal_(0.0, 0.1, generator=g)
    for layer in eng.k_pool:
        eng.k_pool[layer].normal_(0.0, 1.0, generator=g)
        eng.v_pool[layer].normal_(0.0, 1.0, generator=g)
    for i, n in enumerate(lengths):
        eng.set_length(i, n)
    eng.sync_tables()
    torch.cuda.synchronize(device)
    return eng, lengths


def gqa_bytes(lengths):
    """Algorithmic bytes of one K3 launch: KV read 2048 B/token, the appended
    token 2048 B, q+gate in and output (3 x 16 x 256 x 2 B) per sequence."""
    return sum(2048 * n + 2048 + 24576 for n in lengths)


def run_ours(args, rank, world, device, layers):
    from ria_b200 import _ext

    headroom = args.warmup + 2 * args.steps + 4
    t_setup = time.perf_counter()
    eng, lengths = build_engine(args, device, rank, world, headroom, layers, weak_lengths(args, rank, world))
    setup_s = time.perf_counter() - t_setup
    x = torch.randn(args.batch, 2048, device=device).to(torch.bfloat16).float()

    for _ in range(args.warmup):
        eng.step(x)
    torch.cuda.synchronize(device)
    _ext.device_error()
    barrier(world, device)

    hook = EventHook()
    _ext.launch_hook = hook
    lens_timed = []
    clocks = ClockSampler(device)
    clocks.start()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    start.record()
    for _ in range(args.steps):
        lens_timed.append(list(eng.lengths))
        eng.step(x)
    end.record()
    torch.cuda.synchronize(device)
    _ext.launch_hook = None
    clock_info = clocks.stop()
    elapsed_ms = start.elapsed_time(end)
    elapsed_ms = reduce_max(elapsed_ms, world, device)
    barrier(world, device)

    # e2e: host inputs in pinned memory, copies inside the timed region
    x_h = torch.empty(args.batch, 2048, dtype=torch.float32, pin_memory=True)
    x_h.copy_(x.cpu())
    y_h = torch.empty_like(x_h, pin_memory=True)
    x_d = torch.empty_like(x)
    torch.cuda.synchronize(device)
    barrier(world, device)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        x_d.copy_(x_h, non_blocking=True)
        y = eng.step(x_d)
        y_h.copy_(y, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()
    t1.record()
    torch.cuda.synchronize(device)
    e2e_ms = reduce_max(t0.elapsed_time(t1), world, device)
    from ria_b200.sharding import gather_to_rank0

    per_rank = gather_to_rank0({"rank": rank, "device_error": _ext.device_error(), "seqs": len(lengths),
                                "ms": elapsed_ms}, world)
    dev_err = max(r["device_error"] for r in per_rank)

    p = peaks()
    gqa_ms, gqa_n = hook.mean_ms("gqa_decode")
    gdn_ms, gdn_n = hook.mean_ms("gdn_decode")
    gqa_b = statistics.mean(gqa_bytes(ls) for ls in lens_timed)
    gdn_b = args.batch * B_DN
    kernels = {
        "gqa_decode": {"ms_per_launch": gqa_ms, "launches": gqa_n, "bytes_per_launch": gqa_b,
                       "achieved_gbs": gqa_b / (gqa_ms * 1e6), "frac": gqa_b / (gqa_ms * 1e6) / p["hbm_gbs"]},
        "gdn_decode": {"ms_per_launch": gdn_ms, "launches": gdn_n, "bytes_per_launch": gdn_b,
                       "achieved_gbs": gdn_b / (gdn_ms * 1e6), "frac": gdn_b / (gdn_ms * 1e6) / p["hbm_gbs"]},
    }
    dom = max(kernels, key=lambda k: kernels[k]["ms_per_launch"] * kernels[k]["launches"])
    step_bytes = 10 * gqa_b + 30 * gdn_b
    tokens = world * args.batch * args.steps
    line = {
        "metric": METRIC,
        "value": tokens / (elapsed_ms / 1e3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 I/O, fp32 state/accumulate",
        "data": "synthetic (seeded random-init weights, N(0,0.1) states, N(0,1) KV)",
        "config": {
            "workload": "config3: batched ragged hybrid decode step, 30 DeltaNet + 10 GQA layers",
            "sequences_per_gpu": args.batch,
            "kv_len_range": [args.len_lo, args.len_hi],
            "kv_tokens_per_gpu": sum(lengths),
            "kv_block_tokens": 64,
            "parallelism": f"sequence-sharded x{world}, KV-length-balanced (no collective)",
            "l2": "inputs larger than L2 (state+KV ~%.0f GB per step)" % (step_bytes / 1e9),
        },
        "roofline": {
            "kernel": dom, "bound": "hbm", "achieved": kernels[dom]["achieved_gbs"], "peak": p["hbm_gbs"],
            "unit": "GB/s", "frac": kernels[dom]["frac"], "peak_source": p["source"],
            "traffic": TRAFFIC_RATIO[dom] * kernels[dom]["bytes_per_launch"],
            "traffic_source": "ncu small-case ratio x full-launch algorithmic bytes",
        },
        "kernels": kernels,
        "step_hbm_fraction": step_bytes / ((elapsed_ms / args.steps) * 1e6) / p["hbm_gbs"],
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": UNIT,
                "h2d_bytes_per_step": args.batch * 2048 * 4, "d2h_bytes_per_step": args.batch * 2048 * 4},
        "gpu_launches": hook.launches,
        "clocks": clock_info,
        "setup_s": round(setup_s, 1),
        "device_error": dev_err,
    }
    del eng
    torch.cuda.empty_cache()
    return line


def barrier(world, device):
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[device.index])


def reduce_max(v, world, device):
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------- extras (rank 0)
def config1_latency(device, iters=50):
    """Benchmark configuration 1: one GQA layer decode step, batch 1, 4096
    cached tokens (bf16 KV N(0,1)); returns step and kernel times."""
    from ria_b200 import _ext, synthetic
    from ria_b200.engine import gqa_decode, plan_gqa_split
    from ria_b200.weights import GqaWeights, rope_inv_freq

    w = GqaWeights.from_tensors(synthetic.layer_weights_on_device(3, device), device)
    L = 4096
    k = torch.randn(2, 8192, 256, device=device).to(torch.bfloat16)
    v = torch.randn(2, 8192, 256, device=device).to(torch.bfloat16)
    table = torch.arange(128, dtype=torch.int32, device=device).reshape(1, -1)
    inv = rope_inv_freq(device)
    launch = plan_gqa_split([L + 1], device)
    x = torch.randn(1, 2048, device=device)
    for _ in range(10):
        gqa_decode(x, w, k, v, table, inv, launch, seq_len0=L, position0=L)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    s.record()
    for _ in range(iters):
        gqa_decode(x, w, k, v, table, inv, launch, seq_len0=L, position0=L)
    e.record()
    torch.cuda.synchronize(device)
    step_ms = s.elapsed_time(e) / iters
    # the attention kernel (K3 and its split combine) on its own, from a fixed
    # projection row (at batch 1 the layer step issues it inside one C call)
    from ria_b200 import constants as C

    proj = torch.randn(1, C.GQA_PROJ_WIDTH, device=device).to(torch.bfloat16)
    attn = torch.empty(1, C.FULL_Q_DIM, dtype=torch.bfloat16, device=device)
    qkv = [proj[:, a:b] for a, b in (C.GQA_PROJ_Q, C.GQA_PROJ_K, C.GQA_PROJ_V)]

    def attention():
        _ext.gqa_decode_paged(*qkv, w.q_norm, w.k_norm, inv, k, v, table, None, None, attn, launch.workspace,
                              launch.split_pages, launch.max_splits, seq_len0=L, position0=L)

    for _ in range(10):
        attention()
    hook = EventHook(timed=("gqa_decode",))
    _ext.launch_hook = hook
    for _ in range(iters):
        attention()
    torch.cuda.synchronize(device)
    _ext.launch_hook = None
    kms, _ = hook.mean_ms("gqa_decode")
    # the same layer step replayed from a CUDA graph (no per-launch host work)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        gqa_decode(x, w, k, v, table, inv, launch, seq_len0=L, position0=L)
    for _ in range(10):
        graph.replay()
    torch.cuda.synchronize(device)
    s.record()
    for _ in range(iters):
        graph.replay()
    e.record()
    torch.cuda.synchronize(device)
    graph_ms = s.elapsed_time(e) / iters
    kbytes = gqa_bytes([L])
    return {"layer_step_us": step_ms * 1e3, "layer_step_graph_us": graph_ms * 1e3, "gqa_kernel_us": kms * 1e3,
            "kernel_bytes": kbytes, "kernel_gbs": kbytes / (kms * 1e6), "split_pages": launch.split_pages,
            "splits": launch.max_splits}


def config0_deltanet(device, prompt=64, decode=64, reps=5):
    """Benchmark configuration 0: one Gated DeltaNet layer, batch 1, a
    64-token prompt through the chunked prefill (K2 + conv/gate/norm kernels)
    then 64 decode tokens replayed from a CUDA graph (K1), from a zero state.
    One long-lived state serves every request, reset between them (the
    cache's reset-per-turn); after one warm-up request, each of ``reps``
    timed requests is prefill + decode.  Reports tokens/s over the 128 tokens
    of the best request and each phase's time."""
    from ria_b200 import constants as C, synthetic
    from ria_b200.engine import BatchedAttentionState, DecodeGraph
    from ria_b200.weights import DeltaNetWeights

    w = {0: DeltaNetWeights.from_tensors(synthetic.layer_weights_on_device(0, device, seed=0), device)}
    g = torch.Generator(device=device)
    g.manual_seed(11)
    xp = torch.randn(1, prompt, C.HIDDEN, device=device, generator=g).to(torch.bfloat16).float()
    xd = torch.randn(decode, 1, C.HIDDEN, device=device, generator=g).to(torch.bfloat16).float()
    s, m, e = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    nb = (prompt + decode + 2) // C.KV_BLOCK + 2  # the page bookkeeping runs even without GQA layers
    eng = BatchedAttentionState(w, batch=1, pool_blocks=nb, max_blocks_per_seq=nb, device=device)
    eng.step(xd[0])  # library and cuBLAS initialisation outside capture
    eng.reset()
    graph = DecodeGraph(eng)
    best = None
    for rep in range(reps + 1):
        eng.reset()
        torch.cuda.synchronize(device)
        s.record()
        eng.prefill(xp)
        m.record()
        for t in range(decode):
            graph.step(xd[t])
        e.record()
        torch.cuda.synchronize(device)
        r = (s.elapsed_time(m), m.elapsed_time(e))
        if rep > 0:  # request 0 warms the allocator and the prompt-path GEMMs
            best = r if best is None or sum(r) < sum(best) else best
    del graph, eng
    return {"workload": f"config0: one DeltaNet layer, batch 1, {prompt} prompt + {decode} decode tokens",
            "tokens_per_s": (prompt + decode) / (sum(best) * 1e-3), "prefill_ms": best[0],
            "decode_ms_per_token": best[1] / decode, "best_of": reps}


def decode_b1_stack(device, L=4096, iters=30):
    """One sequence through the whole 40-layer stack per token (config 1's
    context length on every GQA layer): per-token latency of the eager step
    and of the step replayed from a CUDA graph (DecodeGraph)."""
    from ria_b200 import constants as C, synthetic
    from ria_b200.engine import BatchedAttentionState, DecodeGraph
    from ria_b200.weights import DeltaNetWeights, GqaWeights

    layers = {}
    for layer in range(C.NUM_LAYERS):
        t = synthetic.layer_weights_on_device(layer, device, seed=0)
        cls = GqaWeights if C.is_full_attention_layer(layer) else DeltaNetWeights
        layers[layer] = cls.from_tensors(t, device)
        del t
    nb = (L + 2 * iters + 64) // C.KV_BLOCK + 2
    eng = BatchedAttentionState(layers, batch=1, pool_blocks=nb, max_blocks_per_seq=nb, device=device)
    g = torch.Generator(device=device)
    g.manual_seed(7)
    for layer in eng.rec:
        eng.rec[layer].normal_(0.0, 0.1, generator=g)
    for layer in eng.k_pool:
        eng.k_pool[layer].normal_(0.0, 1.0, generator=g)
        eng.v_pool[layer].normal_(0.0, 1.0, generator=g)
    eng.set_length(0, L)
    eng.sync_tables()
    x = torch.randn(1, C.HIDDEN, device=device, generator=g)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        eng.step(x)
    torch.cuda.synchronize(device)
    s.record()
    for _ in range(iters):
        eng.step(x)
    e.record()
    torch.cuda.synchronize(device)
    eager_ms = s.elapsed_time(e) / iters
    graph = DecodeGraph(eng)
    for _ in range(3):
        graph.step(x)
    torch.cuda.synchronize(device)
    s.record()
    for _ in range(iters):
        graph.step(x)
    e.record()
    torch.cuda.synchronize(device)
    graph_ms = s.elapsed_time(e) / iters
    del graph, eng, layers
    return {"workload": f"1 sequence, 30 DeltaNet + 10 GQA layers, {L} cached tokens", "eager_ms_per_token": eager_ms,
            "graph_ms_per_token": graph_ms, "graph_tokens_per_s": 1e3 / graph_ms}


PREFILL_FLOP_PER_CHUNK_HEAD = 11_534_336  # 2C^2(3d + 2d) + 6 C d^2 with C = 64, d = 128


def config2_prefill(device, iters=5, warmup=3):
    """Benchmark configuration 2: chunked Gated DeltaNet prefill, 8 sequences x
    8192 tokens, 16 key / 32 value heads, chunk 64, bf16 inputs, fp32 final
    state.  Tensor-bound: reported against the bf16 dense peak."""
    import torch.nn.functional as F

    from ria_b200 import _ext
    from ria_b200.prefill import chunk_gated_delta_rule

    B, T, Hk, Hv = 8, 8192, 16, 32
    g0 = torch.Generator(device=device)
    g0.manual_seed(2)
    q = torch.randn(B, T, Hk, 128, device=device, generator=g0).to(torch.bfloat16)
    k = torch.randn(B, T, Hk, 128, device=device, generator=g0).to(torch.bfloat16)
    v = torch.randn(B, T, Hv, 128, device=device, generator=g0).to(torch.bfloat16)
    a_log = torch.rand(Hv, device=device, generator=g0) * 2.7
    dt_bias = torch.rand(Hv, device=device, generator=g0) * 2 - 1
    g = (-torch.exp(a_log) * F.softplus(torch.randn(B, T, Hv, device=device, generator=g0) + dt_bias)).float()
    beta = torch.sigmoid(torch.randn(B, T, Hv, device=device, generator=g0)).float()
    out = torch.empty(B, T, Hv, 128, dtype=torch.bfloat16, device=device)
    fs = torch.empty(B, Hv, 128, 128, dtype=torch.float32, device=device)
    ws = torch.empty(_ext.gdn_chunk_prefill_workspace_bytes(B, T, Hv), dtype=torch.uint8, device=device)
    for _ in range(warmup):
        chunk_gated_delta_rule(q, k, v, g, beta, None, fs, out, ws)
    hook = EventHook(timed=("gdn_prefill",))
    _ext.launch_hook = hook
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    s.record()
    for _ in range(iters):
        chunk_gated_delta_rule(q, k, v, g, beta, None, fs, out, ws)
    e.record()
    torch.cuda.synchronize(device)
    _ext.launch_hook = None
    ms = s.elapsed_time(e) / iters
    kms, _ = hook.mean_ms("gdn_prefill")
    flops = B * Hv * ((T + 63) // 64) * PREFILL_FLOP_PER_CHUNK_HEAD
    p = peaks()
    cpu = None
    if int(os.environ.get("WORLD_SIZE", "1")) == 1:
        # the reference's chunked rule (oracle restatement of transformers'
        # torch_chunk_gated_delta_rule) on the host cores, bounded sample
        from oracle import attention_oracle as O

        torch.set_num_threads(os.cpu_count() or 1)
        Ts = 1024
        qc, kc, vc = (x[:1, :Ts].float().cpu() for x in (q, k, v))
        qc = qc.repeat_interleave(Hv // Hk, 2)
        kc = kc.repeat_interleave(Hv // Hk, 2)
        gc, bc = g[:1, :Ts].cpu(), beta[:1, :Ts].cpu()
        t0 = time.perf_counter()
        O.chunk_gated_delta_rule(qc, kc, vc, gc, bc)
        dt = time.perf_counter() - t0
        cpu = {"value": Ts / dt, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"1 x {Ts} tokens x {Hv} heads through the chunked rule (fp32, chunk 64)"}
    return {"workload": "config2: chunked DeltaNet prefill 8 x 8192, 32 heads, chunk 64", "tokens_per_s": B * T / (ms * 1e-3),
            "cpu_baseline": cpu,
            "ms": ms, "kernel_ms": kms, "flop": flops,
            "roofline": {"bound": "tensor", "achieved": flops / (kms * 1e9), "peak": p["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": flops / (kms * 1e9) / p["bf16_tflops"], "peak_source": p["source"]}}


def gqa_prefill_extra(device, batch=1, seq=8192, iters=5):
    """K4 on one GQA layer: a prompt of ``seq`` tokens into an empty paged
    cache (q/k norm + RoPE + append + causal attention + gate), timed with
    CUDA events around the whole call.  Tensor-bound: causal FLOPs =
    16 heads x 2 products x 2 x 256 x seq (seq + 1) / 2 per sequence."""
    from ria_b200.profile_cases import gqa_prefill_case

    r = gqa_prefill_case(batch, seq, iters, device)
    p = peaks()
    return {"workload": f"one GQA layer prefill, {batch} x {seq} new tokens, empty cache", "ms": r["ms"],
            "tokens_per_s": r["tokens_per_s"],
            "roofline": {"bound": "tensor", "achieved": r["tflops"], "peak": p["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": r["tflops"] / p["bf16_tflops"], "peak_source": p["source"]}}


MOE_EXPERT_BYTES = 3 * 512 * 2048 * 2  # gate, up, down of one expert (or the shared expert), bf16


def moe_extra(device, batches=(1, 8, 64), iters=20, warmup=3):
    """K5, the MoE block of one decode step (256 experts top-8 + shared
    expert, bf16 weights), at config 4's 64 tokens per GPU and at small
    batches.  Two layers' weights (3.2 GB) alternate between iterations so
    that no iteration finds its experts in L2.  HBM-bound: algorithmic bytes
    = the distinct experts the batch chose + the shared expert + the router
    rows + activations."""
    from ria_b200 import synthetic
    from ria_b200.engine import MoePlan, moe_decode
    from ria_b200.weights import MoeWeights

    ws = []
    for seed in (41, 42):
        t = synthetic.moe_weights(seed, device=device)
        ws.append(MoeWeights.from_tensors(t, device))
        del t
    torch.cuda.empty_cache()
    p = peaks()
    out = {"workload": "MoE block of one layer: 256 experts top-8 + 1 shared expert, hidden 2048, "
                       "intermediate 512, bf16 weights, fp32 activations; two layers' weights alternate; "
                       "CUDA-graph replay"}
    g = torch.Generator(device=device)
    g.manual_seed(5)
    for batch in batches:
        x = torch.randn(batch, 2048, device=device, generator=g) * 2.0
        y = torch.empty_like(x)
        plans = [MoePlan.create(batch, w.num_experts, device) for w in ws]
        # the two layers' blocks captured as one graph, as a decode step replays them
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            for i in range(warmup):
                moe_decode(x, ws[i % 2], plans[i % 2], out=y)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                for i in range(2):
                    moe_decode(x, ws[i], plans[i], out=y)
        torch.cuda.current_stream(device).wait_stream(side)
        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize(device)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters // 2):
            graph.replay()
        e.record()
        torch.cuda.synchronize(device)
        us = s.elapsed_time(e) * 1e3 / (2 * (iters // 2))
        del graph
        active = [len(set(pl.expert_ids.flatten().tolist())) for pl in plans]
        nbytes = (sum(active) / 2 + 1) * MOE_EXPERT_BYTES + 257 * 2048 * 2 + batch * 2048 * 8
        gbs = nbytes / (us * 1e-6) / 1e9
        out[f"b{batch}"] = {"us_per_layer": us, "active_experts": sum(active) / 2, "bytes_per_layer": nbytes,
                            "tokens_per_s_per_layer": batch / (us * 1e-6),
                            "roofline": {"bound": "hbm", "achieved": gbs, "peak": p["hbm_gbs"], "unit": "GB/s",
                                         "frac": gbs / p["hbm_gbs"], "peak_source": p["source"]}}
    del ws
    torch.cuda.empty_cache()
    return out


def config4_e2e(device, batch=64, prompt=2048, gen=256, rank=0, world=1):
    """Benchmark configuration 4 on N GPUs: each GPU serves its share of 64
    requests (512 at N = 8) of the random-init 40-layer 35B-A3B stack, each a
    2048-token random-id prompt, then 256 greedily generated tokens.  Prefill:
    the whole prompt in one pass per layer (chunked DeltaNet K2, GQA prefill
    K4, the prompt MoE as grouped library GEMMs) and the greedy head on the
    last position.  Decode: embedding, 40 x (attention step + MoE block K5),
    greedy head K6, the ids fed back on the device, one CUDA graph per step
    (captured after the first generated step, untimed capture).  All 40
    layers have their own weights (~63 GB).  Reported: prefill time, decode
    time per step with its algorithmic bytes (attention and head weights,
    DeltaNet state read + write, KV read, the weights of the experts each
    layer's batch chose, counted on the first step) and HBM fraction, and the
    whole job's generated tokens/s (prefill + every decode step).  With N > 1
    every rank runs its own 64 requests (different prompts, replicated
    weights, no collective on the path) and each phase's time is the max over
    ranks."""
    from ria_b200 import constants as C, synthetic
    from ria_b200.model import ModelGraph
    from ria_b200.weights import DeltaNetWeights

    torch.cuda.empty_cache()
    model = synthetic.config4_decode_model(device, batch, prompt, extra_tokens=gen + 8, empty=True)
    st, attn, head = model.state, model.state.layers, model.head
    g = torch.Generator(device=device)
    g.manual_seed(404 + rank)
    # library set-up on a short prompt, then a fresh state
    model.prefill(torch.randint(0, head.vocab, (batch, 64), device=device, generator=g, dtype=torch.int32))
    torch.cuda.synchronize(device)
    st.reset()
    ids = torch.randint(0, head.vocab, (batch, prompt), device=device, generator=g, dtype=torch.int32)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    torch.cuda.synchronize(device)
    barrier(world, device)
    ev[0].record()
    model.prefill(ids)  # -> the first generated token
    ev[1].record()
    # the second generated token, eager, counting the experts each layer's batch chose
    active = []
    plain = model._moe

    def counting(layer, x):
        y = plain(layer, x)
        active.append(int(torch.unique(model.plan.expert_ids).numel()))
        return y

    model._moe = counting
    model.step()
    model._moe = plain
    ev[2].record()
    torch.cuda.synchronize(device)
    graph = ModelGraph(model)
    steps = gen - 2
    lens0 = sum(st.lengths) / batch
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    barrier(world, device)
    s.record()
    for _ in range(steps):
        graph.step()
    e.record()
    torch.cuda.synchronize(device)
    prefill_ms = reduce_max(ev[0].elapsed_time(ev[1]), world, device)
    eager_ms = reduce_max(ev[1].elapsed_time(ev[2]), world, device)
    step_ms = reduce_max(s.elapsed_time(e), world, device) / steps
    total_s = (prefill_ms + eager_ms + steps * step_ms) / 1e3
    n_dn = sum(1 for w in attn.values() if isinstance(w, DeltaNetWeights))
    n_gqa = C.NUM_LAYERS - n_dn
    weights = sum(w.w_in.numel() * 2 + w.w_out.numel() * 2 for w in attn.values())
    moe_bytes = sum((a + 1) * MOE_EXPERT_BYTES + 257 * 2048 * 2 for a in active)
    state = n_dn * batch * 2 * 32 * 128 * 128 * 4
    kv = n_gqa * batch * (lens0 + steps / 2) * 2 * 2 * 256 * 2
    nbytes = weights + moe_bytes + state + kv + head.lm_head.numel() * 2
    p = peaks()
    gbs = nbytes / (step_ms * 1e-3) / 1e9
    del graph, model, st, attn, head
    torch.cuda.empty_cache()
    return {"workload": f"config 4 on {world} GPU(s): {batch} sequences per GPU, {batch * world} in total, each a "
                        f"{prompt}-token random-id prompt + {gen} greedy tokens; 40 layers with 256-expert top-8 MoE "
                        "+ shared expert; requests sharded by sequence, no collective",
            "requests": batch * world, "n_gpus": world,
            "prefill_ms": prefill_ms, "prefill_tokens_per_s": world * batch * prompt / (prefill_ms * 1e-3),
            "decode_ms_per_step": step_ms, "decode_tokens_per_s": world * batch / (step_ms * 1e-3),
            "e2e_generated_tokens_per_s": world * batch * gen / total_s,
            "e2e_generated_tokens_per_s_per_gpu": batch * gen / total_s, "e2e_s": total_s,
            "active_experts_per_layer": sum(active) / len(active), "decode_bytes_per_step": nbytes,
            "decode_moe_bytes_share": moe_bytes / nbytes,
            "decode_roofline": {"bound": "hbm", "achieved": gbs, "peak": p["hbm_gbs"], "unit": "GB/s",
                                "frac": gbs / p["hbm_gbs"], "peak_source": p["source"]}}


def strong_scaling(args, rank, world, device, layers):
    """Benchmark configuration 3 as a fixed job: the N = 1 workload's
    args.batch sequences split args.batch / N per GPU by the cost-balanced
    assignment (no collective on the path); the whole job's decode tokens/s,
    elapsed time the max over ranks.  Timed two ways on the same state: the
    eager public step (``BatchedAttentionState.step``, host planning and one
    Python launch per kernel) and the step replayed from a CUDA graph
    (``DecodeGraph``, the engine's loop for small per-GPU batches, where the
    eager step's host work -- about 250 launches -- can exceed the GPU time,
    more so with one such process per GPU on a shared host).  The line's
    ``tokens_per_s`` is the graph figure."""
    from ria_b200.engine import DecodeGraph

    headroom = 2 * (args.warmup + args.steps) + 8
    lengths = strong_lengths(args, rank, world)
    eng, _ = build_engine(args, device, rank, world, headroom, layers, lengths)
    x = torch.randn(len(lengths), 2048, device=device).to(torch.bfloat16).float()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(step):
        for _ in range(args.warmup):
            step(x)
        torch.cuda.synchronize(device)
        barrier(world, device)
        s.record()
        for _ in range(args.steps):
            step(x)
        e.record()
        torch.cuda.synchronize(device)
        return reduce_max(s.elapsed_time(e), world, device)

    eager_ms = timed(eng.step)
    graph = DecodeGraph(eng)
    graph_ms = timed(graph.step)
    kv_max = reduce_max(float(sum(lengths)), world, device)
    del graph, eng
    torch.cuda.empty_cache()
    return {"workload": f"config3 fixed job: {args.batch} sequences in total, {args.batch // world} per GPU",
            "sequences_total": args.batch, "sequences_per_gpu": len(lengths), "kv_tokens_per_gpu_max": int(kv_max),
            "tokens_per_s": args.batch * args.steps / (graph_ms * 1e-3), "ms_per_step": graph_ms / args.steps,
            "step": "CUDA-graph replay (DecodeGraph)",
            "eager_tokens_per_s": args.batch * args.steps / (eager_ms * 1e-3),
            "eager_ms_per_step": eager_ms / args.steps,
            "scaling": "strong", "steps": args.steps, "warmup": args.warmup}


def dropin_b1_stack(device, L=4096, tokens=20, warmup=3):
    """One batch-1 token through all 40 layers via this package's
    ``router_ia.qwen36_attention_cache.step_attention``, called layer by layer
    exactly as router-ia's ``run_forward_token`` calls the reference module
    (qwen36_chat_batch.py:181-207; per-call Python, split planning and the
    registry lookups included; no MoE), with 4096 cached tokens on every GQA
    layer.  Weights are registered in memory (the same seeded weights the
    reference anchor writes to its checkpoint)."""
    from ria_b200 import constants as C, synthetic
    from router_ia import qwen36_attention_cache as cache

    root = Path(tempfile.mkdtemp(prefix="ria_dropin_"))
    for layer in range(C.NUM_LAYERS):
        cache.register_layer_weights(root, layer, synthetic.layer_weights_on_device(layer, device, seed=0))
    dev = f"cuda:{device.index}"
    state = cache.state_for(root, dev)
    state.reset()
    cache.activate(root, state)
    g = torch.Generator(device=device)
    g.manual_seed(17)
    for layer in range(C.NUM_LAYERS):
        if C.is_full_attention_layer(layer):
            state.full_keys[layer] = torch.randn(1, 2, L, 256, device=device, generator=g).to(torch.bfloat16)
            state.full_values[layer] = torch.randn(1, 2, L, 256, device=device, generator=g).to(torch.bfloat16)
        else:
            state.linear_states[layer] = torch.randn(1, 32, 128, 128, device=device, generator=g) * 0.1
    state.tokens_seen = L
    x0 = torch.randn(1, 2048, device=device, generator=g)

    def token(x):
        for layer in range(C.NUM_LAYERS):
            x = cache.step_attention(root, layer, x, dev)
        state.tokens_seen += 1
        return x

    for _ in range(warmup):
        token(x0)
    torch.cuda.synchronize(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(tokens):
        token(x0)
    e.record()
    torch.cuda.synchronize(device)
    ms = s.elapsed_time(e) / tokens
    cache.deactivate(root)
    cache.reset(root)
    return {"ms_per_token": ms, "tokens": tokens, "kv_tokens": L}


def reference_gpu_anchor(L=4096, tokens=20, warmup=3):
    """router-ia's own ``qwen36_attention_cache`` (the unmodified install in
    baseline/_ref) on cuda:0: the same batch-1 40-layer token as
    ``dropin_b1_stack``, through the reference's stock CUDA path (fp16
    projections, fp32 ``torch.cat`` KV of 4096 cached tokens per GQA layer),
    weights read from a synthetic safetensors checkpoint with the reference
    tensor names and kept resident in its VRAM cache (QWEN36_VRAM_CACHE_GB)."""
    ref = import_reference()
    from ria_b200 import constants as C, synthetic
    from ria_b200.weights import write_checkpoint

    device = torch.device("cuda", 0)
    root = Path(tempfile.mkdtemp(prefix="ria_refanchor_"))
    write_checkpoint(root, {layer: {k: v.cpu() for k, v in synthetic.layer_weights_on_device(layer, device, seed=0).items()}
                            for layer in range(C.NUM_LAYERS)})
    dev = "cuda:0"
    state = ref.state_for(root, dev)
    state.reset()
    ref.activate(root, state)
    g = torch.Generator(device=device)
    g.manual_seed(17)
    for layer in range(C.NUM_LAYERS):
        if C.is_full_attention_layer(layer):
            state.full_keys[layer] = torch.randn(1, 2, L, 256, device=device, generator=g).to(torch.bfloat16).float()
            state.full_values[layer] = torch.randn(1, 2, L, 256, device=device, generator=g).to(torch.bfloat16).float()
        else:
            state.linear_states[layer] = torch.randn(1, 32, 128, 128, device=device, generator=g) * 0.1
    state.tokens_seen = L
    x0 = torch.randn(1, 2048, device=device, generator=g)

    def token(x):
        for layer in range(C.NUM_LAYERS):
            x = ref.step_attention(root, layer, x, dev)
        state.tokens_seen += 1
        return x

    for _ in range(warmup):
        token(x0)
    torch.cuda.synchronize(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(tokens):
        token(x0)
    e.record()
    torch.cuda.synchronize(device)
    ms = s.elapsed_time(e) / tokens
    ref.deactivate(root)
    return {"ms_per_token": ms, "tokens": tokens, "kv_tokens": L, "module": str(Path(ref.__file__).relative_to(REPO))}


def gpu_anchor(device):
    """The batch-1 40-layer token through the drop-in module (this process)
    and through the reference's own module on the same GPU (a subprocess, so
    that ``router_ia`` names the reference package there)."""
    ours = dropin_b1_stack(device)
    env = dict(os.environ, QWEN36_VRAM_CACHE_GB="16", CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", "0"))
    ref = None
    try:
        out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--reference-gpu-anchor"], env=env,
                             capture_output=True, text=True, timeout=900)
        lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
        ref = json.loads(lines[-1]) if out.returncode == 0 and lines else {"error": out.stderr[-600:]}
    except (subprocess.TimeoutExpired, OSError, ValueError) as exc:
        ref = {"error": str(exc)[-300:]}
    res = {"workload": "1 sequence, 30 DeltaNet + 10 GQA layers, 4096 cached tokens, one token through "
                       "qwen36_attention_cache.step_attention per layer (no MoE)",
           "ours_ms_per_token": ours["ms_per_token"], "reference": ref}
    if ref and "ms_per_token" in ref:
        res["reference_ms_per_token"] = ref["ms_per_token"]
        res["speedup_vs_reference"] = ref["ms_per_token"] / ours["ms_per_token"]
    return res


def import_reference():
    """router-ia's ``qwen36_attention_cache`` from the unmodified install under
    baseline/_ref (``pip install --target baseline/_ref`` of the reference's
    v2 package).  Raises if it is missing or if this package's module of the
    same name is already imported."""
    if not (REF_DIR / "router_ia" / "qwen36_attention_cache.py").is_file():
        raise RuntimeError("the reference is not installed under baseline/_ref")
    if "router_ia" in sys.modules and not str(getattr(sys.modules["router_ia"], "__file__", "")).startswith(str(REF_DIR)):
        raise RuntimeError("router_ia already names this package's module in this process")
    sys.path.insert(0, str(REF_DIR))
    import router_ia.qwen36_attention_cache as ref

    if not Path(ref.__file__).resolve().is_relative_to(REF_DIR.resolve()):
        raise RuntimeError(f"imported {ref.__file__}, not the reference install")
    return ref


def reference_cpu(args, steps, warmup, sample):
    """router-ia itself on the host cores: the reference's own
    ``step_attention`` (qwen36_attention_cache.py:376-379 -> _linear_stateful
    :224-282 / _full_stateful :285-324, its CPU fp32 path with the per-call
    weight fetch of qwen36_cached_loop.py:527-560) one sequence at a time as
    router-ia runs, on ``sample`` sequences at stratified KV lengths of the
    workload: per timed step, one DeltaNet and one GQA layer step per sampled
    sequence, extrapolated to 30 + 10 layers.  Weights: the seeded synthetic
    layer 0 (DeltaNet) and layer 3 (GQA) written as a safetensors checkpoint
    with the reference tensor names."""
    ref = import_reference()
    from ria_b200 import synthetic
    from ria_b200.weights import write_checkpoint

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    lengths = sorted(synthetic.stratified_lengths(args.batch, args.len_lo, args.len_hi, seed=0))
    picks = [lengths[int((i + 0.5) * len(lengths) / sample)] for i in range(sample)]
    root = Path(tempfile.mkdtemp(prefix="ria_refcpu_"))
    write_checkpoint(root, {0: synthetic.layer_weights(0, 0), 3: synthetic.layer_weights(3, 0)})
    g = torch.Generator().manual_seed(0)
    seqs = []
    for n in picks:
        kc = torch.randn(1, 2, n, 256, generator=g).to(torch.bfloat16).float()
        vc = torch.randn(1, 2, n, 256, generator=g).to(torch.bfloat16).float()
        conv = (torch.randn(1, 8192, 4, generator=g) * 0.1).to(torch.bfloat16)
        rec = torch.randn(1, 32, 128, 128, generator=g) * 0.1
        seqs.append((n, kc, vc, conv, rec))
    x = torch.randn(1, 2048, generator=g).to(torch.bfloat16).float()
    state = ref.state_for(root, "cpu")
    state.reset()
    ref.activate(root, state)
    per_token = []
    for it in range(warmup + steps):
        t_tok = 0.0
        for n, kc, vc, conv, rec in seqs:
            state.linear_states[0], state.linear_conv_states[0] = rec.clone(), conv.clone()
            state.full_keys[3], state.full_values[3] = kc, vc
            state.tokens_seen = n
            t0 = time.perf_counter()
            ref.step_attention(root, 0, x, "cpu")
            t1 = time.perf_counter()
            ref.step_attention(root, 3, x, "cpu")
            t2 = time.perf_counter()
            t_tok += 30 * (t1 - t0) + 10 * (t2 - t1)
        if it >= warmup:
            per_token.append(t_tok / len(seqs))
    ref.deactivate(root)
    sec_per_token = statistics.mean(per_token)
    return {
        "value": 1.0 / sec_per_token,
        "unit": UNIT,
        "cores": torch.get_num_threads(),
        "kind": "reference",
        "sample": (f"router-ia's own step_attention (baseline/_ref) on {sample} sequences at KV lengths {picks} "
                   f"(strata of the workload), one DeltaNet and one GQA layer step each per timed step, "
                   f"extrapolated to 30+10 layers; {steps} timed steps"),
        "cpu": _cpu_model(),
    }


# --------------------------------------------------------------------------- CPU reference (oracle port)
def cpu_reference(args, steps, warmup, sample):
    """router-ia's layer algorithm on the host cores, one sequence at a time
    (as the reference runs): per-token time = 30 x DeltaNet layer + 10 x GQA
    layer at the sequence's KV length, timed on ``sample`` sequences at
    stratified lengths of the workload and extrapolated to the stack."""
    from oracle import attention_oracle as O
    from ria_b200 import synthetic

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    lengths = sorted(synthetic.stratified_lengths(args.batch, args.len_lo, args.len_hi, seed=0))
    picks = [lengths[int((i + 0.5) * len(lengths) / sample)] for i in range(sample)]
    dn_w = {k: v for k, v in synthetic.layer_weights(0, 0).items()}
    gqa_w = {k: v for k, v in synthetic.layer_weights(3, 0).items()}
    # the reference keeps fp32 projections on the CPU path; convert once
    for w in (dn_w, gqa_w):
        for k in list(w):
            if w[k].dim() == 2:
                w[k] = w[k].float()
    g = torch.Generator().manual_seed(0)
    caches = []
    for n in picks:
        kc = torch.randn(1, 2, n, 256, generator=g).to(torch.bfloat16).float()
        vc = torch.randn(1, 2, n, 256, generator=g).to(torch.bfloat16).float()
        conv = (torch.randn(1, 8192, 4, generator=g) * 0.1).to(torch.bfloat16)
        rec = torch.randn(1, 32, 128, 128, generator=g) * 0.1
        caches.append((kc, vc, conv, rec))
    x = torch.randn(1, 2048, generator=g).to(torch.bfloat16).float()
    per_token = []
    for it in range(warmup + steps):
        t_tok = 0.0
        for (kc, vc, conv, rec), n in zip(caches, picks):
            t0 = time.perf_counter()
            O.deltanet_step(dn_w, x, conv, rec)
            t1 = time.perf_counter()
            O.gqa_step(gqa_w, x, kc, vc, n)
            t2 = time.perf_counter()
            t_tok += 30 * (t1 - t0) + 10 * (t2 - t1)
        if it >= warmup:
            per_token.append(t_tok / len(picks))
    sec_per_token = statistics.mean(per_token)
    return {
        "value": 1.0 / sec_per_token,
        "unit": UNIT,
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": (f"{sample} sequences at KV lengths {picks} (strata of the workload), one DeltaNet and one GQA "
                   f"layer step each per timed step, extrapolated to 30+10 layers; {steps} timed steps"),
        "cpu": _cpu_model(),
    }


def _cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.reference_gpu_anchor:
        print(json.dumps(reference_gpu_anchor()), flush=True)
        return

    if args.impl == "reference":
        if rank != 0:
            return
        try:
            ref = reference_cpu(args, steps=args.steps, warmup=args.warmup, sample=args.cpu_sample)
        except RuntimeError as exc:
            print(json.dumps({"impl": "reference", "unavailable": str(exc)}), flush=True)
            return
        line = {
            "metric": METRIC, "impl": "reference", "value": ref["value"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / ref["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (reference CPU path)",
            "data": "synthetic", "config": {"workload": "config3: batched ragged hybrid decode step (CPU sample)",
                                            "sequences_per_gpu": args.batch,
                                            "kv_len_range": [args.len_lo, args.len_hi]},
            "cpu_baseline": ref, "e2e": {"value": ref["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                                         "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    try:
        layers = build_layers(device)
        line = run_ours(args, rank, world, device, layers)
        if not args.no_extras:
            if world > 1:
                # multi-GPU lines, every rank taking part: the fixed 256-sequence
                # job split 256/N (strong scaling) and configuration 4 with 64
                # requests per GPU
                strong = strong_scaling(args, rank, world, device, layers)
                del layers
                torch.cuda.empty_cache()
                c4 = config4_e2e(device, rank=rank, world=world)
                if rank == 0:
                    line["strong_scaling"] = strong
                    line["config4_e2e"] = c4
            else:
                # the fixed job at N = 1 is the headline workload; measured
                # again here so that every N's line times it the same way
                torch.cuda.empty_cache()
                line["strong_scaling"] = strong_scaling(args, rank, world, device, layers)
                del layers
                torch.cuda.empty_cache()
                line["config1_gqa_b1_l4096"] = config1_latency(device)
                line["config2_prefill"] = config2_prefill(device)
                line["gqa_prefill_1x8192"] = gqa_prefill_extra(device)
                line["decode_b1_stack_l4096"] = decode_b1_stack(device)
                line["dropin_vs_reference_b1_l4096"] = gpu_anchor(device)
                line["config0_deltanet_b1"] = config0_deltanet(device)
                line["moe_block"] = moe_extra(device)
                line["config4_e2e"] = config4_e2e(device)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_reference(args, steps=2, warmup=1, sample=args.cpu_sample)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.barrier(device_ids=[device.index])
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
