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
collective on the path); the elapsed time is the max over ranks.

``--impl reference`` times router-ia's algorithm on the host cores (the CPU
oracle port of qwen36_attention_cache's layer steps, one sequence at a time as
the reference runs) on a bounded sample of the same workload.
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
UNIT = "tokens/s"
B_DN = 4_292_736  # algorithmic bytes of K1 per (sequence, layer)
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) over algorithmic
# bytes, from one ncu capture of each kernel on a small case
# (profiles/gqa_decode_kernel_b32_l4096.md: 280.3 / 269.3 MB;
#  profiles/gdn_decode_kernel_b64.md: 222.0 / 274.7 MB, written state partly
#  still in L2 at kernel end).  Traffic of a full launch = ratio x its bytes.
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
def build_engine(args, device, rank, world, headroom):
    from ria_b200 import constants as C, synthetic
    from ria_b200.engine import BatchedAttentionState
    from ria_b200.sharding import balanced_assignment
    from ria_b200.weights import DeltaNetWeights, GqaWeights

    # Each rank decodes args.batch sequences whose KV lengths are a stratified
    # sample of U[len_lo, len_hi] (the same multiset on every rank and at every
    # GPU count: weak scaling with fixed work per GPU).  The job's request list
    # is the ranks' lists concatenated; the cost-balanced assignment keeps
    # each rank's list.
    per_rank = synthetic.stratified_lengths(args.batch, args.len_lo, args.len_hi, seed=0)
    requests = per_rank * world
    lengths = [requests[i] for i in balanced_assignment(requests, world)[rank]]
    layers = {}
    for layer in range(C.NUM_LAYERS):
        t = synthetic.layer_weights_on_device(layer, device, seed=0)
        cls = GqaWeights if C.is_full_attention_layer(layer) else DeltaNetWeights
        layers[layer] = cls.from_tensors(t, device)
        del t
    blocks = [math.ceil((n + headroom) / C.KV_BLOCK) for n in lengths]
    eng = BatchedAttentionState(layers, batch=args.batch, pool_blocks=sum(blocks) + 8,
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


def run_ours(args, rank, world, device):
    from ria_b200 import _ext

    headroom = args.warmup + 2 * args.steps + 4
    t_setup = time.perf_counter()
    eng, lengths = build_engine(args, device, rank, world, headroom)
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
    hook = EventHook(timed=("gqa_decode",))
    _ext.launch_hook = hook
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    s.record()
    for _ in range(iters):
        gqa_decode(x, w, k, v, table, inv, launch, seq_len0=L, position0=L)
    e.record()
    torch.cuda.synchronize(device)
    _ext.launch_hook = None
    kms, _ = hook.mean_ms("gqa_decode")
    step_ms = s.elapsed_time(e) / iters
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


def config4_e2e(device, batch=64, prompt=2048, gen=256):
    """Benchmark configuration 4 on one GPU: its per-GPU share of the 512
    requests (64 sequences) of the random-init 40-layer 35B-A3B stack, each a
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
    whole job's generated tokens/s (prefill + every decode step)."""
    from ria_b200 import constants as C, synthetic
    from ria_b200.model import ModelGraph
    from ria_b200.weights import DeltaNetWeights

    torch.cuda.empty_cache()
    model = synthetic.config4_decode_model(device, batch, prompt, extra_tokens=gen + 8, empty=True)
    st, attn, head = model.state, model.state.layers, model.head
    g = torch.Generator(device=device)
    g.manual_seed(404)
    # library set-up on a short prompt, then a fresh state
    model.prefill(torch.randint(0, head.vocab, (batch, 64), device=device, generator=g, dtype=torch.int32))
    torch.cuda.synchronize(device)
    st.reset()
    ids = torch.randint(0, head.vocab, (batch, prompt), device=device, generator=g, dtype=torch.int32)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    torch.cuda.synchronize(device)
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
    s.record()
    for _ in range(steps):
        graph.step()
    e.record()
    torch.cuda.synchronize(device)
    prefill_ms = ev[0].elapsed_time(ev[1])
    eager_ms = ev[1].elapsed_time(ev[2])
    step_ms = s.elapsed_time(e) / steps
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
    return {"workload": f"config 4 on one GPU: {batch} sequences x ({prompt}-token random-id prompt + {gen} greedy "
                        "tokens), 40 layers with 256-expert top-8 MoE + shared expert",
            "prefill_ms": prefill_ms, "prefill_tokens_per_s": batch * prompt / (prefill_ms * 1e-3),
            "decode_ms_per_step": step_ms, "decode_tokens_per_s": batch / (step_ms * 1e-3),
            "e2e_generated_tokens_per_s": batch * gen / total_s, "e2e_s": total_s,
            "active_experts_per_layer": sum(active) / len(active), "decode_bytes_per_step": nbytes,
            "decode_moe_bytes_share": moe_bytes / nbytes,
            "decode_roofline": {"bound": "hbm", "achieved": gbs, "peak": p["hbm_gbs"], "unit": "GB/s",
                                "frac": gbs / p["hbm_gbs"], "peak_source": p["source"]}}


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

    if args.impl == "reference":
        if rank != 0:
            return
        ref = cpu_reference(args, steps=args.steps, warmup=args.warmup, sample=args.cpu_sample)
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
        line = run_ours(args, rank, world, device)
        if rank == 0 and not args.no_extras:
            line["config1_gqa_b1_l4096"] = config1_latency(device)
            line["config2_prefill"] = config2_prefill(device)
            line["gqa_prefill_1x8192"] = gqa_prefill_extra(device)
            line["decode_b1_stack_l4096"] = decode_b1_stack(device)
            line["config0_deltanet_b1"] = config0_deltanet(device)
            line["moe_block"] = moe_extra(device)
            line["config4_e2e_b64"] = config4_e2e(device)
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
