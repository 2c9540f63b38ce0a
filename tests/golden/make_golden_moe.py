"""Generate the MoE golden fixture by running router-ia's own MoE block.

Run from the repository root on a machine with a router-ia checkout:

    python tests/golden/make_golden_moe.py [--reference /path/to/router-ia]

It imports ``router_ia.qwen36_chat_batch`` from ``<reference>/v2/src`` (the
reference, unmodified), writes a synthetic safetensors checkpoint with the
reference tensor names for one layer's MoE block with ``NUM_EXPERTS`` routed
experts (fewer than the model's 256 keeps the file small; the router and the
block are generic in the expert count), runs ``batched_moe_step`` on the CPU
for ``TOKENS`` residual rows one at a time, and stores in
``tests/golden/reference_moe.npz``: the layer outputs, the chosen expert ids
and router weights, and the shared-expert gate values.  Only seeds are
stored for the inputs; tests regenerate them.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "reference_moe.npz"

LAYER = 0
WEIGHT_SEED = 21
NUM_EXPERTS = 16
TOP_K = 8
TOKENS = 6
INPUT_SEED = 22


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ROUTER_IA_REFERENCE", "/root/reference"))
    args = ap.parse_args()
    ref_src = Path(args.reference) / "v2" / "src"
    if not (ref_src / "router_ia" / "qwen36_chat_batch.py").is_file():
        raise SystemExit(f"router-ia checkout not found under {args.reference}")
    sys.path.insert(0, str(REPO / "router-ia_b200"))
    sys.path.insert(0, str(ref_src))

    import numpy as np
    import torch

    from router_ia import qwen36_chat_batch as chat
    from ria_b200 import synthetic
    from ria_b200.weights import write_checkpoint

    assert Path(chat.__file__).resolve().is_relative_to(ref_src.resolve()), chat.__file__
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    w = synthetic.moe_weights(WEIGHT_SEED, num_experts=NUM_EXPERTS)
    w.update(synthetic.layer_weights(LAYER, 0))  # the layer's attention tensors (layer-kind detection)
    xs = synthetic.hidden_stream(TOKENS, INPUT_SEED)
    outs, ids, wts, sg = [], [], [], []
    with tempfile.TemporaryDirectory() as tmp:
        root = Path(tmp)
        write_checkpoint(root, {LAYER: w})
        for t in range(TOKENS):
            out, e, ww, g, _ = chat.batched_moe_step(root, LAYER, xs[t].reshape(1, -1).float(), TOP_K, "cpu")
            outs.append(out.reshape(-1).float())
            ids.append(e)
            wts.append(ww)
            sg.append(g)
    meta = {"reference_module": "router_ia.qwen36_chat_batch.batched_moe_step (v2/src)", "torch": torch.__version__,
            "layer": LAYER, "weight_seed": WEIGHT_SEED, "num_experts": NUM_EXPERTS, "top_k": TOP_K,
            "tokens": TOKENS, "input_seed": INPUT_SEED}
    np.savez_compressed(OUT, meta=np.array(json.dumps(meta)), out=torch.stack(outs).numpy().astype(np.float32),
                        ids=np.array(ids, dtype=np.int64), weights=np.array(wts, dtype=np.float32),
                        shared_gate=np.array(sg, dtype=np.float32))
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
