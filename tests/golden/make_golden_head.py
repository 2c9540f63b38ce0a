"""Generate the greedy-head golden fixture with router-ia's own functions.

Run from the repository root on a machine with a router-ia checkout:

    python tests/golden/make_golden_head.py [--reference /path/to/router-ia]

The end of router-ia's ``run_forward_token`` (v2/src/router_ia/
qwen36_chat_batch.py:194-199, CPU branch) is ``x = base.rmsnorm(x,
final_norm)`` then ``logits = F.linear(x, lm_head)``, and
``run_generated_token`` picks the next id with ``sample_next(logits,
temperature, top_k)`` (qwen36_mini_chat.py:75-88).  This script imports
``router_ia.qwen36_40layer_loop`` (``base``) and ``router_ia.qwen36_mini_chat``
from ``<reference>/v2/src`` unmodified, applies exactly those calls to seeded
synthetic inputs with a ``VOCAB``-row lm_head (the head is generic in the
vocabulary size; a small one keeps the fixture small) at temperature 0, and
stores the logits and ids in ``tests/golden/reference_head.npz``.  Only seeds
are stored for the inputs; tests regenerate them.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "reference_head.npz"

WEIGHT_SEED = 31
VOCAB = 4099
TOKENS = 6
INPUT_SEED = 32


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ROUTER_IA_REFERENCE", "/root/reference"))
    args = ap.parse_args()
    ref_src = Path(args.reference) / "v2" / "src"
    if not (ref_src / "router_ia" / "qwen36_mini_chat.py").is_file():
        raise SystemExit(f"router-ia checkout not found under {args.reference}")
    sys.path.insert(0, str(REPO / "router-ia_b200"))
    sys.path.insert(0, str(ref_src))

    import numpy as np
    import torch
    import torch.nn.functional as F

    from router_ia import qwen36_40layer_loop as base
    from router_ia.qwen36_mini_chat import sample_next
    from ria_b200 import synthetic

    assert Path(base.__file__).resolve().is_relative_to(ref_src.resolve()), base.__file__
    w = synthetic.head_weights(WEIGHT_SEED, vocab=VOCAB)
    final_norm = w["model.language_model.norm.weight"].float()  # load_final_norm: .float()
    lm_head = w["lm_head.weight"].float()  # load_lm_head: .float()
    xs = synthetic.hidden_stream(TOKENS, INPUT_SEED).reshape(TOKENS, -1) * 3.0
    logits, ids = [], []
    for t in range(TOKENS):
        x = base.rmsnorm(xs[t].reshape(1, -1).float(), final_norm)
        lg = F.linear(x, lm_head)
        logits.append(lg.reshape(-1))
        ids.append(sample_next(lg, 0.0, 0))
    meta = {"reference_functions": "qwen36_40layer_loop.rmsnorm, F.linear, qwen36_mini_chat.sample_next (v2/src)",
            "torch": torch.__version__, "weight_seed": WEIGHT_SEED, "vocab": VOCAB, "tokens": TOKENS,
            "input_seed": INPUT_SEED, "input_scale": 3.0}
    np.savez_compressed(OUT, meta=np.array(json.dumps(meta)), logits=torch.stack(logits).numpy().astype(np.float32),
                        ids=np.array(ids, dtype=np.int64))
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
