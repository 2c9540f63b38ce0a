"""Generate the golden fixtures by running router-ia's own attention code.

Run from the repository root on a machine with a router-ia checkout:

    python tests/golden/make_golden.py [--reference /path/to/router-ia]

It imports ``router_ia.qwen36_attention_cache`` from ``<reference>/v2/src``
(the reference, unmodified), writes a synthetic safetensors checkpoint with the
reference tensor names into a temporary directory (seeded weights from
``ria_b200.synthetic``: layer 0 Gated DeltaNet, layer 3 GQA), runs the
reference's CPU path and stores its outputs in ``tests/golden/reference_steps.npz``:

* ``dn_residual`` (T, 2048): ``step_attention`` residuals for T tokens of a
  DeltaNet layer from a zero state (first half "prompt", second half "decode";
  the reference runs both token by token);
* ``dn_conv_state`` (8192, 4) and ``dn_rec_heads`` (3, 128, 128) for value heads
  0, 17, 31 plus ``dn_rec_norms`` (32,): the final DeltaNet state;
* ``gqa_residual`` (S, 2048), ``gqa_k_new``/``gqa_v_new`` (2, S, 256): a GQA layer
  decoding S tokens after a pre-filled bf16 cache of ``gqa_prefix`` tokens.

Only inputs' seeds are stored; tests regenerate weights and inputs with the
same generators.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "reference_steps.npz"

DN_LAYER, GQA_LAYER = 0, 3
WEIGHT_SEED = 0
DN_TOKENS = 16
DN_INPUT_SEED = 11
GQA_PREFIX = 64
GQA_STEPS = 8
GQA_INPUT_SEED = 12
GQA_CACHE_SEED = 13
REC_HEADS = (0, 17, 31)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ROUTER_IA_REFERENCE", "/root/reference"))
    args = ap.parse_args()
    ref_src = Path(args.reference) / "v2" / "src"
    if not (ref_src / "router_ia" / "qwen36_attention_cache.py").is_file():
        raise SystemExit(f"router-ia checkout not found under {args.reference}")
    # Reference first so that ``router_ia`` is the reference package.
    sys.path.insert(0, str(REPO / "router-ia_b200"))
    sys.path.insert(0, str(ref_src))

    import numpy as np
    import torch

    from router_ia import qwen36_attention_cache as ref
    from ria_b200 import synthetic
    from ria_b200.weights import write_checkpoint

    assert Path(ref.__file__).resolve().is_relative_to(ref_src.resolve()), ref.__file__
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    dn_w = synthetic.layer_weights(DN_LAYER, WEIGHT_SEED)
    gqa_w = synthetic.layer_weights(GQA_LAYER, WEIGHT_SEED)
    with tempfile.TemporaryDirectory() as tmp:
        root = Path(tmp)
        write_checkpoint(root, {DN_LAYER: dn_w, GQA_LAYER: gqa_w})

        state = ref.state_for(root, "cpu")
        state.reset()
        ref.activate(root, state)
        xs = synthetic.hidden_stream(DN_TOKENS, DN_INPUT_SEED)
        dn_res = []
        for t in range(DN_TOKENS):
            dn_res.append(ref.step_attention(root, DN_LAYER, xs[t], "cpu").reshape(-1).clone())
            state.tokens_seen += 1
        rec = state.linear_states[DN_LAYER][0]
        conv = state.linear_conv_states[DN_LAYER][0]

        state.reset()
        kp, vp = synthetic.kv_prefix(GQA_PREFIX, GQA_CACHE_SEED)
        state.full_keys[GQA_LAYER] = kp.float().unsqueeze(0)
        state.full_values[GQA_LAYER] = vp.float().unsqueeze(0)
        state.tokens_seen = GQA_PREFIX
        xg = synthetic.hidden_stream(GQA_STEPS, GQA_INPUT_SEED)
        gqa_res = []
        for t in range(GQA_STEPS):
            gqa_res.append(ref.step_attention(root, GQA_LAYER, xg[t], "cpu").reshape(-1).clone())
            state.tokens_seen += 1
        k_new = state.full_keys[GQA_LAYER][0, :, GQA_PREFIX:]
        v_new = state.full_values[GQA_LAYER][0, :, GQA_PREFIX:]
        ref.deactivate(root)

    meta = {
        "reference_module": "router_ia.qwen36_attention_cache (v2/src)",
        "torch": torch.__version__,
        "weight_seed": WEIGHT_SEED,
        "dn_layer": DN_LAYER,
        "gqa_layer": GQA_LAYER,
        "dn_tokens": DN_TOKENS,
        "dn_input_seed": DN_INPUT_SEED,
        "gqa_prefix": GQA_PREFIX,
        "gqa_steps": GQA_STEPS,
        "gqa_input_seed": GQA_INPUT_SEED,
        "gqa_cache_seed": GQA_CACHE_SEED,
        "rec_heads": list(REC_HEADS),
    }
    np.savez_compressed(
        OUT,
        meta=np.array(json.dumps(meta)),
        dn_residual=torch.stack(dn_res).numpy().astype(np.float32),
        dn_conv_state=conv.float().numpy(),
        dn_rec_heads=rec[list(REC_HEADS)].numpy().astype(np.float32),
        dn_rec_norms=rec.double().flatten(1).norm(dim=1).numpy(),
        gqa_residual=torch.stack(gqa_res).numpy().astype(np.float32),
        gqa_k_new=k_new.numpy().astype(np.float32),
        gqa_v_new=v_new.numpy().astype(np.float32),
    )
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
