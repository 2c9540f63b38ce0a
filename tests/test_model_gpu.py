"""The full decode step (embedding, 4-layer hybrid stack with a MoE block
after every attention layer, greedy head) for B sequences at once.

Three checks: (1) ``DecodeModel.step`` equals, bit for bit, the same pieces
run one at a time on a twin model (embedding gather, then per layer the
attention step and the MoE block, then the head, the ids fed back); (2)
every layer's attention and MoE output of every sequence against the CPU
oracle on the GPU's own input to that layer, at the per-layer bound of the
attention tests (2e-2 max-abs, 1e-2 relative RMS of the layer's
contribution), and the picked ids against the oracle head on the GPU's
final hidden state (an id may differ only where the oracle's best two
logits are within 2e-3); (3) ``ModelGraph`` replays equal eager steps bit
for bit.  B = 3 uses the fused head, B = 10 the library-GEMM head."""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as O
from ria_b200 import _ext, synthetic
from ria_b200 import constants as C
from ria_b200.engine import deltanet_decode, gqa_decode, moe_decode
from ria_b200.model import DecodeModel, HeadWeights, ModelGraph, greedy_head
from ria_b200.weights import DeltaNetWeights, GqaWeights, MoeWeights

pytestmark = pytest.mark.gpu

LAYERS = [0, 1, 2, 3]  # DN DN DN GQA
EXPERTS = 16
VOCAB = 1001


def _weights(dev):
    wt = {layer: synthetic.layer_weights(layer, 4) for layer in LAYERS}
    mt = {layer: synthetic.moe_weights(60 + layer, num_experts=EXPERTS) for layer in LAYERS}
    ht = synthetic.head_weights(61, vocab=VOCAB)
    attn = {layer: (GqaWeights if C.is_full_attention_layer(layer) else DeltaNetWeights).from_tensors(w, dev)
            for layer, w in wt.items()}
    moe = {layer: MoeWeights.from_tensors(w, dev) for layer, w in mt.items()}
    return wt, mt, ht, attn, moe, HeadWeights.from_tensors(ht, dev)


def _model(attn, moe, head, lengths, dev, seed):
    """A model whose sequences hold random DeltaNet / conv state and random KV
    prefixes of the given lengths (the same draws for the same seed)."""
    m = DecodeModel(attn, moe, head, batch=len(lengths), pool_blocks=24, max_blocks_per_seq=4, device=dev)
    st = m.state
    g = torch.Generator().manual_seed(seed)
    ref = []
    for i, n in enumerate(lengths):
        st.set_length(i, n, position=n + 3)
        seq = {}
        for layer in LAYERS:
            if C.is_full_attention_layer(layer):
                k = torch.randn(2, n, 256, generator=g).to(torch.bfloat16)
                v = torch.randn(2, n, 256, generator=g).to(torch.bfloat16)
                rows = st.physical_rows(i, n).to(dev)
                st.k_pool[layer][:, rows] = k.to(dev)
                st.v_pool[layer][:, rows] = v.to(dev)
                seq[layer] = [k.float().unsqueeze(0), v.float().unsqueeze(0)]
            else:
                rec = torch.randn(1, 32, 128, 128, generator=g) * 0.1
                conv = (torch.randn(1, 8192, 4, generator=g) * 0.1).to(torch.bfloat16)
                st.rec[layer][i] = rec[0].to(dev)
                st.conv[layer][i] = conv[0].to(dev)
                seq[layer] = [conv, rec]
        ref.append(seq)
    st.sync_tables()
    m.ids.copy_(torch.randint(0, VOCAB, (len(lengths),), generator=g, dtype=torch.int32).to(dev))
    return m, ref


@pytest.mark.parametrize("lengths", [[0, 70, 131], [5, 64, 0, 17, 100, 63, 1, 128, 40, 9]])
def test_decode_step_matches_pieces_and_oracle(cuda_device, lengths):
    wt, mt, ht, attn, moe, head = _weights(cuda_device)
    model, ref = _model(attn, moe, head, lengths, cuda_device, 8)
    twin, _ = _model(attn, moe, head, lengths, cuda_device, 8)
    B = len(lengths)
    for step in range(2):
        ids_in = model.ids.clone()
        got = model.step().clone()
        # the same step piece by piece on the twin, keeping every input
        st = twin.state
        st.reserve_next()
        launch = st.plan()
        x = head.embedding.index_select(0, twin.ids).float()
        trace = []
        for layer in LAYERS:
            xin = x
            if C.is_full_attention_layer(layer):
                xa = gqa_decode(x, attn[layer], st.k_pool[layer], st.v_pool[layer], st.block_table, st.inv_freq,
                                launch, st.seq_lens, st.positions)
            else:
                xa = deltanet_decode(x, attn[layer], st.rec[layer], st.conv[layer])
            x = moe_decode(xa, moe[layer], twin.plan)
            trace.append((xin, xa, x))
        greedy_head(x, head, twin.ids, twin.head_ws)
        _ext.advance_positions(st.seq_lens, st.positions)
        st.lengths = [n + 1 for n in st.lengths]
        st.positions_host = [p + 1 for p in st.positions_host]
        assert torch.equal(got, twin.ids), "step() differs from its pieces"
        assert O.finite(x), "non-finite hidden state"
        # oracle, layer by layer on the GPU's inputs
        emb = ht["model.language_model.embed_tokens.weight"]
        assert torch.equal(trace[0][0].cpu(), emb[ids_in.cpu().long()].float())
        for i in range(B):
            pos = lengths[i] + 3 + step
            for li, layer in enumerate(LAYERS):
                xin, xa, xm = (t[i:i + 1].cpu() for t in trace[li])
                s = ref[i][layer]
                if C.is_full_attention_layer(layer):
                    ra, s[0], s[1] = O.gqa_step(wt[layer], xin, s[0], s[1], pos)
                else:
                    ra, s[0], s[1] = O.deltanet_step(wt[layer], xin, s[0], s[1])
                assert O.max_abs(xa, ra) < 2e-2 and O.rel_rms(xa - xin, ra - xin) < 1e-2, (step, i, layer, "attn")
                rm, _, _, _ = O.moe_step(mt[layer], xa, top_k=8)
                assert O.max_abs(xm, rm) < 2e-2 and O.rel_rms(xm - xa, rm - xa) < 1e-2, (step, i, layer, "moe")
        ref_logits, ref_ids = O.lm_head_greedy(x.cpu(), ht["model.language_model.norm.weight"], ht["lm_head.weight"])
        for b in range(B):
            g_id = int(got[b])
            if g_id != int(ref_ids[b]):
                top = ref_logits[b].max()
                assert top - ref_logits[b, g_id] <= 2e-3 * max(1.0, abs(float(top))), (step, b)
    assert _ext.device_error() == 0


def test_model_graph_replays_eager_steps(cuda_device):
    _, _, _, attn, moe, head = _weights(cuda_device)
    lengths = [3, 64, 90]
    eager, _ = _model(attn, moe, head, lengths, cuda_device, 9)
    graphed, _ = _model(attn, moe, head, lengths, cuda_device, 9)
    eager.step()
    graphed.step()  # library set-up outside capture
    graph = ModelGraph(graphed)
    for _ in range(3):
        a = eager.step(graph.launch).clone()  # the split plan the graph holds
        b = graph.step().clone()
        assert torch.equal(a, b)
    for layer in LAYERS:
        if C.is_full_attention_layer(layer):
            assert torch.equal(eager.state.k_pool[layer], graphed.state.k_pool[layer])
        else:
            assert torch.equal(eager.state.rec[layer], graphed.state.rec[layer])
    assert eager.state.lengths == graphed.state.lengths
    assert torch.equal(eager.state.seq_lens, graphed.state.seq_lens)
    del graph
