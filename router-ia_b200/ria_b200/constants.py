"""Shapes of the Qwen3.6-35B-A3B attention layers (router-ia
v2/src/router_ia/qwen36_40layer_loop.py:36-50, qwen36_attention_cache.py:17-24)."""

HIDDEN = 2048
NUM_LAYERS = 40
EPS = 1e-6
VOCAB = 151936  # embedding rows and lm_head rows

# Gated DeltaNet ("linear attention") layers
LINEAR_NUM_K_HEADS = 16
LINEAR_NUM_V_HEADS = 32
LINEAR_HEAD_DIM = 128
LINEAR_KEY_DIM = LINEAR_NUM_K_HEADS * LINEAR_HEAD_DIM  # 2048
LINEAR_VALUE_DIM = LINEAR_NUM_V_HEADS * LINEAR_HEAD_DIM  # 4096
LINEAR_CONV_KERNEL = 4
LINEAR_CONV_STATE = LINEAR_CONV_KERNEL
LINEAR_CONV_DIM = LINEAR_KEY_DIM * 2 + LINEAR_VALUE_DIM  # 8192
# Fused input projection of a DeltaNet layer: [qkv | z | b | a]
DN_PROJ_QKV = (0, LINEAR_CONV_DIM)
DN_PROJ_Z = (LINEAR_CONV_DIM, LINEAR_CONV_DIM + LINEAR_VALUE_DIM)
DN_PROJ_B = (DN_PROJ_Z[1], DN_PROJ_Z[1] + LINEAR_NUM_V_HEADS)
DN_PROJ_A = (DN_PROJ_B[1], DN_PROJ_B[1] + LINEAR_NUM_V_HEADS)
DN_PROJ_WIDTH = DN_PROJ_A[1]  # 12352

# GQA full-attention layers
FULL_NUM_HEADS = 16
FULL_NUM_KV_HEADS = 2
FULL_HEAD_DIM = 256
FULL_Q_DIM = FULL_NUM_HEADS * FULL_HEAD_DIM  # 4096
FULL_KV_DIM = FULL_NUM_KV_HEADS * FULL_HEAD_DIM  # 512
FULL_Q_GATE_DIM = FULL_Q_DIM * 2  # 8192
FULL_NUM_KV_GROUPS = FULL_NUM_HEADS // FULL_NUM_KV_HEADS  # 8
ROPE_THETA = 10_000_000.0
ROPE_DIM = int(FULL_HEAD_DIM * 0.25)  # 64
# Fused input projection of a GQA layer: [q_gate | k | v]
GQA_PROJ_Q = (0, FULL_Q_GATE_DIM)
GQA_PROJ_K = (FULL_Q_GATE_DIM, FULL_Q_GATE_DIM + FULL_KV_DIM)
GQA_PROJ_V = (GQA_PROJ_K[1], GQA_PROJ_K[1] + FULL_KV_DIM)
GQA_PROJ_WIDTH = GQA_PROJ_V[1]  # 9216

# Paged KV cache
KV_BLOCK = 64  # tokens per block

DN_WEIGHT_NAMES = (
    "input_layernorm.weight",
    "linear_attn.in_proj_qkv.weight",
    "linear_attn.in_proj_z.weight",
    "linear_attn.in_proj_b.weight",
    "linear_attn.in_proj_a.weight",
    "linear_attn.conv1d.weight",
    "linear_attn.A_log",
    "linear_attn.dt_bias",
    "linear_attn.norm.weight",
    "linear_attn.out_proj.weight",
)
GQA_WEIGHT_NAMES = (
    "input_layernorm.weight",
    "self_attn.q_proj.weight",
    "self_attn.k_proj.weight",
    "self_attn.v_proj.weight",
    "self_attn.q_norm.weight",
    "self_attn.k_norm.weight",
    "self_attn.o_proj.weight",
)


def layer_prefix(layer: int) -> str:
    """Checkpoint prefix of a decoder layer (qwen36_40layer_loop.py:53-54)."""
    return f"model.language_model.layers.{layer}."


def is_full_attention_layer(layer: int) -> bool:
    """The 3:1 hybrid pattern of the 40-layer stack: every fourth layer is GQA."""
    return layer % 4 == 3
