"""ctypes binding of ``libria_attention.so`` (the C ABI in include/ria_attention.h).

This is the only door to the device kernels.  There is no CPU fallback: when
the library is missing or a CUDA device is absent, calls raise.  Each wrapper
takes torch tensors only as carriers of device pointers, strides and the
current stream, and maps a nonzero status to ``RuntimeError`` (``ValueError``
for argument errors), the exception types router-ia raises for the same
conditions.
"""

from __future__ import annotations

import ctypes
import re
from ctypes import c_char_p, c_int, c_int32, c_int64, c_uint, c_void_p, POINTER
from pathlib import Path

import torch

from .build import INCLUDE, LIB_PATH

RIA_OK = 0
RIA_ERR_INVALID = 1

_lib: ctypes.CDLL | None = None

# Optional instrumentation: an object with ``before(name)`` / ``after(name,
# kernels)`` called around each kernel-launching entry point (the benchmark
# records CUDA events and counts launches through it).
launch_hook = None


class _Hooked:
    def __init__(self, name: str, kernels: int = 1):
        self.name, self.kernels = name, kernels

    def __enter__(self):
        if launch_hook is not None:
            launch_hook.before(self.name)

    def __exit__(self, *exc):
        if launch_hook is not None and exc[0] is None:
            launch_hook.after(self.name, self.kernels)
        return False

_SIGNATURES: dict[str, tuple[object, list]] = {
    "ria_last_error_string": (c_char_p, []),
    "ria_abi_version": (c_int, []),
    "ria_device_error": (c_int, [c_int, POINTER(c_uint)]),
    "ria_gdn_decode_step": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_int64, c_int32, c_void_p],
    ),
    "ria_gqa_decode_workspace_bytes": (c_int64, [c_int32, c_int32]),
    "ria_gqa_decode_split_pages": (c_int32, [c_int64, c_int32]),
    "ria_gqa_decode_paged": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_int64, c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_int64,
         c_int32, c_int32, c_int32, c_void_p],
    ),
    "ria_gqa_decode_paged_static": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_int64, c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int64, c_int32, c_int32,
         c_int32, c_void_p],
    ),
    "ria_rmsnorm_gemv": (
        c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32, c_int32, c_void_p]),
    "ria_gemv_residual": (
        c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32, c_int32,
                c_void_p]),
    "ria_deltanet_layer_decode_scratch_bytes": (c_int64, [c_int32]),
    "ria_deltanet_layer_decode": (
        c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                c_int64, c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_int64, c_void_p, c_int64, c_int32,
                c_void_p]),
    "ria_gqa_layer_decode_scratch_bytes": (c_int64, [c_int32, c_int32]),
    "ria_gqa_layer_decode": (
        c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                c_int64, c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int64, c_void_p,
                c_int64, c_void_p, c_int64, c_int32, c_int32, c_int32, c_void_p]),
    "ria_moe_workspace_bytes": (c_int64, [c_int32, c_int32, c_int32]),
    "ria_moe_decode": (
        c_int,
        [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
         c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_int32, c_int32, c_void_p],
    ),
    "ria_moe_prompt_norm": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int32, c_void_p]),
    "ria_silu_mul_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "ria_moe_prompt_combine": (
        c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32,
                c_int32, c_void_p]),
    "ria_lm_head_workspace_bytes": (c_int64, [c_int32]),
    "ria_lm_head_greedy": (
        c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int32, c_void_p, c_int64, c_void_p, c_void_p,
                c_int64, c_int32, c_void_p]),
    "ria_final_norm_f16": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int32, c_int32, c_void_p]),
    "ria_argmax_f16_rows": (c_int, [c_void_p, c_int64, c_int32, c_int32, c_void_p, c_void_p]),
    "ria_gdn_chunk_prefill_workspace_bytes": (c_int64, [c_int32, c_int32, c_int32]),
    "ria_gdn_chunk_prefill": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
         c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int32, c_int32,
         c_int32, c_int32, c_void_p],
    ),
    "ria_gqa_prefill_workspace_bytes": (c_int64, [c_int32, c_int32]),
    "ria_gqa_prefill": (
        c_int,
        [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
         c_void_p, c_int64, c_int32, c_int32, c_void_p],
    ),
    "ria_conv1d_prefill": (
        c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int32, c_int32, c_int32,
                c_void_p]),
    "ria_gdn_gates": (
        c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                c_void_p]),
    "ria_gated_rmsnorm": (
        c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int32, c_int32, c_void_p]),
    "ria_umma_selftest": (c_int, [c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ria_advance_positions": (c_int, [c_void_p, c_void_p, c_int32, c_void_p]),
    "ria_rmsnorm_rows": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int32, c_int32, c_void_p]),
    "ria_rmsnorm_rows_f16": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int32, c_int32, c_void_p]),
    "ria_residual_add": (
        c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32, c_void_p]),
    "ria_conv1d_step": (
        c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_int32, c_void_p]),
    "ria_rope_apply": (c_int, [c_void_p, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p]),
    "ria_kv_append_paged": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int32, c_void_p, c_void_p, c_int64,
                                    c_void_p, c_int32, c_void_p, c_int32, c_int32, c_void_p]),
}


def header_symbols() -> list[str]:
    """Entry points declared in include/ria_attention.h."""
    text = (INCLUDE / "ria_attention.h").read_text()
    return re.findall(r"^RIA_API\s+[\w\s\*]+?\b(ria_\w+)\s*\(", text, flags=re.M)


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is None:
        path = Path(LIB_PATH)
        if not path.exists():
            raise RuntimeError(
                f"router-ia B200 CUDA library not found at {path}; build it with "
                "`python router-ia_b200/ria_b200/build.py` (there is no CPU fallback)"
            )
        handle = ctypes.CDLL(str(path))
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().ria_last_error_string()
    return msg.decode("utf-8", "replace") if msg else ""


def _check(rc: int, what: str) -> None:
    if rc == RIA_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == RIA_ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(msg)


def _stream(t: torch.Tensor) -> int:
    """The current CUDA stream of t's device (the raw handle; the same value
    as ``torch.cuda.current_stream(t.device).cuda_stream`` at a fraction of
    its cost -- it is looked up on every launch)."""
    return torch._C._cuda_getCurrentRawStream(t.get_device())


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("router-ia B200 kernels need CUDA tensors (no CPU fallback)")


def device_error(clear: bool = True) -> int:
    """Device error word set by kernels (0 = none); synchronises the device."""
    code = c_uint(0)
    _check(lib().ria_device_error(1 if clear else 0, ctypes.byref(code)), "ria_device_error")
    return int(code.value)


def gdn_decode_step(mixed, z, b, a, conv_weight, a_log, dt_bias, norm_weight, conv_state, rec_state, slots, out):
    """K1 over ``mixed.shape[0]`` sequences (see ria_gdn_decode_step)."""
    _require_cuda(mixed, z, b, a, conv_weight, conv_state, rec_state, out)
    batch = mixed.shape[0]
    num_slots = rec_state.shape[0]
    if conv_state.shape[0] != num_slots:
        raise ValueError("conv_state and rec_state must have the same number of slots")
    with _Hooked("gdn_decode"):
        rc = lib().ria_gdn_decode_step(
            mixed.data_ptr(), mixed.stride(0), z.data_ptr(), z.stride(0), b.data_ptr(), b.stride(0), a.data_ptr(),
            a.stride(0), conv_weight.data_ptr(), a_log.data_ptr(), dt_bias.data_ptr(), norm_weight.data_ptr(),
            conv_state.data_ptr(), rec_state.data_ptr(), _ptr(slots), num_slots, out.data_ptr(), out.stride(0), batch,
            _stream(mixed))
    _check(rc, "ria_gdn_decode_step")


def gqa_workspace_bytes(batch: int, max_splits: int) -> int:
    return int(lib().ria_gqa_decode_workspace_bytes(batch, max_splits))


def gqa_split_pages(total_blocks: int, num_kv_heads: int = 2) -> int:
    return int(lib().ria_gqa_decode_split_pages(total_blocks, num_kv_heads))


def gqa_decode_paged(q, k, v, q_norm_w, k_norm_w, inv_freq, k_pool, v_pool, block_table, seq_lens, positions,
                     out, workspace, split_pages, max_splits, seq_len0=0, position0=0):
    """K3 over ``q.shape[0]`` sequences (see ria_gqa_decode_paged)."""
    _require_cuda(q, k, v, k_pool, v_pool, block_table, out)
    batch = q.shape[0]
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    with _Hooked("gqa_decode", 2 if int(max_splits) > 1 else 1):
        rc = lib().ria_gqa_decode_paged(
            q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), q_norm_w.data_ptr(),
            k_norm_w.data_ptr(), inv_freq.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.shape[1],
            block_table.data_ptr(), block_table.stride(0), _ptr(seq_lens), _ptr(positions), int(seq_len0),
            int(position0), out.data_ptr(), out.stride(0), _ptr(workspace), ws_bytes, batch, int(split_pages),
            int(max_splits), _stream(q))
    _check(rc, "ria_gqa_decode_paged")


GQA_STATIC_SCRATCH_BYTES = 4 << 20  # RIA_GQA_STATIC_SCRATCH_BYTES


def gqa_decode_paged_static(q, k, v, q_norm_w, k_norm_w, inv_freq, k_pool, v_pool, block_table, seq_lens,
                            positions, out, split_pages, max_splits, seq_len0=0, position0=0):
    """K3 with the split partials in the library's fixed device array instead
    of a caller workspace (see ria_gqa_decode_paged_static): for callers that
    cannot allocate device memory where they decode."""
    _require_cuda(q, k, v, k_pool, v_pool, block_table, out)
    with _Hooked("gqa_decode", 2 if int(max_splits) > 1 else 1):
        rc = lib().ria_gqa_decode_paged_static(
            q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), q_norm_w.data_ptr(),
            k_norm_w.data_ptr(), inv_freq.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.shape[1],
            block_table.data_ptr(), block_table.stride(0), _ptr(seq_lens), _ptr(positions), int(seq_len0),
            int(position0), out.data_ptr(), out.stride(0), q.shape[0], int(split_pages), int(max_splits), _stream(q))
    _check(rc, "ria_gqa_decode_paged_static")


GDN_PREFILL_WORKSPACE_CAP = 2 << 30  # bytes; longer prompts run in blocks of chunks


def gdn_chunk_prefill_workspace_bytes(batch: int, seq_len: int, num_v_heads: int) -> int:
    return int(lib().ria_gdn_chunk_prefill_workspace_bytes(int(batch), int(seq_len), int(num_v_heads)))


def gdn_chunk_prefill(q, k, v, g, beta, initial_state, final_state, out, workspace=None):
    """K2 (see ria_gdn_chunk_prefill).  q, k [B, T, Hk, 128] bf16; v, out
    [B, T, Hv, 128] bf16; g, beta [B, T, Hv] f32; states [B, Hv, 128, 128] f32.
    ``workspace``: uint8 CUDA tensor (allocated here when None, up to
    GDN_PREFILL_WORKSPACE_CAP bytes); returned for reuse."""
    _require_cuda(q, k, v, g, beta, final_state, out)
    B, T, Hk, dk = q.shape
    Hv = v.shape[2]
    for t, name in ((q, "q"), (k, "k"), (v, "v"), (out, "out")):
        if t.dtype != torch.bfloat16 or t.shape[-1] != 128 or t.stride(-1) != 1 or t.stride(-2) != 128:
            raise ValueError(f"{name}: expected [B, T, H, 128] bf16 with contiguous heads")
    if g.dtype != torch.float32 or beta.dtype != torch.float32 or g.stride() != beta.stride() or g.stride(-1) != 1:
        raise ValueError("g and beta: [B, T, Hv] float32 with the same strides")
    if final_state.dtype != torch.float32 or not final_state.is_contiguous():
        raise ValueError("final_state: contiguous [B, Hv, 128, 128] float32")
    if initial_state is not None and (initial_state.dtype != torch.float32 or not initial_state.is_contiguous()):
        raise ValueError("initial_state: contiguous [B, Hv, 128, 128] float32")
    if workspace is None:
        need = gdn_chunk_prefill_workspace_bytes(B, T, Hv)
        one_chunk = gdn_chunk_prefill_workspace_bytes(B, 1, Hv)
        size = max(one_chunk, min(need, GDN_PREFILL_WORKSPACE_CAP // one_chunk * one_chunk)) if need else 16
        workspace = torch.empty(size, dtype=torch.uint8, device=q.device)
    with _Hooked("gdn_prefill"):
        rc = lib().ria_gdn_chunk_prefill(
            q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(),
            v.stride(0), v.stride(1), g.data_ptr(), beta.data_ptr(), g.stride(0), g.stride(1), _ptr(initial_state),
            final_state.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1), workspace.data_ptr(),
            workspace.numel() * workspace.element_size(), B, T, Hk, Hv, _stream(q))
    _check(rc, "ria_gdn_chunk_prefill")
    return workspace


def gqa_prefill(q, k, v, q_norm_w, k_norm_w, inv_freq, k_pool, v_pool, block_table, seq_lens, positions, out,
                workspace=None):
    """K4 (see ria_gqa_prefill): q [B, T, 8192], k, v [B, T, 512] bf16 views
    with unit inner stride; out [B, T, 4096] bf16."""
    _require_cuda(q, k, v, k_pool, v_pool, block_table, seq_lens, positions, out)
    B, T = q.shape[0], q.shape[1]
    need = int(lib().ria_gqa_prefill_workspace_bytes(B, T))
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 16) // 2, dtype=torch.bfloat16, device=q.device)
    with _Hooked("gqa_prefill", 2):
        rc = lib().ria_gqa_prefill(
            q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(),
            v.stride(0), v.stride(1), q_norm_w.data_ptr(), k_norm_w.data_ptr(), inv_freq.data_ptr(),
            k_pool.data_ptr(), v_pool.data_ptr(), k_pool.shape[1], block_table.data_ptr(), block_table.stride(0),
            seq_lens.data_ptr(), positions.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
            workspace.data_ptr(), workspace.numel() * workspace.element_size(), B, T, _stream(q))
    _check(rc, "ria_gqa_prefill")
    return workspace


def conv1d_prefill(x, conv_state, weight, out):
    """x, out [B, T, C] bf16 (unit channel stride); conv_state [B, C, 4] bf16."""
    _require_cuda(x, conv_state, weight, out)
    B, T, Cc = x.shape
    with _Hooked("conv1d_prefill", 2):
        rc = lib().ria_conv1d_prefill(x.data_ptr(), x.stride(0), x.stride(1), conv_state.data_ptr(), weight.data_ptr(),
                                      out.data_ptr(), out.stride(0), out.stride(1), B, T, Cc, _stream(x))
    _check(rc, "ria_conv1d_prefill")


def gdn_gates(a, b, a_log, dt_bias, g, beta):
    """a, b [rows, heads] bf16 views; g, beta [rows, heads] f32 contiguous."""
    _require_cuda(a, b, g, beta)
    rows, heads = a.shape
    with _Hooked("gdn_gates"):
        rc = lib().ria_gdn_gates(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), a_log.data_ptr(),
                                 dt_bias.data_ptr(), g.data_ptr(), beta.data_ptr(), rows, heads, _stream(a))
    _check(rc, "ria_gdn_gates")


def gated_rmsnorm(o, z, weight, out):
    """o, z, out [rows, heads*128] bf16 views (unit inner stride)."""
    _require_cuda(o, z, weight, out)
    rows, width = o.shape
    with _Hooked("gated_rmsnorm"):
        rc = lib().ria_gated_rmsnorm(o.data_ptr(), o.stride(0), z.data_ptr(), z.stride(0), weight.data_ptr(),
                                     out.data_ptr(), out.stride(0), rows, width // 128, _stream(o))
    _check(rc, "ria_gated_rmsnorm")


def umma_selftest(a, b, a_mn_major: int, b_mn_major: bool, f16: bool = False):
    """d = a @ b through one tcgen05 MMA chain (a: [128, k], b: [k, n] fp32
    CUDA tensors; operands rounded to bf16, or fp16 with ``f16``).  a_mn_major:
    0 K-major, 1 MN-major (shared memory), 2 A held in tensor memory."""
    _require_cuda(a, b)
    a = a.float().contiguous()
    b = b.float().contiguous()
    n, k = b.shape[1], a.shape[1]
    d = torch.empty(128, n, dtype=torch.float32, device=a.device)
    with _Hooked("umma_selftest"):
        rc = lib().ria_umma_selftest(int(a_mn_major) | (4 if f16 else 0), int(b_mn_major), n, k, a.data_ptr(), b.data_ptr(),
                                     d.data_ptr(), _stream(a))
    _check(rc, "ria_umma_selftest")
    return d


def advance_positions(seq_lens, positions):
    with _Hooked("advance"):
        rc = lib().ria_advance_positions(seq_lens.data_ptr(), positions.data_ptr(), seq_lens.shape[0], _stream(seq_lens))
    _check(rc, "ria_advance_positions")


GEMV_MAX_BATCH = 8


def rmsnorm_gemv(x, norm_w, w, out):
    """out [B, n] bf16 = w [n, k] fp16 . fp16(rmsnorm(x [B, k] f32) * (1 + norm_w)), B <= 8."""
    _require_cuda(x, norm_w, w, out)
    if w.dtype != torch.float16 or out.dtype != torch.bfloat16:
        raise ValueError(f"rmsnorm_gemv: fp16 weights and a bf16 output expected, got {w.dtype} / {out.dtype}")
    with _Hooked("rmsnorm_gemv"):
        rc = lib().ria_rmsnorm_gemv(x.data_ptr(), x.stride(0), norm_w.data_ptr(), w.data_ptr(), w.stride(0),
                                    out.data_ptr(), out.stride(0), x.shape[0], w.shape[0], w.shape[1], _stream(x))
    _check(rc, "ria_rmsnorm_gemv")


def gemv_residual(a, w, x0, out):
    """out [B, n] f32 = x0 + bf16(w [n, k] . a [B, k] bf16), B <= 8."""
    _require_cuda(a, w, x0, out)
    with _Hooked("gemv_residual"):
        rc = lib().ria_gemv_residual(a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), x0.data_ptr(), x0.stride(0),
                                     out.data_ptr(), out.stride(0), a.shape[0], w.shape[0], w.shape[1], _stream(a))
    _check(rc, "ria_gemv_residual")


def deltanet_layer_scratch_bytes(batch: int) -> int:
    return int(lib().ria_deltanet_layer_decode_scratch_bytes(batch))


def gqa_layer_scratch_bytes(batch: int, max_splits: int) -> int:
    return int(lib().ria_gqa_layer_decode_scratch_bytes(batch, max_splits))


def deltanet_layer_args(w) -> tuple:
    """The weight arguments of ria_deltanet_layer_decode for one layer's
    DeltaNetWeights (device pointers and strides; valid while ``w`` lives)."""
    _require_cuda(w.in_norm, w.w_in, w.conv_w, w.a_log, w.dt_bias, w.norm_w, w.w_out)
    return (w.in_norm.data_ptr(), w.w_in.data_ptr(), w.w_in.stride(0), w.conv_w.data_ptr(), w.a_log.data_ptr(),
            w.dt_bias.data_ptr(), w.norm_w.data_ptr(), w.w_out.data_ptr(), w.w_out.stride(0))


def gqa_layer_args(w) -> tuple:
    """The weight arguments of ria_gqa_layer_decode for one layer's GqaWeights."""
    _require_cuda(w.in_norm, w.w_in, w.q_norm, w.k_norm, w.w_out)
    return (w.in_norm.data_ptr(), w.w_in.data_ptr(), w.w_in.stride(0), w.q_norm.data_ptr(), w.k_norm.data_ptr(),
            w.w_out.data_ptr(), w.w_out.stride(0))


def deltanet_layer_decode(x, wargs, conv_state, rec_state, out, scratch, slots=None):
    """One DeltaNet layer step for x [B <= 8, 2048] f32 in one C call
    (ria_deltanet_layer_decode): out = the layer's residual output."""
    if not (x.is_cuda and out.is_cuda and scratch.is_cuda):
        raise RuntimeError("router-ia B200 kernels need CUDA tensors (no CPU fallback)")
    in_norm, w_in, w_in_s, conv_w, a_log, dt_bias, norm_w, w_out, w_out_s = wargs
    args = (x.data_ptr(), x.stride(0), in_norm, w_in, w_in_s, conv_w, a_log, dt_bias, norm_w, w_out, w_out_s,
            conv_state.data_ptr(), rec_state.data_ptr(), _ptr(slots), rec_state.shape[0], out.data_ptr(),
            out.stride(0), scratch.data_ptr(), scratch.numel() * scratch.element_size(), x.shape[0], _stream(x))
    if launch_hook is None:
        rc = lib().ria_deltanet_layer_decode(*args)
    else:
        with _Hooked("deltanet_layer", 3):
            rc = lib().ria_deltanet_layer_decode(*args)
    if rc:
        _check(rc, "ria_deltanet_layer_decode")


def gqa_layer_decode(x, wargs, inv_freq, k_pool, v_pool, block_table, out, scratch, split_pages, max_splits,
                     seq_lens=None, positions=None, seq_len0=0, position0=0):
    """One GQA layer step for x [B <= 8, 2048] f32 in one C call
    (ria_gqa_layer_decode): out = the layer's residual output."""
    if not (x.is_cuda and out.is_cuda and scratch.is_cuda and k_pool.is_cuda):
        raise RuntimeError("router-ia B200 kernels need CUDA tensors (no CPU fallback)")
    in_norm, w_in, w_in_s, q_norm, k_norm, w_out, w_out_s = wargs
    args = (x.data_ptr(), x.stride(0), in_norm, w_in, w_in_s, q_norm, k_norm, inv_freq.data_ptr(), k_pool.data_ptr(),
            v_pool.data_ptr(), k_pool.shape[1], block_table.data_ptr(), block_table.stride(0), _ptr(seq_lens),
            _ptr(positions), int(seq_len0), int(position0), w_out, w_out_s, out.data_ptr(), out.stride(0),
            scratch.data_ptr(), scratch.numel() * scratch.element_size(), x.shape[0], int(split_pages),
            int(max_splits), _stream(x))
    if launch_hook is None:
        rc = lib().ria_gqa_layer_decode(*args)
    else:
        with _Hooked("gqa_layer", 4 if int(max_splits) > 1 else 3):
            rc = lib().ria_gqa_layer_decode(*args)
    if rc:
        _check(rc, "ria_gqa_layer_decode")


def moe_workspace_bytes(batch: int, num_experts: int, top_k: int) -> int:
    return int(lib().ria_moe_workspace_bytes(batch, num_experts, top_k))


def moe_decode(residual, w, out, expert_ids, expert_weights, shared_gate, workspace, top_k: int):
    """One MoE block for residual [B, 2048] f32 into out (may alias residual).
    ``w`` holds the stacked bf16 weights (a ``weights.MoeWeights``);
    expert_ids [B, k] int32, expert_weights [B, k] f32, shared_gate [B] f32
    receive the routing; workspace a uint8 device buffer."""
    _require_cuda(residual, out, expert_ids, expert_weights, shared_gate, workspace)
    num_experts = w["router"].shape[0]
    with _Hooked("moe", kernels=2):
        rc = lib().ria_moe_decode(
            residual.data_ptr(), residual.stride(0), w["post_norm"].data_ptr(), w["router"].data_ptr(),
            w["shared_gate"].data_ptr(), w["experts_gate"].data_ptr(), w["experts_up"].data_ptr(),
            w["experts_down"].data_ptr(), w["shared_gate_proj"].data_ptr(), w["shared_up_proj"].data_ptr(),
            w["shared_down_proj"].data_ptr(), out.data_ptr(), out.stride(0), expert_ids.data_ptr(),
            expert_weights.data_ptr(), shared_gate.data_ptr(), workspace.data_ptr(), workspace.numel(),
            residual.shape[0], num_experts, top_k, _stream(residual))
    _check(rc, "ria_moe_decode")


def moe_prompt_norm(x, post_norm, h, h_bf16):
    """h [N, 2048] f32, h_bf16 [N, 2048] bf16 <- rmsnorm(x) * (1 + post_norm)."""
    _require_cuda(x, post_norm, h, h_bf16)
    with _Hooked("moe_prompt_norm"):
        rc = lib().ria_moe_prompt_norm(x.data_ptr(), x.stride(0), post_norm.data_ptr(), h.data_ptr(), h_bf16.data_ptr(),
                                       x.shape[0], _stream(x))
    _check(rc, "ria_moe_prompt_norm")


def silu_mul_bf16(gate, up, out):
    """out = bf16(silu(gate) * up), contiguous bf16 tensors of one shape."""
    _require_cuda(gate, up, out)
    with _Hooked("silu_mul"):
        rc = lib().ria_silu_mul_bf16(gate.data_ptr(), up.data_ptr(), out.data_ptr(), out.numel(), _stream(out))
    _check(rc, "ria_silu_mul_bf16")


def moe_prompt_combine(x, expert_out, sorted_position, weights, shared_out, shared_gate, out):
    """out [N, 2048] f32 = x + sum_j weights[:, j] expert_out[sorted_position[:, j]] + shared_gate shared_out."""
    _require_cuda(x, expert_out, sorted_position, weights, shared_out, shared_gate, out)
    with _Hooked("moe_prompt_combine"):
        rc = lib().ria_moe_prompt_combine(x.data_ptr(), x.stride(0), expert_out.data_ptr(), sorted_position.data_ptr(),
                                          weights.data_ptr(), shared_out.data_ptr(), shared_gate.data_ptr(),
                                          out.data_ptr(), out.stride(0), x.shape[0], weights.shape[1], _stream(x))
    _check(rc, "ria_moe_prompt_combine")


LM_HEAD_MAX_BATCH = 8


def lm_head_workspace_bytes(batch: int) -> int:
    return int(lib().ria_lm_head_workspace_bytes(batch))


def lm_head_greedy(x, norm_w, lm_head, next_ids, workspace, logits=None):
    """next_ids [B] int32 = argmax(fp16(rmsnorm(x) * (1 + norm_w)) . lm_head^T)
    for x [B, 2048] f32, B <= 8; lm_head [V, 2048] fp16; logits [B, V] fp16
    (optional) receives the fp16 logits; workspace a zero-filled uint8 buffer."""
    _require_cuda(x, norm_w, lm_head, next_ids, workspace)
    lp = logits.data_ptr() if logits is not None else None
    ls = logits.stride(0) if logits is not None else 0
    with _Hooked("lm_head", kernels=2):
        rc = lib().ria_lm_head_greedy(x.data_ptr(), x.stride(0), norm_w.data_ptr(), lm_head.data_ptr(),
                                      lm_head.stride(0), lm_head.shape[0], lp, ls, next_ids.data_ptr(),
                                      workspace.data_ptr(), workspace.numel(), x.shape[0], _stream(x))
    _check(rc, "ria_lm_head_greedy")


def final_norm_f16(x, weight, out):
    """out [B, n] fp16 = fp16(rmsnorm(x [B, n] f32) * (1 + weight))."""
    _require_cuda(x, weight, out)
    with _Hooked("final_norm"):
        rc = lib().ria_final_norm_f16(x.data_ptr(), x.stride(0), weight.data_ptr(), out.data_ptr(), out.stride(0),
                                      x.shape[0], x.shape[1], _stream(x))
    _check(rc, "ria_final_norm_f16")


def argmax_f16_rows(logits, out):
    """out [B] int32 = first index of each row's largest value; logits [B, V] fp16."""
    _require_cuda(logits, out)
    with _Hooked("argmax"):
        rc = lib().ria_argmax_f16_rows(logits.data_ptr(), logits.stride(0), logits.shape[1], logits.shape[0],
                                       out.data_ptr(), _stream(logits))
    _check(rc, "ria_argmax_f16_rows")


def rmsnorm_rows(x, weight, out):
    """out = rmsnorm(x) * (1 + weight) in out's dtype (bf16 or fp16)."""
    _require_cuda(x, weight, out)
    if out.dtype == torch.float16:
        fn, name = lib().ria_rmsnorm_rows_f16, "ria_rmsnorm_rows_f16"
    elif out.dtype == torch.bfloat16:
        fn, name = lib().ria_rmsnorm_rows, "ria_rmsnorm_rows"
    else:
        raise ValueError(f"rmsnorm_rows: output dtype {out.dtype} (bf16 or fp16)")
    with _Hooked("rmsnorm"):
        rc = fn(x.data_ptr(), x.stride(0), weight.data_ptr(), out.data_ptr(), out.stride(0), x.shape[0], x.shape[1],
                _stream(x))
    _check(rc, name)


def residual_add(x0, proj, out):
    _require_cuda(x0, proj, out)
    with _Hooked("residual_add"):
        rc = lib().ria_residual_add(x0.data_ptr(), x0.stride(0), proj.data_ptr(), proj.stride(0), out.data_ptr(),
                                    out.stride(0), x0.shape[0], x0.shape[1], _stream(x0))
    _check(rc, "ria_residual_add")


def conv1d_step(x, conv_state, weight, out):
    _require_cuda(x, conv_state, weight, out)
    with _Hooked("conv1d_step"):
        rc = lib().ria_conv1d_step(x.data_ptr(), x.stride(0), conv_state.data_ptr(), weight.data_ptr(),
                                   out.data_ptr(), out.stride(0), x.shape[0], x.shape[1], _stream(x))
    _check(rc, "ria_conv1d_step")


def rope_apply(x, inv_freq, rope_dim: int, position: int):
    _require_cuda(x, inv_freq)
    rows, head_dim = x.shape
    with _Hooked("rope_apply"):
        rc = lib().ria_rope_apply(x.data_ptr(), rows, head_dim, rope_dim, inv_freq.data_ptr(), int(position), _stream(x))
    _check(rc, "ria_rope_apply")


def kv_append_paged(k_new, v_new, k_pool, v_pool, block_table, seq_lens=None, seq_len0: int = 0):
    """Write k_new[b], v_new[b] ([B, 512] bf16 or f32) at row seq_lens[b] of
    sequence b's paged cache (see ria_kv_append_paged)."""
    _require_cuda(k_new, v_new, k_pool, v_pool, block_table)
    if k_new.dtype != v_new.dtype or k_new.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"kv_append_paged: bf16 or f32 K/V rows expected, got {k_new.dtype} / {v_new.dtype}")
    with _Hooked("kv_append"):
        rc = lib().ria_kv_append_paged(k_new.data_ptr(), k_new.stride(0), v_new.data_ptr(), v_new.stride(0),
                                       1 if k_new.dtype == torch.float32 else 0, k_pool.data_ptr(), v_pool.data_ptr(),
                                       k_pool.shape[1], block_table.data_ptr(), block_table.stride(0), _ptr(seq_lens),
                                       int(seq_len0), k_new.shape[0], _stream(k_new))
    _check(rc, "ria_kv_append_paged")
