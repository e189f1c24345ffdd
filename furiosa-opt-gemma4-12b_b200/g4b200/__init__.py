"""Host-side binding of libg4b200.so: the reference's `ops.rs` entry points over the C ABI.

Each function here has the name, argument order and in-place semantics of the
`#[device]` function of the same name in the reference crate's `src/ops.rs`, and
forwards to `g4_<name>` of include/g4.h.  Tensors are torch CUDA tensors (torch is used
only to hold device memory and streams); shapes and dtypes are checked up front the way
the reference's typed `HbmTensor<T, Chip, m![...]>` signatures enforce them, and a
non-OK status raises `G4Error` (the reference panics).

The library is loaded from this directory (built by `furiosa-opt-gemma4-12b_b200/build.py`).
There is no fallback: if the library is missing, importing this module fails.
"""

from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

__all__ = [
    "G4Error", "Context", "LIB", "lib_path", "exported_symbols", "header_symbols",
    "embed_token", "copy_hidden_state", "sliding_project_qkv", "full_project_qkv",
    "sliding_attention", "sliding_attention_output", "full_attention_first_page",
    "full_attention_page", "full_attention_output", "decoder_feedforward",
    "final_norm_and_logits", "full_attention_paged", "argmax_bf16", "dequant_nvfp4",
    "dequant_fp8", "sliding_project_qkv_nvfp4", "sliding_attention_output_nvfp4",
    "decoder_feedforward_noalloc", "NOALLOC_MAX_INTERMEDIATE", "full_project_qkv_nvfp4",
    "full_attention_output_nvfp4", "attention_gqa",
]

H, L, W = 3840, 15360, 262144
NS, GS, DS, QS, PS, TS = 8, 2, 256, 4096, 2048, 1024
GF, DF, QF, PF, TF, E = 16, 512, 8192, 512, 512, 32768

_HERE = Path(__file__).resolve().parent
_HEADER = _HERE.parent.parent / "include" / "g4.h"

STATUS = {0: "OK", 1: "BAD_ARG", 2: "CUDA", 3: "NCCL", 4: "TIMEOUT", 5: "UNSUPPORTED", 6: "TOO_LARGE"}
NOALLOC_MAX_INTERMEDIATE = 15360  # G4_NOALLOC_MAX_INTERMEDIATE


class G4Error(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn}: G4_ERR_{STATUS.get(code, code)}: {msg}")
        self.code = code


def lib_path() -> Path:
    return _HERE / "libg4b200.so"


def _load() -> ctypes.CDLL:
    # torch first: the library resolves NCCL at run time and must find torch's copy
    import torch  # noqa: F401

    p = lib_path()
    if not p.exists():
        raise ImportError(f"{p} is missing: build it with furiosa-opt-gemma4-12b_b200/build.py")
    return ctypes.CDLL(str(p), mode=os.RTLD_NOW | os.RTLD_GLOBAL)


LIB = _load()
_vp, _i32, _u32, _i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_int64
LIB.g4_version.restype = ctypes.c_char_p
LIB.g4_ctx_last_error.restype = ctypes.c_char_p
LIB.g4_ctx_last_error.argtypes = [_vp]
LIB.g4_ctx_create.argtypes = [_i32, ctypes.POINTER(_vp)]
LIB.g4_ctx_destroy.argtypes = [_vp]
LIB.g4_ctx_set_stream.argtypes = [_vp, _vp]
LIB.g4_ctx_set_wait_budget.argtypes = [_vp, _u32]
LIB.g4_ctx_set_mlp_kernel.argtypes = [_vp, _i32]
LIB.g4_ctx_set_prefill_pieces.argtypes = [_vp, _i32]
LIB.g4_ctx_poll_device_status.argtypes = [_vp, ctypes.POINTER(_u32)]
LIB.g4_nccl_unique_id.argtypes = [ctypes.c_char_p]
LIB.g4_ctx_init_tp.argtypes = [_vp, _i32, _i32, ctypes.c_char_p]
LIB.g4_ctx_tp_peer_exchange.argtypes = [_vp, ctypes.POINTER(ctypes.c_int)]


def header_symbols() -> list[str]:
    """Every function include/g4.h declares."""
    text = _HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(g4_[a-z0-9_]+)\s*\(", text)))


def exported_symbols() -> list[str]:
    out = []
    for s in header_symbols():
        try:
            getattr(LIB, s)
            out.append(s)
        except AttributeError:
            pass
    return out


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _expect(name: str, t, numel: int, dtypes: tuple) -> None:
    """Shape/dtype check standing in for the reference's typed tensor signatures."""
    import torch

    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name}: expected a torch tensor")
    if not t.is_cuda:
        raise ValueError(f"{name}: must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name}: must be contiguous")
    if t.dtype not in dtypes:
        raise TypeError(f"{name}: dtype {t.dtype} not in {dtypes}")
    if numel is not None and t.numel() != numel:
        raise ValueError(f"{name}: {t.numel()} elements, expected {numel}")


class Context:
    """A g4_ctx on one CUDA device (the reference's `Context::acquire()`).

    `stream` is a torch.cuda.Stream (or None for torch's current stream at creation).
    `tp`: optional (rank, world, nccl_id bytes) to make this a tensor-parallel rank.
    """

    def __init__(self, device: int = 0, stream=None, tp: tuple | None = None):
        import torch

        self.device = device
        h = _vp()
        self._check("g4_ctx_create", LIB.g4_ctx_create(device, ctypes.byref(h)), None)
        self.handle = h
        self.world = 1
        self.rank = 0
        s = stream if stream is not None else torch.cuda.current_stream(device)
        self.stream = s
        self._check("g4_ctx_set_stream", LIB.g4_ctx_set_stream(self.handle, s.cuda_stream))
        if tp is not None:
            rank, world, nid = tp
            self._check("g4_ctx_init_tp", LIB.g4_ctx_init_tp(self.handle, rank, world, nid))
            self.rank, self.world = rank, world

    def _check(self, fn: str, code: int, handle=...) -> None:
        if code != 0:
            hv = self.handle if handle is ... else handle
            msg = LIB.g4_ctx_last_error(hv).decode() if hv is not None else ""
            raise G4Error(fn, code, msg)

    def call(self, fn: str, *args) -> None:
        f = getattr(LIB, fn)
        self._check(fn, f(self.handle, *[(_ptr(a) if not isinstance(a, (ctypes._SimpleCData,)) else a) for a in args]))

    def prepare(self, fn: str, *args):
        """Bind `g4_<op>` (e.g. "g4_decoder_feedforward") to these tensors once and return a
        zero-argument callable that issues it, for host loops that launch the same op on
        the same buffers many times.  The arguments are converted here, not per call, and
        not shape-checked: run the op once through its checked wrapper first."""
        f = getattr(LIB, fn)
        keep = list(args)  # the tensors must outlive the callable
        cargs = [self.handle] + [a if isinstance(a, ctypes._SimpleCData) else _vp(_ptr(a)) for a in args]

        def call() -> None:
            code = f(*cargs)
            if code != 0:
                self._check(fn, code)

        call.args = keep
        return call

    @property
    def tp_peer_exchange(self) -> bool:
        """True if this rank's MLP / o-proj kernels all-reduce over NVLink peer memory
        (False: the NCCL fallback, or not tensor-parallel)."""
        out = ctypes.c_int(0)
        self._check("g4_ctx_tp_peer_exchange", LIB.g4_ctx_tp_peer_exchange(self.handle, ctypes.byref(out)))
        return bool(out.value)

    MLP_KERNELS = {"auto": 0, "stream": 1, "tensor": 2}
    prefill_pieces = 2  # the library's default (g4_ctx_set_prefill_pieces)

    def set_mlp_kernel(self, kind: str) -> None:
        """decoder_feedforward kernel of this context: "auto", "stream" (CUDA-core decode +
        mma.sync) or "tensor" (tcgen05 block-scaled FP4; one GPU only)."""
        self._check("g4_ctx_set_mlp_kernel", LIB.g4_ctx_set_mlp_kernel(self.handle, self.MLP_KERNELS[kind]))

    def set_prefill_pieces(self, pieces: int) -> None:
        """NVFP4 pieces per activation in decoder_feedforward_prefill: 1 (fastest, ~10 %
        activation error), 2 (default, ~1 %) or 3 (~0.1 %)."""
        self._check("g4_ctx_set_prefill_pieces", LIB.g4_ctx_set_prefill_pieces(self.handle, pieces))
        self.prefill_pieces = pieces

    def set_wait_budget(self, timeout_us: int) -> None:
        self._check("g4_ctx_set_wait_budget", LIB.g4_ctx_set_wait_budget(self.handle, timeout_us))

    def poll(self) -> int:
        bits = _u32(0)
        code = LIB.g4_ctx_poll_device_status(self.handle, ctypes.byref(bits))
        if code not in (0,):
            raise G4Error("g4_ctx_poll_device_status", code, LIB.g4_ctx_last_error(self.handle).decode())
        return bits.value

    def close(self) -> None:
        if getattr(self, "handle", None) is not None:
            LIB.g4_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        code = LIB.g4_nccl_unique_id(buf)
        if code != 0:
            raise G4Error("g4_nccl_unique_id", code, "")
        return buf.raw


def _declare(name: str, n_ptr_args: int, tail: list | None = None) -> None:
    f = getattr(LIB, name)
    f.argtypes = [_vp] + [_vp] * n_ptr_args + (tail or [])
    f.restype = _i32


for _n, _k in [("g4_embed_token", 3), ("g4_copy_hidden_state", 2), ("g4_sliding_project_qkv", 17),
               ("g4_full_project_qkv", 15), ("g4_sliding_attention", 5), ("g4_sliding_attention_output", 5),
               ("g4_full_attention_first_page", 7), ("g4_full_attention_page", 7),
               ("g4_full_attention_output", 6), ("g4_decoder_feedforward", 13), ("g4_final_norm_and_logits", 4),
               ("g4_sliding_project_qkv_nvfp4", 20), ("g4_sliding_attention_output_nvfp4", 6),
               ("g4_full_project_qkv_nvfp4", 17), ("g4_full_attention_output_nvfp4", 7)]:
    _declare(_n, _k)
LIB.g4_full_attention_paged.argtypes = [_vp, _vp, _vp, _vp, _i32, _i32, _vp, _vp]
LIB.g4_argmax_bf16.argtypes = [_vp, _vp, _i32, _vp]
LIB.g4_sample_top_k_top_p.argtypes = [_vp, _vp, _i32, ctypes.c_float, _i32, ctypes.c_float, _vp, _i32, _vp, _vp]
LIB.g4_attention_gqa.argtypes = [_vp, _vp, _vp, _vp, _vp, _i32, _vp]
LIB.g4_dequant_nvfp4.argtypes = [_vp, _vp, _vp, _i32, _i32, _vp]
LIB.g4_dequant_fp8.argtypes = [_vp, _vp, _i64, _vp]
LIB.g4_decoder_feedforward_noalloc.argtypes = [_vp, _u32] + [_vp] * 13
LIB.g4_decoder_feedforward_prefill.argtypes = [_vp, _i32] + [_vp] * 13
LIB.g4_decoder_feedforward_noalloc.restype = _i32


def _t():
    import torch

    return torch


# ------------------------------------------------------------------------- ops.rs mirror
def embed_token(ctx: Context, embedding_table, offset, out):
    """ops::embed_token (src/ops.rs:9-36)."""
    t = _t()
    _expect("embedding_table", embedding_table, None, (t.bfloat16,))
    _expect("offset", offset, 1, (t.int32,))
    _expect("out", out, H, (t.bfloat16,))
    ctx.call("g4_embed_token", embedding_table, offset, out)


def copy_hidden_state(ctx: Context, x, out):
    """ops::copy_hidden_state (src/ops.rs:38-42)."""
    t = _t()
    _expect("x", x, H, (t.bfloat16,))
    _expect("out", out, H, (t.bfloat16,))
    ctx.call("g4_copy_hidden_state", x, out)


def sliding_project_qkv(ctx: Context, x, q_weight, k_weight, v_weight, q_weight_scale, k_weight_scale,
                        v_weight_scale, input_rms_weight, q_rms_weight, k_rms_weight, kv_offset, rope_offset,
                        cos, sin, k_cache, v_cache, q_out):
    """ops::sliding_project_qkv (src/ops.rs:44-84); TP: the rank's heads."""
    t = _t()
    n = ctx.world
    u8, bf, i32 = (t.uint8, t.float8_e4m3fn), (t.bfloat16,), (t.int32,)
    _expect("x", x, H, bf)
    _expect("q_weight", q_weight, QS // n * H, u8)
    _expect("k_weight", k_weight, PS // n * H, u8)
    _expect("v_weight", v_weight, PS // n * H, u8)
    _expect("q_weight_scale", q_weight_scale, QS // n, bf)
    _expect("k_weight_scale", k_weight_scale, PS // n, bf)
    _expect("v_weight_scale", v_weight_scale, PS // n, bf)
    _expect("input_rms_weight", input_rms_weight, H, bf)
    _expect("q_rms_weight", q_rms_weight, DS, bf)
    _expect("k_rms_weight", k_rms_weight, DS, bf)
    _expect("kv_offset", kv_offset, 1, i32)
    _expect("rope_offset", rope_offset, 1, i32)
    _expect("cos", cos, E * DS, bf)
    _expect("sin", sin, E * DS, bf)
    _expect("k_cache", k_cache, TS * NS // n * DS, bf)
    _expect("v_cache", v_cache, TS * NS // n * DS, bf)
    _expect("q_out", q_out, NS * GS // n * DS, bf)
    ctx.call("g4_sliding_project_qkv", x, q_weight, k_weight, v_weight, q_weight_scale, k_weight_scale,
             v_weight_scale, input_rms_weight, q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos, sin,
             k_cache, v_cache, q_out)


def sliding_project_qkv_nvfp4(ctx: Context, x, q_weight, k_weight, v_weight, q_block_scale, k_block_scale,
                              v_block_scale, q_global_scale, k_global_scale, v_global_scale, input_rms_weight,
                              q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos, sin, k_cache, v_cache,
                              q_out):
    """NVFP4 variant of sliding_project_qkv."""
    t = _t()
    n = ctx.world
    u8, f8, bf, f32 = (t.uint8,), (t.uint8, t.float8_e4m3fn), (t.bfloat16,), (t.float32,)
    _expect("q_weight", q_weight, QS // n * H // 2, u8)
    _expect("k_weight", k_weight, PS // n * H // 2, u8)
    _expect("v_weight", v_weight, PS // n * H // 2, u8)
    _expect("q_block_scale", q_block_scale, QS // n * H // 16, f8)
    _expect("k_block_scale", k_block_scale, PS // n * H // 16, f8)
    _expect("v_block_scale", v_block_scale, PS // n * H // 16, f8)
    for nm, g in (("q_global_scale", q_global_scale), ("k_global_scale", k_global_scale),
                  ("v_global_scale", v_global_scale)):
        _expect(nm, g, 1, f32)
    _expect("x", x, H, bf)
    _expect("cos", cos, E * DS, bf)
    _expect("sin", sin, E * DS, bf)
    _expect("k_cache", k_cache, TS * NS // n * DS, bf)
    _expect("v_cache", v_cache, TS * NS // n * DS, bf)
    _expect("q_out", q_out, NS * GS // n * DS, bf)
    ctx.call("g4_sliding_project_qkv_nvfp4", x, q_weight, k_weight, v_weight, q_block_scale, k_block_scale,
             v_block_scale, q_global_scale, k_global_scale, v_global_scale, input_rms_weight, q_rms_weight,
             k_rms_weight, kv_offset, rope_offset, cos, sin, k_cache, v_cache, q_out)


def full_project_qkv(ctx: Context, x, q_weight, k_weight, q_weight_scale, k_weight_scale, input_rms_weight,
                     q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos, sin, k_cache, v_cache, q_out):
    """ops::full_project_qkv (src/ops.rs:86-124)."""
    t = _t()
    n = ctx.world
    u8, bf, i32 = (t.uint8, t.float8_e4m3fn), (t.bfloat16,), (t.int32,)
    _expect("x", x, H, bf)
    _expect("q_weight", q_weight, QF // n * H, u8)
    _expect("k_weight", k_weight, PF * H, u8)
    _expect("q_weight_scale", q_weight_scale, QF // n, bf)
    _expect("k_weight_scale", k_weight_scale, PF, bf)
    _expect("input_rms_weight", input_rms_weight, H, bf)
    _expect("q_rms_weight", q_rms_weight, DF, bf)
    _expect("k_rms_weight", k_rms_weight, DF, bf)
    _expect("kv_offset", kv_offset, 1, i32)
    _expect("rope_offset", rope_offset, 1, i32)
    _expect("cos", cos, E * DF, bf)
    _expect("sin", sin, E * DF, bf)
    _expect("k_cache", k_cache, TF * DF, bf)
    _expect("v_cache", v_cache, TF * DF, bf)
    _expect("q_out", q_out, GF // n * DF, bf)
    ctx.call("g4_full_project_qkv", x, q_weight, k_weight, q_weight_scale, k_weight_scale, input_rms_weight,
             q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos, sin, k_cache, v_cache, q_out)


def sliding_attention(ctx: Context, q, k, v, mask, out):
    """ops::sliding_attention (src/ops.rs:126-136)."""
    t = _t()
    n = ctx.world
    bf = (t.bfloat16,)
    _expect("q", q, NS * GS // n * DS, bf)
    _expect("k", k, TS * NS // n * DS, bf)
    _expect("v", v, TS * NS // n * DS, bf)
    _expect("mask", mask, TS, (t.float32,))
    _expect("out", out, NS * GS // n * DS, bf)
    ctx.call("g4_sliding_attention", q, k, v, mask, out)


def sliding_attention_output(ctx: Context, x, post_attn_rms_weight, o_weight, o_weight_scale, residual):
    """ops::sliding_attention_output (src/ops.rs:138-158)."""
    t = _t()
    n = ctx.world
    bf = (t.bfloat16,)
    _expect("x", x, QS // n, bf)
    _expect("post_attn_rms_weight", post_attn_rms_weight, H, bf)
    _expect("o_weight", o_weight, H * QS // n, (t.uint8, t.float8_e4m3fn))
    _expect("o_weight_scale", o_weight_scale, H, bf)
    _expect("residual", residual, H, bf)
    ctx.call("g4_sliding_attention_output", x, post_attn_rms_weight, o_weight, o_weight_scale, residual)


def sliding_attention_output_nvfp4(ctx: Context, x, post_attn_rms_weight, o_weight, o_block_scale,
                                   o_global_scale, residual):
    """NVFP4 variant of sliding_attention_output."""
    t = _t()
    n = ctx.world
    bf = (t.bfloat16,)
    _expect("x", x, QS // n, bf)
    _expect("o_weight", o_weight, H * QS // n // 2, (t.uint8,))
    _expect("o_block_scale", o_block_scale, H * QS // n // 16, (t.uint8, t.float8_e4m3fn))
    _expect("o_global_scale", o_global_scale, 1, (t.float32,))
    _expect("residual", residual, H, bf)
    ctx.call("g4_sliding_attention_output_nvfp4", x, post_attn_rms_weight, o_weight, o_block_scale,
             o_global_scale, residual)


def full_project_qkv_nvfp4(ctx: Context, x, q_weight, k_weight, q_block_scale, k_block_scale, q_global_scale,
                           k_global_scale, input_rms_weight, q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos,
                           sin, k_cache, v_cache, q_out):
    """NVFP4 variant of full_project_qkv."""
    t = _t()
    n = ctx.world
    u8, f8, bf, f32 = (t.uint8,), (t.uint8, t.float8_e4m3fn), (t.bfloat16,), (t.float32,)
    _expect("x", x, H, bf)
    _expect("q_weight", q_weight, QF // n * H // 2, u8)
    _expect("k_weight", k_weight, PF * H // 2, u8)
    _expect("q_block_scale", q_block_scale, QF // n * H // 16, f8)
    _expect("k_block_scale", k_block_scale, PF * H // 16, f8)
    _expect("q_global_scale", q_global_scale, 1, f32)
    _expect("k_global_scale", k_global_scale, 1, f32)
    _expect("cos", cos, E * DF, bf)
    _expect("sin", sin, E * DF, bf)
    _expect("k_cache", k_cache, TF * DF, bf)
    _expect("v_cache", v_cache, TF * DF, bf)
    _expect("q_out", q_out, GF // n * DF, bf)
    ctx.call("g4_full_project_qkv_nvfp4", x, q_weight, k_weight, q_block_scale, k_block_scale, q_global_scale,
             k_global_scale, input_rms_weight, q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos, sin, k_cache,
             v_cache, q_out)


def full_attention_output_nvfp4(ctx: Context, x, running_sum, post_attn_rms_weight, o_weight, o_block_scale,
                                o_global_scale, residual):
    """NVFP4 variant of full_attention_output."""
    t = _t()
    n = ctx.world
    bf = (t.bfloat16,)
    _expect("x", x, GF // n * DF, bf)
    _expect("running_sum", running_sum, GF // n, (t.float32,))
    _expect("o_weight", o_weight, H * QF // n // 2, (t.uint8,))
    _expect("o_block_scale", o_block_scale, H * QF // n // 16, (t.uint8, t.float8_e4m3fn))
    _expect("o_global_scale", o_global_scale, 1, (t.float32,))
    _expect("residual", residual, H, bf)
    ctx.call("g4_full_attention_output_nvfp4", x, running_sum, post_attn_rms_weight, o_weight, o_block_scale,
             o_global_scale, residual)


def attention_gqa(ctx: Context, q, k, v, mask, out) -> None:
    """GQA attention of the sliding geometry over mask.numel() cache rows."""
    t = _t()
    n = ctx.world
    rows = mask.numel()
    bf = (t.bfloat16,)
    _expect("q", q, NS * GS // n * DS, bf)
    _expect("k", k, rows * NS // n * DS, bf)
    _expect("v", v, rows * NS // n * DS, bf)
    _expect("mask", mask, rows, (t.float32,))
    _expect("out", out, NS * GS // n * DS, bf)
    ctx._check("g4_attention_gqa", LIB.g4_attention_gqa(ctx.handle, _ptr(q), _ptr(k), _ptr(v), _ptr(mask), rows,
                                                        _ptr(out)))


def _full_page(fn, ctx, q, k, v, mask, running_max, running_sum, out):
    t = _t()
    n = ctx.world
    bf = (t.bfloat16,)
    _expect("q", q, GF // n * DF, bf)
    _expect("k", k, TF * DF, bf)
    _expect("v", v, TF * DF, bf)
    _expect("mask", mask, TF, (t.float32,))
    _expect("running_max", running_max, GF // n, (t.float32,))
    _expect("running_sum", running_sum, GF // n, (t.float32,))
    _expect("out", out, GF // n * DF, bf)
    ctx.call(fn, q, k, v, mask, running_max, running_sum, out)


def full_attention_first_page(ctx: Context, q, k, v, mask, running_max, running_sum, out):
    """ops::full_attention_first_page (src/ops.rs:160-172)."""
    _full_page("g4_full_attention_first_page", ctx, q, k, v, mask, running_max, running_sum, out)


def full_attention_page(ctx: Context, q, k, v, mask, running_max, running_sum, out):
    """ops::full_attention_page (src/ops.rs:174-186)."""
    _full_page("g4_full_attention_page", ctx, q, k, v, mask, running_max, running_sum, out)


def full_attention_paged(ctx: Context, q, k_pages, v_pages, n_pages: int, last_row: int, running_sum, out):
    """All pages of one full-attention layer in one launch; k_pages/v_pages are int64
    CUDA tensors of page addresses."""
    t = _t()
    _expect("k_pages", k_pages, None, (t.int64,))
    _expect("v_pages", v_pages, None, (t.int64,))
    ctx._check("g4_full_attention_paged",
               LIB.g4_full_attention_paged(ctx.handle, _ptr(q), _ptr(k_pages), _ptr(v_pages), n_pages, last_row,
                                           _ptr(running_sum), _ptr(out)))


def full_attention_output(ctx: Context, x, running_sum, post_attn_rms_weight, o_weight, o_weight_scale, residual):
    """ops::full_attention_output (src/ops.rs:188-211)."""
    t = _t()
    n = ctx.world
    bf = (t.bfloat16,)
    _expect("x", x, GF // n * DF, bf)
    _expect("running_sum", running_sum, GF // n, (t.float32,))
    _expect("post_attn_rms_weight", post_attn_rms_weight, H, bf)
    _expect("o_weight", o_weight, H * QF // n, (t.uint8, t.float8_e4m3fn))
    _expect("o_weight_scale", o_weight_scale, H, bf)
    _expect("residual", residual, H, bf)
    ctx.call("g4_full_attention_output", x, running_sum, post_attn_rms_weight, o_weight, o_weight_scale, residual)


def decoder_feedforward(ctx: Context, residual, pre_ff_rms_weight, up_weight_packed, gate_weight_packed,
                        down_weight_packed, up_weight_scale, gate_weight_scale, down_weight_scale,
                        up_global_scale, gate_global_scale, down_global_scale, post_ff_rms_weight, layer_scalar):
    """ops::decoder_feedforward (src/ops.rs:213-253), in place on residual."""
    t = _t()
    n = ctx.world
    bf, u8, f8, f32 = (t.bfloat16,), (t.uint8,), (t.uint8, t.float8_e4m3fn), (t.float32,)
    _expect("residual", residual, H, bf)
    _expect("pre_ff_rms_weight", pre_ff_rms_weight, H, bf)
    _expect("up_weight_packed", up_weight_packed, L // n * H // 2, u8)
    _expect("gate_weight_packed", gate_weight_packed, L // n * H // 2, u8)
    _expect("down_weight_packed", down_weight_packed, H * L // n // 2, u8)
    _expect("up_weight_scale", up_weight_scale, L // n * H // 16, f8)
    _expect("gate_weight_scale", gate_weight_scale, L // n * H // 16, f8)
    _expect("down_weight_scale", down_weight_scale, H * L // n // 16, f8)
    _expect("up_global_scale", up_global_scale, 1, f32)
    _expect("gate_global_scale", gate_global_scale, 1, f32)
    _expect("down_global_scale", down_global_scale, 1, f32)
    _expect("post_ff_rms_weight", post_ff_rms_weight, H, bf)
    _expect("layer_scalar", layer_scalar, 8, bf)
    ctx.call("g4_decoder_feedforward", residual, pre_ff_rms_weight, up_weight_packed, gate_weight_packed,
             down_weight_packed, up_weight_scale, gate_weight_scale, down_weight_scale, up_global_scale,
             gate_global_scale, down_global_scale, post_ff_rms_weight, layer_scalar)


def sample_top_k_top_p(ctx: Context, logits, temperature: float, top_k: int, top_p: float, banned, uniform,
                       out_index) -> None:
    """Top-k / top-p sampling of logits (bf16 [n]; TP: the rank's vocab slice) on the device
    (g4_sample_top_k_top_p, src/host/sampling.rs:20-72).  `banned`: distinct token ids
    (a host sequence); `uniform`: a float32 CUDA tensor holding the draw in [0, 1);
    `out_index`: an int32 CUDA tensor of one element."""
    t = _t()
    _expect("logits", logits, None, (t.bfloat16,))
    _expect("uniform", uniform, 1, (t.float32,))
    _expect("out_index", out_index, 1, (t.int32,))
    ids = list(banned)
    arr = (ctypes.c_int32 * max(1, len(ids)))(*ids)
    ctx._check("g4_sample_top_k_top_p", LIB.g4_sample_top_k_top_p(
        ctx.handle, _ptr(logits), logits.numel(), float(temperature), int(top_k), float(top_p),
        ctypes.cast(arr, _vp), len(ids), _ptr(uniform), _ptr(out_index)))


PREFILL_MAX_TOKENS = 65536


def decoder_feedforward_prefill(ctx: Context, residual, pre_ff_rms_weight, up_weight_packed, gate_weight_packed,
                                down_weight_packed, up_weight_scale, gate_weight_scale, down_weight_scale,
                                up_global_scale, gate_global_scale, down_global_scale, post_ff_rms_weight,
                                layer_scalar):
    """decoder_feedforward for n tokens at once (g4_decoder_feedforward_prefill), in place
    on residual [n, H]; the weights as for `decoder_feedforward`.  The activations are
    quantised per token to NVFP4 for the block-scaled FP4 tensor cores."""
    t = _t()
    w = ctx.world
    bf, u8, f8, f32 = (t.bfloat16,), (t.uint8,), (t.uint8, t.float8_e4m3fn), (t.float32,)
    if residual.dim() != 2 or residual.shape[1] != H:
        raise ValueError(f"residual: expected [n, {H}], got {list(residual.shape)}")
    n = residual.shape[0]
    if not 1 <= n <= PREFILL_MAX_TOKENS:
        raise ValueError(f"residual: {n} tokens, expected 1..{PREFILL_MAX_TOKENS}")
    _expect("residual", residual, n * H, bf)
    _expect("pre_ff_rms_weight", pre_ff_rms_weight, H, bf)
    _expect("up_weight_packed", up_weight_packed, L // w * H // 2, u8)
    _expect("gate_weight_packed", gate_weight_packed, L // w * H // 2, u8)
    _expect("down_weight_packed", down_weight_packed, H * L // w // 2, u8)
    _expect("up_weight_scale", up_weight_scale, L // w * H // 16, f8)
    _expect("gate_weight_scale", gate_weight_scale, L // w * H // 16, f8)
    _expect("down_weight_scale", down_weight_scale, H * L // w // 16, f8)
    _expect("up_global_scale", up_global_scale, 1, f32)
    _expect("gate_global_scale", gate_global_scale, 1, f32)
    _expect("down_global_scale", down_global_scale, 1, f32)
    _expect("post_ff_rms_weight", post_ff_rms_weight, H, bf)
    _expect("layer_scalar", layer_scalar, 8, bf)
    ctx.call("g4_decoder_feedforward_prefill", ctypes.c_int32(n), residual, pre_ff_rms_weight, up_weight_packed,
             gate_weight_packed, down_weight_packed, up_weight_scale, gate_weight_scale, down_weight_scale,
             up_global_scale, gate_global_scale, down_global_scale, post_ff_rms_weight, layer_scalar)


def final_norm_and_logits(ctx: Context, input, rms_weight, lm_head_weight, out):
    """ops::final_norm_and_logits (src/ops.rs:255-312); TP: the rank's vocab slice."""
    t = _t()
    n = ctx.world
    bf = (t.bfloat16,)
    _expect("input", input, H, bf)
    _expect("rms_weight", rms_weight, H, bf)
    _expect("lm_head_weight", lm_head_weight, W // n * H, bf)
    _expect("out", out, W // n, bf)
    ctx.call("g4_final_norm_and_logits", input, rms_weight, lm_head_weight, out)


def argmax_bf16(ctx: Context, logits, out_index) -> None:
    t = _t()
    _expect("out_index", out_index, 1, (t.int32,))
    ctx._check("g4_argmax_bf16", LIB.g4_argmax_bf16(ctx.handle, _ptr(logits), logits.numel(), _ptr(out_index)))


def dequant_nvfp4(ctx: Context, packed, block_scale, rows: int, cols: int, out) -> None:
    ctx._check("g4_dequant_nvfp4", LIB.g4_dequant_nvfp4(ctx.handle, _ptr(packed), _ptr(block_scale), rows, cols,
                                                         _ptr(out)))


def dequant_fp8(ctx: Context, weight, out) -> None:
    ctx._check("g4_dequant_fp8", LIB.g4_dequant_fp8(ctx.handle, _ptr(weight), weight.numel(), _ptr(out)))


def decoder_feedforward_noalloc(residual, pre_ff_rms_weight, up_weight_packed, gate_weight_packed,
                                down_weight_packed, up_weight_scale, gate_weight_scale, down_weight_scale,
                                up_global_scale, gate_global_scale, down_global_scale, post_ff_rms_weight,
                                layer_scalar, stream=None):
    """decoder_feedforward without a Context, for hosts where this library may not allocate
    device memory (g4_decoder_feedforward_noalloc; no counterpart in the reference).

    Same math and kernel as `decoder_feedforward`, in place on `residual`.  The
    intermediate size n is read from `gate_weight_packed` ([n, H/2] codes); n may be at
    most NOALLOC_MAX_INTERMEDIATE.  Scratch lives in one fixed device array per GPU that
    every call shares, so calls must not overlap on the GPU.  Runs on `stream` (default:
    torch's current stream of residual's device).
    """
    t = _t()
    bf, u8, f8, f32 = (t.bfloat16,), (t.uint8,), (t.uint8, t.float8_e4m3fn), (t.float32,)
    _expect("gate_weight_packed", gate_weight_packed, None, u8)
    if gate_weight_packed.numel() % (H // 2):
        raise ValueError(f"gate_weight_packed: {gate_weight_packed.numel()} bytes is not [n, {H // 2}]")
    n = gate_weight_packed.numel() // (H // 2)
    _expect("residual", residual, H, bf)
    _expect("pre_ff_rms_weight", pre_ff_rms_weight, H, bf)
    _expect("up_weight_packed", up_weight_packed, n * H // 2, u8)
    _expect("down_weight_packed", down_weight_packed, H * n // 2, u8)
    _expect("up_weight_scale", up_weight_scale, n * H // 16, f8)
    _expect("gate_weight_scale", gate_weight_scale, n * H // 16, f8)
    _expect("down_weight_scale", down_weight_scale, H * n // 16, f8)
    _expect("up_global_scale", up_global_scale, 1, f32)
    _expect("gate_global_scale", gate_global_scale, 1, f32)
    _expect("down_global_scale", down_global_scale, 1, f32)
    _expect("post_ff_rms_weight", post_ff_rms_weight, H, bf)
    _expect("layer_scalar", layer_scalar, 8, bf)
    with t.cuda.device(residual.device):
        s = stream if stream is not None else t.cuda.current_stream()
        code = LIB.g4_decoder_feedforward_noalloc(
            s.cuda_stream, n, *[_ptr(a) for a in (
                residual, pre_ff_rms_weight, up_weight_packed, gate_weight_packed, down_weight_packed,
                up_weight_scale, gate_weight_scale, down_weight_scale, up_global_scale, gate_global_scale,
                down_global_scale, post_ff_rms_weight, layer_scalar)])
    if code != 0:
        why = {6: f"intermediate size {n} exceeds the fixed scratch limit of {NOALLOC_MAX_INTERMEDIATE} rows",
               5: f"intermediate size {n} is not 15360, 7680 or a multiple of 128 up to 3840",
               1: "a pointer is null or misaligned"}.get(code, "a CUDA call failed")
        raise G4Error("g4_decoder_feedforward_noalloc", code, why)
