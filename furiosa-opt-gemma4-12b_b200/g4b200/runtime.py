"""Host binding of the decode runtime: Model (src/host/load.rs), Workspace and Decode
(src/host/runtime.rs), greedy generation (src/host/generate.rs without host sampling).

`Model` registers device tensors by checkpoint name (g4_model_set_tensor) and keeps them
alive; `Workspace` owns the KV caches, RoPE tables, offsets and logits
(g4_workspace_create).  `Workspace.generate` is g4_generate_greedy: prefill one position
per step, then greedy decoding, with the position and the token kept on the device and
the whole step replayed as one CUDA graph.
"""

from __future__ import annotations

import ctypes

from . import LIB, Context, G4Error, H, W, _i32, _u32, _vp

_u64 = ctypes.c_uint64
LIB.g4_model_create.argtypes = [_i32, ctypes.POINTER(_vp)]
LIB.g4_model_destroy.argtypes = [_vp]
LIB.g4_model_set_tensor.argtypes = [_vp, ctypes.c_char_p, _vp, _u64]
LIB.g4_model_last_error.argtypes = [_vp]
LIB.g4_model_last_error.restype = ctypes.c_char_p
LIB.g4_model_layer_is_full.argtypes = [_i32]
LIB.g4_workspace_create.argtypes = [_vp, _vp, _i32, ctypes.POINTER(_vp)]
LIB.g4_workspace_set_sampling.argtypes = [_vp, ctypes.c_float, _i32, ctypes.c_float, _vp, _i32, _u64]
LIB.g4_workspace_destroy.argtypes = [_vp]
LIB.g4_workspace_kv_cache.argtypes = [_vp, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_u64)]
LIB.g4_workspace_logits.argtypes = [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_i32)]
LIB.g4_workspace_hidden.argtypes = [_vp, ctypes.POINTER(_vp)]
LIB.g4_decode_run.argtypes = [_vp, _vp, _vp, _i32, _i32]
LIB.g4_decode_begin.argtypes = [_vp, _vp, ctypes.POINTER(_i32), _i32, _i32, _i32]
LIB.g4_decode_steps.argtypes = [_vp, _vp, _vp, _i32, _i32]
LIB.g4_decode_tokens.argtypes = [_vp, _vp, ctypes.POINTER(_i32), _i32, ctypes.POINTER(_i32)]
LIB.g4_decode_predictions.argtypes = [_vp, _vp, ctypes.POINTER(_i32), _i32, ctypes.POINTER(_i32)]
LIB.g4_decode_last_prediction.argtypes = [_vp, _vp, ctypes.POINTER(_i32), ctypes.POINTER(_i32)]
LIB.g4_generate_greedy.argtypes = [_vp, _vp, _vp, ctypes.POINTER(_i32), _i32, _i32, _i32, _i32,
                                   ctypes.POINTER(_i32)]
LIB.g4_model_load_safetensors.argtypes = [_vp, ctypes.c_char_p, _i32, ctypes.POINTER(_vp)]
LIB.g4_checkpoint_check.argtypes = [ctypes.c_char_p, _i32, _i32, ctypes.c_char_p, _u64]
for _f in ("g4_model_load_safetensors", "g4_checkpoint_check", "g4_model_create", "g4_model_destroy", "g4_model_set_tensor", "g4_workspace_create",
           "g4_workspace_destroy", "g4_workspace_kv_cache", "g4_workspace_logits", "g4_workspace_hidden",
           "g4_decode_run", "g4_decode_begin", "g4_decode_steps", "g4_decode_tokens",
           "g4_decode_predictions", "g4_decode_last_prediction", "g4_generate_greedy"):
    getattr(LIB, _f).restype = _i32


def layer_is_full(layer: int) -> bool:
    return bool(LIB.g4_model_layer_is_full(layer))


class Model:
    """g4_model: the decoder's weight set as registered device pointers.

    `tensors` maps checkpoint names (include/g4.h, g4_model_set_tensor) to contiguous CUDA
    tensors in the device formats; the Model keeps references so they outlive it."""

    def __init__(self, n_layers: int, tensors: dict | None = None):
        h = _vp()
        code = LIB.g4_model_create(n_layers, ctypes.byref(h))
        if code != 0:
            raise G4Error("g4_model_create", code, f"n_layers={n_layers}")
        self.handle = h
        self.n_layers = n_layers
        self._keep: list = []
        for name, t in (tensors or {}).items():
            self.set_tensor(name, t)

    def set_tensor(self, name: str, t) -> None:
        if not t.is_contiguous():
            raise ValueError(f"{name}: must be contiguous")
        code = LIB.g4_model_set_tensor(self.handle, name.encode(), t.data_ptr(), t.numel() * t.element_size())
        if code != 0:
            raise G4Error("g4_model_set_tensor", code, LIB.g4_model_last_error(self.handle).decode())
        self._keep.append(t)

    def close(self) -> None:
        if getattr(self, "handle", None) is not None:
            LIB.g4_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def check_checkpoint(path: str, n_layers: int, world: int = 1) -> tuple[bool, str]:
    """g4_checkpoint_check: (True, "") if the safetensors file holds an n_layers text
    decoder the loader accepts for `world` ranks, else (False, reason).  No GPU needed."""
    buf = ctypes.create_string_buffer(512)
    code = LIB.g4_checkpoint_check(str(path).encode(), n_layers, world, buf, 512)
    return code == 0, buf.value.decode()


def load_checkpoint(ctx: Context, path: str, n_layers: int) -> Model:
    """g4_model_load_safetensors: the context rank's shard of every tensor, on the device,
    owned by the returned Model."""
    h = _vp()
    ctx._check("g4_model_load_safetensors",
               LIB.g4_model_load_safetensors(ctx.handle, str(path).encode(), n_layers, ctypes.byref(h)))
    m = Model.__new__(Model)
    m.handle, m.n_layers, m._keep = h, n_layers, []
    return m


def _copy_out(ptr: int, nbytes: int, like):
    """Device bytes at `ptr` into a new CUDA tensor (uint8 view of `nbytes`)."""
    import torch
    from cuda.bindings import runtime as cudart

    out = torch.empty(nbytes, dtype=torch.uint8, device=like)
    err, = cudart.cudaMemcpy(out.data_ptr(), ptr, nbytes, cudart.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
    if int(err) != 0:
        raise RuntimeError(f"cudaMemcpy failed: {err}")
    return out


class Workspace:
    """g4_workspace: KV caches, RoPE tables, offsets, decode scratch and logits."""

    def __init__(self, ctx: Context, model: Model, max_positions: int):
        h = _vp()
        ctx._check("g4_workspace_create", LIB.g4_workspace_create(ctx.handle, model.handle, max_positions,
                                                                  ctypes.byref(h)))
        self.handle, self.ctx, self.model, self.max_positions = h, ctx, model, max_positions

    def kv_cache_ptrs(self, layer: int) -> tuple[int, int, int]:
        k, v, n = _vp(), _vp(), _u64()
        self.ctx._check("g4_workspace_kv_cache", LIB.g4_workspace_kv_cache(self.handle, layer, ctypes.byref(k),
                                                                          ctypes.byref(v), ctypes.byref(n)))
        return k.value, v.value, n.value

    def kv_cache(self, layer: int):
        """Copies of layer `layer`'s K and V caches as bf16 CUDA tensors."""
        import torch

        k, v, n = self.kv_cache_ptrs(layer)
        dev = f"cuda:{self.ctx.device}"
        torch.cuda.synchronize(dev)
        return (_copy_out(k, n, dev).view(torch.bfloat16), _copy_out(v, n, dev).view(torch.bfloat16))

    def set_sampling(self, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0, banned=(),
                     seed: int = 0) -> None:
        """Sampling mode of the following steps (g4_workspace_set_sampling): top_k 0 is
        greedy; otherwise top-k / top-p with the device's per-position draw from `seed`."""
        ids = list(banned)
        arr = (ctypes.c_int32 * max(1, len(ids)))(*ids)
        code = LIB.g4_workspace_set_sampling(self.handle, float(temperature), int(top_k), float(top_p),
                                             ctypes.cast(arr, _vp), len(ids), int(seed) & (2 ** 64 - 1))
        if code != 0:
            raise G4Error("g4_workspace_set_sampling", code, "bad sampling parameters")

    def logits(self):
        import torch

        p, n = _vp(), _i32()
        self.ctx._check("g4_workspace_logits", LIB.g4_workspace_logits(self.handle, ctypes.byref(p), ctypes.byref(n)))
        dev = f"cuda:{self.ctx.device}"
        torch.cuda.synchronize(dev)
        return _copy_out(p.value, n.value * 2, dev).view(torch.bfloat16)

    def hidden(self):
        import torch

        p = _vp()
        self.ctx._check("g4_workspace_hidden", LIB.g4_workspace_hidden(self.handle, ctypes.byref(p)))
        dev = f"cuda:{self.ctx.device}"
        torch.cuda.synchronize(dev)
        return _copy_out(p.value, H * 2, dev).view(torch.bfloat16)

    def run(self, token: int, pos: int) -> None:
        """Decode::run at one position (async)."""
        self.ctx._check("g4_decode_run", LIB.g4_decode_run(self.ctx.handle, self.handle, self.model.handle, token, pos))

    def last_prediction(self) -> tuple[int, int]:
        t, p = _i32(), _i32()
        self.ctx._check("g4_decode_last_prediction",
                        LIB.g4_decode_last_prediction(self.ctx.handle, self.handle, ctypes.byref(t), ctypes.byref(p)))
        return t.value, p.value

    def predictions(self, max_out: int) -> list[int]:
        """Greedy prediction of every step since `begin` (prompt positions included)."""
        out = (_i32 * max(1, max_out))()
        n = _i32()
        self.ctx._check("g4_decode_predictions", LIB.g4_decode_predictions(self.ctx.handle, self.handle, out, max_out,
                                                                           ctypes.byref(n)))
        return list(out[:n.value])

    def begin(self, prompt, start_pos: int, max_new: int) -> None:
        arr = (_i32 * len(prompt))(*[int(x) for x in prompt])
        self.ctx._check("g4_decode_begin", LIB.g4_decode_begin(self.ctx.handle, self.handle, arr, len(prompt),
                                                               start_pos, max_new))

    def steps(self, n: int, use_graph: bool = True) -> None:
        self.ctx._check("g4_decode_steps", LIB.g4_decode_steps(self.ctx.handle, self.handle, self.model.handle, n,
                                                               1 if use_graph else 0))

    def tokens(self, max_out: int) -> list[int]:
        out = (_i32 * max(1, max_out))()
        n = _i32()
        self.ctx._check("g4_decode_tokens", LIB.g4_decode_tokens(self.ctx.handle, self.handle, out, max_out,
                                                                 ctypes.byref(n)))
        return list(out[:n.value])

    def generate(self, prompt, max_new: int, start_pos: int = 0, use_graph: bool = True) -> list[int]:
        arr = (_i32 * len(prompt))(*[int(x) for x in prompt])
        out = (_i32 * max(1, max_new))()
        self.ctx._check("g4_generate_greedy",
                        LIB.g4_generate_greedy(self.ctx.handle, self.handle, self.model.handle, arr, len(prompt),
                                               start_pos, max_new, 1 if use_graph else 0, out))
        return list(out[:max_new])

    def close(self) -> None:
        if getattr(self, "handle", None) is not None:
            LIB.g4_workspace_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def model_from_synthetic(m: dict, device=None) -> Model:
    """A runtime Model over a g4formats.model.synthetic_model dict (its tensors moved to
    `device` first when given)."""
    from g4formats import model as fm

    def dev(t):
        return t if device is None else t.to(device)

    layers = [{k: dev(v) for k, v in lt.items()} for lt in m["layers"]]
    rm = Model(m["n_layers"])
    rm.set_tensor(fm.EMBED, dev(m["embed"]))
    rm.set_tensor(fm.FINAL_NORM, dev(m["final_norm"]))
    for i in range(m["n_layers"]):
        for k, t in layers[i % m["distinct"]].items():
            rm.set_tensor(f"{fm.PREFIX}{i}.{k}", t)
    return rm


__all__ = ["Model", "Workspace", "model_from_synthetic", "layer_is_full", "W"]
