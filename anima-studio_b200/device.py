"""The C-ABI binding (libanima_b200.so via ctypes) and the per-device context.

Plays the part of the reference's GPU object (app/gpu/device.js:59-232): one context per CUDA
device, calls recorded in order on the current torch stream, errors raised as exceptions on the
host. Device memory comes from torch's caching allocator (the reference's BufferPool role).
There is no fallback: without the compiled library or a B200 every operator raises.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("ANIMA_LIB", os.path.join(HERE, "libanima_b200.so"))

ANIMA_F32, ANIMA_BF16, ANIMA_F16, ANIMA_I8, ANIMA_U8 = range(5)
ACT = {None: 0, "none": 0, "gelu": 1, "silu": 2}
W_I8, W_W4, W_BF16, W_F32, W_F16 = range(5)
OUT_STORE, OUT_RESID, OUT_QKV_NORM_ROPE, OUT_HEAD_NORM = range(4)

DTYPE_CODE = {torch.float32: ANIMA_F32, torch.bfloat16: ANIMA_BF16, torch.float16: ANIMA_F16,
              torch.int8: ANIMA_I8, torch.uint8: ANIMA_U8}

# Every entry point declared in include/anima_b200.h (tests check the library exports all of them).
EXPORTS = [
    "anima_ctx_create", "anima_ctx_destroy", "anima_ctx_set_stream", "anima_sync", "anima_last_error",
    "anima_alloc", "anima_free", "anima_upload", "anima_download", "anima_profile_report", "anima_version",
    "anima_unpack_w4", "anima_linear", "anima_matmul", "anima_lora_down", "anima_layernorm_mod", "anima_layernorm_mod_quant",
    "anima_rotate", "anima_rotate_quant", "anima_act_rotate_quant", "anima_quant_rows", "anima_rmsnorm", "anima_qk_norm_rope", "anima_rope",
    "anima_attention", "anima_attention_noalloc", "anima_elementwise", "anima_zero", "anima_patchify", "anima_unpatchify",
    "anima_timestep_embedding", "anima_euler_step", "anima_lincomb", "anima_selftest_wait_timeout",
    "anima_ctx_set_attention_split", "anima_ipc_alloc", "anima_ipc_open", "anima_ipc_close", "anima_ipc_free",
    "anima_peer_barrier", "anima_conv3x3", "anima_channel_norm",
]


class AnimaError(RuntimeError):
    """A failed C-ABI call (status != 0), with the library's message."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"[anima status {status}] {msg}")
        self.status = status


class QAct(C.Structure):
    _fields_ = [("rows", C.c_int), ("cols", C.c_int), ("ld", C.c_int), ("hi", C.c_void_p), ("lo", C.c_void_p),
                ("scale", C.c_void_p)]


class Weight(C.Structure):
    _fields_ = [("kind", C.c_int), ("N", C.c_int), ("K", C.c_int), ("data", C.c_void_p), ("scale", C.c_void_p),
                ("s_rel", C.c_void_p), ("codebook", C.c_void_p), ("bias", C.c_void_p)]


class LinearOpts(C.Structure):
    _fields_ = [("act", C.c_int), ("add", C.c_void_p), ("ld_add", C.c_int), ("out_mode", C.c_int),
                ("out_dtype", C.c_int), ("out", C.c_void_p), ("ldo", C.c_int), ("gate", C.c_void_p),
                ("gate_off", C.c_int), ("norm_q", C.c_void_p), ("norm_k", C.c_void_p), ("rope", C.c_void_p),
                ("rope_rows", C.c_int), ("n_q", C.c_int), ("eps", C.c_float),
                ("lora_t", C.c_void_p), ("ld_t", C.c_int), ("lora_t_lo", C.c_int), ("lora_bt", C.c_void_p), ("ld_bt", C.c_int),
                ("lora_count", C.c_int), ("lora_off", C.c_int * 4), ("lora_n", C.c_int * 4),
                ("lora_r0", C.c_int * 4), ("lora_r", C.c_int * 4),
                ("peer_count", C.c_int), ("peer_kv", C.c_void_p * 8), ("peer_row0", C.c_int), ("peer_rows", C.c_int),
                ("peer_item_rows", C.c_int)]


class PeerGroup(C.Structure):
    _fields_ = [("rank", C.c_int), ("world", C.c_int), ("flags", C.c_void_p * 8), ("counter", C.c_void_p),
                ("timeout_us", C.c_uint)]


class AttentionArgs(C.Structure):
    _fields_ = [("batch", C.c_int), ("heads", C.c_int), ("head_dim", C.c_int), ("Lq", C.c_int), ("Lk", C.c_int),
                ("dtype", C.c_int),
                ("q", C.c_void_p), ("ldq", C.c_longlong), ("q_bstride", C.c_longlong), ("q_off", C.c_int),
                ("k", C.c_void_p), ("ldk", C.c_longlong), ("k_bstride", C.c_longlong), ("k_off", C.c_int),
                ("v", C.c_void_p), ("ldv", C.c_longlong), ("v_bstride", C.c_longlong), ("v_off", C.c_int),
                ("out", C.c_void_p), ("ldo", C.c_longlong), ("o_bstride", C.c_longlong), ("out_dtype", C.c_int),
                ("key_len", C.c_void_p), ("scale", C.c_float), ("group", C.c_int), ("causal", C.c_int)]


_lib = None
_lib_lock = threading.Lock()


def load_library(path: str = LIB_PATH):
    """dlopen libanima_b200.so once and declare the signatures; raises if it is missing."""
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise AnimaError(-1, f"{path} is missing: build it with __graft_entry__.build() "
                                 "(this package has no CPU or fallback path)")
        lib = C.CDLL(path)
        vp, i, f, ll, sz = C.c_void_p, C.c_int, C.c_float, C.c_longlong, C.c_size_t
        sig = {
            "anima_ctx_create": [i, C.POINTER(vp)], "anima_ctx_destroy": [vp], "anima_ctx_set_stream": [vp, vp],
            "anima_sync": [vp], "anima_ctx_set_attention_split": [vp, i], "anima_alloc": [vp, sz, C.POINTER(vp)], "anima_free": [vp, vp],
            "anima_upload": [vp, vp, vp, sz], "anima_download": [vp, vp, vp, sz],
            "anima_profile_report": [vp, C.c_char_p, sz], "anima_version": [],
            "anima_unpack_w4": [vp, vp, vp, vp, i, i, vp],
            "anima_linear": [vp, C.POINTER(QAct), C.POINTER(Weight), C.POINTER(LinearOpts)],
            "anima_matmul": [vp, i, i, i, f, vp, i, C.POINTER(Weight), i, vp, i, i, vp, i],
            "anima_lora_down": [vp, C.POINTER(QAct), vp, i, vp, i],
            "anima_layernorm_mod": [vp, vp, i, i, vp, i, i, f, i, vp, i],
            "anima_layernorm_mod_quant": [vp, vp, i, i, vp, i, i, f, C.POINTER(QAct)],
            "anima_rotate": [vp, vp, i, i, i, i, vp, i],
            "anima_rotate_quant": [vp, vp, i, i, i, i, C.POINTER(QAct)],
            "anima_quant_rows": [vp, vp, i, i, i, i, C.POINTER(QAct)],
            "anima_act_rotate_quant": [vp, vp, i, i, i, i, i, C.POINTER(QAct)],
            "anima_rmsnorm": [vp, vp, i, i, i, vp, f, vp, i],
            "anima_qk_norm_rope": [vp, vp, i, i, i, i, i, vp, vp, vp, i, f],
            "anima_rope": [vp, vp, i, i, i, i, i, i, vp, i],
            "anima_attention": [vp, C.POINTER(AttentionArgs)],
            "anima_attention_noalloc": [vp, C.POINTER(AttentionArgs)],
            "anima_elementwise": [vp, i, vp, vp, vp, ll], "anima_zero": [vp, vp, sz],
            "anima_patchify": [vp, vp, i, i, i, vp], "anima_unpatchify": [vp, vp, i, i, i, vp],
            "anima_timestep_embedding": [vp, vp, i, vp],
            "anima_euler_step": [vp, vp, vp, vp, f, f, f, ll, vp],
            "anima_ipc_alloc": [vp, sz, C.POINTER(vp), C.c_char_p], "anima_ipc_open": [vp, C.c_char_p, C.POINTER(vp)],
            "anima_ipc_close": [vp, vp], "anima_ipc_free": [vp, vp],
            "anima_peer_barrier": [vp, C.POINTER(PeerGroup)],
            "anima_conv3x3": [vp, vp, i, i, i, C.POINTER(Weight), i, vp, i],
            "anima_channel_norm": [vp, vp, ll, i, vp, i, vp],
        }
        for name, args in sig.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = C.c_int
        lib.anima_last_error.argtypes = []
        lib.anima_last_error.restype = C.c_char_p
        _lib = lib
        return lib


def exported_symbols(path: str = LIB_PATH):
    """Names from EXPORTS that the shared object resolves (loads it without calling anything)."""
    lib = C.CDLL(path)
    return [n for n in EXPORTS if hasattr(lib, n)]


def check(status: int):
    if status != 0:
        msg = _lib.anima_last_error().decode(errors="replace") if _lib is not None else "library not loaded"
        raise AnimaError(status, msg)


# Entry points that enqueue one of this library's kernels (anima_zero is a memset).
LAUNCHING = set(EXPORTS) - {"anima_ctx_create", "anima_ctx_destroy", "anima_ctx_set_stream", "anima_sync",
                            "anima_last_error", "anima_alloc", "anima_free", "anima_upload", "anima_download",
                            "anima_profile_report", "anima_version", "anima_zero", "anima_selftest_wait_timeout",
                            "anima_ctx_set_attention_split", "anima_ipc_alloc", "anima_ipc_open", "anima_ipc_close",
                            "anima_ipc_free"}


class KernelTimer:
    """Records CUDA events around selected entry points on the launching stream, keyed by
    (entry point, tag): `with KernelTimer({"anima_linear"}) as kt: ...; kt.summary()`."""

    active = None

    def __init__(self, names):
        self.names = set(names)
        self.events = []

    def __enter__(self):
        KernelTimer.active = self
        return self

    def __exit__(self, *exc):
        KernelTimer.active = None

    def summary(self) -> dict:
        """{(name, tag): (launches, total ms)} after a synchronize."""
        torch.cuda.synchronize()
        out = {}
        for name, tag, e0, e1, work in self.events:
            n, ms, w = out.get((name, tag), (0, 0.0, 0.0))
            out[(name, tag)] = (n + 1, ms + e0.elapsed_time(e1), w + work)
        return out


class Context:
    """One anima_ctx per CUDA device; every call is issued on torch's current stream."""

    _per_device: dict = {}
    launches = 0  # kernels this process enqueued through the library (all devices)

    def __init__(self, device: int):
        self.lib = load_library()
        if not torch.cuda.is_available():
            raise AnimaError(-1, "no CUDA device: the anima operators run only on a B200 (sm_100a)")
        self.device = device
        h = C.c_void_p()
        with torch.cuda.device(device):
            check(self.lib.anima_ctx_create(device, C.byref(h)))
        self.h = h

    @classmethod
    def get(cls, device=None) -> "Context":
        if device is None:
            device = torch.cuda.current_device()
        if isinstance(device, torch.device):
            device = device.index if device.index is not None else torch.cuda.current_device()
        ctx = cls._per_device.get(device)
        if ctx is None:
            ctx = cls._per_device[device] = Context(device)
        return ctx

    def set_attention_split(self, mode: int):
        """-1 automatic stream-K for attention, 0 whole units only, 1 stream-K wherever legal."""
        check(self.lib.anima_ctx_set_attention_split(self.h, int(mode)))

    def bind_stream(self):
        check(self.lib.anima_ctx_set_stream(self.h, C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)))
        return self.h

    def call(self, name: str, *args, tag: str | None = None, work: float = 0.0, kernels: int = 1):
        """Run entry point `name` on torch's current stream; `kernels` = library kernels it enqueues."""
        h = self.bind_stream()
        kt = KernelTimer.active
        if kt is not None and name in kt.names:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            check(getattr(self.lib, name)(h, *args))
            e1.record()
            kt.events.append((name, tag, e0, e1, work))
        else:
            check(getattr(self.lib, name)(h, *args))
        if name in LAUNCHING:
            Context.launches += kernels

    def sync(self):
        """gpu.sync: wait for the stream and raise on a device-side fault or timed-out wait."""
        check(self.lib.anima_sync(self.bind_stream()))

    def profile_report(self) -> str:
        buf = C.create_string_buffer(1 << 16)
        check(self.lib.anima_profile_report(self.bind_stream(), buf, len(buf)))
        return buf.value.decode()


def ptr(t) -> C.c_void_p:
    """Device pointer of a tensor (None -> NULL)."""
    if t is None:
        return C.c_void_p(0)
    return C.c_void_p(t.data_ptr())


def ctx_for(t: torch.Tensor) -> Context:
    if not t.is_cuda:
        raise AnimaError(-1, "anima operators take CUDA tensors (there is no CPU path)")
    return Context.get(t.device.index)
