"""LoRA side paths on (possibly quantized) linears, without touching the base weights (app/lora.js).

y = W x + sum_e scale_e * B_e (A_e x), evaluated next to the int8 GEMM and added in its epilogue
before the activation (ops.js:55-57, 70-87). ConvRot layers receive rotated inputs x_r = x H and
x A^T = x_r (A H)^T, so A is rotated once at load (lora.js:67-84, 103-134). scale = strength *
alpha / r, or strength without an alpha (lora.js:141-149; tools/reference.py:78).

File naming: PEFT ("<prefix><module>.lora_A/B.weight") or kohya ("lora_unet_<module_with_
underscores>.lora_down/up.weight" + ".alpha"); LoKr/LoHa/DoRA tensors are counted as unsupported.
"""

from __future__ import annotations

import ctypes as C
import re
from dataclasses import dataclass

import torch

from . import device as dev
from . import quant
from .device import ctx_for, ptr

SUFFIXES = [(".lora_A.weight", "A"), (".lora_B.weight", "B"), (".lora_down.weight", "A"),
            (".lora_up.weight", "B"), (".alpha", "alpha")]
TE_PREFIXES = ["lora_te_", "lora_te1_", "text_encoder.", "text_encoders.qwen3_06b.transformer.", "te."]
DIT_PREFIXES = ["lora_unet_", "model.diffusion_model.", "diffusion_model.", "base_model.model.", "transformer.",
                "unet."]
UNSUPPORTED = re.compile(r"(lokr_|hada_|\.dora_scale|\.diff$|\.diff_b$|\.w_norm|\.b_norm)")


def norm_name(name: str) -> str:
    return name.replace(".", "_")


def hadamard_rows(a: torch.Tensor) -> torch.Tensor:
    """A H per 256-feature group of every row (lora.js:67-84): the rotation ConvRot inputs get."""
    return quant.rotate(a.float())


def linear_registry(model) -> dict:
    """normalized module name -> (Linear, off, n) for every linear of a model (lora.js:48-65)."""
    from .weights import Linear

    reg = {}
    seen = set()

    def walk(o):
        if id(o) in seen or o is None or isinstance(o, (torch.Tensor, str, int, float)):
            return
        seen.add(id(o))
        if isinstance(o, Linear):
            if o.parts:
                for name, off, n in o.parts:
                    reg[norm_name(name)] = (o, off, n)
            elif o.name:
                reg[norm_name(o.name)] = (o, 0, o.N)
            return
        if isinstance(o, dict):
            for v in o.values():
                walk(v)
        elif isinstance(o, (list, tuple)):
            for v in o:
                walk(v)
        elif hasattr(o, "__dict__"):
            for v in vars(o).values():
                walk(v)

    walk(model)
    return reg


def find_target(module: str, dit_reg: dict, te_reg: dict | None = None):
    """Strip a known prefix and look the module up (lora.js:89-102)."""
    te = False
    name = module
    for p in TE_PREFIXES:
        if name.startswith(p):
            name, te = name[len(p):], True
            break
    if not te:
        for p in DIT_PREFIXES:
            if name.startswith(p):
                name = name[len(p):]
                break
    key = norm_name(name)
    for reg in ([te_reg] if te else [dit_reg, te_reg]):
        if not reg:
            continue
        if key in reg:
            return reg[key]
        if "model_" + key in reg:
            return reg["model_" + key]
    return None


@dataclass
class LoraModule:
    target: tuple       # (Linear, off, n)
    A: torch.Tensor     # [r, K] fp32 on the device, rotated for ConvRot targets
    B: torch.Tensor     # [n, r] fp32 on the device
    r: int
    alpha_scale: float


@dataclass
class Lora:
    modules: list
    matched: int
    total: int
    unsupported: int
    skipped: int


def load_lora(tensors: dict, dit_reg: dict, te_reg: dict | None = None, device="cuda") -> Lora:
    """Group a LoRA file's tensors by module, match them to linears and upload them (lora.js:103-134)."""
    groups: dict = {}
    unsupported = 0
    for key in tensors:
        if UNSUPPORTED.search(key):
            unsupported += 1
            continue
        for suf, role in SUFFIXES:
            if key.endswith(suf):
                groups.setdefault(key[: -len(suf)], {})[role] = key
                break
    modules = []
    skipped = 0
    for module, keys in groups.items():
        if "A" not in keys or "B" not in keys:
            skipped += 1
            continue
        target = find_target(module, dit_reg, te_reg)
        A = tensors[keys["A"]].float()
        B = tensors[keys["B"]].float()
        r = A.shape[0]
        if target is None or A.shape[1] != target[0].K or B.shape[0] != target[2] or B.shape[1] != r:
            skipped += 1
            continue
        if target[0].quantized:
            A = hadamard_rows(A)
        alpha = float(tensors[keys["alpha"]].float().reshape(-1)[0]) if "alpha" in keys else None
        modules.append(LoraModule(target, A.to(device).contiguous(), B.to(device).contiguous(), r,
                                  alpha / r if alpha else 1.0))
    return Lora(modules, len(modules), len(groups), unsupported, skipped)


def attach_loras(registries, active):
    """Replace every side path with [(lora, strength)] (lora.js:141-149)."""
    for reg in registries:
        if reg:
            for (W, _, _) in reg.values():
                W.lora = []
    for lora, strength in active:
        if not strength:
            continue
        for m in lora.modules:
            W, off, n = m.target
            W.lora.append({"A": m.A, "B": m.B, "r": m.r, "scale": strength * m.alpha_scale, "off": off, "n": n})
    for reg in registries:
        if reg:
            for (W, _, _) in reg.values():
                W._lora_cat = None
                W._lora_bt = None
                W._lora_down = None
                W._lora_down_slices = None
                W._lora_up = None
    # the side streams of the K-sliced down-projection, created here (outside any CUDA graph
    # capture) rather than on their first use, which may be inside one
    for lora, strength in active:
        for m in lora.modules if strength else []:
            if m.A.is_cuda:
                _side_streams(m.A.device, 3)
                break


def _cat_A(W):
    """All entries' A stacked [sum r, K] (cached per attach)."""
    cat = getattr(W, "_lora_cat", None)
    if cat is None:
        cat = torch.cat([e["A"] for e in W.lora], 0).contiguous()
        W._lora_cat = cat
    return cat


def lora_delta(x, W) -> torch.Tensor:
    """[M, N] fp32 low-rank update for quantized rows x (ops.js:70-87): T = x_r A^T for all entries
    at once, then each entry's B into its column slice, scaled."""
    M = x.rows
    A = _cat_A(W)
    R = A.shape[0]
    ctx = ctx_for(x.hi)
    T = torch.empty(M, R, dtype=torch.float32, device=x.hi.device)
    qa = x.c()
    ctx.call("anima_lora_down", C.byref(qa), ptr(A), R, ptr(T), R)
    D = torch.empty(M, W.N, dtype=torch.float32, device=x.hi.device)
    ctx.call("anima_zero", ptr(D), D.numel() * 4)
    r0 = 0
    for e in W.lora:
        wb = dev.Weight()
        wb.kind, wb.N, wb.K, wb.data = dev.W_F32, e["n"], e["r"], e["B"].data_ptr()
        Cp = C.c_void_p(D.data_ptr() + 4 * e["off"])
        Tp = C.c_void_p(T.data_ptr() + 4 * r0)
        ctx.call("anima_matmul", M, e["n"], e["r"], C.c_float(e["scale"]), Tp, R, C.byref(wb), 0, Cp, W.N, 1,
                 C.c_void_p(0), 0)
        r0 += e["r"]
    return D


def _fusable(W) -> bool:
    """The fused epilogue takes up to 4 entries with 128-aligned column ranges and ranks that are
    multiples of 4 up to 32; anything else goes through the [M, N] delta (lora_delta)."""
    return (0 < len(W.lora) <= 4 and all(e["off"] % 128 == 0 and e["n"] % 128 == 0 and e["r"] % 4 == 0
                                         and e["r"] <= 32 for e in W.lora))


def _cat_Bt(W):
    """scale_e * B_e^T of every entry in its rows and columns of one [sum r, N] matrix (cached per
    attach; only each entry's own columns are read)."""
    bt = getattr(W, "_lora_bt", None)
    if bt is None:
        R = sum(e["r"] for e in W.lora)
        bt = torch.zeros(R, W.N, dtype=torch.float32, device=W.lora[0]["B"].device)
        r0 = 0
        for e in W.lora:
            bt[r0:r0 + e["r"], e["off"]:e["off"] + e["n"]] = (e["B"].float() * e["scale"]).t()
            r0 += e["r"]
        W._lora_bt = bt
    return bt


def _down_linear(W):
    """All entries' A (rotated, fp32 [R, K]) as an int8 linear for the tensor-core GEMM, in two
    planes so that x_r A^T keeps ~16 bits: A ~= s (hi + lo / 254) per row, hi in rows [0, R) with
    scale s, lo in rows [R, 2R) with scale s / 254, zero rows up to a multiple of 128 (cached per
    attach). T = x_r A^T is then the sum of the two column halves of one GEMM's output."""
    from .weights import Linear

    lin = getattr(W, "_lora_down", None)
    if lin is None:
        A = _cat_A(W).float()
        R, K = A.shape
        s = A.abs().amax(1).clamp(min=1e-30) / 127.0
        a = A / s[:, None]
        hi = torch.round(a)
        lo = torch.round((a - hi) * 254.0)
        n2 = ((2 * R + 127) // 128) * 128
        q = torch.zeros(n2, K, dtype=torch.int8, device=A.device)
        q[:R] = hi.to(torch.int8)
        q[R:2 * R] = lo.to(torch.int8)
        sc = torch.ones(n2, dtype=torch.float32, device=A.device)
        sc[:R] = s
        sc[R:2 * R] = s / 254.0
        lin = Linear("i8", n2, K, q.contiguous(), sc.contiguous(), name=W.name + ".lora_down")
        W._lora_down = lin
    return lin


# How ops.linear applies the side paths: "delta" (default) computes the [M, N] update on the tensor
# cores (the down GEMM below, then T B^T as a two-plane fp16 GEMM) and hands it to the int8 GEMM's
# epilogue as its ADD input, the reference's own structure (ops.js:70-87); "fused" multiplies
# T B^T inside the int8 GEMM's epilogue on CUDA cores (anima_linear_opts.lora_*).
PATH = "delta"


def _up_linear(W):
    """scale_e * B_e of every entry as one fp16 [N, n2] weight over the down GEMM's n2 output
    columns: the entry's rank columns in both the hi half [0, R) and the lo half [R, 2R) of T (whose
    sum is x_r A^T), zero elsewhere (cached per attach)."""
    from .weights import Linear

    lin = getattr(W, "_lora_up", None)
    if lin is None:
        down = _down_linear(W)
        R = sum(e["r"] for e in W.lora)
        b2 = torch.zeros(W.N, down.N, dtype=torch.float32, device=W.lora[0]["B"].device)
        r0 = 0
        for e in W.lora:
            blk = e["B"].float() * e["scale"]
            b2[e["off"]:e["off"] + e["n"], r0:r0 + e["r"]] = blk
            b2[e["off"]:e["off"] + e["n"], R + r0:R + r0 + e["r"]] = blk
            r0 += e["r"]
        lin = Linear("f16", W.N, down.N, b2.half().contiguous(), None, name=W.name + ".lora_up")
        W._lora_up = lin
    return lin


# The down GEMM has few output tiles (ceil(M / 128) x n2 / 128: 32-64 at 1024^2) for the SMs. Where
# its K range is long (MLP layer 2: 8192) it is cut into up to four slices of at least 2048 that run
# as concurrent GEMMs on side streams; shorter slices would not pay for a launch's fixed cost
# (~7 us) and the extra sum. Each slice's partial T is its exact int32 sums times the same scales;
# the partials are added in a fixed order (deterministic), which changes T by fp32 rounding only.
_SIDE_STREAMS: dict = {}
_NUM_SMS: dict = {}


def _side_streams(device, n: int) -> list:
    ss = _SIDE_STREAMS.setdefault(device, [])
    while len(ss) < n:
        ss.append(torch.cuda.Stream(device))
    return ss[:n]


def k_slice_count(M: int, n_down: int, K: int, num_sms: int) -> int:
    """How many K slices the down GEMM ([M, K] x [n_down, K]^T) runs as: doubled while the slices'
    tiles still fit the SMs at once and each slice keeps at least 2048 of K (in 128-wide blocks)."""
    tiles = ((M + 127) // 128) * (n_down // 128)
    S = 1
    while S < 4 and tiles * 2 * S <= num_sms and K % (2 * S * 128) == 0 and K // (2 * S) >= 2048:
        S *= 2
    return S


def _k_slices(M: int, down, device) -> int:
    if device not in _NUM_SMS:
        _NUM_SMS[device] = torch.cuda.get_device_properties(device).multi_processor_count
    return k_slice_count(M, down.N, down.K, _NUM_SMS[device])


def _down_slices(W, S: int) -> list:
    """The down weight cut into S contiguous K slices (cached per attach)."""
    from .weights import Linear

    cache = getattr(W, "_lora_down_slices", None)
    if cache is None or len(cache) != S:
        down = _down_linear(W)
        k = down.K // S
        cache = [Linear("i8", down.N, k, down.data[:, i * k:(i + 1) * k].contiguous(), down.scale,
                        name=f"{down.name}.k{i}") for i in range(S)]
        W._lora_down_slices = cache
    return cache


def down_product(x, W) -> torch.Tensor:
    """T = x_r A^T for all of W's entries: fp32 [M, n2], hi-plane products in columns [0, R) and
    lo-plane products in [R, 2R) (see _down_linear)."""
    from .ops import QuantRows, lincomb, linear

    down = _down_linear(W)
    M = x.rows
    S = _k_slices(M, down, x.hi.device)
    if S == 1:
        return linear(x, down)
    k = down.K // S
    parts = _down_slices(W, S)
    outs = [torch.empty(M, down.N, dtype=torch.float32, device=x.hi.device) for _ in range(S)]
    cur = torch.cuda.current_stream(x.hi.device)
    side = _side_streams(x.hi.device, S - 1)
    for st in side:
        st.wait_stream(cur)
    for i in range(S):
        xs = QuantRows(x.hi[:, i * k:(i + 1) * k], x.lo[:, i * k:(i + 1) * k] if x.lo is not None else None, x.scale)
        if i == 0:
            linear(xs, parts[0], out=outs[0])
        else:
            with torch.cuda.stream(side[i - 1]):
                linear(xs, parts[i], out=outs[i])
    for st in side:
        cur.wait_stream(st)
    return lincomb(outs[0], *[(1.0, o) for o in outs])


def lora_delta_tc(x, W) -> torch.Tensor:
    """[M, N] fp32 low-rank update on the tensor cores: T = x_r A^T (hi and lo halves) by the int8
    GEMM, then T B2^T by the two-plane fp16 GEMM of anima_matmul (T to ~22 bits, scale * B in fp16:
    ~2^-11 of the update, as the fused epilogue)."""
    from .ops import matmul

    return matmul(down_product(x, W), _up_linear(W))


def lora_epilogue(x, W, opts) -> list:
    """Fill the LoRA fields of anima_linear_opts for the fused epilogue: T = x_r A^T of all entries
    (one int8 tensor-core GEMM, `_down_linear`), then the GEMM adds T B^T per entry before its
    activation. Returns the tensors that must stay alive until the GEMM is enqueued, or None when
    W's entries do not fit the fused form."""
    if not _fusable(W) or W.K % 128:
        return None
    A = _cat_A(W)
    R = A.shape[0]
    down = _down_linear(W)
    T = down_product(x, W)                   # [M, 2R (+ padding)]: hi and lo partial products
    bt = _cat_Bt(W)
    opts.lora_t, opts.ld_t, opts.lora_t_lo = T.data_ptr(), down.N, R
    opts.lora_bt, opts.ld_bt = bt.data_ptr(), W.N
    opts.lora_count = len(W.lora)
    r0 = 0
    for i, e in enumerate(W.lora):
        opts.lora_off[i], opts.lora_n[i], opts.lora_r0[i], opts.lora_r[i] = e["off"], e["n"], r0, e["r"]
        r0 += e["r"]
    return [T, bt]
