"""Chronos-2 on the B200 engine: the host side of ``ModelForward.forward`` over the C ABI.

Mirrors, in NumPy, the reference's host ends of a Chronos-2 forward pass:

* ``Chronos2Config`` — chronos2/Chronos2Config.java:45-192 (strict config.json keys)
* ``ModelInput``     — chronos2/ModelInput.java:28-37
* ``ModelLayout``    — chronos2/ModelLayout.java:72-181 (context cut and NaN padding, live keys)
* ``ModelPrep``      — chronos2/ModelPrep.java:37-138 (instance norm, patch tokens, inverse norm)
* ``B200Chronos2Forward.forward`` — chronos2/tornado/Chronos2Forward.java:148-176: the rows are
  regrouped so each group is contiguous, the encoder runs in ``libjitcast_b200.so``
  (``jc_forward_chronos2``), the outputs are put back in the caller's row order.

``random_checkpoint`` writes random-init weights with the reference checkpoint's tensor names and
shapes (Chronos2Weights.java:80-100).
"""

from __future__ import annotations

import ctypes
import json
import math
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import c_int, c_vp, check, precision_code
from .timestral import _TensorView

KEYS = {"architectures", "chronos_config", "chronos_pipeline_class", "d_ff", "d_kv", "d_model", "dense_act_fn",
        "dropout_rate", "feed_forward_proj", "initializer_factor", "is_gated_act", "layer_norm_epsilon", "model_type",
        "num_heads", "num_layers", "pad_token_id", "reg_token_id", "rope_theta", "torch_dtype", "dtype",
        "transformers_version", "use_cache", "vocab_size", "attn_implementation"}
CHRONOS_KEYS = {"context_length", "input_patch_size", "input_patch_stride", "output_patch_size",
                "max_output_patches", "quantiles", "use_reg_token", "use_arcsinh", "time_encoding_scale"}


@dataclass
class Chronos2Config:
    d_model: int
    d_kv: int
    d_ff: int
    num_layers: int
    num_heads: int
    quantiles: list[float]
    context_length: int = 2048
    patch_size: int = 16
    max_output_patches: int = 4
    layer_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    use_reg_token: bool = True
    use_arcsinh: bool = True
    time_encoding_scale: int | None = None

    def __post_init__(self):
        if self.time_encoding_scale is None:
            self.time_encoding_scale = self.context_length

    @property
    def inner(self) -> int:
        return self.num_heads * self.d_kv

    @property
    def num_quantiles(self) -> int:
        return len(self.quantiles)

    @property
    def vocab_size(self) -> int:
        return 2 if self.use_reg_token else 1

    def validate(self) -> "Chronos2Config":
        """Chronos2Config.validate (Chronos2Config.java:163-179)."""
        if min(self.d_model, self.d_kv, self.d_ff, self.num_layers, self.num_heads, self.patch_size,
               self.max_output_patches) < 1:
            raise ValueError("non-positive model dimensions")
        if self.d_kv % 2:
            raise ValueError(f"d_kv must be even for RoPE, got {self.d_kv}")
        if self.context_length < self.patch_size or self.time_encoding_scale < 1:
            raise ValueError("context_length must hold a patch")
        q = self.quantiles
        if any(not 0 < x < 1 for x in q) or any(not a < b for a, b in zip(q, q[1:])):
            raise ValueError("quantiles must be increasing and in (0, 1)")
        return self

    @staticmethod
    def from_json(doc: str | dict) -> "Chronos2Config":
        c = json.loads(doc) if isinstance(doc, str) else dict(doc)
        for k in c:
            if k not in KEYS:
                raise ValueError(f"unknown config key: {k}")
        cc = c.get("chronos_config")
        if cc is None:
            raise ValueError("not a Chronos-2 config: no chronos_config")
        for k in cc:
            if k not in CHRONOS_KEYS:
                raise ValueError(f"unknown config key: {k}")
        arch = c.get("architectures")
        if isinstance(arch, list) and "Chronos2Model" not in arch:
            raise ValueError(f"not a Chronos-2 checkpoint: {arch}")
        act = c.get("dense_act_fn", c.get("feed_forward_proj", "relu"))
        if act != "relu" or c.get("is_gated_act", False) or c.get("feed_forward_proj", "relu") != "relu":
            raise ValueError(f"only the ReLU feed-forward layer is supported, got {act}")
        dtype = c.get("torch_dtype", c.get("dtype", "float32"))
        if dtype != "float32":
            raise ValueError(f"only float32 checkpoints are supported, got {dtype}")
        p = int(cc.get("input_patch_size", 0))
        if p != int(cc.get("output_patch_size", 0)) or p != int(cc.get("input_patch_stride", 0)):
            raise ValueError("input and output patch sizes and the patch stride must be equal")
        ctx = int(cc.get("context_length", 0))
        return Chronos2Config(d_model=int(c.get("d_model", 512)), d_kv=int(c.get("d_kv", 64)),
                              d_ff=int(c.get("d_ff", 2048)), num_layers=int(c.get("num_layers", 6)),
                              num_heads=int(c.get("num_heads", 8)), quantiles=[float(x) for x in cc["quantiles"]],
                              context_length=ctx, patch_size=p,
                              max_output_patches=int(cc.get("max_output_patches", 1)),
                              layer_norm_eps=float(c.get("layer_norm_epsilon", 1e-6)),
                              rope_theta=float(c.get("rope_theta", 10000.0)),
                              use_reg_token=bool(cc.get("use_reg_token", False)),
                              use_arcsinh=bool(cc.get("use_arcsinh", False)),
                              time_encoding_scale=int(cc.get("time_encoding_scale", ctx))).validate()

    def to_json(self) -> dict:
        return {"architectures": ["Chronos2Model"], "d_model": self.d_model, "d_kv": self.d_kv, "d_ff": self.d_ff,
                "num_layers": self.num_layers, "num_heads": self.num_heads, "dense_act_fn": "relu",
                "feed_forward_proj": "relu", "is_gated_act": False, "layer_norm_epsilon": self.layer_norm_eps,
                "rope_theta": self.rope_theta, "torch_dtype": "float32",
                "chronos_config": {"context_length": self.context_length, "input_patch_size": self.patch_size,
                                   "input_patch_stride": self.patch_size, "output_patch_size": self.patch_size,
                                   "max_output_patches": self.max_output_patches, "quantiles": self.quantiles,
                                   "use_reg_token": self.use_reg_token, "use_arcsinh": self.use_arcsinh,
                                   "time_encoding_scale": self.time_encoding_scale}}


def default_quantiles() -> list[float]:
    """The 21 levels 0.01, 0.05, 0.1 … 0.9, 0.95, 0.99."""
    return [0.01] + [round(0.05 * i, 2) for i in range(1, 20)] + [0.99]


def config2() -> Chronos2Config:
    """d_model 768, 12 layers, 12 heads × d_kv 64, d_ff 3072 ReLU, patch 16,
    context 2048 (128 patches) + [REG] + 4 future patches, 21 quantiles."""
    return Chronos2Config(d_model=768, d_kv=64, d_ff=3072, num_layers=12, num_heads=12,
                          quantiles=default_quantiles(), context_length=2048, patch_size=16, max_output_patches=4,
                          use_reg_token=True, use_arcsinh=True).validate()


def weight_shapes(c: Chronos2Config) -> dict[str, tuple[int, ...]]:
    """Every checkpoint tensor and its shape (Chronos2Weights.load)."""
    d, inner, ff, p = c.d_model, c.inner, c.d_ff, c.patch_size
    s: dict[str, tuple[int, ...]] = {"shared.weight": (c.vocab_size, d)}

    def residual(prefix, i, h, o):
        for part, (a, b) in {"hidden_layer": (i, h), "output_layer": (h, o), "residual_layer": (i, o)}.items():
            s[f"{prefix}.{part}.weight"] = (b, a)
            s[f"{prefix}.{part}.bias"] = (b,)

    residual("input_patch_embedding", 3 * p, ff, d)
    for li in range(c.num_layers):
        pre = f"encoder.block.{li}.layer."
        for a in (0, 1):
            s[f"{pre}{a}.layer_norm.weight"] = (d,)
            for proj in "qkv":
                s[f"{pre}{a}.self_attention.{proj}.weight"] = (inner, d)
            s[f"{pre}{a}.self_attention.o.weight"] = (d, inner)
        s[f"{pre}2.layer_norm.weight"] = (d,)
        s[f"{pre}2.mlp.wi.weight"] = (ff, d)
        s[f"{pre}2.mlp.wo.weight"] = (d, ff)
    s["encoder.final_layer_norm.weight"] = (d,)
    residual("output_patch_embedding", d, ff, c.num_quantiles * p)
    return s


def random_checkpoint(c: Chronos2Config, seed: int = 0) -> dict[str, np.ndarray]:
    """Random-init weights: linear W ~ N(0, 1/in), biases ~ U(−0.1, 0.1), norm scales 1, the token
    table ([REG]) ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in sorted(weight_shapes(c).items()):
        if "layer_norm" in name:
            out[name] = np.ones(shape, np.float32)
        elif name.endswith(".bias"):
            out[name] = rng.uniform(-0.1, 0.1, shape).astype(np.float32)
        elif name == "shared.weight":
            out[name] = rng.standard_normal(shape, dtype=np.float32)
        else:
            out[name] = rng.standard_normal(shape, dtype=np.float32) / np.float32(math.sqrt(shape[1]))
    return out


@dataclass
class ModelInput:
    """``context`` [rows, T] with NaN where missing; ``group`` [rows]; optional future covariates."""

    context: np.ndarray
    group: np.ndarray
    output_patches: int
    future_covariates: np.ndarray | None = None

    @property
    def rows(self) -> int:
        return self.context.shape[0]


@dataclass
class ModelLayout:
    rows: int
    patch: int
    context_patches: int
    reg: int
    output_patches: int
    group: np.ndarray
    live: np.ndarray  # [rows, n] bool
    window: np.ndarray
    future: np.ndarray

    @property
    def tokens(self) -> int:
        return self.context_patches + self.reg + self.output_patches

    @property
    def future_start(self) -> int:
        return self.context_patches + self.reg

    @staticmethod
    def of(c: Chronos2Config, inp: ModelInput) -> "ModelLayout":
        ps = c.patch_size
        r = inp.rows
        h = inp.output_patches
        if h < 1:
            raise ValueError(f"output patches must be >= 1, got {h}")
        if len(inp.group) != r:
            raise ValueError("group ids must have one entry per row")
        t = inp.context.shape[1]
        kept = min(t, c.context_length)
        padded = (kept + ps - 1) // ps * ps
        nc = padded // ps
        window = np.full((r, padded), np.nan, np.float32)
        window[:, padded - kept:] = inp.context[:, t - kept:]
        future = np.full((r, h * ps), np.nan, np.float32)
        if inp.future_covariates is not None:
            f = np.asarray(inp.future_covariates, np.float32)
            if f.shape[1] > h * ps:
                raise ValueError(f"{h} output patches cannot hold {f.shape[1]} future steps")
            future[:, :f.shape[1]] = f
        reg = 1 if c.use_reg_token else 0
        live = np.ones((r, nc + reg + h), bool)
        live[:, :nc] = ~np.isnan(window).reshape(r, nc, ps).all(axis=2)
        return ModelLayout(r, ps, nc, reg, h, np.asarray(inp.group).copy(), live, window, future)


def _asinh32(v):
    a = np.abs(v.astype(np.float64))
    r = np.log(a + np.sqrt(a * a + 1.0))
    return np.where(v < 0, -r, r).astype(np.float32)


@dataclass
class ModelPrep:
    tokens: np.ndarray  # [rows, nc + h, 3P]
    loc: np.ndarray
    scale: np.ndarray

    @staticmethod
    def of(c: Chronos2Config, lay: ModelLayout) -> "ModelPrep":
        r, ps, nc, h = lay.rows, c.patch_size, lay.context_patches, lay.output_patches
        x = lay.window
        obs = ~np.isnan(x)
        n = obs.sum(axis=1)
        # sums in double in the reference's loop order (np.add.accumulate runs in order; np.sum pairs terms)
        s = np.add.accumulate(np.where(obs, x.astype(np.float64), 0.0), axis=1)[:, -1]
        loc = np.where(n > 0, (s / np.maximum(n, 1)).astype(np.float32), np.float32(0))
        d = np.where(obs, (x - loc[:, None]).astype(np.float32), np.float32(0)).astype(np.float64)
        sc = np.sqrt(np.add.accumulate(d * d, axis=1)[:, -1] / np.maximum(n, 1)).astype(np.float32)
        sc = np.where(sc == 0, np.float32(1e-5), sc)
        scale = np.where(n > 0, sc, np.float32(1)).astype(np.float32)
        loc = loc.astype(np.float32)

        def scaled(v):
            z = ((v - loc[:, None]) / scale[:, None]).astype(np.float32)
            return _asinh32(z) if c.use_arcsinh else z

        ts = np.float32(c.time_encoding_scale)
        tok = np.empty((r, nc + h, 3 * ps), np.float32)
        tt = np.arange(nc * ps)
        tok[:, :nc, :ps] = ((tt - nc * ps).astype(np.float32) / ts).reshape(nc, ps)[None]
        with np.errstate(invalid="ignore"):
            tok[:, :nc, ps:2 * ps] = np.where(obs, scaled(np.nan_to_num(x)), 0).reshape(r, nc, ps)
        tok[:, :nc, 2 * ps:] = obs.astype(np.float32).reshape(r, nc, ps)
        f = lay.future
        fobs = ~np.isnan(f)
        tf = np.arange(h * ps)
        tok[:, nc:, :ps] = (tf.astype(np.float32) / ts).reshape(h, ps)[None]
        with np.errstate(invalid="ignore"):
            tok[:, nc:, ps:2 * ps] = np.where(fobs, scaled(np.nan_to_num(f)), 0).reshape(r, h, ps)
        tok[:, nc:, 2 * ps:] = fobs.astype(np.float32).reshape(r, h, ps)
        return ModelPrep(tok, loc, scale)

    def finish(self, c: Chronos2Config, lay: ModelLayout, raw: np.ndarray) -> np.ndarray:
        """``sinh(x)·scale + loc`` per row: [rows, Q, h·P] (raw is [rows·h, Q·P], level-major)."""
        r, ps, q, h = lay.rows, c.patch_size, c.num_quantiles, lay.output_patches
        v = np.asarray(raw, np.float32).reshape(r, h, q, ps)
        if c.use_arcsinh:
            with np.errstate(over="ignore"):
                v = np.sinh(v.astype(np.float64)).astype(np.float32)
        out = (v * self.scale[:, None, None, None] + self.loc[:, None, None, None]).astype(np.float32)
        return out.transpose(0, 2, 1, 3).reshape(r, q, h * ps)


class _Desc(ctypes.Structure):
    _fields_ = [("d_model", c_int), ("d_kv", c_int), ("d_ff", c_int), ("num_layers", c_int), ("num_heads", c_int),
                ("patch_size", c_int), ("num_quantiles", c_int), ("use_reg_token", c_int),
                ("layer_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float)]


class Block(ctypes.Structure):
    """jc_chronos2_block."""

    _fields_ = [("rows", c_int), ("context_patches", c_int), ("output_patches", c_int), ("tokens", c_vp),
                ("live", c_vp), ("group_start", c_vp), ("group_end", c_vp)]


_lib.declare("jc_engine_create_chronos2", c_int, [ctypes.POINTER(_Desc), ctypes.POINTER(_TensorView), c_int,
                                                    ctypes.POINTER(c_int), c_int, c_int, ctypes.POINTER(c_vp)])
_lib.declare("jc_forward_chronos2", c_int, [c_vp, ctypes.POINTER(Block), c_vp])
_lib.declare("jc_forward_chronos2_device", c_int, [c_vp, c_int, ctypes.POINTER(Block), c_vp, c_vp])


class Window(ctypes.Structure):
    """jc_chronos2_window."""

    _fields_ = [("layout", Block), ("window", c_vp), ("future", c_vp), ("time_encoding_scale", ctypes.c_float),
                ("use_arcsinh", c_int)]


_lib.declare("jc_forecast_chronos2", c_int, [c_vp, ctypes.POINTER(Window), c_vp])
_lib.declare("jc_engine_profile", c_int, [c_vp, c_int, ctypes.POINTER(ctypes.c_char_p),
                                          ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong),
                                          ctypes.POINTER(ctypes.c_double), c_int, ctypes.POINTER(c_int)])
_lib.declare("jc_forecast_chronos2_device", c_int, [c_vp, c_int, ctypes.POINTER(Window), c_vp, c_vp])


def group_ranges(group: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    r = len(group)
    start = np.empty(r, np.int32)
    end = np.empty(r, np.int32)
    i = 0
    while i < r:
        e = i
        while e < r and group[e] == group[i]:
            e += 1
        start[i:e], end[i:e] = i, e
        i = e
    return start, end


class Chronos2Engine:
    """A Chronos-2 model resident on one or more GPUs (``jc_engine_create_chronos2``)."""

    def __init__(self, config: Chronos2Config, weights: dict[str, np.ndarray], devices=(0,), precision="fp16"):
        self.config = config
        keep = {k: np.ascontiguousarray(v, np.float32) for k, v in weights.items()}
        views = (_TensorView * len(keep))()
        names = []
        for i, (k, v) in enumerate(keep.items()):
            names.append(k.encode())
            views[i] = _TensorView(names[-1], v.ctypes.data, v.ndim,
                                   (ctypes.c_int64 * 4)(*(list(v.shape) + [0] * (4 - v.ndim))))
        desc = _Desc(config.d_model, config.d_kv, config.d_ff, config.num_layers, config.num_heads,
                     config.patch_size, config.num_quantiles, int(config.use_reg_token), config.layer_norm_eps,
                     config.rope_theta)
        devs = (c_int * len(devices))(*devices)
        h = c_vp()
        check(_lib.lib().jc_engine_create_chronos2(ctypes.byref(desc), views, len(keep), devs, len(devices),
                                                   precision_code(precision), ctypes.byref(h)))
        self._h = h

    @property
    def handle(self):
        if not self._h:
            raise RuntimeError("engine is closed")
        return self._h

    def forward_raw(self, lay: ModelLayout, prep: ModelPrep, group_start, group_end,
                    out: np.ndarray | None = None) -> np.ndarray:
        """raw [rows · h, Q · P] for a laid-out input, written into ``out`` when given (a C-contiguous float32 array
        of that shape, e.g. in pinned memory). Inputs already C-contiguous in the right dtype are used in place."""
        c = self.config
        tok = np.ascontiguousarray(prep.tokens, np.float32)
        live = np.ascontiguousarray(lay.live, np.int32)
        gs = np.ascontiguousarray(group_start, np.int32)
        ge = np.ascontiguousarray(group_end, np.int32)
        shape = (lay.rows * lay.output_patches, c.num_quantiles * c.patch_size)
        if out is None:
            out = np.empty(shape, np.float32)
        elif out.shape != shape or out.dtype != np.float32 or not out.flags.c_contiguous:
            raise ValueError(f"out must be a C-contiguous float32 array of shape {shape}")
        raw = out
        blk = Block(lay.rows, lay.context_patches, lay.output_patches, tok.ctypes.data, live.ctypes.data,
                    gs.ctypes.data, ge.ctypes.data)
        check(_lib.lib().jc_forward_chronos2(self.handle, ctypes.byref(blk), raw.ctypes.data))
        return raw

    def forecast(self, lay: ModelLayout, group_start, group_end, out: np.ndarray | None = None) -> np.ndarray:
        """ModelPrep.finish's quantiles [rows, Q, h · P] with ModelPrep.of and finish on the GPU
        (``jc_forecast_chronos2``): the window and future covariates cross instead of the tokens. Written into
        ``out`` when given (C-contiguous float32 of that shape); inputs already C-contiguous are used in place."""
        c = self.config
        win = np.ascontiguousarray(lay.window, np.float32)
        fut = np.ascontiguousarray(lay.future, np.float32)
        live = np.ascontiguousarray(lay.live, np.int32)
        gs = np.ascontiguousarray(group_start, np.int32)
        ge = np.ascontiguousarray(group_end, np.int32)
        shape = (lay.rows, c.num_quantiles, lay.output_patches * c.patch_size)
        if out is None:
            out = np.empty(shape, np.float32)
        elif out.shape != shape or out.dtype != np.float32 or not out.flags.c_contiguous:
            raise ValueError(f"out must be a C-contiguous float32 array of shape {shape}")
        blk = Block(lay.rows, lay.context_patches, lay.output_patches, None, live.ctypes.data, gs.ctypes.data,
                    ge.ctypes.data)
        w = Window(blk, win.ctypes.data, fut.ctypes.data, float(np.float32(c.time_encoding_scale)),
                   int(c.use_arcsinh))
        check(_lib.lib().jc_forecast_chronos2(self.handle, ctypes.byref(w), out.ctypes.data))
        return out

    def set_option(self, key: str, value: int) -> None:
        check(_lib.lib().jc_engine_set_option(self.handle, key.encode(), int(value)))

    def profile(self, slot: int = 0) -> dict[str, dict[str, float]]:
        """Per-stage totals since the last read (engine option ``profile``): ms, launches, flops."""
        cap = 32
        names = (ctypes.c_char_p * cap)()
        ms = (ctypes.c_double * cap)()
        launches = (ctypes.c_longlong * cap)()
        flops = (ctypes.c_double * cap)()
        n = c_int()
        check(_lib.lib().jc_engine_profile(self.handle, slot, names, ms, launches, flops, cap, ctypes.byref(n)))
        return {names[i].decode(): {"ms": ms[i], "launches": launches[i], "flops": flops[i]} for i in range(n.value)}

    def sync(self) -> None:
        check(_lib.lib().jc_engine_sync(self.handle))

    def close(self) -> None:
        if self._h:
            _lib.lib().jc_engine_destroy(self._h)
            self._h = c_vp()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class B200Chronos2Forward:
    """``ModelForward`` on the B200 engine (Chronos2Forward.forward, Chronos2Forward.java:148-176): ModelPrep's
    host ends on the GPU around the encoder (``jc_forecast_chronos2``), or with ``ends="host"`` on the host as
    the reference runs them (``jc_forward_chronos2``)."""

    def __init__(self, engine: Chronos2Engine, ends: str = "device"):
        if ends not in ("host", "device"):
            raise ValueError(f"ends must be 'host' or 'device', got {ends!r}")
        self.engine = engine
        self.config = engine.config
        self.ends = ends

    def forward(self, inp: ModelInput) -> np.ndarray:
        """[rows, Q, outputPatches · P] in each row's own scale."""
        # rows regrouped so each group is contiguous, stable within a group (Chronos2Forward.java:148-194)
        order = np.argsort(np.asarray(inp.group), kind="stable")
        inv = np.empty_like(order)
        inv[order] = np.arange(len(order))
        fut = None if inp.future_covariates is None else np.asarray(inp.future_covariates)[order]
        sorted_inp = ModelInput(np.asarray(inp.context)[order], np.asarray(inp.group)[order], inp.output_patches, fut)
        lay = ModelLayout.of(self.config, sorted_inp)
        gs, ge = group_ranges(lay.group)
        if self.ends == "device":
            return self.engine.forecast(lay, gs, ge)[inv]
        prep = ModelPrep.of(self.config, lay)
        raw = self.engine.forward_raw(lay, prep, gs, ge)
        return prep.finish(self.config, lay, raw)[inv]
