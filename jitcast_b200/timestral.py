"""Timestral on the B200 engine: the host side of ``BlockForward.predictBlock`` over the C ABI.

Mirrors, in NumPy, the reference's host ends of a decode block, which stay on the host in every
reference engine:

* ``TimestralConfig``  — timestral/TimestralConfig.java:53-244 (strict config.json keys)
* ``BlockInput``       — timestral/BlockInput.java:32-46
* ``BlockLayout``      — timestral/BlockLayout.java:77-243 (token layout, key validity, positions)
* ``BlockPrep``        — timestral/BlockPrep.java:40-101 and Scaler.java:36-148 (scaler, patch tokens,
                         monotone quantiles, denormalisation)
* ``B200TimestralForward.predict_block`` — timestral/tornado/TimestralForward.java:187-252: layout and
  prep on the host, the transformer in ``libjitcast_b200.so`` (``jc_forward_timestral``), finish on
  the host.

``random_checkpoint`` writes random-init weights with the reference checkpoint's tensor names and
shapes (TimestralWeights.java:83-115), the synthetic stand-in for a published checkpoint.
"""

from __future__ import annotations

import ctypes
import json
import math
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import _lib
from ._lib import c_int, c_vp, check, precision_code

TARGET, PAST, KNOWN = 0, 1, 2
LAYER_KINDS = {"time": 0, "variate": 1, "time_variate": 2, "variate_time": 3}
_AXES = {0: (True,), 1: (False,), 2: (True, False), 3: (False, True)}

CONFIG_KEYS = {"patch_size", "d_model", "num_heads", "mlp_hidden_dim", "block_schedule", "quantile_knots",
               "block_size", "context_length", "rope_theta", "rope_partial_factor", "norm_eps", "attn_bias",
               "mlp_bias", "time_attn_gate", "variate_attn_gate", "minimum_scale", "use_asinh",
               "stabilize_with_global", "covariate_enabled", "split_context_horizon_attn",
               "attend_missing_patches", "quantile_width_factor"}


@dataclass
class TimestralConfig:
    """The fields of a Timestral ``config.json`` that change the forward pass and decoding."""

    patch_size: int
    d_model: int
    num_heads: int
    mlp_hidden_dim: int
    block_schedule: list[str]
    quantile_knots: list[float]
    block_size: int = 16
    context_length: int = 4096
    rope_theta: float = 10000.0
    rope_partial_factor: float = 0.5
    norm_eps: float = 1e-6
    time_attn_gate: bool = True
    variate_attn_gate: bool = True
    minimum_scale: float = 1e-6
    use_asinh: bool = True
    covariate_enabled: bool = True
    attend_missing_patches: bool = True
    quantile_width_factor: float = 2.0

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads

    @property
    def rope_dim(self) -> int:
        return int(np.float32(self.head_dim) * np.float32(self.rope_partial_factor))

    @property
    def num_quantiles(self) -> int:
        return len(self.quantile_knots)

    @property
    def median_index(self) -> int:
        for i, q in enumerate(self.quantile_knots):
            if q == 0.5:
                return i
        raise ValueError("no 0.5 quantile knot")

    def attention_axes(self) -> list[tuple[bool, ...]]:
        return [_AXES[LAYER_KINDS[k]] for k in self.block_schedule]

    def validate(self) -> "TimestralConfig":
        """TimestralConfig.validate (TimestralConfig.java:211-227)."""
        if self.patch_size < 1 or self.d_model < 1 or self.num_heads < 1 or self.d_model % self.num_heads:
            raise ValueError(f"d_model {self.d_model} is not divisible by num_heads {self.num_heads}")
        if self.rope_dim <= 0 or self.rope_dim % 2:
            raise ValueError(f"rope_partial_factor {self.rope_partial_factor} gives rope_dim {self.rope_dim}")
        for k in self.block_schedule:
            if k not in LAYER_KINDS:
                raise ValueError(f"unknown layer kind {k}")
        if any(not a < b for a, b in zip(self.quantile_knots, self.quantile_knots[1:])):
            raise ValueError("quantile_knots must be increasing")
        self.median_index
        if self.context_length % self.patch_size:
            raise ValueError("context_length must be a multiple of patch_size")
        return self

    @staticmethod
    def from_json(doc: str | dict) -> "TimestralConfig":
        """TimestralConfig.fromJson: unknown keys and unsupported settings fail."""
        c = json.loads(doc) if isinstance(doc, str) else dict(doc)
        for key in c:
            if key not in CONFIG_KEYS:
                raise ValueError(f"unknown config key: {key}")
        for key in ("attn_bias", "mlp_bias", "stabilize_with_global"):
            if c.get(key, False):
                raise ValueError(f"{key} = true is not supported")

        def gate(key):
            g = c.get(key, "sdpa_sigmoid")
            if g not in ("sdpa_sigmoid", "none"):
                raise ValueError(f"unknown attention gate {g}")
            return g == "sdpa_sigmoid"

        return TimestralConfig(
            patch_size=int(c["patch_size"]), d_model=int(c["d_model"]), num_heads=int(c["num_heads"]),
            mlp_hidden_dim=int(c["mlp_hidden_dim"]), block_schedule=list(c["block_schedule"]),
            quantile_knots=[float(q) for q in c["quantile_knots"]], block_size=int(c.get("block_size", 0)),
            context_length=int(c.get("context_length", 0)), rope_theta=float(c.get("rope_theta", 10000.0)),
            rope_partial_factor=float(c.get("rope_partial_factor", 0.5)), norm_eps=float(c.get("norm_eps", 1e-6)),
            time_attn_gate=gate("time_attn_gate"), variate_attn_gate=gate("variate_attn_gate"),
            minimum_scale=float(c.get("minimum_scale", 1e-6)), use_asinh=bool(c.get("use_asinh", True)),
            covariate_enabled=bool(c.get("covariate_enabled", True)),
            attend_missing_patches=bool(c.get("attend_missing_patches", True)),
            quantile_width_factor=float(c.get("quantile_width_factor", 2.0))).validate()

    def to_json(self) -> dict:
        return {"patch_size": self.patch_size, "d_model": self.d_model, "num_heads": self.num_heads,
                "mlp_hidden_dim": self.mlp_hidden_dim, "block_schedule": self.block_schedule,
                "quantile_knots": self.quantile_knots, "block_size": self.block_size,
                "context_length": self.context_length, "rope_theta": self.rope_theta,
                "rope_partial_factor": self.rope_partial_factor, "norm_eps": self.norm_eps,
                "time_attn_gate": "sdpa_sigmoid" if self.time_attn_gate else "none",
                "variate_attn_gate": "sdpa_sigmoid" if self.variate_attn_gate else "none",
                "minimum_scale": self.minimum_scale, "use_asinh": self.use_asinh,
                "covariate_enabled": self.covariate_enabled, "attend_missing_patches": self.attend_missing_patches,
                "quantile_width_factor": self.quantile_width_factor}


def default_knots(q: int = 21) -> list[float]:
    """0.01, 0.05 … 0.95, 0.99 for 21 levels (always contains 0.5)."""
    if q == 21:
        return [0.01] + [round(0.05 * i, 2) for i in range(1, 20)] + [0.99]
    if q == 9:
        return [round(0.1 * i, 1) for i in range(1, 10)]
    return [float(x) for x in np.linspace(0, 1, q + 2)[1:-1]]


def config3() -> TimestralConfig:
    """d 1024, 16 layers, 16 heads, SwiGLU 4096, RoPE (partial 0.5, θ 1e4),
    patch 32, context 4096 (128 tokens), 21 quantiles, every layer time attention with the gate."""
    return TimestralConfig(patch_size=32, d_model=1024, num_heads=16, mlp_hidden_dim=4096,
                           block_schedule=["time"] * 16, quantile_knots=default_knots(21), block_size=16,
                           context_length=4096).validate()


def weight_shapes(c: TimestralConfig) -> dict[str, tuple[int, ...]]:
    """Every checkpoint tensor and its shape (TimestralWeights.load, TimestralWeights.java:83-115)."""
    d, p, f, q = c.d_model, c.patch_size, c.mlp_hidden_dim, c.num_quantiles
    s: dict[str, tuple[int, ...]] = {}
    for part, (i, o) in {"hidden_layer": (2 * p, 4 * d), "output_layer": (4 * d, d),
                         "residual_layer": (2 * p, d)}.items():
        s[f"representation.patch_proj.{part}.weight"] = (o, i)
        s[f"representation.patch_proj.{part}.bias"] = (o,)
    s["representation.forecast_query"] = (d,)
    for li, axes in enumerate(c.attention_axes()):
        pre = f"transformer.layers.{li}"
        for a, is_time in enumerate(axes):
            s[f"{pre}.attn_norms.{a}.scale"] = (d,)
            s[f"{pre}.attns.{a}.wQKV.weight"] = (3 * d, d)
            if c.time_attn_gate if is_time else c.variate_attn_gate:
                s[f"{pre}.attns.{a}._gate.weight"] = (d, d)
            s[f"{pre}.attns.{a}.wO.weight"] = (d, d)
        s[f"{pre}.mlp_norm.scale"] = (d,)
        s[f"{pre}.mlp.w12.weight"] = (2 * f, d)
        s[f"{pre}.mlp.w3.weight"] = (d, f)
    s["transformer.out_norm.scale"] = (d,)
    for part, (i, o) in {"hidden_layer": (d, 4 * d), "output_layer": (4 * d, p * q),
                         "residual_layer": (d, p * q)}.items():
        s[f"head.projection.{part}.weight"] = (o, i)
    return s


def random_checkpoint(c: TimestralConfig, seed: int = 0) -> dict[str, np.ndarray]:
    """Random-init weights: linear W ~ N(0, 1/in), biases ~ U(−0.1, 0.1), norm scales 1, the
    forecast query ~ N(0, 1); one seeded generator, tensors drawn in name order."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in sorted(weight_shapes(c).items()):
        if name.endswith(".scale"):
            out[name] = np.ones(shape, np.float32)
        elif name.endswith(".bias"):
            out[name] = rng.uniform(-0.1, 0.1, shape).astype(np.float32)
        elif name == "representation.forecast_query":
            out[name] = rng.standard_normal(shape, dtype=np.float32)
        else:
            out[name] = (rng.standard_normal(shape, dtype=np.float32) / np.float32(math.sqrt(shape[1])))
    return out


def save_checkpoint(directory: str | Path, c: TimestralConfig, weights: dict[str, np.ndarray]) -> Path:
    """Writes ``config.json`` and ``model.safetensors`` (F32 tensors) as the reference loads them."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    (d / "config.json").write_text(json.dumps(c.to_json(), indent=1))
    header, blobs, off = {}, [], 0
    for name in sorted(weights):
        a = np.ascontiguousarray(weights[name], np.float32)
        header[name] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(d / "model.safetensors", "wb") as fh:
        fh.write(len(h).to_bytes(8, "little"))
        fh.write(h)
        for b in blobs:
            fh.write(b)
    return d


def load_checkpoint(directory: str | Path) -> tuple[TimestralConfig, dict[str, np.ndarray]]:
    d = Path(directory)
    c = TimestralConfig.from_json((d / "config.json").read_text())
    raw = (d / "model.safetensors").read_bytes()
    n = int.from_bytes(raw[:8], "little")
    header = json.loads(raw[8:8 + n])
    base = 8 + n
    w = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        if meta["dtype"] != "F32":
            raise ValueError(f"{name}: expected F32, got {meta['dtype']}")
        s, e = meta["data_offsets"]
        w[name] = np.frombuffer(raw, np.float32, (e - s) // 4, base + s).reshape(meta["shape"])
    return c, w


# ---- host ends of a decode block -------------------------------------------------------------------

@dataclass
class BlockInput:
    """One decode block: ``inputs``/``observed`` [rows, length], ``group`` [rows]."""

    inputs: np.ndarray
    observed: np.ndarray
    group: np.ndarray
    horizon_patches: int
    role: np.ndarray | None = None
    known_future: np.ndarray | None = None
    known_future_mask: np.ndarray | None = None

    @property
    def rows(self) -> int:
        return self.inputs.shape[0]


@dataclass
class BlockLayout:
    rows: int
    patch: int
    context_patches: int
    encoder: int
    horizon: int
    covariates: bool
    group: np.ndarray
    role: np.ndarray
    key_valid: np.ndarray  # [rows, enc] bool
    first: np.ndarray
    window: np.ndarray
    observed: np.ndarray

    @property
    def tokens(self) -> int:
        return self.encoder + self.horizon

    @property
    def known(self) -> np.ndarray:
        return (self.role == KNOWN) & self.covariates

    def positions(self) -> np.ndarray:
        """BlockLayout.position for every (row, token): [rows, enc + h]."""
        tok = np.arange(self.tokens)
        p = np.where(tok < self.encoder, tok, self.context_patches + tok - self.encoder)
        return (p[None, :] - self.first[:, None]).astype(np.int32)

    @staticmethod
    def of(c: TimestralConfig, b: BlockInput) -> "BlockLayout":
        ps = c.patch_size
        r, t = b.inputs.shape
        if t % ps:
            raise ValueError(f"context length {t} is not a multiple of the patch size {ps}")
        h = b.horizon_patches
        if h < 1:
            raise ValueError(f"horizon patches must be >= 1, got {h}")
        cov = bool(b.role is not None and c.covariate_enabled and np.any(np.asarray(b.role) != TARGET))
        ll = t // ps
        window = np.asarray(b.inputs, np.float32)
        obs = np.asarray(b.observed, bool)
        role = np.zeros(r, np.int32)
        if cov:
            if h > c.block_size:
                raise ValueError(f"a block with covariates decodes at most {c.block_size} patches, got {h}")
            role = np.asarray(b.role, np.int32).copy()
            w2 = np.zeros((r, t + h * ps), np.float32)
            o2 = np.zeros((r, t + h * ps), bool)
            w2[:, :t], o2[:, :t] = window, obs
            if b.known_future is not None:
                w2[:, t:] = b.known_future
                o2[:, t:] = b.known_future_mask
            window, obs = w2, o2
        enc = window.shape[1] // ps
        patch_obs = obs.reshape(r, enc, ps).any(axis=2)
        valid = np.logical_or.accumulate(patch_obs, axis=1) if c.attend_missing_patches else patch_obs
        first_row = np.where(patch_obs.any(axis=1), patch_obs.argmax(axis=1), enc)
        group = np.asarray(b.group)
        # each series' first observed patch over all its rows (0 for a series with none), in one pass
        _, inv = np.unique(group, return_inverse=True)
        gmin = np.full(int(inv.max()) + 1 if r else 0, enc, np.int64)
        np.minimum.at(gmin, inv, first_row)
        first = gmin[inv]
        first[first == enc] = 0
        return BlockLayout(r, ps, ll, enc, h, cov, group, role, valid, first, window, obs)

    def group_ranges(self) -> tuple[np.ndarray, np.ndarray]:
        """groupStart / groupEnd per row; rows of a series must be contiguous (TimestralForward.java:610-625)."""
        g = self.group
        r = self.rows
        start = np.empty(r, np.int32)
        end = np.empty(r, np.int32)
        seen = set()
        i = 0
        while i < r:
            if int(g[i]) in seen:
                raise ValueError(f"rows of series {int(g[i])} are not contiguous")
            seen.add(int(g[i]))
            e = i
            while e < r and g[e] == g[i]:
                e += 1
            start[i:e], end[i:e] = i, e
            i = e
        return start, end


_EPS32 = np.float32(np.finfo(np.float32).eps)


def _asinh32(v: np.ndarray) -> np.ndarray:
    a = np.abs(v.astype(np.float64))
    r = np.log(a + np.sqrt(a * a + 1.0))
    return np.where(v < 0, -r, r).astype(np.float32)


def causal_patch_loc_scale(x: np.ndarray, obs: np.ndarray, patch: int, min_scale: float):
    """Scaler.causalPatchLocScale for every row at once (Welford, in double, in the reference's order)."""
    rows, t = x.shape
    loc = np.empty((rows, t), np.float32)
    scale = np.empty((rows, t), np.float32)
    cum_w = np.zeros(rows)
    cum_x = np.zeros(rows)
    m2 = np.zeros(rows)
    prev = np.zeros(rows)
    xd = x.astype(np.float64)
    wd = obs.astype(np.float64)
    for i in range(t):
        w = wd[:, i]
        xi = xd[:, i]
        cum_w += w
        cum_x += w * xi
        mean = cum_x / np.maximum(cum_w, 1.0)
        m2 += (xi - prev) * (xi - mean) * w
        prev = mean
        if i % patch == patch - 1:
            var = m2 / np.maximum(np.maximum(cum_w, 1.0) - 1.0, 1.0)
            loc[:, i - patch + 1:i + 1] = mean.astype(np.float32)[:, None]
            scale[:, i - patch + 1:i + 1] = np.maximum(np.sqrt(var), float(np.float32(min_scale))).astype(
                np.float32)[:, None]
    return loc, scale


def instance_norm(x: np.ndarray, obs: np.ndarray, min_scale: float) -> tuple[float, float, bool]:
    """Scaler.instanceNorm for one known-covariate row: (loc, scale, binary)."""
    n = max(float(obs.sum()), 1.0)
    xo = x[obs].astype(np.float64)
    s = float(np.add.accumulate(xo)[-1]) if xo.size else 0.0  # in the reference's loop order
    loc = np.float32(s / n)
    d = np.where(obs, x - loc, np.float32(0)).astype(np.float64)
    ss = float(np.add.accumulate(d * d)[-1]) if d.size else 0.0
    with np.errstate(over="ignore"):  # a float overflow gives inf, as the reference's (float) cast does
        scale = max(np.float32(math.sqrt(np.float32(ss / n))), np.float32(min_scale))
    zero_one = bool(np.all((x == 0) | (x == 1) | ~obs))
    if zero_one and obs.any():
        return np.float32(0), np.float32(1), True
    return loc, np.float32(scale), False


@dataclass
class BlockPrep:
    tokens: np.ndarray  # [rows, enc, 2P]
    loc: np.ndarray     # [rows, window]
    scale: np.ndarray

    @staticmethod
    def of(c: TimestralConfig, lay: BlockLayout) -> "BlockPrep":
        ps, enc = c.patch_size, lay.encoder
        win, obs = lay.window, lay.observed
        loc, scale = causal_patch_loc_scale(win, obs, ps, c.minimum_scale)
        use = np.full(lay.rows, c.use_asinh)
        for i in np.nonzero(lay.known)[0]:
            l, s, binary = instance_norm(win[i], obs[i], c.minimum_scale)
            loc[i], scale[i] = l, s
            use[i] = c.use_asinh and not binary
        v = (win - loc) / np.maximum(scale, _EPS32)
        v = np.where(use[:, None], _asinh32(v), v)
        scaled = np.where(obs, v, np.float32(0)).astype(np.float32)
        tok = np.empty((lay.rows, enc, 2 * ps), np.float32)
        tok[:, :, :ps] = scaled.reshape(lay.rows, enc, ps)
        tok[:, :, ps:] = np.where(obs, np.float32(0), np.float32(1)).reshape(lay.rows, enc, ps)
        return BlockPrep(tok, loc, scale)

    def finish(self, c: TimestralConfig, lay: BlockLayout, raw: np.ndarray) -> np.ndarray:
        """Monotone quantiles, then denormalisation with the last context patch's frame and
        clamping of infinities: [rows, h·P, Q]."""
        q = c.num_quantiles
        ps, h = c.patch_size, lay.horizon
        v = monotone_quantiles(c, np.asarray(raw, np.float32).reshape(lay.rows, h * ps, q))
        anchor = (lay.context_patches - 1) * ps
        loc = self.loc[:, anchor][:, None, None]
        scale = self.scale[:, anchor][:, None, None]
        with np.errstate(over="ignore", invalid="ignore"):
            s = np.sinh(v.astype(np.float64)).astype(np.float32) if c.use_asinh else v
            out = (s * scale + loc).astype(np.float32)
        return clamp_nonfinite(out)


def quantile_scale(c: TimestralConfig) -> np.ndarray:
    """Quantiles' width_factor · Δp per level, rounded as the reference rounds them."""
    lv = c.quantile_knots
    m = c.median_index
    s = np.zeros(len(lv), np.float32)
    for i in range(len(lv)):
        s[i] = np.float32(lv[i] - lv[i - 1] if i > m else lv[i + 1] - lv[i] if i < m else 0.0)
    return (np.float32(c.quantile_width_factor) * s).astype(np.float32)


def _softplus32(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return np.where(x > 20, x, np.log1p(np.exp(x.astype(np.float64))).astype(np.float32)).astype(np.float32)


def monotone_quantiles(c: TimestralConfig, raw: np.ndarray) -> np.ndarray:
    """Quantiles.apply on the last axis (Quantiles.java:52-70)."""
    sc = quantile_scale(c)
    m = c.median_index
    out = raw.astype(np.float32).copy()
    mid = raw[..., m].astype(np.float32)
    fmax = np.float32(np.finfo(np.float32).max)
    up = np.zeros_like(mid)
    for i in range(m + 1, raw.shape[-1]):
        up = (up + sc[i] * _softplus32(raw[..., i])).astype(np.float32)
        out[..., i] = np.clip(mid + up, -fmax, fmax)
    down = np.zeros_like(mid)
    for i in range(m - 1, -1, -1):
        down = (down + sc[i] * _softplus32(raw[..., i])).astype(np.float32)
        out[..., i] = np.clip(mid - down, -fmax, fmax)
    out[..., m] = np.clip(mid, -fmax, fmax)
    return out


def clamp_nonfinite(v: np.ndarray) -> np.ndarray:
    """Scaler.clampNonFinite along the last axis."""
    fin = np.isfinite(v)
    big = np.where(fin, v, -np.inf).max(axis=-1, keepdims=True)
    small = np.where(fin, v, np.inf).min(axis=-1, keepdims=True)
    x = np.where(v == np.inf, big, np.where(v == -np.inf, small, v))
    return np.where(np.isinf(x), np.float32(0), x).astype(np.float32)


# ---- the engine ---------------------------------------------------------------------------------------

class _TensorView(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", c_vp), ("ndim", c_int), ("shape", ctypes.c_int64 * 4)]


class _Desc(ctypes.Structure):
    _fields_ = [("patch_size", c_int), ("d_model", c_int), ("num_heads", c_int), ("mlp_hidden_dim", c_int),
                ("num_layers", c_int), ("layer_kinds", ctypes.POINTER(ctypes.c_int32)), ("num_quantiles", c_int),
                ("rope_theta", ctypes.c_float), ("rope_partial_factor", ctypes.c_float),
                ("norm_eps", ctypes.c_float), ("time_attn_gate", c_int), ("variate_attn_gate", c_int)]


class Block(ctypes.Structure):
    """jc_timestral_block."""

    _fields_ = [("rows", c_int), ("encoder", c_int), ("horizon", c_int), ("context_patches", c_int),
                ("covariates", c_int), ("tokens", c_vp), ("positions", c_vp), ("key_valid", c_vp),
                ("known", c_vp), ("role", c_vp), ("group_start", c_vp), ("group_end", c_vp)]


_lib.declare("jc_engine_create_timestral", c_int, [ctypes.POINTER(_Desc), ctypes.POINTER(_TensorView), c_int,
                                                     ctypes.POINTER(c_int), c_int, c_int, ctypes.POINTER(c_vp)])
_lib.declare("jc_forward_timestral", c_int, [c_vp, ctypes.POINTER(Block), c_vp])
_lib.declare("jc_forward_timestral_device", c_int, [c_vp, c_int, ctypes.POINTER(Block), c_vp, c_vp])
_lib.declare("jc_forecast_timestral", c_int, [c_vp, c_vp, c_vp])
_lib.declare("jc_forecast_timestral_device", c_int, [c_vp, c_int, c_vp, c_vp, c_vp])
_lib.declare("jc_engine_sync", c_int, [c_vp])
_lib.declare("jc_engine_set_option", c_int, [c_vp, ctypes.c_char_p, ctypes.c_longlong])
_lib.declare("jc_engine_profile", c_int, [c_vp, c_int, ctypes.POINTER(ctypes.c_char_p),
                                          ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong),
                                          ctypes.POINTER(ctypes.c_double), c_int, ctypes.POINTER(c_int)])
_lib.declare("jc_engine_destroy", c_int, [c_vp])


@dataclass
class DeviceInputs:
    """A block's device-forward inputs as host arrays (what jc_timestral_block points at)."""

    rows: int
    encoder: int
    horizon: int
    context_patches: int
    covariates: int
    tokens: np.ndarray | None  # None for WindowInputs, whose tokens the GPU assembles
    positions: np.ndarray
    key_valid: np.ndarray
    known: np.ndarray
    role: np.ndarray
    group_start: np.ndarray
    group_end: np.ndarray
    _keep: list = field(default_factory=list)

    @staticmethod
    def of(lay: BlockLayout, prep: BlockPrep) -> "DeviceInputs":
        gs, ge = lay.group_ranges()
        i32 = lambda a: np.ascontiguousarray(a, np.int32)  # noqa: E731
        return DeviceInputs(lay.rows, lay.encoder, lay.horizon, lay.context_patches, int(lay.covariates),
                            np.ascontiguousarray(prep.tokens, np.float32), i32(lay.positions()),
                            i32(lay.key_valid), i32(lay.known), i32(lay.role), gs, ge)

    def struct(self) -> Block:
        return Block(self.rows, self.encoder, self.horizon, self.context_patches, self.covariates,
                     None if self.tokens is None else self.tokens.ctypes.data, self.positions.ctypes.data, self.key_valid.ctypes.data,
                     self.known.ctypes.data, self.role.ctypes.data, self.group_start.ctypes.data,
                     self.group_end.ctypes.data)


class Window(ctypes.Structure):
    """jc_timestral_window."""

    _fields_ = [("layout", Block), ("window", c_vp), ("observed", c_vp), ("minimum_scale", ctypes.c_float),
                ("use_asinh", c_int), ("median", c_int), ("quantile_scale", c_vp)]


@dataclass
class WindowInputs:
    """A block's inputs for the forward with BlockPrep's host ends on the GPU (what jc_timestral_window points
    at): the layout without tokens, and the raw window with its observed flags."""

    layout: DeviceInputs
    window: np.ndarray    # [rows, encoder · P] float32, BlockLayout.window
    observed: np.ndarray  # [rows, encoder · P] uint8, BlockLayout.observed
    minimum_scale: float
    use_asinh: int
    median: int
    quantile_scale: np.ndarray  # [Q] float32, Quantiles.scale()

    @staticmethod
    def of(c: TimestralConfig, lay: BlockLayout) -> "WindowInputs":
        gs, ge = lay.group_ranges()
        i32 = lambda a: np.ascontiguousarray(a, np.int32)  # noqa: E731
        layout = DeviceInputs(lay.rows, lay.encoder, lay.horizon, lay.context_patches, int(lay.covariates), None,
                              i32(lay.positions()), i32(lay.key_valid), i32(lay.known), i32(lay.role), gs, ge)
        return WindowInputs(layout, np.ascontiguousarray(lay.window, np.float32),
                            np.ascontiguousarray(lay.observed, np.uint8), float(np.float32(c.minimum_scale)),
                            int(c.use_asinh), c.median_index, np.ascontiguousarray(quantile_scale(c), np.float32))

    def struct(self) -> Window:
        return Window(self.layout.struct(), self.window.ctypes.data, self.observed.ctypes.data, self.minimum_scale,
                      self.use_asinh, self.median, self.quantile_scale.ctypes.data)


class DeviceWindow:
    """A block's window inputs resident in one GPU's memory (torch tensors), with the ``jc_timestral_window`` that
    points at them: what ``jc_forecast_timestral_device`` reads, for a caller whose inputs are already in HBM."""

    FIELDS = ("positions", "key_valid", "known", "role", "group_start", "group_end")

    def __init__(self, wi: WindowInputs, device):
        import torch

        up = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
        lay = wi.layout
        self.inputs = wi  # keeps quantile_scale (a host array the call reads) alive
        self.tensors = {k: up(getattr(lay, k)) for k in self.FIELDS}
        self.tensors["window"], self.tensors["observed"] = up(wi.window), up(wi.observed)
        blk = Block(lay.rows, lay.encoder, lay.horizon, lay.context_patches, lay.covariates, None,
                    *(self.tensors[k].data_ptr() for k in self.FIELDS))
        self.struct = Window(blk, self.tensors["window"].data_ptr(), self.tensors["observed"].data_ptr(),
                             wi.minimum_scale, wi.use_asinh, wi.median, wi.quantile_scale.ctypes.data)

    def out_shape(self, c: TimestralConfig) -> tuple[int, int, int]:
        lay = self.inputs.layout
        return (lay.rows, lay.horizon * c.patch_size, c.num_quantiles)

    def forecast(self, engine: "TimestralEngine", out, stream, slot: int = 0) -> None:
        """Enqueues ``jc_forecast_timestral_device`` on ``stream`` (a torch stream) into ``out`` (a float32 CUDA
        tensor of ``out_shape``)."""
        check(_lib.lib().jc_forecast_timestral_device(engine.handle, slot, ctypes.byref(self.struct), out.data_ptr(),
                                                      c_vp(stream.cuda_stream)))


class TimestralEngine:
    """A Timestral model resident on one or more GPUs (``jc_engine_create_timestral``)."""

    def __init__(self, config: TimestralConfig, weights: dict[str, np.ndarray], devices=(0,), precision="bf16"):
        self.config = config
        self.precision = precision
        keep = {k: np.ascontiguousarray(v, np.float32) for k, v in weights.items()}
        views = (_TensorView * len(keep))()
        names = []
        for i, (k, v) in enumerate(keep.items()):
            names.append(k.encode())
            shape = (ctypes.c_int64 * 4)(*(list(v.shape) + [0] * (4 - v.ndim)))
            views[i] = _TensorView(names[-1], v.ctypes.data, v.ndim, shape)
        kinds = (ctypes.c_int32 * len(config.block_schedule))(*[LAYER_KINDS[k] for k in config.block_schedule])
        desc = _Desc(config.patch_size, config.d_model, config.num_heads, config.mlp_hidden_dim,
                     len(config.block_schedule), kinds, config.num_quantiles, config.rope_theta,
                     config.rope_partial_factor, config.norm_eps, int(config.time_attn_gate),
                     int(config.variate_attn_gate))
        devs = (c_int * len(devices))(*devices)
        handle = c_vp()
        check(_lib.lib().jc_engine_create_timestral(ctypes.byref(desc), views, len(keep), devs, len(devices),
                                                    precision_code(precision), ctypes.byref(handle)))
        self._h = handle
        self.devices = tuple(devices)

    @property
    def handle(self):
        if not self._h:
            raise RuntimeError("engine is closed")
        return self._h

    def forward(self, inp: DeviceInputs, out: np.ndarray | None = None) -> np.ndarray:
        """raw [rows · h, P · Q] for a block's device inputs (host buffers), written into ``out`` when given (a
        C-contiguous float32 array of that shape, e.g. in pinned memory)."""
        c = self.config
        shape = (inp.rows * inp.horizon, c.patch_size * c.num_quantiles)
        if out is None:
            out = np.empty(shape, np.float32)
        elif out.shape != shape or out.dtype != np.float32 or not out.flags.c_contiguous:
            raise ValueError(f"out must be a C-contiguous float32 array of shape {shape}")
        blk = inp.struct()
        check(_lib.lib().jc_forward_timestral(self.handle, ctypes.byref(blk), out.ctypes.data))
        return out

    def forecast(self, inp: WindowInputs, out: np.ndarray | None = None) -> np.ndarray:
        """BlockPrep.finish's quantiles [rows, h · P, Q] with the scaler, the tokens and the finish on the GPU
        (``jc_forecast_timestral``), written into ``out`` when given (C-contiguous float32 of that shape)."""
        c = self.config
        shape = (inp.layout.rows, inp.layout.horizon * c.patch_size, c.num_quantiles)
        if out is None:
            out = np.empty(shape, np.float32)
        elif out.shape != shape or out.dtype != np.float32 or not out.flags.c_contiguous:
            raise ValueError(f"out must be a C-contiguous float32 array of shape {shape}")
        blk = inp.struct()
        check(_lib.lib().jc_forecast_timestral(self.handle, ctypes.byref(blk), out.ctypes.data))
        return out

    def set_option(self, key: str, value: int) -> None:
        check(_lib.lib().jc_engine_set_option(self.handle, key.encode(), int(value)))

    def profile(self, slot: int = 0) -> dict[str, dict[str, float]]:
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


def bucket(x: int) -> int:
    """TimestralForward.bucket (TimestralForward.java:93-99): x itself up to 8, then the next multiple of a quarter
    of its power of two, so padding adds at most 25 % and the number of shapes grows with log(x)."""
    if x <= 8:
        return x
    step = (1 << ((x - 1).bit_length() - 1)) // 4
    return (x + step - 1) // step * step


def bucketed_context(block: BlockInput, patch: int) -> BlockInput:
    """The context half of TimestralForward.bucketed (TimestralForward.java:197-231): the window padded in front
    with empty (unobserved, zero) patches up to ``bucket(patches)``. An empty patch is never a valid key and time
    positions count from each series' first observation, so the forecasts do not change; the rows half of the
    bucketing happens inside the engine (its plans are built for bucketed row counts)."""
    r, t = block.inputs.shape
    if t % patch:
        return block  # BlockLayout.of rejects it
    patches = t // patch
    padded = bucket(patches)
    if padded == patches:
        return block
    lead = (padded - patches) * patch
    inputs = np.zeros((r, padded * patch), np.float32)
    observed = np.zeros((r, padded * patch), bool)
    inputs[:, lead:] = block.inputs
    observed[:, lead:] = block.observed
    return BlockInput(inputs, observed, block.group, block.horizon_patches, block.role, block.known_future,
                      block.known_future_mask)


class B200TimestralForward:
    """``BlockForward`` on the B200 engine: the layout on the host, the transformer on the GPUs, and
    BlockPrep's scaler and finish on the GPU around the forward (``jc_forecast_timestral``: the window crosses
    instead of the tokens, the quantiles come back finished; the NumPy host prep of a 8,192-series config-5
    chunk alone takes seconds), or with ``ends="host"`` on the host as the reference runs them
    (TimestralForward.predictExact, TimestralForward.java:234-252; ``jc_forward_timestral``)."""

    def __init__(self, engine: TimestralEngine, ends: str = "device", buckets: bool = True):
        if ends not in ("host", "device"):
            raise ValueError(f"ends must be 'host' or 'device', got {ends!r}")
        self.engine = engine
        self.config = engine.config
        self.ends = ends
        self.buckets = buckets  # timestral.tornado.buckets: the context padded to a bucketed patch count

    def predict_block(self, block: BlockInput) -> np.ndarray:
        if self.buckets:
            block = bucketed_context(block, self.config.patch_size)
        lay = BlockLayout.of(self.config, block)
        if self.ends == "device":
            return self.engine.forecast(WindowInputs.of(self.config, lay))
        prep = BlockPrep.of(self.config, lay)
        raw = self.engine.forward(DeviceInputs.of(lay, prep))
        return prep.finish(self.config, lay, raw)

    predictBlock = predict_block

    def predict_block_sign_flip(self, block: BlockInput) -> np.ndarray:
        """Sign-flip test-time augmentation in one forward. The reference's pipelines forecast a series and its
        negation as two passes and average each quantile level with the negated mirror of its complement
        (SignFlip.average, host/SignFlip.java; TimestralPipeline.java:190-196). Here the block and its
        negation are concatenated (the copies in groups of their own) and run as one block — half the launches
        and weight reads — then averaged the same way: out[q] = (a[q] + −b[c(q)]) / 2."""
        comp = sign_flip_complement(self.config.quantile_knots)
        both = with_negation(block)
        out = self.predict_block(both)
        r = block.rows
        a, b = out[:r], out[r:]
        return ((a + -b[..., comp]) / np.float32(2)).astype(np.float32)


def sign_flip_complement(levels) -> np.ndarray:
    """complement[i] = the level closest to 1 − levels[i] (SignFlip.complement); a quantile set that is not
    symmetric around 0.5 (to 1e-6) is rejected."""
    q = np.asarray(levels, np.float32)
    comp = np.empty(len(q), np.int64)
    for i in range(len(q)):
        target = np.float32(1) - q[i]
        best = 0
        for j in range(1, len(q)):
            if abs(q[j] - target) < abs(q[best] - target):
                best = j
        if abs(q[best] - target) > 1e-6:
            raise ValueError("sign-flip TTA needs a symmetric quantile set")
        comp[i] = best
    return comp


def with_negation(block: BlockInput) -> BlockInput:
    """The block followed by its negation (SignFlip.negate: targets and numeric covariates negated, masks and
    roles kept); the negated rows form groups of their own after the block's."""
    g = np.asarray(block.group)
    offset = int(g.max()) + 1 if len(g) else 0
    cat = lambda a, b: None if a is None else np.concatenate([a, b])  # noqa: E731
    kf = block.known_future
    return BlockInput(np.concatenate([block.inputs, -np.asarray(block.inputs)]),
                      np.concatenate([block.observed, block.observed]),
                      np.concatenate([g, g + offset]).astype(g.dtype), block.horizon_patches,
                      cat(block.role, block.role), cat(kf, None if kf is None else -np.asarray(kf)),
                      cat(block.known_future_mask, block.known_future_mask))
