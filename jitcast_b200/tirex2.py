"""TiRex-2 on the B200 engine: the host side of ``ForwardPass.forward`` over the C ABI.

Mirrors, in NumPy, the reference's host ends of a TiRex-2 forward pass:

* ``TiRex2Config``  — tirex2/TiRex2Config.java:48-246 (config keys of the converted checkpoint, derived
  widths ``mlstm_qk_dim`` and ``ffn_dim``)
* ``ModelBatch``    — tirex2/ModelBatch.java:28-31
* ``structure``     — tirex2/tornado/TornadoForward.java:406-449: known covariates (reverse pass), the rows
  of multi-row groups (variate mixer), their group ranges and target flags; groups must be contiguous
* ``B200TiRex2Forward.forward`` — tirex2/tornado/TornadoForward.java:353-365 and Plan.run :799-827: NaN is
  replaced by 0 plus an is-present flag, the whole forward (scaler and patching, embedding, blocks,
  output embedding, unpatch) runs in ``libjitcast_b200.so`` (``jc_forward_tirex2``) and returns
  ``[rows, Q, context_len + future_len]`` in data units.

``random_checkpoint`` writes random-init weights with the checkpoint's tensor names and shapes
(TiRex2Weights.java:169-247).
"""

from __future__ import annotations

import ctypes
import json
import math
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from ._lib import c_int, c_vp, check, precision_code
from .timestral import _TensorView

MLSTM, SLSTM = 0, 1

NORM_EPS = 1e-6
FFN_ROUND_TO = 64
FFN_PROJ_FACTOR = np.float32(2.6667)
ATTENTION_FFN_FACTOR = 4


@dataclass
class TiRex2Config:
    """The TiRex2Config record (TiRex2Config.java:48-66)."""

    num_blocks: int
    embedding_dim: int
    patch_size: int
    input_ff_dim: int
    output_ff_dim: int
    context_len: int
    future_len: int
    quantiles: list[float]
    recipe: list[int]
    time_mixer_heads: int = 4
    slstm_heads: int = 4
    variate_heads: int = 4
    use_arcsinh: bool = True
    binary_aware: bool = True
    stack_out_norm_eps: float = 1e-7
    use_qk_norm: bool = True
    tta_diff: bool = True
    tta_sign_flip: bool = False

    def validate(self) -> "TiRex2Config":
        """The record's compact constructor (TiRex2Config.java:73-93)."""
        p = self.patch_size
        if p < 1 or self.context_len < 1 or self.future_len < 0 or (self.context_len + self.future_len) % p:
            raise ValueError(f"context_len + future_len ({self.context_len} + {self.future_len}) must be a "
                             f"positive multiple of the patch size {p}")
        for h in (self.time_mixer_heads, self.slstm_heads, self.variate_heads):
            if h < 1 or self.embedding_dim % h:
                raise ValueError(f"embedding_dim {self.embedding_dim} is not divisible by {h} heads")
        q = self.quantiles
        if len(q) % 2 == 0 or np.float32(q[len(q) // 2]) != np.float32(0.5):
            raise ValueError("the quantiles must be an odd number of levels with 0.5 in the middle")
        if any(not 0 < x < 1 for x in q) or any(not a < b for a, b in zip(q, q[1:])):
            raise ValueError("the quantiles must increase strictly within (0, 1)")
        if len(self.recipe) != self.num_blocks:
            raise ValueError(f"recipe has {len(self.recipe)} entries for {self.num_blocks} blocks")
        return self

    @property
    def num_patches(self) -> int:
        return (self.context_len + self.future_len) // self.patch_size

    @property
    def padded_length(self) -> int:
        return self.context_len + self.future_len

    @property
    def num_quantiles(self) -> int:
        return len(self.quantiles)

    @property
    def mlstm_qk_dim(self) -> int:
        return int(np.float32(self.embedding_dim) * np.float32(0.5))

    @property
    def ffn_dim(self) -> int:
        raw = int(np.float32(self.embedding_dim) * FFN_PROJ_FACTOR)
        return (raw + FFN_ROUND_TO - 1) // FFN_ROUND_TO * FFN_ROUND_TO

    @staticmethod
    def from_json(doc: str | dict) -> "TiRex2Config":
        """TiRex2Config.fromJson (TiRex2Config.java:131-211): the ``tirex2.config`` metadata."""
        c = json.loads(doc) if isinstance(doc, str) else dict(doc)

        def num(m, k):
            v = m.get(k)
            if not isinstance(v, (int, float)) or isinstance(v, bool) or float(v) != int(v):
                raise ValueError(f"config key '{k}' missing or not an integer")
            return int(v)

        def sub(m, k):
            v = m.get(k)
            if not isinstance(v, dict):
                raise ValueError(f"config key '{k}' missing")
            return v

        d = num(c, "embedding_dim")
        pin, pout = num(c, "input_patch_size"), num(c, "output_patch_size")
        if pin != pout or num(sub(c, "tokenizer_cfg"), "input_patch_stride") != pin:
            raise ValueError("only non-overlapping patches with input == output size are supported")
        scaler = sub(c, "scaler_cfg")
        out_norm = c.get("stack_out_norm_config")
        if isinstance(out_norm, dict) and out_norm.get("use_rmsnorm") is True:
            raise ValueError("stack_out_norm use_rmsnorm=true is not supported")
        stack = sub(c, "stack_config")
        templates = sub(stack, "templates")
        recipe = []
        for n in stack.get("recipe", []):
            mt = sub(sub(templates, n), "time_mixer").get("model_type")
            if mt == "bi-mlstm":
                recipe.append(MLSTM)
            elif mt == "bi-slstm":
                recipe.append(SLSTM)
            else:
                raise ValueError(f"unknown time mixer {mt}")
        blocks = num(c, "num_blocks")
        if len(recipe) != blocks:
            raise ValueError(f"recipe has {len(recipe)} entries for {blocks} blocks")
        heads = sl = vh = -1

        def same(cur, v, what):
            if cur >= 0 and cur != v:
                raise ValueError(f"templates disagree on {what}: {cur} vs {v}")
            return v

        for t in templates.values():
            tm, vm = sub(t, "time_mixer"), sub(t, "variate_mixer")
            heads = same(heads, num(tm, "num_heads"), "time mixer num_heads")
            if tm.get("num_slstm_heads") is not None:
                sl = same(sl, num(tm, "num_slstm_heads"), "num_slstm_heads")
            vh = same(vh, num(vm, "num_heads"), "variate mixer num_heads")
            if num(tm, "embedding_dim") != d or num(vm, "embedding_dim") != d:
                raise ValueError("mixer embedding_dim differs from the model's")
        eps = float("nan") if out_norm is None else float(out_norm.get("eps", 1e-7))
        return TiRex2Config(num_blocks=blocks, embedding_dim=d, patch_size=pin, input_ff_dim=num(c, "input_ff_dim"),
                            output_ff_dim=int(d * float(c["h_expand"])), context_len=num(c, "context_len"),
                            future_len=num(c, "future_len"), quantiles=[float(q) for q in c["quantiles"]],
                            recipe=recipe, time_mixer_heads=heads, slstm_heads=heads if sl < 0 else sl,
                            variate_heads=vh, use_arcsinh=scaler.get("use_arcsinh") is True,
                            binary_aware=scaler.get("binaryaware") is True, stack_out_norm_eps=eps,
                            use_qk_norm=c.get("use_qk_norm") is not False, tta_diff=c.get("tta_diff") is not False,
                            tta_sign_flip=c.get("tta_sign_flip") is True).validate()

    def to_json(self) -> dict:
        names = {MLSTM: "mlstm_block", SLSTM: "slstm_block"}
        templates = {}
        for kind, name in names.items():
            tm = {"model_type": "bi-mlstm" if kind == MLSTM else "bi-slstm", "num_heads": self.time_mixer_heads,
                  "embedding_dim": self.embedding_dim}
            if kind == SLSTM:
                tm["num_slstm_heads"] = self.slstm_heads
            templates[name] = {"time_mixer": tm, "variate_mixer": {"num_heads": self.variate_heads,
                                                                   "embedding_dim": self.embedding_dim}}
        return {"embedding_dim": self.embedding_dim, "input_patch_size": self.patch_size,
                "output_patch_size": self.patch_size, "tokenizer_cfg": {"input_patch_stride": self.patch_size},
                "scaler_cfg": {"use_arcsinh": self.use_arcsinh, "binaryaware": self.binary_aware},
                "stack_out_norm_config": {"eps": self.stack_out_norm_eps},
                "stack_config": {"templates": templates, "recipe": [names[k] for k in self.recipe]},
                "num_blocks": self.num_blocks, "input_ff_dim": self.input_ff_dim,
                "h_expand": self.output_ff_dim / self.embedding_dim, "context_len": self.context_len,
                "future_len": self.future_len, "quantiles": list(self.quantiles), "use_qk_norm": self.use_qk_norm,
                "tta_diff": self.tta_diff, "tta_sign_flip": self.tta_sign_flip}


def config4() -> TiRex2Config:
    """d 512, 12 blocks (sLSTM at 3, 7, 11, the rest mLSTM), 4 heads, patch 32,
    64 patches (context 1984 + future 64), 9 quantiles, input and output FF widths 2048."""
    recipe = [SLSTM if i % 4 == 3 else MLSTM for i in range(12)]
    return TiRex2Config(num_blocks=12, embedding_dim=512, patch_size=32, input_ff_dim=2048, output_ff_dim=2048,
                        context_len=1984, future_len=64, quantiles=[round(0.1 * i, 1) for i in range(1, 10)],
                        recipe=recipe).validate()


def weight_shapes(c: TiRex2Config) -> dict[str, tuple[int, ...]]:
    """Every checkpoint tensor and its shape (TiRex2Weights.load and Binder.block)."""
    d, p = c.embedding_dim, c.patch_size
    s: dict[str, tuple[int, ...]] = {}

    def linear(prefix, i, o, bias):
        s[f"{prefix}.weight"] = (o, i)
        if bias:
            s[f"{prefix}.bias"] = (o,)

    def residual(prefix, i, h, o):
        linear(f"{prefix}.hidden_layer", i, h, True)
        linear(f"{prefix}.output_layer", h, o, True)
        linear(f"{prefix}.residual_layer", i, o, True)

    residual("input_patch_embedding", 2 * p, c.input_ff_dim, d)
    for i, kind in enumerate(c.recipe):
        cell = f"stack.{i}.time_mixer.fwd_cell"
        if kind == MLSTM:
            qk, h = c.mlstm_qk_dim, c.time_mixer_heads
            linear(f"{cell}.q", d, qk, False)
            linear(f"{cell}.k", d, qk, False)
            linear(f"{cell}.v", d, d, False)
            linear(f"{cell}.ogate_preact", d, d, False)
            linear(f"{cell}.igate_preact", d, h, True)
            linear(f"{cell}.fgate_preact", d, h, True)
            s[f"{cell}.multihead_norm.weight"] = (d,)
            linear(f"{cell}.out_proj", d, d, False)
        else:
            h = c.slstm_heads
            dh = d // h
            for g in ("fgate", "igate", "zgate", "ogate"):
                s[f"{cell}.{g}.weight"] = (h, dh, dh)
            s[f"{cell}._recurrent_kernel_"] = (h, dh, 4, dh)
            s[f"{cell}._bias_"] = (h, 4, dh)
            s[f"{cell}.group_norm.weight"] = (d,)
        tm = f"stack.{i}.time_mixer"
        s[f"{tm}.norm_lstm.weight"] = (d,)
        linear(f"{tm}.combination", 2 * d, d, False)
        s[f"{tm}.norm_ffn.weight"] = (d,)
        linear(f"{tm}.ffn.proj_up_gate", d, c.ffn_dim, False)
        linear(f"{tm}.ffn.proj_up", d, c.ffn_dim, False)
        linear(f"{tm}.ffn.proj_down", c.ffn_dim, d, False)
        vm = f"stack.{i}.variate_mixer"
        s[f"{vm}.norm_attn.weight"] = (d,)
        for w in ("WQ", "WK", "WV", "WO"):
            linear(f"{vm}.attn.{w}", d, d, False)
        s[f"{vm}.norm_ffn.weight"] = (d,)
        linear(f"{vm}.ffn.wi", d, ATTENTION_FFN_FACTOR * d, False)
        linear(f"{vm}.ffn.wo", ATTENTION_FFN_FACTOR * d, d, False)
    s["stack_out_norm.weight"] = (d,)
    residual("output_patch_embedding", d, c.output_ff_dim, c.num_quantiles * p)
    return s


def random_checkpoint(c: TiRex2Config, seed: int = 0, norm_jitter: float = 0.0,
                      forget_bias: tuple[float, float] | None = None) -> dict[str, np.ndarray]:
    """Random-init weights: linear W ~ N(0, 1/in); headwise sLSTM gates and the recurrent kernel ~ N(0, 1/dh);
    biases ~ U(−0.1, 0.1); norm scales 1 (times 1 + N(0, norm_jitter) when tests want every scale to matter).

    ``forget_bias=(lo, hi)`` sets the forget-gate biases as xLSTM initialises them, evenly spaced from lo to hi
    (mLSTM ``fgate_preact.bias`` over the heads, the sLSTM ``_bias_`` forget slot over each head's units), which
    keeps the gates open and the random-init stack well conditioned."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in sorted(weight_shapes(c).items()):
        if name.endswith("norm.weight") or name.endswith("norm_lstm.weight") or name.endswith("norm_ffn.weight") \
                or name.endswith("norm_attn.weight") or name == "stack_out_norm.weight":
            v = np.ones(shape, np.float32)
            if norm_jitter:
                v = v + np.float32(norm_jitter) * rng.standard_normal(shape, dtype=np.float32)
            out[name] = v.astype(np.float32)
        elif name.endswith(".bias") or name.endswith("._bias_"):
            out[name] = rng.uniform(-0.1, 0.1, shape).astype(np.float32)
        elif name.endswith("_recurrent_kernel_") or len(shape) == 3:
            out[name] = rng.standard_normal(shape, dtype=np.float32) / np.float32(math.sqrt(shape[1]))
        else:
            out[name] = rng.standard_normal(shape, dtype=np.float32) / np.float32(math.sqrt(shape[1]))
    if forget_bias is not None:
        lo, hi = forget_bias
        for name, v in out.items():
            if name.endswith("fgate_preact.bias"):
                out[name] = np.linspace(lo, hi, v.size).astype(np.float32)
            elif name.endswith("._bias_"):  # [heads, 4, dh] in the cell's (i, f, z, o) slot order
                v = v.copy()
                v[:, 1, :] = np.linspace(lo, hi, v.shape[2], dtype=np.float32)[None]
                out[name] = v
    return out


@dataclass
class ModelBatch:
    """``x`` [rows, context_len + future_len] with NaN where there is no observation; ``group`` [rows]
    (rows attend across variates only within their group); ``target`` [rows] (covariate rows cannot
    attend to targets)."""

    x: np.ndarray
    group: np.ndarray
    target: np.ndarray

    @property
    def rows(self) -> int:
        return self.x.shape[0]


@dataclass
class Structure:
    """TornadoForward.Structure: known covariates, kept rows (of multi-row groups), each kept row's
    group range within the kept list and its target flag."""

    known: np.ndarray
    kept: np.ndarray
    group_start: np.ndarray
    group_end: np.ndarray
    kept_target: np.ndarray


def structure(c: TiRex2Config, batch: ModelBatch) -> Structure:
    """TornadoForward.structure (TornadoForward.java:406-449)."""
    rows, length = batch.x.shape
    if length != c.padded_length:
        raise ValueError(f"rows have length {length}, expected {c.padded_length}")
    group = np.asarray(batch.group, np.float32)
    target = np.asarray(batch.target, bool)
    fut = ~np.isnan(batch.x[:, length - c.future_len:]) if c.future_len else np.zeros((rows, 0), bool)
    known = [r for r in range(rows) if not target[r] and fut[r].any()]
    kept, start, end, tgt = [], [], [], []
    seen = set()
    r = 0
    while r < rows:
        e = r
        while e < rows and group[e] == group[r]:
            e += 1
        if float(group[r]) in seen:
            raise ValueError(f"rows of group {group[r]} are not contiguous")
        seen.add(float(group[r]))
        if e - r > 1:
            s0 = len(kept)
            for q in range(r, e):
                kept.append(q)
                start.append(s0)
                end.append(s0 + (e - r))
                tgt.append(1 if target[q] else 0)
        r = e
    i32 = lambda v: np.asarray(v, np.int32)
    return Structure(i32(known), i32(kept), i32(start), i32(end), i32(tgt))


class _Desc(ctypes.Structure):
    _fields_ = [("embedding_dim", c_int), ("num_blocks", c_int), ("patch_size", c_int), ("input_ff_dim", c_int),
                ("output_ff_dim", c_int), ("context_len", c_int), ("future_len", c_int), ("num_quantiles", c_int),
                ("block_types", ctypes.POINTER(ctypes.c_int32)), ("time_mixer_heads", c_int),
                ("slstm_heads", c_int), ("variate_heads", c_int), ("use_arcsinh", c_int), ("binary_aware", c_int),
                ("use_qk_norm", c_int), ("stack_out_norm_eps", ctypes.c_float)]


class Batch(ctypes.Structure):
    """jc_tirex2_batch."""

    _fields_ = [("rows", c_int), ("x", c_vp), ("present", c_vp), ("n_known", c_int), ("known", c_vp),
                ("n_kept", c_int), ("kept", c_vp), ("group_start", c_vp), ("group_end", c_vp),
                ("kept_target", c_vp)]


_lib.declare("jc_engine_create_tirex2", c_int, [ctypes.POINTER(_Desc), ctypes.POINTER(_TensorView), c_int,
                                                  ctypes.POINTER(c_int), c_int, c_int, ctypes.POINTER(c_vp)])
_lib.declare("jc_forward_tirex2", c_int, [c_vp, ctypes.POINTER(Batch), c_vp])
_lib.declare("jc_forward_tirex2_device", c_int, [c_vp, c_int, ctypes.POINTER(Batch), c_vp, c_vp])


@dataclass
class DeviceInputs:
    """What TornadoForward.Plan.run uploads (TornadoForward.java:799-815): values with NaN replaced by 0,
    the is-present flags, and the structure lists."""

    x: np.ndarray
    present: np.ndarray
    st: Structure
    _keep: list = field(default_factory=list)

    @staticmethod
    def of(c: TiRex2Config, batch: ModelBatch) -> "DeviceInputs":
        st = structure(c, batch)
        here = ~np.isnan(batch.x)
        x = np.ascontiguousarray(np.where(here, batch.x, 0.0), np.float32)
        return DeviceInputs(x, np.ascontiguousarray(here, np.float32), st)

    def block(self) -> Batch:
        s = self.st
        return Batch(self.x.shape[0], self.x.ctypes.data, self.present.ctypes.data, len(s.known),
                     s.known.ctypes.data, len(s.kept), s.kept.ctypes.data, s.group_start.ctypes.data,
                     s.group_end.ctypes.data, s.kept_target.ctypes.data)


class TiRex2Engine:
    """A TiRex-2 model resident on one or more GPUs (``jc_engine_create_tirex2``)."""

    def __init__(self, config: TiRex2Config, weights: dict[str, np.ndarray], devices=(0,), precision="fp16"):
        self.config = config
        keep = {k: np.ascontiguousarray(v, np.float32) for k, v in weights.items()}
        views = (_TensorView * len(keep))()
        names = []
        for i, (k, v) in enumerate(keep.items()):
            names.append(k.encode())
            views[i] = _TensorView(names[-1], v.ctypes.data, v.ndim,
                                   (ctypes.c_int64 * 4)(*(list(v.shape) + [0] * (4 - v.ndim))))
        kinds = (ctypes.c_int32 * config.num_blocks)(*config.recipe)
        desc = _Desc(config.embedding_dim, config.num_blocks, config.patch_size, config.input_ff_dim,
                     config.output_ff_dim, config.context_len, config.future_len, config.num_quantiles, kinds,
                     config.time_mixer_heads, config.slstm_heads, config.variate_heads, int(config.use_arcsinh),
                     int(config.binary_aware), int(config.use_qk_norm), config.stack_out_norm_eps)
        devs = (c_int * len(devices))(*devices)
        h = c_vp()
        check(_lib.lib().jc_engine_create_tirex2(ctypes.byref(desc), views, len(keep), devs, len(devices),
                                                 precision_code(precision), ctypes.byref(h)))
        self._h = h

    @property
    def handle(self):
        if not self._h:
            raise RuntimeError("engine is closed")
        return self._h

    def forward_inputs(self, di: DeviceInputs, out: np.ndarray | None = None) -> np.ndarray:
        """out [rows, Q, len] for prepared host inputs, written into ``out`` when given (a C-contiguous float32
        array of that shape, e.g. in pinned memory)."""
        c = self.config
        shape = (di.x.shape[0], c.num_quantiles, c.padded_length)
        if out is None:
            out = np.empty(shape, np.float32)
        elif out.shape != shape or out.dtype != np.float32 or not out.flags.c_contiguous:
            raise ValueError(f"out must be a C-contiguous float32 array of shape {shape}")
        blk = di.block()
        check(_lib.lib().jc_forward_tirex2(self.handle, ctypes.byref(blk), out.ctypes.data))
        return out

    def set_option(self, key: str, value: int) -> None:
        check(_lib.lib().jc_engine_set_option(self.handle, key.encode(), int(value)))

    def sync(self) -> None:
        check(_lib.lib().jc_engine_sync(self.handle))

    def profile(self, slot: int = 0) -> dict[str, dict[str, float]]:
        cap = 32
        names = (ctypes.c_char_p * cap)()
        ms = (ctypes.c_double * cap)()
        launches = (ctypes.c_longlong * cap)()
        flops = (ctypes.c_double * cap)()
        n = c_int()
        check(_lib.lib().jc_engine_profile(self.handle, slot, names, ms, launches, flops, cap, ctypes.byref(n)))
        return {names[i].decode(): {"ms": ms[i], "launches": launches[i], "flops": flops[i]} for i in range(n.value)}

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


class B200TiRex2Forward:
    """``ForwardPass`` on the B200 engine (TornadoForward.forward, TornadoForward.java:353-365)."""

    def __init__(self, engine: TiRex2Engine):
        self.engine = engine
        self.config = engine.config

    def forward(self, batch: ModelBatch) -> np.ndarray:
        """``[rows, Q, context_len + future_len]``, rescaled to data units."""
        return self.engine.forward_inputs(DeviceInputs.of(self.config, batch))
