"""ORACLE — test infrastructure only: ctypes access to the C restatement of the reference's FP32
Timestral CPU forward (``oracle/timestral.c``), fed from a config and a checkpoint dict."""

from __future__ import annotations

import ctypes

import numpy as np

from . import lib, threads

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float


class JcoTimestral(ctypes.Structure):
    _fields_ = [("patch_size", _I), ("d_model", _I), ("num_heads", _I), ("mlp_hidden_dim", _I), ("num_layers", _I),
                ("num_quantiles", _I), ("block_size", _I), ("attn_per_layer", _P), ("attn_is_time", _P),
                ("attn_gate", _P), ("quantile_knots", _P), ("rope_theta", _F), ("rope_partial_factor", _F),
                ("norm_eps", _F), ("minimum_scale", _F), ("quantile_width_factor", _F), ("use_asinh", _I),
                ("covariate_enabled", _I), ("attend_missing_patches", _I),
                ("emb_hidden_w", _P), ("emb_hidden_b", _P), ("emb_output_w", _P), ("emb_output_b", _P),
                ("emb_residual_w", _P), ("emb_residual_b", _P), ("forecast_query", _P), ("attn_norm", _P),
                ("wqkv", _P), ("gate_w", _P), ("wo", _P), ("mlp_norm", _P), ("w12", _P), ("w3", _P),
                ("out_norm", _P), ("head_hidden_w", _P), ("head_output_w", _P), ("head_residual_w", _P)]


class JcoBlock(ctypes.Structure):
    _fields_ = [("rows", _I), ("length", _I), ("horizon", _I), ("inputs", _P), ("observed", _P), ("group", _P),
                ("role", _P), ("known_future", _P), ("known_future_mask", _P)]


class JcoPrepared(ctypes.Structure):
    _fields_ = [("rows", _I), ("enc", _I), ("horizon", _I), ("ll", _I), ("covariates", _I), ("window", _P),
                ("obs", _P), ("key_valid", _P), ("first", _P), ("role", _P), ("known", _P), ("group", _P),
                ("pos", _P), ("loc", _P), ("scale", _P), ("tokens", _P)]


def _bind(l):
    l.jco_timestral_predict_block.argtypes = [ctypes.POINTER(JcoTimestral), ctypes.POINTER(JcoBlock), _P, _P, _I]
    l.jco_timestral_predict_block.restype = _I
    l.jco_timestral_prepare.argtypes = [ctypes.POINTER(JcoTimestral), ctypes.POINTER(JcoBlock),
                                        ctypes.POINTER(JcoPrepared)]
    l.jco_timestral_prepare.restype = _I
    l.jco_prepared_free.argtypes = [ctypes.POINTER(JcoPrepared)]
    l.jco_timestral_model.argtypes = [ctypes.POINTER(JcoTimestral), ctypes.POINTER(JcoPrepared), _P, _I]


class Model:
    """A Timestral checkpoint in the oracle's struct (keeps every array alive)."""

    def __init__(self, config, weights: dict[str, np.ndarray]):
        self.c = config
        keep = self._keep = []

        def arr(a, dtype=np.float32):
            a = np.ascontiguousarray(a, dtype)
            keep.append(a)
            return a.ctypes.data

        def ptrs(lst):
            a = (ctypes.c_void_p * max(1, len(lst)))(*[x for x in lst])
            keep.append(a)
            return ctypes.cast(a, ctypes.c_void_p).value

        w = {k: np.ascontiguousarray(v, np.float32) for k, v in weights.items()}
        axes = config.attention_axes()
        per_layer = [len(a) for a in axes]
        is_time, gated, norm, qkv, gate, wo = [], [], [], [], [], []
        for li, ax in enumerate(axes):
            pre = f"transformer.layers.{li}"
            for a, t in enumerate(ax):
                g = config.time_attn_gate if t else config.variate_attn_gate
                is_time.append(int(t))
                gated.append(int(g))
                norm.append(arr(w[f"{pre}.attn_norms.{a}.scale"]))
                qkv.append(arr(w[f"{pre}.attns.{a}.wQKV.weight"]))
                gate.append(arr(w[f"{pre}.attns.{a}._gate.weight"]) if g else None)
                wo.append(arr(w[f"{pre}.attns.{a}.wO.weight"]))
        L = len(axes)
        pe, hp = "representation.patch_proj.", "head.projection."
        self.s = JcoTimestral(
            config.patch_size, config.d_model, config.num_heads, config.mlp_hidden_dim, L, config.num_quantiles,
            config.block_size, arr(per_layer, np.int32), arr(is_time, np.int32), arr(gated, np.int32),
            arr(config.quantile_knots, np.float64), config.rope_theta, config.rope_partial_factor, config.norm_eps,
            config.minimum_scale, config.quantile_width_factor, int(config.use_asinh), int(config.covariate_enabled),
            int(config.attend_missing_patches),
            arr(w[pe + "hidden_layer.weight"]), arr(w[pe + "hidden_layer.bias"]), arr(w[pe + "output_layer.weight"]),
            arr(w[pe + "output_layer.bias"]), arr(w[pe + "residual_layer.weight"]),
            arr(w[pe + "residual_layer.bias"]), arr(w["representation.forecast_query"]), ptrs(norm), ptrs(qkv),
            ptrs(gate), ptrs(wo), ptrs([arr(w[f"transformer.layers.{i}.mlp_norm.scale"]) for i in range(L)]),
            ptrs([arr(w[f"transformer.layers.{i}.mlp.w12.weight"]) for i in range(L)]),
            ptrs([arr(w[f"transformer.layers.{i}.mlp.w3.weight"]) for i in range(L)]),
            arr(w["transformer.out_norm.scale"]), arr(w[hp + "hidden_layer.weight"]),
            arr(w[hp + "output_layer.weight"]), arr(w[hp + "residual_layer.weight"]))
        _bind(lib())

    def _block(self, b):
        keep = []

        def arr(a, dtype):
            if a is None:
                return None
            a = np.ascontiguousarray(a, dtype)
            keep.append(a)
            return a.ctypes.data

        rows, length = np.asarray(b.inputs).shape
        blk = JcoBlock(rows, length, b.horizon_patches, arr(b.inputs, np.float32), arr(b.observed, np.uint8),
                       arr(b.group, np.int32), arr(b.role, np.int32), arr(b.known_future, np.float32),
                       arr(b.known_future_mask, np.uint8))
        return blk, keep

    def predict_block(self, b, nthreads: int | None = None):
        """CpuTimestral.predictBlock: (out [rows, h·P, Q], raw head outputs [rows·h, P·Q])."""
        blk, keep = self._block(b)
        c = self.c
        rows = np.asarray(b.inputs).shape[0]
        out = np.empty((rows, b.horizon_patches * c.patch_size, c.num_quantiles), np.float32)
        raw = np.empty((rows * b.horizon_patches, c.patch_size * c.num_quantiles), np.float32)
        st = lib().jco_timestral_predict_block(ctypes.byref(self.s), ctypes.byref(blk), out.ctypes.data,
                                               raw.ctypes.data, nthreads or threads())
        if st:
            raise ValueError(f"oracle rejected the block ({st})")
        return out, raw

    def prepare(self, b) -> dict[str, np.ndarray]:
        """BlockLayout.of + BlockPrep.of: tokens, positions, key validity, loc/scale."""
        blk, keep = self._block(b)
        p = JcoPrepared()
        st = lib().jco_timestral_prepare(ctypes.byref(self.s), ctypes.byref(blk), ctypes.byref(p))
        if st:
            raise ValueError(f"oracle rejected the block ({st})")
        r, enc, h = p.rows, p.enc, p.horizon
        ps = self.c.patch_size
        w = enc * ps

        def take(ptr, n, dt):
            return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(dt)), (n,)).copy()

        out = {"rows": r, "enc": enc, "horizon": h, "ll": p.ll, "covariates": p.covariates,
               "tokens": take(p.tokens, r * enc * 2 * ps, ctypes.c_float).reshape(r, enc, 2 * ps),
               "positions": take(p.pos, r * (enc + h), ctypes.c_int).reshape(r, enc + h),
               "key_valid": take(p.key_valid, r * enc, ctypes.c_int).reshape(r, enc),
               "known": take(p.known, r, ctypes.c_int), "role": take(p.role, r, ctypes.c_int),
               "loc": take(p.loc, r * w, ctypes.c_float).reshape(r, w),
               "scale": take(p.scale, r * w, ctypes.c_float).reshape(r, w)}
        lib().jco_prepared_free(ctypes.byref(p))
        return out
