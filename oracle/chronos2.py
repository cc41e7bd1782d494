"""ORACLE — test infrastructure only: ctypes access to the C restatement of the reference's FP32
Chronos-2 CPU forward (``oracle/chronos2.c``), fed from a config and a checkpoint dict."""

from __future__ import annotations

import ctypes

import numpy as np

from . import lib, threads

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float


class JcoChronos2(ctypes.Structure):
    _fields_ = ([(n, _I) for n in ("d_model", "d_kv", "d_ff", "num_layers", "num_heads", "context_length",
                                   "patch_size", "num_quantiles", "use_reg_token", "use_arcsinh",
                                   "time_encoding_scale")]
                + [("eps", _F), ("rope_theta", _F), ("shared", _P)]
                + [(n, _P) for n in ("in_hw", "in_hb", "in_ow", "in_ob", "in_rw", "in_rb", "time_norm", "time_q",
                                     "time_k", "time_v", "time_o", "group_norm", "group_q", "group_k", "group_v",
                                     "group_o", "mlp_norm", "wi", "wo", "final_norm", "out_hw", "out_hb", "out_ow",
                                     "out_ob", "out_rw", "out_rb")])


class JcoInput(ctypes.Structure):
    _fields_ = [("rows", _I), ("length", _I), ("output_patches", _I), ("context", _P), ("group", _P),
                ("future", _P), ("future_len", _I)]


class JcoPrepared(ctypes.Structure):
    _fields_ = [("rows", _I), ("nc", _I), ("reg", _I), ("h", _I), ("n", _I), ("live", _P), ("tokens", _P),
                ("loc", _P), ("scale", _P), ("group", _P)]


def _bind(l):
    l.jco_chronos2_forward.argtypes = [ctypes.POINTER(JcoChronos2), ctypes.POINTER(JcoInput), _P, _P, _I]
    l.jco_chronos2_forward.restype = _I
    l.jco_chronos2_prepare.argtypes = [ctypes.POINTER(JcoChronos2), ctypes.POINTER(JcoInput),
                                       ctypes.POINTER(JcoPrepared)]
    l.jco_chronos2_prepare.restype = _I
    l.jco_c2_prepared_free.argtypes = [ctypes.POINTER(JcoPrepared)]


class Model:
    def __init__(self, c, weights):
        self.c = c
        keep = self._keep = []

        def arr(a, dtype=np.float32):
            a = np.ascontiguousarray(a, dtype)
            keep.append(a)
            return a.ctypes.data

        def per_layer(fmt):
            a = (ctypes.c_void_p * c.num_layers)(*[arr(weights[fmt.format(i)]) for i in range(c.num_layers)])
            keep.append(a)
            return ctypes.cast(a, ctypes.c_void_p).value

        blk = "encoder.block.{}.layer."
        ie, oe = "input_patch_embedding.", "output_patch_embedding."
        self.s = JcoChronos2(
            c.d_model, c.d_kv, c.d_ff, c.num_layers, c.num_heads, c.context_length, c.patch_size, c.num_quantiles,
            int(c.use_reg_token), int(c.use_arcsinh), c.time_encoding_scale, c.layer_norm_eps, c.rope_theta,
            arr(weights["shared.weight"]),
            *[arr(weights[ie + f"{p}_layer.{t}"]) for p in ("hidden", "output", "residual") for t in ("weight", "bias")],
            per_layer(blk + "0.layer_norm.weight"), per_layer(blk + "0.self_attention.q.weight"),
            per_layer(blk + "0.self_attention.k.weight"), per_layer(blk + "0.self_attention.v.weight"),
            per_layer(blk + "0.self_attention.o.weight"), per_layer(blk + "1.layer_norm.weight"),
            per_layer(blk + "1.self_attention.q.weight"), per_layer(blk + "1.self_attention.k.weight"),
            per_layer(blk + "1.self_attention.v.weight"), per_layer(blk + "1.self_attention.o.weight"),
            per_layer(blk + "2.layer_norm.weight"), per_layer(blk + "2.mlp.wi.weight"),
            per_layer(blk + "2.mlp.wo.weight"), arr(weights["encoder.final_layer_norm.weight"]),
            *[arr(weights[oe + f"{p}_layer.{t}"]) for p in ("hidden", "output", "residual") for t in ("weight", "bias")])
        _bind(lib())

    def _input(self, inp):
        keep = []

        def arr(a, dtype):
            if a is None:
                return None
            a = np.ascontiguousarray(a, dtype)
            keep.append(a)
            return a.ctypes.data

        ctx = np.asarray(inp.context, np.float32)
        fut = None if inp.future_covariates is None else np.asarray(inp.future_covariates, np.float32)
        s = JcoInput(ctx.shape[0], ctx.shape[1], inp.output_patches, arr(ctx, np.float32), arr(inp.group, np.int32),
                     arr(fut, np.float32), 0 if fut is None else fut.shape[1])
        return s, keep

    def forward(self, inp, nthreads=None):
        """CpuChronos2.forward: (out [rows, Q, h·P], raw [rows·h, Q·P])."""
        s, keep = self._input(inp)
        c = self.c
        r = np.asarray(inp.context).shape[0]
        h = inp.output_patches
        out = np.empty((r, c.num_quantiles, h * c.patch_size), np.float32)
        raw = np.empty((r * h, c.num_quantiles * c.patch_size), np.float32)
        st = lib().jco_chronos2_forward(ctypes.byref(self.s), ctypes.byref(s), out.ctypes.data, raw.ctypes.data,
                                        nthreads or threads())
        if st:
            raise ValueError(f"oracle rejected the input ({st})")
        return out, raw

    def prepare(self, inp):
        s, keep = self._input(inp)
        p = JcoPrepared()
        if lib().jco_chronos2_prepare(ctypes.byref(self.s), ctypes.byref(s), ctypes.byref(p)):
            raise ValueError("oracle rejected the input")
        r, nc, h, n = p.rows, p.nc, p.h, p.n
        ps = self.c.patch_size

        def take(ptr, cnt, dt):
            return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(dt)), (cnt,)).copy()

        out = {"nc": nc, "reg": p.reg, "h": h, "n": n,
               "live": take(p.live, r * n, ctypes.c_int).reshape(r, n),
               "tokens": take(p.tokens, r * (nc + h) * 3 * ps, ctypes.c_float).reshape(r, nc + h, 3 * ps),
               "loc": take(p.loc, r, ctypes.c_float), "scale": take(p.scale, r, ctypes.c_float)}
        lib().jco_c2_prepared_free(ctypes.byref(p))
        return out
