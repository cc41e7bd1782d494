"""ORACLE — test infrastructure only: ctypes access to the C restatement of the reference's FP32
TiRex-2 CPU forward (``oracle/tirex2.c``, CpuReference.forward), fed from a config and a checkpoint dict."""

from __future__ import annotations

import ctypes

import numpy as np

from . import lib, register, threads

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float

_PER_BLOCK = ("norm_lstm", "mq", "mk", "mv", "mo", "ig_w", "ig_b", "fg_w", "fg_b", "head_norm", "out_proj", "sg0",
              "sg1", "sg2", "sg3", "srec", "sbias", "group_norm", "comb", "norm_ffn", "up_gate", "up", "down",
              "norm_attn", "wq", "wk", "wv", "wo", "norm_ffn_attn", "ffn_in", "ffn_out")


class JcoTirex2(ctypes.Structure):
    _fields_ = ([(n, _I) for n in ("d", "blocks", "patch", "in_ff", "out_ff", "context_len", "future_len", "num_q",
                                   "use_arcsinh", "binary_aware", "use_qk_norm", "tm_heads", "slstm_heads",
                                   "var_heads")]
                + [("out_norm_eps", _F), ("block_types", _P)]
                + [(n, _P) for n in ("in_hw", "in_hb", "in_ow", "in_ob", "in_rw", "in_rb")]
                + [(n, _P) for n in _PER_BLOCK]
                + [(n, _P) for n in ("out_norm", "out_hw", "out_hb", "out_ow", "out_ob", "out_rw", "out_rb")])


@register("tirex2")
def _bind(l):
    l.jco_tirex2_forward.argtypes = [ctypes.POINTER(JcoTirex2), _I, _P, _P, _P, _P, _I]
    l.jco_tirex2_forward.restype = _I
    l.jco_tirex2_mlstm_core.argtypes = [_P, _I, _I, _I, _I, _P]
    l.jco_tirex2_slstm_recurrence.argtypes = [_P, _I, _I, _I, _I, _P, _P, _P]


class Model:
    """CpuReference over a checkpoint dict (names of TiRex2Weights)."""

    def __init__(self, c, weights):
        self.c = c
        keep = self._keep = []

        def arr(a, dtype=np.float32):
            a = np.ascontiguousarray(a, dtype)
            keep.append(a)
            return a.ctypes.data

        def per_block(fn):
            ptrs = []
            for i in range(c.num_blocks):
                name = fn(i)
                ptrs.append(arr(weights[name]) if name is not None else None)
            a = (ctypes.c_void_p * c.num_blocks)(*ptrs)
            keep.append(a)
            return ctypes.cast(a, ctypes.c_void_p).value

        def cell(i, part, kind):
            return f"stack.{i}.time_mixer.fwd_cell.{part}" if c.recipe[i] == kind else None

        m = JcoTirex2()
        m.d, m.blocks, m.patch = c.embedding_dim, c.num_blocks, c.patch_size
        m.in_ff, m.out_ff, m.context_len, m.future_len = c.input_ff_dim, c.output_ff_dim, c.context_len, c.future_len
        m.num_q, m.use_arcsinh, m.binary_aware, m.use_qk_norm = (c.num_quantiles, int(c.use_arcsinh),
                                                                 int(c.binary_aware), int(c.use_qk_norm))
        m.tm_heads, m.slstm_heads, m.var_heads = c.time_mixer_heads, c.slstm_heads, c.variate_heads
        m.out_norm_eps = c.stack_out_norm_eps
        m.block_types = arr(np.asarray(c.recipe, np.int32), np.int32)
        for tag, pre in (("in", "input_patch_embedding"), ("out", "output_patch_embedding")):
            for part, k in (("h", "hidden_layer"), ("o", "output_layer"), ("r", "residual_layer")):
                setattr(m, f"{tag}_{part}w", arr(weights[f"{pre}.{k}.weight"]))
                setattr(m, f"{tag}_{part}b", arr(weights[f"{pre}.{k}.bias"]))
        tm = lambda part: (lambda i: f"stack.{i}.time_mixer.{part}")
        vm = lambda part: (lambda i: f"stack.{i}.variate_mixer.{part}")
        M, S = 0, 1
        fields = {
            "norm_lstm": tm("norm_lstm.weight"),
            "mq": lambda i: cell(i, "q.weight", M), "mk": lambda i: cell(i, "k.weight", M),
            "mv": lambda i: cell(i, "v.weight", M), "mo": lambda i: cell(i, "ogate_preact.weight", M),
            "ig_w": lambda i: cell(i, "igate_preact.weight", M), "ig_b": lambda i: cell(i, "igate_preact.bias", M),
            "fg_w": lambda i: cell(i, "fgate_preact.weight", M), "fg_b": lambda i: cell(i, "fgate_preact.bias", M),
            "head_norm": lambda i: cell(i, "multihead_norm.weight", M),
            "out_proj": lambda i: cell(i, "out_proj.weight", M),
            # FlashRNN slot order (i, f, z, o) is fed from the checkpoint's (fgate, igate, zgate, ogate)
            # tensors (TiRex2Weights.java:213-216)
            "sg0": lambda i: cell(i, "fgate.weight", S), "sg1": lambda i: cell(i, "igate.weight", S),
            "sg2": lambda i: cell(i, "zgate.weight", S), "sg3": lambda i: cell(i, "ogate.weight", S),
            "srec": lambda i: cell(i, "_recurrent_kernel_", S), "sbias": lambda i: cell(i, "_bias_", S),
            "group_norm": lambda i: cell(i, "group_norm.weight", S),
            "comb": tm("combination.weight"), "norm_ffn": tm("norm_ffn.weight"),
            "up_gate": tm("ffn.proj_up_gate.weight"), "up": tm("ffn.proj_up.weight"), "down": tm("ffn.proj_down.weight"),
            "norm_attn": vm("norm_attn.weight"), "wq": vm("attn.WQ.weight"), "wk": vm("attn.WK.weight"),
            "wv": vm("attn.WV.weight"), "wo": vm("attn.WO.weight"), "norm_ffn_attn": vm("norm_ffn.weight"),
            "ffn_in": vm("ffn.wi.weight"), "ffn_out": vm("ffn.wo.weight"),
        }
        for k, fn in fields.items():
            setattr(m, k, per_block(fn))
        m.out_norm = arr(weights["stack_out_norm.weight"])
        self.m = m

    def forward(self, batch, nthreads: int | None = None) -> np.ndarray:
        """``[rows, Q, context_len + future_len]`` in data units."""
        c = self.c
        x = np.ascontiguousarray(batch.x, np.float32)
        rows = x.shape[0]
        group = np.ascontiguousarray(batch.group, np.float32)
        target = np.ascontiguousarray(np.asarray(batch.target, bool), np.int32)
        out = np.empty((rows, c.num_quantiles, c.padded_length), np.float32)
        rc = lib().jco_tirex2_forward(ctypes.byref(self.m), rows, x.ctypes.data, group.ctypes.data,
                                      target.ctypes.data, out.ctypes.data, nthreads or threads())
        if rc != 0:
            raise ValueError("oracle rejected the batch")
        return out


def mlstm_core(p: np.ndarray, rows: int, seq: int, heads: int) -> np.ndarray:
    p = np.ascontiguousarray(p, np.float32)
    h = np.empty((rows * seq, heads * 128), np.float32)
    lib().jco_tirex2_mlstm_core(p.ctypes.data, rows, seq, heads, p.shape[1], h.ctypes.data)
    return h


def slstm_recurrence(wx: np.ndarray, rows: int, seq: int, d: int, heads: int, r: np.ndarray,
                     b: np.ndarray) -> np.ndarray:
    wx = np.ascontiguousarray(wx, np.float32)
    r = np.ascontiguousarray(r, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    y = np.empty((rows * seq, d), np.float32)
    lib().jco_tirex2_slstm_recurrence(wx.ctypes.data, rows, seq, d, heads, r.ctypes.data, b.ctypes.data,
                                      y.ctypes.data)
    return y
