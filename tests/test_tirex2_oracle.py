"""The TiRex-2 oracle (C restatement of CpuReference.forward) against a second, independent restatement
written here in float64 NumPy from the cells' equations (Cells.java:31-42 mLSTM, :120-133 sLSTM), on a
tiny random-init model with every path the reference has: mLSTM and sLSTM blocks, known covariates with
the reverse pass and combination, multi-row groups through the variate mixer (with qk-norm and the
covariate→target mask), binary rows, NaN gaps. No golden TiRex-2 activations exist in the reference tree,
so two restatements agreeing is what pins the oracle here.
"""

import math

import numpy as np
import pytest

from jitcast_b200 import tirex2 as tx
from oracle import tirex2 as otx


def tiny_config(**kw):
    base = dict(num_blocks=3, embedding_dim=256, patch_size=8, input_ff_dim=96, output_ff_dim=64, context_len=48,
                future_len=16, quantiles=[0.1, 0.5, 0.9], recipe=[tx.MLSTM, tx.SLSTM, tx.MLSTM],
                time_mixer_heads=2, slstm_heads=2, variate_heads=2)
    base.update(kw)
    return tx.TiRex2Config(**base).validate()


def mixed_batch(c, seed=3):
    """Two univariate series, a group of three rows (target + two covariates, one of them known in the
    future), a binary series, NaN gaps and a late start."""
    rng = np.random.default_rng(seed)
    L, F = c.padded_length, c.future_len
    rows, group, target = [], [], []

    def series(scale=1.0):
        return (np.cumsum(rng.standard_normal(L)) * scale + 5.0).astype(np.float32)

    x = series()
    x[L - F:] = np.nan
    rows.append(x); group.append(0); target.append(True)
    x = series(3.0)
    x[:10] = np.nan
    x[20:27] = np.nan
    x[L - F:] = np.nan
    rows.append(x); group.append(1); target.append(True)
    for j in range(3):  # group 2: a target and two covariates; covariate 1 is known in the future
        x = series()
        if j != 2:
            x[L - F:] = np.nan
        rows.append(x); group.append(2); target.append(j == 0)
    x = (rng.random(L) < 0.3).astype(np.float32)
    x[L - F:] = np.nan
    rows.append(x); group.append(3); target.append(True)
    return tx.ModelBatch(np.stack(rows), np.asarray(group, np.float32), np.asarray(target))


def softcap(z, cap=15.0):
    return cap * np.tanh(z / cap)


def logsig(z):
    return np.minimum(z, 0) - np.log1p(np.exp(-np.abs(z)))


def sig(z):
    return 1 / (1 + np.exp(-z))


def head_ln(x, heads, w, eps=1e-6):
    n, d = x.shape
    v = x.reshape(n, heads, d // heads)
    mu = v.mean(-1, keepdims=True)
    var = ((v - mu) ** 2).mean(-1, keepdims=True)
    return ((v - mu) / np.sqrt(var + eps)).reshape(n, d) * w


def rms(x, w, eps):
    y = x / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return y if w is None else y * w


def numpy_forward(c, W, batch):
    """float64 forward written from the model's equations."""
    W = {k: v.astype(np.float64) for k, v in W.items()}
    silu = lambda v: v / (1 + np.exp(-v))
    d, P, S, L, Q = c.embedding_dim, c.patch_size, c.num_patches, c.padded_length, c.num_quantiles
    x = batch.x.astype(np.float64)
    R = x.shape[0]
    here = ~np.isnan(x)
    loc = np.where(here.any(1), np.nansum(x, 1) / np.maximum(here.sum(1), 1), 0.0)
    sd = np.sqrt(np.nansum((x - loc[:, None]) ** 2, 1) / np.maximum(here.sum(1), 1))
    sd = np.where(here.any(1), np.maximum(sd, 1e-8), 1.0)
    binary = np.array([np.all((r[~np.isnan(r)] == 0) | (r[~np.isnan(r)] == 1)) for r in x]) & c.binary_aware
    loc = np.where(binary, 0.0, loc)
    sd = np.where(binary, 1.0, sd)
    z = (x - loc[:, None]) / sd[:, None]
    z = np.where(binary[:, None] | (not c.use_arcsinh), z, np.arcsinh(z))
    z = np.where(here, z, 0.0)
    tok = np.concatenate([z.reshape(R, S, P), here.reshape(R, S, P).astype(np.float64)], -1).reshape(R * S, 2 * P)

    def lin(a, name, bias=True):
        y = a @ W[name + ".weight"].T
        return y + W[name + ".bias"] if bias and name + ".bias" in W else y

    def resblock(a, pre):
        return lin(silu(lin(a, pre + ".hidden_layer")), pre + ".output_layer") + lin(a, pre + ".residual_layer")

    h = resblock(tok, "input_patch_embedding")
    target = np.asarray(batch.target, bool)
    known = [r for r in range(R) if not target[r] and here[r, L - c.future_len:].any()]

    def mlstm(xn, rows, pre):
        H = c.time_mixer_heads
        q = lin(xn, pre + ".q", False).reshape(rows, S, H, 64)
        k = lin(xn, pre + ".k", False).reshape(rows, S, H, 64)
        v = lin(xn, pre + ".v", False).reshape(rows, S, H, 128)
        o = lin(xn, pre + ".ogate_preact", False)
        ig = softcap(lin(xn, pre + ".igate_preact")).reshape(rows, S, H)
        fg = logsig(softcap(lin(xn, pre + ".fgate_preact"))).reshape(rows, S, H)
        F = np.cumsum(fg, 1)  # [rows, S, H]
        logD = F[:, :, None, :] - F[:, None, :, :] + ig[:, None, :, :]  # [rows, t, s, H]
        causal = np.tril(np.ones((S, S), bool))[None, :, :, None]
        logD = np.where(causal, logD, -np.inf)
        m = np.maximum(F, logD.max(2))  # [rows, t, H]
        C = np.einsum("rthe,rshe->rtsh", q, k) / 8.0 * np.exp(logD - m[:, :, None, :])
        num = np.einsum("rtsh,rshe->rthe", C, v)
        den = C.sum(2)
        hh = num / (np.maximum(np.abs(den), np.exp(-m)) + 1e-6)[..., None]
        hn = head_ln(hh.reshape(rows * S, H * 128), H, W[pre + ".multihead_norm.weight"]) * sig(o)
        return lin(hn, pre + ".out_proj", False)

    def slstm(xn, rows, pre):
        H = c.slstm_heads
        dh = d // H
        xs = xn.reshape(rows * S, H, dh)
        # slot g reads the checkpoint's (fgate, igate, zgate, ogate)[g] tensor
        wx = np.stack([np.einsum("nhj,hoj->nho", xs, W[f"{pre}.{g}.weight"]) for g in
                       ("fgate", "igate", "zgate", "ogate")], 1)  # [n, 4, H, dh]
        wx = wx.reshape(rows, S, 4, H, dh)
        Rk, b = W[pre + "._recurrent_kernel_"], W[pre + "._bias_"]  # [H, dh, 4, dh], [H, 4, dh]
        y = np.zeros((rows, H, dh)); cc = np.zeros_like(y); nn = np.zeros_like(y); mm = np.zeros_like(y)
        out = np.zeros((rows, S, H, dh))
        for t in range(S):
            raw = wx[:, t].transpose(0, 2, 1, 3) + b[None] + np.einsum("rhp,hpge->rhge", y, Rk)
            i, f, zz, o = raw[:, :, 0], raw[:, :, 1], raw[:, :, 2], raw[:, :, 3]
            lf = logsig(f) + mm
            mn = i if t == 0 else np.maximum(i, lf)
            cc = np.exp(lf - mn) * cc + np.exp(i - mn) * np.tanh(zz)
            nn = np.maximum(np.exp(lf - mn) * nn + np.exp(i - mn), 1.0)
            y = sig(o) * cc / nn
            mm = mn
            out[:, t] = y
        return head_ln(out.reshape(rows * S, d), H, W[pre + ".group_norm.weight"])

    for i, kind in enumerate(c.recipe):
        tm = f"stack.{i}.time_mixer"
        cellf = mlstm if kind == tx.MLSTM else slstm
        xn = rms(h, W[tm + ".norm_lstm.weight"], 1e-6)
        y = cellf(xn, R, tm + ".fwd_cell").reshape(R, S, d)
        if known:
            rev = xn.reshape(R, S, d)[known][:, ::-1].reshape(-1, d)
            ro = cellf(rev, len(known), tm + ".fwd_cell").reshape(len(known), S, d)[:, ::-1]
            cat = np.concatenate([y[known], ro], -1).reshape(-1, 2 * d)
            y[known] = lin(cat, tm + ".combination", False).reshape(len(known), S, d)
        y = y.reshape(R * S, d) + h
        fn = rms(y, W[tm + ".norm_ffn.weight"], 1e-6)
        h = lin(silu(lin(fn, tm + ".ffn.proj_up_gate", False)) * lin(fn, tm + ".ffn.proj_up", False),
                tm + ".ffn.proj_down", False) + y
        vm = f"stack.{i}.variate_mixer"
        g = np.asarray(batch.group)
        kept = [r for r in range(R) if (g == g[r]).sum() > 1]
        if kept:
            H = c.variate_heads
            dh = d // H
            xk = h.reshape(R, S, d)[kept].reshape(-1, d)
            nr = rms(xk, W[vm + ".norm_attn.weight"], 1e-6)
            q = lin(nr, vm + ".attn.WQ", False).reshape(-1, H, dh)
            k = lin(nr, vm + ".attn.WK", False).reshape(-1, H, dh)
            v = lin(nr, vm + ".attn.WV", False).reshape(len(kept), S, H, dh)
            if c.use_qk_norm:
                eps32 = float(np.finfo(np.float32).eps)
                q = rms(q, None, eps32)
                k = rms(k, None, eps32)
            q = q.reshape(len(kept), S, H, dh)
            k = k.reshape(len(kept), S, H, dh)
            s = np.einsum("qthe,kthe->thqk", q, k) / math.sqrt(dh)
            gk = g[kept]
            tk = target[kept]
            allow = (gk[:, None] == gk[None, :]) & ~(~tk[:, None] & tk[None, :])
            s = np.where(allow[None, None], s, -np.inf)
            p = np.exp(s - s.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            att = np.einsum("thqk,kthe->qthe", p, v).reshape(-1, d)
            out = lin(att, vm + ".attn.WO", False) + xk
            fn = rms(out, W[vm + ".norm_ffn.weight"], 1e-6)
            mlp = lin(silu(lin(fn, vm + ".ffn.wi", False)), vm + ".ffn.wo", False) + out
            hh = h.reshape(R, S, d)
            hh[kept] = mlp.reshape(len(kept), S, d)
            h = hh.reshape(R * S, d)
    hn = rms(h, W["stack_out_norm.weight"], c.stack_out_norm_eps)
    y = resblock(hn, "output_patch_embedding").reshape(R, S, Q, P)
    sinh_on = c.use_arcsinh & ~binary
    y = np.where(sinh_on[:, None, None, None], np.sinh(np.clip(y, -20, 20)), y)
    y = y * sd[:, None, None, None] + loc[:, None, None, None]
    return y.transpose(0, 2, 1, 3).reshape(R, Q, L)


def rel_err(a, e):
    return np.abs(a - e).max() / max(np.abs(e).max(), 1e-6)


@pytest.mark.parametrize("qk_norm", [True, False])
def test_oracle_matches_numpy_restatement(qk_norm):
    c = tiny_config(use_qk_norm=qk_norm)
    w = tx.random_checkpoint(c, seed=7, norm_jitter=0.1)
    b = mixed_batch(c)
    got = otx.Model(c, w).forward(b, nthreads=2)
    exp = numpy_forward(c, w, b)
    assert got.shape == (b.rows, c.num_quantiles, c.padded_length)
    for q in range(c.num_quantiles):
        assert rel_err(got[:, q], exp[:, q]) < 1e-4, f"quantile {q}: {rel_err(got[:, q], exp[:, q]):.3e}"


def test_structure_lists():
    c = tiny_config()
    b = mixed_batch(c)
    st = tx.structure(c, b)
    assert st.known.tolist() == [4]
    assert st.kept.tolist() == [2, 3, 4]
    assert st.group_start.tolist() == [0, 0, 0] and st.group_end.tolist() == [3, 3, 3]
    assert st.kept_target.tolist() == [1, 0, 0]
    bad = tx.ModelBatch(b.x, np.asarray([0, 1, 0, 2, 2, 3], np.float32), b.target)
    with pytest.raises(ValueError, match="contiguous"):
        tx.structure(c, bad)


def test_config4_shapes_and_json_round_trip():
    c = tx.config4()
    assert c.num_patches == 64 and c.mlstm_qk_dim == 256 and c.ffn_dim == 1408
    assert c.recipe == [0, 0, 0, 1] * 3
    c2 = tx.TiRex2Config.from_json(c.to_json())
    assert c2 == c
    shapes = tx.weight_shapes(c)
    assert shapes["stack.3.time_mixer.fwd_cell._recurrent_kernel_"] == (4, 128, 4, 128)
    assert shapes["stack.0.time_mixer.ffn.proj_up_gate.weight"] == (1408, 512)
    assert shapes["output_patch_embedding.output_layer.weight"] == (9 * 32, 2048)
