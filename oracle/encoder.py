"""Encoder-step ops, restated in NumPy (TEST INFRASTRUCTURE ONLY).

Forward functions round to bfloat16 at the reference's cast points; backward
functions are analytic FP64 derivatives evaluated at the same bf16 inputs
(checked against the kernels with the gradient tolerance).

  rms_norm        kernels/normalization.py:7-22 (+ the bf16 residual add of
                  models/lfm2_5/encoder.py:64-110 and the row mask of
                  layers/convolution.py:29-37)
  qknorm_rope     layers/attention.py:61-77 (per-head q/k RMSNorm) and
                  kernels/rotary.py:7-39
  gated_conv      models/lfm2_5/encoder.py:76-86, kernels/bidirectional.py:38-58
  embed           models/lfm2_5/encoder.py:231 (JAX gathers clamp indices)
  head_loss       a token classification head (full_linear, kernels/linear.py:7-13)
                  with a summed cross-entropy and a valid-token count; the
                  reference's encoder ships no head, so this loss is this
                  build's definition for the training step.

Paths are inside src/minifield_training/ of the reference project.
"""

import numpy as np

from .bf16 import round_bf16 as rb

F = np.float32


def rms_norm(x, w, eps, residual=None, mask=None):
    """(sum, y, rstd): sum = bf16(x + residual) or x; y = bf16(bf16(sum*r) * bf16(w)) * mask."""
    x = rb(x)
    s = rb(x + rb(residual)) if residual is not None else x
    v = s.astype(F)
    r = (F(1) / np.sqrt(np.mean(v * v, axis=-1, keepdims=True, dtype=F) + F(eps))).astype(F)
    y = rb(rb(v * r) * rb(np.asarray(w, F)))
    if mask is not None:
        y = y * np.asarray(mask, F).reshape(*y.shape[:-1], 1)
    return s, y, r[..., 0]


def rms_norm_bwd(s, w, dy, dres=None, mask=None, eps=1e-5):
    """(dx, dw) of y = rms_norm(s) (FP64 at the bf16 input s)."""
    s = np.asarray(s, np.float64)
    dy = np.asarray(dy, np.float64)
    if mask is not None:
        dy = dy * np.asarray(mask, np.float64).reshape(*dy.shape[:-1], 1)
    c = s.shape[-1]
    r = 1.0 / np.sqrt(np.mean(s * s, axis=-1, keepdims=True) + eps)
    n = s * r
    wb = rb(np.asarray(w, F)).astype(np.float64)
    dn = dy * wb
    dx = r * (dn - n * np.mean(dn * n, axis=-1, keepdims=True))
    if dres is not None:
        dx = dx + np.asarray(dres, np.float64)
    dw = np.sum((dy * rb(n.astype(F)).astype(np.float64)).reshape(-1, c), axis=0)
    return dx, dw


def rope_freqs(theta, d=64):
    """theta ** (-arange(0, d, 2) / d) in float32 (rotary.py:31-33)."""
    return (F(theta) ** (-np.arange(0, d, 2, dtype=F) / F(d))).astype(F)


def _rope_tables(positions, freqs):
    ang = (np.asarray(positions, F)[..., None] * freqs[None, :]).astype(F)  # [M, 32]
    ang = np.concatenate((ang, ang), axis=-1)
    return rb(np.cos(ang).astype(F)), rb(np.sin(ang).astype(F))


def qknorm_rope(qkv, wq, wk, positions, freqs, h, hk, eps):
    """(q [M,H,64], k [M,Hk,64], v [M,Hk,64]) from the fused projection [M, (H+2Hk)*64]."""
    m = qkv.shape[0]
    x = rb(qkv).reshape(m, h + 2 * hk, 64)
    cos, sin = _rope_tables(positions, freqs)

    def head(t, w):
        _, n, _ = rms_norm(t, w, eps)
        rot = np.concatenate((-n[..., 32:], n[..., :32]), axis=-1)
        return rb(rb(n * cos[:, None, :]) + rb(rot * sin[:, None, :]))

    return head(x[:, :h], wq), head(x[:, h:h + hk], wk), x[:, h + hk:]


def qknorm_rope_bwd(qkv, wq, wk, positions, freqs, h, hk, dq, dk, dv, eps):
    """(d_qkv [M, (H+2Hk)*64], dwq, dwk) in FP64."""
    m = qkv.shape[0]
    x = rb(qkv).reshape(m, h + 2 * hk, 64).astype(np.float64)
    cos, sin = (t.astype(np.float64) for t in _rope_tables(positions, freqs))

    def head(t, w, g):
        g = np.asarray(g, np.float64)
        gs = g * sin[:, None, :]
        dn = g * cos[:, None, :] + np.concatenate((gs[..., 32:], -gs[..., :32]), axis=-1)
        return rms_norm_bwd(t, w, dn, eps=eps)

    dxq, dwq = head(x[:, :h], wq, dq)
    dxk, dwk = head(x[:, h:h + hk], wk, dk)
    d = np.concatenate((dxq, dxk, np.asarray(dv, np.float64)), axis=1).reshape(m, -1)
    return d, dwq, dwk


def _same(seg, t_len):
    """same[m, i]: token m reads neighbour m + i - 1 (same nonzero segment, same row)."""
    seg = np.asarray(seg).reshape(-1, t_len)
    b = seg.shape[0]
    out = np.zeros((b, t_len, 3), bool)
    for i, off in enumerate((-1, 0, 1)):
        nb = np.zeros_like(seg)
        if off < 0:
            nb[:, 1:] = seg[:, :-1]
        elif off > 0:
            nb[:, :-1] = seg[:, 1:]
        else:
            nb = seg
        out[:, :, i] = (nb == seg) & (seg != 0)
    return out.reshape(-1, 3)


def _shift(a, off, t_len):
    """a[m + off] within rows of t_len (zeros past the row edge)."""
    a3 = a.reshape(-1, t_len, a.shape[-1])
    out = np.zeros_like(a3)
    if off < 0:
        out[:, 1:] = a3[:, :-1]
    elif off > 0:
        out[:, :-1] = a3[:, 1:]
    else:
        out = a3
    return out.reshape(a.shape)


def gated_conv(bcx, taps, seg, t_len):
    """mixed [M, C] = c * conv(b * values) with the reference's bf16 rounding order."""
    bcx = rb(bcx)
    c = bcx.shape[1] // 3
    b, cg, vals = bcx[:, :c], bcx[:, c:2 * c], bcx[:, 2 * c:]
    gated = rb(b * vals)
    tb = rb(np.asarray(taps, F))
    same = _same(seg, t_len)
    result = np.zeros_like(gated)
    for i, off in enumerate((-1, 0, 1)):
        tap = rb(_shift(gated, off, t_len) * tb[:, i][None, :])
        tap = rb(tap * same[:, i:i + 1].astype(F))
        result = rb(result + tap)
    return rb(cg * result)


def gated_conv_bwd(bcx, taps, seg, t_len, dmixed):
    """(d_bcx [M, 3C], d_taps [C, 3]) in FP64 at the bf16 inputs."""
    bcx = rb(bcx).astype(np.float64)
    c = bcx.shape[1] // 3
    b, cg, vals = bcx[:, :c], bcx[:, c:2 * c], bcx[:, 2 * c:]
    gated = rb((b * vals).astype(F)).astype(np.float64)
    tb = rb(np.asarray(taps, F)).astype(np.float64)
    same = _same(seg, t_len).astype(np.float64)
    dm = np.asarray(dmixed, np.float64)
    # d_c multiplies the forward's own bf16-accumulated conv (the value the
    # reference's autodiff sees), not an exact sum.
    conv = np.zeros_like(gated)
    for i, off in enumerate((-1, 0, 1)):
        tap = rb((_shift(gated, off, t_len) * tb[:, i][None, :]).astype(F)).astype(np.float64)
        conv = rb((conv + tap * same[:, i:i + 1]).astype(F)).astype(np.float64)
    dconv = dm * cg
    dgated = np.zeros_like(gated)
    dtaps = np.zeros((c, 3))
    for i, off in enumerate((-1, 0, 1)):
        contrib = dconv * same[:, i:i + 1]
        dgated += _shift(contrib, -off, t_len) * tb[:, i][None, :]
        dtaps[:, i] = np.sum(contrib * _shift(gated, off, t_len), axis=0)
    return np.concatenate((dgated * vals, dm * conv, dgated * b), axis=1), dtaps


def embed(table, ids):
    """bf16 rows of the FP32 table at clamped ids."""
    table = np.asarray(table, F)
    return rb(table[np.clip(np.asarray(ids), 0, table.shape[0] - 1)])


def head_loss(encoded, w, labels, valid):
    """(loss_sum, count, d_encoded, d_w) of the summed token cross-entropy."""
    e = rb(encoded).astype(np.float64)
    wb = rb(np.asarray(w, F)).astype(np.float64)
    logits = rb((e @ wb.T).astype(F)).astype(np.float64)
    mx = logits.max(axis=-1, keepdims=True)
    p = np.exp(logits - mx)
    se = p.sum(axis=-1, keepdims=True)
    p /= se
    k = w.shape[0]
    y = np.clip(np.asarray(labels), 0, k - 1)
    ok = np.asarray(valid) != 0
    lse = (mx + np.log(se))[:, 0]
    loss = float(np.sum((lse - logits[np.arange(len(y)), y])[ok]))
    dl = (p - np.eye(k)[y]) * ok[:, None]
    dl = rb(dl.astype(F)).astype(np.float64)
    return loss, float(ok.sum()), dl @ wb, dl.T @ e
