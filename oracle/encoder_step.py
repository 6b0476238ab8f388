"""Encoder training-step loss and gradients, restated with FP64 autograd (TEST INFRASTRUCTURE ONLY).

A floating-point composition, so it is written with torch on the CPU (float64
tensors, autograd) instead of hand-derived NumPy backward passes. bf16 casts
are emulated with round trips through torch.bfloat16 at the reference's cast
points, and the gradients are the exact FP64 derivatives of that rounded
forward (the casts pass cotangents through unrounded), so the oracle carries
no backward rounding noise of its own. Follows (paths inside
src/minifield_training/):

  encode, _block         models/lfm2_5/encoder.py:64-240
  rms_norm               kernels/normalization.py:7-22
  conv_input_projection  layers/convolution.py:29-37
  centered_convolution   kernels/bidirectional.py:38-58
  project_qkv, rotary    layers/attention.py:61-77, kernels/rotary.py:7-39
  bidirectional attention kernels/bidirectional.py:7-35 (softmax FP32, probabilities cast
                         to the value dtype, inactive queries zeroed)
  swiglu_ffn             layers/feed_forward.py:24-35 (silu(gate) * up rounded once)
  full_linear            kernels/linear.py:7-13 (master cast to bf16 before the product)
  QAT (STE)              strategies/quantization.py:114-126 with oracle.quant's int8 kinds

plus this build's token classification head with a summed cross-entropy over
valid tokens (the reference's encoder has no head).
"""

import numpy as np
import torch

from . import quant

# Arithmetic type of the restatement: FP64 for parity (the default); the
# bench's CPU baseline times the same graph in FP32.
D = torch.float64
_DTYPE = [D]


def _dt():
    return _DTYPE[0]


class _RoundBf16(torch.autograd.Function):
    """bf16 rounding in the forward, the exact (unrounded) gradient in the backward."""

    @staticmethod
    def forward(ctx, t):
        return t.to(torch.bfloat16).to(_dt())

    @staticmethod
    def backward(ctx, g):
        return g


_ROUND = [True]


def rb(t):
    return _RoundBf16.apply(t) if _ROUND[0] else t


def _rms(x, w, eps, mask=None):
    r = torch.rsqrt(torch.mean(x * x, dim=-1, keepdim=True) + eps)
    y = rb(rb(x * r) * rb(w))
    return y * mask[..., None] if mask is not None else y


def _linear(x, w_eff):
    return rb(x @ w_eff.T)


def _qat(w, kind):
    """Effective weight with the straight-through gradient masked by STE."""
    wn = w.detach().numpy().astype(np.float32)
    _, _, ste, dec = quant.fake_quant(wn, kind)
    dec = torch.from_numpy(np.asarray(dec, np.float64)).to(_dt())
    ste = torch.from_numpy(np.asarray(ste, np.float64)).to(_dt())
    return rb(dec) + (w - w.detach()) * ste


def _rope(x, positions, theta, head_dim):
    freqs = torch.from_numpy((np.float32(theta) ** (-np.arange(0, head_dim, 2, dtype=np.float32) /
                                                    np.float32(head_dim))).astype(np.float32))
    ang = (torch.from_numpy(np.asarray(positions, np.float32))[:, None] * freqs[None, :]).to(torch.float32)
    ang = torch.cat((ang, ang), dim=-1)
    cos, sin = rb(torch.cos(ang).to(_dt())), rb(torch.sin(ang).to(_dt()))
    rot = torch.cat((-x[..., head_dim // 2:], x[..., :head_dim // 2]), dim=-1)
    return rb(rb(x * cos[:, None, :]) + rb(rot * sin[:, None, :]))


def _conv(bcx, taps, seg, t_len):
    c = bcx.shape[1] // 3
    b, cg, vals = bcx[:, :c], bcx[:, c:2 * c], bcx[:, 2 * c:]
    gated = rb(b * vals)
    tb = rb(taps)
    seg2 = torch.from_numpy(np.asarray(seg)).reshape(-1, t_len)
    g3 = gated.reshape(-1, t_len, c)
    result = torch.zeros_like(g3)
    for i, off in enumerate((-1, 0, 1)):
        sh = torch.zeros_like(g3)
        nb = torch.zeros_like(seg2)
        if off < 0:
            sh[:, 1:] = g3[:, :-1]
            nb[:, 1:] = seg2[:, :-1]
        elif off > 0:
            sh[:, :-1] = g3[:, 1:]
            nb[:, :-1] = seg2[:, 1:]
        else:
            sh, nb = g3, seg2
        same = ((nb == seg2) & (seg2 != 0)).to(_dt())[..., None]
        tap = rb(rb(sh * tb[:, i]) * same)
        result = rb(result + tap)
    return rb(cg * result.reshape(-1, c))


def _attention(q, k, v, seg, rows, t_len, heads, kv_heads):
    hd = q.shape[-1]
    q4 = q.reshape(rows, t_len, heads, hd)
    k4 = torch.repeat_interleave(k.reshape(rows, t_len, kv_heads, hd), heads // kv_heads, dim=2)
    v4 = torch.repeat_interleave(v.reshape(rows, t_len, kv_heads, hd), heads // kv_heads, dim=2)
    s = torch.einsum("bthd,bshd->bhts", q4, k4) * hd ** -0.5
    seg2 = torch.from_numpy(np.asarray(seg)).reshape(rows, t_len)
    active = seg2 != 0
    valid = (seg2[:, :, None] == seg2[:, None, :]) & active[:, :, None] & active[:, None, :]
    s = torch.where(valid[:, None], s, torch.full_like(s, torch.finfo(s.dtype).min))
    p = torch.softmax(s, dim=-1)
    p = torch.where(active[:, None, :, None], p, torch.zeros_like(p))
    o = rb(torch.einsum("bhts,bshd->bthd", rb(p), v4))
    o = o * active[:, :, None, None]
    return o.reshape(rows * t_len, heads * hd)


def loss_and_grads(cfg, params: dict, ids, mask, seg, pos, labels, rows, bf16=True, compute_dtype=torch.float64):
    """(loss_sum, count, {trainable name: FP64 gradient}) for one local batch.

    ``bf16=False`` drops every bf16 cast (the FP64 version of the same model,
    fake-quantized weights included): the exact path a bf16 run is compared to.
    ``compute_dtype=torch.float32`` runs the same graph in FP32 (CPU timing
    only; parity uses FP64).
    """
    _ROUND[0] = bool(bf16)
    _DTYPE[0] = compute_dtype
    try:
        return _loss_and_grads(cfg, params, ids, mask, seg, pos, labels, rows)
    finally:
        _ROUND[0] = True
        _DTYPE[0] = torch.float64


def _loss_and_grads(cfg, params, ids, mask, seg, pos, labels, rows):
    t_len = cfg.length
    ids, mask, seg, pos, labels = (np.asarray(a).reshape(-1) for a in (ids, mask, seg, pos, labels))
    leaves = {n: torch.tensor(np.asarray(v), dtype=_dt(), requires_grad=n != "lfm2.embed_tokens.weight")
              for n, v in params.items()}
    maskt = torch.from_numpy(mask.astype(np.float64)).to(_dt())
    table = leaves["lfm2.embed_tokens.weight"]
    x = rb(table[torch.from_numpy(np.clip(ids, 0, cfg.vocab - 1)).long()])
    c, eps = cfg.hidden, cfg.norm_eps
    for i, kind in enumerate(cfg.layer_types):
        p = f"lfm2.layers.{i}."
        eff = lambda n: _qat(leaves[p + n], cfg.quant)
        h = _rms(x, leaves[p + "operator_norm.weight"], eps, maskt if kind == "conv" else None)
        if kind == "conv":
            bcx = _linear(h, eff("conv.in_proj.weight"))
            mixed = _conv(bcx, leaves[p + "conv.conv.weight"][:, 0, :], seg, t_len)
            r = _linear(mixed, eff("conv.out_proj.weight"))
        else:
            hd = cfg.head_dim
            q = _linear(h, eff("self_attn.q_proj.weight")).reshape(-1, cfg.heads, hd)
            k = _linear(h, eff("self_attn.k_proj.weight")).reshape(-1, cfg.kv_heads, hd)
            v = _linear(h, eff("self_attn.v_proj.weight")).reshape(-1, cfg.kv_heads, hd)
            q = _rope(_rms(q, leaves[p + "self_attn.q_layernorm.weight"], eps), pos, cfg.rope_theta, hd)
            k = _rope(_rms(k, leaves[p + "self_attn.k_layernorm.weight"], eps), pos, cfg.rope_theta, hd)
            o = _attention(q, k, v, seg, rows, t_len, cfg.heads, cfg.kv_heads)
            r = _linear(o, eff("self_attn.out_proj.weight"))
        x = rb(x + r)
        h2 = _rms(x, leaves[p + "ffn_norm.weight"], eps)
        g = _linear(h2, eff("feed_forward.w1.weight"))
        u = _linear(h2, eff("feed_forward.w3.weight"))
        a = rb(g * torch.sigmoid(g) * u)
        x = rb(x + _linear(a, eff("feed_forward.w2.weight")))
    enc = _rms(x, leaves["lfm2.embedding_norm.weight"], eps, maskt)
    logits = _linear(enc, rb(leaves["head.weight"]))
    lse = torch.logsumexp(logits, dim=-1)
    lab = torch.from_numpy(np.clip(labels, 0, cfg.classes - 1)).long()
    per = lse - logits[torch.arange(len(lab)), lab]
    valid = torch.from_numpy(mask != 0)
    loss = torch.sum(per[valid])
    loss.backward()
    grads = {n: t.grad.numpy() for n, t in leaves.items() if t.requires_grad}
    return float(loss.detach()), float(valid.sum()), grads
