"""One cached decode step of the LFM2.5 causal decoder, FP64 with bf16 rounding points (TEST INFRASTRUCTURE ONLY).

Restates (paths inside src/minifield_training/):

  decode_one / _decode_one_impl  models/lfm2_5/decode.py:325-364, 419-466
  _decode_block                  models/lfm2_5/decode.py:225-262
  prefill / _prefill_impl        models/lfm2_5/decode.py:265-312, 373-416
  _prefill_block                 models/lfm2_5/decode.py:183-222
  conv_block_prefix              layers/convolution.py:77-101, state_tail
                                 kernels/convolution.py:56-79
  attention_block_prefill        layers/attention.py:246-278 (causal attention,
                                 kernels/attention.py:206-222)
  conv_block_step                layers/convolution.py:153-178, 40-48
  gated conv with history        kernels/convolution.py:82-111
  attention_block_step           layers/attention.py:281-322, 61-108
  swiglu_ffn                     layers/feed_forward.py:24-35
  logits (tied head, FP32 cast)  models/lfm2_5/model.py:818-829

with the same cast conventions as oracle.encoder_step: masters cast to bf16
before each product, products rounded to bf16, RMSNorm FP32 statistics ->
bf16 -> times the bf16 gain, attention probabilities rounded to the value
dtype, silu(gate) * up rounded once, the causal conv's tap products and
partial sums each rounded. A state is a dict: "pos" (the position written
this step, = valid length before it), "k"/"v" (per layer [B, cap, Hk, D] or
None) and "hist" (per layer [B, 2, C] or None), values bf16-exact in float64.
"""

import numpy as np
import torch

from .encoder_step import D, _linear, _rms, _rope, rb


def parameter_shapes(cfg) -> dict:
    """Reference parameter names and shapes of the decoder (models/lfm2_5/model.py:127-166)."""
    c, f, kv = cfg.hidden, cfg.ffn, cfg.kv_heads * cfg.head_dim
    shapes = {"model.embed_tokens.weight": (cfg.vocab, c), "model.embedding_norm.weight": (c,)}
    for i, kind in enumerate(cfg.layer_types):
        p = f"model.layers.{i}."
        shapes.update({p + "operator_norm.weight": (c,), p + "ffn_norm.weight": (c,),
                       p + "feed_forward.w1.weight": (f, c), p + "feed_forward.w3.weight": (f, c),
                       p + "feed_forward.w2.weight": (c, f)})
        if kind == "conv":
            shapes.update({p + "conv.in_proj.weight": (3 * c, c), p + "conv.out_proj.weight": (c, c),
                           p + "conv.conv.weight": (c, 1, cfg.conv_kernel)})
        else:
            shapes.update({p + "self_attn.q_proj.weight": (cfg.heads * cfg.head_dim, c),
                           p + "self_attn.k_proj.weight": (kv, c), p + "self_attn.v_proj.weight": (kv, c),
                           p + "self_attn.out_proj.weight": (c, cfg.heads * cfg.head_dim),
                           p + "self_attn.q_layernorm.weight": (cfg.head_dim,),
                           p + "self_attn.k_layernorm.weight": (cfg.head_dim,)})
    return shapes


def new_state(cfg, batch: int, capacity: int) -> dict:
    """Zeroed caches (decode.py:75-134)."""
    k, v, h = [], [], []
    for kind in cfg.layer_types:
        if kind == "full_attention":
            k.append(np.zeros((batch, capacity, cfg.kv_heads, cfg.head_dim)))
            v.append(np.zeros((batch, capacity, cfg.kv_heads, cfg.head_dim)))
            h.append(None)
        else:
            k.append(None)
            v.append(None)
            h.append(np.zeros((batch, cfg.conv_kernel - 1, cfg.hidden)))
    return {"pos": 0, "k": k, "v": v, "hist": h}


def _w(t):
    return rb(t)


def _ffn_tail(P, p, x, r, eps):
    """x + r, then the residual SwiGLU (layers/feed_forward.py:24-35)."""
    x = rb(x + r)
    h2 = _rms(x, P[p + "ffn_norm.weight"], eps)
    gg = _linear(h2, _w(P[p + "feed_forward.w1.weight"]))
    uu = _linear(h2, _w(P[p + "feed_forward.w3.weight"]))
    a = rb(gg * torch.sigmoid(gg) * uu)
    return rb(x + _linear(a, _w(P[p + "feed_forward.w2.weight"])))


def _attention_block_rows(cfg, P, p, x, b, t):
    """The causal attention block (layers/attention.py:111-138) over T tokens per row at positions 0..T-1:
    (block output rows [B*T, C], RoPE'd keys [B, T, Hk, D], values [B, T, Hk, D])."""
    eps, hd = cfg.norm_eps, cfg.head_dim
    positions = np.tile(np.arange(t, dtype=np.int32), b)
    h = _rms(x, P[p + "operator_norm.weight"], eps)
    q = _linear(h, _w(P[p + "self_attn.q_proj.weight"])).reshape(b * t, cfg.heads, hd)
    k = _linear(h, _w(P[p + "self_attn.k_proj.weight"])).reshape(b * t, cfg.kv_heads, hd)
    v = _linear(h, _w(P[p + "self_attn.v_proj.weight"])).reshape(b * t, cfg.kv_heads, hd)
    q = _rope(_rms(q, P[p + "self_attn.q_layernorm.weight"], eps), positions, cfg.rope_theta, hd)
    k = _rope(_rms(k, P[p + "self_attn.k_layernorm.weight"], eps), positions, cfg.rope_theta, hd)
    group = cfg.heads // cfg.kv_heads
    q4 = q.reshape(b, t, cfg.heads, hd)
    k4 = k.reshape(b, t, cfg.kv_heads, hd)
    v4 = v.reshape(b, t, cfg.kv_heads, hd)
    kk = torch.repeat_interleave(k4, group, dim=2)
    vv = torch.repeat_interleave(v4, group, dim=2)
    s = torch.einsum("bthd,bshd->bhts", q4, kk) * hd ** -0.5
    causal = torch.tril(torch.ones(t, t, dtype=torch.bool))
    s = torch.where(causal, s, torch.full_like(s, -1e300))
    prob = rb(torch.softmax(s, dim=-1))
    o = rb(torch.einsum("bhts,bshd->bthd", prob, vv))
    r = _linear(o.reshape(b * t, cfg.heads * hd), _w(P[p + "self_attn.out_proj.weight"]))
    return _ffn_tail(P, p, x, r, eps), k4, v4


def attention_block(cfg, weights: dict, x):
    """One causal attention block over x [B, T, C] (bf16-exact values), every token valid, positions 0..T-1:
    (y [B, T, C], keys [B, T, Hk, D], values [B, T, Hk, D]) in float64 holding bf16-exact values.

    ``weights`` uses the decoder's per-layer names without the layer prefix
    ("operator_norm.weight", "self_attn.q_proj.weight", ..., "ffn_norm.weight",
    "feed_forward.w1.weight" (gate), "feed_forward.w3.weight" (up),
    "feed_forward.w2.weight" (down)).
    """
    with torch.no_grad():
        P = {n: torch.tensor(np.asarray(v, np.float64), dtype=D) for n, v in weights.items()}
        x = np.asarray(x, np.float64)
        b, t, c = x.shape
        y, k4, v4 = _attention_block_rows(cfg, P, "", rb(torch.from_numpy(x.reshape(b * t, c))), b, t)
        return y.reshape(b, t, c).numpy(), k4.numpy(), v4.numpy()


def prefill(cfg, params: dict, ids, capacity: int):
    """(logits [B, V] of the last prompt token, state after the prompt) for a fresh state.

    Every row holds the same T valid tokens (the reference's scalar
    valid_length); its power-of-two padding bucket only adds masked tokens
    after them, which causal attention and the causal convolution never read,
    so the oracle runs on the T tokens themselves.
    """
    with torch.no_grad():
        P = {n: torch.tensor(np.asarray(v, np.float64), dtype=D) for n, v in params.items()}
        ids = np.asarray(ids)
        b, t = ids.shape
        if t <= 0 or t > capacity:
            raise ValueError("Prompt length must fit the cache capacity")
        eps, c = cfg.norm_eps, cfg.hidden
        x = rb(P["model.embed_tokens.weight"][torch.from_numpy(np.clip(ids, 0, cfg.vocab - 1)).long()])  # [B,T,C]
        x = x.reshape(b * t, c)
        state = new_state(cfg, b, capacity)
        state["pos"] = t
        for i, kind in enumerate(cfg.layer_types):
            p = f"model.layers.{i}."
            if kind == "conv":
                h = _rms(x, P[p + "operator_norm.weight"], eps)
                bcx = _linear(h, _w(P[p + "conv.in_proj.weight"])).reshape(b, t, 3 * c)
                gate_b, gate_c, vals = bcx[..., :c], bcx[..., c:2 * c], bcx[..., 2 * c:]
                g = rb(gate_b * vals)
                taps = rb(P[p + "conv.conv.weight"][:, 0, :])
                gp = torch.cat((torch.zeros(b, 2, c, dtype=D), g), dim=1)  # two zero columns before token 0
                acc = rb(rb(rb(gp[:, :t] * taps[:, 0]) + rb(gp[:, 1:t + 1] * taps[:, 1])) + rb(g * taps[:, 2]))
                mixed = rb(gate_c * acc).reshape(b * t, c)
                state["hist"][i] = gp[:, t:t + 2].numpy().copy()  # state_tail at length t (zeros when t == 1)
                r = _linear(mixed, _w(P[p + "conv.out_proj.weight"]))
            else:
                y, k4, v4 = _attention_block_rows(cfg, P, p, x, b, t)
                state["k"][i][:, :t] = k4.numpy()
                state["v"][i][:, :t] = v4.numpy()
                x = y
                continue
            x = _ffn_tail(P, p, x, r, eps)
        last = x.reshape(b, t, c)[:, t - 1]
        enc = _rms(last, P["model.embedding_norm.weight"], eps)
        return _linear(enc, _w(P["model.embed_tokens.weight"])).numpy(), state


def decode_one(cfg, params: dict, ids, state: dict):
    """(logits [B, V] float64 (bf16-exact values), new state) for one token per row."""
    with torch.no_grad():
        P = {n: torch.tensor(np.asarray(v, np.float64), dtype=D) for n, v in params.items()}
        ids = np.asarray(ids).reshape(-1)
        b = ids.shape[0]
        pos = int(state["pos"])
        eps, hd = cfg.norm_eps, cfg.head_dim
        x = rb(P["model.embed_tokens.weight"][torch.from_numpy(np.clip(ids, 0, cfg.vocab - 1)).long()])
        new = {"pos": pos + 1, "k": [], "v": [], "hist": []}
        for i, kind in enumerate(cfg.layer_types):
            p = f"model.layers.{i}."
            h = _rms(x, P[p + "operator_norm.weight"], eps)
            if kind == "conv":
                c = cfg.hidden
                bcx = _linear(h, _w(P[p + "conv.in_proj.weight"]))
                gate_b, gate_c, vals = bcx[:, :c], bcx[:, c:2 * c], bcx[:, 2 * c:]
                g = rb(gate_b * vals)
                taps = rb(P[p + "conv.conv.weight"][:, 0, :])
                hist = torch.tensor(state["hist"][i], dtype=D)
                acc = rb(rb(rb(hist[:, 0] * taps[:, 0]) + rb(hist[:, 1] * taps[:, 1])) + rb(g * taps[:, 2]))
                mixed = rb(gate_c * acc)
                new["hist"].append(torch.stack((hist[:, 1], g), dim=1).numpy())
                new["k"].append(None)
                new["v"].append(None)
                r = _linear(mixed, _w(P[p + "conv.out_proj.weight"]))
            else:
                q = _linear(h, _w(P[p + "self_attn.q_proj.weight"])).reshape(b, cfg.heads, hd)
                k = _linear(h, _w(P[p + "self_attn.k_proj.weight"])).reshape(b, cfg.kv_heads, hd)
                v = _linear(h, _w(P[p + "self_attn.v_proj.weight"])).reshape(b, cfg.kv_heads, hd)
                positions = np.full(b, pos, np.int32)
                q = _rope(_rms(q, P[p + "self_attn.q_layernorm.weight"], eps), positions, cfg.rope_theta, hd)
                k = _rope(_rms(k, P[p + "self_attn.k_layernorm.weight"], eps), positions, cfg.rope_theta, hd)
                kc = torch.tensor(state["k"][i], dtype=D).clone()
                vc = torch.tensor(state["v"][i], dtype=D).clone()
                kc[:, pos], vc[:, pos] = k, v
                group = cfg.heads // cfg.kv_heads
                kk = torch.repeat_interleave(kc[:, :pos + 1], group, dim=2)  # [B, L, H, D]
                vv = torch.repeat_interleave(vc[:, :pos + 1], group, dim=2)
                s = torch.einsum("bhd,blhd->bhl", q, kk) * hd ** -0.5
                prob = rb(torch.softmax(s, dim=-1))
                o = rb(torch.einsum("bhl,blhd->bhd", prob, vv))
                new["k"].append(kc.numpy())
                new["v"].append(vc.numpy())
                new["hist"].append(None)
                r = _linear(o.reshape(b, cfg.heads * hd), _w(P[p + "self_attn.out_proj.weight"]))
            x = _ffn_tail(P, p, x, r, eps)
        enc = _rms(x, P["model.embedding_norm.weight"], eps)
        logits = _linear(enc, _w(P["model.embed_tokens.weight"]))
        return logits.numpy(), new
