"""Fixed-capacity cached decoding of the LFM2.5 causal decoder on the B200 kernels.

Mirrors src/minifield_training/models/lfm2_5/decode.py: ``new_state`` (:75-134)
allocates zeroed per-layer caches (attention K/V [B, capacity, Hk, 64] bf16,
conv history [B, 2, C] bf16); ``Decoder.prefill`` (:373-416) runs a prompt of
T tokens per row through every block (:183-222), fills the caches and returns
the FP32 logits of the last prompt token; ``Decoder.decode_one`` (:419-466)
runs one token per row through every block (:225-262) and returns FP32 logits
of the tied head (model.py:818-829), advancing the state's valid length.

Prefill, per block over the B*T prompt tokens:

  conv       RMSNorm -> in_proj GEMM -> mfb_conv_causal (zero history in, the
             continuation history out) -> out_proj GEMM
  attention  RMSNorm -> fused q|k|v GEMM -> q/k RMSNorm + RoPE at 0..T-1 ->
             causal mfb_attn_fwd -> K/V rows copied into the cache
             (mfb_memcpy2d_d2d) -> out_proj GEMM

The reference pads the prompt to a power-of-two bucket (decode.py:63-67);
the padded tokens sit after every valid one and are masked, so causal
attention and the causal convolution never read them and the prompt runs
at its own length here. Decode, per block:

  conv       RMSNorm -> in_proj GEMM -> mfb_conv_step (gated causal conv over
             the history, history shifted in place) -> out_proj GEMM
  attention  RMSNorm -> fused q|k|v GEMM -> q/k RMSNorm + RoPE at the position
             -> mfb_decode_attn (cache append at the position, split-K
             attention over the valid length) -> out_proj GEMM
  then       residual + RMSNorm (one kernel) -> fused w1|w3 GEMM -> SwiGLU ->
             w2 GEMM, the residual folded into the next block's norm.

The masters are cast to bf16 once at construction (full_linear's cast,
kernels/linear.py:11); the q|k|v and w1|w3 products are single GEMMs over
concatenated rows.
"""

import ctypes

import numpy as np

from .. import _lib
from ..device import DeviceArray
from .encoder import _fwd, rope_freqs

P = ctypes.c_void_p


class DecodeOverflow(ValueError):
    """A token would be written past the fixed cache capacity (decode.py:22-23)."""


def parameter_shapes(cfg) -> dict:
    """Reference decoder parameter names and shapes (models/lfm2_5/model.py:127-166)."""
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


def init_parameters(cfg, seed: int = 0) -> dict:
    """Random init: N(0, 0.02) for matrices, taps and the embedding table; ones for norm gains."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in parameter_shapes(cfg).items():
        if name.endswith("norm.weight") or name.endswith("layernorm.weight"):
            out[name] = np.ones(shape, np.float32)
        else:
            out[name] = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
    return out


class DecodeState:
    """Device caches of one prompt batch plus its logical position (decode.py:34-41).

    ``keys`` / ``values`` / ``history`` are per-layer lists (None where the
    layer has no such cache); ``valid_length`` is the number of written
    positions, which is also the position the next token takes.
    """

    def __init__(self, cfg, batch_size: int, capacity: int):
        if isinstance(capacity, bool) or not isinstance(capacity, int) or capacity <= 0 or capacity & (capacity - 1):
            raise ValueError("Cache capacity must be a positive power of two")
        if isinstance(batch_size, bool) or not isinstance(batch_size, int) or batch_size <= 0:
            raise ValueError("batch_size must be a positive integer")
        self.cfg, self.batch, self.capacity, self.valid_length = cfg, batch_size, capacity, 0
        self.keys, self.values, self.history = [], [], []
        for kind in cfg.layer_types:
            if kind == "full_attention":
                shape = (batch_size, capacity, cfg.kv_heads, cfg.head_dim)
                self.keys.append(DeviceArray.zeros(shape, "bfloat16"))
                self.values.append(DeviceArray.zeros(shape, "bfloat16"))
                self.history.append(None)
            else:
                self.keys.append(None)
                self.values.append(None)
                self.history.append(DeviceArray.zeros((batch_size, cfg.conv_kernel - 1, cfg.hidden), "bfloat16"))


def new_state(cfg, batch_size: int, capacity: int) -> DecodeState:
    """Zeroed fixed-capacity state (decode.py:75-134)."""
    return DecodeState(cfg, batch_size, capacity)


class Decoder:
    """Device weights of the decoder and the single-token step over a DecodeState."""

    def __init__(self, cfg, parameters: dict, *, stream=None):
        if cfg.head_dim != 64 or cfg.conv_kernel != 3:
            raise ValueError("this build decodes head_dim 64 with a 3-tap convolution")
        shapes = parameter_shapes(cfg)
        if set(parameters) != set(shapes):
            raise ValueError("Decoder parameter tree mismatch")
        for name, shape in shapes.items():
            if tuple(np.shape(parameters[name])) != shape:
                raise ValueError(f"Decoder parameter shape mismatch: {name}")
        self.cfg, self.stream = cfg, stream
        f32 = lambda a: DeviceArray.from_numpy(np.ascontiguousarray(a, np.float32), "float32")  # noqa: E731

        def bf16(*names):  # rows of the named matrices, concatenated, cast to bf16 on the device
            host = np.ascontiguousarray(np.concatenate([np.asarray(parameters[n], np.float32) for n in names]))
            src = f32(host)
            out = DeviceArray(host.shape, "bfloat16")
            _lib.call("mfb_cast_f32_bf16", P(src.ptr), P(out.ptr), host.size, None)
            return out

        self.embed = f32(parameters["model.embed_tokens.weight"])
        self.head = bf16("model.embed_tokens.weight")
        self.final_norm = f32(parameters["model.embedding_norm.weight"])
        self.freqs = DeviceArray.from_numpy(rope_freqs(cfg.rope_theta, cfg.head_dim), "float32")
        self.layers = []
        for i, kind in enumerate(cfg.layer_types):
            p = f"model.layers.{i}."
            L = {"kind": kind, "op_norm": f32(parameters[p + "operator_norm.weight"]),
                 "ffn_norm": f32(parameters[p + "ffn_norm.weight"]),
                 "w13": bf16(p + "feed_forward.w1.weight", p + "feed_forward.w3.weight"),
                 "w2": bf16(p + "feed_forward.w2.weight")}
            if kind == "conv":
                L["w_in"] = bf16(p + "conv.in_proj.weight")
                L["w_out"] = bf16(p + "conv.out_proj.weight")
                L["taps"] = f32(np.asarray(parameters[p + "conv.conv.weight"], np.float32)[:, 0, :])
            else:
                L["w_in"] = bf16(p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                                 p + "self_attn.v_proj.weight")
                L["w_out"] = bf16(p + "self_attn.out_proj.weight")
                L["qn"] = f32(parameters[p + "self_attn.q_layernorm.weight"])
                L["kn"] = f32(parameters[p + "self_attn.k_layernorm.weight"])
            self.layers.append(L)
        _lib.call("mfb_device_sync")
        self._scratch, self._graphs, self._prefill_scratch = {}, {}, {}

    def _buffers(self, batch: int, capacity: int):
        key = (batch, capacity)
        if key not in self._scratch:
            cfg, E = self.cfg, DeviceArray
            c, f, h, hk = cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads
            nq = (h + 2 * hk) * cfg.head_dim
            ws = _lib.lib().mfb_decode_workspace_size(batch, capacity, h, cfg.head_dim)
            gemm_ws = max(int(_lib.lib().mfb_gemm_workspace_size(batch, n, k))
                          for n, k in ((3 * c, c), (c, c), (nq, c), (c, h * cfg.head_dim), (2 * f, c), (c, f),
                                       (cfg.vocab, c)))
            meta = E((3, batch), "int32")  # ids, positions, lengths: one upload per step
            self._scratch[key] = dict(
                meta=meta, ids=meta.view(0, (batch,)), pos=meta.view(batch, (batch,)),
                lens=meta.view(2 * batch, (batch,)),
                x=E((batch, c), "bfloat16"), xb=E((batch, c), "bfloat16"), hn=E((batch, c), "bfloat16"),
                proj=E((batch, max(3 * c, nq)), "bfloat16"), mixed=E((batch, c), "bfloat16"),
                r=E((batch, c), "bfloat16"), mid=E((batch, c), "bfloat16"), h2=E((batch, c), "bfloat16"),
                gu=E((batch, 2 * f), "bfloat16"), a=E((batch, f), "bfloat16"), y=E((batch, c), "bfloat16"),
                q=E((batch, h, 64), "bfloat16"), k=E((batch, hk, 64), "bfloat16"), v=E((batch, hk, 64), "bfloat16"),
                o=E((batch, h * 64), "bfloat16"), rq=E((batch, h), "float32"), rk=E((batch, hk), "float32"),
                rstd=E((batch,), "float32"), enc=E((batch, c), "bfloat16"),
                logits16=E((batch, cfg.vocab), "bfloat16"), logits=E((batch, cfg.vocab), "float32"),
                ws=E((max(ws, 16),), "uint8"), gemm_ws=E((max(gemm_ws, 16),), "uint8"))
        return self._scratch[key]

    def _proj(self, x, w, out, m, n, k, B):
        """out[m, n] = x[m, k] . w[n, k]^T (bf16). With the batch's few rows the library runs the product
        swapped (the weight rows on the tensor core's 128-row side) and splits K through the step's
        workspace only for a deep weight (w2).

        On a created stream it launches as a programmatic dependent: the
        weight tiles stream in while the previous kernel (norm, SwiGLU, conv
        step or attention) finishes.
        """
        _lib.call("mfb_gemm_bf16_ws", P(x.ptr), _lib.MAJOR_K, k, P(w.ptr), _lib.MAJOR_K, k, P(out.ptr), n,
                  _lib.DTYPE_BF16, m, n, k, ctypes.c_float(1.0), None, _lib.GEMM_PDL if self.stream else 0,
                  P(B["gemm_ws"].ptr),
                  B["gemm_ws"].nbytes, self.stream)

    def _rms(self, x, res, w, sum_out, y, rstd, m):
        _lib.call("mfb_rmsnorm_fwd", P(x.ptr), P(res.ptr) if res is not None else None, P(w.ptr), None,
                  P(sum_out.ptr) if sum_out is not None else None, P(y.ptr), P(rstd.ptr), m, self.cfg.hidden,
                  ctypes.c_float(self.cfg.norm_eps), self.stream)

    def prefill(self, input_ids, state: DecodeState):
        """FP32 logits [B, vocab] of the token after the prompt; fills the caches of a fresh state.

        ``input_ids`` [B, T] int32; raises the reference's ValueErrors
        (decode.py:382-396) before any kernel runs.
        """
        cfg, s = self.cfg, self.stream
        if state.cfg != cfg:
            raise ValueError("Decode state does not match the decoder config")
        if state.valid_length != 0:
            raise ValueError("Prefill requires a fresh state")
        ids = np.asarray(input_ids)
        if ids.ndim != 2:
            raise ValueError("Prefill input_ids must have shape [batch, tokens]")
        b, t = ids.shape
        if t > cfg.max_position_embeddings:
            raise ValueError("Logical length exceeds model max_position_embeddings")
        if b != state.batch:
            raise ValueError("Prompt batch does not match cache batch")
        if t <= 0 or t > state.capacity:
            raise ValueError("Prompt length must fit the cache capacity")
        ids = np.ascontiguousarray(ids, np.int32)
        c, f, h, hk, hd = cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.head_dim
        m, nq, E = b * t, (h + 2 * hk) * hd, DeviceArray
        # Scratch sized for the reference's power-of-two prompt bucket
        # (decode.py:63-67) and kept per (batch, bucket): at most log2(capacity)
        # buffer sets per batch size, whatever the prompt lengths. A prompt uses
        # the leading b*t rows ([b, t] arrays stay contiguous with row stride t).
        bucket = 1 << (t - 1).bit_length()
        B = self._prefill_scratch.get((b, bucket))
        if B is None:
            mb = b * bucket
            B = dict(ids=E((mb,), "int32"), pos=E((mb,), "int32"), mask=E((mb,), "int32"),
                     qid=E((mb,), "int32"), kid=E((mb,), "int32"),
                     x=E((mb, c), "bfloat16"), xb=E((mb, c), "bfloat16"), hn=E((mb, c), "bfloat16"),
                     proj=E((mb, max(3 * c, nq)), "bfloat16"), mixed=E((mb, c), "bfloat16"),
                     r=E((mb, c), "bfloat16"), mid=E((mb, c), "bfloat16"), h2=E((mb, c), "bfloat16"),
                     gu=E((mb, 2 * f), "bfloat16"), a=E((mb, f), "bfloat16"), y=E((mb, c), "bfloat16"),
                     q=E((mb, h, hd), "bfloat16"), k=E((mb, hk, hd), "bfloat16"), v=E((mb, hk, hd), "bfloat16"),
                     o=E((mb, h * hd), "bfloat16"), lse=E((mb * h,), "float32"), rq=E((mb, h), "float32"),
                     rk=E((mb, hk), "float32"), rstd=E((mb,), "float32"), enc=E((mb, c), "bfloat16"),
                     last=E((b, c), "bfloat16"), logits16=E((b, cfg.vocab), "bfloat16"), ws=E((16,), "uint8"))
            self._prefill_scratch[(b, bucket)] = B
        need = int(_lib.lib().mfb_attn_workspace_size(b, t, t, h, hk, hd))
        if B["ws"].nbytes < need:
            B["ws"] = E((need,), "uint8")
        ws = B["ws"]
        for name, host in (("ids", ids.reshape(-1)), ("pos", np.tile(np.arange(t, dtype=np.int32), b)),
                           ("mask", np.ones((b, t), np.int32))):
            host = np.ascontiguousarray(host)
            _lib.call("mfb_memcpy_h2d", P(B[name].ptr), host.ctypes.data_as(P), host.nbytes, s)
        causal, off, pol = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _lib.call("mfb_attn_ids", _lib.MASK_CAUSAL, P(B["mask"].ptr), None, None, P(B["qid"].ptr),
                  P(B["kid"].ptr), b, t, t, 0, ctypes.byref(causal), ctypes.byref(off), ctypes.byref(pol), s)
        _lib.call("mfb_embed_gather", P(self.embed.ptr), P(B["ids"].ptr), P(B["x"].ptr), m, c, cfg.vocab, s)
        row_kv = hk * hd * 2  # bytes of one token's K (or V) row
        x, prev_mid, prev_y = B["x"], None, None
        for i, L in enumerate(self.layers):
            if prev_mid is None:
                self._rms(x, None, L["op_norm"], None, B["hn"], B["rstd"], m)
            else:
                self._rms(prev_mid, prev_y, L["op_norm"], x, B["hn"], B["rstd"], m)
            if L["kind"] == "conv":
                _fwd(B["hn"], L["w_in"], B["proj"], m, 3 * c, c, s)
                _lib.call("mfb_conv_causal", P(B["proj"].ptr), P(L["taps"].ptr), None, P(state.history[i].ptr),
                          P(B["mixed"].ptr), b, t, c, s)
                _fwd(B["mixed"], L["w_out"], B["r"], m, c, c, s)
            else:
                _fwd(B["hn"], L["w_in"], B["proj"], m, nq, c, s)
                _lib.call("mfb_qknorm_rope_fwd", P(B["proj"].ptr), nq, P(L["qn"].ptr), P(L["kn"].ptr),
                          P(B["pos"].ptr), P(self.freqs.ptr), P(B["q"].ptr), P(B["k"].ptr), P(B["v"].ptr),
                          P(B["rq"].ptr), P(B["rk"].ptr), m, h, hk, ctypes.c_float(cfg.norm_eps), s)
                _lib.call("mfb_attn_fwd", P(B["q"].ptr), P(B["k"].ptr), P(B["v"].ptr), P(B["o"].ptr),
                          P(B["lse"].ptr), P(B["qid"].ptr), P(B["kid"].ptr), b, t, t, h, hk, hd, causal.value,
                          off.value, pol.value, ctypes.c_float(hd ** -0.5), P(ws.ptr), ws.nbytes, s)
                for cache, src in ((state.keys[i], B["k"]), (state.values[i], B["v"])):
                    _lib.call("mfb_memcpy2d_d2d", P(cache.ptr), state.capacity * row_kv, P(src.ptr), t * row_kv,
                              t * row_kv, b, s)
                _fwd(B["o"], L["w_out"], B["r"], m, c, h * hd, s)
            self._rms(x, B["r"], L["ffn_norm"], B["mid"], B["h2"], B["rstd"], m)
            _fwd(B["h2"], L["w13"], B["gu"], m, 2 * f, c, s)
            _lib.call("mfb_swiglu_fwd", P(B["gu"].ptr), P(B["a"].ptr), m, f, s)
            _fwd(B["a"], L["w2"], B["y"], m, c, f, s)
            prev_mid, prev_y = B["mid"], B["y"]
            x = B["xb"] if x is B["x"] else B["x"]
        self._rms(prev_mid, prev_y, self.final_norm, x, B["enc"], B["rstd"], m)
        _lib.call("mfb_memcpy2d_d2d", P(B["last"].ptr), c * 2, P(B["enc"].ptr + (t - 1) * c * 2), t * c * 2, c * 2,
                  b, s)  # the last prompt token of every row
        _fwd(B["last"], self.head, B["logits16"], b, cfg.vocab, c, s)
        logits = DeviceArray((b, cfg.vocab), "float32")
        _lib.call("mfb_cast_bf16_f32", P(B["logits16"].ptr), P(logits.ptr), b * cfg.vocab, s)
        state.valid_length = t
        return logits

    def decode_one(self, input_ids, state: DecodeState, *, out=None, graph: bool = False):
        """FP32 logits [B, vocab] of the next token for each row; writes the caches and advances the state.

        ``out`` (a float32 [B, vocab] DeviceArray) receives the logits instead
        of a new array. ``graph=True`` replays the step as one CUDA graph,
        captured on the first call for this state's caches (needs a created
        stream); the step reads its token ids, positions and lengths from
        device buffers uploaded before each replay, so one graph serves every
        step.
        """
        cfg, s = self.cfg, self.stream
        if state.cfg != cfg:
            raise ValueError("Decode state does not match the decoder config")
        if state.valid_length >= cfg.max_position_embeddings:
            raise ValueError("Decode position exceeds model max_position_embeddings")
        if state.valid_length >= state.capacity:
            raise DecodeOverflow(f"Cannot decode at position {state.valid_length}; capacity is {state.capacity}")
        ids = np.asarray(input_ids, np.int32)
        if ids.ndim == 2 and ids.shape[1] == 1:
            ids = ids[:, 0]
        if ids.ndim != 1 or ids.shape[0] != state.batch:
            raise ValueError("decode_one input_ids must have shape [batch] or [batch, 1] matching the state")
        b = state.batch
        if out is not None and (tuple(out.shape) != (b, cfg.vocab) or out.dtype != "float32"):
            raise ValueError("out must be a float32 [batch, vocab] device array")
        if graph and not s:
            raise ValueError("graph replay needs Decoder(stream=...) from mfb_stream_create")
        B = self._buffers(b, state.capacity)
        pos = state.valid_length
        meta = np.ascontiguousarray(np.stack([ids, np.full(b, pos, np.int32), np.full(b, pos + 1, np.int32)]))
        _lib.call("mfb_memcpy_h2d", P(B["meta"].ptr), meta.ctypes.data_as(P), meta.nbytes, s)
        logits = out if out is not None else DeviceArray((b, cfg.vocab), "float32")
        if graph:
            key = (b, state.capacity) + tuple(a.ptr for a in (*state.keys, *state.values, *state.history)
                                               if a is not None)
            g = self._graphs.get(key)
            if g is None:
                _lib.call("mfb_graph_begin", P(s))
                try:
                    self._step(B, state, B["logits"])
                finally:
                    g_ = P()
                    _lib.call("mfb_graph_end", P(s), ctypes.byref(g_))
                g = self._graphs[key] = g_.value
            _lib.call("mfb_graph_launch", P(g), P(s))
            _lib.call("mfb_memcpy_d2d", P(logits.ptr), P(B["logits"].ptr), logits.nbytes, s)
        else:
            self._step(B, state, logits)
        state.valid_length = pos + 1
        return logits

    def _step(self, B, state: DecodeState, logits):
        """The device work of one decode step (token ids, positions, lengths already in B)."""
        cfg, s = self.cfg, self.stream
        b, c, f, h, hk = state.batch, cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads
        nq = (h + 2 * hk) * cfg.head_dim
        _lib.call("mfb_embed_gather", P(self.embed.ptr), P(B["ids"].ptr), P(B["x"].ptr), b, c, cfg.vocab, s)
        x, prev_mid, prev_y = B["x"], None, None
        for i, L in enumerate(self.layers):
            # Block input (the previous block's mid + FFN output) and its operator norm.
            if prev_mid is None:
                self._rms(x, None, L["op_norm"], None, B["hn"], B["rstd"], b)
            else:
                self._rms(prev_mid, prev_y, L["op_norm"], x, B["hn"], B["rstd"], b)
            if L["kind"] == "conv":
                self._proj(B["hn"], L["w_in"], B["proj"], b, 3 * c, c, B)
                _lib.call("mfb_conv_step", P(B["proj"].ptr), P(L["taps"].ptr), P(state.history[i].ptr),
                          P(B["mixed"].ptr), b, c, s)
                self._proj(B["mixed"], L["w_out"], B["r"], b, c, c, B)
            else:
                self._proj(B["hn"], L["w_in"], B["proj"], b, nq, c, B)
                _lib.call("mfb_qknorm_rope_fwd", P(B["proj"].ptr), nq, P(L["qn"].ptr), P(L["kn"].ptr),
                          P(B["pos"].ptr), P(self.freqs.ptr), P(B["q"].ptr), P(B["k"].ptr), P(B["v"].ptr),
                          P(B["rq"].ptr), P(B["rk"].ptr), b, h, hk, ctypes.c_float(cfg.norm_eps), s)
                _lib.call("mfb_decode_attn", P(B["q"].ptr), P(state.keys[i].ptr), P(state.values[i].ptr),
                          P(B["k"].ptr), P(B["v"].ptr), P(B["pos"].ptr), P(B["lens"].ptr), P(B["o"].ptr), b,
                          state.capacity, h, hk, cfg.head_dim, ctypes.c_float(cfg.head_dim ** -0.5),
                          P(B["ws"].ptr), B["ws"].nbytes, s)
                self._proj(B["o"], L["w_out"], B["r"], b, c, h * cfg.head_dim, B)
            self._rms(x, B["r"], L["ffn_norm"], B["mid"], B["h2"], B["rstd"], b)
            self._proj(B["h2"], L["w13"], B["gu"], b, 2 * f, c, B)
            _lib.call("mfb_swiglu_fwd", P(B["gu"].ptr), P(B["a"].ptr), b, f, s)
            self._proj(B["a"], L["w2"], B["y"], b, c, f, B)
            prev_mid, prev_y = B["mid"], B["y"]
            x = B["xb"] if x is B["x"] else B["x"]  # the next block's input buffer (ping-pong)
        self._rms(prev_mid, prev_y, self.final_norm, x, B["enc"], B["rstd"], b)
        self._proj(B["enc"], self.head, B["logits16"], b, cfg.vocab, c, B)
        _lib.call("mfb_cast_bf16_f32", P(B["logits16"].ptr), P(logits.ptr), b * cfg.vocab, s)

    def close(self):
        """Release the captured decode graphs."""
        graphs, self._graphs = getattr(self, "_graphs", {}), {}
        for g in graphs.values():
            if _lib._lib is not None:
                _lib.lib().mfb_graph_destroy(P(g))

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def prefill(decoder: Decoder, input_ids, state: DecodeState):
    """``(logits, state)`` like models/lfm2_5/decode.py:373 (the state's device caches are filled in place)."""
    return decoder.prefill(input_ids, state), state


def decode_one(decoder: Decoder, input_ids, state: DecodeState):
    """``(logits, state)`` like models/lfm2_5/decode.py:419 (the state's device caches are updated in place)."""
    return decoder.decode_one(input_ids, state), state


__all__ = ["DecodeOverflow", "DecodeState", "Decoder", "decode_one", "init_parameters", "new_state", "prefill",
           "parameter_shapes"]
