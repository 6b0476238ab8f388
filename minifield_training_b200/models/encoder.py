"""LFM2.5-style encoder training step (config 5) on B200: QAT forward, backward,
data-parallel gradient allreduce and the transactional AdamW commit.

Mirrors, with the reference's parameter names and block equations:
  encode / _block        src/minifield_training/models/lfm2_5/encoder.py:64-240
  conv_input_projection  src/minifield_training/layers/convolution.py:29-37
  project_qkv, rope      src/minifield_training/layers/attention.py:61-97
  swiglu_ffn             src/minifield_training/layers/feed_forward.py:24-35
  QAT on projections     src/minifield_training/strategies/quantization.py:114-126
                         over model.projection_names (models/lfm2_5/model.py:169-184)
  step normalization     src/minifield_training/engine/step.py:36-78, :367-395
  AdamW transaction      src/minifield_training/optimizers/adamw.py:384-571
The reference's encoder ships no training head; this step adds a token
classification head ("head.weight" [classes, hidden], a decayed trainable
matrix, not quantized) with a summed cross-entropy over valid tokens and the
valid-token count as the loss terms (engine/step.py:17-19 contract).

Every activation and weight buffer is allocated once per EncoderStep. Each
layer's projections are fake-quantized into fused bf16 weight buffers
(q|k|v and gate|up rows adjacent), and the parameter arenas are ordered so the
fused weight gradients land, FP32, straight in the gradient arena. Activations
are kept for the backward (no rematerialization: 180 GB of HBM holds them).
With a communicator (NCCL through the library's C ABI, comm.Communicator) the
gradient arena (plus the loss and count in its tail) is all-reduced bucket by
bucket on a communication stream as each layer's backward is enqueued,
overlapping the remaining backward; the AdamW commit then runs replicated.
"""

import ctypes
from dataclasses import dataclass

import numpy as np

from .. import _lib
from ..device import DeviceArray, Event
from ..optimizers import adamw

P = ctypes.c_void_p


def _prefix(i):
    return f"lfm2.layers.{i}."


def parameter_shapes(cfg) -> dict:
    """Reference names and shapes (model.py:127-166 with the encoder's lfm2. prefix) plus the head."""
    c, f, kv = cfg.hidden, cfg.ffn, cfg.kv_heads * cfg.head_dim
    shapes = {"lfm2.embed_tokens.weight": (cfg.vocab, c), "lfm2.embedding_norm.weight": (c,),
              "head.weight": (cfg.classes, c)}
    for i, kind in enumerate(cfg.layer_types):
        p = _prefix(i)
        shapes.update({p + "operator_norm.weight": (c,), p + "ffn_norm.weight": (c,),
                       p + "feed_forward.w1.weight": (f, c), p + "feed_forward.w3.weight": (f, c),
                       p + "feed_forward.w2.weight": (c, f)})
        if kind == "conv":
            shapes.update({p + "conv.in_proj.weight": (3 * c, c), p + "conv.out_proj.weight": (c, c),
                           p + "conv.conv.weight": (c, 1, 3)})
        else:
            shapes.update({p + "self_attn.q_proj.weight": (c, c), p + "self_attn.k_proj.weight": (kv, c),
                           p + "self_attn.v_proj.weight": (kv, c), p + "self_attn.out_proj.weight": (c, c),
                           p + "self_attn.q_layernorm.weight": (cfg.head_dim,),
                           p + "self_attn.k_layernorm.weight": (cfg.head_dim,)})
    return shapes


PROJECTION_SUFFIXES = ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                       "self_attn.out_proj.weight", "conv.in_proj.weight", "conv.out_proj.weight",
                       "feed_forward.w1.weight", "feed_forward.w2.weight", "feed_forward.w3.weight")


def projection_names(cfg) -> frozenset:
    return frozenset(n for n in parameter_shapes(cfg) if n.endswith(PROJECTION_SUFFIXES))


def inventory(cfg) -> adamw.Inventory:
    """Decay every unfrozen matrix (model.py:187-209); the token embeddings are frozen."""
    shapes = parameter_shapes(cfg)
    frozen = frozenset({"lfm2.embed_tokens.weight"})
    return adamw.build_inventory(shapes, decayed_names=frozenset(n for n, s in shapes.items()
                                                                 if len(s) == 2 and n not in frozen),
                                 frozen_names=frozen)


def arena_order(cfg):
    """Head first, then layers last to first (the backward's order), fused groups adjacent."""
    order = ["head.weight", "lfm2.embedding_norm.weight"]
    for i in reversed(range(len(cfg.layer_types))):
        p = _prefix(i)
        order += [p + "feed_forward.w1.weight", p + "feed_forward.w3.weight", p + "feed_forward.w2.weight",
                  p + "ffn_norm.weight"]
        if cfg.layer_types[i] == "conv":
            order += [p + "conv.out_proj.weight", p + "conv.in_proj.weight", p + "conv.conv.weight"]
        else:
            order += [p + "self_attn.out_proj.weight", p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                      p + "self_attn.v_proj.weight", p + "self_attn.q_layernorm.weight",
                      p + "self_attn.k_layernorm.weight"]
        order.append(p + "operator_norm.weight")
    order.append("lfm2.embed_tokens.weight")
    return order


def init_parameters(cfg, seed: int = 0) -> dict:
    """Random init: N(0, 0.02) for matrices, taps, embeddings and the head; ones for norm gains."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in parameter_shapes(cfg).items():
        if name.endswith("norm.weight") or name.endswith("layernorm.weight"):
            out[name] = np.ones(shape, np.float32)
        else:
            out[name] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02))
    return out


def rope_freqs(theta: float, head_dim: int = 64) -> np.ndarray:
    """theta ** (-arange(0, D, 2) / D) in float32 (kernels/rotary.py:31-33)."""
    return (np.float32(theta) ** (-np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim))).astype(
        np.float32)


def _gemm(a, a_major, lda, b, b_major, ldb, c, ldc, f32, m, n, k, mask=None, stream=None, ws=None):
    _lib.call("mfb_gemm_bf16_ws", P(a), a_major, lda, P(b), b_major, ldb, P(c), ldc,
              _lib.DTYPE_F32 if f32 else _lib.DTYPE_BF16, m, n, k, ctypes.c_float(1.0),
              P(mask) if mask is not None else None, 0, P(ws.ptr) if ws is not None else None,
              ws.nbytes if ws is not None else 0, stream)


def _fwd(x, w, out, m, n, k, stream):
    """out[m, n] = x[m, k] . w[n, k]^T (bf16)."""
    _gemm(x.ptr, _lib.MAJOR_K, k, w.ptr, _lib.MAJOR_K, k, out.ptr, n, False, m, n, k, stream=stream)


def _dgrad(dy, w, out, m, n, k, stream):
    """out[m, k] = dy[m, n] . w[n, k] (bf16)."""
    _gemm(dy.ptr, _lib.MAJOR_K, n, w.ptr, _lib.MAJOR_MN, k, out.ptr, k, False, m, k, n, stream=stream)


def _wgrad(dy, x, out_ptr, ste, m, n, k, stream, ws=None):
    """out[n, k] (FP32) = dy[m, n]^T . x[m, k], times the STE mask. These products have few
    output tiles and K = the token count: ``ws`` (mfb_gemm_workspace_size bytes) lets the GEMM
    split K so that every SM pair gets work."""
    _gemm(dy.ptr, _lib.MAJOR_MN, n, x.ptr, _lib.MAJOR_MN, k, out_ptr, k, True, n, k, m,
          mask=ste.ptr if ste is not None else None, stream=stream, ws=ws)


@dataclass
class _Layer:
    kind: str
    x: DeviceArray         # layer input (sum), [M, C]
    h: DeviceArray         # operator-normed input
    rstd_op: DeviceArray
    mid: DeviceArray       # x + operator residual
    h2: DeviceArray        # ffn-normed
    rstd_ffn: DeviceArray
    gu: DeviceArray        # [M, 2F]
    a: DeviceArray         # [M, F]
    y: DeviceArray         # ffn output [M, C]
    r: DeviceArray         # operator output [M, C]
    proj: DeviceArray      # conv: bcx [M, 3C]; attention: raw qkv [M, 2048]
    mixed: DeviceArray = None  # conv
    q: DeviceArray = None
    k: DeviceArray = None
    v: DeviceArray = None
    o: DeviceArray = None
    lse: DeviceArray = None
    rstd_q: DeviceArray = None
    rstd_k: DeviceArray = None
    w_in: DeviceArray = None   # fused eff bf16 [3C | 2048, C]
    ste_in: DeviceArray = None
    w_out: DeviceArray = None
    ste_out: DeviceArray = None
    w13: DeviceArray = None
    ste13: DeviceArray = None
    w2: DeviceArray = None
    ste2: DeviceArray = None


class EncoderStep:
    """One logical training step over ``rows`` local sequences of the global batch.

    ``comm`` (a comm.Communicator, or None) all-reduces the gradient sums,
    loss and count; ``stream`` is the CUDA stream handle all kernels run on.
    With a communicator the collectives run on a communication stream of the
    step's own, ordered after the kernels they reduce by events.
    ``shard_optimizer`` (with a communicator) partitions the optimizer state:
    each rank owns a contiguous, bucket-aligned range of the trainable arena
    (``owner_ranges``); each gradient bucket is reduced to its owner instead
    of all-reduced, the AdamW passes run on the owned range (their global
    decisions are allreduces of three doubles), and the owners broadcast the
    updated masters at the end of the step. The next step's forward waits for
    each layer's masters just before that layer, so the broadcast overlaps the
    forward; ``settle()`` orders other work after it. Moments outside a rank's
    range are never touched on that rank.
    """

    def __init__(self, cfg, rows: int, *, seed: int = 0, comm=None, stream=None, shard_optimizer: bool = False):
        self.cfg, self.rows, self.T = cfg, rows, cfg.length
        self.M = m = rows * cfg.length
        self.comm, self.stream = comm, stream
        c, f, h, hk = cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads
        self.nq = (h + 2 * hk) * cfg.head_dim
        inv = inventory(cfg)
        self.layout = adamw.Layout(inv, arena_order(cfg))
        n_grad = self.layout.n_train + 4  # tail: loss sum, count
        grads = DeviceArray.zeros((n_grad,), "float32")
        self.grads = grads
        opt = adamw.AdamWConfig(cfg.learning_rate, beta1=cfg.beta1, beta2=cfg.beta2, epsilon=cfg.epsilon,
                                weight_decay=cfg.weight_decay, clip_norm=cfg.clip_norm)
        self._buckets = reduction_plan(self.layout, len(cfg.layer_types), n_grad)
        self.shard_optimizer = bool(shard_optimizer) and comm is not None
        if self.shard_optimizer:
            # Each rank owns a contiguous, bucket-aligned range of the trainable
            # arena: gradients are reduced to their owner, the AdamW passes run
            # on the owned range, and the owners broadcast the updated masters.
            self._owners = owner_ranges(self._buckets, self.layout.n_train, comm.world)
            self._bcast_plan = broadcast_plan(self._buckets, self.layout.n_train, self._owners)
            self._bcast_events = {key: Event() for key, _ in self._bcast_plan}
            self._gather_start = Event()
            self._pending = False
        self.comm_stream = None
        if comm is not None:
            cs = ctypes.c_void_p()
            _lib.call("mfb_stream_create", ctypes.byref(cs))
            self.comm_stream = cs.value
            self._order_events = (Event(), Event())
        self.state = adamw.initialize_state(init_parameters(cfg, seed), inv, order=arena_order(cfg), grads=grads)
        self.loss_count = grads.view(self.layout.n_train, (2,))
        if self.shard_optimizer:
            lo, hi = self._owners[comm.rank]
            check_hi = self.layout.n_total if comm.rank == comm.world - 1 else hi
            self.transition = adamw.make_sharded_transaction(inv, opt, comm, slices=(lo, check_hi, lo, hi))
        else:
            self.transition = adamw.make_transaction(inv, opt)
        self.params = self.state["params"]
        self.gviews = self.state.gradient_tree()
        self.quant = _lib.QUANT_KINDS[cfg.quant] if cfg.quant else None
        bf, f32 = "bfloat16", "float32"
        E = DeviceArray
        # Shared step inputs and scratch.
        self.ids, self.mask, self.seg, self.pos, self.labels = (E((m,), "int32") for _ in range(5))
        self.freqs = E.from_numpy(rope_freqs(cfg.rope_theta, cfg.head_dim), f32)
        self.qid, self.kid = E((rows, self.T), "int32"), E((rows, self.T), "int32")
        self.x0 = E((m, c), bf)
        self.final = E((m, c), bf)
        self.enc = E((m, c), bf)
        self.rstd_final = E((m,), f32)
        self.d_a, self.d_b = E((m, c), bf), E((m, c), bf)   # residual-stream gradients (ping-pong)
        self.d_mid = E((m, c), bf)
        self.d_h = E((m, c), bf)
        self.d_gu = E((m, 2 * f), bf)
        self.d_proj = E((m, max(3 * c, self.nq)), bf)
        self.d_q, self.d_k, self.d_v = E((m, h, 64), bf), E((m, hk, 64), bf), E((m, hk, 64), bf)
        self.d_o = E((m, c), bf)
        ws = max(_lib.lib().mfb_norm_workspace_size(m, c), _lib.lib().mfb_encoder_workspace_size(c, cfg.classes))
        self.ws = E((ws,), "uint8")
        # Split-K partials of the weight-gradient GEMMs (out features x in features, K = m tokens).
        wg = [(c, f), (2 * f, c), (c, c), (3 * c, c), (self.nq, c)]
        self.gemm_ws = E((max(16, max(int(_lib.lib().mfb_gemm_workspace_size(n, k, m)) for n, k in wg)),), "uint8")
        aws = _lib.lib().mfb_attn_workspace_size(rows, self.T, self.T, h, hk, cfg.head_dim)
        self.attn_ws = E((max(aws, 16),), "uint8")
        self.result = None
        # Normalized loss, gradient divisor and accumulation flag of the commit.
        self._scalars = (E((1,), f32), E((1,), f32), E((1,), "uint8"))
        self.layers = []
        for kind in cfg.layer_types:
            L = _Layer(kind, x=E((m, c), bf), h=E((m, c), bf), rstd_op=E((m,), f32), mid=E((m, c), bf),
                       h2=E((m, c), bf), rstd_ffn=E((m,), f32), gu=E((m, 2 * f), bf), a=E((m, f), bf),
                       y=E((m, c), bf), r=E((m, c), bf),
                       proj=E((m, 3 * c if kind == "conv" else self.nq), bf))
            if kind == "conv":
                L.mixed = E((m, c), bf)
                L.w_in, L.ste_in = E((3 * c, c), bf), E((3 * c, c), "uint8")
            else:
                L.q, L.k, L.v, L.o = E((m, h, 64), bf), E((m, hk, 64), bf), E((m, hk, 64), bf), E((m, c), bf)
                L.lse, L.rstd_q, L.rstd_k = E((rows, h, self.T), f32), E((m, h), f32), E((m, hk), f32)
                L.w_in, L.ste_in = E((self.nq, c), bf), E((self.nq, c), "uint8")
            L.w_out, L.ste_out = E((c, c), bf), E((c, c), "uint8")
            L.w13, L.ste13 = E((2 * f, c), bf), E((2 * f, c), "uint8")
            L.w2, L.ste2 = E((c, f), bf), E((c, f), "uint8")
            self.layers.append(L)
        self.head_eff = E((cfg.classes, c), bf)
        # Initialization ran on the default stream; a created (non-blocking)
        # step stream does not order after it, so finish it here.
        _lib.call("mfb_device_sync")

    # ---- helpers -----------------------------------------------------------------
    def _p(self, name):
        return self.params[name]

    def _g(self, name):
        return self.gviews[name]

    def _quantize(self, name, eff: DeviceArray, ste: DeviceArray, row0: int):
        w = self._p(name)
        rows, cols = w.shape
        e = eff.view(row0 * cols, (rows, cols))
        s = ste.view(row0 * cols, (rows, cols))
        if self.quant is None:
            _lib.call("mfb_cast_f32_bf16", P(w.ptr), P(e.ptr), rows * cols, self.stream)
            _lib.call("mfb_memset", P(s.ptr), 1, rows * cols, self.stream)
        else:
            _lib.call("mfb_fakequant", P(w.ptr), self.quant, rows, cols, None, None, P(s.ptr), None, P(e.ptr),
                      self.stream)

    def _quantize_layer(self, i):
        c, f = self.cfg.hidden, self.cfg.ffn
        L, p = self.layers[i], _prefix(i)
        self._quantize(p + "feed_forward.w1.weight", L.w13, L.ste13, 0)
        self._quantize(p + "feed_forward.w3.weight", L.w13, L.ste13, f)
        self._quantize(p + "feed_forward.w2.weight", L.w2, L.ste2, 0)
        if L.kind == "conv":
            self._quantize(p + "conv.in_proj.weight", L.w_in, L.ste_in, 0)
            self._quantize(p + "conv.out_proj.weight", L.w_out, L.ste_out, 0)
        else:
            kv = self.cfg.kv_heads * self.cfg.head_dim
            self._quantize(p + "self_attn.q_proj.weight", L.w_in, L.ste_in, 0)
            self._quantize(p + "self_attn.k_proj.weight", L.w_in, L.ste_in, c)
            self._quantize(p + "self_attn.v_proj.weight", L.w_in, L.ste_in, c + kv)
            self._quantize(p + "self_attn.out_proj.weight", L.w_out, L.ste_out, 0)

    def _quantize_head(self):
        # The head is not a model projection: full_linear casts its master to bf16.
        hw = self._p("head.weight")
        _lib.call("mfb_cast_f32_bf16", P(hw.ptr), P(self.head_eff.ptr), hw.size, self.stream)

    def quantize(self):
        """Effective bf16 weights and STE masks of every projection for this step."""
        for i in range(len(self.layers)):
            self._quantize_layer(i)
        self._quantize_head()

    def set_batch(self, ids, mask, seg, pos, labels):
        """Upload one local batch (int32 [rows, T] host arrays) and build the attention ids."""
        for dst, src in ((self.ids, ids), (self.mask, mask), (self.seg, seg), (self.pos, pos),
                         (self.labels, labels)):
            a = np.ascontiguousarray(np.asarray(src, np.int32).reshape(-1))
            _lib.call("mfb_memcpy_h2d", P(dst.ptr), a.ctypes.data_as(P), a.nbytes, self.stream)
        self._build_ids()

    def _build_ids(self):
        c_, o_, p_ = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _lib.call("mfb_attn_ids", _lib.MASK_BIDIR, P(self.mask.ptr), P(self.seg.ptr), None, P(self.qid.ptr),
                  P(self.kid.ptr), self.rows, self.T, self.T, 0, ctypes.byref(c_), ctypes.byref(o_),
                  ctypes.byref(p_), self.stream)
        self.attn_flags = (c_.value, o_.value, p_.value)

    # ---- forward -------------------------------------------------------------------
    def _rms(self, x, res, w, mask, sum_out, y, rstd):
        _lib.call("mfb_rmsnorm_fwd", P(x.ptr), P(res.ptr) if res is not None else None, P(w.ptr),
                  P(mask.ptr) if mask is not None else None, P(sum_out.ptr) if res is not None else None, P(y.ptr),
                  P(rstd.ptr), self.M, self.cfg.hidden, ctypes.c_float(self.cfg.norm_eps), self.stream)

    def forward(self):
        self._fwd_embed()
        for i in range(len(self.layers)):
            self._fwd_layer(i)
        self._fwd_final()

    def _fwd_embed(self):
        cfg, m, c = self.cfg, self.M, self.cfg.hidden
        emb = self._p("lfm2.embed_tokens.weight")
        _lib.call("mfb_embed_gather", P(emb.ptr), P(self.ids.ptr), P(self.x0.ptr), m, c, cfg.vocab, self.stream)

    def _fwd_layer(self, i):
        cfg, m, c, f, s = self.cfg, self.M, self.cfg.hidden, self.cfg.ffn, self.stream
        L, p = self.layers[i], _prefix(i)
        prev = self.layers[i - 1] if i > 0 else None
        opmask = self.mask if L.kind == "conv" else None
        if prev is None:
            _lib.call("mfb_memcpy_d2d", P(L.x.ptr), P(self.x0.ptr), L.x.nbytes, s)
            self._rms(L.x, None, self._p(p + "operator_norm.weight"), opmask, None, L.h, L.rstd_op)
        else:
            self._rms(prev.mid, prev.y, self._p(p + "operator_norm.weight"), opmask, L.x, L.h, L.rstd_op)
        if L.kind == "conv":
            _fwd(L.h, L.w_in, L.proj, m, 3 * c, c, s)
            _lib.call("mfb_conv_fwd", P(L.proj.ptr), P(self._p(p + "conv.conv.weight").ptr), P(self.seg.ptr),
                      P(L.mixed.ptr), m, self.T, c, s)
            _fwd(L.mixed, L.w_out, L.r, m, c, c, s)
        else:
            _fwd(L.h, L.w_in, L.proj, m, self.nq, c, s)
            _lib.call("mfb_qknorm_rope_fwd", P(L.proj.ptr), self.nq, P(self._p(p + "self_attn.q_layernorm.weight").ptr),
                      P(self._p(p + "self_attn.k_layernorm.weight").ptr), P(self.pos.ptr), P(self.freqs.ptr),
                      P(L.q.ptr), P(L.k.ptr), P(L.v.ptr), P(L.rstd_q.ptr), P(L.rstd_k.ptr), m, cfg.heads,
                      cfg.kv_heads, ctypes.c_float(cfg.norm_eps), s)
            causal, off, pol = self.attn_flags
            _lib.call("mfb_attn_fwd", P(L.q.ptr), P(L.k.ptr), P(L.v.ptr), P(L.o.ptr), P(L.lse.ptr),
                      P(self.qid.ptr), P(self.kid.ptr), self.rows, self.T, self.T, cfg.heads, cfg.kv_heads,
                      cfg.head_dim, causal, off, pol, ctypes.c_float(cfg.head_dim ** -0.5), P(self.attn_ws.ptr),
                      self.attn_ws.nbytes, s)
            _fwd(L.o, L.w_out, L.r, m, c, c, s)
        self._rms(L.x, L.r, self._p(p + "ffn_norm.weight"), None, L.mid, L.h2, L.rstd_ffn)
        # gate|up GEMM with silu(gate) * up in its epilogue
        _lib.call("mfb_gemm_swiglu_fwd", P(L.h2.ptr), _lib.MAJOR_K, c, P(L.w13.ptr), c, P(L.gu.ptr), P(L.a.ptr),
                  m, f, c, s)
        _fwd(L.a, L.w2, L.y, m, c, f, s)

    def _fwd_final(self):
        prev = self.layers[-1]
        self._rms(prev.mid, prev.y, self._p("lfm2.embedding_norm.weight"), self.mask, self.final, self.enc,
                  self.rstd_final)

    # ---- backward ------------------------------------------------------------------
    def _rms_bwd(self, x, w, rstd, mask, dy, dres, dx, dw):
        _lib.call("mfb_rmsnorm_bwd", P(x.ptr), P(w.ptr), P(rstd.ptr), P(mask.ptr) if mask is not None else None,
                  P(dy.ptr), P(dres.ptr) if dres is not None else None, P(dx.ptr), P(dw.ptr), 0, self.M,
                  self.cfg.hidden, P(self.ws.ptr), self.ws.nbytes, self.stream)

    def _grad_bufs(self, i):
        """Residual-stream gradient buffers (into layer i's output, out of its input).

        Fixed per layer (ping-pong by layer parity), so captured graphs see the
        same pointers on every replay.
        """
        k = len(self.layers) - 1 - i
        return (self.d_a, self.d_b) if k % 2 == 0 else (self.d_b, self.d_a)

    def _bwd_head(self):
        """Head + loss (which also starts the backward) and the final norm's backward."""
        cfg, m, c, s = self.cfg, self.M, self.cfg.hidden, self.stream
        lc = self.loss_count
        _lib.call("mfb_head_loss", P(self.enc.ptr), P(self._p("head.weight").ptr), P(self.labels.ptr),
                  P(self.mask.ptr), P(self.d_h.ptr), P(self._g("head.weight").ptr), P(lc.ptr), m, c, cfg.classes,
                  P(self.ws.ptr), self.ws.nbytes, s)
        d, _ = self._grad_bufs(len(self.layers) - 1)
        self._rms_bwd(self.final, self._p("lfm2.embedding_norm.weight"), self.rstd_final, self.mask, self.d_h, None,
                      d, self._g("lfm2.embedding_norm.weight"))

    def _bwd_layer(self, i):
        """Backward of layer i: d (gradient of its output) -> spare (gradient of its input)."""
        cfg, m, c, f, s = self.cfg, self.M, self.cfg.hidden, self.cfg.ffn, self.stream
        L, p = self.layers[i], _prefix(i)
        d, spare = self._grad_bufs(i)
        # FFN: x_next = mid + y.
        _wgrad(d, L.a, self._g(p + "feed_forward.w2.weight").ptr, L.ste2, m, c, f, s, self.gemm_ws)
        # dH = d . W2 with the SwiGLU backward in its epilogue: d_gu directly
        _lib.call("mfb_gemm_swiglu_bwd", P(d.ptr), _lib.MAJOR_K, c, P(L.w2.ptr), _lib.MAJOR_MN, f, P(L.gu.ptr),
                  P(self.d_gu.ptr), m, f, c, s)
        _dgrad(self.d_gu, L.w13, self.d_h, m, 2 * f, c, s)
        _wgrad(self.d_gu, L.h2, self._g(p + "feed_forward.w1.weight").ptr, L.ste13, m, 2 * f, c, s, self.gemm_ws)
        self._rms_bwd(L.mid, self._p(p + "ffn_norm.weight"), L.rstd_ffn, None, self.d_h, d, self.d_mid,
                      self._g(p + "ffn_norm.weight"))
        # Operator: mid = x + r.
        if L.kind == "conv":
            _dgrad(self.d_mid, L.w_out, self.d_o, m, c, c, s)
            _wgrad(self.d_mid, L.mixed, self._g(p + "conv.out_proj.weight").ptr, L.ste_out, m, c, c, s, self.gemm_ws)
            _lib.call("mfb_conv_bwd", P(L.proj.ptr), P(self._p(p + "conv.conv.weight").ptr), P(self.seg.ptr),
                      P(self.d_o.ptr), P(self.d_proj.ptr), P(self._g(p + "conv.conv.weight").ptr), 0, m, self.T,
                      c, P(self.ws.ptr), self.ws.nbytes, s)
            _dgrad(self.d_proj, L.w_in, self.d_h, m, 3 * c, c, s)
            _wgrad(self.d_proj, L.h, self._g(p + "conv.in_proj.weight").ptr, L.ste_in, m, 3 * c, c, s, self.gemm_ws)
        else:
            _dgrad(self.d_mid, L.w_out, self.d_o, m, c, c, s)
            _wgrad(self.d_mid, L.o, self._g(p + "self_attn.out_proj.weight").ptr, L.ste_out, m, c, c, s, self.gemm_ws)
            causal, off, pol = self.attn_flags
            _lib.call("mfb_attn_bwd", P(L.q.ptr), P(L.k.ptr), P(L.v.ptr), P(L.o.ptr), P(L.lse.ptr),
                      P(self.d_o.ptr), P(self.d_q.ptr), P(self.d_k.ptr), P(self.d_v.ptr), P(self.qid.ptr),
                      P(self.kid.ptr), self.rows, self.T, self.T, cfg.heads, cfg.kv_heads, cfg.head_dim, causal,
                      off, pol, ctypes.c_float(cfg.head_dim ** -0.5), P(self.attn_ws.ptr), self.attn_ws.nbytes, s)
            _lib.call("mfb_qknorm_rope_bwd", P(L.proj.ptr), self.nq,
                      P(self._p(p + "self_attn.q_layernorm.weight").ptr),
                      P(self._p(p + "self_attn.k_layernorm.weight").ptr), P(self.pos.ptr), P(self.freqs.ptr),
                      P(L.rstd_q.ptr), P(L.rstd_k.ptr), P(self.d_q.ptr), P(self.d_k.ptr), P(self.d_v.ptr),
                      P(self.d_proj.ptr), P(self._g(p + "self_attn.q_layernorm.weight").ptr),
                      P(self._g(p + "self_attn.k_layernorm.weight").ptr), 0, m, cfg.heads, cfg.kv_heads,
                      P(self.ws.ptr), self.ws.nbytes, s)
            _dgrad(self.d_proj, L.w_in, self.d_h, m, self.nq, c, s)
            _wgrad(self.d_proj, L.h, self._g(p + "self_attn.q_proj.weight").ptr,
                   L.ste_in, m, self.nq, c, s, self.gemm_ws)
        opmask = self.mask if L.kind == "conv" else None
        self._rms_bwd(L.x, self._p(p + "operator_norm.weight"), L.rstd_op, opmask, self.d_h, self.d_mid, spare,
                      self._g(p + "operator_norm.weight"))

    def backward(self, on_layer_done=None):
        self._bwd_head()
        for i in reversed(range(len(self.layers))):
            self._bwd_layer(i)
            if on_layer_done is not None:
                on_layer_done(i)
        self.d_x0 = self._grad_bufs(0)[1]  # the embeddings are frozen: this gradient is not used

    # ---- the logical step ------------------------------------------------------------
    def capture(self):
        """Record the step as CUDA graphs on this step's stream (a created stream).

        One GPU: one graph (quantize, forward, backward, normalize, commit).
        With a communicator: the forward and the head's backward, one graph per
        layer's backward (so each layer's bucket reduction is launched between
        them), and the commit (replicated optimizer) or the normalization
        (sharded optimizer, whose passes hold collectives). With the sharded
        optimizer the forward is one graph per layer (that layer's
        quantization and forward), so each waits only for its own masters'
        broadcast from the previous step.
        """
        if getattr(self, "graphs", None) is not None:
            return
        if self.stream is None:
            raise ValueError("graph capture needs EncoderStep(stream=...) from mfb_stream_create")

        def rec(fn):
            _lib.call("mfb_graph_begin", P(self.stream))
            try:
                fn()
            finally:
                g = ctypes.c_void_p()
                _lib.call("mfb_graph_end", P(self.stream), ctypes.byref(g))
            return g

        if self.comm is None:
            self.graphs = {"all": rec(self._eager_local_step)}
            self._result_dev = self.result._dev
        elif self.shard_optimizer:
            self.graphs = {"embed": rec(self._fwd_embed),
                           "fwd": [rec(lambda i=i: self._fwd_layer_quantized(i)) for i in range(len(self.layers))],
                           "head": rec(self._head_part),
                           "layers": [rec(lambda i=i: self._bwd_layer(i)) for i in reversed(range(len(self.layers)))],
                           "post": rec(self._normalize)}
        else:
            self.graphs = {"pre": rec(lambda: (self.quantize(), self.forward(), self._bwd_head())),
                           "layers": [rec(lambda i=i: self._bwd_layer(i)) for i in reversed(range(len(self.layers)))],
                           "post": rec(self._commit)}
            self._result_dev = self.result._dev

    def _eager_local_step(self):
        self.quantize()
        self.forward()
        self.backward()
        self._commit()

    def _launch(self, g):
        _lib.call("mfb_graph_launch", g, P(self.stream))

    # ---- sharded optimizer: owned ranges and the masters' broadcast -----------------
    def _fwd_layer_quantized(self, i):
        self._quantize_layer(i)
        self._fwd_layer(i)

    def _head_part(self):
        self._fwd_final()
        self._quantize_head()
        self._bwd_head()

    def _await(self, key):
        """The compute stream waits for the broadcast of ``key``'s masters (if one is pending)."""
        if self._pending:
            self._bcast_events[key].wait_on(self.stream)

    def _broadcast_masters(self):
        """Every owner broadcasts its updated masters, in the next forward's order, on the
        communication stream after the commit; one event per range group."""
        comm, cs, params = self.comm, self.comm_stream, self.state.arenas["params"]
        self._gather_start.record(self.stream)
        self._gather_start.wait_on(cs)
        for key, pieces in self._bcast_plan:
            for lo, hi, root in pieces:
                comm.broadcast(params.view(lo, (hi - lo,)), root, stream=cs)
            self._bcast_events[key].record(cs)
        self._pending = True

    def settle(self):
        """Order the compute stream after the last step's master broadcasts (sharded optimizer):
        afterwards every rank's masters are complete for work on that stream."""
        if self.shard_optimizer and self._pending:
            self._bcast_events["head"].wait_on(self.stream)  # the last broadcast on the stream
            self._pending = False

    def grad_owner(self, name):
        """The rank whose gradient of leaf ``name`` is reduced (sharded optimizer; 0 otherwise)."""
        if not self.shard_optimizer:
            return 0
        off = self.layout.offsets[name]
        return next(r for r, (lo, hi) in enumerate(self._owners) if lo <= off < hi)

    def _sharded_step(self, run):
        """One step with the sharded optimizer; ``run(key, i)`` launches a piece (graph or eager)."""
        run("embed", None)
        self._await("vectors")
        for i in range(len(self.layers)):
            self._await(("layer", i))
            run("fwd", i)
        self._await("head")
        self._pending = False
        run("head", None)
        reducer = self.reducer()
        for i in reversed(range(len(self.layers))):
            run("layers", i)
            reducer.layer_done(i)
        reducer.finish()
        run("post", None)
        loss, div, ok = self._scalars
        self.result = self.transition(self.state, loss, ok, divisor=div, stream=self.stream)
        self._broadcast_masters()
        return self.result

    def reducer(self):
        """A BucketReducer of this step's gradient arena over its communicator and streams:
        allreduces, or with the sharded optimizer reductions to each range's owner (and an
        allreduce of the loss/count tail)."""
        compute_done, reduced = self._order_events
        comm, flat, cs = self.comm, self.grads, self.comm_stream
        n_train = self.layout.n_train

        def reduce_range(lo, hi):
            if not self.shard_optimizer:
                comm.allreduce(flat.view(lo, (hi - lo,)), stream=cs)
                return
            for x, y, root in owner_reductions(lo, hi, self._owners, n_train):
                if root is None:
                    comm.allreduce(flat.view(x, (y - x,)), stream=cs)
                else:
                    comm.reduce(flat.view(x, (y - x,)), root, stream=cs)

        def before():  # the bucket's gradients are complete on the compute stream
            compute_done.record(self.stream)
            compute_done.wait_on(cs)

        def after():  # the compute stream continues once every bucket is reduced
            reduced.record(cs)
            reduced.wait_on(self.stream)

        return BucketReducer(self._buckets, reduce_range, before, after)

    def step(self):
        """quantize -> forward -> backward (+ bucketed gradient reduction) -> normalize -> AdamW commit.

        With the sharded optimizer the step ends by enqueueing the masters'
        broadcast; the next step's forward waits for it layer by layer, and
        ``settle()`` orders any other work after it."""
        graphs = getattr(self, "graphs", None)
        if self.shard_optimizer:
            if graphs is not None:
                def run(key, i):
                    g = graphs[key]
                    if key == "layers":
                        g = g[len(self.layers) - 1 - i]
                    elif key == "fwd":
                        g = g[i]
                    self._launch(g)
            else:
                eager = {"embed": lambda i: self._fwd_embed(), "fwd": self._fwd_layer_quantized,
                         "head": lambda i: self._head_part(), "layers": self._bwd_layer,
                         "post": lambda i: self._normalize()}

                def run(key, i):
                    eager[key](i)
            return self._sharded_step(run)
        if graphs is not None:
            if self.comm is None:
                self._launch(graphs["all"])
            else:
                self._launch(graphs["pre"])
                reducer = self.reducer()
                for g, i in zip(graphs["layers"], reversed(range(len(self.layers)))):
                    self._launch(g)
                    reducer.layer_done(i)
                reducer.finish()
                self._launch(graphs["post"])
            self.result = adamw.CommitResult(self.state, self._result_dev, self.stream)
            return self.result
        self.quantize()
        self.forward()
        if self.comm is not None:
            reducer = self.reducer()
            self.backward(reducer.layer_done)
            reducer.finish()
        else:
            self.backward()
        self._commit()
        return self.result

    def close(self):
        """Release the communication stream (the communicator belongs to the caller)."""
        cs, self.comm_stream = self.comm_stream, None
        if cs is not None and _lib._lib is not None:
            _lib.lib().mfb_stream_sync(P(cs))
            _lib.lib().mfb_stream_destroy(P(cs))

    def _normalize(self):
        loss, div, ok = self._scalars
        lc = self.loss_count
        _lib.call("mfb_step_normalize", P(lc.ptr), P(lc.ptr + 4), None, P(loss.ptr), P(div.ptr), P(ok.ptr),
                  self.stream)

    def _commit(self):
        """Normalize and commit (the replicated transaction; with the sharded optimizer the owned
        range's passes, then the masters' broadcast)."""
        self._normalize()
        loss, div, ok = self._scalars
        if self.shard_optimizer:
            self.result = self.transition(self.state, loss, ok, divisor=div, stream=self.stream)
            self._broadcast_masters()
        else:
            self.result = self.transition(self.state, self.gviews, loss, ok, divisor=div, stream=self.stream)


def reduction_plan(layout, n_layers: int, total: int):
    """Allreduce ranges of the flat gradient buffer, in launch order.

    One range per layer, backward order: the layer's matrices, contiguous in
    the decayed region (arena_order puts layers last to first). Then the rest
    in one or two ranges: the head before the first layer range, and after the
    last one every vector leaf plus the loss/count tail. Together the ranges
    partition [0, total) (checked by the tests).
    """
    plan = []
    for i in reversed(range(n_layers)):
        names = [n for n in layout.trainable if n.startswith(_prefix(i)) and len(layout.specs[n].shape) == 2]
        lo = min(layout.offsets[n] for n in names)
        hi = max(layout.offsets[n] + layout.size(n) for n in names)
        plan.append(("layer", i, lo, hi))
    lo_all = min(p[2] for p in plan)
    hi_all = max(p[3] for p in plan)
    if lo_all > 0:
        plan.append(("rest", -1, 0, lo_all))
    if total > hi_all:
        plan.append(("rest", -1, hi_all, total))
    return plan


def _round4(n):
    return (n + 3) // 4 * 4


def owner_ranges(plan, n_train: int, world: int):
    """[lo, hi) of the trainable arena owned by each rank: contiguous ranges
    tiling [0, n_train) whose cuts fall on bucket starts (the head range, a
    layer's matrices, the vector leaves), each cut the bucket start nearest an
    equal share. A bucket therefore belongs to one rank, except that a range
    may hold several. Starts are multiples of 4 (leaf offsets)."""
    layers = [(lo, hi) for kind, _, lo, hi in plan if kind == "layer"]
    starts = sorted({0} | {lo for lo, _ in layers} | {_round4(max(hi for _, hi in layers))})
    starts = [x for x in starts if x < n_train]
    cuts = [0]
    for k in range(1, world):
        target = k * n_train / world
        cand = [x for x in starts if x >= cuts[-1]]
        cuts.append(min(cand, key=lambda x: abs(x - target)) if cand else n_train)
    cuts.append(n_train)
    return [(cuts[r], cuts[r + 1]) for r in range(world)]


def owner_reductions(lo: int, hi: int, owners, n_train: int):
    """The collectives that reduce gradient range [lo, hi) under the sharded optimizer:
    (x, y, root) reductions of each owned piece to its owner, then (x, y, None) an
    allreduce of the part past the trainable arena (the loss/count tail every rank
    needs)."""
    out = []
    for r, (a, b) in enumerate(owners):
        x, y = max(lo, a), min(hi, b)
        if x < y:
            out.append((x, y, r))
    if hi > n_train:
        out.append((max(lo, n_train), hi, None))
    return out


def broadcast_plan(plan, n_train: int, owners):
    """Master ranges to broadcast after a sharded commit, in the order the next
    forward needs them: the vector leaves (every layer's norm gains), layers
    0, 1, ..., then the head. Each entry is (key, [(lo, hi, owner rank)])."""
    def pieces(lo, hi):
        out = []
        for r, (a, b) in enumerate(owners):
            x, y = max(lo, a), min(hi, b, n_train)
            if x < y:
                out.append((x, y, r))
        return out

    layers = {i: (lo, hi) for kind, i, lo, hi in plan if kind == "layer"}
    lo_all = min(lo for lo, _ in layers.values())
    hi_all = max(hi for _, hi in layers.values())
    out = [("vectors", pieces(hi_all, n_train))]
    out += [(("layer", i), pieces(*layers[i])) for i in sorted(layers)]
    out.append(("head", pieces(0, lo_all)))
    return out


class BucketReducer:
    """SUM-allreduces the flat gradient buffer bucket by bucket (engine/step.py:62's psum).

    ``reduce_range(lo, hi)`` enqueues the reduction of elements [lo, hi);
    ``before()`` runs before each one (it orders the collective after the
    kernels enqueued so far) and ``after()`` once at the end (it orders the
    next kernels after every collective). ``layer_done(i)`` is called after
    layer i's backward is enqueued: its bucket is reduced while the backward of
    the layers below continues. ``finish()`` reduces the remaining ranges (the
    head, the vector leaves and the loss/count tail).
    """

    def __init__(self, plan, reduce_range, before=None, after=None):
        self.reduce_range, self.before, self.after = reduce_range, before, after
        self.by_layer = {i: (lo, hi) for kind, i, lo, hi in plan if kind == "layer"}
        self.rest = [(lo, hi) for kind, _, lo, hi in plan if kind == "rest"]

    def _reduce(self, lo, hi):
        if self.before is not None:
            self.before()
        self.reduce_range(lo, hi)

    def layer_done(self, i):
        self._reduce(*self.by_layer[i])

    def finish(self):
        for lo, hi in self.rest:
            self._reduce(lo, hi)
        if self.after is not None:
            self.after()
