"""Seeded synthetic inputs for the five benchmark configurations.

No dataset is involved: every configuration is synthetic, drawn from
``numpy.random.default_rng(seed)`` in FP32 (the GPU receives bf16 copies).
Packed rows follow the reference's packing convention
(src/minifield_training/batching/packing.py:20-31): segment ids 1..n in row
order, 0 for padding.
"""

from dataclasses import dataclass

import numpy as np

# LFM2.5-350M attention-layer shape (tests/models/lfm2_5/fixtures/encoder_config.json).
HEADS, KV_HEADS, HEAD_DIM, HIDDEN = 16, 8, 64, 1024
ATTENTION_LAYERS = (2, 5, 8, 10, 12, 14)


def packed_segments(seed: int, batch: int, length: int, lo: int = 32, hi: int = 1024) -> np.ndarray:
    """int32 [batch, length] segment ids.

    Per row, lengths L ~ U[lo, hi] (inclusive) are appended while the row has
    room; the last one is truncated to fill the row exactly, and a truncated
    remainder shorter than ``lo`` stays padding (id 0).
    """
    rng = np.random.default_rng(seed)
    ids = np.zeros((batch, length), np.int32)
    for b in range(batch):
        pos, sid = 0, 1
        while pos < length:
            seg = int(rng.integers(lo, hi + 1))
            if pos + seg > length:
                seg = length - pos
                if seg < lo:
                    break
            ids[b, pos : pos + seg] = sid
            pos += seg
            sid += 1
    return ids


def segment_square_sum(segment_ids: np.ndarray) -> int:
    """Sum over rows and nonzero segments of L^2 (valid bidirectional pairs)."""
    total = 0
    for row in segment_ids:
        _, counts = np.unique(row[row != 0], return_counts=True)
        total += int((counts.astype(np.int64) ** 2).sum())
    return total


@dataclass(frozen=True)
class AttentionConfig:
    name: str
    batch: int
    length: int
    heads: int = HEADS
    kv_heads: int = KV_HEADS
    head_dim: int = HEAD_DIM
    causal: bool = True
    packed: bool = False


CONFIG1 = AttentionConfig("cfg1-dense-causal-gqa-fwd-bwd", batch=4, length=512, causal=True, packed=False)
CONFIG2 = AttentionConfig("cfg2-segment-bidirectional-gqa-fwd-bwd", batch=8, length=2048, causal=False, packed=True)


def attention_inputs(cfg: AttentionConfig, seed: int = 0):
    """(q, k, v, d_out, mask, segment_ids) with q,k,v,dO ~ N(0, 1) FP32."""
    rng = np.random.default_rng(seed)
    b, t = cfg.batch, cfg.length
    q = rng.standard_normal((b, t, cfg.heads, cfg.head_dim), dtype=np.float32)
    k = rng.standard_normal((b, t, cfg.kv_heads, cfg.head_dim), dtype=np.float32)
    v = rng.standard_normal((b, t, cfg.kv_heads, cfg.head_dim), dtype=np.float32)
    d_out = rng.standard_normal((b, t, cfg.heads, cfg.head_dim), dtype=np.float32)
    if cfg.packed:
        seg = packed_segments(seed, b, t)
        mask = (seg != 0).astype(np.int32)
    else:
        seg = None
        mask = np.ones((b, t), np.int32)
    return q, k, v, d_out, mask, seg


def attention_flops(cfg: AttentionConfig, segment_ids=None) -> tuple[float, float]:
    """(algorithmic fwd+bwd FLOPs, dense-equivalent fwd+bwd FLOPs).

    fwd = 4 * H * D * (valid pairs); bwd = 2.5 x fwd.
    """
    h, d, b, t = cfg.heads, cfg.head_dim, cfg.batch, cfg.length
    dense_pairs = b * t * t
    if segment_ids is not None:
        pairs = segment_square_sum(segment_ids)
    elif cfg.causal:
        pairs = b * t * t / 2.0
    else:
        pairs = dense_pairs
    return 3.5 * 4.0 * h * d * pairs, 3.5 * 4.0 * h * d * dense_pairs


@dataclass(frozen=True)
class DecodeConfig:
    name: str = "cfg3-kv-cached-gqa-decode-6-layers"
    batch: int = 64
    capacity: int = 4096
    layers: int = 6
    heads: int = HEADS
    kv_heads: int = KV_HEADS
    head_dim: int = HEAD_DIM
    min_len: int = 256


CONFIG3 = DecodeConfig()


def decode_lengths(cfg: DecodeConfig, seed: int = 0) -> np.ndarray:
    """Filled lengths per sequence (after the step's write) ~ U[min_len, capacity]."""
    rng = np.random.default_rng(seed)
    return rng.integers(cfg.min_len, cfg.capacity + 1, size=cfg.batch).astype(np.int32)


def decode_layer_bytes(lengths, cfg: DecodeConfig, elem: int = 2) -> int:
    """Algorithmic HBM bytes of one layer's decode step.

    Reads of the valid K and V prefix (lengths include the new token), the
    query read, the output write and the new key/value read + cache write.
    """
    lengths = np.asarray(lengths, np.int64)
    b = lengths.shape[0]
    kv = int(lengths.sum()) * cfg.kv_heads * cfg.head_dim * 2 * elem
    qo = b * cfg.heads * cfg.head_dim * 2 * elem
    new = b * cfg.kv_heads * cfg.head_dim * 2 * elem * 2
    return kv + qo + new


def decode_layer_inputs(cfg: DecodeConfig, seed: int, layer: int = 0, batch=None, capacity=None):
    """(q [B,H,D], k_cache, v_cache [B,cap,Hk,D], new_k, new_v [B,Hk,D]) ~ N(0, 0.02)."""
    b = cfg.batch if batch is None else batch
    cap = cfg.capacity if capacity is None else capacity
    rng = np.random.default_rng(seed * 1000 + layer + 1)
    s = np.float32(0.02)
    q = rng.standard_normal((b, cfg.heads, cfg.head_dim), dtype=np.float32) * s
    kc = rng.standard_normal((b, cap, cfg.kv_heads, cfg.head_dim), dtype=np.float32) * s
    vc = rng.standard_normal((b, cap, cfg.kv_heads, cfg.head_dim), dtype=np.float32) * s
    nk = rng.standard_normal((b, cfg.kv_heads, cfg.head_dim), dtype=np.float32) * s
    nv = rng.standard_normal((b, cfg.kv_heads, cfg.head_dim), dtype=np.float32) * s
    return q, kc, vc, nk, nv


@dataclass(frozen=True)
class QatConfig:
    name: str = "cfg4-qat-swiglu-ffn-fwd-bwd"
    tokens: int = 16384
    hidden: int = HIDDEN
    ffn: int = 6656
    kind: str = "int8-channel-absmax-v1"


CONFIG4 = QatConfig()


def qat_inputs(cfg: QatConfig, seed: int = 0, tokens=None):
    """(x [M,C] ~ N(0,1), w_gate_up [2F,C], w_down [C,F] ~ N(0,0.02), d_y [M,C] ~ N(0,1))."""
    m = cfg.tokens if tokens is None else tokens
    rng = np.random.default_rng(seed)
    s = np.float32(0.02)
    x = rng.standard_normal((m, cfg.hidden), dtype=np.float32)
    w_gu = rng.standard_normal((2 * cfg.ffn, cfg.hidden), dtype=np.float32) * s
    w_d = rng.standard_normal((cfg.hidden, cfg.ffn), dtype=np.float32) * s
    d_y = rng.standard_normal((m, cfg.hidden), dtype=np.float32)
    return x, w_gu, w_d, d_y


# ---- config 5: data-parallel encoder training step -------------------------------
ENCODER_LAYERS = ("conv", "conv", "full_attention", "conv", "conv", "full_attention", "conv", "conv",
                  "full_attention", "conv", "full_attention", "conv", "full_attention", "conv", "full_attention",
                  "conv")  # tests/models/lfm2_5/fixtures/encoder_config.json layer_types


@dataclass(frozen=True)
class EncoderStepConfig:
    name: str = "cfg5-encoder-dp-qat-train-step"
    global_batch: int = 32
    length: int = 2048
    hidden: int = 1024
    ffn: int = 6656
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 64
    layer_types: tuple = ENCODER_LAYERS
    vocab: int = 65536
    classes: int = 2
    norm_eps: float = 1e-5
    rope_theta: float = 1e6
    quant: str = "int8-channel-absmax-v1"
    learning_rate: float = 3e-4
    beta1: float = 0.9
    beta2: float = 0.95
    weight_decay: float = 0.1
    epsilon: float = 1e-8
    clip_norm: float = 1.0


CONFIG5 = EncoderStepConfig()


def encoder_batch(cfg: EncoderStepConfig, seed: int, rows=None, row0: int = 0):
    """Synthetic packed batch rows [row0, row0 + rows) of the global batch of step ``seed``.

    Returns int32 arrays [rows, T]: token ids ~ U[0, vocab), attention mask
    (segment != 0), segment ids (config-2 packing), per-segment positions and
    class labels ~ U[0, classes).
    """
    rows = cfg.global_batch if rows is None else rows
    seg = packed_segments(seed, cfg.global_batch, cfg.length)[row0:row0 + rows]
    rng = np.random.default_rng(seed + 1_000_003)
    ids = rng.integers(0, cfg.vocab, (cfg.global_batch, cfg.length)).astype(np.int32)[row0:row0 + rows]
    labels = rng.integers(0, cfg.classes, (cfg.global_batch, cfg.length)).astype(np.int32)[row0:row0 + rows]
    mask = (seg != 0).astype(np.int32)
    pos = np.zeros_like(seg)
    for r in range(rows):
        start = 0
        for t in range(1, cfg.length + 1):
            if t == cfg.length or seg[r, t] != seg[r, start]:
                pos[r, start:t] = np.arange(t - start)
                start = t
    pos[seg == 0] = 0
    return ids, mask, seg.astype(np.int32), pos.astype(np.int32), labels


def encoder_matmul_params(cfg: EncoderStepConfig) -> int:
    """Parameters that take part in a matrix product per token (the head excluded)."""
    c, f, kv = cfg.hidden, cfg.ffn, cfg.kv_heads * cfg.head_dim
    n = 0
    for kind in cfg.layer_types:
        n += 3 * c * f
        n += (3 * c * c + c * c) if kind == "conv" else (c * c + 2 * kv * c + c * c)
    return n


def encoder_step_flops(cfg: EncoderStepConfig, segment_ids) -> float:
    """6 * matmul params * tokens + attention fwd+bwd (3.5 x 4 H D sum L^2 per attention layer)."""
    tokens = segment_ids.size
    attn = sum(1 for k in cfg.layer_types if k != "conv") * 3.5 * 4 * cfg.heads * cfg.head_dim * \
        segment_square_sum(segment_ids)
    return 6.0 * encoder_matmul_params(cfg) * tokens + attn


@dataclass(frozen=True)
class DecoderConfig:
    """The LFM2.5 causal decoder's dimensions for cached decoding
    (src/minifield_training/models/lfm2_5/model.py:28-47; the 350M layout: 16
    layers, attention at 2, 5, 8, 10, 12, 14, tied embeddings)."""

    name: str = "lfm2.5-350m-decode-one"
    hidden: int = 1024
    ffn: int = 6656
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 64
    vocab: int = 65536
    layer_types: tuple = ENCODER_LAYERS
    conv_kernel: int = 3
    norm_eps: float = 1e-5
    rope_theta: float = 1000000.0
    max_position_embeddings: int = 128000


DECODER = DecoderConfig()
