"""Write ``reference_kats.npz``: the reference test-suite's known answers.

Every array here is transcribed from the reference's own tests (inputs and
expected values as literals) or computed with the reference test's own
independent formula (the FP64 ``_oracle_attention`` of
tests/kernels/test_attention.py:40-58 and the nearest-level NF4 oracle of
tests/kernels/test_quantization.py:73-121), restated in this script. The
oracle package is deliberately *not* used, so the fixtures pin it.

Sources (paths inside the reference project):
  tests/kernels/test_quantization.py:10-23, 26-35, 38-49, 52-70, 73-121
  tests/kernels/test_bidirectional.py:13-27, 41-65
  tests/kernels/test_linear.py:20-41, 46-62
  tests/kernels/test_attention.py:16-126, 189-257, 306-346, 377-398

Run: ``python tests/golden/make_golden.py`` (deterministic; no GPU, no jax).
"""

import os

import numpy as np

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.npz")

NF4 = np.asarray(
    (-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
     -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
     0.07958029955625534, 0.16093020141124725, 0.24611230194568634,
     0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
     0.7229568362236023, 1.0),
    dtype=np.float32,
)

_B, _T, _P, _H, _HK, _D = 2, 6, 3, 4, 2, 8


def _arrays(*shapes, seed=0):
    g = np.random.default_rng(seed)
    return [np.asarray(g.normal(size=s), np.float32) for s in shapes]


def _oracle_attention(q, k, v, valid):
    rep = q.shape[2] // k.shape[2]
    k = np.repeat(k, rep, axis=2)
    v = np.repeat(v, rep, axis=2)
    s = np.einsum("bthd,bshd->bhts", q, k) * q.shape[-1] ** -0.5
    s = np.where(valid, s, np.finfo(np.float64).min)
    e = np.exp(s - s.max(axis=-1, keepdims=True))
    p = e / e.sum(axis=-1, keepdims=True)
    return np.einsum("bhts,bshd->bthd", p, v)


def _suffix_mask():
    return np.array([[1, 1, 1, 1, 0, 0], [1, 1, 1, 0, 0, 0]], np.int32)


def _causal_valid(m):
    pos = np.arange(m.shape[1])
    return (pos[:, None] >= pos[None, :])[None, None] & (m[:, None, None, :] > 0)


def main():
    g = {}
    # --- quantization -------------------------------------------------------
    w = np.zeros((1, 128), np.float32)
    w[0, :7] = [2, -2, 1, -1, 0.99, -0.99, 0]
    e = np.zeros_like(w)
    e[0, :7] = [2, -2, 2, -2, 0, 0, 0]
    g["ternary_halfaway_in"], g["ternary_halfaway_out"] = w, e

    w = np.zeros((2, 128), np.float32)
    w[0, :4] = [2.0, -2.0, 0.0, 0.16]
    e = np.zeros_like(w)
    e[0, :4] = [2.0, -2.0, 0.0, 2 * 0.07958029955625534]
    g["nf4_codebook_in"], g["nf4_codebook_out"] = w, e

    g["underflow_in"] = np.full((1, 128), 1e-9, np.float32)
    g["underflow_out"] = np.zeros((1, 128), np.float32)

    w = np.zeros((1, 128), np.float32)
    w[0, :7] = [
        1.0003, 0.5,
        np.nextafter(np.float32(0.5), np.float32(0)),
        np.nextafter(np.float32(0.5), np.float32(1)),
        -0.5,
        np.nextafter(np.float32(-0.5), np.float32(0)),
        np.nextafter(np.float32(-0.5), np.float32(-1)),
    ]
    e = np.zeros_like(w)
    e[0, :7] = [1, 1, 0, 1, -1, 0, -1]
    g["ternary_nextafter_in"], g["ternary_nextafter_out"] = w, e

    values = [np.float32(-1), np.float32(1)]
    for left, right in zip(NF4[:-1], NF4[1:]):
        mid = np.float32((np.float64(left) + np.float64(right)) / 2)
        values.extend((np.nextafter(mid, np.float32(-np.inf)), mid, np.nextafter(mid, np.float32(np.inf))))
    w = np.zeros((1, 128), np.float32)
    w[0, : len(values)] = values
    e = np.zeros_like(w)
    for i, x in enumerate(values):
        e[0, i] = NF4[int(np.argmin(np.abs(NF4.astype(np.float64) - np.float64(x))))]
    g["nf4_midpoints_in"], g["nf4_midpoints_out"] = w, e

    # --- bidirectional attention -------------------------------------------
    g["bidir_uniform_q"] = np.zeros((1, 3, 2, 2), np.float32)
    g["bidir_uniform_k"] = np.zeros((1, 3, 1, 2), np.float32)
    g["bidir_uniform_v"] = np.asarray([[[[2.0, 4.0]], [[6.0, 8.0]], [[99.0, 99.0]]]], np.float32)
    g["bidir_uniform_mask"] = np.asarray([[1, 1, 0]], np.int32)
    g["bidir_uniform_out"] = np.broadcast_to(np.asarray([4, 6], np.float32), (1, 3, 2, 2)).copy()
    g["bidir_uniform_dv"] = np.asarray([[[[3, 3]], [[3, 3]], [[0, 0]]]], np.float32)

    g["bidir_packed_q"] = np.zeros((1, 6, 2, 2), np.float32)
    g["bidir_packed_k"] = np.zeros((1, 6, 1, 2), np.float32)
    g["bidir_packed_v"] = np.asarray(
        [[2.0, 4.0], [6.0, 8.0], [1.0, 1.0], [2.0, 2.0], [6.0, 3.0], [99, 99]], np.float32
    ).reshape(1, 6, 1, 2)
    g["bidir_packed_seg"] = np.asarray([[1, 1, 2, 2, 2, 0]], np.int32)
    exp = np.asarray([[4, 6]] * 2 + [[3, 2]] * 3 + [[0, 0]], np.float32)
    g["bidir_packed_out"] = np.broadcast_to(exp[None, :, None], (1, 6, 2, 2)).copy()
    g["bidir_packed_dv"] = np.asarray([[2, 2]] * 5 + [[0, 0]], np.float32).reshape(1, 6, 1, 2)

    # --- linear ------------------------------------------------------------
    x = np.array([[[0.25, -0.5], [1.5, 0.75]]], np.float32)
    wt = np.array([[0.5, -0.25], [0.125, 0.75]], np.float32)
    probe = np.array([[[1.0, -2.0], [0.5, 3.0]]], np.float32)
    g["linear_x"], g["linear_w"], g["linear_probe"] = x, wt, probe
    g["linear_out"] = x @ wt.T
    g["linear_dx"] = probe @ wt
    g["linear_dw"] = probe.reshape(-1, 2).T @ x.reshape(-1, 2)
    g["linear_cast_x"] = np.array([[1024.0, -1024.0]], np.float32)
    g["linear_cast_w"] = np.array([[1.0002, 1.0]], np.float32)
    g["linear_cast_out"] = np.array([[0.0]], np.float32)
    g["linear_cast_dx"] = np.array([[1.0, 1.0]], np.float32)
    g["linear_cast_dw"] = np.array([[1024.0, -1024.0]], np.float32)

    # --- attention (FP64 oracle of the reference's attention tests) ---------
    q, k, v = _arrays((_B, _T, _H, _D), (_B, _T, _HK, _D), (_B, _T, _HK, _D))
    m = _suffix_mask()
    g["causal_q"], g["causal_k"], g["causal_v"], g["causal_mask"] = q, k, v, m
    g["causal_out"] = _oracle_attention(q.astype(np.float64), k.astype(np.float64), v.astype(np.float64),
                                        _causal_valid(m.astype(np.float64)))

    q, pk, pv, k, v = _arrays((_B, _T, _H, _D), (_B, _P, _HK, _D), (_B, _P, _HK, _D),
                              (_B, _T, _HK, _D), (_B, _T, _HK, _D), seed=1)
    pm = np.array([[1, 1, 0], [1, 0, 0]], np.int32)
    prefix = np.broadcast_to(pm[:, None, None, :] > 0, (_B, 1, _T, _P))
    valid = np.concatenate((prefix, _causal_valid(m)), axis=-1)
    g.update(prefix_q=q, prefix_pk=pk, prefix_pv=pv, prefix_k=k, prefix_v=v, prefix_pmask=pm, prefix_smask=m)
    g["prefix_out"] = _oracle_attention(q.astype(np.float64), np.concatenate((pk, k), 1).astype(np.float64),
                                        np.concatenate((pv, v), 1).astype(np.float64), valid)

    q, k, v = _arrays((_B, _T, _H, _D), (_B, _T, _HK, _D), (_B, _T, _HK, _D), seed=2)
    mask = np.array([[1, 1, 1, 1, 1, 0], [1, 1, 1, 0, 0, 0]], np.int32)
    seg = np.array([[1, 1, 1, 2, 2, 0], [1, 1, 2, 0, 0, 0]], np.int32)
    pos = np.arange(_T)
    causal = pos[:, None] >= pos[None, :]
    active = (mask > 0) & (seg != 0)
    same = seg[:, :, None] == seg[:, None, :]
    pv_ = causal[None] & same & (seg[:, :, None] != 0) & active[:, None, :] & active[:, :, None]
    pv_ = pv_ | ((~active)[:, :, None] & (pos[:, None] == pos[None, :])[None])
    out = _oracle_attention(q.astype(np.float64), k.astype(np.float64), v.astype(np.float64), pv_[:, None])
    g.update(packed_q=q, packed_k=k, packed_v=v, packed_mask=mask, packed_seg=seg)
    g["packed_out"] = out * active[:, :, None, None]

    q, k, v = _arrays((_B, 1, _H, _D), (_B, _T, _HK, _D), (_B, _T, _HK, _D), seed=3)
    valid = np.broadcast_to(np.arange(_T)[None, None, None, :] < 4, (_B, 1, 1, _T))
    g.update(cached_q=q, cached_k=k, cached_v=v, cached_len=np.array(4, np.int32))
    g["cached_out"] = _oracle_attention(q.astype(np.float64), k.astype(np.float64), v.astype(np.float64), valid)

    np.savez_compressed(OUT, **{k: np.ascontiguousarray(v) for k, v in g.items()})
    print(f"wrote {OUT} ({len(g)} arrays)")


if __name__ == "__main__":
    main()
