"""Shared helpers for the parity tests."""

import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# Correctness gate for floating-point outputs (bf16 storage) against the FP32/FP64
# oracle: max-abs 2e-2 and relative L2 1e-2. With ``scaled=True`` (gradients and
# GEMM outputs, whose entries grow past O(1)) the max-abs bound is applied per
# element in units of max(1, |reference value|, RMS(reference tensor)): a bf16
# value of magnitude m carries a storage error of up to m * 2^-9 by itself, and
# a sum over K bf16-rounded products carries an absolute error proportional to
# the sum's typical (RMS) magnitude, also for entries that happen to be near 0.
MAX_ABS = 2e-2
REL_L2 = 1e-2


def assert_close(actual, expected, max_abs=MAX_ABS, rel_l2=REL_L2, scaled=False, what=""):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, f"{what}: shape {a.shape} != {e.shape}"
    unit = np.maximum(max(1.0, float(np.sqrt(np.mean(e * e)))), np.abs(e)) if scaled else 1.0
    err = float(np.max(np.abs(a - e) / unit)) if a.size else 0.0
    norm = float(np.linalg.norm(e))
    rl2 = float(np.linalg.norm(a - e)) / norm if norm > 0 else float(np.linalg.norm(a - e))
    assert err <= max_abs, f"{what}: max-abs {err:.3e} > {max_abs:.3e}" + (" (per-element units)" if scaled else "")
    assert rl2 <= rel_l2, f"{what}: rel-L2 {rl2:.3e} > {rel_l2:.1e}"
    return err, rl2


def report_errors(what, actual, expected):
    """Append the unscaled max-abs, the per-element-scaled max-abs and the rel-L2 of one comparison to
    the JSON-lines file named by MFB_PARITY_REPORT (no-op when unset), so the raw errors behind the
    scaled gradient gate can be read off a test run."""
    path = os.environ.get("MFB_PARITY_REPORT")
    if not path:
        return
    import json

    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    unit = np.maximum(max(1.0, float(np.sqrt(np.mean(e * e)))), np.abs(e))
    norm = float(np.linalg.norm(e))
    rec = {"what": what, "max_abs": float(np.max(np.abs(a - e))) if a.size else 0.0,
           "max_abs_scaled": float(np.max(np.abs(a - e) / unit)) if a.size else 0.0,
           "rel_l2": float(np.linalg.norm(a - e)) / norm if norm > 0 else 0.0,
           "ref_max_abs": float(np.max(np.abs(e))) if e.size else 0.0,
           "ref_rms": float(np.sqrt(np.mean(e * e))) if e.size else 0.0}
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "a") as fh:
        fh.write(json.dumps(rec) + "\n")


def header_functions():
    """Names of every function declared in include/*.h."""
    names = []
    inc = os.path.join(ROOT, "include")
    for fn in sorted(os.listdir(inc)):
        if fn.endswith(".h"):
            text = open(os.path.join(inc, fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"\b(mfb_\w+)\s*\(", text)
    return sorted(set(names))


def run_ranks(ctx, target, args_per_rank, timeout_s):
    """Run one child process per rank and wait for all of them, bounded.

    Every rank shares one deadline. A rank still alive at the deadline is
    killed (and reaped), so a stalled rank fails this test instead of keeping
    its GPU context and blocking the interpreter's exit; the assertion names
    the ranks that timed out or exited nonzero.
    """
    import time

    procs = [ctx.Process(target=target, args=args) for args in args_per_rank]
    for p in procs:
        p.start()
    deadline = time.monotonic() + timeout_s
    try:
        for p in procs:
            p.join(max(0.0, deadline - time.monotonic()))
    finally:
        hung = [r for r, p in enumerate(procs) if p.is_alive()]
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(5)
    failed = [(r, p.exitcode) for r, p in enumerate(procs) if p.exitcode != 0 and r not in hung]
    assert not hung and not failed, f"ranks timed out after {timeout_s} s: {hung}; ranks failed (exit code): {failed}"
