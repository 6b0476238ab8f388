#!/usr/bin/env python
"""Benchmark of the B200 hot path (one JSON line on rank 0).

Headline workload (the config its attention metric
is quoted on): segment-masked bidirectional GQA attention forward+backward,
B=8, T=2048, 16/8 heads, head_dim 64, bf16, packed segments U[32,1024].
A step = one forward + backward over the batch through the C ABI
(ids -> forward -> backward). ``value`` = algorithmic TFLOP/s (4*H*D per valid
query/key pair forward, x3.5 forward+backward) over all ranks. Secondary
measurements in the same line: KV-cached decode over 6 layers (config 3,
tokens/s and HBM GB/s), the QAT SwiGLU FFN forward+backward (config 4,
tokens/s and TFLOP/s) and the data-parallel encoder training step (config 5:
16-layer QAT encoder forward+backward, gradient allreduce, AdamW commit;
tokens/s of the fixed global batch of 32 x 2048).

Multi-GPU: one process per GPU (torchrun). Configs 1-4 run one copy per rank
(weak scaling, no collective on their data path). Config 5 splits the global
batch's rows over the ranks (strong scaling) and all-reduces the gradient sums
over NCCL (the library's own communicator, mfb_comm_*), bucket by bucket
during the backward. Timing is the max over ranks of CUDA-event time between
barriers; torch.distributed (gloo) carries only the barrier, the max over
ranks and the NCCL unique id.

``--impl reference`` times the reference algorithm's CPU restatement (the
NumPy oracle; the reference itself is JAX, which is not installed on these
machines) on the host cores, rank 0 only.
"""

import argparse
import ctypes
import json
import os
import subprocess
import sys
import time

os.environ.setdefault("OPENBLAS_NUM_THREADS", str(os.cpu_count() or 1))

import numpy as np  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "attn TFLOP/s (% of peak); KV-decode tokens/s; QAT step tokens/s at 1/2/4/8 GPU"
UNIT = "TFLOP/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-secondary", action="store_true", help="skip the decode / QAT secondary measurements")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", choices=["attention", "attention_cfg1", "decode", "decode_one", "qat", "encoder"],
                    default=None,
                    help="run one workload (profiling); the JSON line then carries only its numbers")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# Distributed plumbing (barrier + max over ranks only).
# ---------------------------------------------------------------------------


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
            self.pg = dist

    def communicator(self):
        """The library's NCCL communicator over all ranks for the gradient exchange (None on one GPU).

        Rank 0 draws the NCCL unique id; the gloo group hands it to the others.
        """
        if not self.pg:
            return None
        if getattr(self, "_comm", None) is None:
            from minifield_training_b200 import comm

            box = [comm.unique_id() if self.rank == 0 else None]
            self.pg.broadcast_object_list(box, src=0)
            self._comm = comm.Communicator(self.world, self.rank, box[0], timeout_s=300.0)
        return self._comm

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch

        t = torch.tensor([x], dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        c = getattr(self, "_comm", None)
        if c is not None:
            c.close()
            self._comm = None
        if self.pg:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# Clock sampling during the timed region.
# ---------------------------------------------------------------------------


class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        """Samples go to MFB_CLOCKS_DIR when set (to keep the CSV), else to a temporary directory."""
        import tempfile

        self.index = index
        self.proc = None
        folder = os.environ.get("MFB_CLOCKS_DIR") or tempfile.mkdtemp(prefix="mfb_clocks_")
        self.path = os.path.join(folder, f"clocks_rank{index}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait()
        self.fh.close()
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# GPU workloads (C-ABI calls on preallocated buffers).
# ---------------------------------------------------------------------------


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return p["hbm_gbs"], p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def traffic_table():
    path = os.path.join(ROOT, "profiles", "traffic.json")
    return json.load(open(path)) if os.path.exists(path) else {}


class Timer:
    """CUDA events on the legacy default stream (the stream every call uses)."""

    def __init__(self):
        from minifield_training_b200.device import Event

        self.a, self.b = Event(), Event()

    def time(self, fn, iters: int) -> float:
        from minifield_training_b200.device import sync

        sync()
        self.a.record()
        for _ in range(iters):
            fn()
        self.b.record()
        sync()
        return self.a.elapsed_ms(self.b) / iters


class AttentionWorkload:
    """Config 2 (or 1): masked GQA attention forward + backward."""

    def __init__(self, cfg, seed):
        from minifield_training_b200 import _lib, workloads
        from minifield_training_b200.device import DeviceArray

        self.L = _lib
        self.cfg = cfg
        q, k, v, do, mask, seg = workloads.attention_inputs(cfg, seed)
        self.host = {"q": q, "k": k, "v": v, "do": do, "mask": mask, "seg": seg}
        b, t, h, d = q.shape
        hk = k.shape[2]
        self.dims = (b, t, t, h, hk, d)
        dev = DeviceArray.from_numpy
        self.q, self.k, self.v, self.do = (dev(x, "bfloat16") for x in (q, k, v, do))
        self.mask = dev(mask, "int32")
        self.seg = dev(seg, "int32") if seg is not None else None
        self.o = DeviceArray(q.shape, "bfloat16")
        self.lse = DeviceArray((b, h, t), "float32")
        self.dq = DeviceArray(q.shape, "bfloat16")
        self.dk = DeviceArray(k.shape, "bfloat16")
        self.dv = DeviceArray(v.shape, "bfloat16")
        self.qid = DeviceArray((b, t), "int32")
        self.kid = DeviceArray((b, t), "int32")
        ws = _lib.lib().mfb_attn_workspace_size(b, t, t, h, hk, d)
        self.ws = DeviceArray((ws,), "uint8")
        self.mode = _lib.MASK_BIDIR if not cfg.causal else _lib.MASK_CAUSAL
        pairs = workloads.segment_square_sum(seg) if seg is not None else b * t * (t + 1) / 2
        self.fwd_flops = 4.0 * h * d * pairs
        self.total_flops = 3.5 * self.fwd_flops
        self.causal = ctypes.c_int()
        self.offset = ctypes.c_int()
        self.policy = ctypes.c_int()
        self.stream = None  # CUDA stream of the three calls (None: the default stream)
        self.ids()

    def ids(self):
        P = ctypes.c_void_p
        b, t, s = self.dims[:3]
        self.L.call("mfb_attn_ids", self.mode, P(self.mask.ptr), P(self.seg.ptr) if self.seg else None, None,
                    P(self.qid.ptr), P(self.kid.ptr), b, t, s, 0, ctypes.byref(self.causal),
                    ctypes.byref(self.offset), ctypes.byref(self.policy), self.stream)

    def fwd(self):
        P = ctypes.c_void_p
        b, t, s, h, hk, d = self.dims
        self.L.call("mfb_attn_fwd", P(self.q.ptr), P(self.k.ptr), P(self.v.ptr), P(self.o.ptr), P(self.lse.ptr),
                    P(self.qid.ptr), P(self.kid.ptr), b, t, s, h, hk, d, self.causal.value, self.offset.value,
                    self.policy.value, ctypes.c_float(d ** -0.5), P(self.ws.ptr), self.ws.nbytes, self.stream)

    def bwd(self):
        P = ctypes.c_void_p
        b, t, s, h, hk, d = self.dims
        self.L.call("mfb_attn_bwd", P(self.q.ptr), P(self.k.ptr), P(self.v.ptr), P(self.o.ptr), P(self.lse.ptr),
                    P(self.do.ptr), P(self.dq.ptr), P(self.dk.ptr), P(self.dv.ptr), P(self.qid.ptr),
                    P(self.kid.ptr), b, t, s, h, hk, d, self.causal.value, self.offset.value, self.policy.value,
                    ctypes.c_float(d ** -0.5), P(self.ws.ptr), self.ws.nbytes, self.stream)

    def step(self):
        self.ids()
        self.fwd()
        self.bwd()

    launches_per_step = 8  # ids, ranges, schedule, fwd, bwd-pre (with the ranges), schedule, bwd-main, dq-convert

    def capture_graphs(self):
        """Capture the step, the forward alone and the backward alone as CUDA graphs on a created
        stream (config 1 is launch-latency bound: 9 small launches per step)."""
        sp = ctypes.c_void_p()
        self.L.call("mfb_stream_create", ctypes.byref(sp))
        self.stream = sp.value
        self.ids()  # host outputs (causal, offset, policy) set before capture
        self.graphs = {}
        for name, fn in (("step", self.step), ("fwd", self.fwd), ("bwd", self.bwd)):
            self.L.call("mfb_graph_begin", self.stream)
            fn()
            g = ctypes.c_void_p()
            self.L.call("mfb_graph_end", self.stream, ctypes.byref(g))
            self.graphs[name] = g.value

    def replay(self, name):
        self.L.call("mfb_graph_launch", self.graphs[name], self.stream)

    def release_graphs(self):
        self.L.call("mfb_stream_sync", self.stream)
        for g in self.graphs.values():
            self.L.call("mfb_graph_destroy", g)
        self.L.call("mfb_stream_destroy", self.stream)
        self.graphs, self.stream = {}, None

    def e2e_setup(self):
        """Pinned host buffers, a second device buffer set and three streams.

        The end-to-end loop pipelines consecutive steps the way a serving or
        training input pipeline would: step i uploads into buffer set i % 2 on
        one stream, computes on a second and downloads on a third, so step
        i + 1's upload and step i - 1's download (opposite PCIe directions)
        overlap step i's kernels. Every step still moves its whole input up
        and its whole output down inside the timed region.
        """
        from minifield_training_b200.device import Event, HostBuffer

        self.pin = {}
        for name in ("q", "k", "v", "do"):
            hb = HostBuffer(self.host[name].shape, np.uint16)
            hb.array[...] = self.host[name].astype(__import__("ml_dtypes").bfloat16).view(np.uint16)
            self.pin[name] = hb
        for name in ("mask", "seg"):
            if self.host[name] is not None:
                hb = HostBuffer(self.host[name].shape, np.int32)
                hb.array[...] = self.host[name]
                self.pin[name] = hb
        self.pin_out = {n: HostBuffer(getattr(self, n).shape, np.uint16) for n in ("o", "dq", "dk", "dv")}
        self.h2d_bytes = sum(hb.array.nbytes for hb in self.pin.values())
        self.d2h_bytes = sum(hb.array.nbytes for hb in self.pin_out.values())
        self.twin = AttentionWorkload(self.cfg, seed=0)
        streams = []
        for _ in range(3):
            sp = ctypes.c_void_p()
            self.L.call("mfb_stream_create", ctypes.byref(sp))
            streams.append(sp.value)
        self.s_in, self.s_comp, self.s_out = streams
        self.e2e_sets = []
        for w in (self, self.twin):
            w.stream = self.s_comp
            self.e2e_sets.append((w, Event(), Event(), Event()))  # uploaded, computed, downloaded
        self.e2e_i = 0

    def e2e_close(self):
        """Finish the pipelined steps and release their streams."""
        self.L.call("mfb_device_sync")
        for s in (self.s_in, self.s_comp, self.s_out):
            self.L.call("mfb_stream_destroy", s)
        self.stream = self.twin.stream = None

    def e2e_step(self):
        from minifield_training_b200.device import d2h, h2d

        w, up, comp, down = self.e2e_sets[self.e2e_i % 2]
        self.e2e_i += 1
        dev = {"q": w.q, "k": w.k, "v": w.v, "do": w.do, "mask": w.mask, "seg": w.seg}
        comp.wait_on(self.s_in)  # the set's inputs were read by its previous step
        for name, hb in self.pin.items():
            h2d(dev[name], hb.ptr, hb.array.nbytes, self.s_in)
        up.record(self.s_in)
        up.wait_on(self.s_comp)
        down.wait_on(self.s_comp)  # the set's outputs of its previous step are downloaded
        w.step()
        comp.record(self.s_comp)
        comp.wait_on(self.s_out)
        for name, hb in self.pin_out.items():
            d2h(hb.ptr, getattr(w, name), hb.array.nbytes, self.s_out)
        down.record(self.s_out)


class DecodeWorkload:
    """Config 3: one decode step over 6 attention layers (append + split-K attention)."""

    def __init__(self, seed):
        from minifield_training_b200 import _lib, workloads
        from minifield_training_b200.device import DeviceArray

        self.L = _lib
        cfg = workloads.CONFIG3
        self.cfg = cfg
        lens = workloads.decode_lengths(cfg, seed)
        self.lens = lens
        dev = DeviceArray.from_numpy
        self.layers = []
        for layer in range(cfg.layers):
            q, kc, vc, nk, nv = workloads.decode_layer_inputs(cfg, seed, layer)
            self.layers.append(tuple(dev(x, "bfloat16") for x in (q, kc, vc, nk, nv)))
        self.pos = dev(lens - 1, "int32")
        self.vl = dev(lens, "int32")
        self.o = DeviceArray((cfg.batch, cfg.heads, cfg.head_dim), "bfloat16")
        ws = _lib.lib().mfb_decode_workspace_size(cfg.batch, cfg.capacity, cfg.heads, cfg.head_dim)
        self.ws = DeviceArray((ws,), "uint8")
        self.bytes = cfg.layers * workloads.decode_layer_bytes(lens, cfg)

    def layer(self, i):
        P = ctypes.c_void_p
        q, kc, vc, nk, nv = self.layers[i]
        c = self.cfg
        self.L.call("mfb_decode_attn", P(q.ptr), P(kc.ptr), P(vc.ptr), P(nk.ptr), P(nv.ptr), P(self.pos.ptr),
                    P(self.vl.ptr), P(self.o.ptr), c.batch, c.capacity, c.heads, c.kv_heads, c.head_dim,
                    ctypes.c_float(c.head_dim ** -0.5), P(self.ws.ptr), self.ws.nbytes, None)

    def step(self):
        for i in range(self.cfg.layers):
            self.layer(i)

    launches_per_step = 6


class DecodeOneWorkload:
    """The LFM2.5 decoder's cached generation (decode.py:373-466): prefill of a
    1024-token prompt for 64 rows into 4096-slot caches, then single-token
    decode_one steps replayed as one CUDA graph each."""

    batch, capacity, prompt = 64, 4096, 1024

    def __init__(self, seed):
        from minifield_training_b200 import _lib, workloads
        from minifield_training_b200.device import DeviceArray
        from minifield_training_b200.models import decode

        self.L, self.dm, cfg = _lib, decode, workloads.DECODER
        self.cfg = cfg
        s = ctypes.c_void_p()
        _lib.call("mfb_stream_create", ctypes.byref(s))
        self.stream = s.value
        self.dec = decode.Decoder(cfg, decode.init_parameters(cfg, seed), stream=self.stream)
        rng = np.random.default_rng(seed)
        self.prompt = rng.integers(0, cfg.vocab, (self.batch, self.prompt)).astype(np.int32)
        self.tokens = rng.integers(0, cfg.vocab, (self.capacity, self.batch)).astype(np.int32)
        self.out = DeviceArray((self.batch, cfg.vocab), "float32")
        self.state = None

    def prefill(self):
        self.state = self.dm.new_state(self.cfg, self.batch, self.capacity)
        self.dec.prefill(self.prompt, self.state)

    def step(self):
        st = self.state
        self.dec.decode_one(self.tokens[st.valid_length], st, out=self.out, graph=True)

    def bytes_per_step(self, first_length, steps):
        """HBM bytes one step must move, averaged over steps that start at first_length valid keys:
        the bf16 weights of every projection and the tied head, the valid K/V cache rows of the
        attention layers (plus the appended row), the gathered FP32 embedding rows and the logits
        (bf16 product written and read, FP32 written)."""
        cfg, b = self.cfg, self.batch
        c, f, kv, q = cfg.hidden, cfg.ffn, cfg.kv_heads * cfg.head_dim, cfg.heads * cfg.head_dim
        weights = 0
        for kind in cfg.layer_types:
            weights += 3 * f * c + (4 * c * c if kind == "conv" else (q + 2 * kv) * c + c * q)
        weights = 2 * (weights + cfg.vocab * c)
        n_attn = sum(1 for k in cfg.layer_types if k == "full_attention")
        mean_len = first_length + (steps + 1) / 2.0
        cache = n_attn * b * mean_len * kv * 2 * 2
        return weights + cache + b * c * 4 + b * cfg.vocab * (2 + 2 + 4)

    def close(self):
        self.dec.close()
        self.L.call("mfb_stream_sync", self.stream)
        self.L.call("mfb_stream_destroy", self.stream)

    def kernels_per_step(self):
        """Kernels one graph replay runs: a split-K GEMM is the GEMM and its reduce."""
        cfg, b = self.cfg, self.batch
        c, f, nq = cfg.hidden, cfg.ffn, (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim

        def gemm(n, k):
            return 2 if self.L.lib().mfb_gemm_workspace_size(b, n, k) > 0 else 1

        n = 1 + 1 + gemm(cfg.vocab, c) + 1  # embedding gather, final norm, tied head, FP32 cast
        for kind in cfg.layer_types:
            n += 2 + gemm(2 * f, c) + 1 + gemm(c, f)  # two norms, w1|w3, SwiGLU, w2
            if kind == "conv":
                n += gemm(3 * c, c) + 1 + gemm(c, c)  # in-proj, conv step, out-proj
            else:
                n += gemm(nq, c) + 2 + gemm(c, cfg.heads * cfg.head_dim)  # q|k|v, qk-norm+RoPE, attention, out
        return n


class QatWorkload:
    """Config 4: int8 fake-quant + SwiGLU FFN GEMM chain forward + backward."""

    def __init__(self, seed, kind=None):
        from minifield_training_b200 import _lib, workloads
        from minifield_training_b200.device import DeviceArray

        self.L = _lib
        cfg = workloads.CONFIG4
        self.cfg = cfg
        self.kind_name = kind or cfg.kind
        x, w_gu, w_d, dy = workloads.qat_inputs(cfg, seed)
        dev = DeviceArray.from_numpy
        m, c, f = cfg.tokens, cfg.hidden, cfg.ffn
        self.m, self.c, self.f = m, c, f
        self.x, self.dy = dev(x, "bfloat16"), dev(dy, "bfloat16")
        self.w_gu, self.w_d = dev(w_gu, "float32"), dev(w_d, "float32")
        self.e_gu, self.e_d = DeviceArray((2 * f, c), "bfloat16"), DeviceArray((c, f), "bfloat16")
        self.s_gu, self.s_d = DeviceArray((2 * f, c), "uint8"), DeviceArray((c, f), "uint8")
        self.gu = DeviceArray((m, 2 * f), "bfloat16")
        self.h = DeviceArray((m, f), "bfloat16")
        self.y = DeviceArray((m, c), "bfloat16")
        self.dgu = DeviceArray((m, 2 * f), "bfloat16")
        self.dx = DeviceArray((m, c), "bfloat16")
        self.dw_gu = DeviceArray((2 * f, c), "float32")
        self.dw_d = DeviceArray((c, f), "float32")
        self.kind = _lib.QUANT_KINDS[self.kind_name]
        self.flops = 3.0 * (2.0 * m * c * 2 * f + 2.0 * m * f * c)
        # Split-K partials for the GEMMs whose output tiles fill the GPU poorly (the weight gradients).
        shapes = [(m, c, f), (c, f, m), (m, c, 2 * f), (2 * f, c, m)]
        sizes = [int(_lib.lib().mfb_gemm_workspace_size(*s)) for s in shapes]
        self.gemm_ws = DeviceArray((max(16, max(sizes)),), "uint8")
        # Two fake-quant passes, six GEMMs (two with SwiGLU epilogues), one reduce per split GEMM.
        self.launches_per_step = 8 + sum(1 for z in sizes if z > 0)

    def gemm(self, a, am, lda, b, bm, ldb, c, ldc, dt, m, n, k, mask=None):
        P = ctypes.c_void_p
        self.L.call("mfb_gemm_bf16_ws", P(a.ptr), am, lda, P(b.ptr), bm, ldb, P(c.ptr), ldc, dt, m, n, k,
                    ctypes.c_float(1.0), P(mask.ptr) if mask is not None else None, 0, P(self.gemm_ws.ptr),
                    self.gemm_ws.nbytes, None)

    def step(self):
        P = ctypes.c_void_p
        L = self.L
        m, c, f = self.m, self.c, self.f
        K, MN, BF, F32 = L.MAJOR_K, L.MAJOR_MN, L.DTYPE_BF16, L.DTYPE_F32
        L.call("mfb_fakequant", P(self.w_gu.ptr), self.kind, 2 * f, c, None, None, P(self.s_gu.ptr), None,
               P(self.e_gu.ptr), None)
        L.call("mfb_fakequant", P(self.w_d.ptr), self.kind, c, f, None, None, P(self.s_d.ptr), None,
               P(self.e_d.ptr), None)
        # gate|up GEMM with the SwiGLU product in its epilogue, then the down projection
        L.call("mfb_gemm_swiglu_fwd", P(self.x.ptr), K, c, P(self.e_gu.ptr), c, P(self.gu.ptr), P(self.h.ptr), m, f,
               c, None)
        self.gemm(self.h, K, f, self.e_d, K, f, self.y, c, BF, m, c, f)
        # dH = dY . W_down with the SwiGLU backward in its epilogue (writes dGU), then the weight gradients
        L.call("mfb_gemm_swiglu_bwd", P(self.dy.ptr), K, c, P(self.e_d.ptr), MN, f, P(self.gu.ptr), P(self.dgu.ptr),
               m, f, c, None)
        self.gemm(self.dy, MN, c, self.h, MN, f, self.dw_d, f, F32, c, f, m, mask=self.s_d)
        self.gemm(self.dgu, K, 2 * f, self.e_gu, MN, c, self.dx, c, BF, m, c, 2 * f)
        self.gemm(self.dgu, MN, 2 * f, self.x, MN, c, self.dw_gu, c, F32, 2 * f, c, m, mask=self.s_gu)


# ---------------------------------------------------------------------------
# CPU legs (oracle restatement of the reference algorithm).
# ---------------------------------------------------------------------------


class EncoderStepWorkload:
    """Config 5: one data-parallel QAT encoder training step over this rank's rows."""

    def __init__(self, dist):
        from minifield_training_b200 import _lib, workloads
        from minifield_training_b200.device import HostBuffer
        from minifield_training_b200.models import encoder as me

        cfg = workloads.CONFIG5
        if cfg.global_batch % dist.world:
            raise ValueError("the global batch must split evenly over the ranks")
        self.cfg, self.rows = cfg, cfg.global_batch // dist.world
        # A created stream, so the step can be captured and replayed as CUDA graphs.
        s = ctypes.c_void_p()
        _lib.call("mfb_stream_create", ctypes.byref(s))
        self.stream = s.value
        # With several ranks the optimizer is sharded: each rank updates the arena range it owns
        # and broadcasts it (overlapped with the next forward), instead of every rank running the
        # whole AdamW transaction.
        self.model = me.EncoderStep(cfg, rows=self.rows, seed=0, comm=dist.communicator(), stream=self.stream,
                                    shard_optimizer=dist.world > 1)
        self.batch = workloads.encoder_batch(cfg, 0, rows=self.rows, row0=dist.rank * self.rows)
        self.model.set_batch(*self.batch)
        full_seg = workloads.packed_segments(0, cfg.global_batch, cfg.length)
        self.global_flops = workloads.encoder_step_flops(cfg, full_seg)
        self.tokens = cfg.global_batch * cfg.length
        # Pinned host copies of the step inputs for the end-to-end leg.
        self.host = [HostBuffer(a.shape, np.int32) for a in self.batch]
        for h, a in zip(self.host, self.batch):
            h.array[...] = a
        self.h2d_bytes = sum(a.nbytes for a in self.batch)
        self.d2h_bytes = 24  # the commit result: code, committed, loss and three norms

    def step(self):
        self.model.step()

    def e2e_step(self):
        from minifield_training_b200.device import h2d

        m = self.model
        for dst, h in zip((m.ids, m.mask, m.seg, m.pos, m.labels), self.host):
            h2d(dst, h.ptr, h.array.nbytes, self.stream)
        m._build_ids()
        res = m.step()
        res.loss  # device -> host read of the step result (synchronizes)

    launches_per_step = None  # counted from the C-ABI calls (see count_launches)

    def count_launches(self):
        """Kernel launches of one step, counted by wrapping the C-ABI entry points once."""
        from minifield_training_b200 import _lib

        per_call = {"mfb_fakequant": 1, "mfb_cast_f32_bf16": 1, "mfb_embed_gather": 1, "mfb_rmsnorm_fwd": 1,
                    "mfb_rmsnorm_bwd": 2, "mfb_gemm_bf16": 1, "mfb_conv_fwd": 1, "mfb_conv_bwd": 2,
                    "mfb_swiglu_fwd": 1, "mfb_swiglu_bwd": 1,
                    "mfb_gemm_swiglu_fwd": 1, "mfb_gemm_swiglu_bwd": 1, "mfb_qknorm_rope_fwd": 1, "mfb_qknorm_rope_bwd": 3,
                    "mfb_attn_fwd": 3, "mfb_attn_bwd": 4, "mfb_head_loss": 3, "mfb_step_normalize": 1,
                    "mfb_adamw_commit": 3, "mfb_adamw_shard_pass": 1}
        orig, count = _lib.call, [0]

        def counting(name, *a):
            count[0] += per_call.get(name, 0)
            if name == "mfb_gemm_bf16_ws":  # the GEMM, and its reduce when the workspace lets K split
                split = a[15] is not None and _lib.lib().mfb_gemm_workspace_size(a[9], a[10], a[11]) > 0
                count[0] += 2 if split else 1
            return orig(name, *a)

        _lib.call = counting
        try:
            self.model.step()
        finally:
            _lib.call = orig
        return count[0]


def _cores():
    return int(os.environ.get("OPENBLAS_NUM_THREADS", os.cpu_count() or 1))


def _cpu_line(value, unit, sample, seconds):
    return {"value": value, "unit": unit, "cores": _cores(), "kind": "port",
            "sample": f"{sample} ({seconds:.1f} s of CPU work)"}


def cpu_attention_sample(cfg=None, rows=None, chunk=2, repeats=1):
    """Time the oracle's FP32 forward+backward over ``rows`` rows of an attention config (default:
    config 2, the whole batch), ``chunk`` rows at a time (a config-2 chunk's score grids take
    about 2.5 GB), ``repeats`` times. Returns (TFLOP/s, seconds, sample text)."""
    from minifield_training_b200 import workloads
    from oracle import attention as oatt

    cfg = cfg or workloads.CONFIG2
    rows = cfg.batch if rows is None else rows
    inputs = workloads.attention_inputs(cfg, 0)
    dt, flops = 0.0, 0.0
    for lo in [lo for _ in range(repeats) for lo in range(0, rows, chunk)]:
        q, k, v, do, mask = (x[lo:min(rows, lo + chunk)] for x in inputs[:5])
        seg = inputs[5][lo:min(rows, lo + chunk)] if inputs[5] is not None else None
        ids = oatt.bidirectional_ids(mask, seg) if cfg.packed else oatt.causal_ids(mask)
        valid = oatt.valid_from_ids(*ids[:4])
        t0 = time.perf_counter()
        oatt.attention_forward(q, k, v, valid, ids[4], np.float32)
        oatt.attention_backward(q, k, v, valid, ids[4], do, np.float32)
        dt += time.perf_counter() - t0
        flops += 3.5 * 4.0 * cfg.heads * cfg.head_dim * oatt.valid_pair_count(*ids[:4])
    what = "the whole batch" if rows == cfg.batch else f"rows 0..{rows - 1}"
    times = f", {repeats} times" if repeats > 1 else ""
    return flops / dt / 1e12, dt, (f"{cfg.name} {what} (B={rows} of {cfg.batch}, T={cfg.length}, "
                                   f"{cfg.heads}/{cfg.kv_heads} heads){times}, FP32 NumPy, {chunk} rows at a time")


def cpu_decode_sample(layers=2):
    """Config 3 on the oracle in FP32: the append + cached attention of ``layers`` of the 6 layers over
    all 64 rows, scaled to the 6-layer step. Returns (tokens/s, GB/s, seconds, sample text)."""
    from minifield_training_b200 import workloads
    from oracle import decode as odec

    cfg = workloads.CONFIG3
    lens = workloads.decode_lengths(cfg, 0)
    dt = 0.0
    for layer in range(layers):
        q, kc, vc, nk, nv = workloads.decode_layer_inputs(cfg, 0, layer)
        t0 = time.perf_counter()
        odec.decode_attention(q, kc, vc, lens, nk, nv, lens - 1, np.float32)
        dt += time.perf_counter() - t0
    step = dt * cfg.layers / layers
    nbytes = cfg.layers * workloads.decode_layer_bytes(lens, cfg)
    return cfg.batch / step, nbytes / step / 1e9, dt, (
        f"{cfg.name}: {layers} of {cfg.layers} layers over all {cfg.batch} rows, scaled to the 6-layer step; "
        "FP32 NumPy (the reference's dense cached attention reads every cache slot, then masks)")


def cpu_qat_sample(kind, tokens=2048):
    """Config 4 on the oracle in FP32: fake-quant of both weights once, then the GEMM chain forward +
    backward on ``tokens`` of the 16384 rows, scaled by rows. Returns (TFLOP/s, tokens/s, seconds, text)."""
    from minifield_training_b200 import workloads
    from oracle import linear as olin

    cfg = workloads.CONFIG4
    x, w_gu, w_d, dy = workloads.qat_inputs(cfg, 0, tokens=tokens)
    t0 = time.perf_counter()
    olin.qat_weights(w_gu, w_d, kind)
    t_quant = time.perf_counter() - t0
    t0 = time.perf_counter()
    olin.swiglu_qat_step(x, w_gu, w_d, kind, dy, np.float32)  # quantizes again, then the chain
    t_chain = max(time.perf_counter() - t0 - t_quant, 1e-9)
    step = t_quant + t_chain * cfg.tokens / tokens
    flops = 3.0 * olin.ffn_flops(cfg.tokens, cfg.hidden, cfg.ffn)
    return flops / step / 1e12, cfg.tokens / step, t_quant * 2 + t_chain, (
        f"{cfg.name} {kind}: both weights fake-quantized once + the chain on {tokens} of {cfg.tokens} "
        "tokens, scaled by rows; FP32 NumPy")


def cpu_encoder_sample(rows=2):
    """Config 5 on the oracle (torch autograd on the CPU, FP32): loss and gradients of ``rows`` 2048-token
    rows through a conv layer and an attention layer at the full hidden/FFN widths, with int8 fake-quant,
    scaled by FLOPs to the 16-layer step over the 32-row global batch. Returns (tokens/s, TFLOP/s,
    seconds, text)."""
    import dataclasses

    import torch

    from minifield_training_b200 import workloads
    from minifield_training_b200.models import encoder as me
    from oracle import encoder_step as oes

    torch.set_num_threads(os.cpu_count() or 1)
    full = workloads.CONFIG5
    sub = dataclasses.replace(full, global_batch=rows, layer_types=("conv", "full_attention"))
    params = me.init_parameters(sub, 0)
    batch = workloads.encoder_batch(sub, 0, rows=rows)
    t0 = time.perf_counter()
    oes.loss_and_grads(sub, params, *batch, rows=rows, compute_dtype=torch.float32)
    dt = time.perf_counter() - t0
    sub_flops = workloads.encoder_step_flops(sub, batch[2])
    full_flops = workloads.encoder_step_flops(full, workloads.packed_segments(0, full.global_batch, full.length))
    step = dt * full_flops / sub_flops
    tokens = full.global_batch * full.length
    return tokens / step, full_flops / step / 1e12, dt, (
        f"{full.name}: {rows} rows x {full.length} tokens through 2 of the 16 layers (conv + attention; hidden "
        f"{full.hidden}, FFN {full.ffn}, int8 fake-quant) forward + backward, torch autograd FP32 on the CPU, "
        "scaled by FLOPs to the 16-layer 32 x 2048 step")


def run_reference(args, dist):
    """The reference algorithm's CPU restatement on the headline config: each step is the whole
    config-2 batch (8 rows, two at a time), as the GPU arm's step."""
    if dist.rank != 0:
        return 0
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_attention_sample(rows=2)
    vals, walls = [], []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        v, _, sample = cpu_attention_sample()
        walls.append(time.perf_counter() - t0)
        vals.append(v)
    value = float(np.median(vals))
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": float(np.mean(walls)) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "cfg2-segment-bidirectional-gqa-fwd-bwd", "batch": 8, "seq_len": 2048, "heads": 16,
                   "kv_heads": 8, "head_dim": 64, "sample": "the whole batch per step"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": _cores(), "kind": "port",
                         "sample": sample + "; the reference is JAX (not installed): NumPy restatement of its "
                                            "algorithm"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Our arm.
# ---------------------------------------------------------------------------


def measure(dist, fn, steps, warmup, clocks=None, stream=None, end_stream=None, settle=None):
    """Max over ranks of the mean step time, CUDA events on the launching stream.

    ``end_stream`` (default ``stream``) is the stream that finishes each step
    last when a step spans several streams. ``settle()``, when given, runs
    before the end event: it orders the timed stream after work a step leaves
    in flight on other streams (the sharded optimizer's master broadcasts,
    which the next step's forward overlaps), so every timed step's work is in
    the timed region.
    """
    from minifield_training_b200.device import Event, sync

    for _ in range(warmup):
        fn()
    sync()
    dist.barrier()
    sync()
    a, b = Event(), Event()
    if clocks:
        clocks.start()
    a.record(stream)
    for _ in range(steps):
        fn()
    if settle is not None:
        settle()
    b.record(end_stream if end_stream is not None else stream)
    sync()
    clk = clocks.stop() if clocks else None
    dist.barrier()
    ms = a.elapsed_ms(b) / steps
    return dist.max(ms), clk


def attention_roofline(att, fwd_ms, bwd_ms, tf_burst, peak_kind, traffic):
    """Roofline entry of the slower attention kernel (forward or backward), each timed alone."""
    if bwd_ms >= fwd_ms:
        dom, dom_ms, dom_flops = "attn_bwd", bwd_ms, 2.5 * att.fwd_flops
    else:
        dom, dom_ms, dom_flops = "attn_fwd", fwd_ms, att.fwd_flops
    achieved = dom_flops / (dom_ms * 1e-3) / 1e12
    return {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": tf_burst, "unit": "TFLOP/s",
            "frac": achieved / tf_burst, "peak_source": f"{peak_kind} bf16 burst", "traffic": traffic.get(dom),
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms, "fwd_tflops": att.fwd_flops / (fwd_ms * 1e-3) / 1e12,
            "bwd_tflops": 2.5 * att.fwd_flops / (bwd_ms * 1e-3) / 1e12}


def attention_e2e(att, dist, steps, n):
    """Pipelined end-to-end leg through the C ABI with pinned host buffers (see e2e_setup)."""
    att.e2e_setup()
    # The timed window carries the pipeline's fill and drain (one step's kernels and download, ~2.5 ms at
    # config 2) once; at least 24 steps keep that a small share of the per-step figure.
    e2e_ms, _ = measure(dist, att.e2e_step, max(24, steps), 2, stream=att.s_in, end_stream=att.s_out)
    att.e2e_close()
    return {"value": n * att.total_flops / (e2e_ms * 1e-3) / 1e12, "unit": UNIT,
            "h2d_bytes_per_step": att.h2d_bytes, "d2h_bytes_per_step": att.d2h_bytes, "ms_per_step": e2e_ms}


def run_ours(args, dist):
    from minifield_training_b200 import device, workloads

    device.set_device(dist.local)
    device.require_b200(dist.local)
    hbm, tf_burst, tf_sus, peak_kind = peaks()
    traffic = traffic_table()
    n = dist.world
    only = args.only
    clocks = Clocks(dist.local)
    clocks.start()  # sampled across every timed phase below
    cpu_legs = dist.world == 1 and not args.no_cpu_baseline

    line = {"metric": METRIC, "unit": UNIT, "n_gpus": n, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic"}
    launches = 0
    if only in (None, "attention"):
        att = AttentionWorkload(workloads.CONFIG2, seed=dist.rank)
        ms, _ = measure(dist, att.step, args.steps, args.warmup)
        value = n * att.total_flops / (ms * 1e-3) / 1e12
        launches += AttentionWorkload.launches_per_step * args.steps
        # Per-kernel timing for the roofline: forward alone, backward alone.
        timer = Timer()
        fwd_ms = dist.max(timer.time(att.fwd, args.steps))
        bwd_ms = dist.max(timer.time(att.bwd, args.steps))
        launches += 3 * args.steps + 4 * args.steps
        roofline = attention_roofline(att, fwd_ms, bwd_ms, tf_burst, peak_kind, traffic)
        e2e = attention_e2e(att, dist, args.steps, n)
        line.update(value=value, ms_per_step=ms, tensor_peak_frac=value / n / tf_burst, roofline=roofline, e2e=e2e)
        line["config"] = {
            "workload": workloads.CONFIG2.name, "batch": 8, "seq_len": 2048, "heads": 16, "kv_heads": 8,
            "head_dim": 64, "segments": "U[32,1024] packed, seed=rank", "flops_per_step": att.total_flops,
            "per_gpu_work": "fixed (weak scaling, independent replicas)",
            "l2": "inputs larger than L2 (~250 MB working set per step)"}
        del att

    secondary = {}
    run_secondary = only is None and not args.no_secondary
    if only == "attention_cfg1" or run_secondary:
        # Config 1: dense causal B=4, T=512; tiny (7.5 GFLOP), so every timing replays CUDA graphs.
        a1 = AttentionWorkload(workloads.CONFIG1, seed=dist.rank)
        a1.capture_graphs()
        ms1, _ = measure(dist, lambda: a1.replay("step"), args.steps, args.warmup, stream=a1.stream)
        f1, _ = measure(dist, lambda: a1.replay("fwd"), args.steps, 2, stream=a1.stream)
        b1, _ = measure(dist, lambda: a1.replay("bwd"), args.steps, 2, stream=a1.stream)
        launches += (8 + 3 + 4) * args.steps
        a1.release_graphs()
        e2e1 = attention_e2e(a1, dist, args.steps, n)
        tflops1 = n * a1.total_flops / (ms1 * 1e-3) / 1e12
        secondary["attention_cfg1"] = {
            "workload": workloads.CONFIG1.name, "batch": 4, "seq_len": 512, "heads": 16, "kv_heads": 8,
            "head_dim": 64, "flops_per_step": a1.total_flops, "ms_per_step": ms1, "tflops": tflops1,
            "tensor_frac": tflops1 / n / tf_burst, "graph": True,
            "roofline": attention_roofline(a1, f1, b1, tf_burst, peak_kind, {}), "e2e": e2e1}
        del a1
    if only == "decode" or run_secondary:
        dec = DecodeWorkload(seed=dist.rank)
        dms, _ = measure(dist, dec.step, args.steps, args.warmup)
        gbs = dec.bytes / (dms * 1e-3) / 1e9
        launches += DecodeWorkload.launches_per_step * args.steps
        secondary["decode"] = {
            "workload": workloads.CONFIG3.name, "tokens_per_s": n * workloads.CONFIG3.batch / (dms * 1e-3),
            "ms_per_step": dms, "hbm_gbs": gbs, "hbm_frac": gbs / hbm, "peak_gbs": hbm,
            "bytes_per_step": dec.bytes, "traffic": traffic.get("decode")}
        del dec
    if only == "decode_one" or run_secondary:
        d1 = DecodeOneWorkload(seed=dist.rank)
        d1.prefill()  # warm-up prompt (allocates the prompt buffers, loads the kernels)
        d1.state = d1.dm.new_state(d1.cfg, d1.batch, d1.capacity)
        device.sync()
        dist.barrier()
        ev0, ev1 = device.Event(), device.Event()
        ev0.record(d1.stream)
        d1.dec.prefill(d1.prompt, d1.state)
        ev1.record(d1.stream)
        device.sync()
        pre_ms = dist.max(ev0.elapsed_ms(ev1))
        first = d1.state.valid_length + args.warmup
        dms1, _ = measure(dist, d1.step, args.steps, args.warmup, stream=d1.stream)
        nbytes = d1.bytes_per_step(first, args.steps)
        gbs = nbytes / (dms1 * 1e-3) / 1e9
        launches += d1.kernels_per_step() * args.steps
        secondary["decode_one"] = {
            "workload": "lfm2.5-350m-decode-one-b64-cap4096", "layers": len(d1.cfg.layer_types),
            "prompt_tokens": d1.prompt.shape[1], "tokens_per_s": n * d1.batch / (dms1 * 1e-3), "ms_per_step": dms1,
            "hbm_gbs": gbs, "hbm_frac": gbs / hbm, "peak_gbs": hbm, "bytes_per_step": nbytes,
            "prefill_ms": pre_ms, "prefill_tokens_per_s": n * d1.prompt.size / (pre_ms * 1e-3),
            "graph": True, "kernels_per_step": d1.kernels_per_step()}
        d1.close()
        del d1
    for kind, key in ((workloads.CONFIG4.kind, "qat"), ("int4-g128-absmax-v1", "qat_int4")):
        if not (only == "qat" or run_secondary):
            break
        qat = QatWorkload(seed=dist.rank, kind=kind)
        qsteps = max(3, args.steps // 2)
        qms, _ = measure(dist, qat.step, qsteps, max(3, args.warmup // 2))
        launches += qat.launches_per_step * qsteps
        secondary[key] = {
            "workload": workloads.CONFIG4.name, "kind": kind,
            "tokens_per_s": n * workloads.CONFIG4.tokens / (qms * 1e-3), "ms_per_step": qms,
            "tflops": qat.flops / (qms * 1e-3) / 1e12, "tensor_frac": qat.flops / (qms * 1e-3) / 1e12 / tf_sus,
            "peak_tflops": tf_sus, "peak_source": f"{peak_kind} bf16 sustained"}
        del qat
    if only == "encoder" or run_secondary:
        enc = EncoderStepWorkload(dist)
        esteps = max(3, args.steps // 5)
        per_step = enc.count_launches()  # one eager step, counting the kernels each call launches
        enc.model.capture()  # then the step replays as CUDA graphs
        ems, _ = measure(dist, enc.step, esteps, max(3, args.warmup // 2), stream=enc.stream,
                         settle=enc.model.settle)
        launches += per_step * esteps
        e2e_ms, _ = measure(dist, enc.e2e_step, max(3, esteps // 2), 1, stream=enc.stream, settle=enc.model.settle)
        res = enc.model.result
        tflops = enc.global_flops / (ems * 1e-3) / 1e12
        secondary["encoder_step"] = {
            "workload": workloads.CONFIG5.name, "tokens_per_s": enc.tokens / (ems * 1e-3), "ms_per_step": ems,
            "global_batch": workloads.CONFIG5.global_batch, "seq_len": workloads.CONFIG5.length,
            "rows_per_gpu": enc.rows, "scaling": "strong", "tflops": tflops,
            "tensor_frac_per_gpu": tflops / n / tf_sus, "peak_tflops": tf_sus,
            "peak_source": f"{peak_kind} bf16 sustained", "flops_per_step": enc.global_flops,
            "quant": workloads.CONFIG5.quant, "committed": res.committed, "loss": res.loss,
            "launches_per_step": per_step,
            "e2e": {"tokens_per_s": enc.tokens / (e2e_ms * 1e-3), "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": enc.h2d_bytes * n, "d2h_bytes_per_step": enc.d2h_bytes * n}}
        del enc
    line["clocks"] = clocks.stop()

    # CPU baselines: the oracle's restatement of the reference algorithm on this host's cores, rank 0 at
    # N=1 only, each on a bounded sample of its config (after every GPU leg, outside their timing).
    if cpu_legs:
        if only in (None, "attention"):
            v, dt, sample = cpu_attention_sample()
            line["cpu_baseline"] = _cpu_line(v, UNIT, sample, dt)
        if "attention_cfg1" in secondary:
            v, dt, sample = cpu_attention_sample(workloads.CONFIG1, repeats=8)
            secondary["attention_cfg1"]["cpu_baseline"] = _cpu_line(v, UNIT, sample, dt)
        if "decode" in secondary:
            tps, gbs, dt, sample = cpu_decode_sample(layers=6)
            secondary["decode"]["cpu_baseline"] = dict(_cpu_line(tps, "tokens/s", sample, dt), hbm_gbs=gbs)
        for key in ("qat", "qat_int4"):
            if key in secondary:
                tf, tps, dt, sample = cpu_qat_sample(secondary[key]["kind"])
                secondary[key]["cpu_baseline"] = dict(_cpu_line(tf, "TFLOP/s", sample, dt), tokens_per_s=tps)
        if "encoder_step" in secondary:
            tps, tf, dt, sample = cpu_encoder_sample()
            secondary["encoder_step"]["cpu_baseline"] = dict(_cpu_line(tps, "tokens/s", sample, dt), tflops=tf)
    line["gpu_launches"] = launches
    line["secondary"] = secondary
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    dist = Dist()
    try:
        if args.impl == "reference":
            return run_reference(args, dist)
        return run_ours(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    sys.exit(main())
