"""Config-5 encoder step on the GPU against oracle/encoder_step.py (FP64 autograd).

A two-layer encoder (conv + attention, hidden 1024, FFN 256, packed segments)
runs the QAT forward and backward through the kernels. For a composed bf16
model the per-op gate (rel-L2 1e-2) is the wrong ruler: two bf16 runs that
round at different points already differ by about that much. So every
trainable leaf's gradient G is compared with the exact FP64 path X of the same
(fake-quantized) model, next to the oracle R that rounds at the reference's
bf16 cast points: rel-L2(G, X) must stay within 1.5x rel-L2(R, X) + 2e-3, and
G and R must agree within rel-L2 2e-2. The loss sum must match R within 2e-3
and the valid count exactly; then one AdamW commit must succeed.
"""

import dataclasses

import numpy as np
import pytest

from tests.gpu_env import require_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    require_gpu()


def _cfg():
    from minifield_training_b200 import workloads
    return dataclasses.replace(workloads.CONFIG5, global_batch=2, length=128, ffn=256,
                               layer_types=("conv", "full_attention"), vocab=1000)


def test_encoder_step_gradients_match_oracle():
    from minifield_training_b200 import workloads
    from minifield_training_b200.device import sync
    from minifield_training_b200.models import encoder as me
    from oracle import encoder_step as oes
    cfg = _cfg()
    step = me.EncoderStep(cfg, rows=2, seed=0)
    batch = workloads.encoder_batch(cfg, 3)
    step.set_batch(*batch)
    step.quantize()
    step.forward()
    step.backward()
    sync()
    loss, count = step.loss_count.numpy()
    ref_loss, ref_count, ref_grads = oes.loss_and_grads(cfg, me.init_parameters(cfg, 0), *batch, rows=2)
    assert count == ref_count
    np.testing.assert_allclose(loss, ref_loss, rtol=2e-3)
    _, _, exact = oes.loss_and_grads(cfg, me.init_parameters(cfg, 0), *batch, rows=2, bf16=False)

    def rl2(a, b):
        return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))

    report, failures = [], []
    for name, ref in ref_grads.items():
        got = step.gviews[name].numpy().astype(np.float64).reshape(-1)
        r, x = ref.reshape(-1), exact[name].reshape(-1)
        g_x, r_x, g_r = rl2(got, x), rl2(r, x), rl2(got, r)
        report.append(f"{name}: G-X {g_x:.2e}  R-X {r_x:.2e}  G-R {g_r:.2e}")
        if g_x > 1.5 * r_x + 2e-3 or g_r > 2e-2:
            failures.append(report[-1])
    print("\n".join(report))
    print(f"loss {loss} vs {ref_loss}")
    assert not failures, failures
    before = step.params["lfm2.layers.1.self_attn.q_proj.weight"].numpy()
    step._commit()
    res = step.result
    assert res.committed and int(res.code) == 0
    np.testing.assert_allclose(res.loss, ref_loss / ref_count, rtol=2e-3)
    after = step.params["lfm2.layers.1.self_attn.q_proj.weight"].numpy()
    assert np.abs(after - before).max() > 0
    assert int(step.state["step"].numpy()[0]) == 1


def test_next_step_consumes_the_committed_state():
    """After a commit, the next forward's loss equals the oracle's loss at the read-back masters."""
    from minifield_training_b200 import workloads
    from minifield_training_b200.device import sync
    from minifield_training_b200.models import encoder as me
    from oracle import encoder_step as oes
    cfg = dataclasses.replace(_cfg(), learning_rate=1e-3)
    step = me.EncoderStep(cfg, rows=2, seed=1)
    batch = workloads.encoder_batch(cfg, 5)
    step.set_batch(*batch)
    assert step.step().committed
    params = {n: v.numpy() for n, v in step.params.items()}
    step.quantize()
    step.forward()
    step.backward()
    sync()
    loss, count = step.loss_count.numpy()
    ref_loss, ref_count, _ = oes.loss_and_grads(cfg, params, *batch, rows=2)
    assert count == ref_count
    np.testing.assert_allclose(loss, ref_loss, rtol=2e-3)


def test_small_steps_lower_the_loss_on_a_fixed_batch():
    from minifield_training_b200 import workloads
    from minifield_training_b200.models import encoder as me
    cfg = dataclasses.replace(_cfg(), learning_rate=1e-5)
    step = me.EncoderStep(cfg, rows=2, seed=1)
    step.set_batch(*workloads.encoder_batch(cfg, 5))
    losses = []
    for _ in range(4):
        res = step.step()
        assert res.committed
        losses.append(res.loss)
    assert all(b < a for a, b in zip(losses, losses[1:])), losses


def test_graph_replay_matches_eager_steps():
    """Two steps replayed from one captured CUDA graph equal two eager steps.

    Same kernels in the same order; the attention backward's dQ atomics may
    sum in another order, so masters are compared at rtol 1e-5.
    """
    import ctypes

    from minifield_training_b200 import _lib, workloads
    from minifield_training_b200.device import sync
    from minifield_training_b200.models import encoder as me
    cfg = _cfg()
    batch = workloads.encoder_batch(cfg, 9)
    stream = ctypes.c_void_p()
    _lib.call("mfb_stream_create", ctypes.byref(stream))
    graph = me.EncoderStep(cfg, rows=2, seed=2, stream=stream.value)
    eager = me.EncoderStep(cfg, rows=2, seed=2)
    graph.set_batch(*batch)
    eager.set_batch(*batch)
    graph.capture()  # records (does not run) one step
    sync()
    assert int(graph.state["step"].numpy()[0]) == 0
    for _ in range(2):
        rg, re_ = graph.step(), eager.step()
        assert rg.committed and re_.committed
        np.testing.assert_allclose(rg.loss, re_.loss, rtol=1e-5)
    sync()
    assert int(graph.state["step"].numpy()[0]) == 2
    for name in graph.params:
        np.testing.assert_allclose(graph.params[name].numpy(), eager.params[name].numpy(), rtol=1e-5, atol=1e-7,
                                   err_msg=name)
