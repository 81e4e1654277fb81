"""Recording and replay (tensorplay-mlu: graph.py:38-92, GraphCapture.cpp:
69-130) on CUDA graphs: replays read the recorded buffers' current contents,
a replayed training step matches the same steps run eagerly, the allocator
holds the recording's blocks until reset, and a body that reads back to the
host is refused without leaving a recording behind."""

from __future__ import annotations

import pytest
import torch

from conftest import assert_close, assert_equal

pytestmark = pytest.mark.gpu


def rand(*shape, seed=0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


@pytest.fixture()
def graph(backend):
    from tensorplay_mlu_b200.graph import Graph

    g = Graph()
    yield g
    g.reset()


def test_replay_reads_the_buffers_current_contents(backend, graph):
    ops = backend.ops
    x = ops.to_device(rand(64, 96, seed=1))
    w = ops.to_device(rand(96, 48, seed=2))
    y = graph.capture(lambda: ops.softmax(ops.gelu(ops.mm(x, w)), -1))
    assert graph.ready
    for seed in (3, 4):
        fresh = rand(64, 96, seed=seed)
        ops.copy_(x, ops.to_device(fresh))
        graph.replay()
        want = ops.softmax(ops.gelu(ops.mm(ops.to_device(fresh), w)), -1)
        assert_equal(ops.to_host(y), ops.to_host(want))


def test_replayed_training_steps_match_eager_steps(backend, graph):
    from tensorplay_mlu_b200.train import DataParallelMLP, MLPConfig, init_params_host, make_batch_host

    ops = backend.ops
    cfg = MLPConfig(d_in=256, d_hidden=1024, batch=128, lr=0.05)
    params = init_params_host(cfg, seed=0)
    x, t = make_batch_host(cfg, seed=0)
    eager = DataParallelMLP(cfg, device=0, host_params=params)
    replayed = DataParallelMLP(cfg, device=0, host_params=params)
    dx, dt = ops.to_device(x), ops.to_device(t)
    for _ in range(3):
        want_loss = eager.step(dx, dt)
    loss = graph.capture(lambda: replayed.step(dx, dt))  # recorded, not run
    assert_equal(ops.to_host(replayed.w1), params[0].to(torch.bfloat16))
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert_equal(ops.to_host(loss), ops.to_host(want_loss))
    for a, b in zip(replayed.params(), eager.params()):
        assert_equal(ops.to_host(a), ops.to_host(b))


def test_recording_holds_its_blocks_until_reset(backend, graph):
    ops = backend.ops
    from tensorplay_mlu_b200 import _native as N

    x = ops.to_device(rand(256, 256, seed=5))
    graph.capture(lambda: ops.add_Tensor(ops.exp(x), ops.sum_dim_IntList(x, [0], keepdim=True)))
    handed_out, held = graph.stats()
    assert handed_out >= 2 and held >= 1  # the exp temporary was given back while recording
    graph.reset()
    assert not graph.ready
    assert graph.stats()[1] == 0
    assert N.lib().tp_b200_take_device_error(torch.cuda.current_device()) == 0


def test_host_read_inside_the_body_is_refused(backend, graph):
    ops = backend.ops
    x = ops.to_device(rand(32, 32, seed=6))
    with pytest.raises(RuntimeError):
        graph.capture(lambda: ops.item(ops.sum(x)))
    assert not graph.ready
    # The device and the allocator are usable, and a new recording works.
    y = graph.capture(lambda: ops.mul_Scalar(x, 2.0))
    graph.replay()
    assert_close(ops.to_host(y), ops.to_host(x) * 2, torch.float32)


def test_one_recording_at_a_time(backend, graph):
    ops = backend.ops
    x = ops.to_device(rand(8, 8, seed=7))
    graph.capture(lambda: ops.neg(x))
    from tensorplay_mlu_b200.graph import Graph

    with pytest.raises(RuntimeError, match="held already"):
        Graph().capture(lambda: ops.neg(x))
    assert graph.ready
