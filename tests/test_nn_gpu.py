"""Normalisation and loss kernels (tensorplay-mlu NNKernels.cpp:59-161 and
:304-397) against the oracle: layer_norm forward / backward over every float
dtype, register-held and long rows, with and without affine parameters;
nll_loss forward / backward with class weights, ignore_index, int32 targets
and every reduction; and the reference's cross-entropy training step
(test_mlu.py:363-378) against PyTorch CPU autograd."""

from __future__ import annotations

import pytest
import torch

import oracle as O
from conftest import assert_close, assert_close_terms

pytestmark = pytest.mark.gpu

FLOATS = [torch.float32, torch.bfloat16, torch.float16, torch.float64]


def rand(*shape, dtype=torch.float32, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


@pytest.fixture(scope="module")
def ops(backend):
    return backend.ops


@pytest.mark.parametrize("dtype", FLOATS)
@pytest.mark.parametrize("shape,norm", [((7, 20), [20]), ((3, 5, 64), [5, 64]), ((9, 1001), [1001]),
                                        ((6, 4096), [4096]), ((3, 16384), [16384]), ((300, 256), [256])])
def test_layer_norm_forward_backward(ops, dtype, shape, norm):
    x = rand(*shape, dtype=dtype, seed=1, scale=3.0) + 0.5
    x = x.to(dtype)
    for affine in (True, False):
        w = rand(*norm, dtype=dtype, seed=2) if affine else None
        b = rand(*norm, dtype=dtype, seed=3) if affine else None
        dev = lambda t: ops.to_device(t) if t is not None else None
        y, mean, rstd = ops.native_layer_norm(dev(x), norm, dev(w), dev(b), 1e-5)
        wy, wm, wr = O.layer_norm(x, norm, w, b, 1e-5)
        assert mean.dtype == wm.dtype and rstd.dtype == wr.dtype
        assert_close(y, wy, dtype, scale=2)
        stat_dtype = torch.float64 if dtype == torch.float64 else torch.float32
        assert_close(mean, wm, stat_dtype if dtype in (torch.float32, torch.float64) else torch.bfloat16)
        assert_close(rstd, wr, stat_dtype if dtype in (torch.float32, torch.float64) else torch.bfloat16)
        dy = rand(*shape, dtype=dtype, seed=4)
        dx, dw, db = ops.native_layer_norm_backward(dev(dy), dev(x), norm, mean, rstd, dev(w), dev(b),
                                                    [True, affine, affine])
        # The oracle's backward from the same (device) statistics.
        hm, hr = ops.to_host(mean).double(), ops.to_host(rstd).double()
        wdx, wdw, wdb = O.layer_norm_backward(dy, x, norm, ops.to_host(mean), ops.to_host(rstd), w)
        # Term magnitudes: per row, dx = rstd (g - mean(g) - xhat mean(g xhat))
        # with g = dy w; dw, db sum dy xhat, dy over the rows.
        D = int(torch.tensor(norm).prod())
        rows = x.numel() // D
        xr = x.double().reshape(rows, D)
        xhat = (xr - hm.reshape(rows, 1)) * hr.reshape(rows, 1)
        g = dy.double().reshape(rows, D) * (w.double().reshape(1, D) if affine else 1.0)
        t_dx = hr.reshape(rows, 1) * (g.abs() + g.abs().mean(1, keepdim=True)
                                      + xhat.abs() * (g * xhat).abs().mean(1, keepdim=True))
        assert_close_terms(dx, wdx, t_dx.reshape(x.shape), dtype)
        if affine:
            dyr = dy.double().reshape(rows, D)
            assert_close_terms(dw, wdw, (dyr * xhat).abs().sum(0).reshape(wdw.shape), dtype)
            assert_close_terms(db, wdb, dyr.abs().sum(0).reshape(wdb.shape), dtype)
        else:
            assert dw is None and db is None


def test_layer_norm_rejects_bad_shapes(ops):
    x = ops.to_device(rand(4, 6))
    with pytest.raises(RuntimeError, match="normalized_shape"):
        ops.native_layer_norm(x, [5], None, None, 1e-5)
    with pytest.raises(RuntimeError):
        ops.native_layer_norm(x, [6], ops.to_device(rand(5)), None, 1e-5)


@pytest.mark.parametrize("dtype", FLOATS)
@pytest.mark.parametrize("reduction", [0, 1, 2])
def test_nll_loss_forward_backward(ops, dtype, reduction):
    n, c = 1000, 37
    g = torch.Generator().manual_seed(5)
    x = torch.log_softmax(rand(n, c, seed=6, scale=2.0), 1).to(dtype)
    t = torch.randint(0, c, (n,), generator=g)
    t[::17] = -100  # ignored samples
    for target_dtype in (torch.int64, torch.int32):
        for w in (None, (rand(c, seed=7).abs() + 0.5).to(dtype)):
            tt = t.to(target_dtype)
            dw = ops.to_device(w) if w is not None else None
            out, total = ops.nll_loss(ops.to_device(x), ops.to_device(tt), dw, reduction, -100)
            want_out, want_total = O.nll_loss(x, tt, w, reduction, -100)
            # Term magnitudes: the weighted picked log-probabilities (and
            # weights) summed by the sum / mean reductions.
            terms_out, _ = O.nll_loss(x.abs(), tt, w, reduction, -100)
            assert_close_terms(out, want_out, terms_out.abs(), dtype)
            assert_close_terms(total, want_total, want_total.abs(), dtype)
            grad = rand(n, dtype=dtype, seed=8) if reduction == 0 else torch.tensor(1.5, dtype=dtype)
            dx = ops.nll_loss_backward(ops.to_device(grad), ops.to_device(x), ops.to_device(tt), dw, reduction,
                                       -100, total)
            want_dx = O.nll_loss_backward(grad, x, tt, w, reduction, -100, want_total)
            assert_close(dx, want_dx, dtype)


def test_nll_loss_target_out_of_range_sets_the_error_word(ops, backend):
    lib = backend._native.lib()
    dev = torch.cuda.current_device()
    lib.tp_b200_take_device_error(dev)
    x = ops.to_device(torch.log_softmax(rand(4, 5), 1))
    t = ops.to_device(torch.tensor([0, 7, 2, 1]))
    out, total = ops.nll_loss(x, t, None, 2, -100)
    torch.cuda.synchronize()
    assert lib.tp_b200_take_device_error(dev) != 0
    # The bad sample counts as ignored: the three valid ones are summed.
    xs = torch.log_softmax(rand(4, 5), 1)
    assert abs(ops.item(out) + float(xs[0, 0] + xs[2, 2] + xs[3, 1])) < 1e-5
    assert ops.item(total) == 3.0


def test_cross_entropy_training_step_matches_host(ops):
    # test_mlu.py:363-378: Linear(12, 32) -> GELU -> Linear(32, 3), cross
    # entropy, full backward; the host side is PyTorch CPU autograd.
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(12, 32), torch.nn.GELU(), torch.nn.Linear(32, 3))
    x, target = torch.randn(16, 12), torch.randint(0, 3, (16,))
    loss_ref = torch.nn.functional.cross_entropy(model(x), target)
    loss_ref.backward()
    w1, b1, w2, b2 = (p.detach() for p in model.parameters())
    d = ops.to_device
    dx, dw1, db1, dw2, db2, dt = d(x), d(w1), d(b1), d(w2), d(b2), d(target)
    h = ops.linear(dx, dw1, db1)
    a = ops.gelu(h)
    logits = ops.linear(a, dw2, db2)
    ls = ops._log_softmax(logits, 1)
    loss, total = ops.nll_loss(ls, dt, None, 1, -100)
    one = d(torch.tensor(1.0))
    dls = ops.nll_loss_backward(one, ls, dt, None, 1, -100, total)
    dlogits = ops._log_softmax_backward_data(dls, ls, 1, torch.float32)
    g_w2 = ops.mm(dlogits.t(), a)
    g_b2 = ops.sum_dim_IntList(dlogits, [0])
    da = ops.mm(dlogits, dw2)
    dh = ops.gelu_backward(da, h)
    g_w1 = ops.mm(dh.t(), dx)
    g_b1 = ops.sum_dim_IntList(dh, [0])
    assert abs(ops.item(loss) - loss_ref.item()) < 1e-4
    for got, p in zip((g_w1, g_b1, g_w2, g_b2), model.parameters()):
        assert (ops.to_host(got) - p.grad).abs().max().item() < 1e-4
    assert abs(ops.item(ops.cross_entropy(logits, dt)) - loss_ref.item()) < 1e-4


@pytest.mark.parametrize("dtype", FLOATS)
def test_dropout_matches_the_oracle_generator(ops, dtype):
    x = rand(333, 257, dtype=dtype, seed=9)
    torch.manual_seed(123)
    out, mask = ops.native_dropout(ops.to_device(x), 0.3, True)
    torch.manual_seed(123)
    seed = int(torch.randint(0, 2 ** 62, (1,)).item())
    want_out, want_mask = O.dropout(x, 0.3, seed)
    assert torch.equal(ops.to_host(mask), want_mask)
    assert torch.equal(ops.to_host(out), want_out)
    kept = want_mask.float().mean().item()
    assert abs(kept - 0.7) < 0.01
    dy = rand(333, 257, dtype=dtype, seed=10)
    dx = ops.native_dropout_backward(ops.to_device(dy), mask, 1 / 0.7)
    want_dx = torch.where(want_mask, (dy.double() / 0.7), torch.zeros((), dtype=torch.float64)).to(dtype)
    assert_close(dx, want_dx, dtype)
    # Evaluation and the edge probabilities need no generator.
    same, m = ops.native_dropout(ops.to_device(x), 0.5, False)
    assert torch.equal(ops.to_host(same), x) and bool(ops.to_host(m).all())
    zero, m = ops.native_dropout(ops.to_device(x), 1.0, True)
    assert not bool(ops.to_host(zero).any()) and not bool(ops.to_host(m).any())


def test_embedding_forward_backward(ops):
    weight = rand(1000, 64, seed=11)
    g = torch.Generator().manual_seed(12)
    idx = torch.randint(0, 1000, (7, 9), generator=g)
    idx[0, :3] = 3  # duplicates and the padding index
    out = ops.embedding(ops.to_device(weight), ops.to_device(idx), 3)
    assert_close(out, O.index_select(weight, 0, idx.reshape(-1)).reshape(7, 9, 64), torch.float32)
    grad = rand(7, 9, 64, seed=13)
    for freq in (False, True):
        got = ops.embedding_dense_backward(ops.to_device(grad), ops.to_device(idx), 1000, 3, freq)
        want = O.index_add_zeros([1000, 64], 0, idx.reshape(-1), grad.reshape(-1, 64))
        terms = O.index_add_zeros([1000, 64], 0, idx.reshape(-1), grad.abs().reshape(-1, 64))
        if freq:
            counts = torch.bincount(idx.reshape(-1), minlength=1000).clamp(min=1).to(torch.float32)
            want = want / counts[:, None]
            terms = terms / counts[:, None]
        want[3] = 0
        terms[3] = 0
        assert_close_terms(got, want, terms, torch.float32)
