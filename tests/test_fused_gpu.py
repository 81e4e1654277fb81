"""The MLP step's fused kernels against the operators they replace.

* tp_b200_gemm_epilogue (gelu): the pre-activation and the activation must
  carry the bits of linear (or mm) followed by gelu -- on the tcgen05
  CTA-pair kernel (products of at least one 256 x 256 tile, including ragged
  edges and operands read transposed in place) and on the decomposed path
  (smaller products);
* tp_b200_gemm_epilogue (gelu_backward): the bits of mm followed by
  gelu_backward;
* tp_b200_mse_loss: the gradient carries the bits of sub followed by mul,
  the loss matches the oracle's mean of the squared (rounded) differences.
Both sides of each bit comparison are also checked against the CPU oracle.
"""

from __future__ import annotations

import pytest
import torch

import oracle as O
from conftest import assert_close, assert_close_terms, assert_equal

pytestmark = pytest.mark.gpu


def _rand(*shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def _epi(N, epilogue, out, aux, a, b, c=None):
    N.check(N.lib().tp_b200_gemm_epilogue(epilogue, N.describe(out), N.describe(aux), N.describe(a), N.describe(b),
                                          N.describe(c) if c is not None else None, 1.0,
                                          1.0 if c is not None else 0.0, 0,
                                          N.stream_of(out.device)), "gemm_epilogue")


SHAPES = [
    (512, 768, 320),    # CTA-pair kernel, whole tiles
    (300, 520, 200),    # CTA-pair kernel, ragged M / N / K
    (8192, 16384, 64),  # the MLP's width, short K
    (128, 256, 64),     # below one 256 x 256 tile: decomposed path
]


@pytest.mark.parametrize("M,Nn,K", SHAPES)
@pytest.mark.parametrize("b_layout", ["k_major", "n_major"])
def test_gelu_epilogue_has_the_bits_of_linear_then_gelu(backend, M, Nn, K, b_layout):
    from tensorplay_mlu_b200 import _native as N

    ops = backend.ops
    x = ops.to_device(_rand(M, K, seed=1))
    bias = ops.to_device(_rand(Nn, seed=3))
    if b_layout == "k_major":       # linear's weight [N, K] read transposed
        w = ops.to_device(_rand(Nn, K, seed=2, scale=K ** -0.5))
        b = w.t()
    else:                            # a plain [K, N] operand
        b = ops.to_device(_rand(K, Nn, seed=2, scale=K ** -0.5))
    h = torch.empty(M, Nn, dtype=torch.bfloat16, device="cuda")
    a = torch.empty_like(h)
    _epi(N, N.EPI_GELU, a, h, x, b, bias)
    want_h = ops.addmm(bias, x, b)
    want_a = ops.gelu(want_h)
    assert_equal(ops.to_host(h), ops.to_host(want_h))
    assert_equal(ops.to_host(a), ops.to_host(want_a))
    # and the pre-activation against the oracle (sampled rows)
    xh, bh, biash = ops.to_host(x), ops.to_host(b), ops.to_host(bias)
    rows = slice(0, min(M, 64))
    ref = O.gemm(xh[rows], bh.contiguous(), biash.view(1, -1).expand(rows.stop, Nn), 1.0, 1.0)
    terms = O.gemm(xh[rows].abs(), bh.contiguous().abs(), biash.abs().view(1, -1).expand(rows.stop, Nn), 1.0, 1.0)
    assert_close_terms(ops.to_host(h)[rows], ref, terms, torch.bfloat16)


@pytest.mark.parametrize("M,Nn,K", SHAPES)
@pytest.mark.parametrize("a_layout", ["k_major", "m_major"])
def test_gelu_backward_epilogue_has_the_bits_of_mm_then_gelu_backward(backend, M, Nn, K, a_layout):
    from tensorplay_mlu_b200 import _native as N

    ops = backend.ops
    if a_layout == "k_major":
        dy = ops.to_device(_rand(M, K, seed=4, scale=1e-3))
    else:
        dy = ops.to_device(_rand(K, M, seed=4, scale=1e-3)).t()
    w = ops.to_device(_rand(K, Nn, seed=5, scale=K ** -0.5))
    h = ops.to_device(_rand(M, Nn, seed=6, scale=2.0))
    d_h = torch.empty(M, Nn, dtype=torch.bfloat16, device="cuda")
    _epi(N, N.EPI_GELU_BACKWARD, d_h, h, dy, w)
    d_a = ops.mm(dy, w)
    want = ops.gelu_backward(d_a, h)
    assert_equal(ops.to_host(d_h), ops.to_host(want))
    assert_close(ops.to_host(want), O.unary_backward(O.GELU_BACKWARD, ops.to_host(d_a), ops.to_host(h)),
                 torch.bfloat16)


def test_epilogue_rejects_bad_arguments(backend):
    from tensorplay_mlu_b200 import _native as N

    x = torch.zeros(256, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="unknown epilogue"):
        _epi(N, 7, x, x.clone(), x, x)
    with pytest.raises(RuntimeError, match="overwrite"):
        _epi(N, N.EPI_GELU_BACKWARD, x, x, x, x)
    with pytest.raises(RuntimeError, match="floating"):
        i = torch.zeros(4, 4, dtype=torch.int32, device="cuda")
        _epi(N, N.EPI_GELU, i, i.clone(), i, i)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("n", [8192 * 4096, 1000003])
def test_mse_loss_and_gradient(backend, dtype, n):
    from tensorplay_mlu_b200 import _native as N

    ops = backend.ops
    out_h = _rand(n, seed=7).to(dtype)
    t_h = _rand(n, seed=8).to(dtype)
    out, t = ops.to_device(out_h), ops.to_device(t_h)
    loss = torch.empty((), dtype=dtype, device="cuda")
    grad = torch.empty_like(out)
    scale = 2.0 / n
    N.check(N.lib().tp_b200_mse_loss(N.describe(loss), N.describe(grad), N.describe(out), N.describe(t), scale,
                                     N.stream_of(out.device)), "mse_loss")
    # gradient: the bits of sub then mul
    diff = ops.sub_Tensor(out, t)
    assert_equal(ops.to_host(grad), ops.to_host(ops.mul_Scalar(diff, scale)))
    # loss: the oracle's mean over the rounded squares
    diff_h = O.binary(O.SUB, out_h, t_h)
    sq = O.unary(O.POW, diff_h, 2.0)
    want = O.reduce(O.MEAN, sq, None, dtype)
    assert_close(ops.to_host(loss), want, dtype)
    assert_close(ops.to_host(loss), ops.to_host(ops.mean(ops.pow_Tensor_Scalar(diff, 2))), dtype)
