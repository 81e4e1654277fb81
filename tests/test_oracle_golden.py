"""The CPU oracle against the golden fixtures (PyTorch CPU outputs on seeded
inputs, tests/golden/make_golden.py) -- the pin that the checker itself is
right before it judges the CUDA path.  CPU only."""

from __future__ import annotations

import os

import pytest
import torch

import oracle as O
from conftest import assert_close, assert_equal

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.pt")
CASES = torch.load(GOLDEN)["cases"]

BINARY = {"add": O.ADD, "sub": O.SUB, "mul": O.MUL, "div": O.DIV, "rsub": O.RSUB}
UNARY = {"exp": O.EXP, "log": O.LOG, "sqrt": O.SQRT, "rsqrt": O.RSQRT, "neg": O.NEG, "abs": O.ABS,
         "pow": O.POW, "relu": O.RELU, "sigmoid": O.SIGMOID, "tanh": O.TANH, "silu": O.SILU,
         "gelu": O.GELU, "gelu_tanh": O.GELU_TANH}
BACKWARD = {"threshold_backward": O.THRESHOLD_BACKWARD, "sigmoid_backward": O.SIGMOID_BACKWARD,
            "tanh_backward": O.TANH_BACKWARD, "gelu_backward": O.GELU_BACKWARD,
            "gelu_tanh_backward": O.GELU_TANH_BACKWARD, "silu_backward": O.SILU_BACKWARD}
REDUCE = {"sum": O.SUM, "mean": O.MEAN, "amax": O.AMAX, "amin": O.AMIN}


def oracle_output(case):
    kind, p, ins = case["kind"], case["params"], case["inputs"]
    if kind == "binary":
        a, b = ins
        if p["op"] == "div":
            b = O.binary_scalar(O.ADD, O.unary(O.ABS, b), 1.0)
            return O.binary(O.DIV, a, b)
        alpha = p.get("alpha", {"add": 0.5, "sub": 2}.get(p["op"], 1))
        return O.binary(BINARY[p["op"]], a, b, alpha)
    if kind == "scalar":
        return O.binary_scalar(BINARY[p["op"]], ins[0], p["s"], p["alpha"])
    if kind == "scalar_chain":
        return O.binary_scalar(O.ADD, O.binary_scalar(O.MUL, ins[0], 3), 1)
    if kind == "unary":
        return O.unary(UNARY[p["op"]], ins[0], p.get("p", 0.0))
    if kind == "unary_backward":
        return O.unary_backward(BACKWARD[p["op"]], ins[0], ins[1], p.get("p", 0.0))
    if kind == "reduce":
        x = ins[0]
        out_dtype = x.dtype
        if p["op"] == "sum" and not x.dtype.is_floating_point:
            out_dtype = torch.int64
        return O.reduce(REDUCE[p["op"]], x, p["dims"], out_dtype)
    if kind == "softmax":
        return O.softmax(ins[0], p["dim"], p["log"])
    if kind == "softmax_backward":
        return O.softmax_backward(ins[0], ins[1], p["dim"], p["log"])
    if kind == "gemm":
        if len(ins) == 3:
            return O.gemm(ins[0], ins[1], ins[2], p["alpha"], p["beta"])
        return O.gemm(ins[0], ins[1])
    if kind == "cast":
        return O.cast(ins[0], p["dtype"])
    if kind == "gather":
        return O.gather(ins[0], p["dim"], ins[1])
    if kind == "index_select":
        return O.index_select(ins[0], p["dim"], ins[1])
    if kind == "scatter":
        return O.scatter(ins[0], p["dim"], ins[1], ins[2], p["reduce"], p["include_self"])
    if kind == "scan":
        return O.scan(ins[0], p["dim"], p["product"])
    if kind == "where":
        return O.where(*ins)
    if kind == "index_add":
        return O.index_add_zeros(p["shape"], p["dim"], ins[0], ins[1])
    if kind == "layer_norm":
        x, w, b = (ins + [None, None])[:3]
        y, mean, rstd = O.layer_norm(x, p["norm"], w, b, p["eps"])
        return {"y": y, "mean": mean, "rstd": rstd}[p["part"]]
    if kind == "layer_norm_backward":
        dy, x, mean, rstd = ins[:4]
        w = ins[4] if len(ins) > 4 else None
        dx, dw, db = O.layer_norm_backward(dy, x, p["norm"], mean, rstd, w)
        return {"dx": dx, "dw": dw, "db": db}[p["part"]]
    if kind == "nll_loss":
        x, t = ins[:2]
        w = ins[2] if len(ins) > 2 else None
        out, total = O.nll_loss(x, t, w, p["reduction"], -100)
        return {"out": out, "total": total}[p["part"]]
    if kind == "nll_loss_backward":
        g, x, t, total = ins[:4]
        w = ins[4] if len(ins) > 4 else None
        return O.nll_loss_backward(g, x, t, w, p["reduction"], -100, total)
    raise AssertionError(kind)


EXACT_KINDS = {"cast", "scalar_chain", "gather", "index_select", "where"}


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_golden(case):
    got = oracle_output(case)
    want = case["output"]
    exact = (case["kind"] in EXACT_KINDS or not want.dtype.is_floating_point
             or case["params"].get("op") in ("amax", "amin", "neg", "abs", "relu"))
    if exact:
        assert_equal(got, want)
    else:
        scale = 1.0
        if case["kind"] == "gemm":
            scale = 4.0  # reduction order: oracle accumulates in double, PyTorch in fp32
        if case["kind"] == "reduce" and case["params"]["op"] == "sum":
            scale = 20.0
        if case["kind"].startswith("layer_norm") or case["kind"].startswith("nll"):
            scale = 4.0  # fp32 / 16-bit statistics and sums rounded in a different order
        got = got.to(want.dtype) if got.dtype != want.dtype else got
        assert_close(got, want, want.dtype, scale)


def test_golden_covers_every_family():
    kinds = {c["kind"] for c in CASES}
    assert {"binary", "scalar", "unary", "unary_backward", "reduce", "softmax", "softmax_backward",
            "gemm", "cast", "scalar_chain", "layer_norm", "layer_norm_backward", "nll_loss",
            "nll_loss_backward", "gather", "index_select", "scatter", "scan", "where", "index_add"} <= kinds


def test_oracle_mlp_step_matches_torch_autograd():
    """The oracle's MLP step (the CPU baseline's workload) against PyTorch
    autograd at a small size, bf16 storage / fp32 math."""
    torch.manual_seed(0)
    D, H, R = 32, 64, 8
    g = torch.Generator().manual_seed(0)
    w1 = (torch.rand(H, D, generator=g) * 2 - 1).mul(D ** -0.5).bfloat16()
    b1 = (torch.rand(H, generator=g) * 2 - 1).mul(D ** -0.5).bfloat16()
    w2 = (torch.rand(D, H, generator=g) * 2 - 1).mul(H ** -0.5).bfloat16()
    b2 = (torch.rand(D, generator=g) * 2 - 1).mul(H ** -0.5).bfloat16()
    x = torch.randn(R, D, generator=g).bfloat16()
    t = torch.randn(R, D, generator=g).bfloat16()
    params = [p.float().requires_grad_() for p in (w1, b1, w2, b2)]
    h = x.float() @ params[0].t() + params[1]
    o = torch.nn.functional.gelu(h) @ params[2].t() + params[3]
    loss = ((o - t.float()) ** 2).mean()
    loss.backward()
    lr = 0.1
    want = [(p - lr * p.grad).detach() for p in params]
    ow = [w1.clone(), b1.clone(), w2.clone(), b2.clone()]
    got_loss = O.mlp_step(x, t, *ow, lr)
    assert abs(got_loss - loss.item()) <= 2e-2 * max(1.0, loss.item())
    for got, ref in zip(ow, want):
        assert (got.float() - ref).abs().max().item() <= 2e-2 * max(ref.abs().max().item(), 1.0)


def test_philox_matches_the_published_known_answers():
    """Philox-4x32-10 (the dropout generator) against the Random123
    known-answer vectors for 10 rounds."""
    kat = [((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
           ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
           ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
            (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1))]
    for ctr, key, want in kat:
        assert tuple(O.philox4x32_10(ctr, key)) == want
