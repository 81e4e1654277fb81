"""Generate the golden fixtures that pin the CPU oracle.

TensorPlay's own CPU kernels (the reference's host path) cannot be installed
here, so the fixtures come from PyTorch 2.11 CPU, which implements the same
operator schemas (ATen) TensorPlay's kernels follow.  Every case is a small,
seeded input; the fixture stores inputs and PyTorch's outputs.  Reference
tests that pin exact values (tensorplay-mlu tests/test_mlu.py:64-132 round
trips and casts, :196-198 integer x*3+1, tests/test_mlu_distributed.py
single-rank identities) are restated as exact cases.

Run:  python tests/golden/make_golden.py     (writes tests/golden/golden.pt)
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "golden.pt")


def rand(*shape, dtype=torch.float32, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


def randint(*shape, low=-1000, high=1000, dtype=torch.int32, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(low, high, shape, generator=g).to(dtype)


def main() -> None:
    cases = []

    def add(kind, name, inputs, output, **params):
        cases.append({"kind": kind, "name": name, "inputs": inputs, "output": output, "params": params})

    float_types = [torch.float32, torch.bfloat16, torch.float16, torch.float64]
    # ---- binary with broadcasting (test_mlu.py:137-145 shapes)
    for dt in float_types:
        a, b = rand(4, 1, 5, dtype=dt), rand(3, 1, dtype=dt, seed=1)
        for op, fn in (("add", lambda x, y: torch.add(x, y, alpha=0.5)),
                       ("sub", lambda x, y: torch.sub(x, y, alpha=2)),
                       ("mul", torch.mul), ("div", lambda x, y: torch.div(x, y.abs() + 1))):
            add("binary", f"{op}_{dt}", [a, b], fn(a, b), op=op)
    for dt in (torch.int32, torch.int64, torch.int16, torch.int8, torch.uint8):
        lo, hi = (0, 100) if dt == torch.uint8 else (-100, 100)
        a, b = randint(6, 5, low=lo, high=hi, dtype=dt), randint(5, low=lo, high=hi, dtype=dt, seed=1)
        add("binary", f"add_{dt}", [a, b], torch.add(a, b, alpha=3), op="add", alpha=3)
        add("binary", f"sub_{dt}", [a, b], torch.sub(a, b), op="sub", alpha=1)
        add("binary", f"mul_{dt}", [a, b], torch.mul(a, b), op="mul", alpha=1)
    # int32 overflow wraps (two's complement), as on the host
    a = torch.tensor([2**31 - 1, -2**31, 123456789], dtype=torch.int32)
    b = torch.tensor([1, -1, 987654321], dtype=torch.int32)
    add("binary", "add_int32_wrap", [a, b], a + b, op="add", alpha=1)
    add("binary", "mul_int32_wrap", [a, b], a * b, op="mul", alpha=1)
    # ---- scalar forms (test_mlu.py:148-158)
    for dt in float_types:
        a = rand(8, 3, dtype=dt)
        add("scalar", f"add2_{dt}", [a], a + 2, op="add", s=2.0, alpha=1.0)
        add("scalar", f"mul3_{dt}", [a], a * 3, op="mul", s=3.0, alpha=1.0)
        add("scalar", f"div4_{dt}", [a], a / 4, op="div", s=4.0, alpha=1.0)
        add("scalar", f"rsub1_{dt}", [a], 1 - a, op="rsub", s=1.0, alpha=1.0)
    ar = torch.arange(10)
    add("scalar_chain", "int_x3_plus1", [ar], ar * 3 + 1)  # test_mlu.py:196-198
    # ---- unary (test_mlu.py:201-216)
    for dt in (torch.float32, torch.bfloat16, torch.float64, torch.float16):
        a = rand(33, 17, dtype=dt)
        pos = (a.abs() + 0.1).to(dt)
        for name, fn, x in (("exp", torch.exp, a), ("log", torch.log, pos), ("sqrt", torch.sqrt, pos),
                            ("rsqrt", torch.rsqrt, pos), ("neg", torch.neg, a), ("abs", torch.abs, a),
                            ("relu", torch.relu, a), ("sigmoid", torch.sigmoid, a), ("tanh", torch.tanh, a),
                            ("silu", F.silu, a), ("gelu", F.gelu, a),
                            ("gelu_tanh", lambda v: F.gelu(v, approximate="tanh"), a)):
            add("unary", f"{name}_{dt}", [x], fn(x), op=name)
        base = (rand(6, 9, dtype=torch.float32).abs() + 0.5).to(dt)
        for e in (2, 1, 0, 0.5, -0.5, 3, 1.7):
            add("unary", f"pow{e}_{dt}", [base], base ** e, op="pow", p=float(e))
    for dt in (torch.int32, torch.int64):
        a = randint(7, 5, low=-9, high=9, dtype=dt)
        add("unary", f"neg_{dt}", [a], torch.neg(a), op="neg")
        add("unary", f"abs_{dt}", [a], torch.abs(a), op="abs")
        add("unary", f"relu_{dt}", [a], torch.relu(a), op="relu")
        add("unary", f"pow3_{dt}", [a], a ** 3, op="pow", p=3.0)
    # ---- activation backward
    for dt in (torch.float32, torch.bfloat16, torch.float64):
        x, dy = rand(16, 32, dtype=dt, seed=2), rand(16, 32, dtype=dt, seed=3)
        math_dt = torch.float64 if dt == torch.float64 else torch.float32
        xr = x.detach().to(math_dt).requires_grad_()
        for name, fn in (("gelu", F.gelu), ("gelu_tanh", lambda v: F.gelu(v, approximate="tanh")),
                         ("silu", F.silu)):
            xr.grad = None
            fn(xr).backward(dy.to(math_dt))
            add("unary_backward", f"{name}_bwd_{dt}", [dy, x], xr.grad.to(dt), op=f"{name}_backward")
        y = torch.sigmoid(x)
        add("unary_backward", f"sigmoid_bwd_{dt}", [dy, y],
            torch.ops.aten.sigmoid_backward(dy, y), op="sigmoid_backward")
        y = torch.tanh(x)
        add("unary_backward", f"tanh_bwd_{dt}", [dy, y], torch.ops.aten.tanh_backward(dy, y),
            op="tanh_backward")
        add("unary_backward", f"threshold_bwd_{dt}", [dy, x],
            torch.ops.aten.threshold_backward(dy, x, 0.0), op="threshold_backward", p=0.0)
    # ---- reductions (test_mlu.py:303-333)
    for dt in (torch.float32, torch.bfloat16, torch.float64):
        a = rand(6, 7, 8, dtype=dt)
        add("reduce", f"sum_all_{dt}", [a], a.sum(), op="sum", dims=None)
        add("reduce", f"sum_d1_{dt}", [a], a.sum(dim=1), op="sum", dims=[1])
        add("reduce", f"sum_d02_{dt}", [a], a.sum(dim=(0, 2)), op="sum", dims=[0, 2])
        add("reduce", f"mean_all_{dt}", [a], a.mean(), op="mean", dims=None)
        add("reduce", f"mean_dm1_{dt}", [a], a.mean(dim=-1), op="mean", dims=[2])
        add("reduce", f"amax_dm1_{dt}", [a], a.amax(dim=-1), op="amax", dims=[2])
        add("reduce", f"amin_d0_{dt}", [a], a.amin(dim=0), op="amin", dims=[0])
        b = rand(3, 5000, dtype=dt, seed=5)
        add("reduce", f"sum_long_{dt}", [b], b.sum(dim=1), op="sum", dims=[1])
    for dt in (torch.int32, torch.int64, torch.int8):
        a = randint(16, 300, low=-100, high=100, dtype=dt)
        add("reduce", f"sum_all_{dt}", [a], a.sum(), op="sum", dims=None)
        add("reduce", f"sum_d0_{dt}", [a], a.sum(dim=0), op="sum", dims=[0])
        add("reduce", f"amax_dm1_{dt}", [a], a.amax(dim=-1), op="amax", dims=[1])
        add("reduce", f"amin_all_{dt}", [a], a.amin(), op="amin", dims=None)
    # ---- softmax (test_mlu.py:344-350)
    for dt in (torch.float32, torch.bfloat16, torch.float64):
        a = rand(5, 6, 7, dtype=dt)
        dy = rand(5, 6, 7, dtype=dt, seed=7)
        for dim in (0, 1, -1):
            y = torch.softmax(a, dim=dim)
            ly = torch.log_softmax(a, dim=dim)
            add("softmax", f"softmax_{dim}_{dt}", [a], y, dim=dim, log=False)
            add("softmax", f"log_softmax_{dim}_{dt}", [a], ly, dim=dim, log=True)
            add("softmax_backward", f"softmax_bwd_{dim}_{dt}", [dy, y],
                torch.ops.aten._softmax_backward_data(dy, y, dim, dt), dim=dim, log=False)
            add("softmax_backward", f"log_softmax_bwd_{dim}_{dt}", [dy, ly],
                torch.ops.aten._log_softmax_backward_data(dy, ly, dim, dt), dim=dim, log=True)
    # ---- GEMM (test_mlu.py:238-286)
    for dt in (torch.float32, torch.bfloat16, torch.float64, torch.int32):
        if dt == torch.int32:
            a, b = randint(37, 19, low=-9, high=9, dtype=dt), randint(19, 23, low=-9, high=9, dtype=dt, seed=3)
        else:
            a, b = rand(37, 19, dtype=dt), rand(19, 23, dtype=dt, seed=3)
        for ta in (False, True):
            for tb in (False, True):
                aa = a.t().contiguous().t() if ta else a
                bb = b.t().contiguous().t() if tb else b
                add("gemm", f"mm_{int(ta)}{int(tb)}_{dt}", [aa, bb], aa @ bb)
    for dt in (torch.float32, torch.bfloat16):
        bias, a, b = rand(23, dtype=dt), rand(37, 19, dtype=dt, seed=1), rand(19, 23, dtype=dt, seed=2)
        add("gemm", f"addmm_{dt}", [a, b, bias], torch.addmm(bias, a, b, beta=0.5, alpha=2.0),
            alpha=2.0, beta=0.5)
        x, y = rand(4, 9, 6, dtype=dt), rand(4, 6, 5, dtype=dt, seed=4)
        add("gemm", f"bmm_{dt}", [x, y], torch.bmm(x, y))
    # ---- layer_norm forward / backward (NNKernels.cpp:59-161), one case per output
    aten = torch.ops.aten
    for dt in float_types:
        for shape, norm, affine in (((6, 20), [20], True), ((3, 4, 16), [4, 16], True), ((5, 33), [33], False)):
            x = rand(*shape, dtype=dt, seed=11, scale=2.0)
            w = rand(*norm, dtype=dt, seed=12) if affine else None
            b = rand(*norm, dtype=dt, seed=13) if affine else None
            y, mean, rstd = aten.native_layer_norm(x, norm, w, b, 1e-5)
            tag = f"{'x'.join(map(str, shape))}_{dt}"
            ins = [x] + ([w, b] if affine else [])
            for part, out in (("y", y), ("mean", mean.reshape(-1)), ("rstd", rstd.reshape(-1))):
                add("layer_norm", f"layer_norm_{part}_{tag}", ins, out, norm=norm, part=part, eps=1e-5)
            dy = rand(*shape, dtype=dt, seed=14)
            dx, dw, db = aten.native_layer_norm_backward(dy, x, norm, mean, rstd, w, b, [True, affine, affine])
            bins = [dy, x, mean.reshape(-1).float() if dt != torch.float64 else mean.reshape(-1),
                    rstd.reshape(-1).float() if dt != torch.float64 else rstd.reshape(-1)] + ([w] if affine else [])
            add("layer_norm_backward", f"layer_norm_backward_dx_{tag}", bins, dx, norm=norm, part="dx")
            if affine:
                add("layer_norm_backward", f"layer_norm_backward_dw_{tag}", bins, dw, norm=norm, part="dw")
                add("layer_norm_backward", f"layer_norm_backward_db_{tag}", bins, db, norm=norm, part="db")
    # ---- nll_loss forward / backward (NNKernels.cpp:304-397), class weights and ignore_index
    for dt in float_types:
        x = torch.log_softmax(rand(9, 7, seed=15, scale=2.0), 1).to(dt)
        t = torch.tensor([0, 3, 6, -100, 2, 2, 5, 1, -100], dtype=torch.int64)
        wt = (rand(7, seed=16).abs() + 0.5).to(dt)
        for red in (0, 1, 2):
            for w_on in (False, True):
                w = wt if w_on else None
                out, total = aten.nll_loss_forward(x, t, w, red, -100)
                tag = f"r{red}_{'w' if w_on else 'nw'}_{dt}"
                ins = [x, t] + ([w] if w_on else [])
                add("nll_loss", f"nll_loss_out_{tag}", ins, out, reduction=red, part="out")
                if red != 0:
                    add("nll_loss", f"nll_loss_total_{tag}", ins, total, reduction=red, part="total")
                g = rand(9, dtype=dt, seed=17) if red == 0 else torch.tensor(1.5, dtype=dt)
                dx = aten.nll_loss_backward(g, x, t, w, red, -100, total)
                add("nll_loss_backward", f"nll_loss_backward_{tag}", [g, x, t, total] + ([w] if w_on else []), dx,
                    reduction=red)
    # ---- index family (IndexKernels.cpp:352-367): gather, index_select, scatter*, scans, where
    g = torch.Generator().manual_seed(21)
    for dt in float_types + [torch.int32, torch.int64]:
        x = rand(5, 6, dtype=dt, seed=22, scale=3.0) if dt.is_floating_point else randint(5, 6, low=-50, high=50, dtype=dt, seed=22)
        idx = torch.randint(0, 5, (4, 6), generator=g)
        add("gather", f"gather_d0_{dt}", [x, idx], torch.gather(x, 0, idx), dim=0)
        idx1 = torch.randint(-6, 6, (5, 3), generator=g)
        add("gather", f"gather_d1_neg_{dt}", [x, idx1], torch.gather(x, 1, idx1 % 6), dim=1)
        sel = torch.tensor([4, 0, 2, 2, -1])
        add("index_select", f"index_select_{dt}", [x, sel], torch.index_select(x, 0, sel % 5), dim=0)
        src = rand(4, 6, dtype=dt, seed=23) if dt.is_floating_point else randint(4, 6, low=-9, high=9, dtype=dt, seed=23)
        add("scatter", f"scatter_add_{dt}", [x, idx, src], torch.scatter_add(x, 0, idx, src), dim=0, reduce="add",
            include_self=True)
        perm = torch.stack([torch.randperm(5, generator=g)[:4] for _ in range(6)], 1)  # no duplicates
        add("scatter", f"scatter_replace_{dt}", [x, perm, src], torch.scatter(x, 0, perm, src), dim=0, reduce=None,
            include_self=True)
        for red in ("sum", "prod", "amax", "amin", "mean"):
            for inc in (True, False):
                want = x.scatter_reduce(0, idx, src, reduce=red, include_self=inc)
                add("scatter", f"scatter_reduce_{red}_{'self' if inc else 'noself'}_{dt}", [x, idx, src], want,
                    dim=0, reduce=red, include_self=inc)
        add("scan", f"cumsum_d1_{dt}", [x], torch.cumsum(x, 1, dtype=dt), dim=1, product=False)
        add("scan", f"cumsum_d0_{dt}", [x], torch.cumsum(x, 0, dtype=dt), dim=0, product=False)
        xs = (x.double() / 4).to(dt) if dt.is_floating_point else (x % 3).to(dt)
        add("scan", f"cumprod_d1_{dt}", [xs], torch.cumprod(xs, 1, dtype=dt), dim=1, product=True)
        cond = torch.rand(5, 1, generator=g) > 0.5
        other = src[:1]
        add("where", f"where_{dt}", [cond, x, other], torch.where(cond, x, other))
        gsrc = rand(5, 6, dtype=dt, seed=24) if dt.is_floating_point else randint(5, 6, low=-9, high=9, dtype=dt, seed=24)
        add("index_add", f"index_select_backward_{dt}", [sel, gsrc], torch.zeros(5, 6, dtype=dt).index_add(0, sel % 5, gsrc),
            shape=[5, 6], dim=0)
    # ---- casts (test_mlu.py:90-98) and round trips (:64-69): exact
    src = rand(3, 9, scale=4.0)
    for s, d in ((torch.float32, torch.float16), (torch.float16, torch.float32),
                 (torch.float32, torch.bfloat16), (torch.float16, torch.bfloat16),
                 (torch.float32, torch.int32), (torch.int64, torch.float32),
                 (torch.float64, torch.float32), (torch.float32, torch.float64),
                 (torch.float64, torch.bfloat16), (torch.int32, torch.bool),
                 (torch.bfloat16, torch.int64), (torch.uint8, torch.float16)):
        x = src.to(s) if s != torch.uint8 else src.abs().to(s)
        add("cast", f"cast_{s}_{d}", [x], x.to(d), dtype=d)
    torch.save({"torch_version": str(torch.__version__), "cases": cases}, OUT)
    print(f"{len(cases)} cases -> {OUT} ({os.path.getsize(OUT)} bytes)")


if __name__ == "__main__":
    main()
