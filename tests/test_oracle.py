"""CPU tests: the oracle against the reference's known answers (tests/golden) and
against float64 numpy restatements on small random cases."""
import json
import os

import numpy as np
import pytest

from conftest import assert_close

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_known_answers.json")


def load_cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


def seq(shape):
    return np.arange(int(np.prod(shape)), dtype=np.float32).reshape(shape)


@pytest.mark.parametrize("case", [c for c in load_cases() if c["op"] == "Conv"], ids=lambda c: c["name"])
def test_conv_known_answers(oracle, case):
    x = np.array(case["x"], np.float32)
    w = np.array(case["w"], np.float32)
    exp = np.array(case["expected"], np.float32)
    if x.ndim == 4:
        for strat in (oracle.ORC_CONV_DIRECT if hasattr(oracle, "ORC_CONV_DIRECT") else 1, 2):
            y = oracle.conv2d(x, w, None, strides=case["strides"], pads=case.get("pads", [0, 0, 0, 0]),
                              dilations=case["dilations"], group=case["group"],
                              auto_pad=case.get("auto_pad", "NOTSET"), strategy=strat)
            assert list(y.shape) == case["expected_shape"]
            # the reference asserts exact equality (conv.rs:1523-1528, 1580-1589, 1680-1691)
            np.testing.assert_array_equal(y, exp)
    else:
        y = oracle.conv_nd_direct(x, w, None, case["strides"], case.get("pads"), case["dilations"], case["group"])
        assert list(y.shape) == case["expected_shape"]
        np.testing.assert_array_equal(y, exp)


@pytest.mark.parametrize("case", [c for c in load_cases() if c["op"] == "MatMul"], ids=lambda c: c["name"])
def test_matmul_known_answers(oracle, case):
    a, b = seq(case["a_shape"]), seq(case["b_shape"])
    y = oracle.matmul(a, b)
    assert list(y.shape) == case["expected_shape"]
    np.testing.assert_array_equal(y, np.array(case["expected"], np.float32).reshape(y.shape))


def test_matmul_shape_validation(oracle):
    case = next(c for c in load_cases() if c["op"] == "MatMulShape")
    for v in case["valid"]:
        assert oracle.matmul_shape(v["a"], v["b"]) == v["out"]
    for v in case["invalid"]:
        with pytest.raises(oracle.OracleError):
            oracle.matmul_shape(v["a"], v["b"])


def test_broadcast_known_answer(oracle):
    case = next(c for c in load_cases() if c["op"] == "Add")
    y = oracle.add(np.array(case["a"], np.float32), np.array(case["b"], np.float32))
    np.testing.assert_array_equal(y, np.array(case["expected"], np.float32))


def np_conv(x, w, b, s, p, d, g):
    x = x.astype(np.float64)
    w = w.astype(np.float64)
    n, c, h, wd = x.shape
    co, cg, kh, kw = w.shape
    oh = (h + p[0] + p[2] - (kh - 1) * d[0] - 1) // s[0] + 1
    ow = (wd + p[1] + p[3] - (kw - 1) * d[1] - 1) // s[1] + 1
    xp = np.zeros((n, c, h + p[0] + p[2], wd + p[1] + p[3]))
    xp[:, :, p[0]:p[0] + h, p[1]:p[1] + wd] = x
    y = np.zeros((n, co, oh, ow))
    cog = co // g
    for gi in range(g):
        for r in range(kh):
            for t in range(kw):
                patch = xp[:, gi * cg:(gi + 1) * cg, r * d[0]: r * d[0] + s[0] * (oh - 1) + 1: s[0],
                           t * d[1]: t * d[1] + s[1] * (ow - 1) + 1: s[1]]
                y[:, gi * cog:(gi + 1) * cog] += np.einsum("nchw,oc->nohw", patch, w[gi * cog:(gi + 1) * cog, :, r, t])
    if b is not None:
        y += b.reshape(1, -1, 1, 1)
    return y


CONV_CASES = [
    # (n, c, h, w, co, k, stride, pad, dil, group)
    (2, 3, 17, 19, 8, 7, 2, 3, 1, 1),
    (1, 16, 9, 9, 12, 3, 1, 1, 1, 1),
    (2, 8, 10, 7, 8, 3, 1, 2, 2, 1),
    (1, 8, 6, 6, 8, 3, 1, 1, 1, 4),
    (3, 5, 5, 5, 6, 1, 1, 0, 1, 1),
    (1, 4, 8, 8, 4, 2, 2, 0, 1, 1),
]


@pytest.mark.parametrize("cs", CONV_CASES)
@pytest.mark.parametrize("strategy", [1, 2])
def test_conv_vs_numpy(oracle, cs, strategy):
    n, c, h, w, co, k, s, p, d, g = cs
    rng = np.random.default_rng(0)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = rng.standard_normal((co, c // g, k, k)).astype(np.float32)
    b = rng.standard_normal(co).astype(np.float32)
    y = oracle.conv2d(x, wt, b, (s, s), (p, p, p, p), (d, d), g, strategy=strategy)
    ref = np_conv(x, wt, b, (s, s), (p, p, p, p), (d, d), g)
    assert_close(y, ref, 1e-5, 1e-4, "conv")
    y64 = oracle.conv2d(x, wt, b, (s, s), (p, p, p, p), (d, d), g, strategy=strategy, acc64=True)
    assert_close(y64, ref, 1e-6, 1e-6, "conv acc64")


def test_conv_strategy_matches_reference(oracle):
    # optimize_convolution_strategy (conv.rs:1425-1452): SIMD=3 for power-of-2 kernels, else Im2Col=2
    assert oracle.conv_strategy(1, 1, 1) == 3
    assert oracle.conv_strategy(3, 3, 1) == 2
    assert oracle.conv_strategy(7, 7, 1) == 2
    assert oracle.conv_strategy(3, 3, 32) == 2
    assert oracle.conv_strategy(1, 1, 2) == 2
    assert oracle.conv_strategy(13, 13, 1) == 1


def test_same_padding(oracle):
    assert oracle.same_pads(3, 3, 1, 1, True) == (1, 1)
    assert oracle.same_pads(224, 7, 2, 1, True) == (2, 3)
    assert oracle.same_pads(224, 7, 2, 1, False) == (3, 2)


@pytest.mark.parametrize("sa,sb", [((3, 5), (5, 4)), ((2, 1, 4, 6), (3, 6, 5)), ((6,), (6, 3)), ((4, 6), (6,)),
                                   ((2, 3, 4), (4,)), ((7,), (7,))])
def test_matmul_vs_numpy(oracle, sa, sb):
    rng = np.random.default_rng(1)
    a = rng.standard_normal(sa).astype(np.float32)
    b = rng.standard_normal(sb).astype(np.float32)
    assert_close(oracle.matmul(a, b), np.matmul(a.astype(np.float64), b.astype(np.float64)), 1e-5, 1e-5)


@pytest.mark.parametrize("ta,tb,cshape,alpha,beta", [(0, 0, (4,), 1.0, 1.0), (1, 0, (3, 4), 0.5, 2.0),
                                                      (0, 1, None, 1.5, 0.0), (1, 1, (3, 1), 1.0, -1.0),
                                                      (0, 1, (), 1.0, 1.0)])
def test_gemm_vs_numpy(oracle, ta, tb, cshape, alpha, beta):
    rng = np.random.default_rng(2)
    m, n, k = 3, 4, 5
    a = rng.standard_normal((k, m) if ta else (m, k)).astype(np.float32)
    b = rng.standard_normal((n, k) if tb else (k, n)).astype(np.float32)
    c = None if cshape is None else rng.standard_normal(cshape).astype(np.float32)
    y = oracle.gemm(a, b, c, alpha, beta, ta, tb)
    ref = alpha * ((a.T if ta else a).astype(np.float64) @ (b.T if tb else b).astype(np.float64))
    if c is not None:
        ref = ref + beta * c.astype(np.float64)
    assert_close(y, ref, 1e-5, 1e-5)


def test_maxpool_semantics(oracle):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 3, 9, 8)).astype(np.float32)
    y, idx = oracle.maxpool2d(x, (3, 3), (2, 2), (1, 1, 1, 1), with_indices=True)
    assert y.shape == (2, 3, 5, 4)
    flat = x.reshape(-1)
    np.testing.assert_array_equal(flat[idx], y)  # indices point at the maxima
    # window max by brute force
    xp = np.full((2, 3, 11, 10), -np.inf, np.float32)
    xp[:, :, 1:10, 1:9] = x
    ref = np.stack([np.stack([xp[:, :, 2 * i:2 * i + 3, 2 * j:2 * j + 3].max(axis=(2, 3)) for j in range(4)], -1)
                    for i in range(5)], -2)
    np.testing.assert_array_equal(y, ref)


def test_maxpool_first_max_and_nan(oracle):
    x = np.array([[[[1, 1], [1, np.nan]]]], np.float32)
    y, idx = oracle.maxpool2d(x, (2, 2), (2, 2), (0, 0, 0, 0), with_indices=True)
    assert y[0, 0, 0, 0] == 1.0 and idx[0, 0, 0, 0] == 0  # f32::max ignores NaN; first max wins


def test_global_avgpool_relu_add_bn(oracle):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 5, 7, 7)).astype(np.float32)
    g = oracle.global_avgpool(x)
    assert g.shape == (2, 5, 1, 1)
    assert_close(g, x.astype(np.float64).mean(axis=(2, 3), keepdims=True), 1e-6, 1e-6)
    r = oracle.relu(np.array([-1.0, 0.0, 2.0, np.nan, -0.0], np.float32))
    np.testing.assert_array_equal(r, [0.0, 0.0, 2.0, 0.0, 0.0])
    a = rng.standard_normal((2, 5, 1, 7)).astype(np.float32)
    b = rng.standard_normal((5, 3, 1)).astype(np.float32)
    np.testing.assert_array_equal(oracle.add(a, b), a + b)
    sc, bi, mu, var = (rng.standard_normal(5).astype(np.float32) for _ in range(4))
    var = np.abs(var) + 0.5
    y = oracle.batchnorm(x, sc, bi, mu, var, 1e-5)
    ref = (x - mu.reshape(1, -1, 1, 1)) / np.sqrt(var.reshape(1, -1, 1, 1) + 1e-5) * sc.reshape(1, -1, 1, 1) \
        + bi.reshape(1, -1, 1, 1)
    assert_close(y, ref, 1e-6, 1e-6)


def test_invalid_inputs(oracle):
    with pytest.raises(oracle.OracleError):
        oracle.add(np.zeros((2, 3), np.float32), np.zeros((3, 2), np.float32))
    with pytest.raises(oracle.OracleError):
        oracle.matmul(np.zeros((2, 3), np.float32), np.zeros((4, 5), np.float32))
    with pytest.raises(oracle.OracleError):
        oracle.gemm(np.zeros((2, 3), np.float32), np.zeros((3, 4), np.float32), np.zeros((3, 4), np.float32))


def test_empty_batch(oracle):
    x = np.zeros((0, 3, 8, 8), np.float32)
    w = np.ones((4, 3, 3, 3), np.float32)
    y = oracle.conv2d(x, w, None, (1, 1), (1, 1, 1, 1))
    assert y.shape == (0, 4, 8, 8)
