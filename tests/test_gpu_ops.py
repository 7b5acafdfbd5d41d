"""GPU parity tests: every op of the path through the C ABI against the oracle.

Tolerances (element passes if |a-b| <= atol or |a-b|/|b| <= rtol):
  3xTF32 and fp32 CUDA-core paths: rtol 1e-5, atol 1e-4 per op;
  tf32 / bf16 fast modes: 2e-2 (rtol and atol);
  pooling indices, Relu, Add, GlobalAveragePool (same summation order): bit-exact.
"""
import numpy as np
import pytest
import torch

from conftest import assert_close

pytestmark = pytest.mark.gpu

TOL = {"3xtf32": (1e-5, 1e-4), "fp32": (1e-5, 1e-4), "tf32": (2e-2, 2e-2), "bf16": (2e-2, 2e-2)}


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def np_(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.fixture(scope="module")
def ctx(ob, handle):
    return ob.ExecutionContext(handle)


def run_conv(ob, ctx, x, w, b, attrs, precision, relu=False, bn=None, residual=None, layout=0):
    conv = ob.Conv(attrs.get("strides", (1, 1)), attrs.get("pads", (0, 0, 0, 0)), attrs.get("dilations", (1, 1)),
                   attrs.get("group", 1), attrs.get("auto_pad", "NOTSET"), precision=precision, relu=relu)
    ins = [cu(x), cu(w)] + ([cu(b)] if b is not None else [])
    bnd = None if bn is None else tuple(cu(v) for v in bn[:4]) + (bn[4],)
    y = conv.compute(ins, ctx, bn=bnd, residual=None if residual is None else cu(residual), layout=layout)[0]
    ctx.handle.synchronize()
    return np_(y)


SMALL = [
    # name, (n, c, h, w), co, k, stride, pad, dil, group
    ("stem_like", (2, 3, 33, 29), 64, 7, 2, 3, 1, 1),
    ("c64_3x3", (2, 64, 14, 14), 64, 3, 1, 1, 1, 1),
    ("c32_1x1_odd_m", (3, 32, 7, 5), 96, 1, 1, 0, 1, 1),
    ("c48_3x3_s2", (2, 48, 15, 15), 128, 3, 2, 1, 1, 1),
    ("c16_dil2", (1, 16, 20, 20), 32, 3, 1, 2, 2, 1),
    ("c128_1x1_wide", (2, 128, 8, 8), 256, 1, 1, 0, 1, 1),
    ("c8_co20", (1, 8, 9, 9), 20, 3, 1, 1, 1, 1),
    ("grouped", (2, 32, 10, 10), 32, 3, 1, 1, 1, 8),
    ("grouped_cg8_s2", (2, 32, 9, 11), 16, 3, 2, 1, 1, 4),
    ("grouped_cg3", (1, 12, 8, 8), 12, 3, 1, 1, 1, 4),
    # grouped 3x3 over row segments: segments past the row end, weight slices
    # narrower than CO, stride 2, no padding, two output channels per input one
    ("grouped_cg32_sliced", (2, 256, 9, 13), 256, 3, 1, 1, 1, 8),
    ("grouped_g32_s2_odd", (3, 128, 15, 17), 128, 3, 2, 1, 1, 32),
    ("grouped_pad0", (2, 64, 12, 12), 64, 3, 1, 0, 1, 16),
    ("grouped_cog8", (2, 32, 8, 30), 64, 3, 1, 1, 1, 8),
    ("c5_odd_channels", (2, 5, 9, 9), 12, 3, 1, 1, 1, 1),
    ("c3_dil2_s2", (2, 3, 17, 19), 16, 3, 2, 2, 2, 1),
    ("c6_5x5_s2", (1, 6, 21, 18), 24, 5, 2, 2, 1, 1),
    ("c3_7x7_s2_even_w", (2, 3, 30, 28), 24, 7, 2, 3, 1, 1),
    ("c4_3x3_s2_p2_even_w", (1, 4, 18, 20), 16, 3, 2, 2, 1, 1),
    # few output tiles, long K: the K loop runs as slices on more SMs, then a
    # reduction pass applies the epilogue
    ("ksplit_3x3_512_7", (2, 512, 7, 7), 512, 3, 1, 1, 1, 1),
    ("ksplit_1x1_2048_7_odd_m", (3, 2048, 5, 7), 512, 1, 1, 0, 1, 1),
    # 4-channel inputs with outputs >= 64 wide: whole input rows per filter row
    ("rows_7x7_s2_b3", (3, 3, 160, 132), 64, 7, 2, 3, 1, 1),
    ("rows_5x5_s1_c4", (2, 4, 70, 80), 24, 5, 1, 2, 1, 1),
    ("rows_3x3_s2_odd", (1, 3, 131, 135), 16, 3, 2, 1, 1, 1),
]


@pytest.mark.parametrize("precision", ["3xtf32", "fp32", "tf32", "bf16"])
@pytest.mark.parametrize("case", SMALL, ids=lambda c: c[0])
def test_conv_small(ob, oracle, ctx, case, precision):
    name, xs, co, k, s, p, d, g = case
    rng = np.random.default_rng(10)
    x = rng.standard_normal(xs).astype(np.float32)
    w = (rng.standard_normal((co, xs[1] // g, k, k)) * np.sqrt(2.0 / (xs[1] // g * k * k))).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, co).astype(np.float32)
    attrs = {"strides": (s, s), "pads": (p, p, p, p), "dilations": (d, d), "group": g}
    y = run_conv(ob, ctx, x, w, b, attrs, precision, relu=True)
    ref = oracle.relu(oracle.conv2d(x, w, b, (s, s), (p, p, p, p), (d, d), g))
    rtol, atol = TOL[precision]
    assert_close(y, ref, rtol, atol, f"{name}/{precision}")


@pytest.mark.parametrize("name", ["conv1d", "conv3d"])
def test_conv_nd_known_answers(ob, ctx, name):
    """The reference's 1-D / 3-D known answers (conv.rs:1487-1529, 1594-1631),
    exact as the reference asserts (small integers are exact in every path)."""
    import json, os
    case = next(c for c in json.load(open(os.path.join(os.path.dirname(__file__), "golden",
                                                         "reference_known_answers.json")))["cases"]
                if c["name"] == name)
    conv = ob.Conv(case["strides"], case["pads"], case["dilations"], case["group"])
    y = np_(conv.compute([cu(case["x"]), cu(case["w"])], ctx)[0])
    assert list(y.shape) == case["expected_shape"]
    np.testing.assert_array_equal(y, np.array(case["expected"], np.float32))


CONV_ND = [
    # name, x shape, co, kernel, strides, pads (begin..., end...), dilations, group, auto_pad
    ("1d_plain", (2, 16, 50), 24, (5,), (1,), (2, 2), (1,), 1, "NOTSET"),
    ("1d_s2_dil2", (3, 8, 61), 16, (3,), (2,), (1, 3), (2,), 1, "NOTSET"),
    ("1d_grouped", (2, 32, 40), 32, (3,), (1,), (1, 1), (1,), 4, "NOTSET"),
    ("1d_same_upper", (1, 12, 33), 20, (4,), (3,), None, (1,), 1, "SAME_UPPER"),
    ("1d_wide_k", (4, 64, 128), 64, (9,), (1,), (4, 4), (1,), 1, "NOTSET"),
    ("3d_plain", (2, 4, 6, 7, 8), 8, (3, 3, 3), (1, 1, 1), (1, 1, 1, 1, 1, 1), (1, 1, 1), 1, "NOTSET"),
    ("3d_strided", (1, 3, 9, 10, 11), 6, (3, 2, 3), (2, 1, 2), (1, 0, 1, 1, 1, 0), (1, 2, 1), 1, "NOTSET"),
    ("3d_grouped", (2, 8, 5, 6, 7), 12, (2, 3, 3), (1, 1, 1), (0, 1, 1, 1, 1, 1), (1, 1, 1), 4, "NOTSET"),
    ("3d_same_lower", (1, 5, 7, 7, 7), 4, (3, 3, 3), (2, 2, 2), None, (1, 1, 1), 1, "SAME_LOWER"),
]


@pytest.mark.parametrize("case", CONV_ND, ids=lambda c: c[0])
def test_conv_nd(ob, oracle, ctx, case):
    """1-D (tensor cores, 3xTF32) and 3-D (CUDA cores, fp32) Conv + bias + Relu
    against the oracle's direct N-d convolution (compute_conv_direct, conv.rs:609-706)."""
    name, xs, co, k, st, pd, dl, g, ap = case
    rng = np.random.default_rng(12)
    x = rng.standard_normal(xs).astype(np.float32)
    ws = (co, xs[1] // g) + tuple(k)
    w = (rng.standard_normal(ws) * np.sqrt(2.0 / np.prod(ws[1:]))).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, co).astype(np.float32)
    conv = ob.Conv(st, pd, dl, g, ap, precision="3xtf32", relu=True)
    y = np_(conv.compute([cu(x), cu(w), cu(b)], ctx)[0])
    sp = len(xs) - 2
    if ap in ("SAME_UPPER", "SAME_LOWER"):
        ps = [oracle.same_pads(xs[2 + i], k[i], st[i], dl[i], ap == "SAME_UPPER") for i in range(sp)]
        pads = [p[0] for p in ps] + [p[1] for p in ps]
    else:
        pads = list(pd)
    ref = oracle.relu(oracle.conv_nd_direct(x, w, b, list(st), pads, list(dl), g))
    assert y.shape == ref.shape
    assert_close(y, ref, 1e-5, 1e-4, name)


def test_conv_stem_config(ob, oracle, ctx, handle):
    """Single Conv+Relu graph (stem 7x7/2, seed 0) through Conv::compute, 3xTF32."""
    nodes, inits, ins, outs = ob.workloads.stem_conv(0)
    x = ob.workloads.stem_input(0)
    y = run_conv(ob, ctx, x, inits["W"], inits["B"], {"strides": (2, 2), "pads": (3, 3, 3, 3)}, "3xtf32", relu=True)
    ref = oracle.relu(oracle.conv2d(x, inits["W"], inits["B"], (2, 2), (3, 3, 3, 3)))
    assert y.shape == (1, 64, 112, 112)
    assert_close(y, ref, 1e-5, 1e-4, "stem")
    # the same through the graph executor (fused Conv+Relu, CUDA graph replay)
    g = ob.Graph(handle, nodes, inits, ins, outs)
    xin = cu(x)
    for _ in range(3):
        out = g.run([xin])[0]
    handle.synchronize()
    assert_close(np_(out), ref, 1e-5, 1e-4, "stem graph")
    st = g.stats()
    assert st["n_fused"] == 1 and st["captured"] == 1
    g.close()


def test_conv_nhwc_layout(ob, oracle, ctx):
    rng = np.random.default_rng(11)
    x = rng.standard_normal((2, 64, 12, 12)).astype(np.float32)
    w = (rng.standard_normal((64, 64, 3, 3)) * 0.06).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, 64).astype(np.float32)
    y = run_conv(ob, ctx, x.transpose(0, 2, 3, 1), w, b, {"pads": (1, 1, 1, 1)}, "3xtf32", layout=1)
    ref = oracle.conv2d(x, w, b, (1, 1), (1, 1, 1, 1))
    assert_close(y.transpose(0, 3, 1, 2), ref, 1e-5, 1e-4, "nhwc")


@pytest.mark.parametrize("precision", ["3xtf32", "fp32"])
def test_conv_fused_bn_residual_relu(ob, oracle, ctx, precision):
    rng = np.random.default_rng(12)
    x = rng.standard_normal((2, 64, 14, 14)).astype(np.float32)
    w = (rng.standard_normal((128, 64, 3, 3)) * 0.06).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, 128).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    beta = rng.uniform(-0.2, 0.2, 128).astype(np.float32)
    mean = rng.normal(0, 0.1, 128).astype(np.float32)
    var = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    res = rng.standard_normal((2, 128, 14, 14)).astype(np.float32)
    y = run_conv(ob, ctx, x, w, b, {"pads": (1, 1, 1, 1)}, precision, relu=True,
                 bn=(gamma, beta, mean, var, 1e-5), residual=res)
    c = oracle.conv2d(x, w, b, (1, 1), (1, 1, 1, 1))
    ref = oracle.relu(oracle.add(oracle.batchnorm(c, gamma, beta, mean, var, 1e-5), res))
    assert_close(y, ref, 1e-5, 1e-4, f"conv+bn+add+relu/{precision}")


def test_conv_tail_split_bn_residual(ob, oracle, ctx):
    """3x3 256->256 at 14x14, 64 images, folded BN + residual + Relu: 196 output tiles
    (1.3 waves), so the first wave runs whole and the last M-tiles run as a K-split
    launch whose reduction pass applies the scale, shift, residual and Relu.  Images
    at both ends (the split rows are the last ones) against the oracle."""
    rng = np.random.default_rng(18)
    x = rng.standard_normal((64, 256, 14, 14)).astype(np.float32)
    w = (rng.standard_normal((256, 256, 3, 3)) * np.sqrt(2.0 / 2304)).astype(np.float32)
    b = rng.uniform(-0.1, 0.1, 256).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, 256).astype(np.float32)
    beta = rng.uniform(-0.2, 0.2, 256).astype(np.float32)
    mean = rng.normal(0, 0.1, 256).astype(np.float32)
    var = rng.uniform(0.5, 1.5, 256).astype(np.float32)
    res = rng.standard_normal((64, 256, 14, 14)).astype(np.float32)
    y = run_conv(ob, ctx, x, w, b, {"pads": (1, 1, 1, 1)}, "3xtf32", relu=True,
                 bn=(gamma, beta, mean, var, 1e-5), residual=res)
    imgs = [0, 1, 37, 52, 60, 61, 62, 63]
    c = oracle.conv2d(np.ascontiguousarray(x[imgs]), w, b, (1, 1), (1, 1, 1, 1))
    ref = oracle.relu(oracle.add(oracle.batchnorm(c, gamma, beta, mean, var, 1e-5), res[imgs]))
    assert_close(y[imgs], ref, 1e-5, 1e-4, f"tail split {imgs}")


SWEEP_NAMES = [s[0] for s in __import__("importlib").import_module("onnx-rs_b200").workloads.SWEEP]


@pytest.mark.parametrize("name", SWEEP_NAMES)
def test_conv_sweep_full_batch(ob, oracle, ctx, name):
    """Conv shape sweep at batch 128 on the GPU; 16 images spread over the batch
    (first, last, both sides of the middle, and every 9th) against the oracle."""
    x, w, b, attrs = ob.workloads.sweep_case(name)
    y = run_conv(ob, ctx, x, w, b, attrs, "3xtf32", relu=True)
    s, p, d, g = attrs["strides"], attrs["pads"], attrs["dilations"], attrs["group"]
    imgs = sorted({0, 63, 64, x.shape[0] - 1} | set(range(5, x.shape[0], 11)))
    ref = oracle.relu(oracle.conv2d(np.ascontiguousarray(x[imgs]), w, b, s, p, d, g))
    assert_close(y[imgs], ref, 1e-5, 1e-4, f"{name}{imgs}")


@pytest.mark.parametrize("case", ["simple_matmul", "vector_vector", "vector_matrix", "matrix_vector",
                                  "batch_no_broadcast", "batch_with_broadcast", "complex_batch_broadcasting",
                                  "singleton_dimension_broadcasting"])
@pytest.mark.parametrize("precision", ["3xtf32", "fp32"])
def test_matmul_reference_cases(ob, oracle, ctx, case, precision):
    import json, os
    cases = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_known_answers.json")))["cases"]
    c = next(c for c in cases if c["name"] == case)
    a = np.arange(int(np.prod(c["a_shape"])), dtype=np.float32).reshape(c["a_shape"])
    b = np.arange(int(np.prod(c["b_shape"])), dtype=np.float32).reshape(c["b_shape"])
    y = ob.MatMul(precision=precision).compute([cu(a), cu(b)], ctx)[0]
    exp = np.array(c["expected"], np.float32).reshape(c["expected_shape"])
    # small integers: exact in fp32, and exact in 3xTF32 (hi parts carry them exactly)
    np.testing.assert_array_equal(np_(y), exp)
    np.testing.assert_array_equal(exp, oracle.matmul(a, b))


@pytest.mark.parametrize("sa,sb", [((4, 64, 96), (96, 128)), ((2, 1, 72, 40), (3, 40, 36)),
                                   ((130, 260), (260, 68)), ((5, 200, 32), (5, 32, 260))])
@pytest.mark.parametrize("precision", ["3xtf32", "tf32", "bf16", "fp32"])
def test_matmul_random(ob, oracle, ctx, sa, sb, precision):
    rng = np.random.default_rng(13)
    a = rng.standard_normal(sa).astype(np.float32)
    b = (rng.standard_normal(sb) / np.sqrt(sb[-2])).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, sb[-1]).astype(np.float32)
    y = ob.MatMul(precision=precision).compute([cu(a), cu(b)], ctx, bias=cu(bias), relu=True)[0]
    ref = oracle.relu(oracle.add(oracle.matmul(a, b), bias))
    rtol, atol = TOL[precision]
    assert_close(np_(y), ref, rtol, atol, f"matmul {sa}x{sb}/{precision}")


def test_matmul_broadcast_config(ob, oracle, ctx, handle):
    """A[8,1,512,768] x B[12,768,3072] + bias, Relu (seed 1): full size on the GPU.
    Output batches (0,0), (3,7) and (7,11) against the oracle; every element of
    all 96 output matrices against a float64 product at the 3xTF32 per-op bar;
    and a checksum of checksums (float64 row sums of every matrix, summed)."""
    a, b, bias = ob.workloads.broadcast_matmul(1)
    nodes, inits, ins, outs = ob.workloads.broadcast_matmul_graph(1)
    y = ob.MatMul().compute([cu(a), cu(b)], ctx, bias=cu(bias), relu=True)[0]
    handle.synchronize()
    yh = np_(y)
    assert yh.shape == (8, 12, 512, 3072)
    for i, j in ((0, 0), (3, 7), (7, 11)):
        ref = oracle.relu(oracle.add(oracle.matmul(a[i, 0], b[j]), bias))
        assert_close(yh[i, j], ref, 1e-5, 1e-4, f"batch ({i},{j})")
    b64 = b.astype(np.float64)
    bias64 = bias.astype(np.float64)
    sums_gpu = np.zeros((8, 12, 512))
    sums_ref = np.zeros((8, 12, 512))
    for i in range(8):
        a64 = a[i, 0].astype(np.float64)
        for j in range(12):
            r = np.maximum(a64 @ b64[j] + bias64, 0.0)
            assert_close(yh[i, j], r, 1e-5, 1e-4, f"batch ({i},{j}) vs float64")
            sums_gpu[i, j] = yh[i, j].astype(np.float64).sum(axis=1)
            sums_ref[i, j] = r.sum(axis=1)
    assert_close(sums_gpu, sums_ref, 1e-5, 1e-4, "row sums")
    # the grand total of 151M non-negative outputs: within the per-op relative
    # bar (the tensor core's truncating accumulation leaves a systematic bias of
    # about -1e-6 relative, which a sum of positive values shows undiluted)
    total_gpu, total_ref = float(sums_gpu.sum()), float(sums_ref.sum())
    assert abs(total_gpu - total_ref) <= 1e-5 * abs(total_ref), (total_gpu, total_ref)
    # graph path (fused MatMul+Add+Relu)
    g = ob.Graph(handle, nodes, inits, ins, outs)
    yg = g.run([cu(a)])[0]
    handle.synchronize()
    assert g.stats()["n_fused"] == 2
    np.testing.assert_array_equal(np_(yg), yh)
    g.close()


@pytest.mark.parametrize("ta,tb,cshape,alpha,beta", [(0, 1, (1000,), 1.0, 1.0), (0, 0, (8, 1000), 0.5, 2.0),
                                                      (1, 1, (), 1.0, 1.0), (1, 0, None, 2.0, 0.0),
                                                      (0, 1, (8, 1), 1.0, -1.0)])
def test_gemm_attributes(ob, oracle, ctx, ta, tb, cshape, alpha, beta):
    rng = np.random.default_rng(14)
    m, n, k = 8, 1000, 512
    a = rng.standard_normal((k, m) if ta else (m, k)).astype(np.float32)
    b = (rng.standard_normal((n, k) if tb else (k, n)) / np.sqrt(k)).astype(np.float32)
    c = None if cshape is None else rng.standard_normal(cshape).astype(np.float32)
    ins = [cu(a), cu(b)] + ([cu(c)] if c is not None else [])
    y = ob.Gemm(alpha, beta, ta, tb).compute(ins, ctx)[0]
    ref = oracle.gemm(a, b, c, alpha, beta, ta, tb)
    assert_close(np_(y), ref, 1e-5, 1e-4, "gemm")


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(37, 129, 61), (130, 260, 264), (8, 1000, 512)])
def test_gemm_fp32_cuda_cores(ob, oracle, ctx, ta, tb, m, n, k):
    """fp32 precision (CUDA-core FFMA GEMM): every transpose combination over odd
    sizes (scalar operand loads and stores at the tile edges), multiples of 4 (16-byte
    vector loads) and the classifier shape, with alpha, beta and a full C."""
    rng = np.random.default_rng(21)
    a = rng.standard_normal((k, m) if ta else (m, k)).astype(np.float32)
    b = (rng.standard_normal((n, k) if tb else (k, n)) / np.sqrt(k)).astype(np.float32)
    c = rng.standard_normal((m, n)).astype(np.float32)
    y = ob.Gemm(0.5, 2.0, ta, tb, precision="fp32").compute([cu(a), cu(b), cu(c)], ctx)[0]
    ref = oracle.gemm(a, b, c, 0.5, 2.0, ta, tb)
    assert_close(np_(y), ref, 1e-5, 1e-4, f"gemm fp32 {m}x{n}x{k} ta={ta} tb={tb}")


def test_maxpool_and_indices(ob, oracle, ctx):
    rng = np.random.default_rng(15)
    x = rng.standard_normal((4, 64, 112, 112)).astype(np.float32)
    y, ind = ob.MaxPool((3, 3), (2, 2), (1, 1, 1, 1)).compute([cu(x)], ctx, with_indices=True)
    ref, rind = oracle.maxpool2d(x, (3, 3), (2, 2), (1, 1, 1, 1), with_indices=True)
    np.testing.assert_array_equal(np_(y), ref)
    np.testing.assert_array_equal(np_(ind), rind)
    y2 = ob.MaxPool((3, 3), (2, 2), (1, 1, 1, 1)).compute([cu(x)], ctx)[0]
    np.testing.assert_array_equal(np_(y2), ref)
    # odd shapes / ceil mode / NaN handling
    x = rng.standard_normal((2, 3, 9, 8)).astype(np.float32)
    x[0, 1, 2, 2] = np.nan
    y, ind = ob.MaxPool((2, 3), (2, 2), (0, 1, 1, 0), ceil_mode=1).compute([cu(x)], ctx, with_indices=True)
    ref, rind = oracle.maxpool2d(x, (2, 3), (2, 2), (0, 1, 1, 0), ceil_mode=1, with_indices=True)
    np.testing.assert_array_equal(np_(y), ref)
    np.testing.assert_array_equal(np_(ind), rind)
    # 3x3 stride 2 without indices (row-segment kernel): output rows that end
    # mid-segment, asymmetric pads, ceil mode, NaN and -inf inputs
    x = rng.standard_normal((3, 12, 15, 37)).astype(np.float32)
    x[1, 4, 3, 5] = np.nan
    x[2, 7, :, 9] = -np.inf
    for pads, ceil in (((1, 0, 0, 1), 1), ((0, 1, 1, 1), 0), ((1, 1, 1, 1), 0)):
        y = ob.MaxPool((3, 3), (2, 2), pads, ceil_mode=ceil).compute([cu(x)], ctx)[0]
        ref = oracle.maxpool2d(x, (3, 3), (2, 2), pads, ceil_mode=ceil)
        np.testing.assert_array_equal(np_(y), ref)


def test_gap_relu_add_bn(ob, oracle, ctx):
    rng = np.random.default_rng(16)
    x = rng.standard_normal((8, 2048, 7, 7)).astype(np.float32)
    np.testing.assert_array_equal(np_(ob.GlobalAveragePool().compute([cu(x)], ctx)[0]), oracle.global_avgpool(x))
    x3 = rng.standard_normal((3, 6, 5, 5)).astype(np.float32)
    np.testing.assert_array_equal(np_(ob.GlobalAveragePool().compute([cu(x3)], ctx)[0]), oracle.global_avgpool(x3))
    r = rng.standard_normal(100003).astype(np.float32)
    r[5] = np.nan
    np.testing.assert_array_equal(np_(ob.Relu().compute([cu(r)], ctx)[0]), oracle.relu(r))
    # 4-byte-offset view (one element per thread) and fewer elements than a vector
    np.testing.assert_array_equal(np_(ob.Relu().compute([cu(r)[1:]], ctx)[0]), oracle.relu(r[1:]))
    np.testing.assert_array_equal(np_(ob.Relu().compute([cu(r[:3])], ctx)[0]), oracle.relu(r[:3]))
    for sa, sb in [((2, 64, 7, 7), (2, 64, 7, 7)), ((8, 12, 16, 32), (32,)), ((2, 1, 5), (3, 1)), ((7,), ())]:
        a = rng.standard_normal(sa).astype(np.float32)
        b = rng.standard_normal(sb).astype(np.float32)
        np.testing.assert_array_equal(np_(ob.Add().compute([cu(a), cu(b)], ctx)[0]), oracle.add(a, b))
    p = [rng.uniform(0.5, 1.5, 6).astype(np.float32) for _ in range(4)]
    y = ob.BatchNormalization(1e-5).compute([cu(x3)] + [cu(v) for v in p], ctx)[0]
    assert_close(np_(y), oracle.batchnorm(x3, *p, 1e-5), 1e-5, 1e-5, "bn")


def test_empty_and_invalid(ob, ctx):
    x = torch.zeros((0, 8, 5, 5), device="cuda")
    w = torch.zeros((8, 8, 3, 3), device="cuda")
    y = ob.Conv(pads=(1, 1, 1, 1)).compute([x, w], ctx)[0]
    assert tuple(y.shape) == (0, 8, 5, 5)
    with pytest.raises(ob.ValidationError):
        ob.Conv(group=3).compute([torch.zeros((1, 8, 5, 5), device="cuda"),
                                  torch.zeros((4, 2, 3, 3), device="cuda")], ctx)
    with pytest.raises(ob.ValidationError):
        ob.MatMul().compute([torch.zeros((2, 3), device="cuda"), torch.zeros((4, 5), device="cuda")], ctx)
    with pytest.raises(ob.ValidationError):
        ob.Add().compute([torch.zeros((2, 3), device="cuda"), torch.zeros((3, 2), device="cuda")], ctx)


@pytest.mark.gpu
@pytest.mark.parametrize("shape,cpad", [((2, 3, 224, 224), 4), ((3, 1, 8, 12), 4), ((2, 2, 5, 7), 4),
                                        ((2, 3, 6, 6), 8), ((1, 5, 4, 4), 8), ((2, 40, 9, 7), 40)])
def test_nchw_to_nhwc_repack(ob, handle, shape, cpad):
    """Layout repack at the graph edge: NCHW -> channel-padded NHWC, bit-exact with
    zero padding channels (four-pixel vectors when HW % 4 == 0, other paths otherwise)."""
    import ctypes
    C = __import__("importlib").import_module("onnx-rs_b200._capi")
    rng = np.random.default_rng(17)
    x = rng.standard_normal(shape).astype(np.float32)
    n, c, hh, ww = shape
    xd = cu(x)
    y = torch.full((n, hh, ww, cpad), 7.0, dtype=torch.float32, device="cuda")
    handle.check(C.lib().onnxb200_nchw_to_nhwc(handle.ptr, n, c, hh, ww, cpad, ctypes.c_void_p(xd.data_ptr()),
                                               ctypes.c_void_p(y.data_ptr())), "repack")
    ref = np.zeros((n, hh, ww, cpad), np.float32)
    ref[..., :c] = x.transpose(0, 2, 3, 1)
    np.testing.assert_array_equal(np_(y), ref)
