"""Writes reference_known_answers.json: the known-answer cases of the onnx-rs
reference's own unit tests for the Conv / MatMul / broadcast path.

The reference is Rust and cannot be built in this image, so its test inputs
and expected outputs are restated here case by case, each citing the test it
comes from.  Every expected value is recomputed with numpy in float64 and the
script fails if a case the reference states correctly disagrees.  Tests whose
stated expectation is arithmetically wrong keep the reference's inputs, record
the correct numpy value, and carry ``"reference_expectation_wrong": true`` with
the reference's (wrong) numbers for the record.

Run: python tests/golden/make_golden.py   (rewrites the JSON beside it)
"""
import json
import os

import numpy as np


def seq(shape):
    """create_test_tensor (src/ops/math/matmul.rs:712-723): 0, 1, 2, ... in row-major order."""
    return np.arange(int(np.prod(shape)), dtype=np.float64).reshape(shape)


def conv_nd(x, w, strides, pads, dil, group):
    """float64 direct convolution, same loops as compute_conv_direct."""
    sd = x.ndim - 2
    n, c = x.shape[:2]
    co = w.shape[0]
    cg, cog = c // group, co // group
    outs = [(x.shape[i + 2] + pads[i] + pads[i + sd] - ((w.shape[i + 2] - 1) * dil[i] + 1)) // strides[i] + 1
            for i in range(sd)]
    y = np.zeros([n, co] + outs)
    for b in range(n):
        for oc in range(co):
            g = oc // cog
            for o in np.ndindex(*outs):
                s = 0.0
                for icg in range(cg):
                    for k in np.ndindex(*w.shape[2:]):
                        idx = [o[i] * strides[i] - pads[i] + k[i] * dil[i] for i in range(sd)]
                        if all(0 <= idx[i] < x.shape[i + 2] for i in range(sd)):
                            s += x[(b, g * cg + icg) + tuple(idx)] * w[(oc, icg) + k]
                y[(b, oc) + o] = s
    return y


def main():
    cases = []

    # conv.rs:1487-1529 test_conv1d
    x = np.array([1, 2, 3, 4, 5], np.float64).reshape(1, 1, 5)
    w = np.array([1, 2, 1], np.float64).reshape(1, 1, 3)
    y = conv_nd(x, w, [1], [0, 0], [1], 1)
    assert y.ravel().tolist() == [8.0, 12.0, 16.0]
    cases.append(dict(name="conv1d", op="Conv", source="src/ops/nn/conv.rs:1487-1529",
                      x=x.tolist(), w=w.tolist(), strides=[1], pads=[0, 0], dilations=[1], group=1,
                      expected=y.tolist(), expected_shape=list(y.shape)))

    # conv.rs:1533-1590 test_conv2d
    x = np.arange(1, 10, dtype=np.float64).reshape(1, 1, 3, 3)
    w = np.array([1, 2, 3, 4], np.float64).reshape(1, 1, 2, 2)
    y = conv_nd(x, w, [1, 1], [0, 0, 0, 0], [1, 1], 1)
    assert y.ravel().tolist() == [37.0, 47.0, 67.0, 77.0]
    cases.append(dict(name="conv2d", op="Conv", source="src/ops/nn/conv.rs:1533-1590",
                      x=x.tolist(), w=w.tolist(), strides=[1, 1], pads=[0, 0, 0, 0], dilations=[1, 1],
                      group=1, expected=y.tolist(), expected_shape=list(y.shape)))

    # conv.rs:1594-1631 test_conv3d
    x = np.arange(1, 9, dtype=np.float64).reshape(1, 1, 2, 2, 2)
    w = np.arange(1, 9, dtype=np.float64).reshape(1, 1, 2, 2, 2)
    y = conv_nd(x, w, [1, 1, 1], [0] * 6, [1, 1, 1], 1)
    assert y.ravel().tolist() == [204.0]
    cases.append(dict(name="conv3d", op="Conv", source="src/ops/nn/conv.rs:1594-1631",
                      x=x.tolist(), w=w.tolist(), strides=[1, 1, 1], pads=[0] * 6, dilations=[1, 1, 1],
                      group=1, expected=y.tolist(), expected_shape=list(y.shape)))

    # conv.rs:1635-1692 test_grouped_conv (reference asserts Direct == Im2Col)
    x = np.arange(1, 37, dtype=np.float64).reshape(1, 4, 3, 3)
    w = np.array([1, 2, 3, 4, 5, 6, 7, 8] * 2, np.float64).reshape(2, 2, 2, 2)
    y = conv_nd(x, w, [1, 1], [0, 0, 0, 0], [1, 1], 2)
    cases.append(dict(name="grouped_conv", op="Conv", source="src/ops/nn/conv.rs:1635-1692",
                      x=x.tolist(), w=w.tolist(), strides=[1, 1], pads=[0, 0, 0, 0], dilations=[1, 1],
                      group=2, expected=y.tolist(), expected_shape=list(y.shape),
                      note="reference checks Direct and Im2Col agree exactly"))

    # conv.rs:1696-1768 test_padding_modes: SAME_UPPER shape 3x3, VALID sum 45
    x = np.arange(1, 10, dtype=np.float64).reshape(1, 1, 3, 3)
    w = np.ones((1, 1, 3, 3))
    y_same = conv_nd(x, w, [1, 1], [1, 1, 1, 1], [1, 1], 1)
    y_valid = conv_nd(x, w, [1, 1], [0, 0, 0, 0], [1, 1], 1)
    assert y_valid.ravel().tolist() == [45.0]
    cases.append(dict(name="padding_same_upper", op="Conv", source="src/ops/nn/conv.rs:1696-1740",
                      x=x.tolist(), w=w.tolist(), strides=[1, 1], auto_pad="SAME_UPPER", dilations=[1, 1],
                      group=1, expected=y_same.tolist(), expected_shape=[1, 1, 3, 3]))
    cases.append(dict(name="padding_valid", op="Conv", source="src/ops/nn/conv.rs:1742-1768",
                      x=x.tolist(), w=w.tolist(), strides=[1, 1], auto_pad="VALID", dilations=[1, 1],
                      group=1, expected=y_valid.tolist(), expected_shape=[1, 1, 1, 1]))

    # conv.rs:1772-1816 test_stride_dilation: stride-2 shape [1,1,2,2] (correct);
    # dilation-2 shape stated [1,1,2,2] but is [1,1,3,3].
    x = np.arange(1, 26, dtype=np.float64).reshape(1, 1, 5, 5)
    w = np.array([1, 2, 3, 4], np.float64).reshape(1, 1, 2, 2)
    y = conv_nd(x, w, [2, 2], [0, 0, 0, 0], [1, 1], 1)
    assert list(y.shape) == [1, 1, 2, 2]
    cases.append(dict(name="stride2", op="Conv", source="src/ops/nn/conv.rs:1791-1807",
                      x=x.tolist(), w=w.tolist(), strides=[2, 2], pads=[0, 0, 0, 0], dilations=[1, 1],
                      group=1, expected=y.tolist(), expected_shape=[1, 1, 2, 2]))
    y = conv_nd(x, w, [1, 1], [0, 0, 0, 0], [2, 2], 1)
    cases.append(dict(name="dilation2", op="Conv", source="src/ops/nn/conv.rs:1809-1815",
                      x=x.tolist(), w=w.tolist(), strides=[1, 1], pads=[0, 0, 0, 0], dilations=[2, 2],
                      group=1, expected=y.tolist(), expected_shape=list(y.shape),
                      reference_expectation_wrong=True, reference_stated_shape=[1, 1, 2, 2]))

    # MatMul cases (src/ops/math/matmul.rs:726-888), inputs = create_test_tensor
    mm = [
        ("simple_matmul", [2, 3], [3, 2], "src/ops/math/matmul.rs:726-744", [5.0, 14.0, 14.0, 50.0]),
        ("vector_vector", [3], [3], "src/ops/math/matmul.rs:747-757", None),
        ("vector_matrix", [2], [2, 3], "src/ops/math/matmul.rs:760-776", [1.0, 3.0, 5.0]),
        ("matrix_vector", [2, 3], [3], "src/ops/math/matmul.rs:779-795", None),
        ("batch_no_broadcast", [2, 2, 3], [2, 3, 2], "src/ops/math/matmul.rs:798-821", [5.0, 14.0, 149.0, 446.0]),
        ("batch_with_broadcast", [2, 3], [2, 3, 2], "src/ops/math/matmul.rs:824-848",
         [5.0, 14.0, 14.0, 50.0, 41.0, 50.0, 122.0, 158.0]),
        ("complex_batch_broadcasting", [2, 1, 2, 3], [3, 3, 2], "src/ops/math/matmul.rs:851-871",
         [5.0, 41.0, 5.0, 446.0]),
        ("singleton_dimension_broadcasting", [2, 1, 2, 3], [1, 3, 2], "src/ops/math/matmul.rs:874-888",
         [5.0, 50.0]),
    ]
    for name, sa, sb, src, wrong in mm:
        a, b = seq(sa), seq(sb)
        y = np.matmul(a, b)
        case = dict(name=name, op="MatMul", source=src, a_shape=sa, b_shape=sb, inputs="create_test_tensor",
                    expected=np.asarray(y).tolist(), expected_shape=list(np.shape(y)))
        if wrong is not None:
            case["reference_expectation_wrong"] = True
            case["reference_stated_values"] = wrong
        cases.append(case)
    # correct reference expectations are checked here
    assert float(np.matmul(seq([3]), seq([3]))) == 5.0
    assert np.matmul(seq([2, 3]), seq([3])).tolist() == [5.0, 14.0]

    # validate_matmul_shapes (matmul.rs:891-946)
    valid = [([2, 3], [3, 4], [2, 4]), ([3], [3], []), ([3], [3, 2], [2]), ([2, 3], [3], [2]),
             ([2, 3, 4], [2, 4, 5], [2, 3, 5]), ([2, 1, 3, 4], [2, 5, 4, 5], [2, 5, 3, 5]),
             ([3, 4], [2, 4, 5], [2, 3, 5]), ([3, 4], [4, 5], [3, 5])]
    invalid = [([2, 3], [4, 5]), ([2], [3]), ([2], [3, 4]), ([2, 3, 4], [3, 4, 5]),
               # test_broadcast_performance (matmul.rs:949-966) expects success; 5 vs 10 cannot broadcast
               ([5, 10, 20], [10, 20, 30])]
    for sa, sb, so in valid:
        assert list(np.matmul(np.zeros(sa), np.zeros(sb)).shape) == so
    cases.append(dict(name="validate_matmul_shapes", op="MatMulShape", source="src/ops/math/matmul.rs:891-946",
                      valid=[dict(a=a, b=b, out=o) for a, b, o in valid],
                      invalid=[dict(a=a, b=b) for a, b in invalid]))

    # broadcast_to [1,3] -> [2,3] (tensor.rs:1991-2013), exercised through Add with zeros
    cases.append(dict(name="broadcast_1x3_to_2x3", op="Add", source="src/ops/tensor.rs:1991-2013",
                      a=[[1.0, 2.0, 3.0]], b=[[0.0, 0.0, 0.0], [0.0, 0.0, 0.0]],
                      expected=[[1.0, 2.0, 3.0], [1.0, 2.0, 3.0]], expected_shape=[2, 3]))

    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_known_answers.json")
    with open(out, "w") as f:
        json.dump(dict(generator="tests/golden/make_golden.py", cases=cases), f, indent=1)
    print(f"wrote {len(cases)} cases to {out}")


if __name__ == "__main__":
    main()
