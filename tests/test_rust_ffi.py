"""The Rust FFI crate (onnx-b200-sys) against the C header, on the CPU: there is
no Rust toolchain in this image, so the crate is checked as text.
src/ffi.rs must be exactly what gen_ffi.py generates from include/onnxb200.h,
declare every exported function, and carry the same struct fields as the
ctypes binding that the GPU tests call through."""
import os
import re
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CRATE = os.path.join(ROOT, "onnx-b200-sys")


def test_ffi_generated_from_header():
    r = subprocess.run([sys.executable, os.path.join(CRATE, "gen_ffi.py"), "--check"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def test_ffi_declares_every_export(ob):
    src = open(os.path.join(CRATE, "src", "ffi.rs")).read()
    block = src[src.index('extern "C" {'):]
    rust_fns = sorted(re.findall(r"pub fn (onnxb200_\w+)\(", block))
    out = subprocess.run(["nm", "-D", "--defined-only", ob.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted(l.split()[-1] for l in out.splitlines() if " T " in l)
    assert rust_fns == exported
    # parameter counts agree with the ctypes signatures
    for name, params in re.findall(r"pub fn (onnxb200_\w+)\((.*?)\)", block):
        n = 0 if not params.strip() else params.count(":")
        assert n == len(ob._capi.SIGNATURES[name][1]), name


def test_ffi_structs_match_ctypes(ob):
    src = open(os.path.join(CRATE, "src", "ffi.rs")).read()
    C = ob._capi
    pairs = {"Options": C.Options, "ConvDesc": C.ConvDesc, "ConvNdDesc": C.ConvNdDesc, "Attr": C.Attr,
             "Node": C.Node, "TensorInfo": C.TensorInfo, "GraphStats": C.GraphStats, "StepProfile": C.StepProfile,
             "ModelInfo": C.ModelInfo, "ShapeInfo": C.ShapeInfo}
    for rust, cty in pairs.items():
        body = re.search(r"pub struct %s \{(.*?)\}" % rust, src, re.S).group(1)
        fields = re.findall(r"pub (\w+):", body)
        names = [f.rstrip("_") for f in fields]
        assert names == [f[0].rstrip("_") for f in cty._fields_], rust


def test_operator_module_covers_the_path():
    src = open(os.path.join(CRATE, "ops", "b200.rs")).read()
    for op in ("Conv", "MatMul", "Gemm", "MaxPool", "GlobalAveragePool", "Relu", "Add", "BatchNormalization"):
        assert f"impl Operator for B200{op}" in src, op
        assert f'register_operator("{op}"' in src, op
    for fn in ("fn compute(", "fn output_shapes(", "fn validate("):
        assert src.count(fn) == 8, fn
