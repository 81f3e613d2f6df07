"""CPU tests of the C ABI boundary (no GPU compute): libq35k.so builds for
sm_100a, loads, and exports exactly what include/q35k.h declares."""

import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "q35k.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(q35k_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib_path():
    import importlib.util

    spec = importlib.util.spec_from_file_location("q35k_build", os.path.join(ROOT, "qwen3.5sharp_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build()


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("q35k_create", "q35k_destroy", "q35k_weight_upload", "q35k_matmul", "q35k_matmul_q8k",
                     "q35k_matmul_dev", "q35k_quantize_q8k", "q35k_dequantize", "q35k_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol(lib_path):
    L = ctypes.CDLL(lib_path)
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (q35k_\w+)", out))
    assert exported == set(declared_functions()), exported ^ set(declared_functions())


def test_python_binding_covers_the_header(lib_path):
    from q35k import _lib

    assert sorted(_lib.exported_symbols()) == declared_functions()


def test_library_is_sm100a_only(lib_path):
    out = subprocess.run(["cuobjdump", "--list-elf", lib_path], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    arches = set(re.findall(r"sm_(\d+a?)", out.stdout))
    assert arches == {"100a"}, arches


def test_no_cpu_fallback_without_gpu(lib_path):
    """Without a visible GPU, context creation fails loudly (no silent CPU path)."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    import q35k

    with pytest.raises(q35k.Q35KError):
        q35k.Context(0)


def test_mirror_argument_errors_without_gpu():
    """Argument checks that the reference performs before any compute."""
    import numpy as np

    import q35k

    with pytest.raises(q35k.NotSupportedException):
        q35k.MulMatQ4K.Gemv(np.zeros(10, np.uint8), np.zeros(100, np.float32), None, 100, 1)
    with pytest.raises(q35k.ArgumentException):
        q35k.Q8K.QuantizeRow(np.zeros(100, np.float32), None, 100)


def test_csharp_binding_covers_the_header():
    """bindings/Q35k.cs (the P/Invoke shim for src/Qwen35Sharp.Kernels/)
    declares every entry point of the header, with the header's argument
    count."""
    cs = open(os.path.join(ROOT, "bindings", "Q35k.cs")).read()
    bound = dict(re.findall(r"static partial \S+ (q35k_\w+)\(([^)]*)\)", cs))
    assert sorted(bound) == declared_functions()
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    for name, args in re.findall(r"\b(q35k_\w+)\s*\(([^)]*)\)", src):
        n_c = 0 if args.strip() in ("", "void") else args.count(",") + 1
        n_cs = 0 if not bound[name].strip() else bound[name].count(",") + 1
        assert n_c == n_cs, (name, n_c, n_cs)
