"""ctypes front end of the CPU oracle (oracle/libkquant_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, as the checker and as the timed CPU reference.
The product (libq35k) never loads it.

PARITY UNPINNED: the reference is C#/.NET and cannot run here, and it ships no
golden vectors for Q4_K/Q5_K/Q6_K; see kquant_oracle.h for what the oracle is
checked against instead.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkquant_oracle.so")

Q4_K, Q5_K, Q6_K = 12, 13, 14
QK = 256
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}
Q8K_BYTES = 292

_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc); returns the .so path."""
    if force or not os.path.exists(LIB_PATH) or _stale():
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def _stale() -> bool:
    so = os.path.getmtime(LIB_PATH)
    for f in ("kquant_scalar.c", "kquant_avx2.c", "kquant_oracle.h"):
        if os.path.getmtime(os.path.join(HERE, f)) > so:
            return True
    return False


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i32, f32p = ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float)
        L.oq_fp16_to_f32.argtypes = [ctypes.c_uint16]
        L.oq_fp16_to_f32.restype = ctypes.c_float
        L.oq_quantize_q8k_scalar.argtypes = [vp, vp, i32]
        L.oq_quantize_q8k_avx2.argtypes = [vp, vp, i32]
        L.oq_dequantize.argtypes = [i32, vp, vp, i32]
        L.oq_dequantize.restype = i32
        L.oq_dot_scalar.argtypes = [i32, vp, vp, i32]
        L.oq_dot_scalar.restype = ctypes.c_float
        L.oq_dot_avx2.argtypes = [i32, vp, vp, i32]
        L.oq_dot_avx2.restype = ctypes.c_float
        L.oq_quantize_q8kx4.argtypes = [vp, vp, i32]
        L.oq_gemm_q4k_semantic.argtypes = [vp, vp, vp, i32, i32, i32, i32]
        L.oq_weight_prepare.argtypes = [i32, vp, i32, i32]
        L.oq_weight_prepare.restype = vp
        L.oq_weight_release.argtypes = [vp]
        L.oq_matmul.argtypes = [vp, vp, vp, i32, i32]
        L.oq_matmul.restype = i32
        L.oq_matmul_q8k.argtypes = [vp, vp, vp, i32, i32]
        L.oq_matmul_q8k.restype = i32
        L.oq_matmul_semantic.argtypes = [vp, vp, vp, i32]
        L.oq_matmul_semantic.restype = i32
        del f32p
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def quantize_q8k(x: np.ndarray, avx2: bool = True) -> np.ndarray:
    """Q8K.QuantizeRow for each row of x [m, k] -> uint8 [m, nb*292]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    m, k = x.shape
    out = np.zeros((m, (k // QK) * Q8K_BYTES), dtype=np.uint8)
    fn = lib().oq_quantize_q8k_avx2 if avx2 else lib().oq_quantize_q8k_scalar
    for r in range(m):
        fn(_ptr(x[r]), _ptr(out[r]), k)
    return out


def dequantize(qtype: int, blocks: np.ndarray, k: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    rows = blocks.size // ((k // QK) * BLOCK_BYTES[qtype])
    out = np.zeros((rows, k), dtype=np.float32)
    flat = blocks.reshape(rows, -1)
    for r in range(rows):
        if lib().oq_dequantize(qtype, _ptr(flat[r]), _ptr(out[r]), k) != 0:
            raise ValueError("dequantize failed")
    return out


def dot(qtype: int, w_row: np.ndarray, q8_row: np.ndarray, k: int, avx2: bool = True) -> float:
    fn = lib().oq_dot_avx2 if avx2 else lib().oq_dot_scalar
    return float(fn(qtype, _ptr(np.ascontiguousarray(w_row)), _ptr(np.ascontiguousarray(q8_row)), k))


def quantize_q8kx4(x4: np.ndarray) -> np.ndarray:
    x4 = np.ascontiguousarray(x4, dtype=np.float32)
    k = x4.shape[1]
    out = np.zeros((k // QK) * 1168, dtype=np.uint8)
    lib().oq_quantize_q8kx4(_ptr(x4), _ptr(out), k)
    return out


class Weight:
    """oq_weight_prepare: raw blocks + the load-time Q4_K panel/meta."""

    def __init__(self, qtype: int, blocks: np.ndarray, n_in: int, n_out: int):
        self.blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        self.qtype, self.n_in, self.n_out = qtype, n_in, n_out
        self.h = lib().oq_weight_prepare(qtype, _ptr(self.blocks), n_in, n_out)
        if not self.h:
            raise ValueError("oq_weight_prepare rejected the weight")

    def __del__(self):
        h = getattr(self, "h", None)
        if h and _lib is not None:
            _lib.oq_weight_release(h)
            self.h = None

    def matmul(self, x: np.ndarray, threads: int = 1) -> np.ndarray:
        """The reference's Linear dispatch (AVX2 executed order, threaded)."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.n_in)
        y = np.zeros((x.shape[0], self.n_out), dtype=np.float32)
        if lib().oq_matmul(self.h, _ptr(x), _ptr(y), x.shape[0], threads) != 0:
            raise RuntimeError("oq_matmul failed")
        return y

    def matmul_q8k(self, q8: np.ndarray, tokens: int, threads: int = 1) -> np.ndarray:
        q8 = np.ascontiguousarray(q8, dtype=np.uint8)
        y = np.zeros((tokens, self.n_out), dtype=np.float32)
        if lib().oq_matmul_q8k(self.h, _ptr(q8), _ptr(y), tokens, threads) != 0:
            raise RuntimeError("oq_matmul_q8k failed")
        return y

    def matmul_semantic(self, x: np.ndarray) -> np.ndarray:
        """Scalar semantics of the same dispatch (single thread)."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.n_in)
        y = np.zeros((x.shape[0], self.n_out), dtype=np.float32)
        if lib().oq_matmul_semantic(self.h, _ptr(x), _ptr(y), x.shape[0]) != 0:
            raise RuntimeError("oq_matmul_semantic failed")
        return y


def gemm_q4k_semantic(blocks: np.ndarray, q8: np.ndarray, rows: int, cols: int, n_in: int) -> np.ndarray:
    out = np.zeros((rows, cols), dtype=np.float32)
    lib().oq_gemm_q4k_semantic(_ptr(np.ascontiguousarray(blocks)), _ptr(np.ascontiguousarray(q8)), _ptr(out),
                               cols, n_in, rows, cols)
    return out


# ---- CpuTopology.ChooseWorkerCount (src/Qwen35Sharp.Kernels/CpuTopology.cs:107-123) ----

def choose_worker_count(logical: int, physical: int, p_cores: int, saw_smt: bool, vm: bool) -> int:
    if logical <= 0:
        logical = 1
    if physical <= 0:
        if vm and logical >= 2 and logical % 2 == 0:
            return logical // 2
        return logical if logical <= 4 else logical // 2
    preferred = p_cores if p_cores > 0 else physical
    if vm and not saw_smt and physical == logical and logical >= 2 and logical % 2 == 0:
        preferred = min(preferred, logical // 2)
    return max(1, min(preferred, logical))


def host_topology() -> dict:
    """Linux topology as CpuTopology reads it: logical CPUs usable by this
    process, physical cores from thread_siblings_list (CpuTopology.cs:419),
    SMT seen, hypervisor flag (CpuTopology.cs:469-476)."""
    cpus = sorted(os.sched_getaffinity(0))
    cores = set()
    saw_smt = False
    for c in cpus:
        p = f"/sys/devices/system/cpu/cpu{c}/topology/thread_siblings_list"
        try:
            s = open(p).read().strip()
        except OSError:
            s = str(c)
        cores.add(s)
        if "," in s or "-" in s:
            saw_smt = True
    vm = os.path.exists("/sys/hypervisor/type")
    try:
        vm = vm or ("hypervisor" in open("/proc/cpuinfo").read())
    except OSError:
        pass
    logical = len(cpus)
    physical = len(cores)
    return dict(logical=logical, physical=physical, saw_smt=saw_smt, vm=vm,
                reference_workers=choose_worker_count(logical, physical, 0, saw_smt, vm))
