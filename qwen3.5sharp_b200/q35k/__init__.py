"""q35k -- Python host mirror of the Qwen35Sharp K-quant kernel entry points,
running on the B200 kernels of libq35k.so (C ABI: include/q35k.h).

The static classes below keep the reference's names, argument meaning and
error behaviour (src/Qwen35Sharp.Kernels/*.cs), so code and tests written
against the reference read the same here:

    MulMatQ4K.Gemv / GemvPrequant / Gemm     (Kernels/MulMatQ4K.cs:12-127)
    Q5K.Gemv / GemvPrequant / Gemm / DequantizeRow   (Kernels/Q5K.cs)
    Q6K.Gemv / GemvPrequant / Gemm / DequantizeRow   (Kernels/Q6K.cs)
    Q4K.DequantizeRow                         (Kernels/Q4K.cs:35-60)
    Q8K.QuantizeRow                           (Kernels/Q8K.cs:12-77)

Where the reference takes a host pointer to GGUF blocks, these take either a
device-resident `Weight` (uploaded once, as LoadWeights does in
Model/Qwen35Model.cs:463-565) or a uint8 numpy array of the raw blocks
(uploaded for the call).  Outputs are written into the given float32 array,
as the reference writes through `float* output`.

Exceptions mirror the reference's: ArgumentException (ValueError),
NotSupportedException (NotImplementedError), InsufficientMemoryException
(MemoryError), InvalidOperationException (RuntimeError) and
TimeoutException (TimeoutError).
"""

from __future__ import annotations

import ctypes
import threading

import numpy as np

from . import _lib
from .synth import BLOCK_BYTES, Q4_K, Q5_K, Q6_K, Q8K_BYTES, QK

__all__ = [
    "Context", "Weight", "MulMatQ4K", "Q4K", "Q5K", "Q6K", "Q8K", "default_context",
    "ArgumentException", "NotSupportedException", "InsufficientMemoryException",
    "InvalidOperationException", "TimeoutException", "InvalidDataException", "GgufIOException", "GgufFile",
    "GgufTensorInfo", "Q4_K", "Q5_K", "Q6_K", "QK", "page_aligned_empty",
]


class Q35KError(Exception):
    code = -1


class ArgumentException(Q35KError, ValueError):
    code = _lib.EINVAL


class NotSupportedException(Q35KError, NotImplementedError):
    code = _lib.ENOTSUP


class InsufficientMemoryException(Q35KError, MemoryError):
    code = _lib.ENOMEM


class InvalidOperationException(Q35KError, RuntimeError):
    code = _lib.ECUDA


class TimeoutException(Q35KError, TimeoutError):
    code = _lib.ETIMEOUT


class InvalidDataException(Q35KError, ValueError):
    """A malformed or truncated GGUF file (the reference's
    InvalidDataException / EndOfStreamException)."""
    code = _lib.EDATA


class GgufIOException(Q35KError, OSError):
    """A GGUF file that cannot be opened or mapped (IOException)."""
    code = _lib.EIO


_EXC = {
    _lib.EINVAL: ArgumentException,
    _lib.ENOTSUP: NotSupportedException,
    _lib.ENOMEM: InsufficientMemoryException,
    _lib.ECUDA: InvalidOperationException,
    _lib.ETIMEOUT: TimeoutException,
    _lib.ENCCL: InvalidOperationException,
    _lib.EDATA: InvalidDataException,
    _lib.EIO: GgufIOException,
}


def _raise(rc: int, msg: str):
    raise _EXC.get(rc, Q35KError)(msg)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint8)


_CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy


def _stream(stream):
    """Map a caller stream to the C ABI: None -> the context's own stream;
    0 (torch's default stream handle) -> cudaStreamLegacy; else the handle."""
    if stream is None:
        return None
    if hasattr(stream, "cuda_stream"):
        stream = stream.cuda_stream
    return stream if stream != 0 else _CUDA_STREAM_LEGACY


def page_aligned_empty(shape, dtype=np.float32) -> np.ndarray:
    """An uninitialised array on pages of its own (an anonymous mapping), for
    a persistent buffer to register with Context.host_register: registering
    page-locks whole pages, so two buffers that share a page cannot both be
    registered."""
    import mmap

    n = int(np.prod(shape)) if np.ndim(shape) else int(shape)
    nbytes = max(n * np.dtype(dtype).itemsize, 1)
    buf = mmap.mmap(-1, (nbytes + mmap.PAGESIZE - 1) // mmap.PAGESIZE * mmap.PAGESIZE)
    return np.frombuffer(buf, dtype=dtype, count=n).reshape(shape)


def _dev_ptr(t) -> int:
    """Device address of a torch tensor / CuPy array / int."""
    if isinstance(t, int):
        return t
    if hasattr(t, "data_ptr"):
        return int(t.data_ptr())
    raise TypeError("expected a device tensor (with .data_ptr()) or an int address")


class Context:
    """One libq35k context on one CUDA device (q35k_create)."""

    def __init__(self, device: int = 0):
        self.L = _lib.load()
        h = ctypes.c_void_p()
        rc = self.L.q35k_create(device, ctypes.byref(h))
        if rc != _lib.OK:
            _raise(rc, self.L.q35k_last_error(None).decode())
        self.h = h
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            self.L.q35k_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int):
        if rc != _lib.OK:
            _raise(rc, self.L.q35k_last_error(self.h).decode())

    def sync(self):
        self._check(self.L.q35k_sync(self.h))

    def set_gemm_mode(self, mode: int):
        """q35k.GEMM_EXACT (default) or q35k.GEMM_FAST (see include/q35k.h)."""
        self._check(self.L.q35k_set_gemm_mode(self.h, mode))

    def upload(self, qtype: int, blocks: np.ndarray, n_in: int, n_out: int) -> "Weight":
        blocks = _u8(blocks)
        nb = n_in // QK if n_in > 0 else 0
        if qtype in BLOCK_BYTES and blocks.size < n_out * nb * BLOCK_BYTES[qtype]:
            raise ArgumentException("blocks buffer is smaller than nOut * nIn/256 blocks")
        h = ctypes.c_void_p()
        self._check(self.L.q35k_weight_upload(self.h, qtype, blocks.ctypes.data, n_in, n_out, ctypes.byref(h)))
        return Weight(self, h, qtype, n_in, n_out)

    def upload_gguf(self, gguf: "GgufFile", name: str) -> "Weight":
        """Upload a Q4_K/Q5_K/Q6_K tensor straight from a mapped GGUF file
        (q35k_weight_upload_gguf; LoadWeights, Model/Qwen35Model.cs:463-565)."""
        h = ctypes.c_void_p()
        self._check(self.L.q35k_weight_upload_gguf(self.h, gguf.h, name.encode(), ctypes.byref(h)))
        info = gguf.tensors[name]
        return Weight(self, h, info.type, int(info.shape[0]), int(info.shape[1]) if len(info.shape) > 1 else 1)

    def host_register(self, a: np.ndarray):
        """Page-lock a persistent host array (q35k_host_register) so that the
        host-pointer calls read and write it in place."""
        self._check(self.L.q35k_host_register(self.h, a.ctypes.data, a.nbytes))

    def host_unregister(self, a: np.ndarray):
        self._check(self.L.q35k_host_unregister(self.h, a.ctypes.data))

    # -- host-pointer calls (synchronous) --
    def matmul(self, w: "Weight", x: np.ndarray, tokens: int | None = None, out: np.ndarray | None = None) -> np.ndarray:
        """y = x @ W^T (q35k_matmul).  `out`: a float32 C-contiguous array of
        at least tokens * nOut values to write into (a caller's persistent
        output buffer, as the reference writes through `float* output`)."""
        x = _f32(x)
        tokens = x.size // w.n_in if tokens is None else tokens
        if x.size < tokens * w.n_in:
            raise ArgumentException("input is smaller than tokens * nIn")
        if out is None:
            y = np.empty((tokens, w.n_out), dtype=np.float32)
        else:
            if out.dtype != np.float32 or not out.flags.c_contiguous or out.size < tokens * w.n_out:
                raise ArgumentException("out must be a C-contiguous float32 array of at least tokens * nOut values")
            y = out
        self._check(self.L.q35k_matmul(self.h, w.h, x.ctypes.data, y.ctypes.data, tokens))
        return y

    def matmul_argmax(self, w: "Weight", x: np.ndarray, tokens: int | None = None) -> np.ndarray:
        """Vocab head + ArgMax (q35k_matmul_argmax): per token the first row
        holding the largest logit, without writing the logits."""
        x = _f32(x)
        tokens = x.size // w.n_in if tokens is None else tokens
        if x.size < tokens * w.n_in:
            raise ArgumentException("input is smaller than tokens * nIn")
        idx = np.empty(tokens, dtype=np.int32)
        self._check(self.L.q35k_matmul_argmax(self.h, w.h, x.ctypes.data, idx.ctypes.data, tokens))
        return idx

    def matmul_shared(self, ws: list, x: np.ndarray, tokens: int | None = None) -> list:
        """Several weights with the same nIn on one input, one quantization of
        it (q35k_matmul_shared; MulMatPanel.QuantizeAndGemm): [x @ W^T for W in ws]."""
        if not ws or len(ws) > MAX_SHARED:
            raise ArgumentException(f"1..{MAX_SHARED} weights per shared call")
        x = _f32(x)
        n_in = ws[0].n_in
        tokens = x.size // n_in if tokens is None else tokens
        if x.size < tokens * n_in:
            raise ArgumentException("input is smaller than tokens * nIn")
        ys = [np.empty((tokens, w.n_out), dtype=np.float32) for w in ws]
        wa = (ctypes.c_void_p * len(ws))(*[w.h for w in ws])
        ya = (ctypes.c_void_p * len(ws))(*[y.ctypes.data for y in ys])
        self._check(self.L.q35k_matmul_shared(self.h, wa, len(ws), x.ctypes.data, ya, tokens))
        return ys

    def matmul_silu(self, w: "Weight", gate: np.ndarray, up: np.ndarray, tokens: int | None = None) -> np.ndarray:
        """ffn_down on SiLU(gate) * up (q35k_matmul_silu; MulMatPanel.SiluQuantizeAndGemm)."""
        gate, up = _f32(gate), _f32(up)
        tokens = gate.size // w.n_in if tokens is None else tokens
        if gate.size < tokens * w.n_in or up.size < tokens * w.n_in:
            raise ArgumentException("gate/up is smaller than tokens * nIn")
        y = np.empty((tokens, w.n_out), dtype=np.float32)
        self._check(self.L.q35k_matmul_silu(self.h, w.h, gate.ctypes.data, up.ctypes.data, y.ctypes.data, tokens))
        return y

    def matmul_q8k(self, w: "Weight", q8: np.ndarray, tokens: int) -> np.ndarray:
        q8 = _u8(q8)
        if q8.size < tokens * (w.n_in // QK) * Q8K_BYTES:
            raise ArgumentException("q8k buffer is smaller than tokens * nIn/256 blocks")
        y = np.empty((tokens, w.n_out), dtype=np.float32)
        self._check(self.L.q35k_matmul_q8k(self.h, w.h, q8.ctypes.data, y.ctypes.data, tokens))
        return y

    def quantize_q8k(self, x: np.ndarray, k: int | None = None) -> np.ndarray:
        x = _f32(x)
        k = x.shape[-1] if k is None else k
        rows = x.size // k
        out = np.empty((rows, (k // QK) * Q8K_BYTES), dtype=np.uint8)
        self._check(self.L.q35k_quantize_q8k(self.h, x.ctypes.data, out.ctypes.data, k, rows))
        return out

    def quantize_q8k_silu(self, gate: np.ndarray, up: np.ndarray, k: int | None = None) -> np.ndarray:
        """BlockQ8K bytes of silu(gate) * up (QuantizeQ8Kx4.Quantize4x8Silu)."""
        gate, up = _f32(gate), _f32(up)
        k = gate.shape[-1] if k is None else k
        rows = gate.size // k
        if up.size < rows * k:
            raise ArgumentException("up is smaller than gate")
        out = np.empty((rows, (k // QK) * Q8K_BYTES), dtype=np.uint8)
        self._check(self.L.q35k_quantize_q8k_silu(self.h, gate.ctypes.data, up.ctypes.data, out.ctypes.data, k, rows))
        return out

    def dequantize(self, qtype: int, blocks: np.ndarray, k: int, rows: int | None = None) -> np.ndarray:
        blocks = _u8(blocks)
        bb = BLOCK_BYTES.get(qtype, 1)
        rows = blocks.size // max(1, (k // QK) * bb) if rows is None else rows
        y = np.empty((rows, k), dtype=np.float32)
        self._check(self.L.q35k_dequantize(self.h, qtype, blocks.ctypes.data, y.ctypes.data, k, rows))
        return y

    # -- device-pointer calls (asynchronous on `stream`: a torch.cuda.Stream,
    #    a cudaStream_t int, or None for the context's own stream) --
    def matmul_dev(self, w: "Weight", d_x, d_y, tokens: int, stream=None):
        self._check(self.L.q35k_matmul_dev(self.h, w.h, _dev_ptr(d_x), _dev_ptr(d_y), tokens, _stream(stream)))

    def matmul_argmax_dev(self, w: "Weight", d_x, d_y, d_idx, tokens: int, stream=None):
        """d_y may be None (logits not written); d_idx: int32[tokens]."""
        self._check(self.L.q35k_matmul_argmax_dev(self.h, w.h, _dev_ptr(d_x), _dev_ptr(d_y) if d_y is not None else None,
                                                  _dev_ptr(d_idx), tokens, _stream(stream)))

    def matmul_shared_dev(self, ws: list, d_x, d_ys: list, tokens: int, stream=None):
        wa = (ctypes.c_void_p * len(ws))(*[w.h for w in ws])
        ya = (ctypes.c_void_p * len(d_ys))(*[_dev_ptr(y) for y in d_ys])
        self._check(self.L.q35k_matmul_shared_dev(self.h, wa, len(ws), _dev_ptr(d_x), ya, tokens, _stream(stream)))

    def matmul_silu_dev(self, w: "Weight", d_gate, d_up, d_y, tokens: int, stream=None):
        self._check(self.L.q35k_matmul_silu_dev(self.h, w.h, _dev_ptr(d_gate), _dev_ptr(d_up), _dev_ptr(d_y), tokens,
                                                _stream(stream)))

    def matmul_q8k_dev(self, w: "Weight", d_q8, d_y, tokens: int, stream=None):
        self._check(self.L.q35k_matmul_q8k_dev(self.h, w.h, _dev_ptr(d_q8), _dev_ptr(d_y), tokens, _stream(stream)))

    def quantize_q8k_dev(self, d_x, d_q8, k: int, rows: int, stream=None):
        self._check(self.L.q35k_quantize_q8k_dev(self.h, _dev_ptr(d_x), _dev_ptr(d_q8), k, rows, _stream(stream)))

    def dequantize_dev(self, qtype: int, d_blocks, d_y, k: int, rows: int, stream=None):
        self._check(self.L.q35k_dequantize_dev(self.h, qtype, _dev_ptr(d_blocks), _dev_ptr(d_y), k, rows,
                                               _stream(stream)))


class GgufTensorInfo:
    """Type, shape (GGUF order, dim 0 innermost) and data-section offset of
    one tensor (Qwen35Sharp.Gguf/GgufTensorInfo.cs)."""

    def __init__(self, name: str, type: int, shape: tuple, offset: int):
        self.name, self.type, self.shape, self.offset = name, type, shape, offset

    @property
    def num_elements(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    def __repr__(self):
        return f"GgufTensorInfo({self.name!r}, type={self.type}, shape={self.shape}, offset={self.offset})"


class GgufFile:
    """A memory-mapped GGUF v2/v3 file (q35k_gguf_open; Qwen35Sharp.Gguf/
    GgufFile.cs).  Host only: needs libq35k.so but no GPU."""

    def __init__(self, path: str):
        self.L = _lib.load()
        h = ctypes.c_void_p()
        rc = self.L.q35k_gguf_open(str(path).encode(), ctypes.byref(h))
        if rc != _lib.OK:
            _raise(rc, self.L.q35k_last_error(None).decode())
        self.h = h
        ver, n, al, off = ctypes.c_int(), ctypes.c_int(), ctypes.c_uint32(), ctypes.c_uint64()
        self.L.q35k_gguf_info(h, ctypes.byref(ver), ctypes.byref(n), ctypes.byref(al), ctypes.byref(off))
        self.version, self.alignment, self.data_offset = ver.value, al.value, off.value
        self.tensors: dict[str, GgufTensorInfo] = {}
        self._index: dict[str, int] = {}
        name, ty, nd, off = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int(), ctypes.c_uint64()
        dims = (ctypes.c_int64 * 4)()
        for i in range(n.value):
            self.L.q35k_gguf_tensor(h, i, ctypes.byref(name), ctypes.byref(ty), ctypes.byref(nd), dims,
                                    ctypes.byref(off))
            nm = name.value.decode()
            self.tensors[nm] = GgufTensorInfo(nm, ty.value, tuple(dims[d] for d in range(nd.value)), off.value)
            self._index[nm] = i

    def close(self):
        if getattr(self, "h", None):
            self.L.q35k_gguf_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def data(self, name: str, nbytes: int) -> np.ndarray:
        """A copy of the first nbytes bytes of tensor `name`."""
        p = ctypes.c_void_p()
        rc = self.L.q35k_gguf_tensor_data(self.h, self._index[name], nbytes, ctypes.byref(p))
        if rc != _lib.OK:
            _raise(rc, self.L.q35k_last_error(None).decode())
        return np.ctypeslib.as_array((ctypes.c_uint8 * nbytes).from_address(p.value)).copy() if nbytes else \
            np.empty(0, np.uint8)

    def get_int(self, key: str, default: int | None = None) -> int:
        v = ctypes.c_int64()
        if self.L.q35k_gguf_get_int(self.h, key.encode(), ctypes.byref(v)) != _lib.OK:
            if default is None:
                raise KeyError(f"GGUF missing or non-integer key '{key}'")
            return default
        return v.value

    def get_float(self, key: str, default: float = 0.0) -> float:
        v = ctypes.c_double()
        if self.L.q35k_gguf_get_float(self.h, key.encode(), ctypes.byref(v)) != _lib.OK:
            return default
        return v.value

    def get_string(self, key: str, default: str = "") -> str:
        v = ctypes.c_char_p()
        if self.L.q35k_gguf_get_string(self.h, key.encode(), ctypes.byref(v)) != _lib.OK:
            return default
        return v.value.decode("utf-8", errors="replace")

    def get_array(self, key: str):
        """(element type, length) of an array value, or None."""
        t, n = ctypes.c_int(), ctypes.c_uint64()
        if self.L.q35k_gguf_get_array(self.h, key.encode(), ctypes.byref(t), ctypes.byref(n)) != _lib.OK:
            return None
        return t.value, n.value


class Weight:
    """A device-resident K-quant weight (q35k_weight_upload)."""

    def __init__(self, ctx: Context, h, qtype: int, n_in: int, n_out: int):
        self.ctx, self.h, self.qtype, self.n_in, self.n_out = ctx, h, qtype, n_in, n_out
        self.nb = n_in // QK

    def free(self):
        if getattr(self, "h", None) and self.ctx.h:
            self.ctx.L.q35k_weight_free(self.ctx.h, self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    @property
    def device_bytes(self) -> int:
        sz = ctypes.c_size_t()
        self.ctx.L.q35k_weight_info(self.h, None, None, None, ctypes.byref(sz))
        return sz.value


# ---------------------------------------------------------------------------
# Row-sharded matmul over several GPUs (q35k_shard_*).
# ---------------------------------------------------------------------------

GATHER_NCCL, GATHER_PEER, GATHER_FUSED = _lib.GATHER_NCCL, _lib.GATHER_PEER, _lib.GATHER_FUSED
GEMM_EXACT, GEMM_FAST = _lib.GEMM_EXACT, _lib.GEMM_FAST
MAX_SHARED = _lib.MAX_SHARED


def shard_rows(n_out: int, nranks: int) -> int:
    """Rows per rank: an equal share (the C library's rule; the last rank may
    hold fewer)."""
    return (n_out + nranks - 1) // nranks


def shard_range(n_out: int, nranks: int, rank: int) -> tuple[int, int]:
    n = shard_rows(n_out, nranks)
    r0 = min(n_out, rank * n)
    return r0, min(n_out, r0 + n)


def nccl_unique_id() -> bytes:
    """An NCCL unique id for q35k_shard_create_rank (share it between ranks)."""
    L = _lib.load()
    buf = ctypes.create_string_buffer(_lib.NCCL_ID_BYTES)
    rc = L.q35k_nccl_unique_id(buf)
    if rc != _lib.OK:
        _raise(rc, L.q35k_last_error(None).decode())
    return buf.raw


class Shard:
    """A group of GPUs sharing row-sharded weights.

    Shard(devices=[0, 1, ...]) drives all of them from this process;
    Shard(nranks=N, rank=r, nccl_id=id, device=d) is this process's rank of a
    one-process-per-GPU group.
    """

    def __init__(self, devices=None, *, nranks=None, rank=None, nccl_id=None, device=None):
        self.L = _lib.load()
        h = ctypes.c_void_p()
        if devices is not None:
            devs = (ctypes.c_int * len(devices))(*devices)
            rc = self.L.q35k_shard_create(len(devices), devs, ctypes.byref(h))
        else:
            idbuf = ctypes.create_string_buffer(nccl_id, _lib.NCCL_ID_BYTES) if nccl_id is not None else None
            rc = self.L.q35k_shard_create_rank(nranks, rank, idbuf, device, ctypes.byref(h))
        if rc != _lib.OK:
            _raise(rc, self.L.q35k_last_error(None).decode())
        self.h = h
        n, r0, loc = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        self.L.q35k_shard_info(self.h, ctypes.byref(n), ctypes.byref(r0), ctypes.byref(loc))
        self.nranks, self.first_rank, self.local_devices = n.value, r0.value, loc.value

    def close(self):
        if getattr(self, "h", None):
            self.L.q35k_shard_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int):
        if rc != _lib.OK:
            _raise(rc, self.L.q35k_shard_last_error(self.h).decode())

    def upload(self, qtype: int, blocks: np.ndarray, n_in: int, n_out: int) -> "ShardedWeight":
        blocks = _u8(blocks)
        h = ctypes.c_void_p()
        self._check(self.L.q35k_shard_weight_upload(self.h, qtype, blocks.ctypes.data, n_in, n_out, ctypes.byref(h)))
        return ShardedWeight(self, h, qtype, n_in, n_out)

    def matmul(self, w: "ShardedWeight", x: np.ndarray, tokens: int | None = None, gather: int = GATHER_NCCL):
        x = _f32(x)
        tokens = tokens if tokens is not None else x.size // w.n_in
        y = np.empty((tokens, w.n_out), dtype=np.float32)
        self._check(self.L.q35k_shard_matmul(self.h, w.h, x.ctypes.data, y.ctypes.data, tokens, gather))
        return y

    def matmul_dev(self, w: "ShardedWeight", d_xs, d_ys, tokens: int, gather: int = GATHER_NCCL, streams=None):
        """streams: one cudaStream_t (int or torch stream) per local device,
        or None for the group's own streams."""
        n = len(d_xs)
        xs = (ctypes.c_void_p * n)(*[_dev_ptr(t) for t in d_xs])
        ys = (ctypes.c_void_p * n)(*[_dev_ptr(t) for t in d_ys])
        ss = None
        if streams is not None:
            ss = (ctypes.c_void_p * n)(*[getattr(t, "cuda_stream", t) for t in streams])
        self._check(self.L.q35k_shard_matmul_dev(self.h, w.h, xs, ys, tokens, gather, ss))

    def sync(self):
        self._check(self.L.q35k_shard_sync(self.h))

    def set_wait_limit(self, milliseconds: int):
        """Bound of the fused gather's wait for the peers (q35k_shard_set_wait_limit)."""
        self._check(self.L.q35k_shard_set_wait_limit(self.h, int(milliseconds)))

    def reset(self):
        """Collective recovery after a TimeoutException (q35k_shard_reset)."""
        self._check(self.L.q35k_shard_reset(self.h))

    def set_trace(self, on: bool = True):
        self._check(self.L.q35k_shard_set_trace(self.h, 1 if on else 0))

    TRACE_PHASES = ("gemv_start", "gemv_end", "gather_start", "peers_seen", "gemv_done_seen", "gather_end")

    def trace(self, local: int = 0) -> dict:
        """Phase timestamps (ns, %globaltimer) of the last fused call on local
        device `local` (q35k_shard_trace)."""
        buf = (ctypes.c_uint64 * 6)()
        self._check(self.L.q35k_shard_trace(self.h, local, buf))
        return dict(zip(self.TRACE_PHASES, list(buf)))


class ShardedWeight:
    def __init__(self, shard: Shard, h, qtype: int, n_in: int, n_out: int):
        self.shard, self.h, self.qtype, self.n_in, self.n_out = shard, h, qtype, n_in, n_out

    def free(self):
        if getattr(self, "h", None) and self.shard.h:
            self.shard.L.q35k_shard_weight_free(self.shard.h, self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


_tls = threading.local()


def default_context(device: int = 0) -> Context:
    """The calling thread's context on `device` (one per thread, as the
    reference keeps one pool + scratch arena per model)."""
    cache = getattr(_tls, "ctx", None)
    if cache is None:
        cache = _tls.ctx = {}
    if device not in cache:
        cache[device] = Context(device)
    return cache[device]


# ---------------------------------------------------------------------------
# Reference-named entry points.
# ---------------------------------------------------------------------------

def _weight(qtype: int, weights, n_in: int, n_out: int) -> Weight:
    if isinstance(weights, Weight):
        if weights.qtype != qtype:
            raise ArgumentException(f"weight type {weights.qtype} does not match {qtype}")
        if weights.n_in != n_in or weights.n_out != n_out:
            raise ArgumentException("nIn/nOut do not match the uploaded weight")
        return weights
    return default_context().upload(qtype, weights, n_in, n_out)


def _store(output, y: np.ndarray):
    if output is None:
        return y
    out = np.asarray(output)
    if out.dtype != np.float32 or not out.flags.c_contiguous:
        raise ArgumentException("output must be a contiguous float32 array")
    out.reshape(-1)[: y.size] = y.reshape(-1)
    return out


def _check_nin(n_in: int):
    if n_in <= 0 or n_in % QK:
        raise NotSupportedException(f"nIn={n_in} is not a multiple of 256")


class _KQuantKernels:
    qtype = 0

    @classmethod
    def Gemv(cls, weights, input, output, nIn: int, nOut: int, pool=None, scratch=None):
        """Q8K.QuantizeRow(input) then one dot per output row (1 token)."""
        _check_nin(nIn)
        w = _weight(cls.qtype, weights, nIn, nOut)
        return _store(output, w.ctx.matmul(w, _f32(input).reshape(-1)[:nIn], 1).reshape(-1))

    @classmethod
    def GemvPrequant(cls, weights, y, output, nIn: int, nOut: int, pool=None):
        """One dot per output row against a caller-quantized Q8_K row."""
        _check_nin(nIn)
        w = _weight(cls.qtype, weights, nIn, nOut)
        return _store(output, w.ctx.matmul_q8k(w, y, 1).reshape(-1))

    @classmethod
    def _gemm(cls, weights, input, output, nIn: int, nOut: int, tokens: int):
        _check_nin(nIn)
        if tokens <= 0:
            raise ArgumentException("tokens must be positive")
        w = _weight(cls.qtype, weights, nIn, nOut)
        return _store(output, w.ctx.matmul(w, input, tokens))


class MulMatQ4K(_KQuantKernels):
    """Q4_K x F32 matmul (Kernels/MulMatQ4K.cs)."""

    qtype = Q4_K

    @classmethod
    def Gemm(cls, packed, rows, input, output, nIn: int, nOut: int, tokens: int, pool=None, scratch=None,
             meta=None):
        """Prefill/decode for any token count (MulMatQ4K.cs:45-127).  `packed`
        and `meta` (the CPU panel formats) are not needed: `rows` is the
        weight (a Weight or raw blocks)."""
        return cls._gemm(rows if rows is not None else packed, input, output, nIn, nOut, tokens)


class Q5K(_KQuantKernels):
    """Q5_K kernels (Kernels/Q5K.cs)."""

    qtype = Q5_K

    @classmethod
    def Gemm(cls, weights, input, output, nIn: int, nOut: int, tokens: int, pool=None):
        return cls._gemm(weights, input, output, nIn, nOut, tokens)

    @staticmethod
    def DequantizeRow(x, y, k: int):
        return _store(y, default_context().dequantize(Q5_K, x, k).reshape(-1))


class Q6K(_KQuantKernels):
    """Q6_K kernels (Kernels/Q6K.cs)."""

    qtype = Q6_K

    @classmethod
    def Gemm(cls, weights, input, output, nIn: int, nOut: int, tokens: int, pool=None, scratch=None):
        return cls._gemm(weights, input, output, nIn, nOut, tokens)

    @staticmethod
    def DequantizeRow(x, y, k: int):
        return _store(y, default_context().dequantize(Q6_K, x, k).reshape(-1))


class Q4K:
    """Q4_K block helpers (Kernels/Q4K.cs)."""

    @staticmethod
    def DequantizeRow(x, y, k: int):
        return _store(y, default_context().dequantize(Q4_K, x, k).reshape(-1))


class Q8K:
    """Q8_K activation quantizer (Kernels/Q8K.cs)."""

    @staticmethod
    def QuantizeRow(x, y, k: int):
        """Bit-exact BlockQ8K bytes of k values; written into y (uint8) if given."""
        if k <= 0 or k % QK:
            raise ArgumentException(f"k={k} is not a multiple of 256")
        q = default_context().quantize_q8k(_f32(x).reshape(-1)[:k], k).reshape(-1)
        if y is None:
            return q
        out = np.asarray(y)
        out.reshape(-1).view(np.uint8)[: q.size] = q
        return out

    @staticmethod
    def RowBytes(k: int) -> int:
        return (k // QK) * Q8K_BYTES
