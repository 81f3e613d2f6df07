"""GGUF ingestion (q35k_gguf_* and q35k_weight_upload_gguf): the reference
reader's behaviour (Qwen35Sharp.Gguf/GgufFile.cs) on synthetic files, and
weights uploaded straight from the mapping.  The parser is host code: every
test here but the last two runs without a GPU."""

import struct

import numpy as np
import pytest

import gguf_writer as gw
import q35k
from q35k import synth
from q35k.synth import Q4_K, Q5_K, Q6_K


def write(tmp_path, blob: bytes, name="m.gguf"):
    p = tmp_path / name
    p.write_bytes(blob)
    return str(p)


def model_blob(alignment=None, version=3):
    kv = [
        ("general.architecture", gw.STRING, "qwen35"),
        ("general.name", gw.STRING, "synthetic"),
        ("qwen35.block_count", gw.U32, 2),
        ("qwen35.embedding_length", gw.U64, 512),
        ("qwen35.rope.freq_base", gw.F32, 1e6),
        ("qwen35.attention.layer_norm_rms_epsilon", gw.F64, 1e-6),
        ("qwen35.context_length", gw.I32, -7),
        ("small.u8", gw.U8, 200), ("small.i8", gw.I8, -5), ("small.u16", gw.U16, 65000),
        ("small.i16", gw.I16, -300), ("small.i64", gw.I64, -(2 ** 40)), ("flag", gw.BOOL, 1),
        ("tokenizer.ggml.tokens", gw.ARRAY, ["a", "bb", "ccc"], gw.STRING),
        ("qwen35.rope.dimension_sections", gw.ARRAY, [11, 11, 10, 0], gw.I32),
    ]
    t = [
        gw.kquant_tensor("blk.0.ffn_gate.weight", Q4_K, synth.kquant_blocks(Q4_K, 40, 512, seed=1), 512, 40),
        gw.kquant_tensor("blk.0.ffn_down.weight", Q5_K, synth.kquant_blocks(Q5_K, 33, 256, seed=2), 256, 33),
        gw.kquant_tensor("output.weight", Q6_K, synth.kquant_blocks(Q6_K, 65, 768, seed=3), 768, 65),
        ("output_norm.weight", gw.F32_TYPE, [512], np.arange(512, dtype=np.float32).tobytes()),
    ]
    return gw.build(kv, t, version=version, alignment=alignment), t


@pytest.mark.parametrize("alignment", [None, 64, 4096])
@pytest.mark.parametrize("version", [2, 3])
def test_tensors_and_metadata_round_trip(tmp_path, alignment, version):
    blob, tensors = model_blob(alignment, version)
    with q35k.GgufFile(write(tmp_path, blob)) as g:
        assert g.version == version
        assert g.alignment == (alignment or 32)
        assert g.data_offset % g.alignment == 0
        assert list(g.tensors) == [t[0] for t in tensors]
        for name, ty, dims, data in tensors:
            info = g.tensors[name]
            assert info.type == ty and info.shape == tuple(dims)
            assert info.offset % g.alignment == 0
            assert info.num_elements == int(np.prod(dims))
            assert g.data(name, len(data)).tobytes() == data
        assert g.get_string("general.architecture") == "qwen35"
        assert g.get_int("qwen35.block_count") == 2
        assert g.get_int("qwen35.embedding_length") == 512
        assert g.get_int("qwen35.context_length") == -7
        assert (g.get_int("small.u8"), g.get_int("small.i8"), g.get_int("small.u16"), g.get_int("small.i16"),
                g.get_int("small.i64")) == (200, -5, 65000, -300, -(2 ** 40))
        assert g.get_float("qwen35.rope.freq_base") == pytest.approx(1e6)
        assert g.get_float("qwen35.attention.layer_norm_rms_epsilon") == 1e-6
        assert g.get_float("qwen35.block_count") == 2.0  # integers coerce to float
        assert g.get_array("tokenizer.ggml.tokens") == (gw.STRING, 3)
        assert g.get_array("qwen35.rope.dimension_sections") == (gw.I32, 4)
        # bool is not an integer, a string is not an integer, a missing key has the default
        assert g.get_int("flag", -1) == -1
        assert g.get_int("general.name", -1) == -1
        assert g.get_string("missing", "dflt") == "dflt"
        with pytest.raises(KeyError):
            g.get_int("missing")


def test_no_tensors_data_section_not_aligned(tmp_path):
    blob = gw.build([("general.name", gw.STRING, "x" * 13)], [])
    with q35k.GgufFile(write(tmp_path, blob)) as g:
        assert g.tensors == {}
        assert g.data_offset == len(blob)  # alignment applies only when there are tensors


def test_duplicate_names_last_wins(tmp_path):
    a = synth.kquant_blocks(Q4_K, 1, 256, seed=4)
    b = synth.kquant_blocks(Q4_K, 1, 256, seed=5)
    blob = gw.build([], [gw.kquant_tensor("w", Q4_K, a, 256, 1), gw.kquant_tensor("w", Q4_K, b, 256, 1)])
    with q35k.GgufFile(write(tmp_path, blob)) as g:
        assert g.data("w", b.nbytes).tobytes() == b.tobytes()


def header(version=3, n_tensors=0, n_kv=0):
    return b"GGUF" + struct.pack("<IQQ", version, n_tensors, n_kv)


@pytest.mark.parametrize("blob,exc,msg", [
    (b"GGUF" + b"\0" * 10, q35k.InvalidDataException, "too small"),
    (b"GGML" + struct.pack("<IQQ", 3, 0, 0), q35k.InvalidDataException, "not a GGUF file"),
    (header(version=1), q35k.NotSupportedException, "version 1"),
    (header(version=4), q35k.NotSupportedException, "version 4"),
    (header(n_tensors=2 ** 31), q35k.InvalidDataException, "implausibly large"),
    (header(n_kv=1) + gw.gstr("") + gw.value(gw.U8, 1), q35k.InvalidDataException, "is empty"),
    (header(n_kv=1) + gw.gstr("k") + struct.pack("<i", 13) + b"\0" * 8, q35k.InvalidDataException,
     "unknown GGUF value type"),
    (header(n_kv=1) + gw.gstr("k") + struct.pack("<iiQ", gw.ARRAY, gw.ARRAY, 1) + b"\0" * 16,
     q35k.InvalidDataException, "nested"),
    (header(n_kv=1) + gw.gstr("k") + struct.pack("<iiQ", gw.ARRAY, gw.U8, 2 ** 31), q35k.InvalidDataException,
     "exceeds int.MaxValue"),
    (header(n_kv=1) + struct.pack("<Q", 2 ** 31) + b"k" * 8, q35k.InvalidDataException, "exceeds 2 GB"),
    (header(n_kv=1) + gw.gstr("general.alignment") + gw.value(gw.U32, 48), q35k.InvalidDataException,
     "not a power of two"),
    (header(n_kv=1) + gw.gstr("general.alignment") + gw.value(gw.U32, 0), q35k.InvalidDataException,
     "not a power of two"),
    (header(n_kv=1) + gw.gstr("general.alignment") + gw.value(gw.I32, -32), q35k.InvalidDataException,
     "out of range"),
    (header(n_tensors=1) + gw.gstr("t") + struct.pack("<I", 0) + struct.pack("<iQ", 12, 0),
     q35k.InvalidDataException, "invalid dim count 0"),
    (header(n_tensors=1) + gw.gstr("t") + struct.pack("<I", 5) + b"\0" * 52, q35k.InvalidDataException,
     "invalid dim count 5"),
    (header(n_tensors=1) + gw.gstr("t") + struct.pack("<Iqq", 2, 256, -1) + struct.pack("<iQ", 12, 0),
     q35k.InvalidDataException, "is negative"),
    (header(n_tensors=1) + gw.gstr("t") + struct.pack("<Iq", 1, 256) + struct.pack("<iQ", 12, 0),
     q35k.InvalidDataException, "past end of file"),
    (header(n_kv=2) + gw.gstr("k") + gw.value(gw.U32, 1), q35k.InvalidDataException, "unexpected end"),
])
def test_malformed_files(tmp_path, blob, exc, msg):
    with pytest.raises(exc, match=msg):
        q35k.GgufFile(write(tmp_path, blob))


def test_missing_file(tmp_path):
    with pytest.raises(q35k.GgufIOException, match="cannot open"):
        q35k.GgufFile(str(tmp_path / "absent.gguf"))


def test_every_truncation_is_an_error_not_a_crash(tmp_path):
    blob, _ = model_blob(alignment=64)
    with q35k.GgufFile(write(tmp_path, blob)) as g:
        data_start = g.data_offset
    # Cut inside the header, metadata or tensor table: always a clean error.
    for cut in list(range(24, data_start, 7)) + [data_start - 1]:
        with pytest.raises((q35k.InvalidDataException, q35k.NotSupportedException)):
            q35k.GgufFile(write(tmp_path, blob[:cut], "cut.gguf"))


def test_random_corruption_never_crashes(tmp_path):
    blob, _ = model_blob()
    rng = np.random.default_rng(7)
    ok = 0
    for trial in range(300):
        b = bytearray(blob)
        for _ in range(rng.integers(1, 4)):
            b[rng.integers(0, 600)] = rng.integers(0, 256)
        try:
            with q35k.GgufFile(write(tmp_path, bytes(b), "c.gguf")) as g:
                for name in g.tensors:
                    g.tensors[name].num_elements
            ok += 1
        except (q35k.InvalidDataException, q35k.NotSupportedException):
            pass
    assert ok > 0  # some corruptions only touch values


def test_tensor_data_past_the_end(tmp_path):
    w = synth.kquant_blocks(Q4_K, 4, 256, seed=9)
    blob = gw.build([], [gw.kquant_tensor("w", Q4_K, w, 256, 4)], pad_data=False)
    with q35k.GgufFile(write(tmp_path, blob[:-10])) as g:
        with pytest.raises(q35k.InvalidDataException, match="past the end"):
            g.data("w", w.nbytes)
        assert g.data("w", w.nbytes - 10).tobytes() == w.tobytes()[:-10]


@pytest.mark.gpu
def test_upload_from_gguf_matches_raw_upload(tmp_path, ctx):
    blob, tensors = model_blob(alignment=64)
    with q35k.GgufFile(write(tmp_path, blob)) as g:
        for name, ty, dims, data in tensors[:3]:
            n_in, n_out = dims
            W = ctx.upload_gguf(g, name)
            assert (W.qtype, W.n_in, W.n_out) == (ty, n_in, n_out)
            R = ctx.upload(ty, np.frombuffer(data, np.uint8), n_in, n_out)
            x = synth.activations(3, n_in, seed=n_in)
            assert (ctx.matmul(W, x) == ctx.matmul(R, x)).all()
            W.free()
            R.free()
        with pytest.raises(q35k.NotSupportedException, match="not Q4_K"):
            ctx.upload_gguf(g, "output_norm.weight")
        with pytest.raises(q35k.ArgumentException, match="no tensor"):
            ctx.upload_gguf(g, "absent.weight")


@pytest.mark.gpu
def test_upload_gguf_rejects_what_load_weights_rejects(tmp_path, ctx):
    w = synth.kquant_blocks(Q4_K, 8, 256, seed=11)
    stack = np.concatenate([w, w])
    blob = gw.build([], [
        ("ragged", Q4_K, [300, 8], w.tobytes()),        # nIn not a multiple of 256
        ("experts", Q4_K, [256, 8, 2], stack.tobytes()),  # a stack of matrices
        ("short", Q4_K, [256, 64], w.tobytes()),        # rows past the end of the file
    ], pad_data=False)
    with q35k.GgufFile(write(tmp_path, blob)) as g:
        with pytest.raises(q35k.NotSupportedException, match="multiple of 256"):
            ctx.upload_gguf(g, "ragged")
        with pytest.raises(q35k.NotSupportedException, match="stack of matrices"):
            ctx.upload_gguf(g, "experts")
        with pytest.raises(q35k.InvalidDataException, match="past the end"):
            ctx.upload_gguf(g, "short")
