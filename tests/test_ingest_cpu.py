"""Checkpoint reading (csrc/ingest.cu, host side, no GPU): the library's
safetensors parser against the reference's own reader (ds_safetensors.c,
compiled unmodified into oracle/_ref) on synthetic checkpoints in the
reference's tensor naming: every tensor's dtype, shape, offset and size,
single file and shards; and the parser's own checks on malformed files."""
import ctypes
import os

import numpy as np
import pytest

import oracle as O
from ds_ocr_b200 import _lib, synth
from st_checkpoint import write_checkpoint, write_safetensors, decoder_tensors


def _ours(lib, path, name):
    dt, nd = ctypes.c_int(), ctypes.c_int()
    shape = (ctypes.c_int64 * 8)()
    off, size = ctypes.c_size_t(), ctypes.c_size_t()
    r = lib.ds_cuda_safetensors_find(path.encode(), name.encode(), ctypes.byref(dt), ctypes.byref(nd), shape,
                                     ctypes.byref(off), ctypes.byref(size))
    if r != 1:
        return r
    return dt.value, list(shape[:nd.value]), off.value, size.value


def _ref(r, path, name):
    dt, nd = ctypes.c_int(), ctypes.c_int()
    shape = (ctypes.c_int64 * 8)()
    off, size = ctypes.c_size_t(), ctypes.c_size_t()
    f = r.ref_st_find(path.encode(), name.encode(), ctypes.addressof(dt), ctypes.addressof(nd),
                      ctypes.addressof(shape), ctypes.addressof(off), ctypes.addressof(size))
    if f != 1:
        return f
    return dt.value, list(shape[:nd.value]), off.value, size.value


@pytest.fixture(scope="module")
def small():
    return synth.Model(n_layers=2, n_experts=8, vocab=512)


@pytest.mark.ref
@pytest.mark.parametrize("shards,norm", [(1, "BF16"), (3, "F32")])
def test_parser_matches_reference_reader(tmp_path, small, shards, norm):
    lib = _lib.load()
    r = O.ref()
    d = str(tmp_path)
    write_checkpoint(small, d, shards=shards, norm_dtype=norm)
    names = list(decoder_tensors(small, norm_dtype=norm))
    assert lib.ds_cuda_safetensors_count(d.encode()) == len(names) == r.ref_st_count(d.encode())
    for n in names:
        assert _ours(lib, d, n) == _ref(r, d, n), n
    assert _ours(lib, d, "model.layers.9.nope") == 0 == _ref(r, d, "model.layers.9.nope")


def test_parser_reads_the_bytes_written(tmp_path):
    lib = _lib.load()
    p = str(tmp_path / "one.safetensors")
    a = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    b = (np.arange(10, dtype=np.uint16) * 3)
    write_safetensors(p, {"a\\u0041\"x": ("F32", a), "b": ("BF16", b), "c": ("I64", np.arange(3, dtype=np.int64))},
                      metadata={"k": "v{]", "n": [1, {"z": 2}]}, pad_header=7)
    assert lib.ds_cuda_safetensors_count(p.encode()) == 3
    # JSON escapes in names: an escaped backslash and quote
    assert _ours(lib, p, 'a\\u0041"x')[:2] == (0, [2, 3, 4])
    dt, shape, off, size = _ours(lib, p, "b")
    assert (dt, shape, size) == (2, [10], 20)
    raw = open(p, "rb").read()
    n = int(np.frombuffer(raw[:8], np.uint64)[0])
    assert np.array_equal(np.frombuffer(raw[8 + n + off:8 + n + off + size], np.uint16), b)
    dt, shape, off, size = _ours(lib, p, "c")
    assert (dt, shape, size) == (4, [3], 24)


@pytest.mark.parametrize("bad", ["short", "length", "json", "offsets", "size"])
def test_parser_rejects_malformed_files(tmp_path, bad):
    lib = _lib.load()
    p = str(tmp_path / "bad.safetensors")
    good = {"w": ("BF16", np.zeros((4, 4), np.uint16))}
    write_safetensors(p, good)
    raw = bytearray(open(p, "rb").read())
    n = int(np.frombuffer(bytes(raw[:8]), np.uint64)[0])
    if bad == "short":
        raw = raw[:5]
    elif bad == "length":
        raw[:8] = np.uint64(len(raw)).tobytes()
    elif bad == "json":
        raw[8] = ord("[")
    elif bad == "offsets":
        h = raw[8:8 + n].decode().replace("[0, 32]", "[0, 64]")
        raw = raw[:8] + h.encode() + raw[8 + n:]
    elif bad == "size":
        h = raw[8:8 + n].decode().replace("[4, 4]", "[4, 5]")
        raw = raw[:8] + h.encode() + raw[8 + n:]  # same header length
    open(p, "wb").write(bytes(raw))
    assert lib.ds_cuda_safetensors_count(p.encode()) < 0
    assert lib.ds_cuda_safetensors_error()


def test_missing_directory_fails(tmp_path):
    lib = _lib.load()
    assert lib.ds_cuda_safetensors_count(str(tmp_path / "none").encode()) < 0
    assert b"cannot open" in lib.ds_cuda_safetensors_error()


def test_parser_survives_mutated_files(tmp_path):
    # truncated, bit-flipped and length-corrupted files: the parser returns
    # a status (a count or < 0), never crashes or reads past the file
    from hypothesis import given, settings, strategies as st

    lib = _lib.load()
    base = str(tmp_path / "base.safetensors")
    write_safetensors(base, {"a": ("F32", np.arange(12, dtype=np.float32).reshape(3, 4)),
                             "b.c": ("BF16", np.arange(8, dtype=np.uint16)),
                             "z": ("I64", np.arange(2, dtype=np.int64))}, metadata={"k": "v"})
    good = open(base, "rb").read()
    p = str(tmp_path / "mut.safetensors")

    @settings(max_examples=300, deadline=None)
    @given(st.integers(0, len(good)), st.lists(st.tuples(st.integers(0, len(good) - 1), st.integers(0, 255)),
                                               max_size=6), st.integers(0, 3))
    def check(cut, flips, length_mode):
        raw = bytearray(good[:max(cut, 0)] if cut < len(good) else good)
        for pos, val in flips:
            if pos < len(raw):
                raw[pos] = val
        if length_mode == 1 and len(raw) >= 8:
            raw[:8] = np.uint64(2**63 - 1).tobytes()
        elif length_mode == 2 and len(raw) >= 8:
            raw[:8] = np.uint64(0).tobytes()
        open(p, "wb").write(bytes(raw))
        r = lib.ds_cuda_safetensors_count(p.encode())
        assert r < 0 or 0 <= r <= 3 + 16

    check()
