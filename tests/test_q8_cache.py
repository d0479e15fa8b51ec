"""The Q8 cache mirror (dianoia_b200/q8_cache.py) after dianoia's
lib/src/q8_cache.dart and its tests (test/failure_recovery_test.dart:27-74):
a written cache opens and gives back every matrix's bytes; a truncated file, a
header length past the end and a matrix offset outside the file raise
FormatException and release the mapping; another key, version or magic is a
miss. The key is FNV-1a 64, checked against the algorithm's published test
vectors. CPU only: the GPU side is in test_q8_cache_gpu.py."""
import json
import os
import struct

import numpy as np
import pytest

from dianoia_b200.q8_cache import (FormatException, MappedFile, Q8Cache, byte_lengths, fnv1a64,
                                   HEADER_REGION)


class Arrays:
    """A CachedMatrix from numpy arrays (format, rows, cols, qs_bytes, scale_bytes)."""

    def __init__(self, fmt, rows, cols, rng):
        self.format, self.rows, self.cols = fmt, rows, cols
        qn, sn = byte_lengths(fmt, rows, cols)
        self.qs_bytes = rng.integers(0, 256, qn, dtype=np.uint8)
        if fmt == "q4":
            self.scale_bytes = rng.uniform(1e-3, 1e-2, sn // 2).astype(np.float16).view(np.uint8)
        else:
            self.scale_bytes = rng.uniform(1e-3, 1e-2, sn // 4).astype(np.float32).view(np.uint8)


@pytest.fixture
def cache_file(tmp_path):
    rng = np.random.default_rng(3)
    mats = {"layers.0.q": Arrays("q8", 64, 128, rng), "layers.0.gate": Arrays("q4", 96, 64, rng),
            "lm_head": Arrays("q8", 40, 96, rng)}
    path = str(tmp_path / "weights.q8cache")
    Q8Cache.write(path, "k123", mats)
    return path, mats


def test_fnv1a64_published_vectors():
    assert fnv1a64(b"") == 0xCBF29CE484222325
    assert fnv1a64(b"a") == 0xAF63DC4C8601EC8C
    assert fnv1a64(b"foobar") == 0x85944171F73967E8
    # continuing a hash equals hashing the concatenation
    assert fnv1a64(b"bar", fnv1a64(b"foo")) == fnv1a64(b"foobar")


def test_key_follows_checkpoint_config_and_format(tmp_path):
    d = tmp_path / "model"
    d.mkdir()
    header = json.dumps({"w": {"dtype": "BF16", "shape": [2, 2], "data_offsets": [0, 8]}}).encode()
    (d / "model.safetensors").write_bytes(struct.pack("<Q", len(header)) + header + bytes(8))
    (d / "config.json").write_text('{"hidden_size": 2}')
    k8 = Q8Cache.key_for(str(d))
    assert len(k8) == 16 and int(k8, 16) >= 0
    assert Q8Cache.key_for(str(d), weights="q8") == k8
    assert Q8Cache.key_for(str(d), weights="q4") != k8
    # by hand: FNV-1a over the length bytes, the header, the file length, config, format text
    st = (d / "model.safetensors").read_bytes()
    h = fnv1a64(st[:8])
    h = fnv1a64(header, h)
    h = fnv1a64(str(len(st)).encode(), h)
    h = fnv1a64(b'{"hidden_size": 2}', h)
    h = fnv1a64(b"LFM3Q8C1 v1 q8 block 32", h)
    assert k8 == f"{h:016x}"
    (d / "config.json").write_text('{"hidden_size": 3}')
    assert Q8Cache.key_for(str(d)) != k8


def test_written_cache_opens_with_every_matrix(cache_file):
    path, mats = cache_file
    cache = Q8Cache.open(path, "k123")
    assert cache is not None
    try:
        assert cache.shapes == [(n, m.rows, m.cols) for n, m in mats.items()]
        for name, m in mats.items():
            o = cache.offsets(name, m.rows, m.cols)
            assert o["format"] == m.format and o["qs"] % 64 == 0 and o["scales"] % 64 == 0
            assert o["qs"] >= HEADER_REGION
            got = cache.matrix(name, m.rows, m.cols)
            assert got.format == m.format
            assert np.array_equal(got.qs_bytes, m.qs_bytes)
            assert np.array_equal(got.scale_bytes, m.scale_bytes)
        assert cache.offsets("layers.0.q", 64, 64) is None   # another shape
        assert cache.matrix("missing", 1, 32) is None
    finally:
        cache.close()
    assert not MappedFile.is_mapped(path)


def test_misses(cache_file, tmp_path):
    path, _ = cache_file
    assert Q8Cache.open(path, "other key") is None
    assert not MappedFile.is_mapped(path)
    assert Q8Cache.open(str(tmp_path / "absent"), "k123") is None
    short = tmp_path / "short"
    short.write_bytes(b"LFM3Q8C1")
    assert Q8Cache.open(str(short), "k123") is None
    other = tmp_path / "other"
    other.write_bytes(b"NOTMAGIC" + bytes(64))
    assert Q8Cache.open(str(other), "k123") is None
    raw = bytearray(open(path, "rb").read())
    n = struct.unpack("<Q", raw[8:16])[0]
    header = json.loads(raw[16:16 + n])
    header["version"] = 2
    text = json.dumps(header, separators=(",", ":")).encode()
    old = tmp_path / "old"
    old.write_bytes(b"LFM3Q8C1" + struct.pack("<Q", len(text)) + text + bytes(raw[16 + len(text):]))
    assert Q8Cache.open(str(old), "k123") is None


def test_truncated_cache_throws_and_releases(cache_file):
    path, _ = cache_file
    raw = open(path, "rb").read()
    open(path, "wb").write(raw[:-1])
    with pytest.raises(FormatException):
        Q8Cache.open(path, "k123")
    assert not MappedFile.is_mapped(path)


def test_header_length_past_the_end_throws(cache_file):
    path, _ = cache_file
    raw = bytearray(open(path, "rb").read())
    raw[8:16] = struct.pack("<Q", len(raw))
    open(path, "wb").write(raw)
    with pytest.raises(FormatException):
        Q8Cache.open(path, "k123")
    assert not MappedFile.is_mapped(path)
    raw[8:16] = struct.pack("<Q", (1 << 64) - 1)  # above 2^63: negative in Dart
    open(path, "wb").write(raw)
    with pytest.raises(FormatException):
        Q8Cache.open(path, "k123")


def test_matrix_offset_outside_the_file_throws(cache_file):
    path, mats = cache_file
    cache = Q8Cache.open(path, "k123")
    name, rows, cols = cache.shapes[0]
    qs = cache.offsets(name, rows, cols)["qs"]
    cache.close()
    raw = bytearray(open(path, "rb").read())
    text = raw[16:16 + 4096].decode("latin-1")
    at = text.index(f'"qs":{qs}')
    raw[16 + at + len('"qs":')] = ord("9")  # a digit more moves it far past the end
    open(path, "wb").write(raw)
    with pytest.raises(FormatException):
        Q8Cache.open(path, "k123")
    assert not MappedFile.is_mapped(path)


@pytest.mark.parametrize("patch", [
    {"rows": 0}, {"cols": 48}, {"format": "q5"}, {"rows": 1.0}, {"scales": 2},
    {"rows": True}, {"qs": -64},
])
def test_entries_that_do_not_fit_throw(cache_file, tmp_path, patch):
    path, _ = cache_file
    raw = bytearray(open(path, "rb").read())
    n = struct.unpack("<Q", raw[8:16])[0]
    header = json.loads(raw[16:16 + n])
    header["tensors"]["layers.0.q"].update(patch)
    text = json.dumps(header, separators=(",", ":")).encode()
    bad = tmp_path / "bad"
    bad.write_bytes(b"LFM3Q8C1" + struct.pack("<Q", len(text)) + text + bytes(raw[16 + len(text):]))
    with pytest.raises(FormatException):
        Q8Cache.open(str(bad), "k123")
    assert not MappedFile.is_mapped(str(bad))


def test_opens_share_one_mapping(cache_file):
    path, _ = cache_file
    a = Q8Cache.open(path, "k123")
    b = Q8Cache.open(path, "k123")
    assert a.file is b.file
    a.close()
    assert MappedFile.is_mapped(path)
    b.close()
    assert not MappedFile.is_mapped(path)


def test_write_each_hands_back_every_matrix_and_checks_shapes(tmp_path):
    rng = np.random.default_rng(9)
    made, done = [], []

    def make(name):
        m = Arrays("q4", 32, 64, rng)
        made.append(name)
        return m

    path = str(tmp_path / "each")
    Q8Cache.write_each(path, "k", [("a", "q4", 32, 64), ("b", "q4", 32, 64)], make, done=done.append)
    assert made == ["a", "b"] and len(done) == 2
    assert not os.path.exists(path + ".partial")
    with pytest.raises(Exception):
        Q8Cache.write_each(str(tmp_path / "bad"), "k", [("a", "q8", 32, 64)], make)
    assert not os.path.exists(str(tmp_path / "bad"))
