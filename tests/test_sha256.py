"""The commitment hash (raster-inference_b200/csrc/sha256.cpp) against
Python's hashlib (CPU).

Every det commitment is a SHA-256 over canonical bytes (transformer_kernels.rs
:1395-1482 in the reference), so both block-compression implementations (the
x86 SHA extensions and the portable loop) and the streaming layer above them
(partial blocks, whole blocks taken straight from the caller, padding) must
give hashlib's digest for every length and every way the bytes arrive."""
import ctypes
import hashlib
import os
import struct
import subprocess

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "..", "raster-inference_b200", "csrc")
SRC = os.path.join(HERE, "sha256_host.cpp")
OUT = os.path.join(HERE, "_build", "libsha256_host.so")
DEPS = [SRC, os.path.join(CSRC, "sha256.cpp"), os.path.join(CSRC, "sha256.h")]


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(OUT) or any(os.path.getmtime(d) > os.path.getmtime(OUT) for d in DEPS):
        os.makedirs(os.path.dirname(OUT), exist_ok=True)
        subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-I" + CSRC, "-o", OUT, SRC], check=True)
    L = ctypes.CDLL(OUT)
    L.rdet_test_sha_stream.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_size_t,
                                       ctypes.c_char_p]
    L.rdet_test_compress.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    return L


def stream_hex(lib, data, seed, max_piece):
    out = ctypes.create_string_buffer(65)
    lib.rdet_test_sha_stream(data, len(data), seed, max_piece, out)
    return out.value.decode()


def padded(data):
    """FIPS 180-4 padding to whole 64-byte blocks."""
    tail = b"\x80" + b"\x00" * ((55 - len(data)) % 64) + struct.pack(">Q", 8 * len(data))
    return data + tail


IV = [0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19]


def compress_hex(lib, impl, data):
    st = (ctypes.c_uint32 * 8)(*IV)
    msg = padded(data)
    rc = lib.rdet_test_compress(impl, st, msg, len(msg) // 64)
    if rc != 0:
        return None
    return b"".join(struct.pack(">I", v) for v in st).hex()


def test_every_length_through_both_block_implementations(lib):
    rng = np.random.default_rng(7)
    have_ext = lib.rdet_test_sha_has_ext() == 1
    for n in list(range(0, 300)) + [1000, 4095, 4096, 4097, 65536 + 13]:
        data = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        want = hashlib.sha256(data).hexdigest()
        assert compress_hex(lib, 0, data) == want, n
        got = compress_hex(lib, 1, data)
        assert got == (want if have_ext else None), n


@pytest.mark.parametrize("max_piece", [0, 1, 7, 8, 63, 64, 65, 200, 5000])
def test_streaming_splits(lib, max_piece):
    rng = np.random.default_rng(max_piece + 1)
    for n in (0, 1, 55, 56, 63, 64, 65, 127, 128, 129, 1000, 10247, 100003):
        data = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert stream_hex(lib, data, 11 + n, max_piece) == hashlib.sha256(data).hexdigest(), (n, max_piece)


def test_canonical_rows_commitment_shape(lib):
    # the act commitment layout (domain tag, row count, then each row as its
    # length and little-endian i32 values) hashed in the pieces the runtime
    # feeds it
    rng = np.random.default_rng(3)
    rows, cols = 37, 2560
    a = rng.integers(-2**31, 2**31, (rows, cols), dtype=np.int64).astype(np.int32)
    msg = b"raster-det-num-act-v1" + struct.pack("<Q", rows)
    for r in a:
        msg += struct.pack("<Q", cols) + r.astype("<i4").tobytes()
    assert stream_hex(lib, msg, 5, 8 + 4 * cols) == hashlib.sha256(msg).hexdigest()


def test_dispatch_uses_the_extensions_when_present(lib):
    assert lib.rdet_test_sha_impl() == lib.rdet_test_sha_has_ext()
