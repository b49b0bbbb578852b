"""safetensors -> detwgt converter (raster-inference_b200/convert.py) on the
CPU: the f32 -> Q16.16 conversion against the reference's golden vectors
(det_num/tests.rs:1551-1611) and the oracle's scalar restatement on seeded
bit patterns, and the whole conversion of the tiny-gemma-dev source values
against the reference's shipped model.detwgt (its SHA-256 is pinned in
tests/golden/tiny_gemma_dev_reference.json)."""
import hashlib
import importlib
import os
import struct

import numpy as np
import pytest

import oracle as O
import tiny_gemma_dev

convert = importlib.import_module("raster-inference_b200.convert")
detwgt = importlib.import_module("raster-inference_b200.detwgt")

STEP = 1.0 / 65536.0
SUBNORMAL_MAX = struct.unpack("<f", struct.pack("<I", 0x007FFFFF))[0]


def test_f32_to_wgt_golden_vectors():
    cases = [(0.0, 0), (1.5, 98304), (0.5 * STEP, 0), (2.5 * STEP, 2), (3.5 * STEP, 4), (-3.5 * STEP, -4),
             (SUBNORMAL_MAX, 0), (40000.0, 2**31 - 1), (-40000.0, -2**31)]
    got = convert.f32_to_wgt_bits(np.array([c[0] for c in cases], dtype=np.float32))
    assert got.tolist() == [c[1] for c in cases]


def test_f32_to_wgt_matches_the_oracle_on_seeded_bit_patterns():
    rng = np.random.default_rng(11)
    raw = rng.integers(0, 2**32, 200_000, dtype=np.uint64).astype(np.uint32)
    # bias toward the interesting range: exponents around 2^-17 .. 2^16
    near = (rng.integers(0x37000000, 0x47800000, 100_000, dtype=np.uint64).astype(np.uint32)
            | (rng.integers(0, 2, 100_000, dtype=np.uint64).astype(np.uint32) << 31))
    bits = np.concatenate([raw, near])
    x = bits.view(np.float32)
    x = x[np.isfinite(x)]
    got = convert.f32_to_wgt_bits(x)
    L = O.lib()
    want = np.array([L.dor_f32_to_act(float(v)) for v in x[:60_000]], dtype=np.int64)
    assert np.array_equal(got[:60_000].astype(np.int64), want)


def test_f32_to_wgt_edges_match_the_oracle():
    f32 = lambda u: struct.unpack("<f", struct.pack("<I", u))[0]
    edges = [32768.0, 32767.998046875, 65536.0, 1e30, f32(0x7F7FFFFF), f32(0x00000001), f32(0x00800000),
             0.5 * STEP, 1.5 * STEP, 32767.5, 16383.25, 1.0 + STEP / 2, -0.0]
    x = np.array(edges + [-e for e in edges], dtype=np.float32)
    L = O.lib()
    assert convert.f32_to_wgt_bits(x).tolist() == [L.dor_f32_to_act(float(v)) for v in x]


def test_non_finite_values_are_rejected():
    for bad in (np.nan, np.inf, -np.inf):
        with pytest.raises(ValueError, match="finite"):
            convert.f32_to_wgt_bits(np.array([1.0, bad], dtype=np.float32))


def _records(blob: bytes):
    """name -> (shape, width, payload length, max row mass, payload) of a
    detwgt v2 artifact, plus the names in file order."""
    assert blob[:8] == detwgt.MAGIC
    (count,) = struct.unpack_from("<Q", blob, 16)
    off, out, order = 24, {}, []
    for _ in range(count):
        (nl,) = struct.unpack_from("<I", blob, off)
        name = blob[off + 4:off + 4 + nl].decode()
        off += 4 + nl
        (rank,) = struct.unpack_from("<I", blob, off)
        shape = struct.unpack_from("<" + "Q" * rank, blob, off + 4)
        off += 4 + 8 * rank
        n, width, plen, mass = struct.unpack_from("<QIQQ", blob, off)
        off += 28
        off += (detwgt.ALIGN - off % detwgt.ALIGN) % detwgt.ALIGN
        out[name] = (shape, width, plen, mass, blob[off:off + plen])
        order.append(name)
        off += plen
    assert off == len(blob)
    return out, order


def _tiny_source(dtype="F32"):
    """The tiny-gemma-dev source tensors as safetensors entries: the recipe's
    Q16.16 values / 65536 (every one a multiple of 1/8, exact in F32, BF16
    and F16)."""
    out = []
    for name, shape, bits in tiny_gemma_dev.tensors():
        x = (np.asarray(bits, dtype=np.float64) / 65536.0).astype(np.float32)
        if dtype == "F32":
            data = x.astype("<f4").tobytes()
        elif dtype == "F16":
            data = x.astype("<f2").tobytes()
        else:
            data = (x.view(np.uint32) >> 16).astype("<u2").tobytes()
        out.append((name, dtype, shape, data))
    return out


@pytest.mark.parametrize("dtype", ["F32", "BF16", "F16"])
def test_tiny_gemma_dev_converts_to_the_reference_artifact(dtype, tmp_path):
    src = tmp_path / "src"
    src.mkdir()
    tiny_gemma_dev.write_bundle(str(src), detwgt.encode)  # config.json (and the recipe's own artifact)
    os.remove(src / "model.detwgt")
    convert.write_safetensors(str(src / "model.safetensors"), _tiny_source(dtype))
    s = convert.convert(str(src), str(tmp_path / "out"))
    blob = (tmp_path / "out" / "model.detwgt").read_bytes()
    # the converter writes sorted names; the recipe's artifact (byte-identical
    # to the reference's shipped model.detwgt) holds the same records
    ref = detwgt.encode(tiny_gemma_dev.tensors())
    assert hashlib.sha256(ref).hexdigest() == tiny_gemma_dev.reference_record()["model_detwgt_sha256"]
    got, order = _records(blob)
    want, _ = _records(ref)
    assert order == sorted(order) and got == want
    assert blob == detwgt.encode(sorted(tiny_gemma_dev.tensors(), key=lambda t: t[0]))
    assert s["tensor_count"] == len(want)
    assert (tmp_path / "out" / "config.json").read_bytes() == (src / "config.json").read_bytes()


def test_row_mass_bound(tmp_path):
    big = np.full((2, 4), 20000.0, dtype=np.float32)  # 4 * 20000 * 65536 > 2^31 per row
    big[0] = 0.5
    src = tmp_path / "m.safetensors"
    (tmp_path / "config.json").write_text("{}")
    convert.write_safetensors(str(src), [("w", "F32", (2, 4), big.tobytes())])
    with pytest.raises(ValueError, match="row 1 has row mass"):
        convert.convert(str(src), str(tmp_path / "out"))
    # rank-1 tensors record their mass but are not bound
    convert.write_safetensors(str(src), [("g", "F32", (8,), np.full(8, 20000.0, dtype=np.float32).tobytes())])
    s = convert.convert(str(src), str(tmp_path / "out2"))
    assert s["tensor_bounds"][0]["max_row_mass"] == 8 * 20000 * 65536 and s["tensor_bounds"][0]["width"] == 32


def test_source_and_output_checks(tmp_path):
    (tmp_path / "a").mkdir()
    with pytest.raises(ValueError, match="missing config.json"):
        convert.convert(str(tmp_path / "a"), str(tmp_path / "o"))
    (tmp_path / "a" / "config.json").write_text("{}")
    with pytest.raises(ValueError, match="missing `model.safetensors`"):
        convert.convert(str(tmp_path / "a"), str(tmp_path / "o"))
    convert.write_safetensors(str(tmp_path / "a" / "model.safetensors"), [("g", "F32", (1,), b"\0\0\0\0")])
    (tmp_path / "busy").mkdir()
    (tmp_path / "busy" / "x").write_text("")
    with pytest.raises(ValueError, match="must not already contain files"):
        convert.convert(str(tmp_path / "a"), str(tmp_path / "busy"))
    with pytest.raises(ValueError, match="unsupported input path"):
        convert.convert(str(tmp_path / "a" / "config.json"), str(tmp_path / "o2"))
    assert convert.main(["--input", str(tmp_path / "a"), "--output-dir", str(tmp_path / "o3"),
                         "--report-bounds", "--report-widths"]) == 0
