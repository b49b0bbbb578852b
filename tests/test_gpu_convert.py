"""safetensors -> detwgt value conversion on the GPU (rdet_convert_to_wgt,
convert.py --device): the f32_to_wgt of det_num/convert.rs:77-93 against the
oracle's scalar restatement on seeded bit patterns and edges, row masses and
the i16 width test against the host form, and the whole conversion of the
tiny-gemma-dev source values (F32, BF16, F16) against the reference's shipped
model.detwgt, all bit-exact."""
import hashlib
import importlib
import os
import struct

import numpy as np
import pytest

import oracle as O  # checker only
import tiny_gemma_dev
from helpers import rdet
from test_convert import _records, _tiny_source

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

convert = importlib.import_module("raster-inference_b200.convert")
detwgt = importlib.import_module("raster-inference_b200.detwgt")


def gpu_convert(values: np.ndarray, dtype: str, shape):
    raw = {"F32": lambda v: v.astype("<f4").tobytes(), "F16": lambda v: v.astype("<f2").tobytes(),
           "BF16": lambda v: (v.astype(np.float32).view(np.uint32) >> 16).astype("<u2").tobytes()}[dtype](values)
    return convert.convert_tensor_gpu(memoryview(raw), dtype, shape, 0)


def test_f32_to_wgt_on_gpu_matches_oracle_and_host():
    rng = np.random.default_rng(12)
    raw = rng.integers(0, 2**32, 300_000, dtype=np.uint64).astype(np.uint32)
    near = (rng.integers(0x37000000, 0x47800000, 300_000, dtype=np.uint64).astype(np.uint32)
            | (rng.integers(0, 2, 300_000, dtype=np.uint64).astype(np.uint32) << 31))
    x = np.concatenate([raw, near]).view(np.float32)
    x = x[np.isfinite(x)]
    f32 = lambda u: struct.unpack("<f", struct.pack("<I", u))[0]
    step = 1.0 / 65536.0
    edges = np.array([32768.0, 32767.998046875, 65536.0, 1e30, f32(0x7F7FFFFF), f32(0x00000001), f32(0x00800000),
                      0.5 * step, 1.5 * step, 2.5 * step, 32767.5, 16383.25, 1.0 + step / 2, -0.0, 40000.0],
                     dtype=np.float32)
    x = np.concatenate([edges, -edges, x[: 600_000 - 2 * edges.size]])
    x = x[: x.size // 1000 * 1000]
    bits, mass = gpu_convert(x, "F32", (x.size // 1000, 1000))
    host_bits, host_mass = convert.convert_tensor(memoryview(x.astype("<f4").tobytes()), "F32",
                                                  (x.size // 1000, 1000))
    assert np.array_equal(bits, host_bits) and np.array_equal(mass, host_mass)
    L = O.lib()
    k = 2 * edges.size + 20_000
    assert [int(b) for b in bits[:k]] == [L.dor_f32_to_act(float(v)) for v in x[:k]]


@pytest.mark.parametrize("dtype", ["BF16", "F16"])
def test_half_width_sources_match_host(dtype):
    rng = np.random.default_rng(13 if dtype == "BF16" else 14)
    w = rng.normal(0, 0.05, (2560, 1536)).astype(np.float32)
    w[7, :5] = [1e4, -1e4, 0.5, -0.25, 3.0]  # a row past the i16 range
    bits, mass = gpu_convert(w, dtype, w.shape)
    raw = {"F16": w.astype("<f2").tobytes(), "BF16": (w.view(np.uint32) >> 16).astype("<u2").tobytes()}[dtype]
    hb, hm = convert.convert_tensor(memoryview(raw), dtype, w.shape)
    assert np.array_equal(bits, hb) and np.array_equal(mass, hm)


def test_non_finite_values_are_rejected_on_gpu():
    for bad in (np.nan, np.inf, -np.inf):
        with pytest.raises(ValueError, match="finite"):
            gpu_convert(np.array([1.0, bad, 2.0, 3.0], dtype=np.float32), "F32", (4,))


@pytest.mark.parametrize("dtype", ["F32", "BF16", "F16"])
def test_tiny_gemma_dev_converts_on_gpu_to_the_reference_artifact(dtype, tmp_path):
    src = tmp_path / "src"
    src.mkdir()
    tiny_gemma_dev.write_bundle(str(src), detwgt.encode)
    os.remove(src / "model.detwgt")
    convert.write_safetensors(str(src / "model.safetensors"), _tiny_source(dtype))
    s = convert.convert(str(src), str(tmp_path / "out"), device=0)
    blob = (tmp_path / "out" / "model.detwgt").read_bytes()
    ref = detwgt.encode(tiny_gemma_dev.tensors())
    assert hashlib.sha256(ref).hexdigest() == tiny_gemma_dev.reference_record()["model_detwgt_sha256"]
    got, order = _records(blob)
    want, _ = _records(ref)
    assert order == sorted(order) and got == want
    assert s["tensor_count"] == len(want)
    # the converted artifact loads and runs
    m = rdet.Model.open(str(tmp_path / "out"), max_prefill=16)
    q = m.new_sequence(24)
    q.prefill(tiny_gemma_dev.lcg_token_ids(16, 280, 0))
    assert len(q.generate(4)) == 4
    m.close()


def test_row_mass_bound_on_gpu(tmp_path):
    big = np.full((2, 4), 20000.0, dtype=np.float32)
    big[0] = 0.5
    src = tmp_path / "m.safetensors"
    (tmp_path / "config.json").write_text("{}")
    convert.write_safetensors(str(src), [("w", "F32", (2, 4), big.tobytes())])
    with pytest.raises(ValueError, match="row 1 has row mass"):
        convert.convert(str(src), str(tmp_path / "out"), device=0)
