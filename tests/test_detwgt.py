"""detwgt v2 encoder/reader and the fail-closed loader checks of
src/shared/model/gemma/io.rs:230-395, on the oracle's reader and on the
product loader (rdet_open validates every byte on the host before touching
the GPU, so these run without one).  CPU only."""
import ctypes as C
import os
import struct
import tempfile

import numpy as np
import pytest

import oracle as O
from helpers import detwgt, mini_config, rdet

GOOD = [("a.weight", (3, 8), np.arange(24, dtype=np.int32) - 12),
        ("b.weight", (4,), np.array([65536, 1 << 20, -5, 7], dtype=np.int32))]


def _mutate(buf: bytes, off: int, data: bytes) -> bytes:
    return buf[:off] + data + buf[off + len(data):]


def corrupt_cases():
    good = detwgt.encode(GOOD)
    cases = {
        "magic": _mutate(good, 0, b"XNWGTV0\0"),
        "version": _mutate(good, 8, struct.pack("<I", 1)),
        "spec": _mutate(good, 12, struct.pack("<I", 2)),
        "truncated": good[:-3],
        "trailing": good + b"\0",
    }
    # first tensor header: name_len(4) name(8) rank(4) dims(16) count(8) width(4) payload_len(8) mass(8)
    o = 24 + 4 + len("a.weight") + 4
    cases["count"] = _mutate(good, o + 16, struct.pack("<Q", 25))
    cases["width"] = _mutate(good, o + 24, struct.pack("<I", 8))
    cases["payload_len"] = _mutate(good, o + 28, struct.pack("<Q", 47))
    cases["row_mass"] = _mutate(good, o + 36, struct.pack("<Q", 1 << 31))
    pad_at = o + 44
    cases["padding"] = _mutate(good, pad_at, b"\x01")
    dup = [GOOD[0], GOOD[0]]
    cases["duplicate"] = detwgt.encode(dup)
    return good, cases


def test_encoder_roundtrip_and_widths():
    good, _ = corrupt_cases()
    assert O.validate_detwgt(good) == 2
    # a: fits i16 -> 16-bit payload; b: does not -> 32-bit
    o = 24 + 4 + 8 + 4 + 16 + 8
    assert struct.unpack_from("<I", good, o)[0] == 16


@pytest.mark.parametrize("case", ["magic", "version", "spec", "truncated", "trailing", "count", "width",
                                  "payload_len", "row_mass", "padding", "duplicate"])
def test_oracle_reader_fails_closed(case):
    _, cases = corrupt_cases()
    with pytest.raises(O.OracleError):
        O.validate_detwgt(cases[case])


@pytest.mark.parametrize("case", ["magic", "version", "spec", "truncated", "trailing", "count", "width",
                                  "payload_len", "row_mass", "padding", "duplicate"])
def test_product_loader_fails_closed(case):
    _, cases = corrupt_cases()
    d = tempfile.mkdtemp()
    detwgt.write_synthetic_model(d, mini_config(num_hidden_layers=1, layer_types=["sliding_attention"],
                                                num_kv_shared_layers=0), 1)
    with open(os.path.join(d, "model.detwgt"), "wb") as f:
        f.write(cases[case])
    with pytest.raises(rdet.RdetError) as e:
        rdet.Model.open(d)
    assert e.value.code == -3, e.value.msg


def test_product_loader_missing_tensor_is_format_error():
    d = tempfile.mkdtemp()
    cfg = mini_config(num_hidden_layers=1, layer_types=["sliding_attention"], num_kv_shared_layers=0)
    detwgt.write_synthetic_model(d, cfg, 1)
    with open(os.path.join(d, "model.detwgt"), "wb") as f:
        f.write(detwgt.encode(GOOD))
    with pytest.raises(rdet.RdetError) as e:
        rdet.Model.open(d)
    assert e.value.code == -3 and ("failed to load tensor" in e.value.msg or "embedding tensor" in e.value.msg)


def test_product_config_validation():
    bad = mini_config(hidden_activation="relu")
    with pytest.raises(rdet.RdetError) as e:
        rdet.Model.synthetic(bad, 1)
    assert e.value.code == -3 and "gelu_pytorch_tanh" in e.value.msg
    bad = mini_config(num_hidden_layers=5)
    with pytest.raises(rdet.RdetError) as e:
        rdet.Model.synthetic(bad, 1)
    assert "layer count mismatch" in e.value.msg


def test_benchmark_activations_follow_f32_to_act():
    """The GEMV microbenchmark's N(0,1) activations are quantized exactly as
    the oracle's f32_to_act (det_num/convert.rs:52-57) quantizes them."""
    import oracle as O
    z = detwgt.normal_f32(3001, 9)
    x = detwgt.normal_acts(3001, 9)
    assert x.dtype == np.int32 and x.size == 3001
    assert abs(float(z.mean())) < 0.1 and 0.9 < float(z.std()) < 1.1
    assert all(int(x[i]) == O.lib().dor_f32_to_act(float(z[i])) for i in range(x.size))
    # halfway and saturating inputs
    edge = np.array([0.5 / 65536, 1.5 / 65536, -2.5 / 65536, 40000.0, -40000.0, 3.0e38], dtype=np.float32)
    assert [int(v) for v in detwgt.f32_to_act(edge)] == [O.lib().dor_f32_to_act(float(v)) for v in edge]


def test_lcg_token_ids_match_fixture_generator():
    from tiny_gemma_dev import lcg_token_ids
    assert detwgt.lcg_token_ids(50, 280, 0) == lcg_token_ids(50, 280, 0)
