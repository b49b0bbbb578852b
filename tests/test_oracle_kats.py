"""Oracle vs the reference's det_num known-answer vectors
(casettek/raster-inference src/shared/numerics/det_num/tests.rs).  CPU only."""
import numpy as np

import oracle as O

L = O.lib()
I32_MAX, I32_MIN = 2**31 - 1, -2**31
I64_MAX, I64_MIN = 2**63 - 1, -2**63


def q16(x):
    return int(round(x * 65536))


def test_mac_and_combine():  # tests.rs:29-292
    assert L.dor_mac_bits(10, 3, 4) == 22
    assert L.dor_mac_bits(I64_MAX - 3, 2, 2) == I64_MIN
    assert L.dor_mac_bits(I64_MIN + 3, -2, 2) == I64_MAX
    assert L.dor_mac_bits(I64_MAX, 1 << 16, 1 << 16) == I64_MIN + (1 << 32) - 1
    assert L.dor_mac_bits(-(1 << 40), 1 << 20, 1 << 21) == (1 << 41) - (1 << 40)
    assert L.dor_mac_bits(0, I32_MIN, I32_MIN) == 1 << 62
    assert L.dor_mac_bits(1 << 62, I32_MIN, I32_MIN) == I64_MIN
    assert L.dor_mac_bits(0, 98304, 131072) == 12884901888
    assert L.dor_acc_combine(I64_MAX, 1) == I64_MIN
    assert L.dor_acc_combine(I64_MIN, -1) == I64_MAX
    assert L.dor_acc_combine(I64_MIN, I64_MIN) == 0


def test_mac_schedule_independence():  # tests.rs:330-397
    rng = np.random.default_rng(5)
    for n in [1, 2, 3, 7, 16, 33, 100]:
        a = rng.integers(I32_MIN, I32_MAX, n, dtype=np.int64)
        b = rng.integers(I32_MIN, I32_MAX, n, dtype=np.int64)
        fwd = 0
        for x, y in zip(a, b):
            fwd = L.dor_mac_bits(fwd, int(x), int(y))
        rev = 0
        for x, y in zip(a[::-1], b[::-1]):
            rev = L.dor_mac_bits(rev, int(x), int(y))
        assert fwd == rev


def test_saturating_and_mul():  # tests.rs:485-579, :1129-1213
    assert L.dor_add_sat(7, 9) == 16
    assert L.dor_add_sat(I32_MAX - 1, 1) == I32_MAX
    assert L.dor_add_sat(I32_MAX, 1) == I32_MAX
    assert L.dor_add_sat(I32_MIN, -1) == I32_MIN
    assert L.dor_sub_sat(20, 3) == 17
    assert L.dor_sub_sat(I32_MIN + 1, 1) == I32_MIN
    assert L.dor_sub_sat(I32_MIN, 1) == I32_MIN
    assert L.dor_sub_sat(I32_MAX, -1) == I32_MAX
    assert L.dor_acc_add_sat(7, 9) == 16
    assert L.dor_acc_add_sat(I64_MAX, 1) == I64_MAX
    assert L.dor_acc_add_sat(I64_MIN, -1) == I64_MIN
    assert L.dor_mul_sat(q16(1.5), q16(2.0)) == q16(3.0)
    assert L.dor_mul_sat(1, 0x8000) == 0
    assert L.dor_mul_sat(3, 0x8000) == 2
    assert L.dor_mul_sat(I32_MAX, I32_MAX) == I32_MAX
    assert L.dor_mul_sat(I32_MIN, I32_MAX) == I32_MIN
    assert L.dor_mul_sat(q16(3.0), q16(0.5)) == q16(1.5)


def test_div():  # tests.rs:588-687
    assert L.dor_div_act(q16(3.0), q16(2.0)) == q16(1.5)
    assert L.dor_div_act(1, q16(2.0)) == 0
    assert L.dor_div_act(-3, q16(2.0)) == -2
    for v, d, e in [(8, 4, 2), (3, 2, 2), (7, 4, 2), (-3, 2, -2), (-5, 4, -1)]:
        assert L.dor_div_acc_by_u32(v, d) == e


def test_norms():  # tests.rs:688-789
    def scale(xs, eps):
        a = np.array(xs, dtype=np.int32)
        return L.dor_rms_norm_scale(O._ptr(a), a.size, eps)
    assert scale([65536], 0) == 65536
    assert scale([65536, 0], 0) == 92682
    assert scale([0], 1 << 32) == 65536
    x = np.array([65536, 0], dtype=np.int32)
    w = np.array([32768, 65536], dtype=np.int32)
    L.dor_rms_norm(O._ptr(x), O._ptr(w), 2, 0)
    assert x.tolist() == [46341, 0]
    x = np.array([65536, -65536], dtype=np.int32)
    w = np.array([65536, 65536], dtype=np.int32)
    L.dor_rms_norm(O._ptr(x), O._ptr(w), 2, 0)
    assert x.tolist() == [65536, -65536]
    x = np.array([65536, 0], dtype=np.int32)
    L.dor_value_rms_norm(O._ptr(x), 2, 0)
    assert x.tolist() == [92682, 0]
    x = np.array([0], dtype=np.int32)
    L.dor_value_rms_norm(O._ptr(x), 1, 1 << 32)
    assert x.tolist() == [0]


def softmax(xs):
    a = np.array(xs, dtype=np.int32)
    w = np.zeros_like(a)
    L.dor_softmax(O._ptr(a), a.size, O._ptr(w))
    return w.tolist()


def test_attention():  # tests.rs:790-898
    q = np.array([q16(1.0), q16(-0.5)], dtype=np.int32)
    k = np.array([q16(0.5), q16(0.25)], dtype=np.int32)
    assert L.dor_attention_score(O._ptr(q), O._ptr(k), 2) == q16(0.375)
    assert softmax([0, 0]) == [32768, 32768]
    assert softmax([0, -45426]) == [43695, 21841]
    assert softmax([0, 0, 0]) == [21846, 21845, 21845]
    w = np.array([q16(0.5), q16(0.5)], dtype=np.int32)
    v = np.array([q16(1.0), 0, 0, q16(1.0)], dtype=np.int32)
    out = np.zeros(2, dtype=np.int32)
    L.dor_weighted_sum(O._ptr(w), 2, O._ptr(v), 2, O._ptr(out))
    assert out.tolist() == [32768, 32768]
    w = np.array([q16(1.0), q16(1.0)], dtype=np.int32)
    v = np.array([I32_MAX, I32_MAX], dtype=np.int32)
    out = np.zeros(1, dtype=np.int32)
    L.dor_weighted_sum(O._ptr(w), 2, O._ptr(v), 1, O._ptr(out))
    assert out.tolist() == [I32_MAX]


def test_tanh_softcap_gelu():  # tests.rs:899-1061
    for x, e in [(0, 0), (1, 1), (q16(0.5), 30527), (q16(-0.5), -30527), (q16(3.0), q16(1.0)), (q16(-3.0), q16(-1.0))]:
        assert L.dor_tanh(x) == e
    assert L.dor_softcap(0, q16(0.5)) == 0
    assert L.dor_softcap(q16(0.5), q16(1.0)) == 30527
    assert L.dor_softcap(q16(-0.5), q16(1.0)) == -30527
    assert L.dor_softcap(q16(3.0), q16(0.5)) == q16(0.5)
    for x, e in [(0, 0), (1, 0), (q16(0.5), 22691), (q16(-0.5), -10077), (q16(2.0), 129512), (q16(-2.0), -1560), (3, 2)]:
        assert L.dor_gelu(x) == e


def test_rope():  # tests.rs:1062-1128
    v = np.array([q16(1.0), 0, q16(0.5), q16(-0.5)], dtype=np.int32)
    L.dor_rope(O._ptr(v), 4, 4, 16 << 32, 1)
    assert v.tolist() == [7835, 8107, 72850, -31750]
    v = np.array([q16(1.0), q16(0.25), q16(0.5), q16(-0.25), q16(3.0)], dtype=np.int32)
    before = v.copy()
    L.dor_rope(O._ptr(v), 4, 4, 16 << 32, 0)
    assert v.tolist() == before.tolist()
    v = np.array([q16(1.0), 0, q16(0.5), q16(-0.5), q16(3.0)], dtype=np.int32)
    L.dor_rope(O._ptr(v), 4, 4, 1000000 << 32, 4096)
    assert v[4] == q16(3.0) and v[1] != 0


def test_requantize_rshift():  # tests.rs:1215-1430
    S = 16
    cases = [(0, 0), ((2 << S) + 0x7fff, 2), ((2 << S) + 0x8000, 2), ((3 << S) + 0x8000, 4), ((2 << S) + 0x8001, 3),
             (-((2 << S) + 0x7fff), -2), (-((2 << S) + 0x8000), -2), (-((3 << S) + 0x8000), -4), (-0x8000, 0),
             (I32_MAX << S, I32_MAX), (I32_MIN << S, I32_MIN), ((I32_MAX + 1) << S, I32_MAX),
             ((I32_MIN - 1) << S, I32_MIN), (I64_MAX, I32_MAX), (I64_MIN, I32_MIN)]
    for a, e in cases:
        assert L.dor_requantize(a) == e, a
    for b, s, e in [(42, 0, 42), (8, 2, 2), (9, 2, 2), (10, 2, 2), (14, 2, 4), (11, 2, 3), (-8, 2, -2), (-9, 2, -2),
                    (-10, 2, -2), (-14, 2, -4), (-1, 1, 0), (1, 63, 0), (I64_MIN, 63, -1)]:
        assert L.dor_rshift_rte(b, s) == e


def test_argmax_first():  # tests.rs:1431-1448
    assert O.argmax_first([4, 9, 3]) == 1
    assert O.argmax_first([4, 9, 9, 3]) == 1
    assert O.argmax_first([7, 7, 7]) == 0
    assert O.argmax_first([-123]) == 0


def test_f32_conversions():  # tests.rs:1551-1696
    step16, step32 = 1.0 / 65536.0, 1.0 / 4294967296.0
    import struct
    sub = struct.unpack("<f", struct.pack("<I", 0x007FFFFF))[0]
    for v, e in [(0.0, 0), (1.5, 98304), (0.5 * step16, 0), (2.5 * step16, 2), (3.5 * step16, 4), (-3.5 * step16, -4),
                 (sub, 0), (40000.0, I32_MAX), (-40000.0, I32_MIN)]:
        assert L.dor_f32_to_act(v) == e
    for v, e in [(0.0, 0), (1.5, 6442450944), (0.5 * step32, 0), (2.5 * step32, 2), (3.5 * step32, 4),
                 (0.000001, 4295), (3e9, I64_MAX), (-3e9, I64_MIN)]:
        assert L.dor_f32_to_acc(v) == e
