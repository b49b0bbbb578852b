"""The byte-limb arithmetic of the batched decode attention on the tensor cores
(csrc/tc_attn_dec.cu), checked on the host with numpy.

Scores: with k_u = k + 2^31 and q_u = q + 2^31 as u32 (byte 3 of x + 2^31 is
byte 3 of x with its top bit flipped), the kernel forms
P_b[a] = sum_dim kbyte_b * qbyte_a (one unsigned int8 product per key limb b
and query limb a), the key's byte sums sum_dim kbyte_b (the all-ones operand
row), and recombines
    sum k q = sum_{a,b} 2^(8(a+b)) P_b[a] - 2^31 sum q_u - 2^31 sum k_u + 2^62 d
in wrapping 64-bit arithmetic.  Weighted values: with v_u = v + 2^31 and
weights w in [0, 2^16] (three byte limbs),
    sum_j w_j v_j = sum_{a<3,b} 2^(8(a+b)) D_b[a] - 2^31 sum_j w_j.
Both must equal the reference's wrapping i64 dot products exactly, and every
limb product sum must fit the signed 32-bit tensor-core accumulator at the
kernel's limits (head_dim 512, 1281 keys per CTA)."""
import numpy as np

M64 = (1 << 64) - 1


def limbs(x):
    """Byte limbs of x + 2^31 (x int32) as an [..., 4] uint8 array."""
    u = (x.astype(np.int64) + (1 << 31)).astype(np.uint32)
    return np.stack([(u >> (8 * b)) & 0xFF for b in range(4)], axis=-1).astype(np.int64)


def wrap_dot(a, b):
    """The reference's wrapping i64 dot product, as an unsigned 64-bit value."""
    return sum(int(x) * int(y) for x, y in zip(a, b)) & M64


def scores_via_limbs(k, q):
    d = k.shape[0]
    kb, qb = limbs(k), limbs(q)
    acc = 0
    for b in range(4):
        for a in range(4):
            p = int(np.dot(kb[:, b], qb[:, a]))
            assert p < (1 << 31)  # the s32 accumulator
            acc += p << (8 * (a + b))
    ksum = sum(int(kb[:, b].sum()) << (8 * b) for b in range(4))  # the ones row
    qsum = int((q.astype(np.int64) + (1 << 31)).sum())
    return (acc - (qsum << 31) - (ksum << 31) + (d << 62)) & M64


def values_via_limbs(w, v):
    vb = limbs(v)
    acc = 0
    for b in range(4):
        for a in range(3):
            wa = (w >> (8 * a)) & 0xFF
            dsum = int(np.dot(wa, vb[:, b]))
            assert dsum < (1 << 31)
            acc += dsum << (8 * (a + b))
    return (acc - (int(w.sum()) << 31)) & M64


def test_score_limb_identity_random_and_extremes():
    rng = np.random.default_rng(7)
    for d in (128, 256, 512):
        cases = [rng.integers(-(1 << 31), 1 << 31, size=(2, d), dtype=np.int64)]
        cases.append(np.full((2, d), -(1 << 31), dtype=np.int64))
        cases.append(np.full((2, d), (1 << 31) - 1, dtype=np.int64))
        mixed = np.where(rng.random((2, d)) < 0.5, -(1 << 31), (1 << 31) - 1)
        cases.append(mixed.astype(np.int64))
        for kq in cases:
            k, q = kq[0].astype(np.int32), kq[1].astype(np.int32)
            assert scores_via_limbs(k, q) == wrap_dot(k, q)


def test_value_limb_identity_random_and_extremes():
    rng = np.random.default_rng(11)
    for n in (1, 64, 1281):
        w = rng.integers(0, (1 << 16) + 1, size=n, dtype=np.int64)
        w[0] = 1 << 16
        v = rng.integers(-(1 << 31), 1 << 31, size=n, dtype=np.int64).astype(np.int32)
        assert values_via_limbs(w, v) == wrap_dot(w, v)
        v_min = np.full(n, -(1 << 31), dtype=np.int32)
        assert values_via_limbs(w, v_min) == wrap_dot(w, v_min)


def test_accumulator_bounds_at_the_kernel_limits():
    # the largest possible limb product sums fit the signed 32-bit accumulator
    assert 255 * 255 * 512 < (1 << 31)       # score products, head_dim 512
    assert 255 * 255 * 1281 < (1 << 31)      # weighted-value products, 1281 keys per CTA
    assert 255 * 512 < (1 << 31)             # the ones row
