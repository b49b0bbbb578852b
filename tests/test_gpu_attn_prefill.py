"""Prefill attention (det_attention_prefill, det_kernels.rs:525-671) on the
tcgen05 tensor cores and on the CUDA cores, against the oracle's
attention_output_into for every (query, head), bit-exact, through the C ABI
(rdet_det_attention_prefill) on device buffers; then whole-model prefills of
4096 tokens at the E4B head geometry (head_dim 256 sliding with window 512,
512 full) against the oracle's per-layer commitments."""
import numpy as np
import pytest

import oracle as O  # checker only
from helpers import lcg_ids, mini_config, rdet, write_model

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

I32_MIN, I32_MAX = -2**31, 2**31 - 1


def oracle_prefill(q, k, v, S, Hq, Hkv, window):
    G = Hq // Hkv
    out = np.zeros_like(q[:S])
    for i in range(S):
        st = max(0, i + 1 - window) if window else 0
        for h in range(Hq):
            out[i, h] = O.attention_one(q[i, h], k[h // G, st:i + 1], v[h // G, st:i + 1])
    return out


def make_inputs(rng, S, cap, Hq, Hkv, d, kind):
    if kind == "normal":  # magnitudes of normed, rotated queries and keys
        q = rng.normal(0, 65536 * 2, (S, Hq, d))
        k = rng.normal(0, 65536 * 2, (Hkv, cap, d))
        v = rng.normal(0, 65536 * 4, (Hkv, cap, d))
        return [np.clip(x, I32_MIN, I32_MAX).astype(np.int32) for x in (q, k, v)]
    if kind == "full_range":  # every limb in use; scores saturate and tie at the i32 limits
        return [rng.integers(I32_MIN, I32_MAX, shape, dtype=np.int64, endpoint=True).astype(np.int32)
                for shape in ((S, Hq, d), (Hkv, cap, d), (Hkv, cap, d))]
    if kind == "saturated_low":  # every score saturates at INT32_MIN: the first key of each window is the max
        q = np.full((S, Hq, d), I32_MAX, dtype=np.int32)
        k = np.full((Hkv, cap, d), I32_MIN, dtype=np.int32)
        v = rng.integers(I32_MIN, I32_MAX, (Hkv, cap, d), dtype=np.int64).astype(np.int32)
        return q, k, v
    if kind == "ties":  # equal scores everywhere: the residual goes to the first key of each window
        q = np.zeros((S, Hq, d), dtype=np.int32)
        k = np.ones((Hkv, cap, d), dtype=np.int32)
        v = rng.integers(I32_MIN, I32_MAX, (Hkv, cap, d), dtype=np.int64).astype(np.int32)
        return q, k, v
    raise ValueError(kind)


CASES = [
    # Hq, Hkv, d, S, window, kind
    (8, 2, 256, 300, 0, "normal"),
    (8, 2, 512, 300, 0, "normal"),
    (8, 2, 256, 700, 128, "normal"),
    (8, 2, 512, 333, 0, "full_range"),
    (8, 2, 256, 200, 40, "full_range"),
    (4, 4, 64, 130, 0, "normal"),      # one query head per KV head: 128 queries per tile
    (8, 1, 128, 257, 50, "normal"),    # eight query heads per KV head: 16 queries per tile
    (16, 1, 64, 100, 0, "full_range"),
    (4, 2, 64, 1, 0, "normal"),        # a one-token prompt
    (2, 1, 192, 65, 0, "ties"),
    (8, 2, 256, 190, 64, "ties"),
    (8, 2, 256, 150, 0, "saturated_low"),
    (4, 1, 64, 77, 20, "saturated_low"),
]


@pytest.mark.parametrize("Hq,Hkv,d,S,window,kind", CASES)
def test_prefill_attention_bit_exact(Hq, Hkv, d, S, window, kind):
    rng = np.random.default_rng(S * 31 + d + Hq)
    cap = S + 7
    q, k, v = make_inputs(rng, S, cap, Hq, Hkv, d, kind)
    ref = oracle_prefill(q, k, v, S, Hq, Hkv, window)
    qd, kd, vd = (torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (q, k, v))
    for tc in (True, False):
        out = torch.full((S, Hq, d), 7, dtype=torch.int32, device="cuda")
        rdet.det_attention_prefill(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), cap, S, Hq, Hkv, d, window,
                                   out.data_ptr(), tensor_cores=tc)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        bad = np.argwhere(got != ref)
        assert bad.size == 0, f"tensor_cores={tc}: {len(bad)} differences, first at {bad[0].tolist()}"


def e4b_heads_config(layers):
    return mini_config(hidden_size=128, intermediate_size=256, num_attention_heads=8, num_key_value_heads=2,
                       head_dim=256, global_head_dim=512, sliding_window=512, hidden_size_per_layer_input=16,
                       num_hidden_layers=len(layers), num_kv_shared_layers=0, vocab_size=300, layer_types=layers)


def test_prefill_4096_tokens_e4b_heads_against_oracle():
    """A 4096-token prompt through a sliding (head_dim 256, window 512) and a
    full (head_dim 512) layer: every layer output, the final hidden states,
    the logits and the KV caches equal the oracle's, and the tensor-core and
    CUDA-core contexts agree."""
    cfg = e4b_heads_config(["sliding_attention", "full_attention"])
    d = write_model(cfg, seed=17)
    ids = lcg_ids(4096, 300, 5)
    om = O.Model(d, threads=O.cpu_count())
    hid, logits, lh = om.seq().prefill(ids)
    for tc in (True, False):
        m = rdet.Model.open(d, max_prefill=4096, layer_commitments=True, tensor_cores=tc)
        s = m.new_sequence(4100)
        s.prefill(ids)
        assert [s.commitment(rdet.BUF_LAYER_OUTPUT, l) for l in range(2)] == lh, f"tensor_cores={tc}"
        assert s.commitment(rdet.BUF_HIDDEN) == O.act_commitment(hid)
        assert np.array_equal(s.read(rdet.BUF_LOGITS), logits)
        m.close()
