"""Whole-path parity, CUDA vs oracle, on the tiny-gemma-dev bundle
and on seeded synthetic models covering every det
feature: sliding / full layers, partial RoPE, KV sharing, k_eq_v with global
KV heads, PLE, softcap, tied and untied lm_head, i16 and i32 weights,
bidirectional window, prompts longer than the window."""
import tempfile

import numpy as np
import pytest

import oracle as O
import tiny_gemma_dev
from helpers import detwgt, lcg_ids, mini_config, rdet, write_model

pytestmark = pytest.mark.gpu


def run_both(model_dir, ids, n_decode, layer_commitments=True):
    om = O.Model(model_dir, threads=8)
    gm = rdet.Model.open(model_dir, max_prefill=max(len(ids), 8), layer_commitments=layer_commitments)
    os_, gs = om.seq(), gm.new_sequence(len(ids) + n_decode + 4)
    hid, logits, lh = os_.prefill(ids)
    gs.prefill(ids)
    assert gs.commitment(rdet.BUF_HIDDEN) == O.act_commitment(hid)
    assert np.array_equal(gs.read(rdet.BUF_LOGITS), logits)
    if layer_commitments:
        assert [gs.commitment(rdet.BUF_LAYER_OUTPUT, l) for l in range(om.L)] == lh
    assert gs.commitment(rdet.BUF_KV) == os_.kv_commitment()
    for step in range(n_decode):
        t = O.argmax_first(logits)
        assert gs.select() == t, step
        h, logits, lh = os_.decode(t)
        gs.decode(t)
        assert np.array_equal(gs.read(rdet.BUF_LOGITS), logits), step
        assert [gs.commitment(rdet.BUF_LAYER_OUTPUT, l) for l in range(om.L)] == lh, step
        assert gs.commitment(rdet.BUF_KV) == os_.kv_commitment(), step
    return om, gm


def test_tiny_gemma_dev_config1():
    d = tiny_gemma_dev.write_bundle(tempfile.mkdtemp(), detwgt.encode)
    run_both(d, tiny_gemma_dev.lcg_token_ids(16, 280, 0), 8)


VARIANTS = {
    "default": (mini_config(), 16),
    "no_share_untied_i32": (mini_config(num_kv_shared_layers=0, tie_word_embeddings=False,
                                        final_logit_softcapping=None), 32),
    "k_eq_v_global_kv": (mini_config(attention_k_eq_v=True, num_global_key_value_heads=1), 16),
    "bidirectional_window": (mini_config(use_bidirectional_attention="all", sliding_window=10), 16),
    "no_ple_full_rotary": (mini_config(hidden_size_per_layer_input=None,
                                       rope_parameters={"full_attention": {"partial_rotary_factor": 1.0}}), 16),
    "gqa8": (mini_config(num_attention_heads=8, num_key_value_heads=1, layer_types=["full_attention"] * 2 +
                         ["sliding_attention"] * 4, num_kv_shared_layers=1), 16),
}


@pytest.mark.parametrize("variant", sorted(VARIANTS))
def test_synthetic_variants(variant):
    cfg, width = VARIANTS[variant]
    cfg["text_config"] = {k: v for k, v in cfg["text_config"].items() if v is not None}
    d = write_model(cfg, seed=11, width=width)
    ids = lcg_ids(21, cfg["text_config"]["vocab_size"], 3)
    run_both(d, ids, 12)


def test_single_token_prompt_and_window_edge():
    cfg = mini_config(sliding_window=1)
    d = write_model(cfg, seed=5)
    run_both(d, [7], 5)


def test_synthetic_on_device_equals_artifact():
    cfg = mini_config()
    d = write_model(cfg, seed=21, width=16)
    ids = lcg_ids(9, 97, 1)
    a = rdet.Model.open(d, max_prefill=16)
    b = rdet.Model.synthetic(cfg, seed=21, width=16, max_prefill=16)
    assert a.weight_bytes == b.weight_bytes
    sa, sb = a.new_sequence(32), b.new_sequence(32)
    sa.prefill(ids)
    sb.prefill(ids)
    assert np.array_equal(sa.read(rdet.BUF_LOGITS), sb.read(rdet.BUF_LOGITS))
    assert sa.generate(6) == sb.generate(6)
    assert sa.commitment(rdet.BUF_KV) == sb.commitment(rdet.BUF_KV)


def test_routine_granular_prefill_equals_one_shot():
    cfg = mini_config(num_kv_shared_layers=0)
    d = write_model(cfg, seed=2)
    ids = lcg_ids(13, 97, 9)
    m = rdet.Model.open(d, max_prefill=16)
    s1, s2 = m.new_sequence(32), m.new_sequence(32)
    s1.prefill(ids)
    s2.prefill_begin(ids)
    s2.prefill_range(0, 2)
    s2.prefill_range(2, 5)
    s2.prefill_range(5, 6)
    s2.prefill_finalize()
    for b in (rdet.BUF_HIDDEN, rdet.BUF_LOGITS, rdet.BUF_KV):
        assert s1.commitment(b) == s2.commitment(b)
    with pytest.raises(rdet.RdetError):
        s2.prefill_range(3, 4)  # not in flight


def test_generate_equals_stepwise_and_batch_decode():
    cfg = mini_config()
    d = write_model(cfg, seed=4)
    m = rdet.Model.open(d, max_prefill=16)
    ids = lcg_ids(10, 97, 4)
    a, b, c = m.new_sequence(64), m.new_sequence(64), m.new_sequence(64)
    for s in (a, b, c):
        s.prefill(ids)
    ga = a.generate(20)
    gb = []
    for _ in range(20):
        t = b.select()
        gb.append(t)
        b.decode(t)
    assert ga == gb
    assert a.commitment(rdet.BUF_KV) == b.commitment(rdet.BUF_KV)
    # ragged batch of two sequences at different positions
    x = m.new_sequence(64)
    x.prefill(ids[:4])
    gc, gx = [], []
    for _ in range(5):
        tc, tx = c.select(), x.select()
        gc.append(tc)
        gx.append(tx)
        rdet.decode_batch(m, [c, x], [tc, tx])
    assert gc == ga[:5]


def test_errors_are_reported():
    cfg = mini_config()
    d = write_model(cfg, seed=4)
    m = rdet.Model.open(d, max_prefill=8)
    s = m.new_sequence(8)
    with pytest.raises(rdet.RdetError) as e:
        s.prefill([1000])
    assert e.value.code == -6
    with pytest.raises(rdet.RdetError):
        s.decode(1)  # not prefilled
    with pytest.raises(rdet.RdetError):
        s.prefill(list(range(9)))  # longer than max_prefill
    s.prefill([1, 2, 3, 4, 5, 6, 7, 8])
    with pytest.raises(rdet.RdetError):
        s.decode(1)  # KV cache full


def test_e4b_head_dims_long_prompt():
    # E4B head geometry (d=256 sliding, d_g=512 full, 8 query / 2 KV heads,
    # window 512) on a narrow model, with a prompt longer than the window
    cfg = mini_config(hidden_size=256, intermediate_size=512, num_attention_heads=8, num_key_value_heads=2,
                      head_dim=256, global_head_dim=512, sliding_window=512, hidden_size_per_layer_input=32,
                      num_hidden_layers=4, num_kv_shared_layers=1, vocab_size=300,
                      layer_types=["sliding_attention", "full_attention", "sliding_attention", "sliding_attention"])
    d = write_model(cfg, seed=8)
    run_both(d, lcg_ids(600, 300, 2), 4)


@pytest.mark.parametrize("variant", ["default", "k_eq_v_global_kv", "gqa8", "bidirectional_window"])
def test_tensor_core_prefill_long_prompt(variant):
    # prompts of >= 32 tokens take the tcgen05 prefill linear (several M tiles,
    # a partial last tile); the no-tensor-core context must agree with it
    cfg, width = VARIANTS[variant]
    cfg = {"text_config": {k: v for k, v in cfg["text_config"].items() if v is not None}}
    d = write_model(cfg, seed=21, width=width)
    ids = lcg_ids(300, cfg["text_config"]["vocab_size"], 9)
    run_both(d, ids, 3)
    cuda = rdet.Model.open(d, max_prefill=len(ids), tensor_cores=False)
    s = cuda.new_sequence(len(ids) + 4)
    s.prefill(ids)
    tc = rdet.Model.open(d, max_prefill=len(ids))
    assert tc.tensor_core_prefill and not cuda.tensor_core_prefill
    t = tc.new_sequence(len(ids) + 4)
    t.prefill(ids)
    assert s.commitment(rdet.BUF_HIDDEN) == t.commitment(rdet.BUF_HIDDEN)
    assert np.array_equal(s.read(rdet.BUF_LOGITS), t.read(rdet.BUF_LOGITS))


def check_batched_equals_solo(cfg, width, lens, steps, seed):
    cfg = {"text_config": {k: v for k, v in cfg["text_config"].items() if v is not None}}
    V = cfg["text_config"]["vocab_size"]
    d = write_model(cfg, seed=seed, width=width)
    m = rdet.Model.open(d, max_prefill=max(max(lens), len(lens)))
    batch = [m.new_sequence(n + steps + 4) for n in lens]
    solo = [m.new_sequence(n + steps + 4) for n in lens]
    for i, n in enumerate(lens):
        ids = lcg_ids(n, V, 100 + i)
        batch[i].prefill(ids)
        solo[i].prefill(ids)
    L = m.L
    for step in range(steps):
        toks = rdet.select_batch(m, batch)  # one launch over every row
        assert toks == [s.select() for s in solo] == [s.select() for s in batch], step
        rdet.decode_batch(m, batch, toks)
        for s, t in zip(solo, toks):
            s.decode(t)
        for i, (a, b) in enumerate(zip(batch, solo)):
            assert np.array_equal(a.read(rdet.BUF_LOGITS), b.read(rdet.BUF_LOGITS)), (step, i)
            assert a.commitment(rdet.BUF_HIDDEN) == b.commitment(rdet.BUF_HIDDEN), (step, i)
            assert a.commitment(rdet.BUF_LAYER_OUTPUT, L // 2) == b.commitment(rdet.BUF_LAYER_OUTPUT, L // 2)
            assert a.commitment(rdet.BUF_KV) == b.commitment(rdet.BUF_KV), (step, i)
            assert a.position == b.position


@pytest.mark.parametrize("variant,B", [("default", 5), ("default", 40), ("k_eq_v_global_kv", 40),
                                       ("gqa8", 33), ("no_share_untied_i32", 34), ("bidirectional_window", 6)])
def test_batched_ragged_decode_equals_solo(variant, B):
    # ragged batch: each sequence has its own length (some past the window);
    # >= 32 rows take the tensor-core GEMMs, fewer the CUDA-core linear
    cfg, width = VARIANTS[variant]
    lens = [1 + (7 * i * i + 3 * i) % 37 for i in range(B)]
    check_batched_equals_solo(cfg, width, lens, 4, seed=30 + B)


def test_batched_ragged_decode_e4b_head_dims():
    cfg = mini_config(hidden_size=256, intermediate_size=512, num_attention_heads=8, num_key_value_heads=2,
                      head_dim=256, global_head_dim=512, sliding_window=512, hidden_size_per_layer_input=32,
                      num_hidden_layers=4, num_kv_shared_layers=1, vocab_size=300,
                      layer_types=["sliding_attention", "full_attention", "sliding_attention", "sliding_attention"])
    lens = [5 + (97 * i) % 640 for i in range(36)]
    check_batched_equals_solo(cfg, 16, lens, 3, seed=44)
