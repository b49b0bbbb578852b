"""Writes the E4B-shape parity fixtures (tests/golden/e4b_fixtures.json).

The BASELINE configs 3, 4 and 5 run on the seeded random-init model of the
E4B stand-in shape (raster-inference_b200/configs/e4b_text_standin.json,
seed 20260501, i16 weights: the model bench.py times).  The reference
publishes no goldens at that shape, and running its det path there on the CPU
takes tens of minutes per config, far too long for a test.  So this script
runs the CPU oracle (the C++ restatement of the reference det path, pinned to
the reference's own goldens) once, here, and records what it produced: SHA-256
commitments (det_layer_prefill / det_layer_decode / det_hidden_to_logits at
det_kernels.rs:678-821, :866-1133, :1217-1267; commitments as
transformer_kernels.rs:1395-1482) and greedy tokens (argmax_first,
det_num/ops.rs:463-478).  tests/test_gpu_e4b.py rebuilds the same model on
the GPU and checks the CUDA path against these values bit for bit.

Inputs (the same draws bench.py makes):
  config 3: one prompt of 512 and one of 2048 token ids, LCG seed
            20260501 + 11 + length; prefill only.
  config 4: 4096 ids, LCG seed 20260501; prefill, then 256 greedy tokens.
  config 5: the 64 ragged lengths 128 + draw % 3969 (LCG seed 20260501 + 7),
            sequence i's ids from LCG seed 20260501 + 100 + i; 128 greedy
            tokens each.  The oracle runs a subset of 4 of the 64 sequences
            (all 64 would take hours on the CPU); the GPU test decodes all 64
            in one batch and checks these 4.

    python tests/golden/make_e4b_fixtures.py [config3] [config4] [config5]

Each part merges into the output file as it finishes.  Expect roughly 10, 15
and 20 minutes on 8 host cores.
"""
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402  (the checker)

OUT = os.path.join(HERE, "e4b_fixtures.json")
CONFIG = os.path.join(ROOT, "raster-inference_b200", "configs", "e4b_text_standin.json")
SEED = 20260501
CONFIG3_LENGTHS = (512, 2048)
CONFIG4_PROMPT, CONFIG4_TOKENS = 4096, 256
CONFIG5_BATCH, CONFIG5_TOKENS = 64, 128
CONFIG5_PICKED = (29, 54, 63, 27)  # lengths 419, 235, 1997, 3675


def lcg_ids(n, vocab, seed):
    """The reference fixture's LCG (det_goldens.rs:348-356), draw = s >> 33."""
    s, out = seed, []
    for _ in range(n):
        s = (s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        out.append((s >> 33) % vocab)
    return out


def config5_lengths():
    return [128 + (x % 3969) for x in lcg_ids(CONFIG5_BATCH, 1 << 30, SEED + 7)]


def log(msg):
    print(f"[{time.strftime('%H:%M:%S')}] {msg}", flush=True)


def merge(key, value):
    data = {}
    if os.path.exists(OUT):
        with open(OUT) as f:
            data = json.load(f)
    data.update({"model": {"config": "raster-inference_b200/configs/e4b_text_standin.json", "seed": SEED,
                           "width": 16},
                 "generator": "tests/golden/make_e4b_fixtures.py (CPU oracle)"})
    data[key] = value
    with open(OUT, "w") as f:
        json.dump(data, f, indent=1, sort_keys=True)
        f.write("\n")


def own_cache_layers(m):
    """Layers [0, n) all hold a KV cache of their own (the later ones share
    their donor's), so the commitment over them is not None."""
    n = 0
    while n < m.L and m.layers[n]["donor"] < 0:
        n += 1
    return n


def prefill_record(m, s, ids):
    hid, logits, layer_hashes = s.prefill(ids)
    return {
        "embedding": O.act_commitment(m.embed(ids)),
        "final_hidden": O.act_commitment(hid),
        "logits": O.vec_commitment(logits),
        "layer_outputs": layer_hashes,
        "kv": s.kv_commitment(),
        "kv_own_layers": s.kv_commitment(own_cache_layers(m)),
        "next_token": O.argmax_first(logits),
    }, logits


def greedy(s, logits, n):
    """n x (select_output_token, decode_transition), as rdet_generate."""
    toks = []
    for _ in range(n):
        t = O.argmax_first(logits)
        toks.append(t)
        _, logits, _ = s.decode(t, want_layer_hashes=False)
    return toks, logits


def main(parts):
    with open(CONFIG) as f:
        cfg = json.load(f)
    V = cfg["text_config"]["vocab_size"]
    t0 = time.time()
    m = O.Model(None, threads=O.cpu_count(), synthetic=(cfg, SEED, 16))
    log(f"model generated in {time.time() - t0:.0f} s")
    if "config3" in parts:
        rec = {}
        for n in CONFIG3_LENGTHS:
            t0 = time.time()
            seed = SEED + 11 + n
            r, _ = prefill_record(m, m.seq(), lcg_ids(n, V, seed))
            r["ids_seed"] = seed
            rec[str(n)] = r
            log(f"config 3 prefill {n}: {time.time() - t0:.0f} s")
        merge("config3", rec)
    if "config4" in parts:
        t0 = time.time()
        s = m.seq()
        r, logits = prefill_record(m, s, lcg_ids(CONFIG4_PROMPT, V, SEED))
        log(f"config 4 prefill: {time.time() - t0:.0f} s")
        t0 = time.time()
        toks, logits = greedy(s, logits, CONFIG4_TOKENS)
        log(f"config 4 decode of {CONFIG4_TOKENS}: {time.time() - t0:.0f} s")
        merge("config4", {"prompt_tokens": CONFIG4_PROMPT, "ids_seed": SEED, "prefill": r, "tokens": toks,
                          "final_logits": O.vec_commitment(logits), "final_kv": s.kv_commitment(),
                          "final_kv_own_layers": s.kv_commitment(own_cache_layers(m))})
    if "config5" in parts:
        lens = config5_lengths()
        seqs = {}
        for i in CONFIG5_PICKED:
            t0 = time.time()
            s = m.seq()
            seed = SEED + 100 + i
            _, logits, _ = s.prefill(lcg_ids(lens[i], V, seed), want_hidden=False, want_layer_hashes=False)
            toks, logits = greedy(s, logits, CONFIG5_TOKENS)
            seqs[str(i)] = {"length": lens[i], "ids_seed": seed, "tokens": toks,
                            "final_logits": O.vec_commitment(logits),
                            "final_kv_own_layers": s.kv_commitment(own_cache_layers(m))}
            log(f"config 5 sequence {i} (length {lens[i]}): {time.time() - t0:.0f} s")
        merge("config5", {"batch": CONFIG5_BATCH, "lengths_seed": SEED + 7, "tokens_per_sequence": CONFIG5_TOKENS,
                          "sequences": seqs})
    m.close()


if __name__ == "__main__":
    main(set(sys.argv[1:]) or {"config3", "config4", "config5"})
